// fg_common.cuh -- error plumbing and block-level primitives shared by the kernels.
#pragma once

#include <cuda_runtime.h>
#include <cfloat>
#include <cstdint>
#include <cstdio>

#include "fusiongpu.h"

namespace fg {

// ---- host-side error reporting (thread-local message behind fg_last_error) ----
void set_error(const char* fmt, ...);
int fail(int status, const char* fmt, ...);
int check_launch(const char* what);

// A device attribute of the current device, read once per device and cached
// (launch paths ask for shared-memory limits and SM counts on every call).
int device_attr(cudaDeviceAttr attr);
// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) only when `bytes` exceeds
// what was last granted to `func` (the attribute is per function, not per launch).
cudaError_t ensure_smem(const void* func, int bytes);

#define FG_REQUIRE(cond, ...)                                          \
    do {                                                               \
        if (!(cond)) return ::fg::fail(FG_ERR_INVALID_ARG, __VA_ARGS__); \
    } while (0)

#define FG_CUDA_TRY(call)                                                                  \
    do {                                                                                   \
        cudaError_t _e = (call);                                                           \
        if (_e != cudaSuccess)                                                             \
            return ::fg::fail(FG_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(_e));     \
    } while (0)

inline bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
inline size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Bump allocator over a caller-provided workspace (256-byte aligned slices).
struct Carve {
    char* base;
    size_t cap, used = 0;
    Carve(void* p, size_t c) : base(static_cast<char*>(p)), cap(c) {}
    template <class T>
    T* take(size_t n) {
        size_t off = round_up(used, 256);
        used = off + n * sizeof(T);
        return (base && used <= cap) ? reinterpret_cast<T*>(base + off) : nullptr;
    }
    bool ok() const { return base != nullptr && used <= cap; }
};

// ---- device helpers --------------------------------------------------------------

// Order-preserving map float -> uint32 (total order; -0.0 sorts before +0.0).
__device__ __forceinline__ uint32_t f2key(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Exclusive scan of one int per thread over a block of NT threads.
// `s_warp` needs NT/32 ints.  Returns the prefix; `total` gets the block sum.
// Contains __syncthreads(): every thread of the block must call it.
template <int NT>
__device__ __forceinline__ int block_exclusive_scan(int v, int* s_warp, int& total) {
    static_assert(NT % 32 == 0 && NT <= 1024, "block size");
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[w] = x;
    __syncthreads();
    if (w == 0) {
        int t = (lane < NT / 32) ? s_warp[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            int y = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += y;
        }
        if (lane < NT / 32) s_warp[lane] = t;
    }
    __syncthreads();
    const int wbase = w ? s_warp[w - 1] : 0;
    total = s_warp[NT / 32 - 1];
    __syncthreads();
    return wbase + x - v;
}

// Finds the k-th smallest (1-based, 1 <= k <= n) of n uint32 keys held in
// memory visible to the block.  Four 8-bit MSD passes with a shared
// histogram.  Returns the k-th key and how many keys are strictly smaller.
// `s_hist` needs 256 uint32, `s_b` 2 uint32.
template <int NT>
__device__ void block_radix_select(const uint32_t* keys, int n, int k, uint32_t* s_hist,
                                   uint32_t* s_b, uint32_t& kth, int& n_less) {
    uint32_t prefix = 0, mask = 0, kk = (uint32_t)k, less = 0;
#pragma unroll 1
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = threadIdx.x; i < 256; i += NT) s_hist[i] = 0;
        __syncthreads();
        for (int i = threadIdx.x; i < n; i += NT) {
            const uint32_t key = keys[i];
            if ((key & mask) == prefix) atomicAdd(&s_hist[(key >> shift) & 255u], 1u);
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            const int lane = threadIdx.x;
            uint32_t c[8], s = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                c[j] = s_hist[lane * 8 + j];
                s += c[j];
            }
            uint32_t incl = s;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            const uint32_t excl = incl - s;
            if (excl < kk && kk <= incl) {
                uint32_t run = excl;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (run + c[j] >= kk) {
                        s_b[0] = (uint32_t)(lane * 8 + j);
                        s_b[1] = run;
                        break;
                    }
                    run += c[j];
                }
            }
        }
        __syncthreads();
        const uint32_t b = s_b[0], below = s_b[1];
        prefix |= b << shift;
        mask |= 255u << shift;
        kk -= below;
        less += below;
        __syncthreads();
    }
    kth = prefix;
    n_less = (int)less;
}

// Ascending bitonic sort of n_pow2 (power of two) uint64 keys in shared memory.
template <int NT>
__device__ void block_bitonic_sort(unsigned long long* s, int n_pow2) {
    for (int k = 2; k <= n_pow2; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n_pow2; i += NT) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const unsigned long long a = s[i], b = s[ixj];
                    const bool up = (i & k) == 0;
                    if ((a > b) == up) {
                        s[i] = b;
                        s[ixj] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
}

// ---- warp-level selection (no block barriers) -----------------------------------

__device__ __forceinline__ unsigned lanemask_lt() {
    unsigned m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

// k-th smallest (1-based, 1 <= k <= n) of n uint32 keys, by one warp.
// `hist`: 256 uint32 of shared memory owned by this warp.
__device__ inline void warp_radix_select(const uint32_t* keys, int n, int k, uint32_t* hist, uint32_t& kth,
                                         int& n_less) {
    const int lane = threadIdx.x & 31;
    uint32_t prefix = 0, mask = 0, kk = (uint32_t)k, less = 0;
#pragma unroll 1
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = lane; i < 256; i += 32) hist[i] = 0;
        __syncwarp();
        for (int i = lane; i < n; i += 32) {
            const uint32_t key = keys[i];
            if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
        }
        __syncwarp();
        uint32_t c[8], sum = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            c[j] = hist[lane * 8 + j];
            sum += c[j];
        }
        uint32_t incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        const uint32_t excl = incl - sum;
        const bool mine = excl < kk && kk <= incl;
        uint32_t b = 0, below = 0;
        if (mine) {
            uint32_t run = excl;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (run + c[j] >= kk) {
                    b = (uint32_t)(lane * 8 + j);
                    below = run;
                    break;
                }
                run += c[j];
            }
        }
        const int src = __ffs(__ballot_sync(0xffffffffu, mine)) - 1;
        b = __shfl_sync(0xffffffffu, b, src);
        below = __shfl_sync(0xffffffffu, below, src);
        prefix |= b << shift;
        mask |= 255u << shift;
        kk -= below;
        less += below;
        __syncwarp();
    }
    kth = prefix;
    n_less = (int)less;
}

// The k smallest keys (ties: lower index first), written in index order as
// (key << 32 | payload(i)) to dst[0..k).  kth/n_less from warp_radix_select.
template <class Payload>
__device__ inline void warp_collect_smallest(const uint32_t* keys, int n, int k, uint32_t kth, int n_less,
                                             unsigned long long* dst, Payload payload) {
    const int lane = threadIdx.x & 31;
    const unsigned lt = lanemask_lt();
    const int need_eq = k - n_less;
    int eq_base = 0, out = 0;
    for (int c0 = 0; c0 < n; c0 += 32) {
        const int i = c0 + lane;
        const bool in = i < n;
        const uint32_t key = in ? keys[i] : 0xffffffffu;
        const bool eq = in && key == kth;
        const unsigned eqb = __ballot_sync(0xffffffffu, eq);
        const bool sel = in && (key < kth || (eq && eq_base + __popc(eqb & lt) < need_eq));
        const unsigned sb = __ballot_sync(0xffffffffu, sel);
        if (sel) dst[out + __popc(sb & lt)] = ((unsigned long long)key << 32) | (uint32_t)payload(i);
        eq_base += __popc(eqb);
        out += __popc(sb);
    }
    __syncwarp();
}

// Ascending bitonic sort of n_pow2 uint64 keys in shared memory by one warp.
__device__ inline void warp_bitonic_sort(unsigned long long* s, int n_pow2) {
    const int lane = threadIdx.x & 31;
    for (int k = 2; k <= n_pow2; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = lane; i < n_pow2; i += 32) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const unsigned long long a = s[i], b = s[ixj];
                    if ((a > b) == ((i & k) == 0)) {
                        s[i] = b;
                        s[ixj] = a;
                    }
                }
            }
            __syncwarp();
        }
    }
}

__host__ __device__ inline int next_pow2(int x) {
    int p = 1;
    while (p < x) p <<= 1;
    return p;
}

}  // namespace fg
