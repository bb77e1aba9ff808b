// coarse_tc.cu -- coarse quantizer on the 5th-generation tensor cores
// (replaces cuVS CAGRA search over the centroids, cagra_adapter.cuh:38-68).
//
// 1. Queries and centroids are split into bf16 hi + lo parts and laid out as
//    A = [q_hi | q_hi | q_lo], B = [c_hi | c_lo | c_hi] (K = 3*dim, zero padded to
//    a multiple of 64), so one bf16 GEMM A.B^T = q_hi.c_hi + q_hi.c_lo + q_lo.c_hi
//    approximates q.c to about 2^-16 relative.
// 2. coarse_gemm_kernel: persistent, warp-specialised CTA per SM over a balanced
//    range of (128-query tile, 128-centroid tile) pairs; A resident in shared
//    memory (reloaded where the range enters the next query tile), B through a
//    3-stage TMA ring of 32 KB K blocks (two centroid tiles, 128-byte swizzle,
//    no multicast), one tcgen05.mma of N = 256 per K step for two consecutive
//    centroid tiles, issued by one thread into two TMEM accumulators; the
//    epilogue computes d~ = |q|^2 + |c|^2 - 2 q.c with |c|^2 read from shared
//    memory.
//    top_m <= 4: a single pass in which every (query, range, column part) keeps
//    its 4 or 8 smallest d~ in registers (coarse_topk_finish_kernel certifies).
//    Larger top_m:
//    Pass 0 writes d~ for a prefix of NS centroids; the S-th smallest of those (S =
//    max(2P, P+32)) bounds the S-th smallest over all centroids.  Pass 1 covers every
//    centroid and appends only (d~, id) within that bound to a per-query list, so
//    no nq x nlist matrix is ever written.
// 3. coarse_finish_kernel: per query, the S smallest appended d~ are rescored with
//    exact fp32 distances (the oracle's arithmetic) and sorted by (distance, id).
//    The top P is certified exact when the P-th exact distance is below the
//    S-th d~ minus an error bound E(q) on |d~ - d| (every excluded centroid has
//    d~ >= the S-th); otherwise -- list overflow, a failed wait in the GEMM, or
//    a certificate that does not hold -- the query is rescored exactly against
//    every centroid.  Rankings therefore equal the exact ones bit for bit,
//    whatever the tensor-core rounding.
#include <cuda_bf16.h>

#include <algorithm>

#include "fg_common.cuh"
#include "tc_common.cuh"

namespace fg {


constexpr int TC_M = 128;       // queries per tile (UMMA M, TMEM lanes)
constexpr int TC_N = 128;       // centroids per tile (UMMA N)
constexpr int TC_TILE = 128;    // row padding of both operands
constexpr int TC_KB = 64;       // bf16 elements per K block (one 128-byte swizzle row)
constexpr int TC_MAX_KB = 6;    // A resident (6 x 16 KB) + TC_NST B stages (32 KB each) = 192 KB
constexpr int TC_GRP = 2;       // centroid tiles per MMA group (UMMA N = 256)
constexpr int TC_NST = 3;       // B ring: one K block of a group's TC_GRP tiles per stage
constexpr int TC_SMEM_MAX = 227 * 1024;  // dynamic shared memory per CTA; the rest holds column norms
constexpr int TC_PARTS = 4;              // column parts of a tile: one epilogue warp per (lane quarter, part)
constexpr int TC_CPW = TC_N / TC_PARTS;  // 32 columns of each tile per epilogue thread
constexpr int TC_EPI_WARPS = 4 * TC_PARTS;
constexpr int TC_NT = 64 + TC_EPI_WARPS * 32;

__host__ __device__ inline int tc_kpad(int dim) { return (3 * dim + TC_KB - 1) / TC_KB * TC_KB; }

// Row-wise split: pattern 0 -> [hi | hi | lo], 1 -> [hi | lo | hi]; norms[r] = |x_r|^2.
__global__ void split_bf16_kernel(const float* __restrict__ x, long long n, int dim, int kpad, int pattern,
                                  __nv_bfloat16* __restrict__ out, float* __restrict__ norms,
                                  unsigned* __restrict__ max_norm_bits) {
    const long long r = (long long)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (r >= n) return;
    const float* xr = x + r * dim;
    __nv_bfloat16* o = out + r * kpad;
    float acc = 0.0f;
    for (int j = lane; j < dim; j += 32) {
        const float v = xr[j];
        const __nv_bfloat16 hi = __float2bfloat16_rn(v);
        const __nv_bfloat16 lo = __float2bfloat16_rn(v - __bfloat162float(hi));
        o[j] = hi;
        o[dim + j] = pattern ? lo : hi;
        o[2 * dim + j] = pattern ? hi : lo;
        acc = fmaf(v, v, acc);
    }
    for (int j = 3 * dim + lane; j < kpad; j += 32) o[j] = __float2bfloat16_rn(0.0f);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) {
        norms[r] = acc;
        if (max_norm_bits) atomicMax(max_norm_bits, __float_as_uint(acc));
    }
}

// Warp roles of the persistent GEMM CTA (576 threads, one CTA per SM):
//   warp 0, lane 0: TMA producer (the query tile A, then B through a ring of
//                   TC_NST stages, one 256 x 64 K block per stage)
//   warp 1, lane 0: MMA issuer (and warp 1 owns the TMEM allocation)
//   warps 2..17:    epilogue; warp w reads TMEM lanes 32*(w%4) .. +31 (its 32
//                   queries) and columns 32*((w-2)/4) .. +31 of each tile
// The (query tile, centroid tile) pairs are numbered query-tile-major and every
// CTA takes one contiguous range of L of them, so the work is balanced over the
// SMs whatever the shape; where a range crosses into the next query tile the
// producer reloads A once the MMAs on the old one have finished (a_empty).  A
// range covers one "segment" of a query tile: segment = CTA index minus the
// first CTA of that query tile, at most maxseg per query tile.
// Within a range, two consecutive tiles of one query tile form a group whose
// MMAs run as one UMMA of N = 256 (half the tcgen05.mma instructions, waits
// and commits per flop of 128-wide tiles, which bound the MMA issuer); a tile
// left over at the end of a range or of a query tile is a group of one (N =
// 128).  Producer, issuer and epilogue walk the same groups.  TMEM holds two
// 128 x 256 fp32 accumulators (all 512 columns), so the epilogue of group i
// runs while the MMAs of group i+1 fill the other one.
struct GemmArgs {
    int kt;              // 64-wide K blocks
    long long q0;        // first query row of this launch (row of the A tensor map)
    int nq;              // query rows of this launch
    int ncols;           // centroid columns [0, ncols)
    int ntiles;          // centroid tiles: ceil(ncols / TC_N)
    long long total;     // (query tile, centroid tile) pairs
    int per_cta;         // L: pairs per CTA
    int maxseg;          // segments per query tile (lists per query = maxseg * TC_PARTS)
    const float* qn;     // |q|^2, indexed by q0 + row
    const float* cn;     // |c|^2
    uint32_t* out;       // GEMM_MATRIX: order key of d~ at out[row * ldo + col]
    long long ldo;
    const float* tq;     // GEMM_FILTER: per-query bound
    int cap;             // GEMM_FILTER: capacity of each (query, segment, part) list
    int* cnt;            // GEMM_FILTER: [nq][maxseg * TC_PARTS] appended counts (may exceed cap)
    uint32_t* list_k;    // [nq][maxseg * TC_PARTS][cap or T] keys of d~
    int32_t* list_i;     // same shape: centroid ids
    int* err;
    int norm_smem;       // column norms staged in shared memory (+inf past ncols)
};

enum { GEMM_MATRIX = 0, GEMM_FILTER = 1, GEMM_TOPK = 2 };
constexpr int TC_TOPK_MAXP = 4;  // top_m up to which the single-pass GEMM_TOPK path runs

// Candidates kept per (query, segment, part) list in the single-pass path:
// P + 2 or more, so that the list's largest kept value usually lies well above
// the P-th distance and the certificate holds.
__host__ __device__ constexpr int topk_len(int P) { return P <= 2 ? 4 : 8; }

// v[j] for a lane-varying j by a five-level select tree: every index is
// static, so v stays in registers.
__device__ __forceinline__ float select32(const float (&v)[32], int j) {
    float a[16], b[8], c[4], d[2];
#pragma unroll
    for (int t = 0; t < 16; ++t) a[t] = (j & 1) ? v[2 * t + 1] : v[2 * t];
#pragma unroll
    for (int t = 0; t < 8; ++t) b[t] = (j & 2) ? a[2 * t + 1] : a[2 * t];
#pragma unroll
    for (int t = 0; t < 4; ++t) c[t] = (j & 4) ? b[2 * t + 1] : b[2 * t];
#pragma unroll
    for (int t = 0; t < 2; ++t) d[t] = (j & 8) ? c[2 * t + 1] : c[2 * t];
    return (j & 16) ? d[1] : d[0];
}

// Insert x into the ascending list bd (x < bd[T-1]); equal keys keep their
// order, so an earlier column stays ahead.  Every slot's update is
// independent of the others: no serial compare-swap chain.
template <int T>
__device__ __forceinline__ void insert_sorted(float (&bd)[T], int32_t (&bi)[T], float x, int32_t xi) {
    bool lt[T];
#pragma unroll
    for (int t = 0; t < T; ++t) lt[t] = x < bd[t];
#pragma unroll
    for (int t = T - 1; t > 0; --t) {
        bd[t] = lt[t - 1] ? bd[t - 1] : (lt[t] ? x : bd[t]);
        bi[t] = lt[t - 1] ? bi[t - 1] : (lt[t] ? xi : bi[t]);
    }
    bd[0] = lt[0] ? x : bd[0];
    bi[0] = lt[0] ? xi : bi[0];
}

// Minimum of 32 values by a tree.
__device__ __forceinline__ float min32(const float (&v)[32]) {
    float m[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) m[j] = fminf(v[j], v[j + 16]);
#pragma unroll
    for (int w = 8; w; w >>= 1)
#pragma unroll
        for (int j = 0; j < w; ++j) m[j] = fminf(m[j], m[j + w]);
    return m[0];
}

// Norms of the 32 columns col0.. (0 past ncols), from shared or global memory.
__device__ __forceinline__ void load_norms(const float* cn, int col0, int ncols, float (&c)[32]) {
    if (col0 + 32 <= ncols) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
            const float4 c4 = *reinterpret_cast<const float4*>(cn + col0 + j);
            c[j] = c4.x;
            c[j + 1] = c4.y;
            c[j + 2] = c4.z;
            c[j + 3] = c4.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) c[j] = (col0 + j < ncols) ? cn[col0 + j] : 0.0f;
    }
}

template <int MODE, int T>
__global__ void __launch_bounds__(TC_NT, 1)
    coarse_gemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                       const GemmArgs g) {
    extern __shared__ __align__(1024) unsigned char dsmem[];
    __shared__ __align__(8) uint64_t a_full, a_empty, b_full[TC_NST], b_empty[TC_NST], acc_full[2], acc_empty[2];
    __shared__ uint32_t tmem_slot;
    __shared__ int s_fail;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const long long p0 = (long long)blockIdx.x * g.per_cta;
    const long long p1 = p0 + g.per_cta < g.total ? p0 + g.per_cta : g.total;
    if (p0 >= p1) return;  // uniform for the whole CTA
    constexpr int A_KB = TC_M * TC_KB * 2;  // 16 KB per K block
    constexpr int B_KB = TC_N * TC_KB * 2;  // 16 KB per K block
    constexpr int B_ST = TC_GRP * B_KB;     // one stage
    unsigned char* base = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(dsmem) + 1023) & ~static_cast<uintptr_t>(1023));
    unsigned char* sa = base;
    unsigned char* sb = base + g.kt * A_KB;
    float* sn = reinterpret_cast<float*>(sb + TC_NST * B_ST);

    if (tid == 0) {
        s_fail = 0;
        tc::mbar_init(&a_full, 1);
        tc::mbar_init(&a_empty, 1);
        for (int i = 0; i < TC_NST; ++i) {
            tc::mbar_init(&b_full[i], 1);
            tc::mbar_init(&b_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            tc::mbar_init(&acc_full[i], 1);
            tc::mbar_init(&acc_empty[i], TC_EPI_WARPS * 32);
        }
        tc::fence_mbar_init();
    }
    if (warp == 1) {
        tc::tmem_alloc(&tmem_slot, 2 * TC_GRP * TC_N);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t taddr = tmem_slot;
    volatile int* fail = &s_fail;

    if (warp == 0) {
        if (lane == 0) {  // ---- TMA producer
            long long cur = -1;
            int na = 0;
            long long kb = 0;
            for (long long pi = p0, gs = 1; pi < p1; pi += gs) {
                const long long mt = pi / g.ntiles;
                const int t = (int)(pi - mt * g.ntiles);
                gs = (pi + 1 < p1 && t + 1 < g.ntiles) ? 2 : 1;
                if (mt != cur) {
                    if (na > 0 && !tc::mbar_wait_or_fail(&a_empty, (na - 1) & 1, fail)) break;
                    tc::mbar_arrive_expect_tx(&a_full, (uint32_t)(g.kt * A_KB));
                    for (int k = 0; k < g.kt; ++k)
                        tc::tma_load_2d(sa + k * A_KB, &ta, &a_full, k * TC_KB, (int)(g.q0 + mt * TC_M));
                    ++na;
                    cur = mt;
                }
                bool ok = true;
                for (int k = 0; k < g.kt; ++k, ++kb) {
                    const int st = (int)(kb % TC_NST);
                    if (!tc::mbar_wait_or_fail(&b_empty[st], (uint32_t)(((kb / TC_NST) & 1) ^ 1), fail)) {
                        ok = false;
                        break;
                    }
                    tc::mbar_arrive_expect_tx(&b_full[st], (uint32_t)(gs * B_KB));
                    tc::tma_load_2d(sb + st * B_ST, &tb, &b_full[st], k * TC_KB, t * TC_N);
                    if (gs == 2) tc::tma_load_2d(sb + st * B_ST + B_KB, &tb, &b_full[st], k * TC_KB, (t + 1) * TC_N);
                }
                if (!ok) break;
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // ---- MMA issuer
            constexpr uint32_t idesc1 = tc::idesc_bf16_f32(TC_M, TC_N);
            constexpr uint32_t idesc2 = tc::idesc_bf16_f32(TC_M, 2 * TC_N);
            long long cur = -1;
            int na = 0;
            long long kb = 0;
            int li = 0;
            for (long long pi = p0, gs = 1; pi < p1; pi += gs, ++li) {
                const long long mt = pi / g.ntiles;
                gs = (pi + 1 < p1 && (int)(pi - mt * g.ntiles) + 1 < g.ntiles) ? 2 : 1;
                const uint32_t idesc = gs == 2 ? idesc2 : idesc1;
                if (mt != cur) {
                    if (!tc::mbar_wait_or_fail(&a_full, na & 1, fail)) break;
                    ++na;
                    cur = mt;
                }
                const int acc = li & 1;
                if (!tc::mbar_wait_or_fail(&acc_empty[acc], ((li >> 1) & 1) ^ 1, fail)) break;
                tc::fence_after_sync();
                bool ok = true;
                for (int k = 0; k < g.kt; ++k, ++kb) {
                    const int st = (int)(kb % TC_NST);
                    if (!tc::mbar_wait_or_fail(&b_full[st], (uint32_t)((kb / TC_NST) & 1), fail)) {
                        ok = false;
                        break;
                    }
                    tc::fence_after_sync();
                    const uint64_t da = tc::desc_kmajor_sw128(sa + k * A_KB);
                    const uint64_t db = tc::desc_kmajor_sw128(sb + st * B_ST);
#pragma unroll
                    for (int kk = 0; kk < TC_KB / 16; ++kk)
                        tc::umma_bf16(taddr + (uint32_t)(acc * TC_GRP * TC_N), da + 2 * kk, db + 2 * kk, idesc,
                                      (k | kk) != 0);
                    tc::umma_commit(&b_empty[st]);  // the stage may be refilled once these MMAs finish
                }
                if (!ok) break;
                tc::umma_commit(&acc_full[acc]);  // the accumulator is ready for the epilogue
                if (pi + gs == p1 || (pi + gs) / g.ntiles != mt) tc::umma_commit(&a_empty);  // last use of this A
            }
        }
    } else {  // ---- epilogue warps 2..17
        const int q4 = warp & 3;
        const int part = (warp - 2) >> 2;  // which 32 columns of each tile
        long long cur = -1;
        int row = 0;
        bool valid = false;
        long long qg = 0, lidx = 0;
        float qnr = 0.0f, bound = 0.0f;
        int n = 0;
        bool first = true;
        // GEMM_TOPK: the T smallest u = cn - 2 dp of this thread's columns in the
        // segment, ascending.  u orders the columns as d~ = qn + u does (qn is
        // constant per thread and adding it is monotone); qn is added when written.
        float bd[T];
        int32_t bi[T];
        auto flush = [&]() {
            if (!valid) return;
            if (MODE == GEMM_FILTER) g.cnt[lidx] = n;
            if (MODE == GEMM_TOPK) {
                const long long o = lidx * (long long)T;
#pragma unroll
                for (int t = 0; t < T; ++t) {
                    g.list_k[o + t] = bi[t] >= 0 ? f2key(qnr + bd[t]) : 0xffffffffu;
                    g.list_i[o + t] = bi[t];
                }
            }
        };
        // column norms: staged in shared memory once per CTA (+inf past ncols,
        // so padded columns never enter a list), else read per tile from global
        const float* cnp = g.cn;
        if (g.norm_smem) {
            const int nfl = g.ntiles * TC_N;
            for (int i = tid - 64; i < nfl; i += TC_EPI_WARPS * 32) sn[i] = i < g.ncols ? g.cn[i] : INFINITY;
            asm volatile("bar.sync 1, %0;" ::"r"(TC_EPI_WARPS * 32) : "memory");
        }
        int li = 0;
        for (long long pi = p0, gs = 1; pi < p1; pi += gs, ++li) {
            const long long mt = pi / g.ntiles;
            const int t0 = (int)(pi - mt * g.ntiles);
            gs = (pi + 1 < p1 && t0 + 1 < g.ntiles) ? 2 : 1;
            if (mt != cur) {
                flush();
                cur = mt;
                row = (int)(mt * TC_M) + q4 * 32 + lane;
                valid = row < g.nq;
                qg = g.q0 + row;
                qnr = valid ? g.qn[qg] : 0.0f;
                bound = (MODE == GEMM_FILTER && valid) ? g.tq[qg] : 0.0f;
                const long long first_cta = (mt * g.ntiles) / g.per_cta;
                lidx = (qg * g.maxseg + ((long long)blockIdx.x - first_cta)) * TC_PARTS + part;
                n = 0;
                first = true;
            }
            const int acc = li & 1, ph = (li >> 1) & 1;
            if (!__all_sync(0xffffffffu, tc::mbar_wait_or_fail(&acc_full[acc], ph, fail))) break;
            tc::fence_after_sync();
#pragma unroll 1
            for (int sub = 0; sub < (int)gs; ++sub) {
                const int t = t0 + sub;
                float v[32];
                tc::tmem_ld_32x32(taddr + ((uint32_t)(q4 * 32) << 16) +
                                      (uint32_t)(acc * TC_GRP * TC_N + sub * TC_N + part * TC_CPW),
                                  v);
                if (sub + 1 == (int)gs) {
                    tc::fence_before_sync();
                    tc::mbar_arrive(&acc_empty[acc]);
                }
                // GEMM_TOPK keeps every lane in the loop: its candidate rounds are warp-collective
                if (!valid && MODE != GEMM_TOPK) continue;
                const int col0 = t * TC_N + part * TC_CPW;
                const int ncol = min(TC_CPW, g.ncols - col0);
                float c[32];
                if (g.norm_smem) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        const float4 c4 = *reinterpret_cast<const float4*>(sn + col0 + j);
                        c[j] = c4.x;
                        c[j + 1] = c4.y;
                        c[j + 2] = c4.z;
                        c[j + 3] = c4.w;
                    }
                } else {
                    load_norms(cnp, col0, g.ncols, c);
                }
                if (MODE == GEMM_MATRIX) {
                    uint32_t* o = g.out + (long long)row * g.ldo + col0;
                    if (ncol == TC_CPW && (g.ldo & 3) == 0) {  // 16-byte aligned row chunks
#pragma unroll
                        for (int j = 0; j < 32; j += 4) {
                            uint4 k4;
                            k4.x = f2key(qnr + c[j] - 2.0f * v[j]);
                            k4.y = f2key(qnr + c[j + 1] - 2.0f * v[j + 1]);
                            k4.z = f2key(qnr + c[j + 2] - 2.0f * v[j + 2]);
                            k4.w = f2key(qnr + c[j + 3] - 2.0f * v[j + 3]);
                            *reinterpret_cast<uint4*>(o + j) = k4;
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (j < ncol) o[j] = f2key(qnr + c[j] - 2.0f * v[j]);
                    }
                } else if (MODE == GEMM_TOPK) {
                    if (g.norm_smem) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] = fmaf(-2.0f, v[j], c[j]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] = (j < ncol) ? fmaf(-2.0f, v[j], c[j]) : INFINITY;
                    }
                    if (first) {
                        // fill the list from the segment's first chunk: T rounds of
                        // taking out the minimum (lowest column first on equal values)
#pragma unroll
                        for (int r = 0; r < T; ++r) {
                            const float mn = min32(v);
                            unsigned em = 0;
#pragma unroll
                            for (int j = 0; j < 32; ++j) em |= (v[j] == mn) ? (1u << j) : 0u;
                            const int jm = __ffs(em) - 1;
                            bd[r] = mn;
                            bi[r] = (mn < INFINITY) ? col0 + jm : -1;
#pragma unroll
                            for (int j = 0; j < 32; ++j) v[j] = (j == jm) ? INFINITY : v[j];
                        }
                        first = false;
                        continue;
                    }
                    unsigned cand = 0;
                    if (valid && min32(v) < bd[T - 1]) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) cand |= (v[j] < bd[T - 1]) ? (1u << j) : 0u;
                    }
                    // one candidate per lane per round: the warp runs as many rounds as
                    // its busiest lane has candidates (one or two once the lists fill)
                    while (__any_sync(0xffffffffu, cand != 0u)) {
                        if (cand) {
                            const int j = __ffs(cand) - 1;
                            cand &= cand - 1u;
                            const float x = select32(v, j);
                            if (x < bd[T - 1]) insert_sorted<T>(bd, bi, x, col0 + j);
                        }
                    }
                } else {
                    unsigned pass = 0;
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        v[j] = qnr + c[j] - 2.0f * v[j];
                        pass |= (j < ncol && v[j] <= bound) ? (1u << j) : 0u;
                    }
                    if (pass) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            if (pass & (1u << j)) {
                                if (n < g.cap) {
                                    g.list_k[lidx * g.cap + n] = f2key(v[j]);
                                    g.list_i[lidx * g.cap + n] = col0 + j;
                                }
                                ++n;
                            }
                        }
                    }
                }
            }
        }
        flush();
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) tc::tmem_dealloc(taddr, 2 * TC_GRP * TC_N);
    if (tid == 0 && s_fail) atomicExch(g.err, 1);
}

// Exact squared distance in the oracle's order: one fmaf per dimension, t = 0..dim-1.
// Rows of 4-float alignment load eight float4 ahead of their fmafs, so one
// lane keeps eight loads in flight instead of waiting on each.
__device__ __forceinline__ float l2_seq_dev(const float* __restrict__ a_smem, const float* __restrict__ b, int dim) {
    float d = 0.0f;
    if ((dim & 3) == 0) {
        const float4* b4 = reinterpret_cast<const float4*>(b);
        const float4* q4 = reinterpret_cast<const float4*>(a_smem);
        const int n4 = dim >> 2;
        int t = 0;
        for (; t + 8 <= n4; t += 8) {
            float4 x[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) x[u] = __ldg(b4 + t + u);
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const float4 q = q4[t + u];
                float df = q.x - x[u].x;
                d = fmaf(df, df, d);
                df = q.y - x[u].y;
                d = fmaf(df, df, d);
                df = q.z - x[u].z;
                d = fmaf(df, df, d);
                df = q.w - x[u].w;
                d = fmaf(df, df, d);
            }
        }
        for (; t < n4; ++t) {
            const float4 x = __ldg(b4 + t);
            const float4 q = q4[t];
            float df = q.x - x.x;
            d = fmaf(df, df, d);
            df = q.y - x.y;
            d = fmaf(df, df, d);
            df = q.z - x.z;
            d = fmaf(df, df, d);
            df = q.w - x.w;
            d = fmaf(df, df, d);
        }
    } else {
        for (int t = 0; t < dim; ++t) {
            const float df = a_smem[t] - __ldg(b + t);
            d = fmaf(df, df, d);
        }
    }
    return d;
}

// The bound E on |d~ - d| for one query: split-bf16 products, fp32
// accumulation and the norms' rounding.
__device__ __forceinline__ float approx_err(float qq, float cc) {
    return 0x1p-12f * sqrtf(qq) * sqrtf(cc) + 0x1p-16f * (qq + cc);
}

// Candidates whose approximate distance exceeds the P-th smallest
// approximate distance dPa by more than 2E cannot be in the exact top P: P
// others are nearer by more than zero.  The slack covers rounding of thr.
__device__ __forceinline__ float rescore_limit(float dPa, float E) {
    return dPa + 2.0f * E + fabsf(dPa) * 0x1p-20f;
}

constexpr int FIN_WARPS = 4;      // queries per finish CTA (one warp each)
constexpr int FIN_TOT = 2048;     // appended candidates a warp gathers per query
constexpr int TC_MAX_S = 512;     // superset bound of the tensor-core path

// Warp per query: the bound for pass 1 is the S-th smallest key of the query's
// prefix row (exact order statistic of a subset, so an upper bound on the
// S-th smallest over all centroids).
__global__ void __launch_bounds__(256) coarse_bound_kernel(const uint32_t* __restrict__ M0, int NS, long long ldm,
                                                           int nq, int S, float* __restrict__ tq) {
    __shared__ uint32_t hist[8][256];
    const int w = threadIdx.x >> 5;
    const int q = blockIdx.x * 8 + w;
    if (q >= nq) return;
    uint32_t kth;
    int n_less;
    warp_radix_select(M0 + (size_t)q * ldm, NS, S, hist[w], kth, n_less);
    if ((threadIdx.x & 31) == 0) tq[q] = key2f(kth);
}

// Per-warp shared memory of the finish kernel: the query, a histogram, the
// gathered keys, the first gathered position of each of the query's segment
// lists (segs of them: 4 per CTA whose range touches the query's tile, so a
// small batch spread over every SM has several hundred), the superset.
struct FinishSmem {
    int dim4, spow, segs;
    __host__ __device__ int seg_words() const { return (segs + 3) / 4 * 4 + 4; }
    __host__ __device__ int per_warp_bytes() const {
        return dim4 * 4 + 256 * 4 + FIN_TOT * 4 + seg_words() * 4 + spow * 8 * 2;  // 16-byte multiples
    }
};

// Warp per query: gather the appended (key, id) of every list segment, keep the
// S smallest keys, rescore them exactly, sort by (distance, id), certify;
// otherwise rescore all centroids exactly through the warp's scratch row.
__global__ void __launch_bounds__(FIN_WARPS * 32) coarse_finish_kernel(
    const float* __restrict__ centroids, int nlist, int dim, const float* __restrict__ queries, int nq,
    const int* __restrict__ cnt, int gy, const uint32_t* __restrict__ list_k, const int32_t* __restrict__ list_i,
    int cap, int S, int P, const float* __restrict__ qn, const unsigned* __restrict__ max_cn_bits,
    const int* __restrict__ err, uint32_t* __restrict__ fb, uint32_t* __restrict__ out_ids,
    float* __restrict__ out_d, int* __restrict__ n_fallback) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * FIN_WARPS + w;
    if (q >= nq) return;
    const FinishSmem L{(dim + 3) / 4 * 4, next_pow2(S > P ? S : P), gy};
    unsigned char* mine = smem + (size_t)w * L.per_warp_bytes();
    float* sq = reinterpret_cast<float*>(mine);
    uint32_t* hist = reinterpret_cast<uint32_t*>(mine + L.dim4 * 4);
    uint32_t* wk = hist + 256;
    int32_t* pre = reinterpret_cast<int32_t*>(wk + FIN_TOT);  // first gathered position of each segment
    unsigned long long* sx = reinterpret_cast<unsigned long long*>(pre + L.seg_words());
    unsigned long long* ex = sx + L.spow;
    for (int t = lane; t < dim; t += 32) sq[t] = queries[(size_t)q * dim + t];

    // gather the segments' keys; a key's id stays in its global segment list
    int total = 0;
    bool over = false;
    for (int y = 0; y < gy && !over; ++y) {
        const int c = cnt[(size_t)q * gy + y];
        over |= c > cap;
        const int take = min(c, cap);
        if (total + take > FIN_TOT) {
            over = true;
            break;
        }
        if (lane == 0) pre[y] = total;
        const size_t seg = ((size_t)q * gy + y) * cap;
        for (int i = lane; i < take; i += 32) wk[total + i] = list_k[seg + i];
        total += take;
    }
    if (lane == 0 && !over) pre[gy] = total;
    __syncwarp();
    bool certified = false;
    if (*err == 0 && !over && total >= S) {
        uint32_t kth;
        int n_less;
        warp_radix_select(wk, total, S, hist, kth, n_less);
        warp_collect_smallest(wk, total, S, kth, n_less, sx, [&](int i) {
            // the segment holding gathered position i: the last y with pre[y] <= i
            // (empty segments share their successor's start)
            int y = 0, hi = gy - 1;
            while (y < hi) {
                const int mid = (y + hi + 1) >> 1;
                if (pre[mid] <= i) y = mid; else hi = mid - 1;
            }
            return list_i[((size_t)q * gy + y) * cap + (i - pre[y])];
        });
        for (int i = S + lane; i < L.spow; i += 32) sx[i] = ~0ull;
        __syncwarp();
        warp_bitonic_sort(sx, L.spow);  // by approximate key
        const float E = approx_err(qn[q], __uint_as_float(*max_cn_bits));
        const float thr = rescore_limit(key2f((uint32_t)(sx[P - 1] >> 32)), E);
        // rescore exactly the sorted prefix within thr.  Every lane runs every
        // round (spow is below 32 when nlist is), so the ballot sees the whole warp.
        int r = 0;
        for (int i0 = 0; i0 < L.spow; i0 += 32) {
            const int i = i0 + lane;
            const bool in = i < L.spow;
            const unsigned long long e = in ? sx[i] : ~0ull;
            unsigned long long key = ~0ull;
            const bool take = in && i < S && key2f((uint32_t)(e >> 32)) <= thr;
            if (take) {
                const uint32_t cid = (uint32_t)(e & 0xffffffffu);
                key = ((unsigned long long)f2key(l2_seq_dev(sq, centroids + (size_t)cid * dim, dim)) << 32) | cid;
            }
            r += __popc(__ballot_sync(0xffffffffu, take));
            if (in) ex[i] = key;
        }
        __syncwarp();
        warp_bitonic_sort(ex, next_pow2(r > P ? r : P));
        const float dp = key2f((uint32_t)(ex[P - 1] >> 32));
        const float T = key2f(kth);
        certified = (S >= nlist) || (dp < T - E);
    }
    if (!certified) {
        uint32_t* rk = fb + ((size_t)blockIdx.x * FIN_WARPS + w) * nlist;
        for (int c = lane; c < nlist; c += 32) rk[c] = f2key(l2_seq_dev(sq, centroids + (size_t)c * dim, dim));
        __syncwarp();
        uint32_t kth;
        int n_less;
        warp_radix_select(rk, nlist, P, hist, kth, n_less);
        warp_collect_smallest(rk, nlist, P, kth, n_less, ex, [](int i) { return i; });
        const int ppow = next_pow2(P);
        for (int i = P + lane; i < ppow; i += 32) ex[i] = ~0ull;
        __syncwarp();
        warp_bitonic_sort(ex, ppow);
        if (lane == 0) atomicAdd(n_fallback, 1);
    }
    for (int j = lane; j < P; j += 32) {
        const unsigned long long e = ex[j];
        out_ids[(size_t)q * P + j] = (uint32_t)(e & 0xffffffffu);
        out_d[(size_t)q * P + j] = key2f((uint32_t)(e >> 32));
    }
}

// Warp per query, single-pass path: the topt smallest d~ of every (segment,
// part) list are rescored exactly and sorted by (distance, id).  Every
// centroid outside a full list has d~ >= that list's largest kept d~, so with
// B = the smallest such value over the full lists, the first P are the exact
// top-P when their P-th distance is below B - E.  Otherwise every centroid is
// rescored through the warp's scratch row.
__global__ void __launch_bounds__(FIN_WARPS * 32) coarse_topk_finish_kernel(
    const float* __restrict__ centroids, int nlist, int dim, const float* __restrict__ queries, int nq, int nlists,
    int topt, const uint32_t* __restrict__ list_k, const int32_t* __restrict__ list_i, int P,
    const float* __restrict__ qn,
    const unsigned* __restrict__ max_cn_bits, const int* __restrict__ err, uint32_t* __restrict__ fb,
    uint32_t* __restrict__ out_ids, float* __restrict__ out_d, int* __restrict__ n_fallback) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * FIN_WARPS + w;
    if (q >= nq) return;
    const int ncand = nlists * topt;
    const int cpow = next_pow2(ncand);
    const FinishSmem L{(dim + 3) / 4 * 4, next_pow2(P), 0};
    // per warp: query, histogram (fallback select), candidate keys [cpow]
    unsigned char* mine = smem + (size_t)w * ((size_t)L.dim4 * 4 + 256 * 4 + (size_t)cpow * 8);
    float* sq = reinterpret_cast<float*>(mine);
    uint32_t* hist = reinterpret_cast<uint32_t*>(mine + L.dim4 * 4);
    unsigned long long* ex = reinterpret_cast<unsigned long long*>(hist + 256);
    for (int t = lane; t < dim; t += 32) sq[t] = queries[(size_t)q * dim + t];
    __syncwarp();
    // B: the smallest largest-kept d~ over the full lists (an unfilled list holds
    // every centroid of its columns)
    float B = INFINITY;
    for (int l = lane; l < nlists; l += 32) {
        const size_t o = ((size_t)q * nlists + l) * topt + (topt - 1);
        if (list_i[o] >= 0) B = fminf(B, key2f(list_k[o]));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) B = fminf(B, __shfl_xor_sync(0xffffffffu, B, o));
    // (approximate key, centroid) of every kept candidate
    for (int i = lane; i < cpow; i += 32) {
        unsigned long long e = ~0ull;
        if (i < ncand) {
            const size_t o = (size_t)q * ncand + i;
            const int32_t cid = list_i[o];
            if (cid >= 0 && cid < nlist) e = ((unsigned long long)list_k[o] << 32) | (uint32_t)cid;
        }
        ex[i] = e;
    }
    __syncwarp();
    // the P-th smallest by P rounds of a warp minimum
    unsigned long long kp = 0ull;
    for (int p = 0; p < P; ++p) {
        unsigned long long mn = ~0ull;
        for (int i = lane; i < ncand; i += 32) {
            const unsigned long long e = ex[i];
            if ((p == 0 || e > kp) && e < mn) mn = e;
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const unsigned long long x = __shfl_xor_sync(0xffffffffu, mn, o);
            mn = x < mn ? x : mn;
        }
        kp = mn;
    }
    bool certified = false;
    if (*err == 0 && kp != ~0ull) {
        const float E = approx_err(qn[q], __uint_as_float(*max_cn_bits));
        const float thr = rescore_limit(key2f((uint32_t)(kp >> 32)), E);
        // compact the candidates within thr to the front, in place: a chunk's
        // entries are all read (ballot) before any lane writes, and writes
        // land at or below the chunk being read
        int r = 0;
        for (int c0 = 0; c0 < ncand; c0 += 32) {
            const int i = c0 + lane;
            const unsigned long long e = i < ncand ? ex[i] : ~0ull;
            const bool take = e != ~0ull && key2f((uint32_t)(e >> 32)) <= thr;
            const unsigned b = __ballot_sync(0xffffffffu, take);
            if (take) ex[r + __popc(b & lanemask_lt())] = e;
            r += __popc(b);
            __syncwarp();
        }
        const int rpow = next_pow2(r > P ? r : P);
        for (int i = lane; i < rpow; i += 32) {
            unsigned long long key = ~0ull;
            if (i < r) {
                const uint32_t cid = (uint32_t)(ex[i] & 0xffffffffu);
                key = ((unsigned long long)f2key(l2_seq_dev(sq, centroids + (size_t)cid * dim, dim)) << 32) | cid;
            }
            ex[i] = key;
        }
        __syncwarp();
        warp_bitonic_sort(ex, rpow);
        const float dp = key2f((uint32_t)(ex[P - 1] >> 32));
        certified = (B == INFINITY) || (dp < B - E);
    }
    if (!certified) {
        uint32_t* rk = fb + ((size_t)blockIdx.x * FIN_WARPS + w) * nlist;
        for (int c = lane; c < nlist; c += 32) rk[c] = f2key(l2_seq_dev(sq, centroids + (size_t)c * dim, dim));
        __syncwarp();
        uint32_t kth;
        int n_less;
        warp_radix_select(rk, nlist, P, hist, kth, n_less);
        warp_collect_smallest(rk, nlist, P, kth, n_less, ex, [](int i) { return i; });
        const int ppow = next_pow2(P);
        for (int i = P + lane; i < ppow; i += 32) ex[i] = ~0ull;
        __syncwarp();
        warp_bitonic_sort(ex, ppow);
        if (lane == 0) atomicAdd(n_fallback, 1);
    }
    for (int j = lane; j < P; j += 32) {
        const unsigned long long e = ex[j];
        out_ids[(size_t)q * P + j] = (uint32_t)(e & 0xffffffffu);
        out_d[(size_t)q * P + j] = key2f((uint32_t)(e >> 32));
    }
}

// ---- host side ---------------------------------------------------------------

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

static int make_map(CUtensorMap* m, const void* base, long long rows, int kpad, int box_rows) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(FG_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
    if (!aligned(base, 16)) return fail(FG_ERR_INVALID_ARG, "TMA operand not 16-byte aligned");
    cuuint64_t dims[2] = {(cuuint64_t)kpad, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)kpad * 2};
    cuuint32_t box[2] = {TC_KB, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(FG_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return FG_OK;
}

bool coarse_tc_supported(int dim, int P) {
    const int S = std::max(2 * P, P + 32);
    return tc_kpad(dim) / TC_KB <= TC_MAX_KB && S <= TC_MAX_S;
}

namespace {
// Persistent GEMM grid: the (query tile, centroid tile) pairs split into
// contiguous ranges of `per_cta`, one per CTA, at most one CTA per SM.
struct GemmGrid {
    int ntiles;       // centroid tiles
    long long total;  // pairs
    int per_cta, ctas, maxseg;
};

GemmGrid gemm_grid(long long nq, int ncols) {
    GemmGrid gg;
    int nsm = device_attr(cudaDevAttrMultiProcessorCount);
    if (nsm <= 0) nsm = 148;
    const long long mtiles = (std::max(nq, 1ll) + TC_M - 1) / TC_M;
    gg.ntiles = (ncols + TC_N - 1) / TC_N;
    gg.total = mtiles * gg.ntiles;
    gg.per_cta = (int)((gg.total + nsm - 1) / nsm);
    gg.ctas = (int)((gg.total + gg.per_cta - 1) / gg.per_cta);
    // a query tile's ntiles pairs touch at most ceil(ntiles / L) + 1 ranges
    gg.maxseg = std::min(gg.ctas, (gg.ntiles + gg.per_cta - 1) / gg.per_cta + 1);
    return gg;
}

struct CoarsePlan {
    int S;       // exactly rescored superset
    int NS;      // prefix of centroids whose S-th smallest d~ bounds the S-th over all
    int cap;     // capacity of one (query, segment, part) list
    GemmGrid g1;  // the pass over every centroid
    int nlists;   // lists per query: g1.maxseg * TC_PARTS
    int fin_cta;
};

CoarsePlan coarse_plan(long long nq, int nlist, int P) {
    CoarsePlan c;
    c.S = std::min(nlist, std::max(2 * P, P + 32));
    int ns = std::max({1024, 8 * c.S, nlist / 8});
    ns = (ns + TC_N - 1) / TC_N * TC_N;
    c.NS = std::min(nlist, std::min(ns, 8192));
    const long long expect = (long long)c.S * nlist / c.NS;
    c.g1 = gemm_grid(nq, nlist);
    c.nlists = c.g1.maxseg * TC_PARTS;
    c.cap = (int)std::min<long long>(FIN_TOT, std::max<long long>(4 * expect, c.S + 256));
    c.cap = std::min(c.cap, std::max(topk_len(TC_TOPK_MAXP), std::min(c.g1.per_cta, c.g1.ntiles) * TC_CPW));
    c.fin_cta = (int)((std::max(nq, 1ll) + FIN_WARPS - 1) / FIN_WARPS);
    return c;
}
}  // namespace

size_t coarse_tc_workspace(long long nq, int nlist, int dim, int P) {
    const int kpad = tc_kpad(dim);
    const CoarsePlan c = coarse_plan(nq, nlist, P);
    size_t b = 0;
    b += round_up(round_up((size_t)nq, TC_TILE) * kpad * 2, 256) + round_up(round_up((size_t)nlist, TC_TILE) * kpad * 2, 256);
    b += round_up((size_t)nq * 4, 256) * 2 + round_up((size_t)nlist * 4, 256) + 256 * 3;
    b += round_up((size_t)nq * round_up(c.NS, 4) * 4, 256);     // prefix keys
    b += round_up((size_t)nq * c.nlists * 4, 256);              // list counts
    b += round_up((size_t)nq * c.nlists * c.cap * 4, 256) * 2;  // lists
    b += round_up((size_t)c.fin_cta * FIN_WARPS * nlist * 4, 256);  // fallback rows
    return b + 4096;
}

int coarse_tc(const float* centroids, int nlist, int dim, const float* queries, long long nq, int P,
              uint32_t* out_ids, float* out_d, void* ws, size_t ws_bytes, cudaStream_t s, int* n_fallback_host) {
    const int kpad = tc_kpad(dim);
    const int kt = kpad / TC_KB;
    if (!coarse_tc_supported(dim, P))
        return fail(FG_ERR_UNSUPPORTED, "tensor-core coarse path needs 3*dim <= 384 and top_m <= 256");
    if (nq > 0x7fffffffll) return fail(FG_ERR_INVALID_ARG, "too many queries");
    const CoarsePlan c = coarse_plan(nq, nlist, P);
    const long long nq_pad = (long long)round_up((size_t)nq, TC_TILE);
    const long long nl_pad = (long long)round_up((size_t)nlist, TC_TILE);
    Carve cv(ws, ws_bytes);
    __nv_bfloat16* A = cv.take<__nv_bfloat16>((size_t)nq_pad * kpad);
    __nv_bfloat16* B = cv.take<__nv_bfloat16>((size_t)nl_pad * kpad);
    float* qn = cv.take<float>((size_t)nq);
    float* tq = cv.take<float>((size_t)nq);
    float* cn = cv.take<float>((size_t)nlist);
    unsigned* maxc = cv.take<unsigned>(4);
    int* err = cv.take<int>(4);
    int* nfb = cv.take<int>(4);
    const long long ldm = (long long)round_up((size_t)c.NS, 4);
    uint32_t* M0 = cv.take<uint32_t>((size_t)nq * ldm);
    int* cnt = cv.take<int>((size_t)nq * c.nlists);
    uint32_t* lk = cv.take<uint32_t>((size_t)nq * c.nlists * c.cap);
    int32_t* li = cv.take<int32_t>((size_t)nq * c.nlists * c.cap);
    uint32_t* fb = cv.take<uint32_t>((size_t)c.fin_cta * FIN_WARPS * nlist);
    if (!cv.ok()) return fail(FG_ERR_WORKSPACE, "coarse workspace too small (%zu < %zu)", ws_bytes,
                              coarse_tc_workspace(nq, nlist, dim, P));
    FG_CUDA_TRY(cudaMemsetAsync(maxc, 0, 4, s));
    FG_CUDA_TRY(cudaMemsetAsync(err, 0, 4, s));
    FG_CUDA_TRY(cudaMemsetAsync(nfb, 0, 4, s));
    if (nq_pad > nq) FG_CUDA_TRY(cudaMemsetAsync(A + (size_t)nq * kpad, 0, (size_t)(nq_pad - nq) * kpad * 2, s));
    if (nl_pad > nlist)
        FG_CUDA_TRY(cudaMemsetAsync(B + (size_t)nlist * kpad, 0, (size_t)(nl_pad - nlist) * kpad * 2, s));
    split_bf16_kernel<<<(unsigned)((nlist + 7) / 8), 256, 0, s>>>(centroids, nlist, dim, kpad, 1, B, cn, maxc);
    int rc = check_launch("split_bf16_kernel(centroids)");
    if (rc) return rc;
    split_bf16_kernel<<<(unsigned)((nq + 7) / 8), 256, 0, s>>>(queries, nq, dim, kpad, 0, A, qn, nullptr);
    if ((rc = check_launch("split_bf16_kernel(queries)"))) return rc;
    CUtensorMap ta, tb;
    if ((rc = make_map(&ta, A, nq_pad, kpad, TC_M))) return rc;
    if ((rc = make_map(&tb, B, nl_pad, kpad, TC_N))) return rc;
    const int smem_base = 1024 + kt * TC_M * TC_KB * 2 + TC_NST * TC_GRP * TC_N * TC_KB * 2;

    GemmArgs g{};
    g.kt = kt;
    g.q0 = 0;
    g.nq = (int)nq;
    g.qn = qn;
    g.cn = cn;
    g.err = err;
    // Sets the launch's columns and range split; returns its dynamic shared
    // memory, which holds the column norms too where they fit.
    auto set_grid = [&](const GemmGrid& gg, int ncols) {
        g.ncols = ncols;
        g.ntiles = gg.ntiles;
        g.total = gg.total;
        g.per_cta = gg.per_cta;
        g.maxseg = gg.maxseg;
        const int norm_bytes = gg.ntiles * TC_N * (int)sizeof(float);
        g.norm_smem = smem_base + norm_bytes <= TC_SMEM_MAX;
        return g.norm_smem ? smem_base + norm_bytes : smem_base;
    };

    const int T = topk_len(P);
    const int topk_fsm = FIN_WARPS * ((dim + 3) / 4 * 4 * 4 + 256 * 4 + next_pow2(c.nlists * T) * 8);
    if (P <= TC_TOPK_MAXP && topk_fsm <= 227 * 1024) {
        // single pass: each (query, segment, part) keeps its T smallest d~ in
        // registers; a warp per query rescores and certifies them.  Lists of
        // segments that no CTA covers stay empty (ids -1).
        FG_CUDA_TRY(cudaMemsetAsync(li, 0xff, (size_t)nq * c.nlists * T * sizeof(int32_t), s));
        const int smem1 = set_grid(c.g1, nlist);
        g.list_k = lk;
        g.list_i = li;
        if (T == 4) {
            FG_CUDA_TRY(ensure_smem(reinterpret_cast<const void*>(&coarse_gemm_kernel<GEMM_TOPK, 4>), smem1));
            coarse_gemm_kernel<GEMM_TOPK, 4><<<c.g1.ctas, TC_NT, smem1, s>>>(ta, tb, g);
        } else {
            FG_CUDA_TRY(ensure_smem(reinterpret_cast<const void*>(&coarse_gemm_kernel<GEMM_TOPK, 8>), smem1));
            coarse_gemm_kernel<GEMM_TOPK, 8><<<c.g1.ctas, TC_NT, smem1, s>>>(ta, tb, g);
        }
        if ((rc = check_launch("coarse_gemm_kernel(top-k)"))) return rc;
        FG_CUDA_TRY(
            ensure_smem(reinterpret_cast<const void*>(&coarse_topk_finish_kernel), topk_fsm));
        coarse_topk_finish_kernel<<<c.fin_cta, FIN_WARPS * 32, topk_fsm, s>>>(
            centroids, nlist, dim, queries, (int)nq, c.nlists, T, lk, li, P, qn, maxc, err, fb, out_ids, out_d, nfb);
        if ((rc = check_launch("coarse_topk_finish_kernel"))) return rc;
        if (n_fallback_host) {
            FG_CUDA_TRY(cudaMemcpyAsync(n_fallback_host, nfb, sizeof(int), cudaMemcpyDeviceToHost, s));
            FG_CUDA_TRY(cudaStreamSynchronize(s));
        }
        return FG_OK;
    }

    // pass 0: keys of d~ to the first NS centroids, then the S-th smallest per query
    const GemmGrid g0 = gemm_grid(nq, c.NS);
    const int smem0 = set_grid(g0, c.NS);
    FG_CUDA_TRY(ensure_smem(reinterpret_cast<const void*>(&coarse_gemm_kernel<GEMM_MATRIX, 1>), smem0));
    g.out = M0;
    g.ldo = ldm;
    coarse_gemm_kernel<GEMM_MATRIX, 1><<<g0.ctas, TC_NT, smem0, s>>>(ta, tb, g);
    if ((rc = check_launch("coarse_gemm_kernel(prefix)"))) return rc;
    coarse_bound_kernel<<<(unsigned)((nq + 7) / 8), 256, 0, s>>>(M0, c.NS, ldm, (int)nq, c.S, tq);
    if ((rc = check_launch("coarse_bound_kernel"))) return rc;

    // pass 1: every centroid; each query row appends those within its bound
    // (counts of segments that no CTA covers stay 0)
    FG_CUDA_TRY(cudaMemsetAsync(cnt, 0, (size_t)nq * c.nlists * sizeof(int), s));
    const int smem1 = set_grid(c.g1, nlist);
    FG_CUDA_TRY(ensure_smem(reinterpret_cast<const void*>(&coarse_gemm_kernel<GEMM_FILTER, 1>), smem1));
    g.out = nullptr;
    g.tq = tq;
    g.cap = c.cap;
    g.cnt = cnt;
    g.list_k = lk;
    g.list_i = li;
    coarse_gemm_kernel<GEMM_FILTER, 1><<<c.g1.ctas, TC_NT, smem1, s>>>(ta, tb, g);
    if ((rc = check_launch("coarse_gemm_kernel(filter)"))) return rc;

    // pass 2: select, rescore exactly, certify (or fall back)
    const FinishSmem FL{(dim + 3) / 4 * 4, next_pow2(std::max(c.S, P)), c.nlists};
    const int fin_smem = FIN_WARPS * FL.per_warp_bytes();
    FG_CUDA_TRY(ensure_smem(reinterpret_cast<const void*>(&coarse_finish_kernel), fin_smem));
    coarse_finish_kernel<<<c.fin_cta, FIN_WARPS * 32, fin_smem, s>>>(centroids, nlist, dim, queries, (int)nq, cnt,
                                                                     c.nlists, lk, li, c.cap, c.S, P, qn, maxc, err,
                                                                     fb, out_ids, out_d, nfb);
    if ((rc = check_launch("coarse_finish_kernel"))) return rc;
    if (n_fallback_host) {
        FG_CUDA_TRY(cudaMemcpyAsync(n_fallback_host, nfb, sizeof(int), cudaMemcpyDeviceToHost, s));
        FG_CUDA_TRY(cudaStreamSynchronize(s));
    }
    return FG_OK;
}

}  // namespace fg

namespace fg {

// ---- k-means assignment on the tensor cores ------------------------------------
// The nearest centroid of every point is the coarse search with top_m = 1: the
// split-bf16 GEMM bounds and filters, the exact rescore (the same fmaf chain as
// l2_argmin) ranks by (distance, id) and the certificate or the exact fallback
// makes the result identical to l2_argmin's.  Points go through in chunks that
// keep the workspace near 1.5 GB.

static long long assign_chunk(long long n, int k, int dim) {
    const long long probe = 65536;
    const size_t per = coarse_tc_workspace(probe, k, dim, 1) / (size_t)probe + 8;
    long long r = (long long)(((size_t)1536 << 20) / std::max<size_t>(per, 1));
    r = std::max(4096ll, std::min(r, 262144ll));
    return std::max(1ll, std::min(r, n));
}

size_t assign_tc_workspace(long long n, int k, int dim) {
    const long long r = assign_chunk(n, k, dim);
    return coarse_tc_workspace(r, k, dim, 1) + round_up((size_t)r * 4, 256) + 512;
}

int assign_tc(const float* X, long long n, int dim, const float* C, int k, int32_t* out, void* ws, size_t ws_bytes,
              cudaStream_t s) {
    if (n <= 0) return FG_OK;
    const long long r = assign_chunk(n, k, dim);
    Carve cv(ws, ws_bytes);
    float* d = cv.take<float>((size_t)r);
    const size_t used = round_up(cv.used, 256);
    if (!cv.ok() || used > ws_bytes) return fail(FG_ERR_WORKSPACE, "assignment workspace too small");
    for (long long q0 = 0; q0 < n; q0 += r) {
        const long long nr = std::min(r, n - q0);
        const int rc = coarse_tc(C, k, dim, X + (size_t)q0 * dim, nr, 1, reinterpret_cast<uint32_t*>(out + q0), d,
                                 static_cast<char*>(ws) + used, ws_bytes - used, s, nullptr);
        if (rc) return rc;
    }
    return FG_OK;
}

}  // namespace fg
