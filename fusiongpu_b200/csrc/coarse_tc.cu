// coarse_tc.cu -- coarse quantizer on the 5th-generation tensor cores
// (replaces cuVS CAGRA search over the centroids, cagra_adapter.cuh:38-68).
//
// 1. Queries and centroids are split into bf16 hi + lo parts and laid out as
//    A = [q_hi | q_hi | q_lo], B = [c_hi | c_lo | c_hi] (K = 3*dim, zero padded to
//    a multiple of 64), so one bf16 GEMM A.B^T = q_hi.c_hi + q_hi.c_lo + q_lo.c_hi
//    approximates q.c to about 2^-16 relative.
// 2. coarse_gemm_kernel: one 128x128 tile per CTA, operands staged by TMA (128-byte
//    swizzle, no multicast), tcgen05.mma issued by one thread, accumulator in TMEM,
//    epilogue writes d~ = |q|^2 + |c|^2 - 2 q.c.
// 3. the S = max(2P, P+32) smallest d~ per query (two-stage radix select).
// 4. coarse_rescore_kernel: exact fp32 distances (the oracle's arithmetic) of the S
//    candidates, sorted by (distance, id).  The top P is certified exact when the
//    P-th exact distance is below the smallest excluded d~ minus an error bound
//    E(q) on |d~ - d|; otherwise (or if the GEMM reported a failed wait) the query is
//    rescored exactly against every centroid.  Rankings therefore equal the exact
//    ones bit for bit, whatever the tensor-core rounding.
#include <cuda_bf16.h>

#include <algorithm>

#include "fg_common.cuh"
#include "tc_common.cuh"

namespace fg {

int rows_topk(const float* v, long long ldv, long long rows, int ncols, int k, int32_t* out_i, float* out_v,
              long long out_ld, float* stage_v, int32_t* stage_i, cudaStream_t s);
size_t rows_topk_stage_bytes(long long rows, int ncols, int k);

constexpr int TC_TILE = 128;    // M = N = 128 per CTA
constexpr int TC_KB = 64;       // bf16 elements per K block (one 128-byte swizzle row)
constexpr int TC_MAX_KB = 6;    // all K blocks resident: 2 * 6 * 16 KB = 192 KB
constexpr int TC_NT = 128;
constexpr int RS_NT = 256;

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

__global__ void __launch_bounds__(TC_NT, 1)
    coarse_gemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, int kt,
                       long long q0, int nq_chunk, int nlist, const float* __restrict__ qn,
                       const float* __restrict__ cn, float* __restrict__ out, long long ldo, int* err) {
    extern __shared__ __align__(1024) unsigned char dsmem[];
    __shared__ __align__(8) uint64_t bars[2];
    __shared__ uint32_t tmem_slot;
    __shared__ int s_fail;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // 1024-byte aligned operand area: A blocks then B blocks, 16 KB each
    unsigned char* base = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(dsmem) + 1023) & ~static_cast<uintptr_t>(1023));
    unsigned char* sa = base;
    unsigned char* sb = base + kt * (TC_TILE * TC_KB * 2);
    const int m0 = blockIdx.x * TC_TILE;  // row inside the chunk
    const int n0 = blockIdx.y * TC_TILE;

    if (tid == 0) {
        s_fail = 0;
        tc::mbar_init(&bars[0], 1);
        tc::mbar_init(&bars[1], 1);
        tc::fence_mbar_init();
    }
    if (warp == 0) {
        tc::tmem_alloc(&tmem_slot, TC_TILE);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t taddr = tmem_slot;

    if (tid == 0) {
        tc::mbar_arrive_expect_tx(&bars[0], (uint32_t)(2 * kt * TC_TILE * TC_KB * 2));
        for (int k = 0; k < kt; ++k) {
            tc::tma_load_2d(sa + k * (TC_TILE * TC_KB * 2), &ta, &bars[0], k * TC_KB, (int)(q0 + m0));
            tc::tma_load_2d(sb + k * (TC_TILE * TC_KB * 2), &tb, &bars[0], k * TC_KB, n0);
        }
        if (tc::mbar_wait(&bars[0], 0)) {
            constexpr uint32_t idesc = tc::idesc_bf16_f32(TC_TILE, TC_TILE);
            for (int k = 0; k < kt; ++k) {
                const uint64_t da = tc::desc_kmajor_sw128(sa + k * (TC_TILE * TC_KB * 2));
                const uint64_t db = tc::desc_kmajor_sw128(sb + k * (TC_TILE * TC_KB * 2));
#pragma unroll
                for (int kk = 0; kk < TC_KB / 16; ++kk)  // K = 16 per MMA: +32 bytes in the swizzle row
                    tc::umma_bf16(taddr, da + 2 * kk, db + 2 * kk, idesc, (k | kk) != 0);
            }
            tc::umma_commit(&bars[1]);
        } else {
            s_fail = 1;
        }
    }
    __syncthreads();
    // block-uniform: the TMEM loads below are .sync.aligned
    const bool ok = __syncthreads_and(!s_fail && tc::mbar_wait(&bars[1], 0));
    tc::fence_after_sync();
    if (ok) {
        const int row = m0 + warp * 32 + lane;
        const float qnr = row < nq_chunk ? qn[q0 + row] : 0.0f;
#pragma unroll 1
        for (int c = 0; c < TC_TILE / 32; ++c) {
            float v[32];
            tc::tmem_ld_32x32(taddr + ((uint32_t)(warp * 32) << 16) + (uint32_t)(c * 32), v);
            if (row < nq_chunk) {
                float* o = out + (long long)row * ldo + n0 + c * 32;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int col = n0 + c * 32 + j;
                    if (col < nlist) o[j] = qnr + cn[col] - 2.0f * v[j];
                }
            }
        }
    }
    if (!ok && tid == 0) atomicExch(err, 1);
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(taddr, TC_TILE);
}

__device__ __forceinline__ float l2_seq_dev(const float* __restrict__ a_smem, const float* __restrict__ b, int dim) {
    float d = 0.0f;
    if ((dim & 3) == 0) {
        const float4* b4 = reinterpret_cast<const float4*>(b);
        for (int t = 0; t < dim / 4; ++t) {
            const float4 x = __ldg(b4 + t);
            const float4 q = *reinterpret_cast<const float4*>(a_smem + 4 * t);
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

// One CTA per query of the chunk: exact rescoring of the S candidates and the
// certificate; exact fallback over all centroids when it fails.
__global__ void __launch_bounds__(RS_NT) coarse_rescore_kernel(
    const float* __restrict__ centroids, int nlist, int dim, const float* __restrict__ queries, long long q0,
    const int32_t* __restrict__ cand_i, const float* __restrict__ cand_d, int S, int P,
    const float* __restrict__ qn, const unsigned* __restrict__ max_cn_bits, const int* __restrict__ err,
    uint32_t* __restrict__ row_keys, long long ldk, uint32_t* __restrict__ out_ids, float* __restrict__ out_d,
    int* __restrict__ n_fallback) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ uint32_t hist[256];
    __shared__ uint32_t sb[2];
    __shared__ int warp[RS_NT / 32];
    const int row = blockIdx.x;
    const long long q = q0 + row;
    const int tid = threadIdx.x;
    const int dim4 = (dim + 3) / 4 * 4;
    float* sq = reinterpret_cast<float*>(smem);
    unsigned long long* sk = reinterpret_cast<unsigned long long*>(smem + dim4 * 4 + (dim4 * 4 % 8));
    for (int t = tid; t < dim; t += RS_NT) sq[t] = queries[q * dim + t];
    __syncthreads();
    const int spow = next_pow2(S > P ? S : P);
    bool certified = false;
    if (*err == 0) {
        for (int i = tid; i < spow; i += RS_NT) {
            unsigned long long key = ~0ull;
            if (i < S) {
                const int cid = cand_i[(long long)row * S + i];
                if (cid >= 0 && cid < nlist)
                    key = ((unsigned long long)f2key(l2_seq_dev(sq, centroids + (size_t)cid * dim, dim)) << 32) |
                          (unsigned)cid;
            }
            sk[i] = key;
        }
        __syncthreads();
        block_bitonic_sort<RS_NT>(sk, spow);
        const float dp = key2f((uint32_t)(sk[P - 1] >> 32));
        const float T = cand_d[(long long)row * S + S - 1];
        const float qq = qn[q];
        const float cc = __uint_as_float(*max_cn_bits);
        const float E = 0x1p-12f * sqrtf(qq) * sqrtf(cc) + 0x1p-16f * (qq + cc);
        certified = (S >= nlist) || (dp < T - E);
    }
    if (!certified) {
        uint32_t* rk = row_keys + (long long)row * ldk;
        for (int c = tid; c < nlist; c += RS_NT) rk[c] = f2key(l2_seq_dev(sq, centroids + (size_t)c * dim, dim));
        __syncthreads();
        uint32_t kth;
        int n_less;
        block_radix_select<RS_NT>(rk, nlist, P, hist, sb, kth, n_less);
        const int need_eq = P - n_less;
        int eq_base = 0, out_base = 0;
        for (int r0 = 0; r0 < nlist; r0 += RS_NT) {
            const int c = r0 + tid;
            const bool in = c < nlist;
            const uint32_t key = in ? rk[c] : 0xffffffffu;
            const int is_eq = (in && key == kth) ? 1 : 0;
            int eq_tot, s_tot;
            const int eq_pre = block_exclusive_scan<RS_NT>(is_eq, warp, eq_tot);
            const bool sel = in && (key < kth || (is_eq && eq_base + eq_pre < need_eq));
            eq_base += eq_tot;
            const int s_pre = block_exclusive_scan<RS_NT>(sel ? 1 : 0, warp, s_tot);
            if (sel) sk[out_base + s_pre] = ((unsigned long long)key << 32) | (unsigned)c;
            out_base += s_tot;
        }
        const int ppow = next_pow2(P);
        for (int i = P + tid; i < ppow; i += RS_NT) sk[i] = ~0ull;
        __syncthreads();
        block_bitonic_sort<RS_NT>(sk, ppow);
        if (tid == 0) atomicAdd(n_fallback, 1);
    }
    for (int j = tid; j < P; j += RS_NT) {
        const unsigned long long e = sk[j];
        out_ids[q * P + j] = (uint32_t)(e & 0xffffffffu);
        out_d[q * P + j] = key2f((uint32_t)(e >> 32));
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

static int make_map(CUtensorMap* m, const void* base, long long rows, int kpad) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return fail(FG_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
    if (!aligned(base, 16)) return fail(FG_ERR_INVALID_ARG, "TMA operand not 16-byte aligned");
    cuuint64_t dims[2] = {(cuuint64_t)kpad, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)kpad * 2};
    cuuint32_t box[2] = {TC_KB, TC_TILE};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(FG_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return FG_OK;
}

bool coarse_tc_supported(int dim) { return tc_kpad(dim) / TC_KB <= TC_MAX_KB; }

static int superset(int P, int nlist) { return std::min(nlist, std::max(2 * P, P + 32)); }

static long long tc_chunk_rows(long long nq, int nlist) {
    long long r = std::max<long long>(128, (256ll << 20) / ((long long)nlist * 4));
    r = r / 128 * 128;
    return std::min(nq, r);
}

size_t coarse_tc_workspace(long long nq, int nlist, int dim, int P) {
    const int kpad = tc_kpad(dim);
    const int S = superset(P, nlist);
    const long long rows = tc_chunk_rows(std::max(nq, 1ll), nlist);
    size_t b = 0;
    b += round_up((size_t)round_up(nq, TC_TILE) * kpad * 2, 256) + round_up((size_t)round_up(nlist, TC_TILE) * kpad * 2, 256);
    b += round_up((size_t)nq * 4, 256) + round_up((size_t)nlist * 4, 256) + 256 * 3;
    b += round_up((size_t)rows * nlist * 4, 256);
    b += round_up((size_t)rows * S * 4, 256) * 2;
    b += rows_topk_stage_bytes(rows, nlist, S);
    return b + 2048;
}

int coarse_tc(const float* centroids, int nlist, int dim, const float* queries, long long nq, int P,
              uint32_t* out_ids, float* out_d, void* ws, size_t ws_bytes, cudaStream_t s, int* n_fallback_host) {
    const int kpad = tc_kpad(dim);
    const int kt = kpad / TC_KB;
    if (kt > TC_MAX_KB) return fail(FG_ERR_UNSUPPORTED, "tensor-core coarse path needs 3*dim <= 384");
    const int S = superset(P, nlist);
    const long long rows = tc_chunk_rows(nq, nlist);
    // operands padded to whole 128-row tiles (zero rows), so no TMA box exceeds its tensor
    const long long nq_pad = (long long)round_up((size_t)nq, TC_TILE);
    const long long nl_pad = (long long)round_up((size_t)nlist, TC_TILE);
    Carve cv(ws, ws_bytes);
    __nv_bfloat16* A = cv.take<__nv_bfloat16>((size_t)nq_pad * kpad);
    __nv_bfloat16* B = cv.take<__nv_bfloat16>((size_t)nl_pad * kpad);
    float* qn = cv.take<float>((size_t)nq);
    float* cn = cv.take<float>((size_t)nlist);
    unsigned* maxc = cv.take<unsigned>(4);
    int* err = cv.take<int>(4);
    int* nfb = cv.take<int>(4);
    float* M = cv.take<float>((size_t)rows * nlist);
    int32_t* ci = cv.take<int32_t>((size_t)rows * S);
    float* cd = cv.take<float>((size_t)rows * S);
    const size_t stage = rows_topk_stage_bytes(rows, nlist, S);
    float* sv = stage ? cv.take<float>(stage / 8) : nullptr;
    int32_t* si = stage ? cv.take<int32_t>(stage / 8) : nullptr;
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
    if ((rc = make_map(&ta, A, nq_pad, kpad))) return rc;
    if ((rc = make_map(&tb, B, nl_pad, kpad))) return rc;
    const int smem = 1024 + 2 * kt * TC_TILE * TC_KB * 2;
    FG_CUDA_TRY(cudaFuncSetAttribute(coarse_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    const int spow = next_pow2(std::max(S, P));
    const int rs_smem = ((dim + 3) / 4 * 4) * 4 + 8 + spow * 8;
    FG_CUDA_TRY(cudaFuncSetAttribute(coarse_rescore_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, rs_smem));
    for (long long q0 = 0; q0 < nq; q0 += rows) {
        const int r = (int)std::min(rows, nq - q0);
        dim3 grid((unsigned)((r + TC_TILE - 1) / TC_TILE), (unsigned)((nlist + TC_TILE - 1) / TC_TILE));
        coarse_gemm_kernel<<<grid, TC_NT, smem, s>>>(ta, tb, kt, q0, r, nlist, qn, cn, M, nlist, err);
        if ((rc = check_launch("coarse_gemm_kernel"))) return rc;
        if ((rc = rows_topk(M, nlist, r, nlist, S, ci, cd, S, sv, si, s))) return rc;
        coarse_rescore_kernel<<<r, RS_NT, rs_smem, s>>>(centroids, nlist, dim, queries, q0, ci, cd, S, P, qn, maxc,
                                                        err, reinterpret_cast<uint32_t*>(M), nlist, out_ids, out_d,
                                                        nfb);
        if ((rc = check_launch("coarse_rescore_kernel"))) return rc;
    }
    if (n_fallback_host) {
        FG_CUDA_TRY(cudaMemcpyAsync(n_fallback_host, nfb, sizeof(int), cudaMemcpyDeviceToHost, s));
        FG_CUDA_TRY(cudaStreamSynchronize(s));
    }
    return FG_OK;
}

}  // namespace fg
