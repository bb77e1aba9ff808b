// rerank.cu -- exact rerank of the candidate list (replaces run_gpu_rerank /
// heuristic_rerank_kernel, gpu_global.cu:603-673).
//
// One CTA per query walks the candidates in mini-batches of `mini_batch`
// inside a single launch (the reference launches once per mini-batch).  Each
// mini-batch: exact squared L2 of the new candidates against the raw base
// vectors (fmaf in dimension order, as nvcc compiles the reference's
// `local_d += diff*diff`), a stable merge of [running top-k ; new] by
// distance, and the reference's early stop: when at most epsilon*k of the
// new top-k ids were absent from the previous top-k, the stable counter
// grows, otherwise it resets; at `beta` the query is finished.
//
// ref_compat reproduces the reference's 128-thread block sort, which only
// sees the first 128 entries of the k + mini_batch window (gpu_global.cu:644-650).
#include "fg_common.cuh"

namespace fg {

constexpr int RR_NT = 256;

struct RerankArgs {
    const float* queries;
    int dim;
    const int32_t* top_ids;
    const int32_t* top_counts;
    int rm;
    const void* base;  // [nbase][dim] float or uint8
    long long nbase;
    int k, mb, nw;
    float eps;
    int beta;
    int32_t* out_ids;
    float* out_dists;
};

// Exact squared L2 in dimension order (fmaf, as nvcc contracts the reference's
// `local_d += diff*diff`), eight 16-byte loads in flight.
__device__ __forceinline__ float exact_l2(const float* __restrict__ sq, const float* __restrict__ v, int dim) {
    float d = 0.0f;
    if ((dim & 3) == 0) {
        const float4* v4 = reinterpret_cast<const float4*>(v);
        const int n4 = dim >> 2;
        int t = 0;
        for (; t + 8 <= n4; t += 8) {
            float4 x[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) x[u] = __ldg(v4 + t + u);
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const float4 q = *reinterpret_cast<const float4*>(sq + 4 * (t + u));
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
            const float4 x = __ldg(v4 + t);
            const float4 q = *reinterpret_cast<const float4*>(sq + 4 * t);
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
            const float df = sq[t] - __ldg(v + t);
            d = fmaf(df, df, d);
        }
    }
    return d;
}

// The same for uint8 rows (C5's raw vectors): each byte converts exactly to
// float, so the result equals exact_l2 on a float copy.  Sixteen bytes per load.
__device__ __forceinline__ float exact_l2(const float* __restrict__ sq, const uint8_t* __restrict__ v, int dim) {
    float d = 0.0f;
    if ((dim & 15) == 0) {
        const uint4* v16 = reinterpret_cast<const uint4*>(v);
        const int n16 = dim >> 4;
        int t = 0;
        for (; t + 4 <= n16; t += 4) {
            uint4 x[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) x[u] = __ldg(v16 + t + u);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const uint32_t w[4] = {x[u].x, x[u].y, x[u].z, x[u].w};
#pragma unroll
                for (int e = 0; e < 16; ++e) {
                    const float xv = (float)((w[e >> 2] >> (8 * (e & 3))) & 0xffu);
                    const float df = sq[16 * (t + u) + e] - xv;
                    d = fmaf(df, df, d);
                }
            }
        }
        for (; t < n16; ++t) {
            const uint4 x = __ldg(v16 + t);
            const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const float xv = (float)((w[e >> 2] >> (8 * (e & 3))) & 0xffu);
                const float df = sq[16 * t + e] - xv;
                d = fmaf(df, df, d);
            }
        }
    } else {
        for (int t = 0; t < dim; ++t) {
            const float df = sq[t] - (float)__ldg(v + t);
            d = fmaf(df, df, d);
        }
    }
    return d;
}

template <class T>
__global__ void __launch_bounds__(RR_NT) rerank_kernel(const RerankArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int warp[RR_NT / 32];
    __shared__ int s_stab;
    float* s_q = reinterpret_cast<float*>(smem);
    const int dim4 = (a.dim + 3) / 4 * 4;
    float* fd = s_q + dim4;          // running top-k distances (ascending)
    int32_t* fid = reinterpret_cast<int32_t*>(fd + a.k);
    float* wd = reinterpret_cast<float*>(fid + a.k);  // this mini-batch's candidates
    int32_t* wi = reinterpret_cast<int32_t*>(wd + a.mb);
    float* nd = reinterpret_cast<float*>(wi + a.mb);  // merged top-k
    int32_t* ni = reinterpret_cast<int32_t*>(nd + a.k);

    const int q = blockIdx.x, tid = threadIdx.x, k = a.k;
    const float* qv = a.queries + (size_t)q * a.dim;
    for (int t = tid; t < a.dim; t += RR_NT) s_q[t] = qv[t];
    for (int t = tid; t < k; t += RR_NT) {
        fd[t] = FLT_MAX;
        fid[t] = -1;
    }
    if (tid == 0) s_stab = 0;
    __syncthreads();
    const int total = a.top_counts[q];

    for (int off = 0; off < a.rm; off += a.mb) {
        if (off >= total) break;
        const int eff = min(a.mb, total - off);
        // The window is [top-k ; mini-batch].  Its tail past eff is (FLT_MAX, -1)
        // padding, which sorts after k earlier entries and can never enter the
        // top-k, so only m = min(eff, nw - k) new entries take part.
        const int m = min(eff, a.nw - k);
        for (int i = tid; i < m; i += RR_NT) {
            const int32_t vid = a.top_ids[(size_t)q * a.rm + off + i];
            float dist = FLT_MAX;
            if (vid >= 0 && (long long)vid < a.nbase)
                dist = exact_l2(s_q, static_cast<const T*>(a.base) + (size_t)vid * a.dim, a.dim);
            wd[i] = dist;
            wi[i] = vid;
        }
        __syncthreads();
        // stable ranks: old entries come before new ones on equal distance
        for (int j = tid; j < k; j += RR_NT) {  // old entry j (the top-k is sorted)
            const float d = fd[j];
            int r = j;
            for (int u = 0; u < m; ++u) r += wd[u] < d;
            if (r < k) {
                nd[r] = d;
                ni[r] = fid[j];
            }
        }
        for (int i = tid; i < m; i += RR_NT) {  // new entry i
            const float d = wd[i];
            int lo = 0, hi = k;  // old entries with distance <= d
            while (lo < hi) {
                const int mid = (lo + hi) >> 1;
                if (fd[mid] <= d) lo = mid + 1; else hi = mid;
            }
            int r = lo;
            for (int u = 0; u < m; ++u) {
                const float du = wd[u];
                r += (du < d) || (du == d && u < i);
            }
            if (r < k) {
                nd[r] = d;
                ni[r] = wi[i];
            }
        }
        __syncthreads();
        int ch = 0;
        for (int i = tid; i < k; i += RR_NT) {
            const int32_t nid = ni[i];
            if (nid == -1) continue;
            bool found = false;
            for (int j = 0; j < k; ++j)
                if (fid[j] == nid) {
                    found = true;
                    break;
                }
            ch += found ? 0 : 1;
        }
        int chg;
        (void)block_exclusive_scan<RR_NT>(ch, warp, chg);
        if (tid == 0) {
            if ((float)chg / (float)k <= a.eps)
                s_stab++;
            else
                s_stab = 0;
        }
        for (int i = tid; i < k; i += RR_NT) {
            fd[i] = nd[i];
            fid[i] = ni[i];
        }
        __syncthreads();
        if (s_stab >= a.beta) break;
    }
    for (int i = tid; i < k; i += RR_NT) {
        a.out_ids[(size_t)q * k + i] = fid[i];
        a.out_dists[(size_t)q * k + i] = fd[i];
    }
}

int rerank(const float* queries, int nq, int dim, const int32_t* top_ids, const int32_t* top_counts,
           const void* base, int base_u8, long long nbase, const fg_search_params* p, int32_t* out_ids,
           float* out_dists, cudaStream_t stream) {
    FG_REQUIRE(p, "null params");
    FG_REQUIRE(nq >= 0 && dim > 0, "bad nq/dim");
    FG_REQUIRE(p->final_k >= 1 && p->mini_batch >= 1 && p->rerank_m >= 1, "final_k, mini_batch, rerank_m must be >= 1");
    FG_REQUIRE(!p->ref_compat || p->final_k <= 128,
               "ref_compat needs final_k <= 128 (the reference's block sort has 128 slots)");
    if (nq == 0) return FG_OK;
    FG_REQUIRE(queries && top_ids && top_counts && base && out_ids && out_dists, "null buffer");
    FG_REQUIRE(dim % 4 != 0 || aligned(queries, 16), "queries must be 16-byte aligned");
    FG_REQUIRE(dim % (base_u8 ? 16 : 4) != 0 || aligned(base, 16), "base must be 16-byte aligned");
    RerankArgs a;
    a.queries = queries;
    a.dim = dim;
    a.top_ids = top_ids;
    a.top_counts = top_counts;
    a.rm = p->rerank_m;
    a.base = base;
    a.nbase = nbase;
    a.k = p->final_k;
    a.mb = p->mini_batch;
    a.nw = a.k + a.mb;
    if (p->ref_compat && a.nw > 128) a.nw = 128;
    a.eps = p->epsilon;
    a.beta = p->beta;
    a.out_ids = out_ids;
    a.out_dists = out_dists;
    const size_t smem = (size_t)((dim + 3) / 4 * 4) * 4 + (size_t)a.k * 16 + (size_t)a.mb * 8;
    int dev = 0, smem_max = 0;
    FG_CUDA_TRY(cudaGetDevice(&dev));
    FG_CUDA_TRY(cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    if (smem > (size_t)smem_max - 1024)
        return fail(FG_ERR_UNSUPPORTED, "rerank needs %zu bytes of shared memory", smem);
    if (base_u8) {
        FG_CUDA_TRY(cudaFuncSetAttribute(rerank_kernel<uint8_t>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem));
        rerank_kernel<uint8_t><<<nq, RR_NT, smem, stream>>>(a);
    } else {
        FG_CUDA_TRY(cudaFuncSetAttribute(rerank_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem));
        rerank_kernel<float><<<nq, RR_NT, smem, stream>>>(a);
    }
    return check_launch("rerank_kernel");
}

}  // namespace fg
