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
// The candidate rows of a mini-batch are first copied into shared memory by
// the whole CTA (coalesced 16-byte loads, all in flight together); each
// distance chain then runs from shared memory.  The counter is not evaluated
// on the last mini-batch, where it cannot change the result.
//
// ref_compat reproduces the reference's 128-thread block sort, which only
// sees the first 128 entries of the k + mini_batch window (gpu_global.cu:644-650).
#include <algorithm>
#include <cstdlib>

#include "fg_common.cuh"

namespace fg {

constexpr int RR_NT = 128;

struct RerankArgs {
    const float* queries;
    int dim;
    const int32_t* top_ids;
    const int32_t* top_counts;
    int rm;
    const void* base;  // [nbase][dim] float or uint8
    long long nbase;
    int k, mb, nw;
    int rch;  // candidate rows staged in shared memory at a time
    float eps;
    int beta;
    int32_t* out_ids;
    float* out_dists;
};

// Shared-memory layout of the rerank CTA; every array starts on 16 bytes.
struct RerankLayout {
    int q, fd, fid, wd, wi, nd, ni, rows, fixed;
};

__host__ __device__ inline RerankLayout rerank_layout(int dim, int k, int mb) {
    auto r16 = [](int b) { return (b + 15) / 16 * 16; };
    RerankLayout L;
    int o = 0;
    L.q = o;
    o += r16(dim * 4);
    L.fd = o;
    o += r16(k * 4);
    L.fid = o;
    o += r16(k * 4);
    L.wd = o;
    o += r16(((mb + 3) & ~3) * 4);
    L.wi = o;
    o += r16(mb * 4);
    L.nd = o;
    o += r16(k * 4);
    L.ni = o;
    o += r16(k * 4);
    L.rows = o;
    L.fixed = o;
    return L;
}

// Candidate rows staged in shared memory: a float row is dim floats, a uint8
// row dim bytes, each padded to an odd number of 16-byte units so that the
// lanes of a quarter-warp reading their own rows hit distinct banks.
template <class T>
__host__ __device__ inline int row_stride_bytes(int dim) {
    const int u = ((int)sizeof(T) * dim + 15) / 16;
    return ((u & 1) ? u : u + 1) * 16;
}

// Exact squared L2 of a candidate row in shared memory, in dimension order
// (fmaf, as nvcc contracts the reference's `local_d += diff*diff`).
__device__ __forceinline__ float exact_l2_row(const float* __restrict__ sq, const float* __restrict__ v, int dim) {
    float d = 0.0f;
    if ((dim & 3) == 0) {
#pragma unroll 8
        for (int t = 0; t < dim; t += 4) {
            const float4 x = *reinterpret_cast<const float4*>(v + t);
            const float4 q = *reinterpret_cast<const float4*>(sq + t);
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
            const float df = sq[t] - v[t];
            d = fmaf(df, df, d);
        }
    }
    return d;
}

// The same for uint8 rows (C5's raw vectors): each byte converts exactly to
// float, so the result equals the float version on a float copy.
__device__ __forceinline__ float exact_l2_row(const float* __restrict__ sq, const uint8_t* __restrict__ v, int dim) {
    float d = 0.0f;
    if ((dim & 15) == 0) {
#pragma unroll 2
        for (int t = 0; t < dim; t += 16) {
            const uint4 x = *reinterpret_cast<const uint4*>(v + t);
            const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                const float xv = (float)((w[e >> 2] >> (8 * (e & 3))) & 0xffu);
                const float df = sq[t + e] - xv;
                d = fmaf(df, df, d);
            }
        }
    } else {
        for (int t = 0; t < dim; ++t) {
            const float df = sq[t] - (float)v[t];
            d = fmaf(df, df, d);
        }
    }
    return d;
}

// Copies rows [c0, c0 + nr) of this mini-batch (ids in wi) into `rows` with
// asynchronous 16-byte copies: every copy of the chunk is in flight at once,
// so a chunk costs about one memory latency.  Rows of invalid ids are skipped.
// The caller waits (cp_async_wait_all) and synchronises before reading.
template <class T>
__device__ __forceinline__ void stage_rows(const RerankArgs& a, const int32_t* wi, int c0, int nr,
                                           unsigned char* rows, int stride) {
    const int row_bytes = (int)sizeof(T) * a.dim;
    if ((row_bytes & 15) == 0) {
        const int per_row = row_bytes >> 4;
        const int total = nr * per_row;
        const bool pow2 = (per_row & (per_row - 1)) == 0;
        const int sh = pow2 ? __ffs(per_row) - 1 : 0;
        for (int e = threadIdx.x; e < total; e += RR_NT) {
            const int r = pow2 ? e >> sh : e / per_row, c = e - r * per_row;
            const int32_t vid = wi[c0 + r];
            if (vid >= 0 && (long long)vid < a.nbase) {
                const unsigned char* src = static_cast<const unsigned char*>(a.base) + (size_t)vid * row_bytes + 16 * c;
                const uint32_t dst = (uint32_t)__cvta_generic_to_shared(rows + (size_t)r * stride + 16 * c);
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
            }
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    } else {
        const int total = nr * a.dim;
        for (int e = threadIdx.x; e < total; e += RR_NT) {
            const int r = e / a.dim, c = e - r * a.dim;
            const int32_t vid = wi[c0 + r];
            if (vid >= 0 && (long long)vid < a.nbase)
                reinterpret_cast<T*>(rows + (size_t)r * stride)[c] =
                    static_cast<const T*>(a.base)[(size_t)vid * a.dim + c];
        }
    }
}

__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

template <class T>
__global__ void __launch_bounds__(RR_NT, 8) rerank_kernel(const RerankArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int warp[RR_NT / 32];
    __shared__ int s_stab;
    const RerankLayout L = rerank_layout(a.dim, a.k, a.mb);
    float* s_q = reinterpret_cast<float*>(smem + L.q);
    float* fd = reinterpret_cast<float*>(smem + L.fd);      // running top-k distances (ascending)
    int32_t* fid = reinterpret_cast<int32_t*>(smem + L.fid);
    float* wd = reinterpret_cast<float*>(smem + L.wd);      // this mini-batch's candidates (+inf padded to 4)
    int32_t* wi = reinterpret_cast<int32_t*>(smem + L.wi);
    float* nd = reinterpret_cast<float*>(smem + L.nd);      // merged top-k
    int32_t* ni = reinterpret_cast<int32_t*>(smem + L.ni);
    unsigned char* rows = smem + L.rows;                     // [a.rch][stride]
    const int stride = row_stride_bytes<T>(a.dim);

    const int q = blockIdx.x, tid = threadIdx.x, k = a.k;
    const int total = a.top_counts[q];
    const float* qv = a.queries + (size_t)q * a.dim;
    for (int t = tid; t < a.dim; t += RR_NT) s_q[t] = qv[t];
    for (int t = tid; t < k; t += RR_NT) {
        fd[t] = FLT_MAX;
        fid[t] = -1;
    }
    if (tid == 0) s_stab = 0;
    // the first mini-batch's ids are read alongside the count, before it is
    // known how many are valid (the row holds rm entries; extra ones are unused)
    const int m_first = min(min(a.mb, a.nw - k), a.rm);
    for (int i = tid; i < m_first; i += RR_NT) wi[i] = a.top_ids[(size_t)q * a.rm + i];
    __syncthreads();

    bool result_in_n = false;  // the last mini-batch leaves the result in nd/ni
    for (int off = 0; off < a.rm; off += a.mb) {
        if (off >= total) break;
        const int eff = min(a.mb, total - off);
        // The window is [top-k ; mini-batch].  Its tail past eff is (FLT_MAX, -1)
        // padding, which sorts after k earlier entries and can never enter the
        // top-k, so only m = min(eff, nw - k) new entries take part.
        const int m = min(eff, a.nw - k);
        if (off > 0) {
            for (int i = tid; i < m; i += RR_NT) wi[i] = a.top_ids[(size_t)q * a.rm + off + i];
            __syncthreads();
        }
        for (int c0 = 0; c0 < m; c0 += a.rch) {
            const int nr = min(a.rch, m - c0);
            stage_rows<T>(a, wi, c0, nr, rows, stride);
            cp_async_wait_all();
            __syncthreads();
            for (int i = tid; i < nr; i += RR_NT) {
                const int32_t vid = wi[c0 + i];
                wd[c0 + i] = (vid >= 0 && (long long)vid < a.nbase)
                                 ? exact_l2_row(s_q, reinterpret_cast<const T*>(rows + (size_t)i * stride), a.dim)
                                 : FLT_MAX;
            }
            __syncthreads();
        }
        // +inf padding to a multiple of 4 ranks below no distance (all are
        // finite: exact or FLT_MAX)
        const int m4 = (m + 3) & ~3;
        if (tid < m4 - m) wd[m + tid] = INFINITY;
        __syncthreads();
        // stable ranks, old and new entries at once: old entries come before
        // new ones on equal distance, new ones keep their order.  In the first
        // mini-batch every old entry is (FLT_MAX, -1): the merged list is those
        // placeholders with each finite new entry at its rank among the new ones.
        const float4* w4 = reinterpret_cast<const float4*>(wd);
        const bool first_batch = off == 0;
        if (first_batch) {
            for (int t = tid; t < k; t += RR_NT) {
                nd[t] = FLT_MAX;
                ni[t] = -1;
            }
            __syncthreads();
        }
        for (int t = first_batch ? k + tid : tid; t < k + m; t += RR_NT) {
            if (t < k) {  // old entry t (the top-k is sorted)
                const float d = fd[t];
                int r = t;
#pragma unroll 4
                for (int u = 0; u < m4 / 4; ++u) {
                    const float4 x = w4[u];
                    r += (x.x < d) + (x.y < d) + (x.z < d) + (x.w < d);
                }
                if (r < k) {
                    nd[r] = d;
                    ni[r] = fid[t];
                }
            } else {  // new entry i
                const int i = t - k;
                const float d = wd[i];
                int lo = 0, hi = k;  // old entries with distance <= d
                if (first_batch) {
                    lo = d < FLT_MAX ? 0 : k;
                } else {
                    while (lo < hi) {
                        const int mid = (lo + hi) >> 1;
                        if (fd[mid] <= d) lo = mid + 1; else hi = mid;
                    }
                }
                int r = lo;
#pragma unroll 4
                for (int u = 0; u < m4 / 4; ++u) {
                    const float4 x = w4[u];
                    const int b = 4 * u;
                    r += (x.x < d) || (x.x == d && b < i);
                    r += (x.y < d) || (x.y == d && b + 1 < i);
                    r += (x.z < d) || (x.z == d && b + 2 < i);
                    r += (x.w < d) || (x.w == d && b + 3 < i);
                }
                if (r < k) {
                    nd[r] = d;
                    ni[r] = wi[i];
                }
            }
        }
        __syncthreads();
        // the stability counter only decides whether another mini-batch runs
        // (uniform over the block, so the scan's barriers are all or none)
        const bool last = off + a.mb >= total || off + a.mb >= a.rm;
        if (!last) {
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
        }
        if (last) {
            result_in_n = true;
            break;
        }
        for (int i = tid; i < k; i += RR_NT) {
            fd[i] = nd[i];
            fid[i] = ni[i];
        }
        __syncthreads();
        if (s_stab >= a.beta) break;
    }
    const float* rd = result_in_n ? nd : fd;
    const int32_t* ri = result_in_n ? ni : fid;
    for (int i = tid; i < k; i += RR_NT) {
        a.out_ids[(size_t)q * k + i] = ri[i];
        a.out_dists[(size_t)q * k + i] = rd[i];
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
    const int stride = base_u8 ? row_stride_bytes<uint8_t>(dim) : row_stride_bytes<float>(dim);
    const int mmax = std::max(1, std::min(a.mb, a.nw - a.k));  // new entries per mini-batch
    // about 24 KB of staged rows: eight 128-thread CTAs per SM (measured on C2
    // against 64 and 96 rows: 0.130 / 0.134 / 0.167 ms at nprobe 2, 0.61 / 0.66 /
    // 0.86 ms at nprobe 8)
    a.rch = std::max(8, std::min(mmax, 24576 / stride));
    if (const char* e = getenv("FG_RERANK_CHUNK")) a.rch = std::max(8, std::min(mmax, atoi(e)));  // tuning override
    const size_t smem = (size_t)rerank_layout(dim, a.k, a.mb).fixed + (size_t)a.rch * stride;
    int smem_max = 0;
    smem_max = device_attr(cudaDevAttrMaxSharedMemoryPerBlockOptin);
    if (smem > (size_t)smem_max - 1024)
        return fail(FG_ERR_UNSUPPORTED, "rerank needs %zu bytes of shared memory", smem);
    if (base_u8) {
        FG_CUDA_TRY(ensure_smem(reinterpret_cast<const void*>(&rerank_kernel<uint8_t>), (int)smem));
        rerank_kernel<uint8_t><<<nq, RR_NT, smem, stream>>>(a);
    } else {
        FG_CUDA_TRY(ensure_smem(reinterpret_cast<const void*>(&rerank_kernel<float>), (int)smem));
        rerank_kernel<float><<<nq, RR_NT, smem, stream>>>(a);
    }
    return check_launch("rerank_kernel");
}

}  // namespace fg
