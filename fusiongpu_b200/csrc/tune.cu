// tune.cu -- the search-parameter tuner (tune_parameters.cu:459-1013) on the GPU.
//
// For a sample of queries with exact ground truth it derives the four search
// parameters the reference's tune_parameters tool recommends:
//   top_m           P99.5 of the coarse rank of each true neighbour's list
//   p1_lists        elbow of the hits-per-coarse-rank histogram
//   limit_k         largest PQ rank (inside its own list) of the neighbours
//                   whose list is among the first p1_lists probes
//   threshold_coeff largest ratio of the farthest neighbour's PQ distance to
//                   the smallest phase-1 cutoff of its query
// The reference does this with one host loop per (query, neighbour) and a
// cudaMalloc + three tiny kernels per list; here every query (or pair) is one
// CTA: the coarse ranks, the PQ and exact ranks inside a list, and the
// phase-1 cutoffs (radix select over the list's PQ distances) each take one
// launch.  The expressions follow the reference's: the coarse distances are
// the host's (separate multiply and add), the LUT, PQ and exact distances its
// device kernels' (nvcc contracts `acc += d * d` into fmaf).
#include <algorithm>
#include <climits>
#include <cmath>
#include <vector>

#include "fg_common.cuh"

namespace fg {

constexpr int TU_NT = 256;
constexpr int32_t TU_NONE = 0x7f7f7f7f;  // "no list" (cudaMemset byte 0x7f)

__device__ __forceinline__ float l2_unfused(const float* a, const float* b, int dim) {
    float d = 0.0f;
    for (int j = 0; j < dim; ++j) {
        const float df = __fsub_rn(a[j], b[j]);
        d = __fadd_rn(d, __fmul_rn(df, df));
    }
    return d;
}

__device__ __forceinline__ float l2_fused(const float* a, const float* b, int dim) {
    float d = 0.0f;
    for (int j = 0; j < dim; ++j) {
        const float df = __fsub_rn(a[j], b[j]);
        d = __fmaf_rn(df, df, d);
    }
    return d;
}

// owner[id] = lowest list holding id (the reference's first-match scan over
// lists in order, tune_parameters.cu:548-559)
__global__ void tune_owner_kernel(const int32_t* __restrict__ offsets, const int32_t* __restrict__ ids,
                                  long long nbase, int32_t* __restrict__ owner) {
    const int c = blockIdx.x;
    for (int j = offsets[c] + threadIdx.x; j < offsets[c + 1]; j += blockDim.x) {
        const int32_t id = ids[j];
        if (id >= 0 && id < nbase) atomicMin(&owner[id], c);
    }
}

// firstpos[id] = first position of id inside its owner list
__global__ void tune_firstpos_kernel(const int32_t* __restrict__ offsets, const int32_t* __restrict__ ids,
                                     long long nbase, const int32_t* __restrict__ owner,
                                     int32_t* __restrict__ firstpos) {
    const int c = blockIdx.x;
    for (int j = offsets[c] + threadIdx.x; j < offsets[c + 1]; j += blockDim.x) {
        const int32_t id = ids[j];
        if (id >= 0 && id < nbase && owner[id] == c) atomicMin(&firstpos[id], j);
    }
}

__device__ __forceinline__ int32_t list_of(const int32_t* gt, long long nbase, const int32_t* owner, int nlist,
                                           size_t pair) {
    const int32_t id = gt[pair];
    if (id < 0 || id >= nbase) return -1;
    const int32_t c = owner[id];
    return (c >= 0 && c < nlist) ? c : -1;
}

// Coarse rank (1-based) of each neighbour's list among all lists ordered by
// (host distance, list id): one CTA per query.
__global__ void __launch_bounds__(TU_NT)
    tune_cluster_rank_kernel(const float* __restrict__ centroids, int nlist, int dim, const float* __restrict__ queries,
                             const int32_t* __restrict__ gt, int k, const int32_t* __restrict__ owner, long long nbase,
                             int32_t* __restrict__ out_rank) {
    extern __shared__ __align__(16) float tsm[];
    float* sq = tsm;
    float* td = sq + dim;
    int* tc = reinterpret_cast<int*>(td + k);
    unsigned* cnt = reinterpret_cast<unsigned*>(tc + k);
    const int q = blockIdx.x, lane = threadIdx.x & 31;
    for (int j = threadIdx.x; j < dim; j += TU_NT) sq[j] = queries[(size_t)q * dim + j];
    __syncthreads();
    for (int t = threadIdx.x; t < k; t += TU_NT) {
        const int c = list_of(gt, nbase, owner, nlist, (size_t)q * k + t);
        tc[t] = c;
        td[t] = c >= 0 ? l2_unfused(sq, centroids + (size_t)c * dim, dim) : 0.0f;
        cnt[t] = 0;
    }
    __syncthreads();
    for (int b0 = 0; b0 < nlist; b0 += TU_NT) {
        const int c = b0 + threadIdx.x;
        const bool ok = c < nlist;
        const float d = ok ? l2_unfused(sq, centroids + (size_t)c * dim, dim) : 0.0f;
        for (int t = 0; t < k; ++t) {
            const float dt = td[t];
            const int ct = tc[t];
            const bool before = ok && ct >= 0 && (d < dt || (d == dt && c < ct));
            const unsigned bal = __ballot_sync(0xffffffffu, before);
            if (lane == 0 && bal) atomicAdd(&cnt[t], (unsigned)__popc(bal));
        }
    }
    __syncthreads();
    for (int t = threadIdx.x; t < k; t += TU_NT)
        out_rank[(size_t)q * k + t] = tc[t] >= 0 ? (int32_t)cnt[t] + 1 : -1;
}

// LUT of (query, list c) as the tuner's precompute_lut_kernel computes it
// (tune_parameters.cu:98-121): residual first, then fmaf per sub-dimension.
__device__ void tune_lut(const float* sq, const float* __restrict__ cen, const float* __restrict__ codebook, int pq_m,
                         int sd, float* lut) {
    for (int e = threadIdx.x; e < pq_m * 256; e += TU_NT) {
        const int m = e >> 8;
        const float* cb = codebook + (size_t)e * sd;
        float acc = 0.0f;
        for (int d = 0; d < sd; ++d) {
            const float r = __fsub_rn(sq[m * sd + d], cen[m * sd + d]);
            const float df = __fsub_rn(r, cb[d]);
            acc = __fmaf_rn(df, df, acc);
        }
        lut[e] = acc;
    }
}

__device__ __forceinline__ float tune_pq(const uint8_t* __restrict__ code, const float* lut, int pq_m) {
    float s = 0.0f;
    for (int m = 0; m < pq_m; ++m) s = __fadd_rn(s, lut[(m << 8) + code[m]]);
    return s;
}

struct TuneIndex {
    const float* codebook;
    const int32_t* offsets;
    const uint8_t* codes;
    const int32_t* ids;
    const float* centroids;
    int nlist, dim, pq_m;
};

// PQ rank and exact rank of each neighbour inside its own list, and its PQ
// distance: one CTA per (query, neighbour).
__global__ void __launch_bounds__(TU_NT)
    tune_pq_rank_kernel(TuneIndex ix, const float* __restrict__ base, long long nbase, const float* __restrict__ queries,
                        const int32_t* __restrict__ gt, int k, const int32_t* __restrict__ owner,
                        const int32_t* __restrict__ firstpos, int32_t* __restrict__ out_pq_rank,
                        int32_t* __restrict__ out_ex_rank, float* __restrict__ out_pq) {
    extern __shared__ __align__(16) float tsm[];
    const int dim = ix.dim, pq_m = ix.pq_m, sd = dim / pq_m;
    float* lut = tsm;
    float* sq = lut + pq_m * 256;
    float* st = sq + dim;
    unsigned* red = reinterpret_cast<unsigned*>(st + 2);
    const size_t pair = blockIdx.x;
    const int q = (int)(pair / k);
    const int c = list_of(gt, nbase, owner, ix.nlist, pair);
    if (c < 0) {
        if (threadIdx.x == 0) {
            out_pq_rank[pair] = -1;
            out_ex_rank[pair] = -1;
            out_pq[pair] = -1.0f;
        }
        return;
    }
    const int32_t id = gt[pair];
    for (int j = threadIdx.x; j < dim; j += TU_NT) sq[j] = queries[(size_t)q * dim + j];
    if (threadIdx.x < 2) red[threadIdx.x] = 0;
    __syncthreads();
    tune_lut(sq, ix.centroids + (size_t)c * dim, ix.codebook, pq_m, sd, lut);
    __syncthreads();
    if (threadIdx.x == 0) {
        st[0] = tune_pq(ix.codes + (size_t)firstpos[id] * pq_m, lut, pq_m);
        st[1] = l2_fused(sq, base + (size_t)id * dim, dim);
    }
    __syncthreads();
    const float pt = st[0], et = st[1];
    unsigned npq = 0, nex = 0;
    for (int j = ix.offsets[c] + threadIdx.x; j < ix.offsets[c + 1]; j += TU_NT) {
        npq += tune_pq(ix.codes + (size_t)j * pq_m, lut, pq_m) < pt ? 1u : 0u;
        const int32_t v = ix.ids[j];
        if (v >= 0 && v < nbase) nex += l2_fused(sq, base + (size_t)v * dim, dim) < et ? 1u : 0u;
    }
    for (int o = 16; o; o >>= 1) {
        npq += __shfl_xor_sync(0xffffffffu, npq, o);
        nex += __shfl_xor_sync(0xffffffffu, nex, o);
    }
    if ((threadIdx.x & 31) == 0) {
        atomicAdd(&red[0], npq);
        atomicAdd(&red[1], nex);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        out_pq_rank[pair] = (int32_t)red[0] + 1;
        out_ex_rank[pair] = (int32_t)red[1] + 1;
        out_pq[pair] = pt;
    }
}

// Smallest phase-1 cutoff of each query: over the first P lists by (host
// distance, id), the (min(limit_k, len) )-th smallest PQ distance of each
// non-empty list (tune_parameters.cu:830-890).  NaN when every list is empty.
// `rows`: one uint32 scratch row of `ldr` >= max(nlist, longest list) per CTA;
// `sel`: P ints per CTA.
__global__ void __launch_bounds__(TU_NT)
    tune_cutoff_kernel(TuneIndex ix, const float* __restrict__ queries, int q0, int P, int limit_k,
                       uint32_t* __restrict__ rows, size_t ldr, int32_t* __restrict__ sel, float* __restrict__ out_cut) {
    extern __shared__ __align__(16) float tsm[];
    const int dim = ix.dim, pq_m = ix.pq_m, sd = dim / pq_m, nlist = ix.nlist;
    float* lut = tsm;
    float* sq = lut + pq_m * 256;
    uint32_t* hist = reinterpret_cast<uint32_t*>(sq + dim);
    uint32_t* sb = hist + 256;
    int* swarp = reinterpret_cast<int*>(sb + 2);
    const int q = q0 + blockIdx.x;
    uint32_t* row = rows + (size_t)blockIdx.x * ldr;
    int32_t* my_sel = sel + (size_t)blockIdx.x * P;
    for (int j = threadIdx.x; j < dim; j += TU_NT) sq[j] = queries[(size_t)q * dim + j];
    __syncthreads();
    for (int c = threadIdx.x; c < nlist; c += TU_NT) row[c] = f2key(l2_unfused(sq, ix.centroids + (size_t)c * dim, dim));
    __syncthreads();
    uint32_t kth;
    int nless;
    block_radix_select<TU_NT>(row, nlist, P, hist, sb, kth, nless);
    // the first P lists: every key below the P-th, then ties in id order
    const int need_ties = P - nless;
    int ties = 0, taken = 0;
    for (int b0 = 0; b0 < nlist; b0 += TU_NT) {
        const int c = b0 + threadIdx.x;
        const uint32_t key = c < nlist ? row[c] : 0xffffffffu;
        const int tie = (c < nlist && key == kth) ? 1 : 0;
        int tie_tot;
        const int tie_rank = ties + block_exclusive_scan<TU_NT>(tie, swarp, tie_tot);
        const int take = (c < nlist && (key < kth || (tie && tie_rank < need_ties))) ? 1 : 0;
        int take_tot;
        const int pos = taken + block_exclusive_scan<TU_NT>(take, swarp, take_tot);
        if (take) my_sel[pos] = c;
        ties += tie_tot;
        taken += take_tot;
    }
    __syncthreads();
    float best = INFINITY;
    bool have = false;
    for (int s = 0; s < P; ++s) {
        const int c = my_sel[s];
        const int lo = ix.offsets[c], len = ix.offsets[c + 1] - lo;
        if (len <= 0) continue;
        tune_lut(sq, ix.centroids + (size_t)c * dim, ix.codebook, pq_m, sd, lut);
        __syncthreads();
        for (int j = threadIdx.x; j < len; j += TU_NT)
            row[j] = f2key(tune_pq(ix.codes + (size_t)(lo + j) * pq_m, lut, pq_m));
        __syncthreads();
        int idx = min(limit_k - 1, len - 1);
        if (idx < 0) idx = 0;
        uint32_t kk;
        int nl2;
        block_radix_select<TU_NT>(row, len, idx + 1, hist, sb, kk, nl2);
        best = fminf(best, key2f(kk));
        have = true;
        __syncthreads();  // row and lut are rewritten by the next list
    }
    if (threadIdx.x == 0) out_cut[q] = have ? best : NAN;
}

// ---- host side: the reference's statistics (tune_parameters.cu:168-456) ----------

// (int)(size * p) in float arithmetic, clamped (tune_parameters.cu:169-184)
template <class T>
static T percentile(std::vector<T> v, float p) {
    if (v.empty()) return T(0);
    std::sort(v.begin(), v.end());
    int i = static_cast<int>(static_cast<float>(v.size()) * p);
    if (i >= (int)v.size()) i = (int)v.size() - 1;
    if (i < 0) i = 0;
    return v[i];
}

// Elbow of the hits-per-rank curve (tune_parameters.cu:199-456): on the log of
// the hits, smoothed with a (1/4, 1/2, 1/4) stencil, each rank i = 2..min(n-2,
// 29) with cumulative coverage >= 0.8 is scored by |curvature| * 10, the
// slowdown of the relative drop * 8, an efficiency bonus 4 * (1 - (i/32)^2)
// and a penalty of 5 where the raw curve changes direction; the best score
// wins (the first on equal scores).  Without a candidate: the first rank with
// coverage >= 0.6.  Returns the 1-based rank and its coverage.
static void elbow(const std::vector<int>& hits, long long total, int& point, float& coverage) {
    const int n = (int)hits.size();
    point = 1;
    coverage = 0.0f;
    if (n == 0 || total == 0) return;
    std::vector<float> cov(n), lg(n), sm(n), curv(n, 0.0f), vol(n, 0.0f);
    long long run = 0;
    for (int i = 0; i < n; ++i) {
        run += hits[i];
        cov[i] = static_cast<float>(run) / static_cast<float>(total);
        lg[i] = std::log(static_cast<float>(hits[i]) + 1.0f);
    }
    for (int i = 0; i < n; ++i) {
        if (i == 0 || i == n - 1) {
            sm[i] = lg[i];
        } else {
            float s = 0.25f * lg[i - 1];
            s = s + 0.50f * lg[i];
            sm[i] = s + 0.25f * lg[i + 1];
        }
    }
    for (int i = 1; i + 1 < n; ++i) {
        const float t = sm[i + 1] - 2.0f * sm[i];
        curv[i] = t + sm[i - 1];
        const float up = static_cast<float>(hits[i - 1] - hits[i]);
        const float dn = static_cast<float>(hits[i] - hits[i + 1]);
        if (up * dn < 0.0f) vol[i] = 1.0f;
    }
    int best_i = -1;
    float best = -1e9f;
    for (int i = 2; i + 1 < n && i < 30; ++i) {
        if (cov[i] < 0.60f) continue;
        const float cs = std::fabs(curv[i]) * 10.0f;
        const float before = static_cast<float>(hits[i - 1] - hits[i]) / (static_cast<float>(hits[i - 1]) + 1.0f);
        const float after = static_cast<float>(hits[i] - hits[i + 1]) / (static_cast<float>(hits[i]) + 1.0f);
        const float ds = after < before ? (before - after) * 8.0f : 0.0f;
        const float r = static_cast<float>(i) / 32.0f;
        const float bonus = 4.0f * (1.0f - r * r);
        float score = cs + ds;
        score = score + bonus;
        score = score - vol[i] * 5.0f;
        if (cov[i] >= 0.80f && score > best) {
            best = score;
            best_i = i;
        }
    }
    if (best_i >= 0) {
        point = best_i + 1;
        coverage = cov[best_i];
        return;
    }
    for (int i = 0; i < n; ++i)
        if (cov[i] >= 0.60f) {
            point = i + 1;
            coverage = cov[i];
            return;
        }
}

namespace {
struct Scratch {
    void* p = nullptr;
    ~Scratch() {
        if (p) cudaFree(p);
    }
};
}  // namespace

int tune(const fg_ivfpq_view* v, const float* base, long long nbase, const float* queries, int nq, const int32_t* gt,
         int k, fg_tune_result* out, int32_t* h_cluster_rank, int32_t* h_pq_rank, int32_t* h_exact_rank,
         float* h_ratio, cudaStream_t s) {
    FG_REQUIRE(v && out, "null index or result");
    FG_REQUIRE(nq >= 1 && k >= 1 && nbase >= 1, "bad tune shape");
    FG_REQUIRE(base && queries && gt, "null buffer");
    FG_REQUIRE(v->pq_codebook && v->list_offsets && v->pq_codes && v->vector_ids && v->centroids, "null index array");
    FG_REQUIRE(v->nlist >= 1 && v->dim >= 1 && v->pq_m >= 1 && v->dim % v->pq_m == 0, "bad index shape");
    const int nlist = v->nlist, dim = v->dim, pq_m = v->pq_m;
    std::vector<int32_t> hoff((size_t)nlist + 1);
    FG_CUDA_TRY(cudaMemcpyAsync(hoff.data(), v->list_offsets, hoff.size() * 4, cudaMemcpyDeviceToHost, s));
    FG_CUDA_TRY(cudaStreamSynchronize(s));
    int lmax = 0;
    for (int c = 0; c < nlist; ++c) {
        FG_REQUIRE(hoff[c + 1] >= hoff[c], "list offsets decrease at list %d", c);
        lmax = std::max(lmax, hoff[c + 1] - hoff[c]);
    }
    int dev = 0, smem_max = 0;
    FG_CUDA_TRY(cudaGetDevice(&dev));
    FG_CUDA_TRY(cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    const size_t np = (size_t)nq * k;
    const size_t smem_rank = (size_t)dim * 4 + (size_t)k * 12;
    const size_t smem_pq = ((size_t)pq_m * 256 + dim + 2 + 2) * 4;
    const size_t smem_cut = ((size_t)pq_m * 256 + dim + 256 + 2 + TU_NT / 32) * 4;
    FG_REQUIRE(smem_rank <= (size_t)smem_max && smem_pq <= (size_t)smem_max && smem_cut <= (size_t)smem_max,
               "tuner needs more shared memory than the device has (dim %d, pq_m %d, k %d)", dim, pq_m, k);

    // device scratch: owner, firstpos [nbase]; per-pair outputs; cutoffs
    const size_t ldr = (size_t)std::max(nlist, std::max(lmax, 1));
    const int chunk = (int)std::max<size_t>(1, std::min<size_t>((size_t)nq, (size_t)(256u << 20) / (ldr * 4)));
    const int Pmax = nlist;  // p1 is known only after the first pass
    Scratch sc;
    size_t off = 0;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += round_up(bytes, 256);
        return o;
    };
    const size_t o_owner = take((size_t)nbase * 4), o_first = take((size_t)nbase * 4), o_cr = take(np * 4),
                 o_pr = take(np * 4), o_er = take(np * 4), o_pq = take(np * 4), o_cut = take((size_t)nq * 4),
                 o_rows = take((size_t)chunk * ldr * 4), o_sel = take((size_t)chunk * Pmax * 4);
    FG_CUDA_TRY(cudaMalloc(&sc.p, off));
    char* b = static_cast<char*>(sc.p);
    int32_t* owner = reinterpret_cast<int32_t*>(b + o_owner);
    int32_t* first = reinterpret_cast<int32_t*>(b + o_first);
    int32_t* d_cr = reinterpret_cast<int32_t*>(b + o_cr);
    int32_t* d_pr = reinterpret_cast<int32_t*>(b + o_pr);
    int32_t* d_er = reinterpret_cast<int32_t*>(b + o_er);
    float* d_pq = reinterpret_cast<float*>(b + o_pq);
    float* d_cut = reinterpret_cast<float*>(b + o_cut);
    uint32_t* rows = reinterpret_cast<uint32_t*>(b + o_rows);
    int32_t* sel = reinterpret_cast<int32_t*>(b + o_sel);

    FG_CUDA_TRY(cudaMemsetAsync(owner, 0x7f, (size_t)nbase * 4, s));
    FG_CUDA_TRY(cudaMemsetAsync(first, 0x7f, (size_t)nbase * 4, s));
    tune_owner_kernel<<<nlist, 128, 0, s>>>(v->list_offsets, v->vector_ids, nbase, owner);
    int rc = check_launch("tune_owner_kernel");
    if (rc) return rc;
    tune_firstpos_kernel<<<nlist, 128, 0, s>>>(v->list_offsets, v->vector_ids, nbase, owner, first);
    if ((rc = check_launch("tune_firstpos_kernel"))) return rc;
    FG_CUDA_TRY(cudaFuncSetAttribute(tune_cluster_rank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)smem_rank));
    tune_cluster_rank_kernel<<<nq, TU_NT, smem_rank, s>>>(v->centroids, nlist, dim, queries, gt, k, owner, nbase, d_cr);
    if ((rc = check_launch("tune_cluster_rank_kernel"))) return rc;
    const TuneIndex ix{v->pq_codebook, v->list_offsets, v->pq_codes, v->vector_ids, v->centroids, nlist, dim, pq_m};
    FG_CUDA_TRY(cudaFuncSetAttribute(tune_pq_rank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_pq));
    tune_pq_rank_kernel<<<(unsigned)np, TU_NT, smem_pq, s>>>(ix, base, nbase, queries, gt, k, owner, first, d_pr, d_er,
                                                           d_pq);
    if ((rc = check_launch("tune_pq_rank_kernel"))) return rc;

    std::vector<int32_t> cr(np), pr(np), er(np);
    std::vector<float> pqt(np);
    FG_CUDA_TRY(cudaMemcpyAsync(cr.data(), d_cr, np * 4, cudaMemcpyDeviceToHost, s));
    FG_CUDA_TRY(cudaMemcpyAsync(pr.data(), d_pr, np * 4, cudaMemcpyDeviceToHost, s));
    FG_CUDA_TRY(cudaMemcpyAsync(er.data(), d_er, np * 4, cudaMemcpyDeviceToHost, s));
    FG_CUDA_TRY(cudaMemcpyAsync(pqt.data(), d_pq, np * 4, cudaMemcpyDeviceToHost, s));
    FG_CUDA_TRY(cudaStreamSynchronize(s));

    // top_m and p1_lists from the coarse ranks
    std::vector<int> ranks;
    ranks.reserve(np);
    for (size_t i = 0; i < np; ++i)
        if (cr[i] > 0) ranks.push_back(cr[i]);
    fg_tune_result r{};
    r.top_m = percentile(ranks, 0.995f);
    const int max_rank = ranks.empty() ? 0 : *std::max_element(ranks.begin(), ranks.end());
    std::vector<int> hits((size_t)max_rank, 0);
    for (int x : ranks) ++hits[x - 1];
    elbow(hits, (long long)ranks.size(), r.p1_lists, r.coverage_at_elbow);
    r.n_ranked = (int)ranks.size();

    // limit_k from the PQ ranks of neighbours in the first p1 lists
    std::vector<int> all_pq, p1_pq;
    for (size_t i = 0; i < np; ++i) {
        if (pr[i] <= 0) continue;
        all_pq.push_back(pr[i]);
        if (cr[i] > 0 && cr[i] <= r.p1_lists) p1_pq.push_back(pr[i]);
    }
    r.limit_k = p1_pq.empty() ? percentile(all_pq, 0.98f) : *std::max_element(p1_pq.begin(), p1_pq.end());
    r.n_in_p1 = (int)p1_pq.size();

    // threshold_coeff from the phase-1 cutoffs
    const int P = std::min(std::max(r.p1_lists, 1), nlist);
    const size_t smem_c = smem_cut;
    FG_CUDA_TRY(cudaFuncSetAttribute(tune_cutoff_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_c));
    for (int q0 = 0; q0 < nq; q0 += chunk) {
        const int nb = std::min(chunk, nq - q0);
        tune_cutoff_kernel<<<nb, TU_NT, smem_c, s>>>(ix, queries, q0, P, r.limit_k, rows, ldr, sel, d_cut);
        if ((rc = check_launch("tune_cutoff_kernel"))) return rc;
    }
    std::vector<float> cut((size_t)nq);
    FG_CUDA_TRY(cudaMemcpyAsync(cut.data(), d_cut, (size_t)nq * 4, cudaMemcpyDeviceToHost, s));
    FG_CUDA_TRY(cudaStreamSynchronize(s));
    std::vector<float> ratios;
    for (int q = 0; q < nq; ++q) {
        float ratio = NAN;
        const size_t far = (size_t)q * k + (k - 1);
        if (!std::isnan(cut[q]) && pr[far] > 0 && pqt[far] >= 0.0f && cut[q] > 0.0f) {
            ratio = pqt[far] / cut[q];
            ratios.push_back(ratio);
        }
        if (h_ratio) h_ratio[q] = ratio;
    }
    r.threshold_coeff = ratios.empty() ? 2.0f : *std::max_element(ratios.begin(), ratios.end());
    r.n_ratios = (int)ratios.size();
    if (h_cluster_rank) std::copy(cr.begin(), cr.end(), h_cluster_rank);
    if (h_pq_rank) std::copy(pr.begin(), pr.end(), h_pq_rank);
    if (h_exact_rank) std::copy(er.begin(), er.end(), h_exact_rank);
    *out = r;
    return FG_OK;
}

}  // namespace fg

extern "C" int fg_tune_elbow(const int32_t* hits, int32_t n, int64_t total, int32_t* point, float* coverage) {
    if (n < 0 || (n > 0 && !hits) || !point || !coverage) return fg::fail(FG_ERR_INVALID_ARG, "bad elbow arguments");
    std::vector<int> h(hits, hits + n);
    int p = 1;
    fg::elbow(h, (long long)total, p, *coverage);
    *point = p;
    return FG_OK;
}

extern "C" int fg_tune(const fg_ivfpq_view* index, const float* base, int64_t nbase, const float* queries, int32_t nq,
                       const int32_t* gt_ids, int32_t k, fg_tune_result* out, int32_t* cluster_ranks,
                       int32_t* pq_ranks, int32_t* exact_ranks, float* ratios, void* stream) {
    return fg::tune(index, base, nbase, queries, nq, gt_ids, k, out, cluster_ranks, pq_ranks, exact_ranks, ratios,
                    static_cast<cudaStream_t>(stream));
}
