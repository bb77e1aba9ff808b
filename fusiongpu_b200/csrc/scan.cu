// scan.cu -- candidate generation for a batch of queries (replaces the
// reference's run_gpu_batch_logic, gpu_global.cu:679-874).
//
// One CTA per query does, without leaving the SM or the host stepping in:
//   prune the probe list            (gpu_global.cu:31-77)
//   per probed list: residual LUT   (gpu_global.cu:79-166) built in shared memory
//   phase 1: ADC scan of the first p1_lists lists, top-limit_k per list and the
//            limit_k-th distance as the list cutoff (gpu_global.cu:321-390)
//   threshold = min positive cutoff * coeff (gpu_global.cu:394-426)
//   phase 2: ADC scan of the remaining lists, keep distance <= threshold
//            (gpu_global.cu:428-527, including the 128-slot overflow rule)
//   the sorted top rerank_m candidates (gpu_global.cu:533-576)
//
// Candidates go to a shared-memory buffer in emission order (probe index j,
// then position in the list), which is the order the stable sort of the
// reference breaks distance ties by under an in-order schedule.  When the
// buffer fills, it is cut to its best `rsel` entries and every later candidate
// whose distance is not below the rsel-th is dropped on arrival: those can no
// longer reach the output.
//
// The ADC arithmetic is bit-identical to the reference: each LUT entry is the
// same fmaf expression as gpu_global.cu:115-157 / 274-313, and the ADC sum runs
// over subspaces in order with round-to-nearest adds.
#include "fg_common.cuh"

namespace fg {

constexpr int SCAN_NT = 512;
constexpr int REF_BLOCK = 128;      // blockDim of the reference's scan/gather kernels
constexpr int REF_P1_CLAMP = 1024;  // 128 threads x 8 items (gpu_global.cu:343-346)

struct ScanArgs {
    const float* codebook;
    const int32_t* offsets;
    const uint8_t* codes;
    const int32_t* vids;
    const float* centroids;
    int nlist, dim, pq_m, sub_dim;  // pq_m/sub_dim are read by the generic (M = 0) kernel
    const float* queries;
    const uint32_t* probe_ids;
    const float* probe_dists;
    int top_m, p1, limit_k;
    float coeff, prune_ratio;
    int rerank_m, rsel, ref_compat, lmax, cap, sort_n;
    int write_pad;  // write (-1, FLT_MAX) / ref_compat zeros past each query's count
    int32_t* top_ids;
    float* top_dists;
    int32_t* top_counts;
    int32_t* cand_counts;
};

struct ScanMisc {
    uint32_t hist[256];
    int warp[SCAN_NT / 32];
    uint32_t b[2];
    int carry[REF_BLOCK];
    unsigned char passf[SCAN_NT];
    int buf_n, count, nb_list;
    uint32_t prune_key;
    float thr;
};

struct ScanLayout {
    int lut, res, pid, cut, lkey, ckey, cid, sortb, misc, total;
};

__host__ __device__ inline int take16(int& o, int bytes) {
    int r = o;
    o += (bytes + 15) / 16 * 16;
    return r;
}

__host__ __device__ inline ScanLayout scan_layout(int M, int dim, int top_m, int p1, int lmax,
                                                  int cap, int sort_n) {
    ScanLayout L;
    int o = 0;
    L.lut = take16(o, M * 256 * 4);
    L.res = take16(o, dim * 4);
    L.pid = take16(o, top_m * 4);
    L.cut = take16(o, (p1 > 0 ? p1 : 1) * 4);
    L.lkey = take16(o, (lmax > 0 ? lmax : 1) * 4);
    const int prefix = o;  // LUT..lkey are dead once the final sort starts
    L.ckey = take16(o, cap * 4);
    L.cid = take16(o, cap * 4);
    if (sort_n * 8 <= prefix) {
        L.sortb = 0;
    } else {
        L.sortb = take16(o, sort_n * 8);
    }
    L.misc = take16(o, (int)sizeof(ScanMisc));
    L.total = o;
    return L;
}

// ||r - c||^2 of one subspace, the expression of gpu_global.cu:115-157.
template <int SD>
__device__ __forceinline__ float sub_dist(const float* r, const float* c) {
    if constexpr (SD == 4) {
        const float4 rv = *reinterpret_cast<const float4*>(r);
        const float4 cv = __ldg(reinterpret_cast<const float4*>(c));
        const float dx = rv.x - cv.x, dy = rv.y - cv.y, dz = rv.z - cv.z, dw = rv.w - cv.w;
        return fmaf(dx, dx, fmaf(dy, dy, fmaf(dz, dz, __fmul_rn(dw, dw))));
    } else if constexpr (SD == 8) {
        const float4 r0 = *reinterpret_cast<const float4*>(r);
        const float4 r1 = *reinterpret_cast<const float4*>(r + 4);
        const float4 c0 = __ldg(reinterpret_cast<const float4*>(c));
        const float4 c1 = __ldg(reinterpret_cast<const float4*>(c + 4));
        const float a0 = r0.x - c0.x, a1 = r0.y - c0.y, a2 = r0.z - c0.z, a3 = r0.w - c0.w;
        const float a4 = r1.x - c1.x, a5 = r1.y - c1.y, a6 = r1.z - c1.z, a7 = r1.w - c1.w;
        const float d = fmaf(a0, a0, fmaf(a1, a1, fmaf(a2, a2, __fmul_rn(a3, a3))));
        return fmaf(a4, a4, fmaf(a5, a5, fmaf(a6, a6, fmaf(a7, a7, d))));
    } else if constexpr (SD == 2) {
        const float2 rv = *reinterpret_cast<const float2*>(r);
        const float2 cv = __ldg(reinterpret_cast<const float2*>(c));
        const float d0 = rv.x - cv.x, d1 = rv.y - cv.y;
        return fmaf(d1, d1, fmaf(d0, d0, 0.0f));
    } else {
        float d = 0.0f;
#pragma unroll
        for (int i = 0; i < SD; ++i) {
            const float df = r[i] - __ldg(c + i);
            d = fmaf(df, df, d);
        }
        return d;
    }
}

__device__ __forceinline__ float sub_dist_rt(const float* r, const float* c, int sd) {
    if (sd == 4) return sub_dist<4>(r, c);
    if (sd == 8) return sub_dist<8>(r, c);
    float d = 0.0f;
    for (int i = 0; i < sd; ++i) {
        const float df = r[i] - __ldg(c + i);
        d = fmaf(df, df, d);
    }
    return d;
}

// ADC distance of one PQ code row: sum of LUT entries in subspace order.
// M = 0: runtime pq_m (`mrt`), byte loads.
template <int M>
__device__ __forceinline__ float adc(const uint8_t* __restrict__ row, const float* __restrict__ lut, int mrt = 0) {
    float d = 0.0f;
    if constexpr (M == 0) {
        for (int m = 0; m < mrt; ++m) d = __fadd_rn(d, lut[m * 256 + __ldg(row + m)]);
    } else if constexpr (M % 16 == 0) {
        const uint4* r4 = reinterpret_cast<const uint4*>(row);
#pragma unroll
        for (int w = 0; w < M / 16; ++w) {
            const uint4 v = __ldg(r4 + w);
            const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int b = 0; b < 16; ++b) {
                const uint32_t code = (wd[b >> 2] >> (8 * (b & 3))) & 0xffu;
                d = __fadd_rn(d, lut[(16 * w + b) * 256 + code]);
            }
        }
    } else {
        static_assert(M % 4 == 0, "pq_m must be a multiple of 4");
        const uint32_t* r1 = reinterpret_cast<const uint32_t*>(row);
#pragma unroll
        for (int w = 0; w < M / 4; ++w) {
            const uint32_t v = __ldg(r1 + w);
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const uint32_t code = (v >> (8 * b)) & 0xffu;
                d = __fadd_rn(d, lut[(4 * w + b) * 256 + code]);
            }
        }
    }
    return d;
}

template <int M, int SD>
__device__ __forceinline__ void build_lut(const ScanArgs& a, const float* qv, uint32_t c, float* res,
                                          float* lut) {
    const float* cv = a.centroids + (size_t)c * a.dim;
    for (int t = threadIdx.x; t < a.dim; t += SCAN_NT) res[t] = qv[t] - cv[t];
    __syncthreads();
    if constexpr (M == 0) {
        const int sd = a.sub_dim;
        for (int e = threadIdx.x; e < a.pq_m * 256; e += SCAN_NT) {
            const int m = e >> 8;
            lut[e] = sub_dist_rt(res + m * sd, a.codebook + (size_t)e * sd, sd);
        }
    } else {
        for (int e = threadIdx.x; e < M * 256; e += SCAN_NT) {
            const int m = e >> 8;
            lut[e] = sub_dist<SD>(res + m * SD, a.codebook + (size_t)e * SD);
        }
    }
    __syncthreads();
}

// Cut the candidate buffer down to its best `rsel` entries (by key, then
// position), keeping their order, and raise the pruning bar to the rsel-th key.
__device__ void reduce_buffer(int rsel, uint32_t* ckey, int32_t* cid, ScanMisc* ms) {
    const int n = ms->buf_n;
    uint32_t kth;
    int n_less;
    block_radix_select<SCAN_NT>(ckey, n, rsel, ms->hist, ms->b, kth, n_less);
    const int need_eq = rsel - n_less;
    int eq_base = 0, out_base = 0;
    for (int r0 = 0; r0 < n; r0 += SCAN_NT) {
        const int i = r0 + threadIdx.x;
        const bool in = i < n;
        const uint32_t key = in ? ckey[i] : 0xffffffffu;
        const int32_t idv = in ? cid[i] : 0;
        const int is_eq = (in && key == kth) ? 1 : 0;
        int eq_tot, k_tot;
        const int eq_pre = block_exclusive_scan<SCAN_NT>(is_eq, ms->warp, eq_tot);
        const bool keep = in && (key < kth || (is_eq && eq_base + eq_pre < need_eq));
        eq_base += eq_tot;
        const int k_pre = block_exclusive_scan<SCAN_NT>(keep ? 1 : 0, ms->warp, k_tot);
        // destinations never pass their sources, and every source of this
        // round was read before the scans' barriers
        if (keep) {
            ckey[out_base + k_pre] = key;
            cid[out_base + k_pre] = idv;
        }
        out_base += k_tot;
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        ms->buf_n = out_base;
        ms->prune_key = kth;
    }
    __syncthreads();
}

// Append the flagged candidates of this round, in thread order.
__device__ __forceinline__ void append(const ScanArgs& a, bool emit, uint32_t key, int32_t id,
                                       uint32_t* ckey, int32_t* cid, ScanMisc* ms) {
    int tot;
    const int pre = block_exclusive_scan<SCAN_NT>(emit ? 1 : 0, ms->warp, tot);
    if (tot == 0) return;
    if (ms->buf_n + tot > a.cap) reduce_buffer(a.rsel, ckey, cid, ms);
    const int base = ms->buf_n;
    if (emit) {
        ckey[base + pre] = key;
        cid[base + pre] = id;
    }
    __syncthreads();
    if (threadIdx.x == 0) ms->buf_n = base + tot;
    __syncthreads();
}

template <int M, int SD>
__global__ void __launch_bounds__(SCAN_NT) ivfpq_batch_kernel(const ScanArgs a) {
    static_assert(SCAN_NT % REF_BLOCK == 0, "phase-2 overflow ranks need whole 128-thread groups");
    extern __shared__ __align__(16) unsigned char smem[];
    constexpr bool RT = (M == 0);
    const int MM = RT ? a.pq_m : M;
    const ScanLayout L = scan_layout(MM, a.dim, a.top_m, a.p1, a.lmax, a.cap, a.sort_n);
    float* lut = reinterpret_cast<float*>(smem + L.lut);
    float* res = reinterpret_cast<float*>(smem + L.res);
    uint32_t* pid = reinterpret_cast<uint32_t*>(smem + L.pid);
    float* cut = reinterpret_cast<float*>(smem + L.cut);
    uint32_t* lkey = reinterpret_cast<uint32_t*>(smem + L.lkey);
    uint32_t* ckey = reinterpret_cast<uint32_t*>(smem + L.ckey);
    int32_t* cid = reinterpret_cast<int32_t*>(smem + L.cid);
    unsigned long long* sortb = reinterpret_cast<unsigned long long*>(smem + L.sortb);
    ScanMisc* ms = reinterpret_cast<ScanMisc*>(smem + L.misc);

    const int tid = threadIdx.x;
    const int q = blockIdx.x;
    const int P = a.top_m;
    const float* qv = a.queries + (size_t)q * a.dim;

    // prune (gpu_global.cu:43-51); ids outside [0, nlist) are skipped
    const float best = a.probe_dists[(size_t)q * P];
    const float pthr = best * a.prune_ratio;
    for (int j = tid; j < P; j += SCAN_NT) {
        const float d = a.probe_dists[(size_t)q * P + j];
        const uint32_t id = a.probe_ids[(size_t)q * P + j];
        pid[j] = (d > pthr || id >= (uint32_t)a.nlist) ? FG_INVALID_PROBE : id;
    }
    if (tid == 0) {
        ms->buf_n = 0;
        ms->count = 0;
        ms->prune_key = 0xffffffffu;
    }
    __syncthreads();

    // ---- phase 1 --------------------------------------------------------------
    for (int j = 0; j < a.p1; ++j) {
        const uint32_t c = pid[j];
        int start = 0, len = 0;
        if (c != FG_INVALID_PROBE) {
            start = a.offsets[c];
            len = a.offsets[c + 1] - start;
        }
        if (len <= 0) {
            if (tid == 0) cut[j] = 0.0f;
            continue;
        }
        const int wc = len < a.limit_k ? len : a.limit_k;
        const int scan = (a.ref_compat && len > REF_P1_CLAMP) ? REF_P1_CLAMP : len;
        build_lut<M, SD>(a, qv, c, res, lut);
        for (int i = tid; i < scan; i += SCAN_NT)
            lkey[i] = f2key(adc<M>(a.codes + (size_t)(start + i) * MM, lut, MM));
        __syncthreads();
        uint32_t kth;
        int n_less;
        block_radix_select<SCAN_NT>(lkey, scan, wc, ms->hist, ms->b, kth, n_less);
        if (tid == 0) {
            cut[j] = key2f(kth);
            ms->count += wc;
        }
        const int need_eq = wc - n_less;
        int eq_base = 0;
        for (int r0 = 0; r0 < scan; r0 += SCAN_NT) {
            const int i = r0 + tid;
            const bool in = i < scan;
            const uint32_t key = in ? lkey[i] : 0xffffffffu;
            const int is_eq = (in && key == kth) ? 1 : 0;
            int eq_tot;
            const int eq_pre = block_exclusive_scan<SCAN_NT>(is_eq, ms->warp, eq_tot);
            const bool sel = in && (key < kth || (is_eq && eq_base + eq_pre < need_eq));
            eq_base += eq_tot;
            const bool emit = sel && key < ms->prune_key;
            append(a, emit, key, emit ? __ldg(a.vids + start + i) : 0, ckey, cid, ms);
        }
    }

    // ---- threshold (gpu_global.cu:394-426) -----------------------------------
    if (tid == 0) {
        float mn = FLT_MAX;
        for (int j = 0; j < a.p1; ++j)
            if (cut[j] > 0.0f && cut[j] < mn) mn = cut[j];
        ms->thr = (mn < FLT_MAX) ? mn * a.coeff : FLT_MAX;
    }
    __syncthreads();
    const float thr = ms->thr;

    // ---- phase 2 --------------------------------------------------------------
    for (int j = a.p1; j < P; ++j) {
        const uint32_t c = pid[j];
        int start = 0, len = 0;
        if (c != FG_INVALID_PROBE) {
            start = a.offsets[c];
            len = a.offsets[c + 1] - start;
        }
        if (len <= 0) continue;
        if (tid == 0) ms->nb_list = 0;
        build_lut<M, SD>(a, qv, c, res, lut);
        for (int c0 = 0; c0 < len; c0 += SCAN_NT) {
            const int i = c0 + tid;
            float d = 0.0f;
            bool pass = false;
            if (i < len) {
                d = adc<M>(a.codes + (size_t)(start + i) * MM, lut, MM);
                pass = d <= thr;
            }
            int p_tot;
            const int p_pre = block_exclusive_scan<SCAN_NT>(pass ? 1 : 0, ms->warp, p_tot);
            const int rank = ms->nb_list + p_pre;
            const uint32_t key = f2key(d);
            const bool emit = pass && (!a.ref_compat || rank < REF_BLOCK) && key < ms->prune_key;
            append(a, emit, key, emit ? __ldg(a.vids + start + i) : 0, ckey, cid, ms);
            if (tid == 0) ms->nb_list += p_tot;
            __syncthreads();
        }
        const int s_count = ms->nb_list;
        if (!a.ref_compat || s_count <= REF_BLOCK) {
            if (tid == 0) ms->count += s_count;
            __syncthreads();
            continue;
        }
        // overflow: each of the reference's 128 threads re-emits its first
        // (s_count - 128) passing vectors (gpu_global.cu:508-526)
        const int quota = s_count - REF_BLOCK;
        if (tid < REF_BLOCK) ms->carry[tid] = 0;
        if (tid == 0) ms->count += REF_BLOCK;
        __syncthreads();
        for (int c0 = 0; c0 < len; c0 += SCAN_NT) {
            const int i = c0 + tid;
            float d = 0.0f;
            bool pass = false;
            if (i < len) {
                d = adc<M>(a.codes + (size_t)(start + i) * MM, lut, MM);
                pass = d <= thr;
            }
            ms->passf[tid] = pass ? 1 : 0;
            __syncthreads();
            // rank among the passing vectors of the same reference thread (i mod 128)
            const int t = tid % REF_BLOCK;
            int rank = ms->carry[t];
            for (int u = t; u < tid; u += REF_BLOCK) rank += ms->passf[u];
            const bool re = pass && rank < quota;
            int r_tot;
            (void)block_exclusive_scan<SCAN_NT>(re ? 1 : 0, ms->warp, r_tot);
            if (tid == 0) ms->count += r_tot;
            const uint32_t key = f2key(d);
            const bool emit = re && key < ms->prune_key;
            append(a, emit, key, emit ? __ldg(a.vids + start + i) : 0, ckey, cid, ms);
            if (tid < REF_BLOCK) {
                int add = 0;
                for (int u = tid; u < SCAN_NT; u += REF_BLOCK) add += ms->passf[u];
                ms->carry[tid] += add;
            }
            __syncthreads();
        }
    }

    // ---- select, sort and gather (gpu_global.cu:838-871) ---------------------
    __syncthreads();
    if (ms->buf_n > a.rsel) reduce_buffer(a.rsel, ckey, cid, ms);
    const int n = ms->buf_n;
    const int npow = next_pow2(n > 0 ? n : 1);
    for (int i = tid; i < npow; i += SCAN_NT)
        sortb[i] = (i < n) ? ((unsigned long long)ckey[i] << 32) | (unsigned)i : ~0ull;
    __syncthreads();
    block_bitonic_sort<SCAN_NT>(sortb, npow);
    const int count = ms->count;
    const int rm = a.rerank_m;
    const int ak = count < rm ? count : rm;
    const int pend = a.write_pad ? rm : (ak < rm ? ak : rm);
    for (int p = tid; p < pend; p += SCAN_NT) {
        const size_t o = (size_t)q * rm + p;
        if (a.ref_compat && p >= REF_BLOCK) {
            // never written by the reference's 128-thread gather; modelled as
            // freshly allocated (zeroed) device memory
            a.top_ids[o] = 0;
            a.top_dists[o] = 0.0f;
        } else if (p < ak) {
            const unsigned long long e = sortb[p];
            a.top_ids[o] = cid[(unsigned)(e & 0xffffffffu)];
            a.top_dists[o] = key2f((uint32_t)(e >> 32));
        } else {
            a.top_ids[o] = -1;
            a.top_dists[o] = FLT_MAX;
        }
    }
    if (tid == 0) {
        a.top_counts[q] = ak;
        if (a.cand_counts) a.cand_counts[q] = count;
    }
}

using ScanKernel = void (*)(const ScanArgs);

static ScanKernel pick_scan_kernel(int M, int SD) {
#define FG_SCAN_CASE(m, sd) \
    if (M == m && SD == sd) return ivfpq_batch_kernel<m, sd>;
    FG_SCAN_CASE(16, 4)
    FG_SCAN_CASE(16, 8)
    FG_SCAN_CASE(32, 2)
    FG_SCAN_CASE(32, 3)
    FG_SCAN_CASE(32, 4)
    FG_SCAN_CASE(48, 2)
    FG_SCAN_CASE(64, 2)
    FG_SCAN_CASE(96, 8)
    FG_SCAN_CASE(128, 1)
#undef FG_SCAN_CASE
    if (M <= 256 && SD <= 16) return ivfpq_batch_kernel<0, 0>;  // generic runtime shape
    return nullptr;
}

int batch_logic(const fg_ivfpq_view* ix, const float* queries, int nq, const uint32_t* probe_ids,
                const float* probe_dists, const fg_search_params* p, int32_t* top_ids,
                float* top_dists, int32_t* top_counts, int32_t* cand_counts, cudaStream_t stream,
                bool write_pad) {
    FG_REQUIRE(ix && p, "null index or params");
    FG_REQUIRE(nq >= 0, "nq < 0");
    FG_REQUIRE(ix->dim > 0 && ix->pq_m > 0 && ix->dim % ix->pq_m == 0, "dim %d not divisible by pq_m %d",
               ix->dim, ix->pq_m);
    FG_REQUIRE(p->top_m >= 1 && p->top_m <= 4096, "top_m %d outside [1, 4096]", p->top_m);
    FG_REQUIRE(p->p1_lists >= 0, "p1_lists < 0");
    FG_REQUIRE(p->limit_k >= 1, "limit_k < 1");
    FG_REQUIRE(p->rerank_m >= 1, "rerank_m < 1");
    FG_REQUIRE(!p->ref_compat || p->limit_k <= REF_P1_CLAMP,
               "ref_compat needs limit_k <= 1024 (the reference leaves ranks >= 1024 unwritten)");
    FG_REQUIRE(ix->max_list_len >= 0 && ix->max_list_len < (1 << 19), "max_list_len %d", ix->max_list_len);
    if (nq == 0) return FG_OK;
    FG_REQUIRE(queries && probe_ids && probe_dists && top_ids && top_dists && top_counts,
               "null buffer");
    FG_REQUIRE(ix->pq_codebook && ix->list_offsets && ix->pq_codes && ix->vector_ids && ix->centroids,
               "null index array");
    FG_REQUIRE(aligned(ix->pq_codes, 16) && aligned(ix->pq_codebook, 16) && aligned(queries, 16),
               "codes, codebook and queries must be 16-byte aligned");
    FG_REQUIRE(ix->nlist >= 1 && ix->total >= 0, "empty index");
    const int M = ix->pq_m, SD = ix->dim / ix->pq_m;
    ScanKernel k = pick_scan_kernel(M, SD);
    if (!k) return fail(FG_ERR_UNSUPPORTED, "no scan kernel for pq_m=%d sub_dim=%d", M, SD);

    ScanArgs a;
    a.codebook = ix->pq_codebook;
    a.offsets = ix->list_offsets;
    a.codes = ix->pq_codes;
    a.vids = ix->vector_ids;
    a.centroids = ix->centroids;
    a.nlist = ix->nlist;
    a.dim = ix->dim;
    a.pq_m = M;
    a.sub_dim = SD;
    a.queries = queries;
    a.probe_ids = probe_ids;
    a.probe_dists = probe_dists;
    a.top_m = p->top_m;
    a.p1 = p->top_m < p->p1_lists ? p->top_m : p->p1_lists;
    a.limit_k = p->limit_k;
    a.coeff = p->threshold_coeff;
    a.prune_ratio = p->prune_ratio;
    a.rerank_m = p->rerank_m;
    a.rsel = p->ref_compat ? (p->rerank_m < REF_BLOCK ? p->rerank_m : REF_BLOCK) : p->rerank_m;
    a.ref_compat = p->ref_compat ? 1 : 0;
    int lmax = ix->max_list_len;
    if (a.ref_compat && lmax > REF_P1_CLAMP) lmax = REF_P1_CLAMP;
    a.lmax = lmax > 0 ? lmax : 1;
    a.sort_n = next_pow2(a.rsel);
    a.top_ids = top_ids;
    a.top_dists = top_dists;
    a.top_counts = top_counts;
    a.cand_counts = cand_counts;
    a.write_pad = write_pad ? 1 : 0;

    int dev = 0, smem_max = 0, smem_sm = 0;
    FG_CUDA_TRY(cudaGetDevice(&dev));
    FG_CUDA_TRY(cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    FG_CUDA_TRY(cudaDeviceGetAttribute(&smem_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev));
    // a roomy buffer (fewer cuts) when it fits and costs no resident CTA, else
    // the minimum rsel + one round
    a.cap = 2 * a.rsel + SCAN_NT;
    ScanLayout L = scan_layout(M, a.dim, a.top_m, a.p1, a.lmax, a.cap, a.sort_n);
    const ScanLayout Lmin = scan_layout(M, a.dim, a.top_m, a.p1, a.lmax, a.rsel + SCAN_NT, a.sort_n);
    auto per_sm = [&](int bytes) { return smem_sm / (bytes + 1024); };
    if (L.total > smem_max || per_sm(Lmin.total) > per_sm(L.total)) {
        a.cap = a.rsel + SCAN_NT;
        L = Lmin;
    }
    if (L.total > smem_max)
        return fail(FG_ERR_UNSUPPORTED, "scan needs %d bytes of shared memory (max %d): rerank_m=%d "
                    "max_list_len=%d", L.total, smem_max, a.rerank_m, a.lmax);
    FG_CUDA_TRY(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total));
    k<<<nq, SCAN_NT, L.total, stream>>>(a);
    return check_launch("ivfpq_batch_kernel");
}

// ---- candidate budget: prune + count + offsets (gpu_global.cu:31-77, 709-725) ----
// counts[q] = total length of the probed lists that survive the prune
// (distance <= best * prune_ratio); offsets = exclusive scan of counts with
// offsets[nq] = the batch total.  The probe list is not modified.

constexpr int BUD_NT = 128;

__global__ void __launch_bounds__(BUD_NT)
    budget_count_kernel(const int32_t* __restrict__ offs, int nlist, const uint32_t* __restrict__ pid,
                        const float* __restrict__ pd, int top_m, float ratio, int32_t* __restrict__ counts) {
    const int q = blockIdx.x;
    const float thr = pd[(size_t)q * top_m] * ratio;
    long long c = 0;
    for (int j = threadIdx.x; j < top_m; j += BUD_NT) {
        const uint32_t id = pid[(size_t)q * top_m + j];
        if (id != FG_INVALID_PROBE && (int)id < nlist && !(pd[(size_t)q * top_m + j] > thr)) c += offs[id + 1] - offs[id];
    }
    for (int o = 16; o; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    __shared__ long long sw[BUD_NT / 32];
    if ((threadIdx.x & 31) == 0) sw[threadIdx.x >> 5] = c;
    __syncthreads();
    if (threadIdx.x == 0) {
        long long t = 0;
        for (int w = 0; w < BUD_NT / 32; ++w) t += sw[w];
        counts[q] = (int32_t)t;
    }
}

__global__ void __launch_bounds__(1024) budget_scan_kernel(const int32_t* __restrict__ counts, int nq,
                                                           int32_t* __restrict__ offsets) {
    __shared__ int sw[32];
    int run = 0;
    for (int b0 = 0; b0 < nq; b0 += 1024) {
        const int i = b0 + threadIdx.x;
        const int v = i < nq ? counts[i] : 0;
        int tot;
        const int ex = block_exclusive_scan<1024>(v, sw, tot);
        if (i < nq) offsets[i] = run + ex;
        run += tot;
    }
    if (threadIdx.x == 0) offsets[nq] = run;
}

int probe_budget(const int32_t* list_offsets, int nlist, const uint32_t* probe_ids, const float* probe_dists, int nq,
                 int top_m, float prune_ratio, int32_t* counts, int32_t* offsets, cudaStream_t s) {
    FG_REQUIRE(nq >= 0 && top_m >= 1 && nlist >= 1, "bad budget shape");
    FG_REQUIRE(list_offsets && counts && (nq == 0 || (probe_ids && probe_dists)), "null buffer");
    if (nq > 0) {
        budget_count_kernel<<<nq, BUD_NT, 0, s>>>(list_offsets, nlist, probe_ids, probe_dists, top_m, prune_ratio,
                                                   counts);
        int rc = check_launch("budget_count_kernel");
        if (rc) return rc;
    }
    if (offsets) {
        budget_scan_kernel<<<1, 1024, 0, s>>>(counts, nq, offsets);
        return check_launch("budget_scan_kernel");
    }
    return FG_OK;
}

}  // namespace fg
