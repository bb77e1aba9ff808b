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
#include <algorithm>
#include <cstdlib>
#include <string>

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
    int* work_counter;  // team kernel: zeroed counter for dynamic query fetching (null: static round robin)
    int small;      // team kernel: 1 when no query can emit more than rsel candidates (the buffer is never
                    // cut) and one warp selects each list; 2 the same with team-wide selection
    int write_pad;  // write (-1, FLT_MAX) / ref_compat zeros past each query's count
    int32_t* top_ids;
    float* top_dists;
    int32_t* top_counts;
    int32_t* cand_counts;
    // split path (one CTA per probed list): per-query phase-1 cutoffs [nq][p1],
    // candidate counts [nq], candidate keys [nq][capg] and fallback flags [nq]
    float* cut_g;
    int32_t* cnt_g;
    unsigned long long* cand_g;
    int32_t* flags;       // split select: 1 where the query falls back to the per-query kernel
    const int32_t* only;  // per-query kernel: run only the queries flagged here (null: all)
    int capg;
    int* work;            // split: [0] phase-1 pairs, [1] phase-2 pairs, [2], [3] their work counters
    int4* pairs1;         // split: the (query, probe) pairs with a non-empty list of each phase,
    int4* pairs2;         //        as (q * top_m + j, list, start, length), grouped by list
    int* hist;            // split: per-list pair counts, then offsets: phase 1 [nlist + 1], phase 2 [nlist + 1]
    int2* groups;         // group kernel: (first record, records) of up to GRP_G queries probing one list
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

// ||r - c||^2 of one subspace from values in registers: the expression of
// gpu_global.cu:115-157.  Every LUT entry and every on-the-fly ADC term is
// this one function, so both scan kernels produce identical floats.
template <int SD>
__device__ __forceinline__ float sd_arith(const float (&r)[SD], const float (&c)[SD]) {
    if constexpr (SD == 4) {
        const float dx = r[0] - c[0], dy = r[1] - c[1], dz = r[2] - c[2], dw = r[3] - c[3];
        return fmaf(dx, dx, fmaf(dy, dy, fmaf(dz, dz, __fmul_rn(dw, dw))));
    } else if constexpr (SD == 8) {
        const float a0 = r[0] - c[0], a1 = r[1] - c[1], a2 = r[2] - c[2], a3 = r[3] - c[3];
        const float a4 = r[4] - c[4], a5 = r[5] - c[5], a6 = r[6] - c[6], a7 = r[7] - c[7];
        const float d = fmaf(a0, a0, fmaf(a1, a1, fmaf(a2, a2, __fmul_rn(a3, a3))));
        return fmaf(a4, a4, fmaf(a5, a5, fmaf(a6, a6, fmaf(a7, a7, d))));
    } else if constexpr (SD == 2) {
        const float d0 = r[0] - c[0], d1 = r[1] - c[1];
        return fmaf(d1, d1, fmaf(d0, d0, 0.0f));
    } else {
        float d = 0.0f;
#pragma unroll
        for (int i = 0; i < SD; ++i) {
            const float df = r[i] - c[i];
            d = fmaf(df, df, d);
        }
        return d;
    }
}

// SD consecutive floats; GLOBAL reads through the read-only path.
template <int SD, bool GLOBAL>
__device__ __forceinline__ void load_sub(const float* p, float (&v)[SD]) {
    if constexpr (SD % 4 == 0) {
#pragma unroll
        for (int i = 0; i < SD / 4; ++i) {
            const float4 x = GLOBAL ? __ldg(reinterpret_cast<const float4*>(p) + i)
                                    : reinterpret_cast<const float4*>(p)[i];
            v[4 * i] = x.x;
            v[4 * i + 1] = x.y;
            v[4 * i + 2] = x.z;
            v[4 * i + 3] = x.w;
        }
    } else if constexpr (SD == 2) {
        const float2 x = GLOBAL ? __ldg(reinterpret_cast<const float2*>(p)) : *reinterpret_cast<const float2*>(p);
        v[0] = x.x;
        v[1] = x.y;
    } else {
#pragma unroll
        for (int i = 0; i < SD; ++i) v[i] = GLOBAL ? __ldg(p + i) : p[i];
    }
}

// SD consecutive floats at a 32-bit shared-memory address.
template <int SD>
__device__ __forceinline__ void lds_sub(uint32_t addr, float (&v)[SD]) {
    if constexpr (SD % 4 == 0) {
#pragma unroll
        for (int i = 0; i < SD / 4; ++i)
            asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                         : "=f"(v[4 * i]), "=f"(v[4 * i + 1]), "=f"(v[4 * i + 2]), "=f"(v[4 * i + 3])
                         : "r"(addr + 16 * i));
    } else if constexpr (SD == 2) {
        asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v[0]), "=f"(v[1]) : "r"(addr));
    } else {
#pragma unroll
        for (int i = 0; i < SD; ++i) asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v[i]) : "r"(addr + 4 * i));
    }
}

// r in shared memory, c in global memory.
template <int SD>
__device__ __forceinline__ float sub_dist(const float* r, const float* c) {
    float rv[SD], cv[SD];
    load_sub<SD, false>(r, rv);
    load_sub<SD, true>(c, cv);
    return sd_arith<SD>(rv, cv);
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
    if (a.only && !a.only[q]) return;
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

// ---- team kernel: codebook resident in shared memory --------------------------
//
// The same per-query algorithm as ivfpq_batch_kernel, run by teams of NT
// (64, 128 or 256) threads inside a persistent CTA of up to 1024 threads per SM.  The CTA
// copies the PQ codebook into shared memory once; each team then takes
// queries in turn and synchronises on its own named barrier, so up to eight
// queries share an SM and one team's barrier waits are filled by the others'
// work.  With LUT the
// team builds each list's residual table from the resident codebook; without
// it (short lists, where a table of M x 256 entries would outnumber the
// lookups) every ADC term is computed on the fly from the codebook.  Both
// produce the floats of the LUT path: one sd_arith expression per term, summed
// over subspaces in order.

constexpr int TEAM_THREADS = 1024;  // threads of a team CTA: TEAM_THREADS / NT teams of NT
constexpr double TEAM_OTF_MAX_LEN = 400.0;  // typical list length up to which the team kernel (on-the-fly terms) runs

template <int NT>
struct TeamMisc {
    uint32_t hist[256];
    int warp[NT / 32];
    uint32_t b[2];
    int carry[REF_BLOCK];
    unsigned char passf[NT];
    int buf_n, count, nb_list, next_q;
    uint32_t prune_key;
    float thr;
};

struct TeamLayout {
    int lut, res, pid, cut, lkey, ckey, cid, sortb, misc, total;
};

template <int NT>
__host__ __device__ inline TeamLayout team_layout(int M, int dim, int top_m, int p1, int lmax, int cap,
                                                  int sort_n, bool lut) {
    TeamLayout L;
    int o = 0;
    L.lut = lut ? take16(o, M * 256 * 4) : 0;
    L.res = take16(o, dim * 4);
    L.pid = take16(o, top_m * 4);
    L.cut = take16(o, (p1 > 0 ? p1 : 1) * 4);
    L.lkey = take16(o, (lmax > 0 ? lmax : 1) * 4);
    const int prefix = o;  // dead once the final sort starts
    L.ckey = take16(o, cap * 4);
    L.cid = take16(o, cap * 4);
    L.sortb = (sort_n * 8 <= prefix) ? 0 : take16(o, sort_n * 8);
    L.misc = take16(o, (int)sizeof(TeamMisc<NT>));
    L.total = o;
    return L;
}

template <int NT>
__device__ __forceinline__ void team_sync(int bar) {
    asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(NT) : "memory");
}

// block_exclusive_scan over one team (thread tt of NT, barrier `bar`).
template <int NT>
__device__ __forceinline__ int team_exclusive_scan(int v, int tt, int bar, int* s_warp, int& total) {
    const int lane = tt & 31, w = tt >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) s_warp[w] = x;
    team_sync<NT>(bar);
    if (w == 0) {
        int t = (lane < NT / 32) ? s_warp[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += y;
        }
        if (lane < NT / 32) s_warp[lane] = t;
    }
    team_sync<NT>(bar);
    const int wbase = w ? s_warp[w - 1] : 0;
    total = s_warp[NT / 32 - 1];
    team_sync<NT>(bar);
    return wbase + x - v;
}

// block_radix_select over one team.
template <int NT>
__device__ void team_radix_select(const uint32_t* keys, int n, int k, int tt, int bar, uint32_t* s_hist,
                                  uint32_t* s_b, uint32_t& kth, int& n_less) {
    uint32_t prefix = 0, mask = 0, kk = (uint32_t)k, less = 0;
#pragma unroll 1
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tt; i < 256; i += NT) s_hist[i] = 0;
        team_sync<NT>(bar);
        for (int i = tt; i < n; i += NT) {
            const uint32_t key = keys[i];
            if ((key & mask) == prefix) atomicAdd(&s_hist[(key >> shift) & 255u], 1u);
        }
        team_sync<NT>(bar);
        if (tt < 32) {
            const int lane = tt;
            uint32_t c[8], sum = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                c[j] = s_hist[lane * 8 + j];
                sum += c[j];
            }
            uint32_t incl = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            const uint32_t excl = incl - sum;
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
        team_sync<NT>(bar);
        const uint32_t b = s_b[0], below = s_b[1];
        prefix |= b << shift;
        mask |= 255u << shift;
        kk -= below;
        less += below;
        team_sync<NT>(bar);
    }
    kth = prefix;
    n_less = (int)less;
}

// block_bitonic_sort over one team.
template <int NT>
__device__ void team_bitonic_sort(unsigned long long* sb, int n_pow2, int tt, int bar) {
    for (int k = 2; k <= n_pow2; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = tt; i < n_pow2; i += NT) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const unsigned long long x = sb[i], y = sb[ixj];
                    const bool up = (i & k) == 0;
                    if ((x > y) == up) {
                        sb[i] = y;
                        sb[ixj] = x;
                    }
                }
            }
            team_sync<NT>(bar);
        }
    }
}

template <int NT>
struct TeamBufs {
    uint32_t* ckey;
    int32_t* cid;
    TeamMisc<NT>* ms;
};

// reduce_buffer over one team.
template <int NT>
__device__ void team_reduce_buffer(int rsel, int tt, int bar, const TeamBufs<NT>& tb) {
    TeamMisc<NT>* ms = tb.ms;
    const int n = ms->buf_n;
    uint32_t kth;
    int n_less;
    team_radix_select<NT>(tb.ckey, n, rsel, tt, bar, ms->hist, ms->b, kth, n_less);
    const int need_eq = rsel - n_less;
    int eq_base = 0, out_base = 0;
    for (int r0 = 0; r0 < n; r0 += NT) {
        const int i = r0 + tt;
        const bool in = i < n;
        const uint32_t key = in ? tb.ckey[i] : 0xffffffffu;
        const int32_t idv = in ? tb.cid[i] : 0;
        const int is_eq = (in && key == kth) ? 1 : 0;
        int eq_tot, k_tot;
        const int eq_pre = team_exclusive_scan<NT>(is_eq, tt, bar, ms->warp, eq_tot);
        const bool keep = in && (key < kth || (is_eq && eq_base + eq_pre < need_eq));
        eq_base += eq_tot;
        const int k_pre = team_exclusive_scan<NT>(keep ? 1 : 0, tt, bar, ms->warp, k_tot);
        if (keep) {
            tb.ckey[out_base + k_pre] = key;
            tb.cid[out_base + k_pre] = idv;
        }
        out_base += k_tot;
        team_sync<NT>(bar);
    }
    if (tt == 0) {
        ms->buf_n = out_base;
        ms->prune_key = kth;
    }
    team_sync<NT>(bar);
}

// append over one team.
template <int NT>
__device__ __forceinline__ void team_append(const ScanArgs& a, bool emit, uint32_t key, int32_t id, int tt, int bar,
                                            const TeamBufs<NT>& tb) {
    TeamMisc<NT>* ms = tb.ms;
    int tot;
    const int pre = team_exclusive_scan<NT>(emit ? 1 : 0, tt, bar, ms->warp, tot);
    if (tot == 0) return;
    if (ms->buf_n + tot > a.cap) team_reduce_buffer<NT>(a.rsel, tt, bar, tb);
    const int base = ms->buf_n;
    if (emit) {
        tb.ckey[base + pre] = key;
        tb.cid[base + pre] = id;
    }
    team_sync<NT>(bar);
    if (tt == 0) ms->buf_n = base + tot;
    team_sync<NT>(bar);
}

// k-th smallest (1-based) of n keys by one warp, as team_radix_select but
// without team barriers: 8-bit MSD passes that start below the bytes every
// key shares.
__device__ void warp_select_keys(const uint32_t* keys, int n, int k, uint32_t* hist, uint32_t& kth, int& n_less) {
    const int lane = threadIdx.x & 31;
    uint32_t kand = 0xffffffffu, kor = 0u;
    for (int i = lane; i < n; i += 32) {
        const uint32_t x = keys[i];
        kand &= x;
        kor |= x;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        kand &= __shfl_xor_sync(0xffffffffu, kand, o);
        kor |= __shfl_xor_sync(0xffffffffu, kor, o);
    }
    const uint32_t diff = kand ^ kor;
    int top = 24;
    while (top > 0 && ((diff >> top) & 255u) == 0u) top -= 8;
    uint32_t mask = top == 24 ? 0u : (0xffffffffu << (top + 8));
    uint32_t prefix = kand & mask, kk = (uint32_t)k, less = 0;
#pragma unroll 1
    for (int shift = top; shift >= 0; shift -= 8) {
        for (int i = lane; i < 256; i += 32) hist[i] = 0;
        __syncwarp();
        for (int i0 = 0; i0 < n; i0 += 32) {
            const int i = i0 + lane;
            const uint32_t key = i < n ? keys[i] : 0u;
            const bool in = i < n && (key & mask) == prefix;
            const uint32_t dg = (key >> shift) & 255u;
            if (in) atomicAdd(&hist[dg], 1u);
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
        uint32_t b = 0, below = 0, cb = 0;
        if (mine) {
            uint32_t run = excl;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (run + c[j] >= kk) {
                    b = (uint32_t)(lane * 8 + j);
                    below = run;
                    cb = c[j];
                    break;
                }
                run += c[j];
            }
        }
        const int src = __ffs(__ballot_sync(0xffffffffu, mine)) - 1;
        b = __shfl_sync(0xffffffffu, b, src);
        below = __shfl_sync(0xffffffffu, below, src);
        cb = __shfl_sync(0xffffffffu, cb, src);
        prefix |= b << shift;
        mask |= 255u << shift;
        kk -= below;
        less += below;
        __syncwarp();
        if (cb == 1u && shift > 0) {
            // one key left under the prefix: it is the k-th, and no key
            // below it shares the prefix
            for (int i0 = 0; i0 < n; i0 += 32) {
                const int i = i0 + lane;
                const uint32_t key = i < n ? keys[i] : 0u;
                const unsigned m = __ballot_sync(0xffffffffu, i < n && (key & mask) == prefix);
                if (m) {
                    prefix = __shfl_sync(0xffffffffu, key, __ffs(m) - 1);
                    break;
                }
            }
            break;
        }
    }
    kth = prefix;
    n_less = (int)less;
}

constexpr int WARP_SELECT_MAX = 1024;  // lists up to this length are selected by one warp
constexpr int RANK_SORT_MAX = 256;     // candidate sets up to this size are sorted by ranks

// ADC distance of one code row with every term computed from the resident
// codebook `cb` ([M][256][SD]) and the list residual `res`.
template <int M, int SD>
__device__ __forceinline__ float adc_otf(const uint8_t* __restrict__ row, const float* cb, const float* res) {
    float d = 0.0f;
    if constexpr (M % 16 == 0) {
        const uint4* r4 = reinterpret_cast<const uint4*>(row);
#pragma unroll
        for (int w = 0; w < M / 16; ++w) {
            const uint4 v = __ldg(r4 + w);
            const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int b = 0; b < 16; ++b) {
                const int m = 16 * w + b;
                const uint32_t code = (wd[b >> 2] >> (8 * (b & 3))) & 0xffu;
                float rv[SD], cv[SD];
                load_sub<SD, false>(res + m * SD, rv);
                load_sub<SD, false>(cb + ((size_t)m * 256 + code) * SD, cv);
                d = __fadd_rn(d, sd_arith<SD>(rv, cv));
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
                const int m = 4 * w + b;
                const uint32_t code = (v >> (8 * b)) & 0xffu;
                float rv[SD], cv[SD];
                load_sub<SD, false>(res + m * SD, rv);
                load_sub<SD, false>(cb + ((size_t)m * 256 + code) * SD, cv);
                d = __fadd_rn(d, sd_arith<SD>(rv, cv));
            }
        }
    }
    return d;
}

// Whether the on-the-fly ADC of (M, SD) runs skewed: the resident codebook is
// stored as [code][subspace][SD] and the lanes of one shared-memory phase
// (Z = 32 / SD lanes: 128 bytes of 4*SD-byte terms) walk the subspaces offset
// by lane % Z, so that at every step they read Z different subspaces.  With
// M*SD a multiple of 32 the codebook entry (k, m) then lies in bank group
// m % Z for every code k, and so does the residual of subspace m: both reads
// are free of bank conflicts whatever the codes.
template <int M, int SD>
struct AdcSkew {
    static constexpr int Z = (SD == 1 || SD == 2 || SD == 4 || SD == 8) ? 32 / SD : 0;
    static constexpr bool value = Z > 0 && (M * SD) % 32 == 0 && M % Z == 0;
};

// Byte t of a code row held in registers (static t).
template <int W>
__device__ __forceinline__ uint32_t code_byte(const uint32_t (&w)[W], int t) {
    return (w[t >> 2] >> (8 * (t & 3))) & 0xffu;
}

// ADC of one code row, skewed: lane offset j = lane % Z.  Step s (0 .. M+Z-2)
// handles subspace s - j when that is in [0, M); the row's bytes are first
// rotated by j so that the byte of step s sits at static position s mod M.
// Each lane still adds its terms in subspace order, so the sum is the same
// float as adc_otf's.
// The M code bytes of one row, rotated up by j (0 <= j < Z): byte p of the
// result is byte (p - j) mod M of the row.
template <int M, int Z>
__device__ __forceinline__ void load_rotated(const uint8_t* __restrict__ row, int j, uint32_t (&w)[M / 4]) {
    constexpr int W = M / 4;
    if constexpr (M % 16 == 0) {
        const uint4* r4 = reinterpret_cast<const uint4*>(row);
#pragma unroll
        for (int u = 0; u < M / 16; ++u) {
            const uint4 v = __ldg(r4 + u);
            w[4 * u] = v.x;
            w[4 * u + 1] = v.y;
            w[4 * u + 2] = v.z;
            w[4 * u + 3] = v.w;
        }
    } else {
        const uint32_t* r1 = reinterpret_cast<const uint32_t*>(row);
#pragma unroll
        for (int u = 0; u < W; ++u) w[u] = __ldg(r1 + u);
    }
    // rotate the M bytes up by j: words by j / 4 (barrel), then bytes by j % 4
    {
        const int jw = j >> 2;
#pragma unroll
        for (int b = 1; b < (Z + 3) / 4; b <<= 1) {
            if (jw & b) {
                uint32_t t[W];
#pragma unroll
                for (int u = 0; u < W; ++u) t[u] = w[(u - b + W) % W];
#pragma unroll
                for (int u = 0; u < W; ++u) w[u] = t[u];
            }
        }
        const int jb = 8 * (j & 3);
        if (jb) {
            uint32_t t[W];
#pragma unroll
            for (int u = 0; u < W; ++u) t[u] = __funnelshift_l(w[(u - 1 + W) % W], w[u], jb);
#pragma unroll
            for (int u = 0; u < W; ++u) w[u] = t[u];
        }
    }
}

template <int M, int SD>
__device__ __forceinline__ float adc_otf_skew(const uint8_t* __restrict__ row, const float* cbT, const float* res) {
    constexpr int Z = AdcSkew<M, SD>::Z;
    constexpr int W = M / 4;
    const int j = (threadIdx.x & 31) % Z;
    uint32_t w[W];
    load_rotated<M, Z>(row, j, w);
    // 32-bit shared addresses: + 4*SD*s is the residual of subspace s - j, + 4*SD*(k*M + s)
    // the codebook entry (k, s - j)
    const uint32_t rl = static_cast<uint32_t>(__cvta_generic_to_shared(res)) - 4u * SD * j;
    const uint32_t cl = static_cast<uint32_t>(__cvta_generic_to_shared(cbT)) - 4u * SD * j;
    float d = 0.0f;
#pragma unroll
    for (int st = 0; st < M + Z - 1; ++st) {
        const bool act = (st < Z - 1 || st >= M) ? (st >= j && st < j + M) : true;
        if (act) {
            const uint32_t k = code_byte<W>(w, st % M);
            float rv[SD], cv[SD];
            lds_sub<SD>(rl + 4u * SD * st, rv);
            lds_sub<SD>(cl + 4u * SD * (k * M + st), cv);
            d = __fadd_rn(d, sd_arith<SD>(rv, cv));
        }
    }
    return d;
}

// Skewed ADC of every row of a list, the rows of one lane streamed back to
// back: lane tt takes rows tt, tt + NT, ...  Period r (M steps) finishes the
// previous row's subspaces M-j .. M-1 in its first j steps and starts row r in
// the rest, so a lane idles only in the Z - 1 drain steps after its last row
// (adc_otf_skew idles Z - 1 steps per row).  Shared-memory reads keep the
// bank pattern of adc_otf_skew (lane j reads subspaces s with s mod Z = (step
// - j) mod Z), and each row's terms are still added in subspace order from
// 0.0f, so every key equals f2key(adc_otf_skew(row)).  Writes lkey[i] for i <
// n; the caller syncs the team.
template <int M, int SD, int NT>
__device__ __forceinline__ void adc_skew_stream(const uint8_t* __restrict__ rows, int n, int tt, const float* cbT,
                                                const float* res, uint32_t* lkey) {
    constexpr int Z = AdcSkew<M, SD>::Z;
    constexpr int W = M / 4;
    constexpr int HW = (Z - 1 + 3) / 4;  // words holding byte positions < Z - 1
    const int j = (threadIdx.x & 31) % Z;
    const int nr = n > tt ? (n - tt + NT - 1) / NT : 0;  // rows of this lane
    const int tw = tt & ~31;
    const int nw = n > tw ? (n - tw + NT - 1) / NT : 0;  // rows of the warp's first lane: the most
    // byte masks: position p < j takes the previous row
    uint32_t pm[HW];
#pragma unroll
    for (int u = 0; u < HW; ++u) {
        const int e = j - 4 * u;
        pm[u] = e >= 4 ? 0xffffffffu : (e <= 0 ? 0u : (1u << (8 * e)) - 1u);
    }
    // 32-bit shared addresses: + 4*SD*s is the residual of subspace s - j, + 4*SD*(k*M + s)
    // the codebook entry (k, s - j)
    const uint32_t rl = static_cast<uint32_t>(__cvta_generic_to_shared(res)) - 4u * SD * j;
    const uint32_t cl = static_cast<uint32_t>(__cvta_generic_to_shared(cbT)) - 4u * SD * j;
    uint32_t prev[HW];
#pragma unroll
    for (int u = 0; u < HW; ++u) prev[u] = 0u;
    float dprev = 0.0f;
    for (int r = 0; r < nw; ++r) {
        uint32_t w[W];
        if (r < nr) {
            load_rotated<M, Z>(rows + (size_t)(tt + r * NT) * M, j, w);
        } else {
#pragma unroll
            for (int u = 0; u < W; ++u) w[u] = 0u;
        }
        uint32_t h[HW];
#pragma unroll
        for (int u = 0; u < HW; ++u) h[u] = (prev[u] & pm[u]) | (w[u] & ~pm[u]);
        float dcur = 0.0f;
#pragma unroll
        for (int st = 0; st < M; ++st) {
            if (st < Z - 1) {
                const bool tail = st < j;  // previous row, subspace st - j + M
                const int sp = tail ? st + M : st;
                const uint32_t k = code_byte<HW>(h, st);
                float rv[SD], cv[SD];
                lds_sub<SD>(rl + 4u * SD * sp, rv);
                lds_sub<SD>(cl + 4u * SD * (k * M + sp), cv);
                const float t = sd_arith<SD>(rv, cv);
                if (tail)
                    dprev = __fadd_rn(dprev, t);
                else
                    dcur = __fadd_rn(dcur, t);
            } else {
                const uint32_t k = code_byte<W>(w, st);
                float rv[SD], cv[SD];
                lds_sub<SD>(rl + 4u * SD * st, rv);
                lds_sub<SD>(cl + 4u * SD * (k * M + st), cv);
                dcur = __fadd_rn(dcur, sd_arith<SD>(rv, cv));
            }
        }
        if (r > 0 && r - 1 < nr) lkey[tt + (r - 1) * NT] = f2key(dprev);
        dprev = dcur;
#pragma unroll
        for (int u = 0; u < HW; ++u) prev[u] = w[u];
    }
    // drain: the last row's subspaces M-j .. M-1
#pragma unroll
    for (int st = 0; st < Z - 1; ++st) {
        if (st < j) {
            const uint32_t k = code_byte<HW>(prev, st);
            float rv[SD], cv[SD];
            lds_sub<SD>(rl + 4u * SD * (st + M), rv);
            lds_sub<SD>(cl + 4u * SD * (k * M + st + M), cv);
            dprev = __fadd_rn(dprev, sd_arith<SD>(rv, cv));
        }
    }
    if (nw > 0 && nw - 1 < nr) lkey[tt + (nw - 1) * NT] = f2key(dprev);
}

// adc_skew_stream for G queries probing the same list: each step reads the
// codebook entry once and adds its term for every query (residuals res + g *
// rstride), so the codebook traffic per term falls G-fold.  Every query's
// terms are still added in subspace order from 0.0f: lkey[g * lstride + i] is
// the key adc_skew_stream writes for query g.  The caller syncs the team.
template <int M, int SD, int NT, int G>
__device__ __forceinline__ void adc_skew_stream_multi(const uint8_t* __restrict__ rows, int n, int tt,
                                                      const float* cbT, const float* res, int rstride,
                                                      uint32_t* lkey, int lstride) {
    constexpr int Z = AdcSkew<M, SD>::Z;
    constexpr int W = M / 4;
    constexpr int HW = (Z - 1 + 3) / 4;
    const int j = (threadIdx.x & 31) % Z;
    const int nr = n > tt ? (n - tt + NT - 1) / NT : 0;
    const int tw = tt & ~31;
    const int nw = n > tw ? (n - tw + NT - 1) / NT : 0;
    uint32_t pm[HW];
#pragma unroll
    for (int u = 0; u < HW; ++u) {
        const int e = j - 4 * u;
        pm[u] = e >= 4 ? 0xffffffffu : (e <= 0 ? 0u : (1u << (8 * e)) - 1u);
    }
    uint32_t rl[G];
#pragma unroll
    for (int g = 0; g < G; ++g)
        rl[g] = static_cast<uint32_t>(__cvta_generic_to_shared(res + (size_t)g * rstride)) - 4u * SD * j;
    const uint32_t cl = static_cast<uint32_t>(__cvta_generic_to_shared(cbT)) - 4u * SD * j;
    uint32_t prev[HW];
#pragma unroll
    for (int u = 0; u < HW; ++u) prev[u] = 0u;
    float dprev[G];
#pragma unroll
    for (int g = 0; g < G; ++g) dprev[g] = 0.0f;
    for (int r = 0; r < nw; ++r) {
        uint32_t w[W];
        if (r < nr) {
            load_rotated<M, Z>(rows + (size_t)(tt + r * NT) * M, j, w);
        } else {
#pragma unroll
            for (int u = 0; u < W; ++u) w[u] = 0u;
        }
        uint32_t h[HW];
#pragma unroll
        for (int u = 0; u < HW; ++u) h[u] = (prev[u] & pm[u]) | (w[u] & ~pm[u]);
        float dcur[G];
#pragma unroll
        for (int g = 0; g < G; ++g) dcur[g] = 0.0f;
#pragma unroll
        for (int st = 0; st < M; ++st) {
            if (st < Z - 1) {
                const bool tail = st < j;  // previous row, subspace st - j + M
                const int sp = tail ? st + M : st;
                const uint32_t k = code_byte<HW>(h, st);
                float cv[SD];
                lds_sub<SD>(cl + 4u * SD * (k * M + sp), cv);
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    float rv[SD];
                    lds_sub<SD>(rl[g] + 4u * SD * sp, rv);
                    const float t = sd_arith<SD>(rv, cv);
                    if (tail)
                        dprev[g] = __fadd_rn(dprev[g], t);
                    else
                        dcur[g] = __fadd_rn(dcur[g], t);
                }
            } else {
                const uint32_t k = code_byte<W>(w, st);
                float cv[SD];
                lds_sub<SD>(cl + 4u * SD * (k * M + st), cv);
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    float rv[SD];
                    lds_sub<SD>(rl[g] + 4u * SD * st, rv);
                    dcur[g] = __fadd_rn(dcur[g], sd_arith<SD>(rv, cv));
                }
            }
        }
        if (r > 0 && r - 1 < nr) {
#pragma unroll
            for (int g = 0; g < G; ++g) lkey[g * lstride + tt + (r - 1) * NT] = f2key(dprev[g]);
        }
#pragma unroll
        for (int g = 0; g < G; ++g) dprev[g] = dcur[g];
#pragma unroll
        for (int u = 0; u < HW; ++u) prev[u] = w[u];
    }
#pragma unroll
    for (int st = 0; st < Z - 1; ++st) {
        if (st < j) {
            const uint32_t k = code_byte<HW>(prev, st);
            float cv[SD];
            lds_sub<SD>(cl + 4u * SD * (k * M + st + M), cv);
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float rv[SD];
                lds_sub<SD>(rl[g] + 4u * SD * (st + M), rv);
                dprev[g] = __fadd_rn(dprev[g], sd_arith<SD>(rv, cv));
            }
        }
    }
    if (nw > 0 && nw - 1 < nr) {
#pragma unroll
        for (int g = 0; g < G; ++g) lkey[g * lstride + tt + (nw - 1) * NT] = f2key(dprev[g]);
    }
}

// Residual of list c for this query; with LUT also the list's table from the
// resident codebook.  Ends on the team barrier.
template <int M, int SD, bool LUT, int NT>
__device__ __forceinline__ void team_prepare_list(const ScanArgs& a, const float* qv, uint32_t c, const float* cb,
                                                  float* res, float* lut, int tt, int bar) {
    const float* cv = a.centroids + (size_t)c * a.dim;
    for (int t = tt; t < a.dim; t += NT) res[t] = qv[t] - cv[t];
    team_sync<NT>(bar);
    if constexpr (LUT) {
        for (int e = tt; e < M * 256; e += NT) {
            const int m = e >> 8;
            float rv[SD], cv2[SD];
            load_sub<SD, false>(res + m * SD, rv);
            load_sub<SD, false>(cb + (size_t)e * SD, cv2);
            lut[e] = sd_arith<SD>(rv, cv2);
        }
        team_sync<NT>(bar);
    }
}

template <int M, int SD, bool LUT>
__device__ __forceinline__ float team_adc(const ScanArgs& a, int start, int i, const float* cb, const float* res,
                                          const float* lut) {
    const uint8_t* row = a.codes + (size_t)(start + i) * M;
    if constexpr (LUT)
        return adc<M>(row, lut);
    else if constexpr (AdcSkew<M, SD>::value)
        return adc_otf_skew<M, SD>(row, cb, res);
    else
        return adc_otf<M, SD>(row, cb, res);
}

template <int M, int SD, bool LUT, int NT>
__global__ void __launch_bounds__(TEAM_THREADS, 1)
    ivfpq_team_kernel(const ScanArgs a, int nq, int nteams, int team_bytes) {
    // the ref_compat phase-2 overflow ranks need whole 128-thread groups: the
    // host launches teams of 64 threads only without ref_compat
    static_assert(NT % REF_BLOCK == 0 || NT == 64, "team size");
    extern __shared__ __align__(16) unsigned char smem[];
    constexpr int CBF = M * 256 * SD;  // codebook floats
    float* cb = reinterpret_cast<float*>(smem);
    {
        static_assert(CBF % 4 == 0, "the codebook copies as float4");
        if constexpr (!LUT && AdcSkew<M, SD>::value) {
            // [subspace][code][SD] -> [code][subspace][SD], walking the
            // destination in order (conflict-free stores; the reads hit L2)
            for (int e = threadIdx.x; e < M * 256; e += blockDim.x) {
                const int k = e / M, m = e - k * M;
                float v[SD];
                load_sub<SD, true>(a.codebook + ((size_t)m * 256 + k) * SD, v);
#pragma unroll
                for (int t = 0; t < SD; ++t) cb[(size_t)e * SD + t] = v[t];
            }
        } else {
            const float4* src = reinterpret_cast<const float4*>(a.codebook);
            float4* dst = reinterpret_cast<float4*>(cb);
            for (int i = threadIdx.x; i < CBF / 4; i += blockDim.x) dst[i] = __ldg(src + i);
        }
    }
    __syncthreads();
    const int team = threadIdx.x / NT, tt = threadIdx.x % NT;
    const int bar = 1 + team;
    unsigned char* ts = smem + (size_t)(CBF * 4 + 15) / 16 * 16 + (size_t)team * team_bytes;
    const TeamLayout L = team_layout<NT>(M, a.dim, a.top_m, a.p1, a.lmax, a.cap, a.sort_n, LUT);
    float* lut = reinterpret_cast<float*>(ts + L.lut);
    float* res = reinterpret_cast<float*>(ts + L.res);
    uint32_t* pid = reinterpret_cast<uint32_t*>(ts + L.pid);
    float* cut = reinterpret_cast<float*>(ts + L.cut);
    uint32_t* lkey = reinterpret_cast<uint32_t*>(ts + L.lkey);
    unsigned long long* sortb = reinterpret_cast<unsigned long long*>(ts + L.sortb);
    const TeamBufs<NT> tb{reinterpret_cast<uint32_t*>(ts + L.ckey), reinterpret_cast<int32_t*>(ts + L.cid),
                          reinterpret_cast<TeamMisc<NT>*>(ts + L.misc)};
    TeamMisc<NT>* ms = tb.ms;
    const int P = a.top_m;

    // first query by position, then (with a counter) whichever is next, so
    // teams that drew cheap queries take more and the launch ends together
    for (int q = blockIdx.x * nteams + team; q < nq;) {
        const float* qv = a.queries + (size_t)q * a.dim;
        // prune (gpu_global.cu:43-51); ids outside [0, nlist) are skipped
        const float best = a.probe_dists[(size_t)q * P];
        const float pthr = best * a.prune_ratio;
        for (int j = tt; j < P; j += NT) {
            const float d = a.probe_dists[(size_t)q * P + j];
            const uint32_t id = a.probe_ids[(size_t)q * P + j];
            pid[j] = (d > pthr || id >= (uint32_t)a.nlist) ? FG_INVALID_PROBE : id;
        }
        if (tt == 0) {
            ms->buf_n = 0;
            ms->count = 0;
            ms->prune_key = 0xffffffffu;
        }
        team_sync<NT>(bar);

        // ---- phase 1 ----------------------------------------------------------
        for (int j = 0; j < a.p1; ++j) {
            const uint32_t c = pid[j];
            int start = 0, len = 0;
            if (c != FG_INVALID_PROBE) {
                start = a.offsets[c];
                len = a.offsets[c + 1] - start;
            }
            if (len <= 0) {
                if (tt == 0) cut[j] = 0.0f;
                continue;
            }
            const int wc = len < a.limit_k ? len : a.limit_k;
            const int scan = (a.ref_compat && len > REF_P1_CLAMP) ? REF_P1_CLAMP : len;
            team_prepare_list<M, SD, LUT, NT>(a, qv, c, cb, res, lut, tt, bar);
            if constexpr (!LUT && AdcSkew<M, SD>::value)
                adc_skew_stream<M, SD, NT>(a.codes + (size_t)start * M, scan, tt, cb, res, lkey);
            else
                for (int i = tt; i < scan; i += NT) lkey[i] = f2key(team_adc<M, SD, LUT>(a, start, i, cb, res, lut));
            team_sync<NT>(bar);
            if (a.small == 1 && scan <= WARP_SELECT_MAX) {
                // one warp selects and emits (the buffer can never need a cut)
                if (tt < 32) {
                    uint32_t kth;
                    int n_less;
                    warp_select_keys(lkey, scan, wc, ms->hist, kth, n_less);
                    const unsigned lt = lanemask_lt();
                    const int need_eq = wc - n_less;
                    const uint32_t pk = ms->prune_key;
                    int eq_base = 0, bn = ms->buf_n;
                    for (int i0 = 0; i0 < scan; i0 += 32) {
                        const int i = i0 + tt;
                        const bool in = i < scan;
                        const uint32_t key = in ? lkey[i] : 0xffffffffu;
                        const bool is_eq = in && key == kth;
                        const unsigned eqb = __ballot_sync(0xffffffffu, is_eq);
                        const bool sel = in && (key < kth || (is_eq && eq_base + __popc(eqb & lt) < need_eq));
                        eq_base += __popc(eqb);
                        const bool emit = sel && key < pk;
                        const unsigned eb = __ballot_sync(0xffffffffu, emit);
                        if (emit) {
                            const int pos = bn + __popc(eb & lt);
                            tb.ckey[pos] = key;
                            tb.cid[pos] = start + i;
                        }
                        bn += __popc(eb);
                    }
                    if (tt == 0) {
                        ms->buf_n = bn;
                        cut[j] = key2f(kth);
                        ms->count += wc;
                    }
                }
                team_sync<NT>(bar);
                continue;
            }
            uint32_t kth;
            int n_less;
            team_radix_select<NT>(lkey, scan, wc, tt, bar, ms->hist, ms->b, kth, n_less);
            if (tt == 0) {
                cut[j] = key2f(kth);
                ms->count += wc;
            }
            const int need_eq = wc - n_less;
            int eq_base = 0;
            for (int r0 = 0; r0 < scan; r0 += NT) {
                const int i = r0 + tt;
                const bool in = i < scan;
                const uint32_t key = in ? lkey[i] : 0xffffffffu;
                const int is_eq = (in && key == kth) ? 1 : 0;
                int eq_tot;
                const int eq_pre = team_exclusive_scan<NT>(is_eq, tt, bar, ms->warp, eq_tot);
                const bool sel = in && (key < kth || (is_eq && eq_base + eq_pre < need_eq));
                eq_base += eq_tot;
                const bool emit = sel && key < ms->prune_key;
                team_append<NT>(a, emit, key, emit ? start + i : 0, tt, bar, tb);
            }
        }

        // ---- threshold (gpu_global.cu:394-426) ---------------------------------
        team_sync<NT>(bar);
        if (tt == 0) {
            float mn = FLT_MAX;
            for (int j = 0; j < a.p1; ++j)
                if (cut[j] > 0.0f && cut[j] < mn) mn = cut[j];
            ms->thr = (mn < FLT_MAX) ? mn * a.coeff : FLT_MAX;
        }
        team_sync<NT>(bar);
        const float thr = ms->thr;

        // ---- phase 2 ------------------------------------------------------------
        for (int j = a.p1; j < P; ++j) {
            const uint32_t c = pid[j];
            int start = 0, len = 0;
            if (c != FG_INVALID_PROBE) {
                start = a.offsets[c];
                len = a.offsets[c + 1] - start;
            }
            if (len <= 0) continue;
            if (tt == 0) ms->nb_list = 0;
            team_prepare_list<M, SD, LUT, NT>(a, qv, c, cb, res, lut, tt, bar);
            for (int c0 = 0; c0 < len; c0 += NT) {
                const int i = c0 + tt;
                float d = 0.0f;
                bool pass = false;
                if (i < len) {
                    d = team_adc<M, SD, LUT>(a, start, i, cb, res, lut);
                    pass = d <= thr;
                }
                int p_tot;
                const int p_pre = team_exclusive_scan<NT>(pass ? 1 : 0, tt, bar, ms->warp, p_tot);
                const int rank = ms->nb_list + p_pre;
                const uint32_t key = f2key(d);
                const bool emit = pass && (!a.ref_compat || rank < REF_BLOCK) && key < ms->prune_key;
                team_append<NT>(a, emit, key, emit ? start + i : 0, tt, bar, tb);
                if (tt == 0) ms->nb_list += p_tot;
                team_sync<NT>(bar);
            }
            const int s_count = ms->nb_list;
            if (!a.ref_compat || s_count <= REF_BLOCK) {
                if (tt == 0) ms->count += s_count;
                team_sync<NT>(bar);
                continue;
            }
            // overflow: each of the reference's 128 threads re-emits its first
            // (s_count - 128) passing vectors (gpu_global.cu:508-526)
            const int quota = s_count - REF_BLOCK;
            if (tt < REF_BLOCK) ms->carry[tt] = 0;
            if (tt == 0) ms->count += REF_BLOCK;
            team_sync<NT>(bar);
            for (int c0 = 0; c0 < len; c0 += NT) {
                const int i = c0 + tt;
                float d = 0.0f;
                bool pass = false;
                if (i < len) {
                    d = team_adc<M, SD, LUT>(a, start, i, cb, res, lut);
                    pass = d <= thr;
                }
                ms->passf[tt] = pass ? 1 : 0;
                team_sync<NT>(bar);
                // rank among the passing vectors of the same reference thread (i mod 128)
                const int t = tt % REF_BLOCK;
                int rank = ms->carry[t];
                for (int u = t; u < tt; u += REF_BLOCK) rank += ms->passf[u];
                const bool re = pass && rank < quota;
                int r_tot;
                (void)team_exclusive_scan<NT>(re ? 1 : 0, tt, bar, ms->warp, r_tot);
                if (tt == 0) ms->count += r_tot;
                const uint32_t key = f2key(d);
                const bool emit = re && key < ms->prune_key;
                team_append<NT>(a, emit, key, emit ? start + i : 0, tt, bar, tb);
                if (tt < REF_BLOCK) {
                    int add = 0;
                    for (int u = tt; u < NT; u += REF_BLOCK) add += ms->passf[u];
                    ms->carry[tt] += add;
                }
                team_sync<NT>(bar);
            }
        }

        // ---- select, sort and gather (gpu_global.cu:838-871) -------------------
        team_sync<NT>(bar);
        if (ms->buf_n > a.rsel) team_reduce_buffer<NT>(a.rsel, tt, bar, tb);
        const int n = ms->buf_n;
        const int npow = next_pow2(n > 0 ? n : 1);
        if (n <= RANK_SORT_MAX) {
            // rank sort: entry i goes to the number of entries before it in
            // (key, position) order; the keys are read as broadcasts
            for (int i = tt; i < n; i += NT) {
                const uint32_t key = tb.ckey[i];
                int r = 0;
                int u = 0;
                for (; u + 4 <= n; u += 4) {
                    const uint4 k4 = *reinterpret_cast<const uint4*>(tb.ckey + u);
                    r += (k4.x < key) || (k4.x == key && u < i);
                    r += (k4.y < key) || (k4.y == key && u + 1 < i);
                    r += (k4.z < key) || (k4.z == key && u + 2 < i);
                    r += (k4.w < key) || (k4.w == key && u + 3 < i);
                }
                for (; u < n; ++u) {
                    const uint32_t ku = tb.ckey[u];
                    r += (ku < key) || (ku == key && u < i);
                }
                sortb[r] = ((unsigned long long)key << 32) | (unsigned)i;
            }
            team_sync<NT>(bar);
        } else {
            for (int i = tt; i < npow; i += NT)
                sortb[i] = (i < n) ? ((unsigned long long)tb.ckey[i] << 32) | (unsigned)i : ~0ull;
            team_sync<NT>(bar);
            team_bitonic_sort<NT>(sortb, npow, tt, bar);
        }
        const int count = ms->count;
        const int rm = a.rerank_m;
        const int ak = count < rm ? count : rm;
        const int pend = a.write_pad ? rm : (ak < rm ? ak : rm);
        for (int p = tt; p < pend; p += NT) {
            const size_t o = (size_t)q * rm + p;
            if (a.ref_compat && p >= REF_BLOCK) {
                a.top_ids[o] = 0;
                a.top_dists[o] = 0.0f;
            } else if (p < ak) {
                const unsigned long long e = sortb[p];
                a.top_ids[o] = __ldg(a.vids + tb.cid[(unsigned)(e & 0xffffffffu)]);
                a.top_dists[o] = key2f((uint32_t)(e >> 32));
            } else {
                a.top_ids[o] = -1;
                a.top_dists[o] = FLT_MAX;
            }
        }
        if (tt == 0) {
            a.top_counts[q] = ak;
            if (a.cand_counts) a.cand_counts[q] = count;
            ms->next_q = a.work_counter ? gridDim.x * nteams + atomicAdd(a.work_counter, 1) : q + gridDim.x * nteams;
        }
        team_sync<NT>(bar);  // the next query reuses every buffer
        q = ms->next_q;
    }
}

using TeamKernel = void (*)(const ScanArgs, int, int, int);

// ---- split path: one CTA per (query, probed list) -----------------------------
//
// For long lists (hundreds of vectors per list, tens of probes per query) the
// per-query kernel serialises a query's probes inside one CTA, with block
// barriers around every LUT, selection and emission round.  The split path
// gives every (query, probed list) pair a CTA of its own for its turn:
//
//   split_pairs_*     list the pairs whose list is non-empty (a shard of a
//                     list-sharded index owns only some of each query's
//                     probes), grouped by list; persistent CTAs of the two
//                     phase kernels take them from work counters;
//   split_p1_pair     phase 1 (the first p1 probes): LUT, ADC of the list,
//                     the limit_k smallest by (distance, position), the cutoff
//                     (gpu_global.cu:79-166, 212-253, 321-390);
//   split_p2_pair     phase 2 (the other probes): threshold from the query's
//                     phase-1 cutoffs (gpu_global.cu:394-426), LUT, ADC, the
//                     passing vectors with the reference's 128-slot buffer and
//                     overflow re-emission in ref_compat mode (:428-527);
//   split_select_kernel  per query: the rerank_m smallest candidates, sorted,
//                     with their vector ids (gpu_global.cu:533-576, 838-871).
//
// Candidates go to a per-query region of capg 64-bit keys in global memory as
// (distance key << 32 | order), order = probe index << 20 | position (plus
// 1 << 19 for an overflow re-emission).  Sorting by that key is sorting by
// distance with ties in emission order -- the order the per-query kernel
// appends in -- so the slots themselves can be taken in any order.  A query
// whose candidates overflow its region, or whose ties at the selection
// boundary overflow the sort buffer, is flagged and recomputed by the
// per-query kernel.  Every float is the same expression as in the per-query
// kernel, so both paths return identical results.

constexpr int SPLIT_NT = 128;
constexpr int SEL_NT = 512;

__host__ __device__ inline int split_keys_bytes(int lmax) { return ((lmax > 0 ? lmax : 1) * 4 + 15) / 16 * 16; }

constexpr int SPLIT_P2_NT = 256;  // phase-2 CTAs outside ref_compat (more warps hide the code loads)
#ifndef FG_SPLIT_P1_NT
#define FG_SPLIT_P1_NT 256
#endif
constexpr int SPLIT_P1_NT = FG_SPLIT_P1_NT;  // phase-1 CTAs; also the rows that set its bound

struct SplitMisc {
    int4 rec;  // persistent phase kernels: the pair taken next
    uint32_t hist[256];
    int warp[SPLIT_P2_NT / 32];
    uint32_t b[2];
    int base, n_pass;
    float thr;
};

// The probed list of pair (q, j) after the prune, as start/len (len 0: skipped).
__device__ __forceinline__ void split_probe(const ScanArgs& a, int q, int j, uint32_t& c, int& start, int& len) {
    const int P = a.top_m;
    const float best = a.probe_dists[(size_t)q * P];
    const float d = a.probe_dists[(size_t)q * P + j];
    c = a.probe_ids[(size_t)q * P + j];
    start = 0;
    len = 0;
    if (d > best * a.prune_ratio || c >= (uint32_t)a.nlist) {
        c = FG_INVALID_PROBE;
        return;
    }
    start = a.offsets[c];
    len = a.offsets[c + 1] - start;
}

// LUT of (query, list c) in shared memory: the entries of build_lut, for the
// first MB subspaces (all M by default); the residual covers every dimension.
template <int M, int SD, int NT = SPLIT_NT, int MB = M>
__device__ __forceinline__ void split_lut(const ScanArgs& a, const float* qv, uint32_t c, float* res, float* lut) {
    const float* cv = a.centroids + (size_t)c * a.dim;
    for (int t = threadIdx.x; t < a.dim; t += NT) res[t] = qv[t] - cv[t];
    __syncthreads();
    if constexpr (SD == 2) {
        // two codewords per thread: one 16-byte codebook load, one 8-byte store
#pragma unroll 4
        for (int e2 = threadIdx.x; e2 < MB * 128; e2 += NT) {
            const int m = e2 >> 7;
            const float4 cb = __ldg(reinterpret_cast<const float4*>(a.codebook) + e2);
            const float2 r = *reinterpret_cast<const float2*>(res + m * 2);
            const float rv[2] = {r.x, r.y}, c0[2] = {cb.x, cb.y}, c1[2] = {cb.z, cb.w};
            reinterpret_cast<float2*>(lut)[e2] = make_float2(sd_arith<2>(rv, c0), sd_arith<2>(rv, c1));
        }
    } else {
#pragma unroll 4
        for (int e = threadIdx.x; e < MB * 256; e += NT) {
            const int m = e >> 8;
            lut[e] = sub_dist<SD>(res + m * SD, a.codebook + (size_t)e * SD);
        }
    }
    __syncthreads();
}

// Keys of rows [0, n) of the list: thread t takes rows t, t + SPLIT_NT, ...
template <int M, int NT = SPLIT_NT>
__device__ __forceinline__ void split_keys(const ScanArgs& a, int start, int n, const float* lut, uint32_t* keys) {
    for (int i = threadIdx.x; i < n; i += NT) keys[i] = f2key(adc<M>(a.codes + (size_t)(start + i) * M, lut));
    __syncthreads();
}

// ADC key of one row, or 0xffffffff once the running sum exceeds `bound`:
// every LUT entry is a sum of squares (>= 0), so under round-to-nearest the
// running sum never decreases and such a row's full distance exceeds bound too.
// Rows within the bound are summed to the end in subspace order, so their keys
// are adc<M>'s bit for bit.  `first` holds the row's first 16 codes; a later
// 16-code word is loaded only while the row is alive, and issued halfway
// through the word before it (a row dead after 8 terms is dead after 16), so
// the rows rejected in their first word -- nearly all of them past a tight
// bound -- cost one 16-byte load instead of M bytes.
template <int M>
__device__ __forceinline__ uint32_t adc_bounded_lazy(uint4 first, const uint8_t* row, const float* lut,
                                                     float bound) {
    const uint4* r4 = reinterpret_cast<const uint4*>(row);
    float d = 0.0f;
    bool alive = true;
    uint4 v = first, next = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int w = 0; w < M / 16; ++w) {
        if (alive) {
            const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int b = 0; b < 16; ++b) {
                const uint32_t code = (wd[b >> 2] >> (8 * (b & 3))) & 0xffu;
                d = __fadd_rn(d, lut[(16 * w + b) * 256 + code]);
                if (b == 7 && w + 1 < M / 16 && d <= bound) next = __ldg(r4 + w + 1);
            }
            alive = d <= bound;
            v = next;
        }
    }
    return alive ? f2key(d) : 0xffffffffu;
}

// keys[i] for rows i = first, first + NT, ... < n of the list at `start`, each
// bounded by `bound`; the next row's first 16 codes are loaded while a row's
// sum runs.
template <int M, int NT>
__device__ __forceinline__ void keys_bounded(const ScanArgs& a, int start, int first, int n, const float* lut,
                                             float bound, uint32_t* keys) {
    static_assert(M % 16 == 0, "16-code chunks");
    int i = first + threadIdx.x;
    if (i >= n) return;
    const uint8_t* rows = a.codes + (size_t)start * M;
    uint4 cur = __ldg(reinterpret_cast<const uint4*>(rows + (size_t)i * M));
    for (; i < n; i += NT) {
        const bool more = i + NT < n;
        uint4 nxt = cur;
        if (more) nxt = __ldg(reinterpret_cast<const uint4*>(rows + (size_t)(i + NT) * M));
        keys[i] = adc_bounded_lazy<M>(cur, rows + (size_t)i * M, lut, bound);
        cur = nxt;
    }
}

// Terms 16w .. 16w + 15 of a row computed from the codebook instead of a LUT:
// the LUT entry's expression (sd_arith on the same residual and codeword), so
// the same floats, added in subspace order.  The codewords of TB terms are
// loaded before they are summed.
template <int SD>
__device__ __forceinline__ float otf_word(uint4 v, int w, const float* res, const float* cb, float d) {
    constexpr int TB = SD <= 2 ? 16 : (SD <= 4 ? 4 : 2);
    const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int b0 = 0; b0 < 16; b0 += TB) {
        float cv[TB][SD];
#pragma unroll
        for (int k = 0; k < TB; ++k) {
            const int b = b0 + k;
            const uint32_t code = (wd[b >> 2] >> (8 * (b & 3))) & 0xffu;
            load_sub<SD, true>(cb + ((size_t)(16 * w + b) * 256 + code) * SD, cv[k]);
        }
#pragma unroll
        for (int k = 0; k < TB; ++k) {
            float rv[SD];
            load_sub<SD, false>(res + (16 * w + b0 + k) * SD, rv);
            d = __fadd_rn(d, sd_arith<SD>(rv, cv[k]));
        }
    }
    return d;
}

// adc_bounded_lazy with a LUT of the first 16 subspaces only: past a tight
// bound nearly every row is rejected within its first 16 terms, so the other
// subspaces' LUT entries would mostly go unread; a row still alive after them
// finishes from the codebook (otf_word).  Bit for bit adc<M>'s key for rows
// within the bound.
template <int M, int SD>
__device__ __forceinline__ uint32_t adc_bounded_prefix(uint4 first, const uint8_t* row, const float* lut,
                                                       const float* res, const float* cb, float bound) {
    const uint4* r4 = reinterpret_cast<const uint4*>(row);
    float d = 0.0f;
    uint4 next = make_uint4(0u, 0u, 0u, 0u);
    {
        const uint32_t wd[4] = {first.x, first.y, first.z, first.w};
#pragma unroll
        for (int b = 0; b < 16; ++b) {
            const uint32_t code = (wd[b >> 2] >> (8 * (b & 3))) & 0xffu;
            d = __fadd_rn(d, lut[b * 256 + code]);
            if (b == 7 && M / 16 > 1 && d <= bound) next = __ldg(r4 + 1);
        }
    }
    bool alive = d <= bound;
#pragma unroll 1
    for (int w = 1; w < M / 16; ++w) {
        if (!alive) break;
        const uint4 v = next;
        if (w + 1 < M / 16) next = __ldg(r4 + w + 1);
        d = otf_word<SD>(v, w, res, cb, d);
        alive = d <= bound;
    }
    return alive ? f2key(d) : 0xffffffffu;
}

// keys_bounded over a LUT of the first 16 subspaces (adc_bounded_prefix).
template <int M, int SD, int NT>
__device__ __forceinline__ void keys_bounded_prefix(const ScanArgs& a, int start, int n, const float* lut,
                                                    const float* res, float bound, uint32_t* keys) {
    static_assert(M % 16 == 0, "16-code chunks");
    int i = threadIdx.x;
    if (i < n) {
        const uint8_t* rows = a.codes + (size_t)start * M;
        uint4 cur = __ldg(reinterpret_cast<const uint4*>(rows + (size_t)i * M));
        for (; i < n; i += NT) {
            const bool more = i + NT < n;
            uint4 nxt = cur;
            if (more) nxt = __ldg(reinterpret_cast<const uint4*>(rows + (size_t)(i + NT) * M));
            keys[i] = adc_bounded_prefix<M, SD>(cur, rows + (size_t)i * M, lut, res, a.codebook, bound);
            cur = nxt;
        }
    }
    __syncthreads();
}

template <int M, int SD, int NT>
__device__ void split_p1_pair(const ScanArgs& a, int q, int j, uint32_t c, int start, int len, unsigned char* smem) {
    float* lut = reinterpret_cast<float*>(smem);
    float* res = lut + M * 256;
    uint32_t* keys = reinterpret_cast<uint32_t*>(res + (a.dim + 3) / 4 * 4);
    SplitMisc* ms = reinterpret_cast<SplitMisc*>(reinterpret_cast<unsigned char*>(keys) + split_keys_bytes(a.lmax));
    if (len <= 0) {
        if (threadIdx.x == 0) a.cut_g[(size_t)q * a.p1 + j] = 0.0f;
        return;
    }
    const int wc = len < a.limit_k ? len : a.limit_k;
    const int scan = (a.ref_compat && len > REF_P1_CLAMP) ? REF_P1_CLAMP : len;
    split_lut<M, SD, NT>(a, a.queries + (size_t)q * a.dim, c, res, lut);
    uint32_t kth;
    int n_less;
    if constexpr (M % 16 == 0) {
        // the first NT rows in full; their wc-th smallest distance bounds
        // the list's wc-th from above, so a later row whose partial sum passes
        // it cannot be among the wc selected, and it gets the largest key
        // (which changes neither the wc-th key nor the count below it)
        const int head = (scan < NT || wc > NT) ? scan : NT;
        split_keys<M, NT>(a, start, head, lut, keys);
        if (scan > head && wc <= head) {
            block_radix_select<NT>(keys, head, wc, ms->hist, ms->b, kth, n_less);
            keys_bounded<M, NT>(a, start, head, scan, lut, key2f(kth), keys);
            __syncthreads();
        }
    } else {
        split_keys<M, NT>(a, start, scan, lut, keys);
    }
    unsigned long long* dst = a.cand_g + (size_t)q * a.capg;
    const unsigned long long jo = (unsigned long long)((uint32_t)j << 20);
    // The rows still in the running (key below 0xffffffff) go to a compact
    // (key, position) list in the LUT's space, dead by now; the selection runs
    // over them alone (the others all lie above the wc-th key, so the wc-th
    // key and the count below it do not change).
    {
        const int ccap = M * 128;
        uint32_t* ckey = reinterpret_cast<uint32_t*>(lut);
        int32_t* cpos = reinterpret_cast<int32_t*>(lut) + ccap;
        int n_t = 0;
        for (int i = threadIdx.x; i < scan; i += NT) n_t += keys[i] != 0xffffffffu ? 1 : 0;
        int n_c;
        int o = block_exclusive_scan<NT>(n_t, ms->warp, n_c);
        if (n_c <= ccap) {
            for (int i = threadIdx.x; i < scan; i += NT)
                if (keys[i] != 0xffffffffu) {
                    ckey[o] = keys[i];
                    cpos[o++] = i;
                }
            __syncthreads();
            block_radix_select<NT>(ckey, n_c, wc, ms->hist, ms->b, kth, n_less);
            int eq_t = 0, sel_t = 0;
            for (int u = threadIdx.x; u < n_c; u += NT) {
                eq_t += ckey[u] == kth ? 1 : 0;
                sel_t += ckey[u] <= kth ? 1 : 0;
            }
            int eq_tot;
            (void)block_exclusive_scan<NT>(eq_t, ms->warp, eq_tot);
            if (eq_tot == wc - n_less) {
                // every row at the cutoff is selected: no position order needed
                if (threadIdx.x == 0) {
                    a.cut_g[(size_t)q * a.p1 + j] = key2f(kth);
                    ms->base = atomicAdd(a.cnt_g + q, wc);
                }
                int tot;
                const int pre = block_exclusive_scan<NT>(sel_t, ms->warp, tot);
                int slot = ms->base + pre;
                for (int u = threadIdx.x; u < n_c; u += NT)
                    if (ckey[u] <= kth) {
                        if (slot < a.capg) dst[slot] = ((unsigned long long)ckey[u] << 32) | jo | (uint32_t)cpos[u];
                        ++slot;
                    }
                return;
            }
        }
    }
    // ties at the cutoff beyond what is selected (or too many rows in the
    // running): the full selection in position order
    block_radix_select<NT>(keys, scan, wc, ms->hist, ms->b, kth, n_less);
    if (threadIdx.x == 0) {
        a.cut_g[(size_t)q * a.p1 + j] = key2f(kth);
        ms->base = atomicAdd(a.cnt_g + q, wc);
    }
    // the wc selected rows in position order: keys below kth, then the first
    // need_eq equal to it (the stable order of gpu_global.cu:321-390)
    const int need_eq = wc - n_less;
    int eq_base = 0, out = 0;
    for (int r0 = 0; r0 < scan; r0 += NT) {
        const int i = r0 + threadIdx.x;
        const bool in = i < scan;
        const uint32_t key = in ? keys[i] : 0xffffffffu;
        const int is_eq = (in && key == kth) ? 1 : 0;
        int eq_tot, s_tot;
        const int eq_pre = block_exclusive_scan<NT>(is_eq, ms->warp, eq_tot);
        const bool sel = in && (key < kth || (is_eq && eq_base + eq_pre < need_eq));
        const int s_pre = block_exclusive_scan<NT>(sel ? 1 : 0, ms->warp, s_tot);
        if (sel) {
            const int slot = ms->base + out + s_pre;
            if (slot < a.capg) dst[slot] = ((unsigned long long)key << 32) | jo | (uint32_t)i;
        }
        eq_base += eq_tot;
        out += s_tot;
    }
}

template <int M, int SD, int NT>
__device__ void split_p2_pair(const ScanArgs& a, int q, int j, uint32_t c, int start, int len, unsigned char* smem) {
    float* lut = reinterpret_cast<float*>(smem);
    float* res = lut + M * 256;
    uint32_t* keys = reinterpret_cast<uint32_t*>(res + (a.dim + 3) / 4 * 4);
    SplitMisc* ms = reinterpret_cast<SplitMisc*>(reinterpret_cast<unsigned char*>(keys) + split_keys_bytes(a.lmax));
    if (len <= 0) return;
    const int tid = threadIdx.x;
    if (tid == 0) {
        // threshold = min positive phase-1 cutoff * coeff (gpu_global.cu:394-426)
        float mn = FLT_MAX;
        for (int u = 0; u < a.p1; ++u) {
            const float cu = a.cut_g[(size_t)q * a.p1 + u];
            if (cu > 0.0f && cu < mn) mn = cu;
        }
        ms->thr = (mn < FLT_MAX) ? mn * a.coeff : FLT_MAX;
    }
    const float* qv = a.queries + (size_t)q * a.dim;
    if constexpr (M % 16 == 0)
        split_lut<M, SD, NT, 16>(a, qv, c, res, lut);  // the first 16 subspaces
    else
        split_lut<M, SD, NT>(a, qv, c, res, lut);
    const float thr = ms->thr;
    if constexpr (M % 16 == 0)
        keys_bounded_prefix<M, SD, NT>(a, start, len, lut, res, thr, keys);
    else
        split_keys<M, NT>(a, start, len, lut, keys);
    unsigned long long* dst = a.cand_g + (size_t)q * a.capg;
    const unsigned long long jo = (unsigned long long)((uint32_t)j << 20);
    auto passes = [&](int i) { return keys[i] != 0xffffffffu && key2f(keys[i]) <= thr; };
    if (!a.ref_compat) {
        int n_t = 0;
        for (int i = tid; i < len; i += NT) n_t += passes(i) ? 1 : 0;
        int tot;
        const int pre = block_exclusive_scan<NT>(n_t, ms->warp, tot);
        if (tot == 0) return;
        if (tid == 0) ms->base = atomicAdd(a.cnt_g + q, tot);
        __syncthreads();
        int slot = ms->base + pre;
        for (int i = tid; i < len; i += NT)
            if (passes(i)) {
                if (slot < a.capg) dst[slot] = ((unsigned long long)keys[i] << 32) | jo | (uint32_t)i;
                ++slot;
            }
        return;
    }
    // ref_compat: the reference's 128 threads (thread t: rows t, t + 128, ...)
    // keep the first 128 passing vectors in list order in a shared buffer, and
    // past 128 each thread re-emits its own first (count - 128) passing ones
    // (gpu_global.cu:466-526).  This instance has 128 threads, so thread t is
    // the reference's thread t.
    if constexpr (NT != REF_BLOCK) return;  // launched with NT == 128 under ref_compat
    else {
        int n_t = 0;
        for (int i = tid; i < len; i += SPLIT_NT) n_t += passes(i) ? 1 : 0;
        int s_count;
        (void)block_exclusive_scan<SPLIT_NT>(n_t, ms->warp, s_count);
        if (s_count == 0) return;
        const int quota = s_count > REF_BLOCK ? s_count - REF_BLOCK : 0;
        const int re_t = n_t < quota ? n_t : quota;
        // regular emissions of this thread: rows whose list-order rank is < 128
        int reg_t = 0;
        {
            int carry = 0;
            for (int r0 = 0; r0 < len && carry < REF_BLOCK; r0 += SPLIT_NT) {
                const int i = r0 + tid;
                const int pf = (i < len && passes(i)) ? 1 : 0;
                int tot;
                const int pre = block_exclusive_scan<SPLIT_NT>(pf, ms->warp, tot);
                if (pf && carry + pre < REF_BLOCK) ++reg_t;
                carry += tot;
            }
        }
        int tot;
        const int pre = block_exclusive_scan<SPLIT_NT>(reg_t + re_t, ms->warp, tot);
        if (tid == 0) ms->base = atomicAdd(a.cnt_g + q, tot);
        __syncthreads();
        int slot = ms->base + pre;
        {
            int carry = 0;
            for (int r0 = 0; r0 < len && carry < REF_BLOCK; r0 += SPLIT_NT) {
                const int i = r0 + tid;
                const int pf = (i < len && passes(i)) ? 1 : 0;
                int tot2;
                const int pre2 = block_exclusive_scan<SPLIT_NT>(pf, ms->warp, tot2);
                if (pf && carry + pre2 < REF_BLOCK) {
                    if (slot < a.capg) dst[slot] = ((unsigned long long)keys[i] << 32) | jo | (uint32_t)i;
                    ++slot;
                }
                carry += tot2;
            }
        }
        int left = re_t;
        for (int i = tid; i < len && left > 0; i += SPLIT_NT)
            if (passes(i)) {
                if (slot < a.capg) dst[slot] = ((unsigned long long)keys[i] << 32) | jo | (1u << 19) | (uint32_t)i;
                ++slot;
                --left;
            }
    }
}

// The (query, probe) pairs whose list is non-empty after the prune, as
// records grouped by list (a counting sort: count, scan, scatter), so that the
// ~nq * top_m / nlist queries probing one list run back to back and its codes
// are read from DRAM about once per batch instead of once per query.  An empty
// phase-1 probe gets its cutoff 0 here.  A shard of a list-sharded index owns
// only some of each query's probes: the phase kernels run on its pairs alone.
// The order inside a list does not matter: candidates are ranked by (distance,
// probe, position) whatever the order they arrive in.
__global__ void __launch_bounds__(256) split_pairs_count_kernel(const ScanArgs a, int nq) {
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (long long)nq * a.top_m) return;
    const int q = (int)(t / a.top_m), j = (int)(t % a.top_m);
    uint32_t c;
    int start, len;
    split_probe(a, q, j, c, start, len);
    if (len <= 0) {
        if (j < a.p1) a.cut_g[(size_t)q * a.p1 + j] = 0.0f;
        return;
    }
    atomicAdd(a.hist + (j < a.p1 ? 0 : a.nlist + 1) + c, 1);
}

// Exclusive scan of one phase's per-list counts (CTA 0: phase 1, CTA 1:
// phase 2) in place; the phase's pair count goes to work[phase].
__global__ void __launch_bounds__(1024) split_pairs_scan_kernel(const ScanArgs a) {
    __shared__ int warp[32];
    int* h = a.hist + (size_t)blockIdx.x * (a.nlist + 1);
    const int n = a.nlist, per = (n + 1023) / 1024;
    const int b = min(n, (int)threadIdx.x * per), e = min(n, b + per);
    int sum = 0;
    for (int i = b; i < e; ++i) sum += h[i];
    int tot;
    int pre = block_exclusive_scan<1024>(sum, warp, tot);
    for (int i = b; i < e; ++i) {
        const int v = h[i];
        h[i] = pre;
        pre += v;
    }
    if (threadIdx.x == 0) a.work[blockIdx.x] = tot;
}

__global__ void __launch_bounds__(256) split_pairs_scatter_kernel(const ScanArgs a, int nq) {
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (long long)nq * a.top_m) return;
    const int q = (int)(t / a.top_m), j = (int)(t % a.top_m);
    uint32_t c;
    int start, len;
    split_probe(a, q, j, c, start, len);
    if (len <= 0) return;
    const bool p2 = j >= a.p1;
    const int pos = atomicAdd(a.hist + (p2 ? a.nlist + 1 : 0) + c, 1);
    (p2 ? a.pairs2 : a.pairs1)[pos] = make_int4(q * a.top_m + j, (int)c, start, len);
}

// Persistent CTAs taking the pairs of one phase from a work counter.  Thread
// 0 keeps the next pair's index, claimed one pair ahead, and loads its record
// while the current pair runs, so neither the atomic nor the load waits.
template <int M, int SD, int NT, bool P2>
__global__ void __launch_bounds__(NT, 1024 / NT) split_phase_kernel(const ScanArgs a) {
    extern __shared__ __align__(16) unsigned char smem[];
    SplitMisc* ms = reinterpret_cast<SplitMisc*>(smem + (size_t)M * 256 * 4 + (size_t)(a.dim + 3) / 4 * 16 +
                                                 split_keys_bytes(a.lmax));
    int* ctr = a.work + (P2 ? 3 : 2);
    const int4* recs = P2 ? a.pairs2 : a.pairs1;
    const int count = a.work[P2 ? 1 : 0];
    const int4 none = make_int4(-1, 0, 0, 0);
    int nidx = 0;
    if (threadIdx.x == 0) {
        const int i0 = atomicAdd(ctr, 1);
        nidx = atomicAdd(ctr, 1);
        ms->rec = i0 < count ? recs[i0] : none;
    }
    __syncthreads();
    for (;;) {
        const int4 r = ms->rec;
        if (r.x < 0) break;
        int4 nrec = none;
        int nnidx = 0;
        if (threadIdx.x == 0) {
            if (nidx < count) nrec = recs[nidx];
            nnidx = atomicAdd(ctr, 1);
        }
        const int q = r.x / a.top_m, j = r.x - q * a.top_m;
        if constexpr (P2)
            split_p2_pair<M, SD, NT>(a, q, j, (uint32_t)r.y, r.z, r.w, smem);
        else
            split_p1_pair<M, SD, NT>(a, q, j, (uint32_t)r.y, r.z, r.w, smem);
        __syncthreads();  // every thread has read this pair's record and shared state
        if (threadIdx.x == 0) {
            ms->rec = nrec;
            nidx = nnidx;
        }
        __syncthreads();
    }
}

// ---- group kernel: short lists, the queries probing one list together ------------
//
// Short lists without phase 2 (every probe within p1_lists) and many probes
// per query (C2 at nprobe 8-12; group_chosen has the measured crossover).
// The phase-1 pair records, grouped by list, are cut into groups of up to
// GRP_G consecutive records of one list; a team of GRP_NT threads takes a
// group, computes the group's residuals, runs the skewed on-the-fly ADC over
// the list once for all of its queries (each codebook read serves every
// query of the group) and then has one warp per query select and emit that
// query's limit_k smallest by (distance, position) into the query's
// candidate region -- split_select_kernel ranks them.  The codebook is
// resident in shared memory for the launch, as in ivfpq_team_kernel.

constexpr int GRP_G = 3;      // queries per group, one selecting warp each (4 spilled registers on C2)
constexpr int GRP_MIN_TOP_M = 8;  // the group kernel runs by default from this many probes per query
constexpr int GRP_NT = 128;   // threads per team
constexpr int GRP_TEAMS = 7;  // teams per CTA at most (896 threads: 72 registers each)

struct GroupLayout {
    int res, lkey, hist, misc, total, dpad, lpad;
};

__host__ __device__ inline GroupLayout group_layout(int dim, int lmax) {
    GroupLayout L;
    L.dpad = (dim + 3) / 4 * 4;
    L.lpad = ((lmax > 0 ? lmax : 1) + 3) / 4 * 4;
    int o = 0;
    L.res = take16(o, GRP_G * L.dpad * 4);
    L.lkey = take16(o, GRP_G * L.lpad * 4);
    L.hist = take16(o, (GRP_NT / 32) * 256 * 4);
    L.misc = take16(o, 16);
    L.total = o;
    return L;
}

// Groups of the phase-1 records (grouped by list; after the scatter hist[c]
// is the end of list c's records): a record starts a group when its index
// within its list is a multiple of GRP_G.  work[4] counts the groups.
__global__ void __launch_bounds__(256) group_cut_kernel(const ScanArgs a) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= a.work[0]) return;
    const int c = a.pairs1[i].y;
    const int s = c > 0 ? a.hist[c - 1] : 0, e = a.hist[c];
    if ((i - s) % GRP_G) return;
    const int gi = atomicAdd(a.work + 4, 1);
    a.groups[gi] = make_int2(i, min(GRP_G, e - i));
}

template <int M, int SD, int G>
__device__ __forceinline__ void group_adc(const ScanArgs& a, int start, int scan, int tt, const float* cb,
                                          const float* res, int dpad, uint32_t* lkey, int lpad) {
    adc_skew_stream_multi<M, SD, GRP_NT, G>(a.codes + (size_t)start * M, scan, tt, cb, res, dpad, lkey, lpad);
}

template <int M, int SD>
__global__ void __launch_bounds__(GRP_TEAMS * GRP_NT, 1) ivfpq_group_kernel(const ScanArgs a, int team_bytes) {
    extern __shared__ __align__(16) unsigned char smem[];
    static_assert(AdcSkew<M, SD>::value, "skewed on-the-fly ADC shape");
    constexpr int CBF = M * 256 * SD;
    float* cb = reinterpret_cast<float*>(smem);
    // [subspace][code][SD] -> [code][subspace][SD], as ivfpq_team_kernel
    for (int e = threadIdx.x; e < M * 256; e += blockDim.x) {
        const int k = e / M, m = e - k * M;
        float v[SD];
        load_sub<SD, true>(a.codebook + ((size_t)m * 256 + k) * SD, v);
#pragma unroll
        for (int t = 0; t < SD; ++t) cb[(size_t)e * SD + t] = v[t];
    }
    __syncthreads();
    const int team = threadIdx.x / GRP_NT, tt = threadIdx.x % GRP_NT;
    const int bar = 1 + team;
    unsigned char* ts = smem + (size_t)(CBF * 4 + 15) / 16 * 16 + (size_t)team * team_bytes;
    const GroupLayout L = group_layout(a.dim, a.lmax);
    float* res = reinterpret_cast<float*>(ts + L.res);
    uint32_t* lkey = reinterpret_cast<uint32_t*>(ts + L.lkey);
    uint32_t* hist = reinterpret_cast<uint32_t*>(ts + L.hist);
    int* next = reinterpret_cast<int*>(ts + L.misc);
    const int ngroups = a.work[4];
    const int w = tt >> 5, lane = tt & 31;
    for (;;) {
        if (tt == 0) *next = atomicAdd(a.work + 5, 1);
        team_sync<GRP_NT>(bar);
        const int gi = *next;
        if (gi >= ngroups) break;
        const int2 g2 = a.groups[gi];
        const int first = g2.x, gcnt = g2.y;
        const int4 r0 = a.pairs1[first];
        const uint32_t c = (uint32_t)r0.y;
        const int start = r0.z, len = r0.w;
        const int wc = len < a.limit_k ? len : a.limit_k;
        const int scan = (a.ref_compat && len > REF_P1_CLAMP) ? REF_P1_CLAMP : len;
        const float* cv = a.centroids + (size_t)c * a.dim;
        for (int e = tt; e < gcnt * a.dim; e += GRP_NT) {
            const int g = e / a.dim, t = e - g * a.dim;
            const int q = a.pairs1[first + g].x / a.top_m;
            res[g * L.dpad + t] = a.queries[(size_t)q * a.dim + t] - cv[t];
        }
        team_sync<GRP_NT>(bar);
        switch (gcnt) {
            case 1: group_adc<M, SD, 1>(a, start, scan, tt, cb, res, L.dpad, lkey, L.lpad); break;
            case 2: group_adc<M, SD, 2>(a, start, scan, tt, cb, res, L.dpad, lkey, L.lpad); break;
            default: group_adc<M, SD, 3>(a, start, scan, tt, cb, res, L.dpad, lkey, L.lpad); break;
        }
        team_sync<GRP_NT>(bar);
        if (w < gcnt) {
            // warp w: query w of the group selects its wc smallest by (key,
            // position) and appends them to its region (gpu_global.cu:321-390)
            const int qj = a.pairs1[first + w].x;
            const int q = qj / a.top_m, j = qj - q * a.top_m;
            const uint32_t* keys = lkey + w * L.lpad;
            uint32_t kth;
            int n_less;
            warp_select_keys(keys, scan, wc, hist + w * 256, kth, n_less);
            int base = 0;
            if (lane == 0) {
                base = atomicAdd(a.cnt_g + q, wc);
                a.cut_g[(size_t)q * a.p1 + j] = key2f(kth);
            }
            base = __shfl_sync(0xffffffffu, base, 0);
            unsigned long long* dst = a.cand_g + (size_t)q * a.capg;
            const unsigned long long jo = (unsigned long long)((uint32_t)j << 20);
            const unsigned lt = lanemask_lt();
            const int need_eq = wc - n_less;
            int eq_base = 0, out = 0;
            for (int i0 = 0; i0 < scan; i0 += 32) {
                const int i = i0 + lane;
                const bool in = i < scan;
                const uint32_t key = in ? keys[i] : 0xffffffffu;
                const bool is_eq = in && key == kth;
                const unsigned eqb = __ballot_sync(0xffffffffu, is_eq);
                const bool sel = in && (key < kth || (is_eq && eq_base + __popc(eqb & lt) < need_eq));
                const unsigned sb = __ballot_sync(0xffffffffu, sel);
                if (sel) {
                    const int slot = base + out + __popc(sb & lt);
                    if (slot < a.capg) dst[slot] = ((unsigned long long)key << 32) | jo | (uint32_t)i;
                }
                eq_base += __popc(eqb);
                out += __popc(sb);
            }
        }
        team_sync<GRP_NT>(bar);  // the next group reuses every buffer
    }
}

// k-th smallest high word (1-based) of n 64-bit keys in global memory; the
// block_radix_select scheme (four 8-bit MSD passes).
__device__ void sel_radix_select_hi(const unsigned long long* keys, int n, int k, uint32_t* s_hist, uint32_t* s_b,
                                    uint32_t& kth, int& n_less) {
    uint32_t prefix = 0, mask = 0, kk = (uint32_t)k, less = 0;
#pragma unroll 1
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = threadIdx.x; i < 256; i += SEL_NT) s_hist[i] = 0;
        __syncthreads();
        for (int i = threadIdx.x; i < n; i += SEL_NT) {
            const uint32_t key = (uint32_t)(keys[i] >> 32);
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
                const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
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

struct SelMisc {
    uint32_t hist[256];
    uint32_t b[2];
    int n_col;
};

__global__ void __launch_bounds__(SEL_NT) split_select_kernel(const ScanArgs a, int nq, int sort_cap) {
    extern __shared__ __align__(16) unsigned char smem[];
    unsigned long long* sortb = reinterpret_cast<unsigned long long*>(smem);
    SelMisc* ms = reinterpret_cast<SelMisc*>(smem + (size_t)sort_cap * 8);
    const int q = blockIdx.x;
    if (q >= nq) return;
    const int tid = threadIdx.x;
    const int count = a.cnt_g[q];
    const int rm = a.rerank_m;
    const int ak = count < rm ? count : rm;
    const int nsel = a.ref_compat ? (ak < REF_BLOCK ? ak : REF_BLOCK) : ak;
    const unsigned long long* cand = a.cand_g + (size_t)q * a.capg;
    bool ok = count <= a.capg;
    int n_sort = 0;
    if (ok && nsel > 0) {
        if (count <= sort_cap) {
            for (int i = tid; i < count; i += SEL_NT) sortb[i] = cand[i];
            n_sort = count;
        } else {
            uint32_t kth;
            int n_less;
            sel_radix_select_hi(cand, count, nsel, ms->hist, ms->b, kth, n_less);
            if (tid == 0) ms->n_col = 0;
            __syncthreads();
            for (int i = tid; i < count; i += SEL_NT) {
                const unsigned long long e = cand[i];
                if ((uint32_t)(e >> 32) <= kth) {
                    const int s = atomicAdd(&ms->n_col, 1);
                    if (s < sort_cap) sortb[s] = e;
                }
            }
            __syncthreads();
            n_sort = ms->n_col;
            ok = n_sort <= sort_cap;  // more ties at the boundary than the buffer holds
        }
    }
    if (tid == 0) a.flags[q] = ok ? 0 : 1;
    if (!ok) return;  // the per-query kernel writes this query
    const int npow = next_pow2(n_sort > 0 ? n_sort : 1);
    for (int i = n_sort + tid; i < npow; i += SEL_NT) sortb[i] = ~0ull;
    __syncthreads();
    if (n_sort > 1) block_bitonic_sort<SEL_NT>(sortb, npow);
    const int pend = a.write_pad ? rm : ak;
    const int P = a.top_m;
    for (int p = tid; p < pend; p += SEL_NT) {
        const size_t o = (size_t)q * rm + p;
        if (a.ref_compat && p >= REF_BLOCK) {
            a.top_ids[o] = 0;  // never written by the reference's 128-thread gather (zeroed memory)
            a.top_dists[o] = 0.0f;
        } else if (p < ak) {
            const unsigned long long e = sortb[p];
            const uint32_t ord = (uint32_t)(e & 0xffffffffu);
            const uint32_t c = a.probe_ids[(size_t)q * P + (ord >> 20)];
            a.top_ids[o] = __ldg(a.vids + a.offsets[c] + (ord & 0x7ffffu));
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

using SplitKernel = void (*)(const ScanArgs);

// P2: 0 phase 1, 1 phase 2 in ref_compat (128 threads), 2 phase 2 otherwise
template <int P2>
static SplitKernel pick_split_kernel(int M, int SD) {
#define FG_SPLIT_CASE(m, sd)                                                                        \
    if (M == m && SD == sd)                                                                       \
        return P2 == 2 ? split_phase_kernel<m, sd, SPLIT_P2_NT, true>                             \
                       : (P2 == 1 ? split_phase_kernel<m, sd, SPLIT_NT, true>                     \
                                  : split_phase_kernel<m, sd, SPLIT_P1_NT, false>);
    FG_SPLIT_CASE(4, 4)  // small test indexes
    FG_SPLIT_CASE(16, 4)
    FG_SPLIT_CASE(16, 8)
    FG_SPLIT_CASE(32, 2)
    FG_SPLIT_CASE(32, 3)
    FG_SPLIT_CASE(32, 4)
    FG_SPLIT_CASE(48, 2)
    FG_SPLIT_CASE(64, 2)
    FG_SPLIT_CASE(96, 8)
    FG_SPLIT_CASE(128, 1)
#undef FG_SPLIT_CASE
    return nullptr;
}

template <bool LUT, int NT>
static TeamKernel pick_team_kernel(int M, int SD) {
#define FG_TEAM_CASE(m, sd) \
    if (M == m && SD == sd) return ivfpq_team_kernel<m, sd, LUT, NT>;
    FG_TEAM_CASE(4, 4)  // small test indexes
    FG_TEAM_CASE(16, 4)
    FG_TEAM_CASE(16, 8)
    FG_TEAM_CASE(32, 2)
    FG_TEAM_CASE(32, 3)
    FG_TEAM_CASE(32, 4)
    FG_TEAM_CASE(48, 2)
    FG_TEAM_CASE(64, 2)
    FG_TEAM_CASE(96, 8)
    FG_TEAM_CASE(128, 1)
#undef FG_TEAM_CASE
    return nullptr;
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

// ---- the split path's choice and workspace ---------------------------------------

// Typical length of a probed list: the mean over all lists, or half the
// longest (rebalancing caps lists at twice the mean), whichever is larger.  A
// shard of a list-sharded index keeps every list slot but owns only some
// lists, so its mean over all slots understates the lists it scans.
static double typical_list_len(const fg_ivfpq_view* ix) {
    return std::max((double)ix->total / std::max(ix->nlist, 1), 0.5 * ix->max_list_len);
}

static int split_rsel(const fg_search_params* p) {
    return p->ref_compat ? (p->rerank_m < REF_BLOCK ? p->rerank_m : REF_BLOCK) : p->rerank_m;
}

static int split_capg(const fg_search_params* p) {
    const int r = split_rsel(p);
    return (std::max(4096, 2 * r) + 31) / 32 * 32;
}

// Whether the split path runs for this index, parameters and batch: long
// lists (typical length above the team kernel's limit) and a supported shape,
// unless FG_SCAN_KERNEL names another kernel (FG_SCAN_KERNEL=split forces it).
static bool split_chosen(const fg_ivfpq_view* ix, const fg_search_params* p, int nq) {
    if (!ix || !p || nq <= 0 || ix->pq_m <= 0 || ix->dim % ix->pq_m) return false;
    const int M = ix->pq_m, SD = ix->dim / ix->pq_m;
    if (!pick_split_kernel<0>(M, SD) || p->top_m > 4096 || ix->max_list_len >= (1 << 19) ||
        (long long)nq * p->top_m >= (1LL << 31))
        return false;
    const char* force = getenv("FG_SCAN_KERNEL");
    const std::string mode = force ? force : "";
    if (mode == "split") return true;
    if (!mode.empty()) return false;
    return typical_list_len(ix) > TEAM_OTF_MAX_LEN;
}

struct SplitWs {
    float* cut;
    int* work;  // pair counts and work counters, then the per-list pair counts, then the per-query candidate counts
    int* hist;
    int32_t* cnt;
    int32_t* flags;
    int4* pairs;
    int2* groups;
    unsigned long long* cand;
};

static size_t split_carve(void* ws, int nq, int nlist, const fg_search_params* p, int capg, SplitWs* out) {
    const int p1 = std::max(1, std::min(p->top_m, p->p1_lists));
    size_t o = 0;
    auto take = [&](size_t bytes) {
        const size_t r = o;
        o += (bytes + 255) / 256 * 256;
        return r;
    };
    const size_t oc = take((size_t)nq * p1 * 4), ow = take(32), oh = take((size_t)2 * (nlist + 1) * 4),
                 on = take((size_t)nq * 4),
                 of = take((size_t)nq * 4), op = take((size_t)nq * std::max(p->top_m, p1) * 16),
                 og = take((size_t)nq * p1 * 8), oa = take((size_t)nq * capg * 8);
    if (out) {
        char* b = static_cast<char*>(ws);
        out->cut = reinterpret_cast<float*>(b + oc);
        out->work = reinterpret_cast<int*>(b + ow);
        out->hist = reinterpret_cast<int*>(b + oh);
        out->cnt = reinterpret_cast<int32_t*>(b + on);
        out->flags = reinterpret_cast<int32_t*>(b + of);
        out->pairs = reinterpret_cast<int4*>(b + op);
        out->groups = reinterpret_cast<int2*>(b + og);
        out->cand = reinterpret_cast<unsigned long long*>(b + oa);
    }
    return o;
}

// Persistent grid of a split phase kernel: its resident CTAs on every SM, at
// most one per pair.
static int split_grid(SplitKernel k, int nt, int bytes, long long pairs, int* grid) {
    int occ = 0;
    FG_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, reinterpret_cast<const void*>(k), nt, bytes));
    const long long nsm = std::max(1, device_attr(cudaDevAttrMultiProcessorCount));
    *grid = (int)std::max(1LL, std::min(pairs, nsm * std::max(occ, 1)));
    return FG_OK;
}

// Launches the split path: zero the counters, list the non-empty (query,
// probe) pairs, phase 1 and phase 2 over them (persistent CTAs), per-query
// selection, then the per-query kernel for the queries the selection flagged
// (its CTAs for the others return at once).
static int batch_logic_split(ScanArgs a, const fg_ivfpq_view* ix, int nq, void* ws, cudaStream_t stream,
                             int smem_max) {
    const int M = ix->pq_m, SD = ix->dim / ix->pq_m;
    fg_search_params pp{};
    pp.top_m = a.top_m;
    pp.p1_lists = a.p1;
    pp.rerank_m = a.rerank_m;
    pp.ref_compat = a.ref_compat;
    SplitWs w;
    split_carve(ws, nq, ix->nlist, &pp, split_capg(&pp), &w);
    a.cut_g = w.cut;
    a.cnt_g = w.cnt;
    a.flags = w.flags;
    a.cand_g = w.cand;
    a.capg = split_capg(&pp);
    a.work = w.work;
    a.hist = w.hist;
    a.pairs1 = w.pairs;
    a.pairs2 = w.pairs + (size_t)nq * a.p1;
    // the fallback kernel's shared memory must fit, as on the per-query path
    ScanKernel k = pick_scan_kernel(M, SD);
    a.cap = a.rsel + SCAN_NT;
    const ScanLayout L = scan_layout(M, a.dim, a.top_m, a.p1, a.lmax, a.cap, a.sort_n);
    if (!k || L.total > smem_max)
        return fail(FG_ERR_UNSUPPORTED, "scan needs %d bytes of shared memory (max %d): rerank_m=%d "
                    "max_list_len=%d", L.total, smem_max, a.rerank_m, a.lmax);
    // the counters, the per-list counts and the per-query counts are adjacent: one memset
    FG_CUDA_TRY(cudaMemsetAsync(w.work, 0, reinterpret_cast<char*>(w.cnt + nq) - reinterpret_cast<char*>(w.work),
                                stream));
    {
        const long long n = (long long)nq * a.top_m;
        const unsigned blocks = (unsigned)((n + 255) / 256);
        split_pairs_count_kernel<<<blocks, 256, 0, stream>>>(a, nq);
        int rc = check_launch("split_pairs_count_kernel");
        if (rc) return rc;
        split_pairs_scan_kernel<<<2, 1024, 0, stream>>>(a);
        if ((rc = check_launch("split_pairs_scan_kernel"))) return rc;
        split_pairs_scatter_kernel<<<blocks, 256, 0, stream>>>(a, nq);
        if ((rc = check_launch("split_pairs_scatter_kernel"))) return rc;
    }
    const int dpad = (a.dim + 3) / 4 * 4;
    if (a.p1 > 0) {
        SplitKernel k1 = pick_split_kernel<0>(M, SD);
        const int bytes = M * 256 * 4 + dpad * 4 + split_keys_bytes(a.lmax) + (int)sizeof(SplitMisc);
        if (bytes > smem_max) return fail(FG_ERR_UNSUPPORTED, "split phase 1 needs %d bytes of shared memory", bytes);
        FG_CUDA_TRY(ensure_smem(reinterpret_cast<const void*>(k1), bytes));
        int grid = 1;
        int rc = split_grid(k1, SPLIT_P1_NT, bytes, (long long)nq * a.p1, &grid);
        if (rc) return rc;
        k1<<<grid, SPLIT_P1_NT, bytes, stream>>>(a);
        rc = check_launch("split_phase_kernel (phase 1)");
        if (rc) return rc;
    }
    if (a.top_m > a.p1) {
        ScanArgs a2 = a;
        a2.lmax = std::max(ix->max_list_len, 1);  // phase 2 has no 1024-row clamp
        SplitKernel k2 = a.ref_compat ? pick_split_kernel<1>(M, SD) : pick_split_kernel<2>(M, SD);
        const int nt2 = a.ref_compat ? SPLIT_NT : SPLIT_P2_NT;
        const int bytes = M * 256 * 4 + dpad * 4 + split_keys_bytes(a2.lmax) + (int)sizeof(SplitMisc);
        if (bytes > smem_max) return fail(FG_ERR_UNSUPPORTED, "split phase 2 needs %d bytes of shared memory", bytes);
        FG_CUDA_TRY(ensure_smem(reinterpret_cast<const void*>(k2), bytes));
        int grid = 1;
        int rc = split_grid(k2, nt2, bytes, (long long)nq * (a.top_m - a.p1), &grid);
        if (rc) return rc;
        k2<<<grid, nt2, bytes, stream>>>(a2);
        rc = check_launch("split_phase_kernel (phase 2)");
        if (rc) return rc;
    }
    const int sort_cap = next_pow2(std::max(256, 2 * a.rsel));
    const int sbytes = sort_cap * 8 + (int)sizeof(SelMisc);
    if (sbytes > smem_max) return fail(FG_ERR_UNSUPPORTED, "split select needs %d bytes of shared memory", sbytes);
    FG_CUDA_TRY(ensure_smem(reinterpret_cast<const void*>(&split_select_kernel), sbytes));
    split_select_kernel<<<nq, SEL_NT, sbytes, stream>>>(a, nq, sort_cap);
    int rc = check_launch("split_select_kernel");
    if (rc) return rc;
    a.only = w.flags;
    FG_CUDA_TRY(ensure_smem(reinterpret_cast<const void*>(k), L.total));
    k<<<nq, SCAN_NT, L.total, stream>>>(a);
    return check_launch("ivfpq_batch_kernel");
}

using GroupKernel = void (*)(const ScanArgs, int);

static GroupKernel pick_group_kernel(int M, int SD) {
#define FG_GROUP_CASE(m, sd) \
    if (M == m && SD == sd) return ivfpq_group_kernel<m, sd>;
    FG_GROUP_CASE(16, 4)
    FG_GROUP_CASE(16, 8)
    FG_GROUP_CASE(32, 2)
    FG_GROUP_CASE(32, 4)
    FG_GROUP_CASE(48, 2)
    FG_GROUP_CASE(64, 2)
#undef FG_GROUP_CASE
    return nullptr;
}

// Whether the group kernel runs: short lists (typical length up to the team
// kernel's limit), no phase 2 (top_m <= p1_lists), a skewed-ADC shape and at
// least GRP_MIN_TOP_M probes per query, unless FG_SCAN_KERNEL names another
// kernel (FG_SCAN_KERNEL=group forces it at any top_m).  Measured on C2 (4,104
// lists of ~244, 10,000 queries): 2.82 -> 2.44 ms per step at nprobe 8, a tie
// at 4, and slower at 1 and 2 (0.39 -> 0.53, 0.63 -> 0.76 ms), where a list
// has only 2.4 or 4.9 probing queries and the separate selection kernel
// (0.12 ms) outweighs the shared codebook reads.
static bool group_chosen(const fg_ivfpq_view* ix, const fg_search_params* p, int nq) {
    if (!ix || !p || nq <= 0 || ix->pq_m <= 0 || ix->dim % ix->pq_m) return false;
    const int M = ix->pq_m, SD = ix->dim / ix->pq_m;
    if (!pick_group_kernel(M, SD) || p->top_m > p->p1_lists || ix->max_list_len >= (1 << 19) ||
        (long long)nq * p->top_m >= (1LL << 31))
        return false;
    const char* force = getenv("FG_SCAN_KERNEL");
    const std::string mode = force ? force : "";
    if (mode == "group") return true;
    if (!mode.empty()) return false;
    return p->top_m >= GRP_MIN_TOP_M && typical_list_len(ix) <= TEAM_OTF_MAX_LEN;
}

// Candidate region of a query on the group path: every probe is a phase-1
// probe, so a query emits at most top_m * min(limit_k, longest list).
static int group_capg(const fg_ivfpq_view* ix, const fg_search_params* p) {
    const long long m = (long long)p->top_m * std::min(p->limit_k, std::max(ix->max_list_len, 1));
    return (int)((std::max(m, 32LL) + 31) / 32 * 32);
}

constexpr int GROUP_NOT_LAUNCHED = -1;

// Launches the group path: zero the counters, list the phase-1 pairs grouped
// by list, cut them into groups, the group kernel, per-query selection, then
// the per-query kernel for any query the selection flagged.  Returns
// GROUP_NOT_LAUNCHED (nothing queued) when the codebook and one team do not
// fit in shared memory.
static int batch_logic_group(ScanArgs a, const fg_ivfpq_view* ix, int nq, void* ws, cudaStream_t stream,
                             int smem_max) {
    const int M = ix->pq_m, SD = ix->dim / ix->pq_m;
    GroupKernel gk = pick_group_kernel(M, SD);
    ScanKernel k = pick_scan_kernel(M, SD);
    const int cb_bytes = (M * 256 * SD * 4 + 15) / 16 * 16;
    const GroupLayout GL = group_layout(a.dim, a.lmax);
    const int nteams = std::min(GRP_TEAMS, (smem_max - cb_bytes) / GL.total);
    a.cap = a.rsel + SCAN_NT;
    const ScanLayout L = scan_layout(M, a.dim, a.top_m, a.p1, a.lmax, a.cap, a.sort_n);
    if (!gk || !k || nteams < 1 || L.total > smem_max) return GROUP_NOT_LAUNCHED;
    fg_search_params pp{};
    pp.top_m = a.top_m;
    pp.p1_lists = a.p1;
    pp.rerank_m = a.rerank_m;
    pp.ref_compat = a.ref_compat;
    pp.limit_k = a.limit_k;
    const int capg = group_capg(ix, &pp);
    SplitWs w;
    split_carve(ws, nq, ix->nlist, &pp, capg, &w);
    a.cut_g = w.cut;
    a.cnt_g = w.cnt;
    a.flags = w.flags;
    a.cand_g = w.cand;
    a.capg = capg;
    a.work = w.work;
    a.hist = w.hist;
    a.pairs1 = w.pairs;
    a.pairs2 = w.pairs + (size_t)nq * a.p1;
    a.groups = w.groups;
    FG_CUDA_TRY(cudaMemsetAsync(w.work, 0, reinterpret_cast<char*>(w.cnt + nq) - reinterpret_cast<char*>(w.work),
                                stream));
    const long long n = (long long)nq * a.top_m;
    const unsigned blocks = (unsigned)((n + 255) / 256);
    split_pairs_count_kernel<<<blocks, 256, 0, stream>>>(a, nq);
    int rc = check_launch("split_pairs_count_kernel");
    if (rc) return rc;
    split_pairs_scan_kernel<<<2, 1024, 0, stream>>>(a);
    if ((rc = check_launch("split_pairs_scan_kernel"))) return rc;
    split_pairs_scatter_kernel<<<blocks, 256, 0, stream>>>(a, nq);
    if ((rc = check_launch("split_pairs_scatter_kernel"))) return rc;
    group_cut_kernel<<<(unsigned)(((long long)nq * a.p1 + 255) / 256), 256, 0, stream>>>(a);
    if ((rc = check_launch("group_cut_kernel"))) return rc;
    const int bytes = cb_bytes + nteams * GL.total;
    FG_CUDA_TRY(ensure_smem(reinterpret_cast<const void*>(gk), bytes));
    const int nsm = std::max(1, device_attr(cudaDevAttrMultiProcessorCount));
    gk<<<nsm, nteams * GRP_NT, bytes, stream>>>(a, GL.total);
    if ((rc = check_launch("ivfpq_group_kernel"))) return rc;
    const int sort_cap = next_pow2(std::max(256, std::min(2 * a.rsel, capg)));
    const int sbytes = sort_cap * 8 + (int)sizeof(SelMisc);
    if (sbytes > smem_max) return fail(FG_ERR_UNSUPPORTED, "split select needs %d bytes of shared memory", sbytes);
    FG_CUDA_TRY(ensure_smem(reinterpret_cast<const void*>(&split_select_kernel), sbytes));
    split_select_kernel<<<nq, SEL_NT, sbytes, stream>>>(a, nq, sort_cap);
    if ((rc = check_launch("split_select_kernel"))) return rc;
    if (capg >= 2 * a.rsel) {  // only then can a query overflow the selection buffer
        a.only = w.flags;
        FG_CUDA_TRY(ensure_smem(reinterpret_cast<const void*>(k), L.total));
        k<<<nq, SCAN_NT, L.total, stream>>>(a);
        return check_launch("ivfpq_batch_kernel");
    }
    return FG_OK;
}

size_t batch_logic_workspace(const fg_ivfpq_view* ix, const fg_search_params* p, int nq) {
    if (split_chosen(ix, p, nq)) return split_carve(nullptr, nq, ix->nlist, p, split_capg(p), nullptr) + 256;
    if (group_chosen(ix, p, nq)) return split_carve(nullptr, nq, ix->nlist, p, group_capg(ix, p), nullptr) + 256;
    return 0;
}

int batch_logic(const fg_ivfpq_view* ix, const float* queries, int nq, const uint32_t* probe_ids,
                const float* probe_dists, const fg_search_params* p, int32_t* top_ids,
                float* top_dists, int32_t* top_counts, int32_t* cand_counts, cudaStream_t stream,
                bool write_pad, int* work_counter, void* ws, size_t ws_bytes) {
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
    a.small = 0;
    a.work_counter = work_counter;
    a.cut_g = nullptr;
    a.cnt_g = nullptr;
    a.cand_g = nullptr;
    a.flags = nullptr;
    a.only = nullptr;
    a.capg = 0;
    a.work = nullptr;
    a.hist = nullptr;
    a.pairs1 = nullptr;
    a.pairs2 = nullptr;
    a.groups = nullptr;

    int smem_max = 0, smem_sm = 0;
    smem_max = device_attr(cudaDevAttrMaxSharedMemoryPerBlockOptin);
    smem_sm = device_attr(cudaDevAttrMaxSharedMemoryPerMultiprocessor);
    if (smem_max <= 0 || smem_sm <= 0) return fail(FG_ERR_CUDA, "cannot read the device's shared-memory limits");

    if (split_chosen(ix, p, nq)) {
        const size_t need = split_carve(nullptr, nq, ix->nlist, p, split_capg(p), nullptr);
        if (ws && ws_bytes >= need) return batch_logic_split(a, ix, nq, ws, stream, smem_max);
        if (getenv("FG_SCAN_KERNEL") && std::string(getenv("FG_SCAN_KERNEL")) == "split")
            return fail(FG_ERR_WORKSPACE, "FG_SCAN_KERNEL=split needs %zu workspace bytes", need);
    }
    if (group_chosen(ix, p, nq)) {
        const size_t need = split_carve(nullptr, nq, ix->nlist, p, group_capg(ix, p), nullptr);
        const bool forced = getenv("FG_SCAN_KERNEL") && std::string(getenv("FG_SCAN_KERNEL")) == "group";
        if (ws && ws_bytes >= need) {
            const int rc = batch_logic_group(a, ix, nq, ws, stream, smem_max);
            if (rc != GROUP_NOT_LAUNCHED) return rc;
            if (forced) return fail(FG_ERR_UNSUPPORTED, "FG_SCAN_KERNEL=group: the group kernel does not fit");
        } else if (forced) {
            return fail(FG_ERR_WORKSPACE, "FG_SCAN_KERNEL=group needs %zu workspace bytes", need);
        }
    }
    // The team kernel when the codebook and at least one team fit in shared
    // memory (two teams for on-the-fly ADC).  FG_SCAN_KERNEL=block|team|team_lut|team_otf
    // and FG_SCAN_TEAM_NT=64|128|256 override the choice (for tests and measurements).
    const char* force = getenv("FG_SCAN_KERNEL");
    const std::string mode = force ? force : "";
    const double avg_len = typical_list_len(ix);
    // measured: on long lists (C3: 680, C5: 1000 vectors per list at nprobe 64)
    // the per-query CTA kernel is faster than any team configuration
    if (mode != "block" && (!mode.empty() || avg_len <= TEAM_OTF_MAX_LEN)) {
        bool lut = mode == "team_lut";
        const bool forced = mode == "team_lut" || mode == "team_otf";
        const int min_teams = forced ? 1 : 2;  // one team leaves an SM mostly idle
        // the most candidates one query can emit: phase-1 lists give at most
        // limit_k each, phase-2 lists at most their length.  Below rsel the
        // buffer is never cut and the final sort never holds more.
        const long long p1n = std::min(a.top_m, a.p1);
        const long long maxcand = std::max(1LL, p1n * std::min(a.limit_k, a.lmax) +
                                                    (long long)(a.top_m - p1n) * std::max(ix->max_list_len, 1));
        const bool small = maxcand < a.rsel;
        const int sort_n = small ? next_pow2((int)maxcand) : a.sort_n;
        const int cb_bytes = (M * 256 * SD * 4 + 15) / 16 * 16;
        const int avail = smem_max - cb_bytes;
        struct Pick {
            TeamKernel k = nullptr;
            int nt = 0, nteams = 0, cap = 0, bytes = 0;
        } best;
        const char* fnt = getenv("FG_SCAN_TEAM_NT");  // 64, 128 or 256: only that team size
        // Small per-query work (few probed vectors) favours many small teams,
        // more work per query teams of 128 (measured on C2: 64 at nprobe 2, 128
        // at nprobe 8); when shared memory caps the team count, larger teams.
        const double est = (double)a.top_m * avg_len;
        const int pref_nt = (est <= 1024.0 && !a.ref_compat) ? 64 : 128;
        const int only_nt = fnt ? atoi(fnt) : 0;
        int pass_nt = only_nt;
        Pick by_nt[3];  // teams of 64, 128, 256
        auto consider = [&](TeamKernel k, int nt, int min_cap, int roomy_cap, int tbytes_min, int tbytes_roomy) {
            // (a forced 64 yields to 128 under ref_compat, which needs whole 128-thread groups)
            const int want_nt = (pass_nt == 64 && a.ref_compat) ? 128 : pass_nt;
            if (!k || avail <= 0 || (want_nt && nt != want_nt)) return;
            const int maxt = std::min(TEAM_THREADS / nt, 15);  // named barriers 1..15
            int nteams = std::min(maxt, avail / tbytes_min);
            if (nteams < min_teams) return;
            int cap = min_cap, tbytes = tbytes_min;
            if (std::min(maxt, avail / tbytes_roomy) == nteams) {
                cap = roomy_cap;
                tbytes = tbytes_roomy;
            }
            by_nt[nt == 64 ? 0 : nt == 128 ? 1 : 2] = Pick{k, nt, nteams, cap, tbytes};
        };
        auto consider_all = [&]() {
            if (!a.ref_compat) {
                const int c0 = small ? (int)maxcand + 64 : a.rsel + 64, c1 = small ? c0 : 2 * a.rsel + 64;
                consider(lut ? pick_team_kernel<true, 64>(M, SD) : pick_team_kernel<false, 64>(M, SD), 64, c0, c1,
                         team_layout<64>(M, a.dim, a.top_m, a.p1, a.lmax, c0, sort_n, lut).total,
                         team_layout<64>(M, a.dim, a.top_m, a.p1, a.lmax, c1, sort_n, lut).total);
            }
            {
                const int c0 = small ? (int)maxcand + 128 : a.rsel + 128, c1 = small ? c0 : 2 * a.rsel + 128;
                consider(lut ? pick_team_kernel<true, 128>(M, SD) : pick_team_kernel<false, 128>(M, SD), 128, c0, c1,
                         team_layout<128>(M, a.dim, a.top_m, a.p1, a.lmax, c0, sort_n, lut).total,
                         team_layout<128>(M, a.dim, a.top_m, a.p1, a.lmax, c1, sort_n, lut).total);
            }
            {
                const int c0 = small ? (int)maxcand + 256 : a.rsel + 256, c1 = small ? c0 : 2 * a.rsel + 256;
                consider(lut ? pick_team_kernel<true, 256>(M, SD) : pick_team_kernel<false, 256>(M, SD), 256, c0, c1,
                         team_layout<256>(M, a.dim, a.top_m, a.p1, a.lmax, c0, sort_n, lut).total,
                         team_layout<256>(M, a.dim, a.top_m, a.p1, a.lmax, c1, sort_n, lut).total);
            }
        };
        consider_all();
        if (!forced && lut && !by_nt[0].k && !by_nt[1].k && !by_nt[2].k) {
            lut = false;  // no two teams with tables fit: on-the-fly terms
            consider_all();
        }
        // the size with the most resident threads, unless the preferred size
        // keeps at least 90 % of them
        for (const Pick& p : by_nt)
            if (p.k && p.nteams * p.nt > best.nteams * best.nt) best = p;
        for (const Pick& p : by_nt)
            if (p.k && p.nt == pref_nt && 10 * p.nteams * p.nt >= 9 * best.nteams * best.nt) best = p;
        if (best.k) {
            a.cap = best.cap;
            a.sort_n = sort_n;
            const char* fws = getenv("FG_SCAN_WARP_SELECT");  // 0: team-wide selection always
            a.small = small ? ((fws && fws[0] == '0') ? 2 : 1) : 0;
            int nsm = 0;
            nsm = std::max(1, device_attr(cudaDevAttrMultiProcessorCount));
            const int grid = std::max(1, std::min(nsm, (nq + best.nteams - 1) / best.nteams));
            const int bytes = cb_bytes + best.nteams * best.bytes;
            FG_CUDA_TRY(ensure_smem(reinterpret_cast<const void*>(best.k), bytes));
            best.k<<<grid, best.nteams * best.nt, bytes, stream>>>(a, nq, best.nteams, best.bytes);
            return check_launch("ivfpq_team_kernel");
        }
        if (mode == "team" || mode == "team_lut" || mode == "team_otf")
            return fail(FG_ERR_UNSUPPORTED, "FG_SCAN_KERNEL=%s: the team kernel does not fit (pq_m=%d sub_dim=%d)",
                        mode.c_str(), M, SD);
    }
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
    FG_CUDA_TRY(ensure_smem(reinterpret_cast<const void*>(k), L.total));
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
