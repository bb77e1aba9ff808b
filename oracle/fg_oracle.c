/*
 * fg_oracle.c -- TEST INFRASTRUCTURE ONLY (see fg_oracle.h).
 *
 * A plain-C restatement of the reference's IVF-PQ arithmetic, used as the
 * checker for the CUDA product.  Compile with -ffp-contract=off: every fused
 * multiply-add below is written out with fmaf() where the reference's CUDA
 * code computes one (explicit fmaf() calls, or nvcc's default contraction of
 * `acc += diff * diff`), and nowhere else.
 *
 * Where the reference is nondeterministic (atomic emission order into the
 * per-query candidate buffer, gpu_global.cu:349,483,495,519) the oracle fixes
 * one legal schedule: candidates are emitted in (probe index j, position in
 * list) order, so ties in the stable sort by distance (gpu_global.cu:853-861)
 * are broken by that emission order.  Phase-2 overflow (gpu_global.cu:508-526)
 * likewise buffers the first 128 passing vectors in list order.
 */
#include "fg_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define FGO_INVALID 0xFFFFFFFFu
#define FGO_REF_BLOCK 128      /* blockDim of the reference's scan/gather/rerank kernels */
#define FGO_REF_P1_CLAMP 1024  /* 128 threads x 8 items, gpu_global.cu:343-346 */

static void set_threads(int nthreads) {
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#else
    (void)nthreads;
#endif
}

/* ---- distances --------------------------------------------------------- */

/* Sub-space distance ||r - c||^2 as the reference's LUT build and direct ADC
 * both write it (gpu_global.cu:115-157 and :274-313, identical expressions). */
static inline float sub_dist(const float* r, const float* c, int sd) {
    if (sd == 4) {
        float dx = r[0] - c[0], dy = r[1] - c[1], dz = r[2] - c[2], dw = r[3] - c[3];
        return fmaf(dx, dx, fmaf(dy, dy, fmaf(dz, dz, dw * dw)));
    }
    if (sd == 8) {
        float a[8];
        for (int i = 0; i < 8; ++i) a[i] = r[i] - c[i];
        float d = fmaf(a[0], a[0], fmaf(a[1], a[1], fmaf(a[2], a[2], a[3] * a[3])));
        return fmaf(a[4], a[4], fmaf(a[5], a[5], fmaf(a[6], a[6], fmaf(a[7], a[7], d))));
    }
    float d = 0.0f;
    for (int i = 0; i < sd; ++i) {
        float df = r[i] - c[i];
        d = fmaf(df, df, d);
    }
    return d;
}

/* Exact squared L2 as nvcc compiles `acc += diff * diff` (contracted to an
 * FMA): the rerank (gpu_global.cu:636), and the oracle's coarse/GT/k-means. */
static inline float l2_seq(const float* a, const float* b, int dim) {
    float d = 0.0f;
    for (int j = 0; j < dim; ++j) {
        float df = a[j] - b[j];
        d = fmaf(df, df, d);
    }
    return d;
}

int fgo_lut(const float* residual, const float* codebook, int pq_m, int sub_dim, float* lut) {
    for (int m = 0; m < pq_m; ++m)
        for (int k = 0; k < 256; ++k)
            lut[m * 256 + k] = sub_dist(residual + m * sub_dim,
                                        codebook + ((size_t)m * 256 + k) * sub_dim, sub_dim);
    return 0;
}

/* ADC sum in subspace order, as compute_pq_dist_vectorized (gpu_global.cu:212-253). */
static inline float adc(const uint8_t* code, const float* lut, int pq_m) {
    float d = 0.0f;
    for (int m = 0; m < pq_m; ++m) d += lut[m * 256 + code[m]];
    return d;
}

/* ---- small sort helpers ---------------------------------------------- */

typedef struct { float d; uint32_t key2; int32_t id; } cand_t;

static int cmp_cand(const void* a, const void* b) {
    const cand_t* x = (const cand_t*)a;
    const cand_t* y = (const cand_t*)b;
    if (x->d < y->d) return -1;
    if (x->d > y->d) return 1;
    return (x->key2 < y->key2) ? -1 : (x->key2 > y->key2);
}

typedef struct { cand_t* v; size_t n, cap; } cvec;

static int cvec_push(cvec* c, float d, int32_t id, uint32_t key2) {
    if (c->n == c->cap) {
        size_t nc = c->cap ? c->cap * 2 : 1024;
        cand_t* nv = (cand_t*)realloc(c->v, nc * sizeof(cand_t));
        if (!nv) return -1;
        c->v = nv;
        c->cap = nc;
    }
    c->v[c->n].d = d;
    c->v[c->n].id = id;
    c->v[c->n].key2 = key2;
    c->n++;
    return 0;
}

/* ---- coarse (exact) --------------------------------------------------- */

int fgo_coarse(const float* centroids, int nlist, int dim, const float* queries, int nq,
               int top_m, uint32_t* out_ids, float* out_dists, int nthreads) {
    if (top_m < 1 || top_m > nlist || dim < 1 || nq < 0) return 1;
    set_threads(nthreads);
    int err = 0;
#pragma omp parallel
    {
        cand_t* all = (cand_t*)malloc((size_t)nlist * sizeof(cand_t));
        if (!all) {
#pragma omp atomic write
            err = 2;
        }
#pragma omp for schedule(dynamic, 8)
        for (int q = 0; q < nq; ++q) {
            if (!all) continue;
            const float* qv = queries + (size_t)q * dim;
            for (int c = 0; c < nlist; ++c) {
                all[c].d = l2_seq(qv, centroids + (size_t)c * dim, dim);
                all[c].key2 = (uint32_t)c;
                all[c].id = c;
            }
            qsort(all, (size_t)nlist, sizeof(cand_t), cmp_cand);
            for (int j = 0; j < top_m; ++j) {
                out_ids[(size_t)q * top_m + j] = (uint32_t)all[j].id;
                out_dists[(size_t)q * top_m + j] = all[j].d;
            }
        }
        free(all);
    }
    return err;
}

/* ---- batch logic: prune, LUT, phase 1, threshold, phase 2, sort, gather --- */

int fgo_batch_logic(const fgo_index* idx, const float* queries, int nq,
                    const uint32_t* probe_ids, const float* probe_dists, const fgo_params* p,
                    int32_t* top_ids, float* top_dists, int32_t* top_counts,
                    fgo_qstat* stats, int nthreads) {
    const int P = p->top_m, rm = p->rerank_m, M = idx->pq_m, sd = idx->sub_dim, D = idx->dim;
    if (P < 1 || P > 4096 || p->limit_k < 1 || rm < 1 || p->p1_lists < 0) return 1;
    if (M * sd != D) return 1;
    if (p->ref_compat && p->limit_k > FGO_REF_P1_CLAMP) return 1;
    int max_len = 0;
    for (int c = 0; c < idx->nlist; ++c) {
        int len = idx->offsets[c + 1] - idx->offsets[c];
        if (len > max_len) max_len = len;
    }
    if (max_len >= (1 << 19)) return 1;
    const int P1 = P < p->p1_lists ? P : p->p1_lists;
    set_threads(nthreads);
    int err = 0;
#pragma omp parallel
    {
        float* lut = (float*)malloc((size_t)M * 256 * sizeof(float));
        float* res = (float*)malloc((size_t)D * sizeof(float));
        uint32_t* pid = (uint32_t*)malloc((size_t)P * sizeof(uint32_t));
        float* cut = (float*)malloc((size_t)(P1 > 0 ? P1 : 1) * sizeof(float));
        cand_t* ld = (cand_t*)malloc((size_t)(max_len > 0 ? max_len : 1) * sizeof(cand_t));
        unsigned char* pass = (unsigned char*)malloc((size_t)(max_len > 0 ? max_len : 1));
        cvec cv = {0, 0, 0};
        if (!lut || !res || !pid || !cut || !ld || !pass) {
#pragma omp atomic write
            err = 2;
        }
#pragma omp for schedule(dynamic, 4)
        for (int q = 0; q < nq; ++q) {
            if (err) continue;
            const float* qv = queries + (size_t)q * D;
            cv.n = 0;
            int overflow = 0;
            /* prune (gpu_global.cu:43-51) */
            float best = probe_dists[(size_t)q * P];
            float pthr = best * p->prune_ratio;
            for (int j = 0; j < P; ++j)
                pid[j] = (probe_dists[(size_t)q * P + j] > pthr) ? FGO_INVALID
                                                                 : probe_ids[(size_t)q * P + j];
            /* phase 1 (gpu_global.cu:321-390) */
            for (int j = 0; j < P1; ++j) {
                cut[j] = 0.0f;
                uint32_t c = pid[j];
                if (c == FGO_INVALID) continue;
                int start = idx->offsets[c], len = idx->offsets[c + 1] - start;
                if (len == 0) continue;
                int wc = len < p->limit_k ? len : p->limit_k;
                int scan = (p->ref_compat && len > FGO_REF_P1_CLAMP) ? FGO_REF_P1_CLAMP : len;
                for (int t = 0; t < D; ++t) res[t] = qv[t] - idx->centroids[(size_t)c * D + t];
                fgo_lut(res, idx->codebook, M, sd, lut);
                for (int i = 0; i < scan; ++i) {
                    ld[i].d = adc(idx->codes + (size_t)(start + i) * M, lut, M);
                    ld[i].key2 = (uint32_t)i;
                    ld[i].id = idx->ids[start + i];
                }
                qsort(ld, (size_t)scan, sizeof(cand_t), cmp_cand);
                for (int r = 0; r < wc && r < scan; ++r)
                    cvec_push(&cv, ld[r].d, ld[r].id, ((uint32_t)j << 20) | ld[r].key2);
                if (wc - 1 < scan) cut[j] = ld[wc - 1].d;
            }
            /* threshold (gpu_global.cu:394-426) */
            float mn = FLT_MAX;
            for (int j = 0; j < P1; ++j)
                if (cut[j] > 0.0f && cut[j] < mn) mn = cut[j];
            float thr = (mn < FLT_MAX) ? mn * p->threshold_coeff : FLT_MAX;
            /* phase 2 (gpu_global.cu:428-527) */
            for (int j = P1; j < P; ++j) {
                uint32_t c = pid[j];
                if (c == FGO_INVALID) continue;
                int start = idx->offsets[c], len = idx->offsets[c + 1] - start;
                if (len == 0) continue;
                for (int t = 0; t < D; ++t) res[t] = qv[t] - idx->centroids[(size_t)c * D + t];
                fgo_lut(res, idx->codebook, M, sd, lut);
                int s_count = 0;
                for (int i = 0; i < len; ++i) {
                    ld[i].d = adc(idx->codes + (size_t)(start + i) * M, lut, M);
                    pass[i] = ld[i].d <= thr;
                    s_count += pass[i];
                }
                const uint32_t jb = (uint32_t)j << 20;
                if (!p->ref_compat || s_count <= FGO_REF_BLOCK) {
                    for (int i = 0; i < len; ++i)
                        if (pass[i]) cvec_push(&cv, ld[i].d, idx->ids[start + i], jb | (uint32_t)i);
                } else {
                    /* the first 128 passing are buffered in shared memory ... */
                    overflow++;
                    int emitted = 0;
                    for (int i = 0; i < len && emitted < FGO_REF_BLOCK; ++i)
                        if (pass[i]) {
                            cvec_push(&cv, ld[i].d, idx->ids[start + i], jb | (uint32_t)i);
                            emitted++;
                        }
                    /* ... then each of the 128 threads re-emits its first
                     * (s_count - 128) passing vectors (gpu_global.cu:508-526) */
                    int quota = s_count - FGO_REF_BLOCK;
                    int rank_t[FGO_REF_BLOCK];
                    memset(rank_t, 0, sizeof(rank_t));
                    for (int i = 0; i < len; ++i) {
                        if (!pass[i]) continue;
                        int t = i % FGO_REF_BLOCK;
                        if (rank_t[t] < quota) {
                            cvec_push(&cv, ld[i].d, idx->ids[start + i],
                                      jb | (1u << 19) | (uint32_t)i);
                            rank_t[t]++;
                        }
                    }
                }
            }
            /* stable sort by distance, then gather (gpu_global.cu:556-576) */
            int count = (int)cv.n;
            qsort(cv.v, cv.n, sizeof(cand_t), cmp_cand);
            int ak = count < rm ? count : rm;
            top_counts[q] = ak;
            for (int r = 0; r < rm; ++r) {
                size_t o = (size_t)q * rm + r;
                if (p->ref_compat && r >= FGO_REF_BLOCK) {
                    /* never written by the reference's 128-thread gather; modelled
                     * as freshly allocated (zeroed) device memory */
                    top_ids[o] = 0;
                    top_dists[o] = 0.0f;
                } else if (r < ak) {
                    top_ids[o] = cv.v[r].id;
                    top_dists[o] = cv.v[r].d;
                } else {
                    top_ids[o] = -1;
                    top_dists[o] = FLT_MAX;
                }
            }
            if (stats) {
                stats[q].count = count;
                stats[q].p2_overflow = overflow;
                stats[q].threshold = thr;
            }
        }
        free(lut); free(res); free(pid); free(cut); free(ld); free(pass); free(cv.v);
    }
    return err;
}

/* ---- heuristic rerank (gpu_global.cu:603-673) ----------------------------- */

int fgo_rerank(const float* queries, int nq, int dim, const int32_t* top_ids,
               const int32_t* top_counts, const float* base, int64_t nbase,
               const fgo_params* p, int32_t* out_ids, float* out_dists, int nthreads) {
    const int k = p->final_k, mb = p->mini_batch, rm = p->rerank_m;
    if (k < 1 || mb < 1 || rm < 1) return 1;
    if (p->ref_compat && k > FGO_REF_BLOCK) return 1;
    const int cap = k + mb;
    const int nw = (p->ref_compat && cap > FGO_REF_BLOCK) ? FGO_REF_BLOCK : cap;
    set_threads(nthreads);
    int err = 0;
#pragma omp parallel
    {
        cand_t* w = (cand_t*)malloc((size_t)cap * sizeof(cand_t));
        int32_t* fid = (int32_t*)malloc((size_t)k * sizeof(int32_t));
        float* fd = (float*)malloc((size_t)k * sizeof(float));
        if (!w || !fid || !fd) {
#pragma omp atomic write
            err = 2;
        }
#pragma omp for schedule(dynamic, 4)
        for (int q = 0; q < nq; ++q) {
            if (err) continue;
            const float* qv = queries + (size_t)q * dim;
            for (int i = 0; i < k; ++i) { fid[i] = -1; fd[i] = FLT_MAX; }
            int stab = 0, total = top_counts[q];
            for (int off = 0; off < rm; off += mb) {
                if (off >= total) break;
                int eff = mb < total - off ? mb : total - off;
                for (int i = 0; i < k; ++i) { w[i].d = fd[i]; w[i].id = fid[i]; w[i].key2 = (uint32_t)i; }
                for (int i = 0; i < mb && k + i < nw; ++i) {
                    float dist = FLT_MAX;
                    int32_t vid = -1;
                    if (i < eff) {
                        vid = top_ids[(size_t)q * rm + off + i];
                        if (vid >= 0 && (int64_t)vid < nbase)
                            dist = l2_seq(qv, base + (size_t)vid * dim, dim);
                    }
                    w[k + i].d = dist;
                    w[k + i].id = vid;
                    w[k + i].key2 = (uint32_t)(k + i);
                }
                qsort(w, (size_t)nw, sizeof(cand_t), cmp_cand);
                int chg = 0;
                for (int i = 0; i < k; ++i) {
                    int nid = w[i].id;
                    if (nid == -1) continue;
                    int f = 0;
                    for (int j = 0; j < k; ++j)
                        if (fid[j] == nid) { f = 1; break; }
                    if (!f) chg++;
                }
                if ((float)chg / (float)k <= p->epsilon) stab++; else stab = 0;
                for (int i = 0; i < k; ++i) { fid[i] = w[i].id; fd[i] = w[i].d; }
                if (stab >= p->beta) break;
            }
            for (int i = 0; i < k; ++i) {
                out_ids[(size_t)q * k + i] = fid[i];
                out_dists[(size_t)q * k + i] = fd[i];
            }
        }
        free(w); free(fid); free(fd);
    }
    return err;
}

int fgo_search(const fgo_index* idx, const float* base, int64_t nbase, const float* queries,
               int nq, const fgo_params* p, int32_t* out_ids, float* out_dists, int nthreads) {
    size_t P = (size_t)p->top_m, rm = (size_t)p->rerank_m;
    uint32_t* pids = (uint32_t*)malloc((size_t)nq * P * sizeof(uint32_t));
    float* pd = (float*)malloc((size_t)nq * P * sizeof(float));
    int32_t* tid = (int32_t*)malloc((size_t)nq * rm * sizeof(int32_t));
    float* td = (float*)malloc((size_t)nq * rm * sizeof(float));
    int32_t* tc = (int32_t*)malloc((size_t)nq * sizeof(int32_t));
    int rc = (!pids || !pd || !tid || !td || !tc) ? 2 : 0;
    if (!rc) rc = fgo_coarse(idx->centroids, idx->nlist, idx->dim, queries, nq, p->top_m, pids, pd, nthreads);
    if (!rc) rc = fgo_batch_logic(idx, queries, nq, pids, pd, p, tid, td, tc, NULL, nthreads);
    if (!rc) rc = fgo_rerank(queries, nq, idx->dim, tid, tc, base, nbase, p, out_ids, out_dists, nthreads);
    free(pids); free(pd); free(tid); free(td); free(tc);
    return rc;
}

/* ---- exact k-NN (ground truth): ties broken by smaller id ------------------ */

int fgo_knn_exact(const float* base, int64_t n, int dim, const float* queries, int nq, int k,
                  int32_t* out_ids, float* out_dists, int nthreads) {
    if (k < 1 || k > n) return 1;
    set_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
    for (int q = 0; q < nq; ++q) {
        const float* qv = queries + (size_t)q * dim;
        float* hd = out_dists + (size_t)q * k;
        int32_t* hi = out_ids + (size_t)q * k;
        int cnt = 0;
        /* insertion into a sorted array of size k (k is small in tests) */
        for (int64_t i = 0; i < n; ++i) {
            float d = l2_seq(qv, base + (size_t)i * dim, dim);
            if (cnt == k && !(d < hd[k - 1])) continue;
            int pos = cnt < k ? cnt : k - 1;
            while (pos > 0 && d < hd[pos - 1]) {
                hd[pos] = hd[pos - 1];
                hi[pos] = hi[pos - 1];
                --pos;
            }
            hd[pos] = d;
            hi[pos] = (int32_t)i;
            if (cnt < k) cnt++;
        }
    }
    return 0;
}

/* ---- build side ------------------------------------------------------------ */

/* MT19937 (Matsumoto & Nishimura 1998), the generator the reference seeds for
 * k-means initialisation (kmeans_gpu.cuh:260). */
typedef struct { uint32_t mt[624]; int i; } mt19937_t;

static void mt_seed(mt19937_t* s, uint32_t seed) {
    s->mt[0] = seed;
    for (int i = 1; i < 624; ++i)
        s->mt[i] = 1812433253u * (s->mt[i - 1] ^ (s->mt[i - 1] >> 30)) + (uint32_t)i;
    s->i = 624;
}

static uint32_t mt_next(mt19937_t* s) {
    if (s->i >= 624) {
        for (int k = 0; k < 624; ++k) {
            uint32_t y = (s->mt[k] & 0x80000000u) | (s->mt[(k + 1) % 624] & 0x7fffffffu);
            s->mt[k] = s->mt[(k + 397) % 624] ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
        }
        s->i = 0;
    }
    uint32_t y = s->mt[s->i++];
    y ^= y >> 11;
    y ^= (y << 7) & 0x9d2c5680u;
    y ^= (y << 15) & 0xefc60000u;
    y ^= y >> 18;
    return y;
}

uint32_t fgo_mt19937_first(uint32_t seed, int skip) {
    mt19937_t s;
    mt_seed(&s, seed);
    for (int i = 0; i < skip; ++i) mt_next(&s);
    return mt_next(&s);
}

/* ---- std::shuffle over MT19937, as the reference's PQ trainer draws it -----
 * pq_utils.h:24-26 and :90-93 call std::shuffle(v.begin(), v.end(), mt19937)
 * on a std::vector<int>.  With GCC's libstdc++ that is a Fisher-Yates shuffle
 * (element i swaps with a uniform position in [0, i], i = 1 .. n-1) whose
 * bounded integers come from Lemire's multiply-shift method with rejection
 * ("Fast Random Integer Generation in an Interval", ACM TOMACS 29(1), 2019)
 * on the 32-bit generator; when the generator's range covers n*n, one draw
 * in [0, (i+1)(i+2)) yields the swap positions of elements i and i+1 (the
 * quotient and the remainder by i+2), after a single draw in [0, 1] for
 * element 1 when n is even.  Pinned against std::shuffle itself by the CPU
 * tests (oracle/_ref). */
static uint32_t mt_below(mt19937_t* g, uint32_t range) {
    uint64_t prod = (uint64_t)mt_next(g) * range;
    uint32_t low = (uint32_t)prod;
    if (low < range) {
        const uint32_t thr = (uint32_t)(0u - range) % range;
        while (low < thr) {
            prod = (uint64_t)mt_next(g) * range;
            low = (uint32_t)prod;
        }
    }
    return (uint32_t)(prod >> 32);
}

static void swap_i32(int32_t* a, int64_t i, int64_t j) {
    const int32_t t = a[i];
    a[i] = a[j];
    a[j] = t;
}

void fgo_std_shuffle(int32_t* a, int64_t n, uint32_t seed) {
    if (n <= 1) return;
    mt19937_t g;
    mt_seed(&g, seed);
    if (0xffffffffull / (uint64_t)n >= (uint64_t)n) {
        int64_t i = 1;
        if (n % 2 == 0) {
            swap_i32(a, 1, (int64_t)mt_below(&g, 2u));
            i = 2;
        }
        while (i < n) {
            const uint64_t b1 = (uint64_t)i + 2;
            const uint32_t x = mt_below(&g, (uint32_t)(((uint64_t)i + 1) * b1));
            swap_i32(a, i, (int64_t)(x / b1));
            swap_i32(a, i + 1, (int64_t)(x % b1));
            i += 2;
        }
        return;
    }
    for (int64_t i = 1; i < n; ++i) swap_i32(a, i, (int64_t)mt_below(&g, (uint32_t)(i + 1)));
}

/* Strided initial centroids: point (i*stride + rng() % stride) % n for
 * centroid i, stride = max(1, n/k) (kmeans_gpu.cuh:259-267). */
int fgo_kmeans_init(const float* data, int64_t n, int dim, int k, uint32_t seed, float* centroids) {
    if (k < 1 || n < 1) return 1;
    mt19937_t s;
    mt_seed(&s, seed);
    int64_t stride = n / k > 1 ? n / k : 1;
    for (int i = 0; i < k; ++i) {
        int64_t id = ((int64_t)i * stride + (int64_t)(mt_next(&s) % (uint32_t)stride)) % n;
        memcpy(centroids + (size_t)i * dim, data + (size_t)id * dim, (size_t)dim * sizeof(float));
    }
    return 0;
}

/* Nearest centroid by exact L2; the lowest index wins ties. */
int fgo_assign(const float* data, int64_t n, int dim, const float* centroids, int k,
               int32_t* out_assign, int nthreads) {
    set_threads(nthreads);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        const float* x = data + (size_t)i * dim;
        float best = FLT_MAX;
        int32_t bc = 0;
        for (int c = 0; c < k; ++c) {
            float d = l2_seq(x, centroids + (size_t)c * dim, dim);
            if (d < best) { best = d; bc = c; }
        }
        out_assign[i] = bc;
    }
    return 0;
}

/* Centroid = mean of members, summed in point order in double and rounded
 * once; an empty cluster keeps its previous centroid. */
int fgo_kmeans_update(const float* data, int64_t n, int dim, const int32_t* assign, int k,
                      float* centroids, int32_t* counts) {
    double* acc = (double*)calloc((size_t)k * dim, sizeof(double));
    if (!acc) return 2;
    for (int c = 0; c < k; ++c) counts[c] = 0;
    for (int64_t i = 0; i < n; ++i) {
        int c = assign[i];
        counts[c]++;
        const float* x = data + (size_t)i * dim;
        double* a = acc + (size_t)c * dim;
        for (int j = 0; j < dim; ++j) a[j] += (double)x[j];
    }
    for (int c = 0; c < k; ++c) {
        if (counts[c] == 0) continue;
        for (int j = 0; j < dim; ++j)
            centroids[(size_t)c * dim + j] = (float)(acc[(size_t)c * dim + j] / (double)counts[c]);
    }
    free(acc);
    return 0;
}

int fgo_kmeans(const float* data, int64_t n, int dim, int k, int iters, uint32_t seed,
               float* centroids, int nthreads) {
    int32_t* as = (int32_t*)malloc((size_t)n * sizeof(int32_t));
    int32_t* cnt = (int32_t*)malloc((size_t)k * sizeof(int32_t));
    int rc = (!as || !cnt) ? 2 : fgo_kmeans_init(data, n, dim, k, seed, centroids);
    for (int it = 0; it < iters && !rc; ++it) {
        rc = fgo_assign(data, n, dim, centroids, k, as, nthreads);
        if (!rc) rc = fgo_kmeans_update(data, n, dim, as, k, centroids, cnt);
    }
    free(as);
    free(cnt);
    return rc;
}

/* List rebalancing (build_global.cu:62-169): a FIFO queue of lists, starting
 * with the non-empty input lists in order.  A list longer than
 * (size_t)(2 * n/k) and not shorter than 32 is split by k-means on its points
 * (sub_k = clamp(ceil(len/avg), 2, len/2), `iters` steps, `seed`) and the
 * exact assignment; its non-empty children go to the back of the queue.  Any
 * other list is final and numbered in the order it leaves the queue.  A split
 * whose points all land in one child makes that child final (the reference
 * would split it again forever).  Returns the list count in *out_nlist; when
 * it exceeds cap nothing is written and 3 is returned. */
typedef struct {
    int32_t* ids;
    int64_t len;
    float* cen;
} fgo_list;

typedef struct {
    fgo_list* v;
    int64_t n, cap;
} fgo_lists;

static int lists_push(fgo_lists* L, fgo_list x) {
    if (L->n == L->cap) {
        int64_t nc = L->cap ? 2 * L->cap : 64;
        fgo_list* nv = (fgo_list*)realloc(L->v, (size_t)nc * sizeof(fgo_list));
        if (!nv) return 2;
        L->v = nv;
        L->cap = nc;
    }
    L->v[L->n++] = x;
    return 0;
}

int fgo_rebalance(const float* data, int64_t n, int dim, const int32_t* assign,
                  const float* centroids, int k, int iters, uint32_t seed, int32_t* out_assign,
                  float* out_centroids, int cap, int32_t* out_nlist, int nthreads) {
    if (n < 1 || k < 1 || dim < 1) return 1;
    const double avg = (double)n / k;
    const size_t split_above = (size_t)(avg * 2);
    fgo_lists queue = {0}, done = {0};
    int64_t head = 0;
    int rc = 0;
    int64_t* cnt = (int64_t*)calloc((size_t)k, sizeof(int64_t));
    if (!cnt) return 2;
    for (int64_t i = 0; i < n; ++i) {
        if (assign[i] < 0 || assign[i] >= k) { free(cnt); return 1; }
        cnt[assign[i]]++;
    }
    for (int c = 0; c < k && !rc; ++c) {
        if (!cnt[c]) continue;
        fgo_list x;
        x.len = 0;
        x.ids = (int32_t*)malloc((size_t)cnt[c] * sizeof(int32_t));
        x.cen = (float*)malloc((size_t)dim * sizeof(float));
        if (!x.ids || !x.cen) { rc = 2; break; }
        memcpy(x.cen, centroids + (size_t)c * dim, (size_t)dim * sizeof(float));
        rc = lists_push(&queue, x);
    }
    free(cnt);
    /* members in ascending id order; queue slot j = j-th non-empty cluster */
    if (!rc) {
        int64_t* slot = (int64_t*)malloc((size_t)k * sizeof(int64_t));
        if (!slot) rc = 2;
        else {
            int64_t j = 0;
            for (int c = 0; c < k; ++c) slot[c] = -1;
            for (int64_t i = 0; i < n; ++i) slot[assign[i]] = 0;
            for (int c = 0; c < k; ++c)
                if (slot[c] == 0) slot[c] = j++;
            for (int64_t i = 0; i < n; ++i) {
                fgo_list* x = &queue.v[slot[assign[i]]];
                x->ids[x->len++] = (int32_t)i;
            }
            free(slot);
        }
    }
    while (!rc && head < queue.n) {
        fgo_list b = queue.v[head++];
        if ((size_t)b.len <= split_above || b.len < 32) {
            rc = lists_push(&done, b);
            continue;
        }
        int sub_k = (int)ceil((double)b.len / avg);
        if (sub_k < 2) sub_k = 2;
        if (sub_k > (int)b.len / 2) sub_k = (int)b.len / 2;
        float* sub = (float*)malloc((size_t)b.len * dim * sizeof(float));
        float* sc = (float*)malloc((size_t)sub_k * dim * sizeof(float));
        int32_t* sa = (int32_t*)malloc((size_t)b.len * sizeof(int32_t));
        int64_t* kc = (int64_t*)calloc((size_t)sub_k, sizeof(int64_t));
        if (!sub || !sc || !sa || !kc) rc = 2;
        if (!rc) {
            for (int64_t i = 0; i < b.len; ++i)
                memcpy(sub + (size_t)i * dim, data + (size_t)b.ids[i] * dim, (size_t)dim * sizeof(float));
            rc = fgo_kmeans(sub, b.len, dim, sub_k, iters, seed, sc, nthreads);
        }
        if (!rc) rc = fgo_assign(sub, b.len, dim, sc, sub_k, sa, nthreads);
        int nonempty = 0;
        if (!rc) {
            for (int64_t i = 0; i < b.len; ++i) kc[sa[i]]++;
            for (int c = 0; c < sub_k; ++c) nonempty += kc[c] ? 1 : 0;
        }
        for (int c = 0; c < sub_k && !rc; ++c) {
            if (!kc[c]) continue;
            fgo_list x;
            x.len = 0;
            x.ids = (int32_t*)malloc((size_t)kc[c] * sizeof(int32_t));
            x.cen = (float*)malloc((size_t)dim * sizeof(float));
            if (!x.ids || !x.cen) { free(x.ids); free(x.cen); rc = 2; break; }
            for (int64_t i = 0; i < b.len; ++i)
                if (sa[i] == c) x.ids[x.len++] = b.ids[i];
            memcpy(x.cen, sc + (size_t)c * dim, (size_t)dim * sizeof(float));
            rc = nonempty == 1 ? lists_push(&done, x) : lists_push(&queue, x);
        }
        free(sub); free(sc); free(sa); free(kc);
        free(b.ids); free(b.cen);
    }
    if (!rc) {
        *out_nlist = (int32_t)done.n;
        if (done.n > cap) rc = 3;
    }
    if (!rc) {
        for (int64_t c = 0; c < done.n; ++c) {
            for (int64_t i = 0; i < done.v[c].len; ++i) out_assign[done.v[c].ids[i]] = (int32_t)c;
            memcpy(out_centroids + (size_t)c * dim, done.v[c].cen, (size_t)dim * sizeof(float));
        }
    }
    for (int64_t i = head; i < queue.n; ++i) { free(queue.v[i].ids); free(queue.v[i].cen); }
    for (int64_t i = 0; i < done.n; ++i) { free(done.v[i].ids); free(done.v[i].cen); }
    free(queue.v);
    free(done.v);
    return rc;
}

/* Residual PQ training as pq_utils.h:77-138 computes it: the first `sample`
 * rows of std::shuffle(0..n-1, MT19937(12345)) give the residuals (in that
 * order); per subspace m, an independent 256-way k-means (pq_utils.h:17-72):
 * codeword c starts as the sample row at position c of
 * std::shuffle(0..S-1, MT19937(1234 + m)); `iters` Lloyd steps assign each
 * row to the first nearest codeword by `d += diff * diff` evaluated as a
 * rounded product then a rounded sum (the reference is built without FMA
 * contraction), and move each non-empty codeword to the mean of its rows,
 * summed in sample order in double and rounded to float. */
static void pq_assign_sep(const float* sub, int64_t S, int sd, const float* cb, int32_t* as) {
    for (int64_t i = 0; i < S; ++i) {
        float best = FLT_MAX;
        int32_t bc = 0;
        for (int c = 0; c < 256; ++c) {
            float d = 0.0f;
            for (int t = 0; t < sd; ++t) {
                const float df = sub[(size_t)i * sd + t] - cb[(size_t)c * sd + t];
                d = d + df * df; /* two roundings: this file is built with -ffp-contract=off */
            }
            if (d < best) { best = d; bc = c; }
        }
        as[i] = bc;
    }
}

int fgo_pq_train(const float* data, int64_t n, int dim, const int32_t* assign,
                 const float* centroids, int pq_m, int sample, int iters, float* codebook,
                 int nthreads) {
    if (pq_m < 1 || dim % pq_m) return 1;
    const int sd = dim / pq_m;
    int64_t S = sample < n ? sample : n;
    if (S < 256) return 1;
    float* res = (float*)malloc((size_t)S * dim * sizeof(float));
    int32_t* perm = (int32_t*)malloc((size_t)n * sizeof(int32_t));
    if (!res || !perm) { free(res); free(perm); return 2; }
    for (int64_t i = 0; i < n; ++i) perm[i] = (int32_t)i;
    fgo_std_shuffle(perm, n, 12345u);
    for (int64_t i = 0; i < S; ++i) {
        const int64_t id = perm[i];
        const float* x = data + (size_t)id * dim;
        const float* c = centroids + (size_t)assign[id] * dim;
        for (int j = 0; j < dim; ++j) res[(size_t)i * dim + j] = x[j] - c[j];
    }
    free(perm);
    int rc = 0;
    set_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
    for (int m = 0; m < pq_m; ++m) {
        float* sub = (float*)malloc((size_t)S * sd * sizeof(float));
        float* cb = codebook + (size_t)m * 256 * sd;
        int32_t* as = (int32_t*)malloc((size_t)S * sizeof(int32_t));
        int32_t* cnt = (int32_t*)malloc(256 * sizeof(int32_t));
        int32_t* idx = (int32_t*)malloc((size_t)S * sizeof(int32_t));
        if (!sub || !as || !cnt || !idx) {
#pragma omp atomic write
            rc = 2;
        } else {
            for (int64_t i = 0; i < S; ++i)
                for (int t = 0; t < sd; ++t) sub[(size_t)i * sd + t] = res[(size_t)i * dim + m * sd + t];
            for (int64_t i = 0; i < S; ++i) idx[i] = (int32_t)i;
            fgo_std_shuffle(idx, S, 1234u + (uint32_t)m);
            for (int c = 0; c < 256; ++c)
                memcpy(cb + (size_t)c * sd, sub + (size_t)idx[c] * sd, (size_t)sd * sizeof(float));
            for (int it = 0; it < iters; ++it) {
                pq_assign_sep(sub, S, sd, cb, as);
                fgo_kmeans_update(sub, S, sd, as, 256, cb, cnt);
            }
        }
        free(sub); free(as); free(cnt); free(idx);
    }
    free(res);
    return rc;
}

/* The rows fg_pq_train samples and the codeword seeds of each subspace, for
 * tests: rows[0..S) = first S of std::shuffle(0..n-1, MT19937(12345));
 * init[m*256 + c] = position c of std::shuffle(0..S-1, MT19937(1234 + m)). */
int fgo_pq_sample_rows(int64_t n, int64_t S, int pq_m, int32_t* rows, int32_t* init) {
    int32_t* perm = (int32_t*)malloc((size_t)(n > S ? n : S) * sizeof(int32_t));
    if (!perm) return 2;
    for (int64_t i = 0; i < n; ++i) perm[i] = (int32_t)i;
    fgo_std_shuffle(perm, n, 12345u);
    memcpy(rows, perm, (size_t)S * sizeof(int32_t));
    for (int m = 0; m < pq_m; ++m) {
        for (int64_t i = 0; i < S; ++i) perm[i] = (int32_t)i;
        fgo_std_shuffle(perm, S, 1234u + (uint32_t)m);
        memcpy(init + (size_t)m * 256, perm, 256 * sizeof(int32_t));
    }
    free(perm);
    return 0;
}

/* code[i][m] = nearest sub-codeword of the residual (first minimum wins), with
 * the reference encoder's contracted `dist += diff * diff` (kmeans_gpu.cuh:427-441). */
int fgo_pq_encode(const float* data, int64_t n, int dim, const int32_t* assign,
                  const float* centroids, const float* codebook, int pq_m, uint8_t* codes,
                  int nthreads) {
    if (pq_m < 1 || dim % pq_m) return 1;
    const int sd = dim / pq_m;
    set_threads(nthreads);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        const float* x = data + (size_t)i * dim;
        const float* c = centroids + (size_t)assign[i] * dim;
        for (int m = 0; m < pq_m; ++m) {
            float best = FLT_MAX;
            int bk = 0;
            for (int k = 0; k < 256; ++k) {
                const float* e = codebook + ((size_t)m * 256 + k) * sd;
                float d = 0.0f;
                for (int t = 0; t < sd; ++t) {
                    float r = x[m * sd + t] - c[m * sd + t];
                    float df = r - e[t];
                    d = fmaf(df, df, d);
                }
                if (d < best) { best = d; bk = k; }
            }
            codes[(size_t)i * pq_m + m] = (uint8_t)bk;
        }
    }
    return 0;
}

/* ---- search-parameter tuner (tune_parameters.cu:169-1013) ------------------
 * Same statistics as the reference's tune_search_parameters for given sample
 * queries and ground truth: coarse distances as the reference's host code
 * computes them (separate multiply and add), LUT / PQ / exact distances as its
 * device kernels do (fmaf per dimension). */

static float l2_host(const float* a, const float* b, int dim) {
    float d = 0.0f;
    for (int j = 0; j < dim; ++j) {
        float df = a[j] - b[j];
        float sq = df * df;
        d = d + sq;
    }
    return d;
}

static void tune_lut(const float* q, const float* cen, const float* codebook, int pq_m, int sd, float* lut) {
    for (int m = 0; m < pq_m; ++m)
        for (int j = 0; j < 256; ++j) {
            const float* cb = codebook + ((size_t)m * 256 + j) * sd;
            float acc = 0.0f;
            for (int d = 0; d < sd; ++d) {
                float r = q[m * sd + d] - cen[m * sd + d];
                float df = r - cb[d];
                acc = fmaf(df, df, acc);
            }
            lut[m * 256 + j] = acc;
        }
}

static float tune_pq(const uint8_t* code, const float* lut, int pq_m) {
    float s = 0.0f;
    for (int m = 0; m < pq_m; ++m) s = s + lut[m * 256 + code[m]];
    return s;
}

typedef struct {
    float d;
    int c;
} fgo_dc;

static int cmp_dc(const void* a, const void* b) {
    const fgo_dc* x = (const fgo_dc*)a;
    const fgo_dc* y = (const fgo_dc*)b;
    if (x->d < y->d) return -1;
    if (y->d < x->d) return 1;
    return (x->c > y->c) - (x->c < y->c);
}

static int cmp_f(const void* a, const void* b) {
    float x = *(const float*)a, y = *(const float*)b;
    return (x > y) - (x < y);
}

static int cmp_i(const void* a, const void* b) {
    int x = *(const int*)a, y = *(const int*)b;
    return (x > y) - (x < y);
}

/* sorted copy's element (int)((float)n * p), clamped (tune_parameters.cu:169-184) */
static int pct_int(const int* v, int64_t n, float p) {
    if (n <= 0) return 0;
    int* s = (int*)malloc((size_t)n * sizeof(int));
    memcpy(s, v, (size_t)n * sizeof(int));
    qsort(s, (size_t)n, sizeof(int), cmp_i);
    int i = (int)((float)n * p);
    if (i >= n) i = (int)n - 1;
    if (i < 0) i = 0;
    int r = s[i];
    free(s);
    return r;
}

/* elbow of the hits-per-rank curve (tune_parameters.cu:199-456) */
void fgo_tune_elbow(const int* hits, int n, int64_t total, int* point, float* coverage) {
    *point = 1;
    *coverage = 0.0f;
    if (n == 0 || total == 0) return;
    float* cov = (float*)calloc((size_t)n, sizeof(float));
    float* lg = (float*)calloc((size_t)n, sizeof(float));
    float* sm = (float*)calloc((size_t)n, sizeof(float));
    float* cu = (float*)calloc((size_t)n, sizeof(float));
    float* vo = (float*)calloc((size_t)n, sizeof(float));
    int64_t run = 0;
    for (int i = 0; i < n; ++i) {
        run += hits[i];
        cov[i] = (float)run / (float)total;
        lg[i] = logf((float)hits[i] + 1.0f);
    }
    for (int i = 0; i < n; ++i) {
        if (i == 0 || i == n - 1) {
            sm[i] = lg[i];
        } else {
            float a = 0.25f * lg[i - 1];
            float b = 0.50f * lg[i];
            float c = 0.25f * lg[i + 1];
            sm[i] = (a + b) + c;
        }
    }
    for (int i = 1; i + 1 < n; ++i) {
        float two = 2.0f * sm[i];
        cu[i] = (sm[i + 1] - two) + sm[i - 1];
        float d1 = (float)(hits[i - 1] - hits[i]);
        float d2 = (float)(hits[i] - hits[i + 1]);
        if (d1 * d2 < 0.0f) vo[i] = 1.0f;
    }
    int best_i = -1;
    float best = -1e9f;
    for (int i = 2; i + 1 < n && i < 30; ++i) {
        if (cov[i] < 0.60f) continue;
        float cs = fabsf(cu[i]) * 10.0f;
        float before = (float)(hits[i - 1] - hits[i]) / ((float)hits[i - 1] + 1.0f);
        float after = (float)(hits[i] - hits[i + 1]) / ((float)hits[i] + 1.0f);
        float ds = 0.0f;
        if (after < before) ds = (before - after) * 8.0f;
        float r = (float)i / 32.0f;
        float bonus = 4.0f * (1.0f - r * r);
        float score = ((cs + ds) + bonus) - vo[i] * 5.0f;
        if (cov[i] >= 0.80f && score > best) {
            best = score;
            best_i = i;
        }
    }
    if (best_i >= 0) {
        *point = best_i + 1;
        *coverage = cov[best_i];
    } else {
        for (int i = 0; i < n; ++i)
            if (cov[i] >= 0.60f) {
                *point = i + 1;
                *coverage = cov[i];
                break;
            }
    }
    free(cov); free(lg); free(sm); free(cu); free(vo);
}

int fgo_tune(const fgo_index* idx, const float* base, int64_t nbase, const float* queries, int nq,
             const int32_t* gt, int k, fgo_tune_result* out, int32_t* cluster_ranks,
             int32_t* pq_ranks, int32_t* exact_ranks, float* ratios, int nthreads) {
    const int dim = idx->dim, pq_m = idx->pq_m, sd = idx->sub_dim, nlist = idx->nlist;
    const int64_t np = (int64_t)nq * k;
    int32_t* owner = (int32_t*)malloc((size_t)nbase * sizeof(int32_t));
    int32_t* first = (int32_t*)malloc((size_t)nbase * sizeof(int32_t));
    int32_t* cr = (int32_t*)malloc((size_t)np * sizeof(int32_t));
    int32_t* pr = (int32_t*)malloc((size_t)np * sizeof(int32_t));
    int32_t* er = (int32_t*)malloc((size_t)np * sizeof(int32_t));
    float* pqt = (float*)malloc((size_t)np * sizeof(float));
    float* cut = (float*)malloc((size_t)nq * sizeof(float));
    if (!owner || !first || !cr || !pr || !er || !pqt || !cut) return 2;
    for (int64_t i = 0; i < nbase; ++i) owner[i] = first[i] = -1;
    for (int c = 0; c < nlist; ++c)
        for (int j = idx->offsets[c]; j < idx->offsets[c + 1]; ++j) {
            int32_t id = idx->ids[j];
            if (id >= 0 && id < nbase && owner[id] < 0) {
                owner[id] = c;
                first[id] = j;
            }
        }
    set_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t p = 0; p < np; ++p) {
        const int q = (int)(p / k);
        const float* qv = queries + (size_t)q * dim;
        int32_t id = gt[p];
        int c = (id >= 0 && id < nbase) ? owner[id] : -1;
        cr[p] = pr[p] = er[p] = -1;
        pqt[p] = -1.0f;
        if (c < 0) continue;
        float dc = l2_host(qv, idx->centroids + (size_t)c * dim, dim);
        int before = 0;
        for (int c2 = 0; c2 < nlist; ++c2) {
            float d2 = l2_host(qv, idx->centroids + (size_t)c2 * dim, dim);
            if (d2 < dc || (d2 == dc && c2 < c)) ++before;
        }
        cr[p] = before + 1;
        float* lut = (float*)malloc((size_t)pq_m * 256 * sizeof(float));
        tune_lut(qv, idx->centroids + (size_t)c * dim, idx->codebook, pq_m, sd, lut);
        float pt = tune_pq(idx->codes + (size_t)first[id] * pq_m, lut, pq_m);
        float et = l2_seq(qv, base + (size_t)id * dim, dim);
        int npq = 0, nex = 0;
        for (int j = idx->offsets[c]; j < idx->offsets[c + 1]; ++j) {
            if (tune_pq(idx->codes + (size_t)j * pq_m, lut, pq_m) < pt) ++npq;
            int32_t v = idx->ids[j];
            if (v >= 0 && v < nbase && l2_seq(qv, base + (size_t)v * dim, dim) < et) ++nex;
        }
        free(lut);
        pr[p] = npq + 1;
        er[p] = nex + 1;
        pqt[p] = pt;
    }
    fgo_tune_result r;
    memset(&r, 0, sizeof(r));
    int* ranks = (int*)malloc((size_t)np * sizeof(int));
    int64_t nr = 0;
    int max_rank = 0;
    for (int64_t p = 0; p < np; ++p)
        if (cr[p] > 0) {
            ranks[nr++] = cr[p];
            if (cr[p] > max_rank) max_rank = cr[p];
        }
    r.top_m = pct_int(ranks, nr, 0.995f);
    int* hits = (int*)calloc((size_t)(max_rank > 0 ? max_rank : 1), sizeof(int));
    for (int64_t i = 0; i < nr; ++i) hits[ranks[i] - 1]++;
    fgo_tune_elbow(hits, max_rank, nr, &r.p1_lists, &r.coverage_at_elbow);
    r.n_ranked = (int)nr;
    int* allq = (int*)malloc((size_t)np * sizeof(int));
    int64_t na = 0, n1 = 0;
    int mx1 = 0;
    for (int64_t p = 0; p < np; ++p) {
        if (pr[p] <= 0) continue;
        allq[na++] = pr[p];
        if (cr[p] > 0 && cr[p] <= r.p1_lists) {
            ++n1;
            if (pr[p] > mx1) mx1 = pr[p];
        }
    }
    r.limit_k = n1 ? mx1 : pct_int(allq, na, 0.98f);
    r.n_in_p1 = (int)n1;
    const int P = r.p1_lists < nlist ? (r.p1_lists > 1 ? r.p1_lists : 1) : nlist;
#pragma omp parallel for schedule(dynamic, 1)
    for (int q = 0; q < nq; ++q) {
        const float* qv = queries + (size_t)q * dim;
        fgo_dc* all = (fgo_dc*)malloc((size_t)nlist * sizeof(fgo_dc));
        for (int c = 0; c < nlist; ++c) {
            all[c].d = l2_host(qv, idx->centroids + (size_t)c * dim, dim);
            all[c].c = c;
        }
        qsort(all, (size_t)nlist, sizeof(fgo_dc), cmp_dc);
        float* lut = (float*)malloc((size_t)pq_m * 256 * sizeof(float));
        float best = 0.0f;
        int have = 0;
        for (int s = 0; s < P; ++s) {
            int c = all[s].c;
            int lo = idx->offsets[c], len = idx->offsets[c + 1] - lo;
            if (len <= 0) continue;
            tune_lut(qv, idx->centroids + (size_t)c * dim, idx->codebook, pq_m, sd, lut);
            float* d = (float*)malloc((size_t)len * sizeof(float));
            for (int j = 0; j < len; ++j) d[j] = tune_pq(idx->codes + (size_t)(lo + j) * pq_m, lut, pq_m);
            qsort(d, (size_t)len, sizeof(float), cmp_f);
            int i = r.limit_k - 1 < len - 1 ? r.limit_k - 1 : len - 1;
            if (i < 0) i = 0;
            if (!have || d[i] < best) best = d[i];
            have = 1;
            free(d);
        }
        cut[q] = have ? best : NAN;
        free(lut);
        free(all);
    }
    float mx = 0.0f;
    int nrat = 0;
    for (int q = 0; q < nq; ++q) {
        float ratio = NAN;
        int64_t far = (int64_t)q * k + (k - 1);
        if (!isnan(cut[q]) && pr[far] > 0 && pqt[far] >= 0.0f && cut[q] > 0.0f) {
            ratio = pqt[far] / cut[q];
            if (!nrat || ratio > mx) mx = ratio;
            ++nrat;
        }
        if (ratios) ratios[q] = ratio;
    }
    r.threshold_coeff = nrat ? mx : 2.0f;
    r.n_ratios = nrat;
    if (cluster_ranks) memcpy(cluster_ranks, cr, (size_t)np * sizeof(int32_t));
    if (pq_ranks) memcpy(pq_ranks, pr, (size_t)np * sizeof(int32_t));
    if (exact_ranks) memcpy(exact_ranks, er, (size_t)np * sizeof(int32_t));
    *out = r;
    free(owner); free(first); free(cr); free(pr); free(er); free(pqt); free(cut);
    free(ranks); free(hits); free(allq);
    return 0;
}

/* ---- graph index (the product's CAGRA-style build and search) ---------------
 * No reference implementation exists (the reference's only graph is cuVS
 * CAGRA over its centroids, a library absent here); this restates the
 * product's documented algorithm step by step so the CUDA kernels can be
 * checked bit for bit. */

static float half_bits_to_float(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ff, bits;
    if (e == 0) {
        if (m == 0) {
            bits = sign;
        } else { /* subnormal: normalise */
            int sh = 0;
            while (!(m & 0x400)) { m <<= 1; ++sh; }
            m &= 0x3ff;
            bits = sign | ((uint32_t)(127 - 15 + 1 - sh) << 23) | (m << 13);
        }
    } else if (e == 31) {
        bits = sign | 0x7f800000u | (m << 13);
    } else {
        bits = sign | ((e + 127 - 15) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static float dist_metric(const float* a, const float* b, int dim, int metric) {
    if (metric == 1) {
        float acc = 0.0f;
        for (int j = 0; j < dim; ++j) acc = fmaf(a[j], b[j], acc);
        return -acc;
    }
    return l2_seq(a, b, dim);
}

typedef struct {
    float d;
    int32_t id;
} fgo_did;

static int cmp_did(const void* x, const void* y) {
    const fgo_did* a = (const fgo_did*)x;
    const fgo_did* b = (const fgo_did*)y;
    if (a->d < b->d) return -1;
    if (b->d < a->d) return 1;
    return (a->id > b->id) - (a->id < b->id);
}

static int cmp_u32(const void* x, const void* y) {
    uint32_t a = *(const uint32_t*)x, b = *(const uint32_t*)y;
    return (a > b) - (a < b);
}

int fgo_graph_build(const float* data, int64_t n, int dim, int D, int I, int L, int P, int iters,
                    uint32_t seed, int metric, int32_t* graph, float* entry_centroids,
                    int32_t* entry_nodes, int nthreads) {
    if (n < 2 || D < 2 || (D & 1) || I < D || L < 1 || L > n || P < 1 || P > L) return 1;
    float* cen = (float*)malloc((size_t)L * dim * sizeof(float));
    int32_t* as = (int32_t*)malloc((size_t)n * sizeof(int32_t));
    int32_t* order = (int32_t*)malloc((size_t)n * sizeof(int32_t));
    int64_t* off = (int64_t*)calloc((size_t)L + 1, sizeof(int64_t));
    int32_t* g0 = (int32_t*)malloc((size_t)n * I * sizeof(int32_t));
    int32_t* pr = (int32_t*)malloc((size_t)n * D * sizeof(int32_t));
    int32_t* nn = (int32_t*)malloc((size_t)L * P * sizeof(int32_t));
    if (!cen || !as || !order || !off || !g0 || !pr || !nn) return 2;
    int rc = fgo_kmeans(data, n, dim, L, iters, seed, cen, nthreads);
    if (!rc) rc = fgo_assign(data, n, dim, cen, L, as, nthreads);
    if (rc) return rc;
    for (int64_t i = 0; i < n; ++i) off[as[i] + 1]++;
    for (int c = 0; c < L; ++c) off[c + 1] += off[c];
    {
        int64_t* fill = (int64_t*)malloc((size_t)L * sizeof(int64_t));
        memcpy(fill, off, (size_t)L * sizeof(int64_t));
        for (int64_t i = 0; i < n; ++i) order[fill[as[i]]++] = (int32_t)i;
        free(fill);
    }
    /* nearest lists of every list */
    for (int c = 0; c < L; ++c) {
        fgo_did* all = (fgo_did*)malloc((size_t)L * sizeof(fgo_did));
        for (int c2 = 0; c2 < L; ++c2) {
            all[c2].d = l2_seq(cen + (size_t)c * dim, cen + (size_t)c2 * dim, dim);
            all[c2].id = c2;
        }
        qsort(all, (size_t)L, sizeof(fgo_did), cmp_did);
        for (int j = 0; j < P; ++j) nn[(size_t)c * P + j] = all[j].id;
        free(all);
    }
    /* initial k-NN graph */
    for (int64_t i = 0; i < n * I; ++i) g0[i] = -1;
    for (int c = 0; c < L; ++c) {
        int lists[4096];
        int nl = 0;
        lists[nl++] = c;
        for (int j = 0; j < P && nl < P; ++j)
            if (nn[(size_t)c * P + j] != c) lists[nl++] = nn[(size_t)c * P + j];
        int64_t nc = 0;
        for (int l = 0; l < nl; ++l) nc += off[lists[l] + 1] - off[lists[l]];
        uint32_t* cand = (uint32_t*)malloc((size_t)(nc > 0 ? nc : 1) * sizeof(uint32_t));
        int64_t t = 0;
        for (int l = 0; l < nl; ++l)
            for (int64_t r = off[lists[l]]; r < off[lists[l] + 1]; ++r) cand[t++] = (uint32_t)order[r];
        qsort(cand, (size_t)nc, sizeof(uint32_t), cmp_u32);
        const int64_t kk = nc < I + 1 ? nc : I + 1;
        set_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 16)
        for (int64_t r = off[c]; r < off[c + 1]; ++r) {
            const int32_t self = order[r];
            fgo_did* d = (fgo_did*)malloc((size_t)nc * sizeof(fgo_did));
            for (int64_t j = 0; j < nc; ++j) {
                d[j].d = dist_metric(data + (size_t)self * dim, data + (size_t)cand[j] * dim, dim, metric);
                d[j].id = (int32_t)cand[j];
            }
            qsort(d, (size_t)nc, sizeof(fgo_did), cmp_did);
            int o = 0;
            for (int64_t j = 0; j < kk && o < I; ++j)
                if (d[j].id != self) g0[(size_t)self * I + o++] = d[j].id;
            free(d);
        }
        free(cand);
    }
    /* pruning by detour count */
    set_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 64)
    for (int64_t u = 0; u < n; ++u) {
        const int32_t* nb = g0 + (size_t)u * I;
        uint32_t* key = (uint32_t*)malloc((size_t)I * sizeof(uint32_t));
        for (int i = 0; i < I; ++i) {
            if (nb[i] < 0) {
                key[i] = (0xffffu << 16) | (uint32_t)i;
                continue;
            }
            int cnt = 0;
            for (int j = 0; j < i; ++j) {
                if (nb[j] < 0) continue;
                const int32_t* wl = g0 + (size_t)nb[j] * I;
                for (int x = 0; x < i; ++x)
                    if (wl[x] == nb[i]) { ++cnt; break; }
            }
            key[i] = ((uint32_t)(cnt < 0xffff ? cnt : 0xffff) << 16) | (uint32_t)i;
        }
        qsort(key, (size_t)I, sizeof(uint32_t), cmp_u32);
        for (int r = 0; r < D; ++r) pr[(size_t)u * D + r] = nb[key[r] & 0xffffu];
        free(key);
    }
    /* reverse edges: for each v, sources u in (rank, u) order */
    int64_t* rcount = (int64_t*)calloc((size_t)n + 1, sizeof(int64_t));
    for (int i = 0; i < D; ++i)
        for (int64_t u = 0; u < n; ++u) {
            int32_t v = pr[(size_t)u * D + i];
            if (v >= 0) rcount[v + 1]++;
        }
    for (int64_t v = 0; v < n; ++v) rcount[v + 1] += rcount[v];
    int32_t* rsrc = (int32_t*)malloc((size_t)(rcount[n] > 0 ? rcount[n] : 1) * sizeof(int32_t));
    int64_t* rfill = (int64_t*)malloc((size_t)n * sizeof(int64_t));
    memcpy(rfill, rcount, (size_t)n * sizeof(int64_t));
    for (int i = 0; i < D; ++i)
        for (int64_t u = 0; u < n; ++u) {
            int32_t v = pr[(size_t)u * D + i];
            if (v >= 0) rsrc[rfill[v]++] = (int32_t)u;
        }
    /* final lists */
    for (int64_t u = 0; u < n; ++u) {
        int32_t* out = graph + (size_t)u * D;
        const int32_t* pu = pr + (size_t)u * D;
        int cnt = 0, half = D / 2, taken = 0;
        for (int r = 0; r < half; ++r) {
            int32_t v = pu[r], dup = 0;
            for (int x = 0; x < cnt; ++x) dup |= out[x] == v;
            if (v >= 0 && !dup) out[cnt++] = v;
        }
        for (int64_t e = rcount[u]; e < rcount[u + 1] && taken < D - half && cnt < D; ++e) {
            int32_t v = rsrc[e], dup = 0;
            for (int x = 0; x < cnt; ++x) dup |= out[x] == v;
            if (!dup) { out[cnt++] = v; ++taken; }
        }
        for (int r = half; r < D && cnt < D; ++r) {
            int32_t v = pu[r], dup = 0;
            for (int x = 0; x < cnt; ++x) dup |= out[x] == v;
            if (v >= 0 && !dup) out[cnt++] = v;
        }
        for (; cnt < D; ++cnt) out[cnt] = -1;
    }
    /* entry points: centroids and each list's medoid by the metric */
    if (entry_centroids) memcpy(entry_centroids, cen, (size_t)L * dim * sizeof(float));
    if (entry_nodes)
        for (int c = 0; c < L; ++c) {
            float best = FLT_MAX;
            int32_t bid = -1;
            for (int64_t r = off[c]; r < off[c + 1]; ++r) {
                const int32_t id = order[r];
                const float d = dist_metric(data + (size_t)id * dim, cen + (size_t)c * dim, dim, metric);
                if (bid < 0 || d < best || (d == best && id < bid)) {
                    best = d;
                    bid = id;
                }
            }
            entry_nodes[c] = bid;
        }
    free(rcount); free(rsrc); free(rfill);
    free(cen); free(as); free(order); free(off); free(g0); free(pr); free(nn);
    return 0;
}

static uint32_t gmix32(uint32_t h) {
    h ^= h >> 16;
    h *= 0x85ebca6bu;
    h ^= h >> 13;
    h *= 0xc2b2ae35u;
    h ^= h >> 16;
    return h;
}

/* one warp's distance: lane l sums its 16-byte chunks l, l+32, ... with fmaf,
 * then the xor butterfly 16, 8, 4, 2, 1 */
static float warp_dist_emul(const float* x, const float* q, int dim, int E, int metric) {
    float v[32], w[32];
    const int nch = dim / E;
    for (int l = 0; l < 32; ++l) {
        float acc = 0.0f;
        for (int c = l; c < nch; c += 32)
            for (int e = 0; e < E; ++e) {
                const float a = x[c * E + e], b = q[c * E + e];
                if (metric == 1) {
                    acc = fmaf(a, b, acc);
                } else {
                    const float df = a - b;
                    acc = fmaf(df, df, acc);
                }
            }
        v[l] = acc;
    }
    for (int o = 16; o; o >>= 1) {
        for (int l = 0; l < 32; ++l) w[l] = v[l] + v[l ^ o];
        memcpy(v, w, sizeof(v));
    }
    return metric == 1 ? -v[0] : v[0];
}

static uint32_t fkey(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

static float fkey_inv(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static int cmp_u64(const void* x, const void* y) {
    uint64_t a = *(const uint64_t*)x, b = *(const uint64_t*)y;
    return (a > b) - (a < b);
}

#define FGO_GS_HASH 4096

int fgo_graph_search(const void* data, int dtype, int64_t n, int dim, const int32_t* graph, int D,
                     const float* entry_cen, const int32_t* entry_nodes, int n_entries,
                     int entry_probes, const void* queries, int nq, int itopk, int width,
                     int max_iter, int k, uint32_t seed, int metric, int32_t* out_ids,
                     float* out_dists, uint64_t* counters, int nthreads) {
    const int E = dtype == 1 ? 8 : 4;
    if (dim % E || k < 1 || k > itopk || width < 1) return 1;
    if (max_iter == 0) max_iter = 2 * ((itopk + width - 1) / width) + 10;
    const int WD = width * D;
    uint64_t evals = 0, expanded = 0;
    set_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1) reduction(+ : evals, expanded)
    for (int q = 0; q < nq; ++q) {
        float* qv = (float*)malloc((size_t)dim * sizeof(float));
        float* xv = (float*)malloc((size_t)dim * sizeof(float));
        uint8_t* vis = (uint8_t*)calloc((size_t)n, 1);
        int32_t* vlist = (int32_t*)malloc((size_t)(FGO_GS_HASH + WD + itopk) * sizeof(int32_t));
        uint64_t* top = (uint64_t*)malloc((size_t)itopk * sizeof(uint64_t));
        uint8_t* ex = (uint8_t*)calloc((size_t)itopk, 1);
        uint64_t* cand = (uint64_t*)malloc((size_t)WD * sizeof(uint64_t));
        uint64_t* mt = (uint64_t*)malloc((size_t)itopk * sizeof(uint64_t));
        uint8_t* me = (uint8_t*)malloc((size_t)itopk);
        int32_t* slot = (int32_t*)malloc((size_t)WD * sizeof(int32_t));
        int nvis = 0, ntop = 0;
        for (int j = 0; j < dim; ++j)
            qv[j] = dtype == 1 ? half_bits_to_float(((const uint16_t*)queries)[(size_t)q * dim + j])
                               : ((const float*)queries)[(size_t)q * dim + j];
        for (int iter = -1; iter < max_iter; ++iter) {
            if (iter < 0) {
                int S = 0;
                if (entry_probes > 0 && n_entries > 0) {
                    S = entry_probes < n_entries ? entry_probes : n_entries;
                    if (S > WD) S = WD;
                    fgo_dc* ed = (fgo_dc*)malloc((size_t)n_entries * sizeof(fgo_dc));
                    for (int c = 0; c < n_entries; ++c) {
                        ed[c].d = dist_metric(qv, entry_cen + (size_t)c * dim, dim, metric);
                        ed[c].c = c;
                    }
                    qsort(ed, (size_t)n_entries, sizeof(fgo_dc), cmp_dc);
                    for (int s = 0; s < S; ++s) slot[s] = entry_nodes[ed[s].c];
                    free(ed);
                }
                for (int s = S; s < WD; ++s) {
                    uint32_t x = gmix32(seed ^ gmix32((uint32_t)((int64_t)q * WD + s) * 0x9e3779b9u + 0x7f4a7c15u));
                    slot[s] = (int32_t)((uint64_t)x % (uint64_t)n);
                }
            } else {
                int32_t par[2048];
                int np = 0;
                for (int t = 0; t < ntop && np < width; ++t)
                    if (!ex[t]) {
                        par[np++] = (int32_t)(top[t] & 0xffffffffu);
                        ex[t] = 1;
                    }
                if (np == 0) break;
                expanded += (uint64_t)np;
                if (nvis > FGO_GS_HASH / 2) {
                    for (int x = 0; x < nvis; ++x) vis[vlist[x]] = 0;
                    nvis = 0;
                    for (int t = 0; t < ntop; ++t) {
                        int32_t v = (int32_t)(top[t] & 0xffffffffu);
                        vis[v] = 1;
                        vlist[nvis++] = v;
                    }
                }
                for (int s = 0; s < WD; ++s) {
                    int pi = s / D;
                    slot[s] = pi < np ? graph[(size_t)par[pi] * D + (s - pi * D)] : -1;
                }
            }
            int m = 0;
            for (int s = 0; s < WD; ++s) {
                int32_t v = slot[s];
                if (v < 0 || v >= n || vis[v]) continue;
                vis[v] = 1;
                vlist[nvis++] = v;
                for (int j = 0; j < dim; ++j)
                    xv[j] = dtype == 1 ? half_bits_to_float(((const uint16_t*)data)[(size_t)v * dim + j])
                                       : ((const float*)data)[(size_t)v * dim + j];
                float d = warp_dist_emul(xv, qv, dim, E, metric);
                cand[m++] = ((uint64_t)fkey(d) << 32) | (uint32_t)v;
            }
            evals += (uint64_t)m;
            qsort(cand, (size_t)m, sizeof(uint64_t), cmp_u64);
            /* merge */
            int i = 0, j = 0, r = 0;
            while (r < itopk && (i < ntop || j < m)) {
                if (i < ntop && (j >= m || top[i] < cand[j])) {
                    mt[r] = top[i];
                    me[r++] = ex[i++];
                } else {
                    mt[r] = cand[j++];
                    me[r++] = 0;
                }
            }
            ntop = r;
            memcpy(top, mt, (size_t)r * sizeof(uint64_t));
            memcpy(ex, me, (size_t)r);
        }
        for (int r = 0; r < k; ++r) {
            if (r < ntop) {
                out_ids[(size_t)q * k + r] = (int32_t)(top[r] & 0xffffffffu);
                out_dists[(size_t)q * k + r] = fkey_inv((uint32_t)(top[r] >> 32));
            } else {
                out_ids[(size_t)q * k + r] = -1;
                out_dists[(size_t)q * k + r] = FLT_MAX;
            }
        }
        free(qv); free(xv); free(vis); free(vlist); free(top); free(ex); free(cand); free(mt); free(me);
        free(slot);
    }
    if (counters) {
        counters[0] = evals;
        counters[1] = expanded;
    }
    return 0;
}
