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

/* Residual PQ training: a strided sample of `sample` residuals (seed 12345),
 * then an independent 256-way k-means per subspace (seed 1234 + m, `iters`
 * Lloyd steps), as pq_utils.h:77-138 structures it. */
int fgo_pq_train(const float* data, int64_t n, int dim, const int32_t* assign,
                 const float* centroids, int pq_m, int sample, int iters, float* codebook,
                 int nthreads) {
    if (pq_m < 1 || dim % pq_m) return 1;
    const int sd = dim / pq_m;
    int64_t S = sample < n ? sample : n;
    if (S < 256) return 1;
    float* res = (float*)malloc((size_t)S * dim * sizeof(float));
    if (!res) return 2;
    mt19937_t s;
    mt_seed(&s, 12345u);
    int64_t stride = n / S > 1 ? n / S : 1;
    for (int64_t i = 0; i < S; ++i) {
        int64_t id = (i * stride + (int64_t)(mt_next(&s) % (uint32_t)stride)) % n;
        const float* x = data + (size_t)id * dim;
        const float* c = centroids + (size_t)assign[id] * dim;
        for (int j = 0; j < dim; ++j) res[(size_t)i * dim + j] = x[j] - c[j];
    }
    int rc = 0;
    set_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 1)
    for (int m = 0; m < pq_m; ++m) {
        float* sub = (float*)malloc((size_t)S * sd * sizeof(float));
        float* cb = codebook + (size_t)m * 256 * sd;
        int32_t* as = (int32_t*)malloc((size_t)S * sizeof(int32_t));
        int32_t* cnt = (int32_t*)malloc(256 * sizeof(int32_t));
        if (!sub || !as || !cnt) {
#pragma omp atomic write
            rc = 2;
        } else {
            for (int64_t i = 0; i < S; ++i)
                for (int t = 0; t < sd; ++t) sub[(size_t)i * sd + t] = res[(size_t)i * dim + m * sd + t];
            fgo_kmeans_init(sub, S, sd, 256, 1234u + (uint32_t)m, cb);
            for (int it = 0; it < iters; ++it) {
                fgo_assign(sub, S, sd, cb, 256, as, 1);
                fgo_kmeans_update(sub, S, sd, as, 256, cb, cnt);
            }
        }
        free(sub); free(as); free(cnt);
    }
    free(res);
    return rc;
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
