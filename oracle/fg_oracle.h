/*
 * fg_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement (plain C + OpenMP) of the reference's IVF-PQ search and
 * build arithmetic.  Only tests, the smoke check and bench.py's CPU-baseline
 * leg load this library; the product never links it.
 *
 * Reference files restated (Hello-day/FusionGPU):
 *   gpu_global.cu:31-77    prune + count               -> fgo_batch_logic
 *   gpu_global.cu:79-166   residual LUT                -> fgo_lut
 *   gpu_global.cu:212-319  ADC (LUT / direct)          -> fgo_lut + adc
 *   gpu_global.cu:321-390  phase-1 scan                -> fgo_batch_logic
 *   gpu_global.cu:394-426  threshold                   -> fgo_batch_logic
 *   gpu_global.cu:428-527  phase-2 scan (+ overflow)   -> fgo_batch_logic
 *   gpu_global.cu:533-576  compact / sort / gather     -> fgo_batch_logic
 *   gpu_global.cu:603-673  heuristic rerank            -> fgo_rerank
 *   kmeans_gpu.cuh:234-324 Lloyd k-means               -> fgo_kmeans
 *   kmeans_gpu.cuh:403-445 residual PQ encode          -> fgo_pq_encode
 *   pq_utils.h:17-138      residual PQ training        -> fgo_pq_train
 */
#ifndef FG_ORACLE_H
#define FG_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int dim, pq_m, sub_dim, nlist, total;
    const float*   codebook;   /* [pq_m][256][sub_dim]          */
    const int32_t* offsets;    /* [nlist + 1]                   */
    const int32_t* ids;        /* [total]                       */
    const uint8_t* codes;      /* [total][pq_m]                 */
    const float*   centroids;  /* [nlist][dim]                  */
} fgo_index;

typedef struct {
    int   top_m, p1_lists, limit_k;
    float threshold_coeff, prune_ratio;
    int   rerank_m, final_k, mini_batch;
    float epsilon;
    int   beta;
    int   ref_compat;          /* 1 = reproduce the reference's gather/rerank/scan quirks */
} fgo_params;

/* per-query diagnostics of fgo_batch_logic */
typedef struct {
    int32_t count;             /* candidates emitted (d_atomic in the reference)       */
    int32_t p2_overflow;       /* phase-2 lists whose passing count exceeded 128       */
    float   threshold;         /* phase-2 threshold                                    */
} fgo_qstat;

int fgo_coarse(const float* centroids, int nlist, int dim, const float* queries, int nq,
               int top_m, uint32_t* out_ids, float* out_dists, int nthreads);

int fgo_lut(const float* residual, const float* codebook, int pq_m, int sub_dim, float* lut);

int fgo_batch_logic(const fgo_index* idx, const float* queries, int nq,
                    const uint32_t* probe_ids, const float* probe_dists, const fgo_params* p,
                    int32_t* top_ids, float* top_dists, int32_t* top_counts,
                    fgo_qstat* stats, int nthreads);

int fgo_rerank(const float* queries, int nq, int dim, const int32_t* top_ids,
               const int32_t* top_counts, const float* base, int64_t nbase,
               const fgo_params* p, int32_t* out_ids, float* out_dists, int nthreads);

int fgo_search(const fgo_index* idx, const float* base, int64_t nbase, const float* queries,
               int nq, const fgo_params* p, int32_t* out_ids, float* out_dists, int nthreads);

int fgo_knn_exact(const float* base, int64_t n, int dim, const float* queries, int nq, int k,
                  int32_t* out_ids, float* out_dists, int nthreads);

/* build side */
uint32_t fgo_mt19937_first(uint32_t seed, int skip);
/* std::shuffle(a, a + n, std::mt19937(seed)) as GCC's libstdc++ performs it */
void fgo_std_shuffle(int32_t* a, int64_t n, uint32_t seed);
/* the sample rows and per-subspace codeword seeds of fgo_pq_train */
int fgo_pq_sample_rows(int64_t n, int64_t S, int pq_m, int32_t* rows, int32_t* init);
int fgo_kmeans_init(const float* data, int64_t n, int dim, int k, uint32_t seed, float* centroids);
int fgo_assign(const float* data, int64_t n, int dim, const float* centroids, int k,
               int32_t* out_assign, int nthreads);
int fgo_kmeans_update(const float* data, int64_t n, int dim, const int32_t* assign, int k,
                      float* centroids, int32_t* counts);
int fgo_kmeans(const float* data, int64_t n, int dim, int k, int iters, uint32_t seed,
               float* centroids, int nthreads);
int fgo_rebalance(const float* data, int64_t n, int dim, const int32_t* assign,
                  const float* centroids, int k, int iters, uint32_t seed, int32_t* out_assign,
                  float* out_centroids, int cap, int32_t* out_nlist, int nthreads);
int fgo_pq_train(const float* data, int64_t n, int dim, const int32_t* assign,
                 const float* centroids, int pq_m, int sample, int iters, float* codebook,
                 int nthreads);
int fgo_pq_encode(const float* data, int64_t n, int dim, const int32_t* assign,
                  const float* centroids, const float* codebook, int pq_m, uint8_t* codes,
                  int nthreads);

/* Search-parameter tuner (tune_parameters.cu:459-1013): same fields as
 * fg_tune_result of the product's C ABI. */
typedef struct {
    int32_t top_m, p1_lists, limit_k;
    float threshold_coeff, coverage_at_elbow;
    int32_t n_ranked, n_in_p1, n_ratios;
} fgo_tune_result;

void fgo_tune_elbow(const int* hits, int n, int64_t total, int* point, float* coverage);
int fgo_tune(const fgo_index* idx, const float* base, int64_t nbase, const float* queries, int nq,
             const int32_t* gt, int k, fgo_tune_result* out, int32_t* cluster_ranks,
             int32_t* pq_ranks, int32_t* exact_ranks, float* ratios, int nthreads);

/* Graph index: the product's build and search, restated (fg_graph_build /
 * fg_graph_search of the product's C ABI; no reference implementation).
 * data for the build is fp32; for the search dtype 0 = fp32, 1 = fp16 bits.
 * metric 0 = L2, 1 = inner product (distance = -dot). */
int fgo_graph_build(const float* data, int64_t n, int dim, int D, int I, int L, int P, int iters,
                    uint32_t seed, int metric, int32_t* graph, float* entry_centroids,
                    int32_t* entry_nodes, int nthreads);
int fgo_graph_search(const void* data, int dtype, int64_t n, int dim, const int32_t* graph, int D,
                     const float* entry_cen, const int32_t* entry_nodes, int n_entries,
                     int entry_probes, const void* queries, int nq, int itopk, int width,
                     int max_iter, int k, uint32_t seed, int metric, int32_t* out_ids,
                     float* out_dists, uint64_t* counters, int nthreads);

#ifdef __cplusplus
}
#endif
#endif
