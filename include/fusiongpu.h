/*
 * fusiongpu.h -- C ABI of the B200 (sm_100a) IVF-PQ search engine.
 *
 * Plain C: pointers, sizes and an opaque stream handle (a cudaStream_t passed
 * as void*; NULL = the legacy default stream).  Every entry point returns an
 * fg_status; on failure fg_last_error() gives a message (thread-local).
 * All vector/index buffers are caller-owned DEVICE memory unless the name
 * says "host".  Scratch memory is caller-owned too: query the *_workspace_size
 * function and pass a device buffer at least that large (256-byte aligned).
 * No entry point allocates device memory, and calls on different workspaces
 * may run concurrently on different streams.
 *
 * Each entry point names the reference interface (Hello-day/FusionGPU) it
 * replaces.
 */
#ifndef FUSIONGPU_H
#define FUSIONGPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FG_INVALID_PROBE 0xFFFFFFFFu

/* Distance used by the exact k-NN and the graph index: squared L2, or the
 * negated inner product (smaller is nearer in both). */
typedef enum {
    FG_METRIC_L2 = 0,
    FG_METRIC_IP = 1
} fg_metric;

/* Element type of the graph index's vectors. */
typedef enum {
    FG_DTYPE_F32 = 0,
    FG_DTYPE_F16 = 1
} fg_dtype;

typedef enum {
    FG_OK = 0,
    FG_ERR_INVALID_ARG = 1,   /* a size, pointer or parameter is out of range         */
    FG_ERR_CUDA = 2,          /* a CUDA runtime call or kernel launch failed          */
    FG_ERR_WORKSPACE = 3,     /* workspace missing, misaligned or too small           */
    FG_ERR_UNSUPPORTED = 4,   /* a shape this build has no kernel for                 */
    FG_ERR_DEVICE = 5         /* a kernel reported an error status from the device    */
} fg_status;

/* Read-only device view of an IVF-PQ index.  Same arrays as the reference's
 * IVFIndexGPU (defs.h:49-56) and ivf_data.bin (build_global.cu:242-252), with
 * the compile-time DIM / PQ_M of defs.h:9-12 made runtime fields. */
typedef struct {
    const float*   pq_codebook;   /* [pq_m][256][dim/pq_m]                       */
    const int32_t* list_offsets;  /* [nlist + 1], list c = [offsets[c], offsets[c+1]) */
    const uint8_t* pq_codes;      /* [total][pq_m], row-major, lists contiguous   */
    const int32_t* vector_ids;    /* [total]                                      */
    const float*   centroids;     /* [nlist][dim]                                 */
    int32_t nlist;
    int32_t dim;
    int32_t pq_m;
    int32_t total;
    int32_t max_list_len;         /* longest list (kernels size shared memory by it) */
} fg_ivfpq_view;

/* Search parameters.  Names and defaults follow the reference's flags
 * (search_pipeline.cu:562-588, defs.h:17-41). */
typedef struct {
    int32_t top_m;            /* nprobe: probed lists per query (-m)                  */
    int32_t p1_lists;         /* lists scanned in phase 1 (--p1_lists)                */
    int32_t limit_k;          /* candidates kept per phase-1 list (--limit_k)         */
    float   threshold_coeff;  /* phase-2 threshold factor (--threshold_coeff)         */
    float   prune_ratio;      /* drop probes farther than best * ratio (-p)           */
    int32_t rerank_m;         /* rerank depth (-r)                                    */
    int32_t final_k;          /* results per query (-k)                               */
    int32_t mini_batch;       /* rerank mini-batch (-mb)                              */
    float   epsilon;          /* rerank change-rate bound (-e)                        */
    int32_t beta;             /* rerank stable rounds before stopping (--beta)        */
    int32_t ref_compat;       /* 1: reproduce the reference's 128-lane gather, 128-entry
                                 rerank window, 1024-vector phase-1 clamp and phase-2
                                 overflow re-emission; 0: full rerank_m / k+mini_batch */
} fg_search_params;

const char* fg_version(void);
const char* fg_last_error(void);
void fg_search_params_default(fg_search_params* p);

/* ---- coarse quantizer: replaces search_cagra_index (cagra_adapter.cuh:38-68)
 * Exact top_m nearest centroids per query by squared L2, ascending by
 * (distance, centroid id).  out_ids/out_dists: [nq][top_m]. */
int fg_coarse_workspace_size(int32_t nlist, int32_t dim, int32_t nq, int32_t top_m, size_t* bytes);
int fg_coarse_search(const float* centroids, int32_t nlist, int32_t dim, const float* queries,
                     int32_t nq, int32_t top_m, uint32_t* out_ids, float* out_dists,
                     void* workspace, size_t workspace_bytes, void* stream);

/* The same ranking through one fixed path: exact fp32 CUDA-core tiles, or the
 * tcgen05 tensor-core GEMM (split-bf16 operands staged by TMA) whose top
 * candidates are rescored exactly and certified against an error bound, with
 * an exact per-query fallback.  fg_coarse_search picks the tensor-core path
 * when 3*dim <= 384.  n_fallback (HOST int, may be NULL): when given, the call
 * waits for the stream and stores how many queries needed the exact fallback.
 * Both return the same ids and distances. */
int fg_coarse_search_simt(const float* centroids, int32_t nlist, int32_t dim, const float* queries,
                          int32_t nq, int32_t top_m, uint32_t* out_ids, float* out_dists,
                          void* workspace, size_t workspace_bytes, void* stream);
int fg_coarse_search_tc(const float* centroids, int32_t nlist, int32_t dim, const float* queries,
                        int32_t nq, int32_t top_m, uint32_t* out_ids, float* out_dists,
                        void* workspace, size_t workspace_bytes, int32_t* n_fallback, void* stream);

/* ---- allocation-free coarse search (no counterpart in the reference)
 * For callers that cannot give this library device memory when they call it:
 * plugins whose host runtime owns every device pool and forbids its plugins
 * the CUDA allocator, and serving loops that must never reach cudaMalloc or
 * cudaFree (both can synchronise the whole device).  Same results as
 * fg_coarse_search_simt, with the scratch in a fixed 16 MiB device array built
 * into the library (held on every GPU that loads it).  Returns
 * FG_ERR_INVALID_ARG when one query's scratch row (4*nlist bytes, plus
 * 8*top_m per 8192 centroids past the first 8192) exceeds it.  The first call
 * on each device resolves the array's address and caches it for the life of
 * the process; make that first call before any stream capture, and do not
 * call this entry point on a device after cudaDeviceReset there (the cached
 * address would be stale).  All calls on a device share the array: calls
 * whose GPU work overlaps race and must be serialised by the caller. */
int fg_coarse_search_noalloc(const float* centroids, int32_t nlist, int32_t dim, const float* queries,
                             int32_t nq, int32_t top_m, uint32_t* out_ids, float* out_dists,
                             void* stream);

/* ---- candidate generation: replaces run_gpu_batch_logic (gpu_global.cu:679-874)
 * Prune, phase-1 ADC scan with per-list top-limit_k, threshold, phase-2 ADC
 * scan, and the sorted top rerank_m candidates per query.  Short lists (mean
 * length <= 400) run in a persistent kernel that keeps the PQ codebook in
 * shared memory and computes each ADC term on the fly; long lists in one CTA
 * per query with a per-(query, list) LUT in shared memory.  Both produce the
 * reference's floats bit for bit.  FG_SCAN_KERNEL=block|team|team_lut|team_otf
 * and FG_SCAN_TEAM_NT=64|128|256 in the environment override the choice.
 * probe_ids/probe_dists: [nq][top_m] as fg_coarse_search writes them
 * (FG_INVALID_PROBE entries are skipped).  top_ids/top_dists: [nq][rerank_m];
 * top_counts: [nq] = min(#candidates, rerank_m).  Needs no workspace.  The
 * probe list is not modified. */
int fg_batch_logic(const fg_ivfpq_view* index, const float* queries, int32_t nq,
                   const uint32_t* probe_ids, const float* probe_dists,
                   const fg_search_params* params, int32_t* top_ids, float* top_dists,
                   int32_t* top_counts, int32_t* candidate_counts, void* stream);

/* The same with a caller workspace of at least fg_batch_logic_workspace_size
 * bytes (256-byte aligned; 0 bytes, and any pointer, when the size is 0).
 * With it, long lists (typical length above 400: the larger of the mean
 * over all lists and half the longest) run the split path: the (query,
 * probed list) pairs grouped by list, each pair taken by one resident CTA for
 * phase 1 and for phase 2, candidates in a per-query region of the
 * workspace, then one selection CTA per query -- the same results as
 * fg_batch_logic, bit for bit.  Short lists with top_m between 8 and
 * p1_lists (every probe in phase 1) run the group kernel instead: up to 3
 * queries probing one list share its codebook reads, candidates in the same
 * per-query regions (top_m * limit_k keys each).  fg_search uses it.  The
 * split path's region holds max(4096, 2 * rerank_m) 8-byte keys per query
 * (10,000 queries, rerank_m 4096: 655 MB), so split very large batches; a
 * query whose candidates overflow its region is recomputed by the per-query
 * kernel.  The size is 0 when neither path applies. */
int fg_batch_logic_workspace_size(const fg_ivfpq_view* index, const fg_search_params* params, int32_t nq,
                                  size_t* bytes);
int fg_batch_logic_ws(const fg_ivfpq_view* index, const float* queries, int32_t nq,
                      const uint32_t* probe_ids, const float* probe_dists,
                      const fg_search_params* params, int32_t* top_ids, float* top_dists,
                      int32_t* top_counts, int32_t* candidate_counts, void* workspace,
                      size_t workspace_bytes, void* stream);

/* ---- candidate budget: replaces prune_and_count_fused_kernel + the offsets
 * scan (gpu_global.cu:31-77, 709-725).  counts[q] = summed length of the
 * probed lists whose distance is <= probe_dists[q][0] * prune_ratio (the
 * lists fg_batch_logic scans); offsets [nq+1] (may be NULL) = exclusive scan
 * of counts, offsets[nq] = the batch total.  fg_batch_logic does not need it;
 * it serves callers that size buffers or report pruning statistics. */
int fg_probe_budget(const int32_t* list_offsets, int32_t nlist, const uint32_t* probe_ids,
                    const float* probe_dists, int32_t nq, int32_t top_m, float prune_ratio,
                    int32_t* counts, int32_t* offsets, void* stream);

/* ---- exact rerank: replaces run_gpu_rerank (gpu_global.cu:603-673)
 * Mini-batches of `mini_batch` candidates, exact fp32 squared L2 against the
 * raw base vectors [nbase][dim], merged into a running top-final_k with the
 * reference's early stop.  out_ids/out_dists: [nq][final_k]. */
int fg_rerank(const float* queries, int32_t nq, int32_t dim, const int32_t* top_ids,
              const int32_t* top_counts, const float* base, int64_t nbase,
              const fg_search_params* params, int32_t* out_ids, float* out_dists, void* stream);

/* The same with uint8 raw vectors [nbase][dim] (C5's base): each byte
 * converts exactly to float, so results equal fg_rerank on a float copy;
 * 16-byte loads when dim % 16 == 0 (then the base must be 16-byte aligned). */
int fg_rerank_u8(const float* queries, int32_t nq, int32_t dim, const int32_t* top_ids,
                 const int32_t* top_counts, const uint8_t* base, int64_t nbase,
                 const fg_search_params* params, int32_t* out_ids, float* out_dists, void* stream);

/* ---- full search: coarse + candidate generation + rerank on one stream.
 * Replaces one SearchPipeline::submit_batch (search_pipeline.cu:311-377)
 * minus the host copies.  Allocation- and synchronisation-free (capturable
 * into a CUDA graph); one workspace per concurrently running call.  The scan
 * hands out queries through a counter in the workspace. */
int fg_search_workspace_size(const fg_ivfpq_view* index, const fg_search_params* params,
                             int32_t nq, size_t* bytes);
int fg_search(const fg_ivfpq_view* index, const float* base, int64_t nbase, const float* queries,
              int32_t nq, const fg_search_params* params, int32_t* out_ids, float* out_dists,
              void* workspace, size_t workspace_bytes, void* stream);
/* fg_search over uint8 raw vectors (fg_rerank_u8 for the last stage). */
int fg_search_u8(const fg_ivfpq_view* index, const uint8_t* base, int64_t nbase, const float* queries,
                 int32_t nq, const fg_search_params* params, int32_t* out_ids, float* out_dists,
                 void* workspace, size_t workspace_bytes, void* stream);
/* *mapped = 1 when kernels on the current device can read and write the host
 * memory at p through the address p itself (page-locked memory under unified
 * addressing), else 0.  Such memory may be passed as out_ids / out_dists of
 * fg_search: the rerank kernel then writes the results straight into host
 * memory, so no device-to-host copy follows the search.  No counterpart in the
 * reference, which copies results back after each batch
 * (search_pipeline.cu:311-377). */
int fg_host_memory_mapped(const void* p, int32_t* mapped);

/* ---- sharded search: the exchange step (no counterpart in the single-GPU
 * reference, whose search runs on device 0 only, search_pipeline.cu:560).
 * Each GPU searches the lists it owns with fg_search; fg_map_ids turns its
 * shard-local vector ids into global ones (out[i] = map[in[i]], negative or
 * out-of-range ids become -1); after an all-gather of the per-GPU results
 * laid out [nshards][nq][k] (each row ascending by distance),
 * fg_merge_topk keeps the k smallest per query by (distance, global id).
 * nshards * k <= 4096. */
int fg_map_ids(const int32_t* in, int64_t n, const int32_t* map, int64_t nmap, int32_t* out,
               void* stream);
int fg_merge_topk(const float* dists, const int32_t* ids, int32_t nshards, int32_t nq, int32_t k,
                  int32_t* out_ids, float* out_dists, void* stream);

/* The exchange as ONE all-gather: fg_pack_topk turns each GPU's [nq][k]
 * result into one uint64 tensor, key = orderable(distance) << 32 | global id
 * (global id = map[id], or the id itself when map is null; -1 for an id
 * outside the map), each row of k keys sorted ascending; after the all-gather
 * of those keys ([nshards][nq][k], rows as fg_pack_topk wrote them)
 * fg_merge_topk_keys merges the nshards sorted rows of each query, keeps the
 * k smallest keys, i.e. by (distance, global id), and unpacks them.
 * k <= 4096, nshards * k <= 4096. */
int fg_pack_topk(const int32_t* ids, const float* dists, int32_t nq, int32_t k, const int32_t* map,
                 int64_t nmap, uint64_t* keys, void* stream);
int fg_merge_topk_keys(const uint64_t* keys, int32_t nshards, int32_t nq, int32_t k, int32_t* out_ids,
                       float* out_dists, void* stream);

/* ---- search-parameter tuner: replaces tune_search_parameters
 * (tune_parameters.cu:459-1013).  For nq sample queries with their exact k
 * nearest base vectors gt_ids [nq][k] (ascending distance; fg_knn_exact),
 * derives the reference's four recommendations:
 *   top_m           = P99.5 of the coarse rank (1-based, lists ordered by
 *                     (distance, id)) of each neighbour's list;
 *   p1_lists        = the elbow of the hits-per-coarse-rank histogram;
 *   limit_k         = the largest PQ rank inside its own list of the
 *                     neighbours whose list ranks <= p1_lists (P98 of all PQ
 *                     ranks when there is none);
 *   threshold_coeff = the largest ratio, over queries, of the farthest
 *                     neighbour's PQ distance to the smallest phase-1 cutoff
 *                     (the min(limit_k, len)-th smallest PQ distance of each
 *                     non-empty list among the first p1_lists); 2 if none.
 * A neighbour's list is the lowest-numbered list holding its id.  Optional
 * HOST outputs (NULL to skip): cluster_ranks, pq_ranks, exact_ranks [nq][k]
 * (-1 where the id is in no list) and ratios [nq] (NaN where a query gives
 * none).  Synchronises the stream and allocates its own device scratch. */
typedef struct {
    int32_t top_m;
    int32_t p1_lists;
    int32_t limit_k;
    float   threshold_coeff;
    float   coverage_at_elbow;  /* share of neighbours within the first p1_lists lists */
    int32_t n_ranked;           /* neighbours found in some list                       */
    int32_t n_in_p1;            /* of those, in a list ranked <= p1_lists               */
    int32_t n_ratios;           /* queries that gave a threshold ratio                  */
} fg_tune_result;

int fg_tune(const fg_ivfpq_view* index, const float* base, int64_t nbase, const float* queries,
            int32_t nq, const int32_t* gt_ids, int32_t k, fg_tune_result* out,
            int32_t* cluster_ranks, int32_t* pq_ranks, int32_t* exact_ranks, float* ratios,
            void* stream);

/* The elbow rule fg_tune applies to the hits-per-coarse-rank histogram
 * (find_elbow_point, tune_parameters.cu:199-456), on host arrays: hits[i] =
 * neighbours whose list ranks i+1, total = their sum.  Writes the 1-based
 * elbow rank and the coverage there. */
int fg_tune_elbow(const int32_t* hits, int32_t n, int64_t total, int32_t* point, float* coverage);

/* ---- graph index (no counterpart in the reference, whose only graph is
 * cuVS CAGRA over its centroids, cagra_adapter.cuh:10-68): a fixed-degree
 * k-NN graph after the CAGRA design, for the C4 configuration.
 *
 * fg_graph_build: 1. IVF partition of the data (fg_kmeans with nlist lists,
 * kmeans_iters steps, seed; exact assignment).  2. Initial graph of degree
 * intermediate_degree: each point's exact nearest neighbours (metric) among
 * the members of its list's probe_lists nearest lists (itself dropped, ties
 * by id).  3. Pruning to graph_degree: neighbour v_i (rank i) of u scores the
 * number of detours u->v_j->v_i with j < i and rank(v_i in N(v_j)) < i;
 * fewest detours first, ties by rank.  4-5. Final list: the first
 * graph_degree/2 pruned neighbours, then up to graph_degree/2 reverse
 * neighbours (sources u ordered by (rank, u)), then the rest of the pruned
 * list, without duplicates; -1 pads.  data: [n][dim] of dtype (device);
 * graph: [n][graph_degree] int32 (device).  Optional entry points for the
 * search (device, may be NULL): entry_centroids [nlist][dim] float (the IVF
 * centroids) and entry_nodes [nlist] (each list's member nearest its
 * centroid by the metric, ties by id; -1 for an empty list).  Synchronises;
 * allocates its own scratch. */
typedef struct {
    int32_t graph_degree;         /* D, even (64)                             */
    int32_t intermediate_degree;  /* initial k-NN degree, >= D (128)          */
    int32_t nlist;                /* IVF lists that supply the candidates     */
    int32_t probe_lists;          /* lists whose members are candidates       */
    int32_t kmeans_iters;
    uint32_t seed;
    int32_t metric;               /* fg_metric                                */
} fg_graph_build_params;

int fg_graph_build(const void* data, int32_t dtype, int64_t n, int32_t dim,
                   const fg_graph_build_params* params, int32_t* graph,
                   float* entry_centroids, int32_t* entry_nodes, void* stream);

/* fg_graph_search: CTA per query.  A top list of itopk (distance, id)
 * entries is seeded with search_width*degree start nodes: the entry nodes of
 * the query's entry_probes nearest entry centroids (exact metric distance,
 * fmaf in dimension order, ties by list id; selected for the whole batch by
 * one tiled pass before the search), then pseudo-random nodes (murmur3
 * finaliser of seed, query and slot) for the remaining slots.  Each
 * iteration expands the first search_width unexplored entries: their
 * neighbours not yet visited (open-addressing hash of 4096 slots in shared
 * memory, reset to the top list when half full) get distances (one warp per
 * vector, 16-byte loads, lane-strided fmaf then a fixed xor-butterfly sum)
 * and are merged in by (distance, id).  Stops when no unexplored entry
 * remains or after max_iterations (0: 2*ceil(itopk / search_width) + 10).
 * data / queries: [n][dim] / [nq][dim] of dtype, rows 16 bytes aligned (dim
 * multiple of 8 for f16, 4 for f32); entry_centroids / entry_nodes /
 * n_entries as fg_graph_build writes them (NULL / 0 when entry_probes is 0);
 * out_ids/out_dists [nq][k] ascending (IP distance = -dot).  counters
 * (device, may be NULL): [0] += distance evaluations, [1] += expanded nodes,
 * [2] += index checks that failed (a graph entry or buffer index out of
 * range; the access is skipped, so a corrupt graph gives wrong results
 * instead of a fault).  The workspace (fg_graph_search_workspace_size) holds
 * the entry selection; none is needed when entry_probes is 0. */
typedef struct {
    int32_t itopk;           /* internal top-list size (128)        */
    int32_t search_width;    /* parents per iteration (4)           */
    int32_t max_iterations;  /* 0 = automatic                       */
    int32_t k;               /* results per query, <= itopk         */
    uint32_t seed;           /* pseudo-random start nodes           */
    int32_t metric;          /* fg_metric                           */
    int32_t entry_probes;    /* nearest entry lists seeded (0: none), <= 4096 */
} fg_graph_search_params;

int fg_graph_search_workspace_size(int32_t dtype, int32_t dim, int32_t nq, int32_t n_entries,
                                   const fg_graph_search_params* params, size_t* bytes);
int fg_graph_search(const void* data, int32_t dtype, int64_t n, int32_t dim, const int32_t* graph,
                    int32_t degree, const float* entry_centroids, const int32_t* entry_nodes,
                    int32_t n_entries, const void* queries, int32_t nq,
                    const fg_graph_search_params* params, int32_t* out_ids, float* out_dists,
                    uint64_t* counters, void* workspace, size_t workspace_bytes, void* stream);

/* ---- index build (device pointers; the reference takes host pointers) ----- */

/* Strided k-means seeding: centroid i = data[(i*stride + r_i % stride) % n],
 * stride = max(1, n/k), r_i = the i-th output of MT19937(seed)
 * (kmeans_gpu.cuh:259-267).  workspace: at least k*8 bytes. */
int fg_kmeans_init(const float* data, int64_t n, int32_t dim, int32_t k, uint32_t seed,
                   float* centroids, void* workspace, size_t workspace_bytes, void* stream);

/* Nearest centroid by exact squared L2, lowest index on ties.  Replaces
 * gpu_assign_to_centroids / gpu_assign_initial_clusters (kmeans_gpu.cuh:329-394).
 * For dim <= 128 (k >= 64, n >= 4096) the assignment runs on the tensor cores
 * (the coarse search with top_m = 1: split-bf16 tcgen05 GEMM, exact rescore,
 * certificate or exact fallback) in the caller's workspace (at least
 * fg_assign_workspace_size bytes; 0 when the CUDA-core path runs); the result
 * is identical to the CUDA-core path.  fg_kmeans uses the same dispatch. */
int fg_assign_workspace_size(int64_t n, int32_t dim, int32_t k, size_t* bytes);
int fg_assign(const float* data, int64_t n, int32_t dim, const float* centroids, int32_t k,
              int32_t* out_assign, void* workspace, size_t workspace_bytes, void* stream);

/* Stable counting sort of point ids by assignment: order[] lists the points
 * of cluster 0, then cluster 1, ... each in increasing id; offsets [k+1]. */
int fg_sort_by_list_workspace_size(int64_t n, int32_t k, size_t* bytes);
int fg_sort_by_list(const int32_t* assign, int64_t n, int32_t k, int32_t* order, int32_t* offsets,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Centroid update without float atomics: members summed in point order in
 * double, one rounding to float; empty clusters keep their centroid.
 * Replaces accumulate/compute_centroids (kmeans_gpu.cuh:81-116). */
int fg_kmeans_update(const float* data, int32_t dim, const int32_t* order, const int32_t* offsets,
                     int32_t k, float* centroids, void* stream);

/* Lloyd k-means: init + iters x (assign, sort, update).  Replaces
 * run_kmeans_gpu (kmeans_gpu.cuh:234-324). */
int fg_kmeans_workspace_size(int64_t n, int32_t dim, int32_t k, size_t* bytes);
int fg_kmeans(const float* data, int64_t n, int32_t dim, int32_t k, int32_t iters, uint32_t seed,
              float* centroids, void* workspace, size_t workspace_bytes, void* stream);

/* Residual PQ codebook training, the codebook the reference's
 * train_residual_pq_codebooks (pq_utils.h:77-138) writes, bit for bit: the
 * sample is the first `sample` rows of std::shuffle(0..n-1, MT19937(12345))
 * (GCC's shuffle, restated on the host), and each subspace runs a 256-way
 * k-means seeded with the rows at the first 256 positions of
 * std::shuffle(0..S-1, MT19937(1234 + m)), distances `d += diff * diff` with
 * two roundings, means summed in sample order in double.  n < 2^31.
 * Synchronises the host (the shuffles run there). */
int fg_pq_train_workspace_size(int64_t n, int32_t dim, int32_t pq_m, int32_t sample, size_t* bytes);
int fg_pq_train(const float* data, int64_t n, int32_t dim, const int32_t* assign,
                const float* centroids, int32_t pq_m, int32_t sample, int32_t iters,
                float* codebook, void* workspace, size_t workspace_bytes, void* stream);

/* code[i][m] = nearest sub-codeword of the residual.  Replaces
 * encode_residuals_to_pq_gpu (kmeans_gpu.cuh:450-508). */
int fg_pq_encode(const float* data, int64_t n, int32_t dim, const int32_t* assign,
                 const float* centroids, const float* codebook, int32_t pq_m, uint8_t* codes,
                 void* stream);

/* Gather codes into list order: out_codes[r] = codes[order[r]] (rows of pq_m
 * bytes), out_ids[r] = order[r].  Replaces build_global.cu:226-240. */
int fg_gather_lists(const uint8_t* codes, int64_t n, int32_t pq_m, const int32_t* order,
                    uint8_t* out_codes, int32_t* out_ids, void* stream);

/* List rebalancing: replaces build_global.cu:62-169.  With avg = n/k, every
 * list longer than (size_t)(2*avg) and not shorter than 32 points is split
 * into sub_k = clamp(ceil(len/avg), 2, len/2) lists by fg_kmeans on its
 * points (`iters` steps, `seed`; the reference uses 15 and 42) and
 * fg_assign; the children go to the back of a FIFO queue that starts with the
 * non-empty input lists in order, and a list leaves the queue as final when it
 * is small enough.  Final lists are numbered in the order they leave the
 * queue.  A split whose points all land in one child ends there (the
 * reference would repeat it forever).  out_assign [n] (may alias assign) and
 * out_centroids [cap][dim] are device memory; *out_nlist (host) receives the
 * list count, also when it exceeds cap (then FG_ERR_WORKSPACE and nothing is
 * written: call again with cap >= *out_nlist).  Synchronises the stream; the
 * control loop runs on the host and allocates its own device scratch. */
int fg_rebalance(const float* data, int64_t n, int32_t dim, const int32_t* assign,
                 const float* centroids, int32_t k, int32_t iters, uint32_t seed,
                 int32_t* out_assign, float* out_centroids, int32_t cap, int32_t* out_nlist,
                 void* stream);

/* Exact k nearest base vectors (ground truth), ascending by (distance, id). */
int fg_knn_workspace_size(int64_t nbase, int32_t dim, int32_t nq, int32_t k, size_t* bytes);
int fg_knn_exact(const float* base, int64_t nbase, int32_t dim, const float* queries, int32_t nq,
                 int32_t k, int32_t* out_ids, float* out_dists, void* workspace,
                 size_t workspace_bytes, void* stream);
/* The same with a metric: FG_METRIC_IP ranks by -(q . x) (sum of fmaf in
 * dimension order, negated), written to out_dists. */
int fg_knn(const float* base, int64_t nbase, int32_t dim, const float* queries, int32_t nq,
           int32_t k, int32_t metric, int32_t* out_ids, float* out_dists, void* workspace,
           size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif
#endif
