/*
 * ref_defs.h -- TEST INFRASTRUCTURE ONLY.
 *
 * Stands in for the reference's defs.h so that its sources can be compiled
 * from where they lie with other (DIM, PQ_M) than the hard-coded 128/32
 * (defs.h:9-12 are plain #defines, not #ifndef-guarded).  Defining the
 * reference header's include guard first makes its `#include "defs.h"` a
 * no-op; the constants and the three structs below have the same names and
 * member layout as the reference's (defs.h:9-104) because the reference
 * source refers to them by name.
 */
#ifndef FG_REF_DEFS_H
#define FG_REF_DEFS_H
#define DEFS_H_

#include <cstdint>
#include <vector>
#include <cuda_runtime.h>

#ifndef REF_DIM
#error "REF_DIM must be defined"
#endif
#ifndef REF_PQ_M
#error "REF_PQ_M must be defined"
#endif

#define DIM REF_DIM
#define PQ_M REF_PQ_M
#define PQ_K 256
#define PQ_SUB_DIM (DIM / PQ_M)
#ifndef REF_K_CLUSTERS
#define REF_K_CLUSTERS 2048
#endif
#define K_CLUSTERS REF_K_CLUSTERS
#define DEFAULT_BATCH_SIZE 128
#define DEFAULT_TOP_M 20
#define DEFAULT_RERANK_M 10000
#define DEFAULT_P1_LISTS 12
#define DEFAULT_LIMIT_K 50
#define DEFAULT_THRESHOLD_COEFF 1.0f
#define DEFAULT_RERANK_MINI_BATCH 128
#define DEFAULT_RERANK_EPSILON 0.1f
#define DEFAULT_RERANK_BETA 2

using pq_code_t = uint8_t;

template <typename T>
struct point_t {
    T coordinates[DIM];
};

struct IVFIndexGPU {
    float* d_pq_codebook;
    int* d_cluster_offsets;
    uint8_t* d_all_pq_codes;
    int* d_all_vector_ids;
    float* d_centroids;
    int num_clusters;
};

struct BatchLogicEvents {
    cudaEvent_t evt_start, evt_prune_count, evt_precompute_p1, evt_precompute, evt_scan_offset,
        evt_resize_sync, evt_scan_phase1_end, evt_d2h_p1_start, evt_d2h_p1_end, evt_precompute_p2,
        evt_h2d_threshold, evt_scan_cand, evt_compact, evt_sort, evt_gather;
};

struct GPUStageTimings {
    float prune_count_ms = 0, precompute_p1_ms = 0, precompute_ms = 0, scan_offset_ms = 0,
          resize_sync_ms = 0, scan_phase1_ms = 0, d2h_p1_ms = 0, cpu_sort_ms = 0,
          precompute_p2_ms = 0, h2d_threshold_ms = 0, scan_phase2_ms = 0, compact_ms = 0,
          sort_ms = 0, gather_ms = 0, total_ms = 0;
    long long total_candidates = 0, total_max_candidates = 0;
};

#endif
