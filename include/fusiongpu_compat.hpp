// fusiongpu_compat.hpp -- the reference's C++ entry points, with their exact
// signatures, implemented over the C ABI of fusiongpu.h.
//
// Drop-in use in a FusionGPU build: compile gpu_global.cu's callers
// (search_pipeline.cu, build_global.cu) against this header instead of linking
// gpu_global.cu and kmeans_gpu.cuh.  In exactly one translation unit define
// FG_COMPAT_IMPLEMENTATION before including it.  DIM and PQ_M come from the
// reference's defs.h when it was included first; otherwise from -D flags (the
// defaults below mirror defs.h:9-12).
//
// Replaced functions (Hello-day/FusionGPU):
//   run_gpu_batch_logic           gpu_global.cu:679-874
//   run_gpu_rerank                gpu_global.cu:667-673
//   run_kmeans_gpu                kmeans_gpu.cuh:234-324
//   gpu_assign_initial_clusters   kmeans_gpu.cuh:329-362
//   gpu_assign_to_centroids       kmeans_gpu.cuh:367-394
//   encode_residuals_to_pq_gpu    kmeans_gpu.cuh:450-508
//   train_residual_pq_codebooks   pq_utils.h:77-138 (host CPU there, GPU here)
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "fusiongpu.h"

#ifndef DEFS_H_
// The reference's defs.h was not included: declare its names here with the
// same members and order (defs.h:9-12, 49-79), since callers refer to them.
#ifndef DIM
#define DIM 128
#endif
#ifndef PQ_M
#define PQ_M 32
#endif
#ifndef PQ_K
#define PQ_K 256
#endif
#ifndef PQ_SUB_DIM
#define PQ_SUB_DIM (DIM / PQ_M)
#endif
struct IVFIndexGPU {
    float* d_pq_codebook;
    int* d_cluster_offsets;
    uint8_t* d_all_pq_codes;
    int* d_all_vector_ids;
    float* d_centroids;
    int num_clusters;
};
struct BatchLogicEvents {
    cudaEvent_t evt_start, evt_prune_count, evt_precompute_p1, evt_precompute, evt_scan_offset, evt_resize_sync,
        evt_scan_phase1_end, evt_d2h_p1_start, evt_d2h_p1_end, evt_precompute_p2, evt_h2d_threshold, evt_scan_cand,
        evt_compact, evt_sort, evt_gather;
};
template <typename T>
struct point_t {
    T coordinates[DIM];
};
#endif

// Candidate generation with the reference's arguments and results
// (ref_compat).  Written as the reference writes them: d_top_ids/d_top_dists
// [bs][rerank_m] (ranks >= 128 as id 0 / distance 0, the values the
// reference's 128-thread gather leaves in freshly zeroed buffers),
// d_top_counts, d_atomic (candidates per query), d_counts and d_offsets
// [bs+1] (the per-query budget and its scan, d_offsets[bs] = batch total).
// The flat pools, the global LUT buffer, the cutoff/threshold/compact buffers
// and pool_cap are accepted and not used (the fused kernel needs no scratch);
// the probe list is not pruned in place, and the host is never blocked.
// Events, when given, bracket the budget and the fused kernel.
void run_gpu_batch_logic(const IVFIndexGPU& idx, float* d_queries, uint32_t* d_cagra_top_m, float* d_cagra_dists,
                         float* d_global_tables, int*& d_flat_ids, float*& d_flat_dists, int*& d_flat_ids_alt,
                         float*& d_flat_dists_alt, size_t& current_pool_cap, int* d_counts, int* d_offsets,
                         int* d_atomic, int* d_top_ids, float* d_top_dists, int* d_top_counts, int batch_size,
                         int top_m, int rerank_m, int final_k, float prune_ratio, float* d_list_cutoffs,
                         float* d_thresholds, int* d_compact_offsets, cudaStream_t stream_main,
                         BatchLogicEvents* events, int p1_lists, int limit_k, float threshold_coeff);

// Exact rerank with the reference's arguments (one launch instead of
// ceil(rm/mb)); d_stable_cnt and d_finished are not used.
void run_gpu_rerank(float* d_queries, int* d_top_ids, int* d_top_counts, float* d_base_vecs, int* d_final_ids,
                    float* d_final_dists, int* d_stable_cnt, bool* d_finished, int batch_size, int rerank_m,
                    int final_k, int total_vecs, int mini_batch_size, float epsilon, int beta, cudaStream_t stream);

// Build helpers on host arrays, as the reference's (synchronous).
void run_kmeans_gpu(const float* h_data, int n, int dim, int k, std::vector<float>& h_centroids, int max_iter = 20);
void gpu_assign_to_centroids(const float* h_data, const float* h_centroids, int n, int dim, int k,
                             std::vector<int>& assignments);
void gpu_assign_initial_clusters(const float* h_data, const float* h_centroids, int n, int dim, int k,
                                 std::vector<std::vector<int>>& buckets);
void encode_residuals_to_pq_gpu(const float* h_data, int n, int dim, const std::vector<int>& h_cluster_ids,
                                const std::vector<float>& h_centroids, const std::vector<float>& h_codebook,
                                uint8_t* h_codes, int pq_m, int pq_k, int sub_dim);
void train_residual_pq_codebooks(const point_t<float>* points, int n, const std::vector<int>& vec_cluster_ids,
                                 const std::vector<float>& clusters, std::vector<float>& codebook,
                                 int sample_size = 50000, int max_iter = 8);

// Errors: the reference ignores them; these print fg_last_error() to stderr
// and leave the outputs unwritten.  fg_compat_last_status() returns the status
// of the most recent call on this thread.
int fg_compat_last_status();

#ifdef FG_COMPAT_IMPLEMENTATION
#include <cstdio>

namespace fg_compat_detail {
inline thread_local int g_status = FG_OK;
inline bool ok(int rc, const char* what) {
    g_status = rc;
    if (rc != FG_OK) std::fprintf(stderr, "%s: %s\n", what, fg_last_error());
    return rc == FG_OK;
}
struct DevBuf {
    void* p = nullptr;
    explicit DevBuf(size_t n) {
        if (n && cudaMalloc(&p, n) != cudaSuccess) p = nullptr;
    }
    ~DevBuf() {
        if (p) cudaFree(p);
    }
    template <class T>
    T* as() const { return static_cast<T*>(p); }
};
inline fg_search_params ref_params(int top_m, int rerank_m, int final_k, float prune_ratio, int p1, int limit_k,
                                   float coeff) {
    fg_search_params p;
    fg_search_params_default(&p);
    p.top_m = top_m;
    p.rerank_m = rerank_m;
    p.final_k = final_k;
    p.prune_ratio = prune_ratio;
    p.p1_lists = p1;
    p.limit_k = limit_k;
    p.threshold_coeff = coeff;
    p.ref_compat = 1;
    return p;
}
}  // namespace fg_compat_detail

int fg_compat_last_status() { return fg_compat_detail::g_status; }

void run_gpu_batch_logic(const IVFIndexGPU& idx, float* d_queries, uint32_t* d_cagra_top_m, float* d_cagra_dists,
                         float*, int*&, float*&, int*&, float*&, size_t&, int* d_counts, int* d_offsets, int* d_atomic,
                         int* d_top_ids,
                         float* d_top_dists, int* d_top_counts, int batch_size, int top_m, int rerank_m, int final_k,
                         float prune_ratio, float*, float*, int*, cudaStream_t stream_main, BatchLogicEvents* events,
                         int p1_lists, int limit_k, float threshold_coeff) {
    using namespace fg_compat_detail;
    // ref_compat clamps phase-1 lists at 1024 vectors, so 1024 bounds the
    // per-list scratch whatever the longest list is.
    fg_ivfpq_view v{idx.d_pq_codebook, idx.d_cluster_offsets, idx.d_all_pq_codes, idx.d_all_vector_ids,
                    idx.d_centroids, idx.num_clusters, DIM, PQ_M, 0, 1024};
    const fg_search_params p = ref_params(top_m, rerank_m, final_k, prune_ratio, p1_lists, limit_k, threshold_coeff);
    if (events) cudaEventRecord(events->evt_start, stream_main);
    if (d_counts &&
        !ok(fg_probe_budget(idx.d_cluster_offsets, idx.num_clusters, d_cagra_top_m, d_cagra_dists, batch_size, top_m,
                            prune_ratio, d_counts, d_offsets, stream_main),
            "run_gpu_batch_logic"))
        return;
    ok(fg_batch_logic(&v, d_queries, batch_size, d_cagra_top_m, d_cagra_dists, &p, d_top_ids, d_top_dists,
                      d_top_counts, d_atomic, stream_main),
       "run_gpu_batch_logic");
    if (events) {
        for (cudaEvent_t e : {events->evt_prune_count, events->evt_precompute, events->evt_scan_offset,
                              events->evt_resize_sync, events->evt_scan_phase1_end, events->evt_scan_cand,
                              events->evt_compact, events->evt_sort, events->evt_gather})
            cudaEventRecord(e, stream_main);
    }
}

void run_gpu_rerank(float* d_queries, int* d_top_ids, int* d_top_counts, float* d_base_vecs, int* d_final_ids,
                    float* d_final_dists, int*, bool*, int batch_size, int rerank_m, int final_k, int total_vecs,
                    int mini_batch_size, float epsilon, int beta, cudaStream_t stream) {
    using namespace fg_compat_detail;
    fg_search_params p = ref_params(1, rerank_m, final_k, 100.0f, 0, 1, 1.0f);
    p.mini_batch = mini_batch_size;
    p.epsilon = epsilon;
    p.beta = beta;
    ok(fg_rerank(d_queries, batch_size, DIM, d_top_ids, d_top_counts, d_base_vecs, total_vecs, &p, d_final_ids,
                 d_final_dists, stream),
       "run_gpu_rerank");
}

void run_kmeans_gpu(const float* h_data, int n, int dim, int k, std::vector<float>& h_centroids, int max_iter) {
    using namespace fg_compat_detail;
    size_t wsb = 0;
    if (!ok(fg_kmeans_workspace_size(n, dim, k, &wsb), "run_kmeans_gpu")) return;
    DevBuf x((size_t)n * dim * 4), c((size_t)k * dim * 4), ws(wsb);
    cudaMemcpy(x.p, h_data, (size_t)n * dim * 4, cudaMemcpyHostToDevice);
    if (!ok(fg_kmeans(x.as<float>(), n, dim, k, max_iter, 42, c.as<float>(), ws.p, wsb, nullptr), "run_kmeans_gpu"))
        return;
    h_centroids.resize((size_t)k * dim);
    cudaMemcpy(h_centroids.data(), c.p, (size_t)k * dim * 4, cudaMemcpyDeviceToHost);
}

void gpu_assign_to_centroids(const float* h_data, const float* h_centroids, int n, int dim, int k,
                             std::vector<int>& assignments) {
    using namespace fg_compat_detail;
    size_t wb = 0;
    if (!ok(fg_assign_workspace_size(n, dim, k, &wb), "gpu_assign_to_centroids")) return;
    DevBuf x((size_t)n * dim * 4), c((size_t)k * dim * 4), a((size_t)n * 4), ws(wb ? wb : 256);
    cudaMemcpy(x.p, h_data, (size_t)n * dim * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(c.p, h_centroids, (size_t)k * dim * 4, cudaMemcpyHostToDevice);
    if (!ok(fg_assign(x.as<float>(), n, dim, c.as<float>(), k, a.as<int32_t>(), ws.p, wb, nullptr),
            "gpu_assign_to_centroids"))
        return;
    assignments.resize(n);
    cudaMemcpy(assignments.data(), a.p, (size_t)n * 4, cudaMemcpyDeviceToHost);
}

void gpu_assign_initial_clusters(const float* h_data, const float* h_centroids, int n, int dim, int k,
                                 std::vector<std::vector<int>>& buckets) {
    std::vector<int> a;
    gpu_assign_to_centroids(h_data, h_centroids, n, dim, k, a);
    buckets.assign(k, {});
    for (int i = 0; i < (int)a.size(); ++i) buckets[a[i]].push_back(i);
}

void encode_residuals_to_pq_gpu(const float* h_data, int n, int dim, const std::vector<int>& h_cluster_ids,
                                const std::vector<float>& h_centroids, const std::vector<float>& h_codebook,
                                uint8_t* h_codes, int pq_m, int, int) {
    using namespace fg_compat_detail;
    DevBuf x((size_t)n * dim * 4), a((size_t)n * 4), c(h_centroids.size() * 4), cb(h_codebook.size() * 4),
        out((size_t)n * pq_m);
    cudaMemcpy(x.p, h_data, (size_t)n * dim * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(a.p, h_cluster_ids.data(), (size_t)n * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(c.p, h_centroids.data(), h_centroids.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(cb.p, h_codebook.data(), h_codebook.size() * 4, cudaMemcpyHostToDevice);
    if (!ok(fg_pq_encode(x.as<float>(), n, dim, a.as<int32_t>(), c.as<float>(), cb.as<float>(), pq_m,
                         out.as<uint8_t>(), nullptr),
            "encode_residuals_to_pq_gpu"))
        return;
    cudaMemcpy(h_codes, out.p, (size_t)n * pq_m, cudaMemcpyDeviceToHost);
}

void train_residual_pq_codebooks(const point_t<float>* points, int n, const std::vector<int>& vec_cluster_ids,
                                 const std::vector<float>& clusters, std::vector<float>& codebook, int sample_size,
                                 int max_iter) {
    using namespace fg_compat_detail;
    const int dim = DIM, pq_m = PQ_M;
    size_t wsb = 0;
    if (!ok(fg_pq_train_workspace_size(n, dim, pq_m, sample_size, &wsb), "train_residual_pq_codebooks")) return;
    DevBuf x((size_t)n * dim * 4), a((size_t)n * 4), c(clusters.size() * 4), cb((size_t)pq_m * 256 * (dim / pq_m) * 4),
        ws(wsb);
    cudaMemcpy(x.p, points, (size_t)n * dim * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(a.p, vec_cluster_ids.data(), (size_t)n * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(c.p, clusters.data(), clusters.size() * 4, cudaMemcpyHostToDevice);
    if (!ok(fg_pq_train(x.as<float>(), n, dim, a.as<int32_t>(), c.as<float>(), pq_m, sample_size, max_iter,
                        cb.as<float>(), ws.p, wsb, nullptr),
            "train_residual_pq_codebooks"))
        return;
    codebook.resize((size_t)pq_m * 256 * (dim / pq_m));
    cudaMemcpy(codebook.data(), cb.p, codebook.size() * 4, cudaMemcpyDeviceToHost);
}
#endif  // FG_COMPAT_IMPLEMENTATION
