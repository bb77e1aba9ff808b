/*
 * ref_gpu_global_wrap.cu -- TEST INFRASTRUCTURE ONLY.
 *
 * Compiles the reference's search kernels (gpu_global.cu, included by path
 * through REF_SRC) and exposes its two entry points, run_gpu_batch_logic
 * (gpu_global.cu:679-874) and run_gpu_rerank (gpu_global.cu:667-673), behind a
 * plain C ABI so that the parity tests can run the reference's own code on
 * the GPU and pin the CPU oracle against it.  The wrapper owns the scratch
 * buffers the reference expects its caller (SearchPipeline, search_pipeline.cu
 * :179-211) to allocate.
 */
#include "ref_defs.h"
#include REF_SRC

#include <cstring>

extern "C" int ref_gg_dim(void) { return DIM; }
extern "C" int ref_gg_pq_m(void) { return PQ_M; }

/* All pointers are device pointers.  probe_ids is modified in place (prune).
 * top_ids/top_dists must be [bs][rerank_m]; entries the reference does not
 * write keep their previous contents. */
extern "C" int ref_run_batch_logic(const float* codebook, const int* offsets, const uint8_t* codes,
                                   const int* vec_ids, const float* centroids, int nlist,
                                   float* queries, uint32_t* probe_ids, float* probe_dists,
                                   int bs, int top_m, int rerank_m, int final_k, float prune_ratio,
                                   int p1_lists, int limit_k, float threshold_coeff,
                                   int* top_ids, float* top_dists, int* top_counts,
                                   int* out_candidate_counts) {
    IVFIndexGPU idx;
    idx.d_pq_codebook = const_cast<float*>(codebook);
    idx.d_cluster_offsets = const_cast<int*>(offsets);
    idx.d_all_pq_codes = const_cast<uint8_t*>(codes);
    idx.d_all_vector_ids = const_cast<int*>(vec_ids);
    idx.d_centroids = const_cast<float*>(centroids);
    idx.num_clusters = nlist;

    float* tables = nullptr;
    int *counts = nullptr, *offs = nullptr, *atomic = nullptr, *coffs = nullptr;
    float *cutoffs = nullptr, *thr = nullptr;
    int *fid = nullptr, *fid_alt = nullptr;
    float *fd = nullptr, *fd_alt = nullptr;
    size_t cap = (size_t)bs * 2000;  // SearchPipeline's initial pool (search_pipeline.cu:166)
    int p1 = p1_lists > 0 ? p1_lists : 1;
    cudaMalloc(&tables, (size_t)bs * top_m * PQ_M * PQ_K * sizeof(float));
    cudaMalloc(&counts, bs * sizeof(int));
    cudaMalloc(&offs, (bs + 1) * sizeof(int));
    cudaMalloc(&atomic, bs * sizeof(int));
    cudaMalloc(&coffs, (bs + 1) * sizeof(int));
    cudaMalloc(&cutoffs, (size_t)bs * p1 * sizeof(float));
    cudaMalloc(&thr, bs * sizeof(float));
    cudaMalloc(&fid, cap * sizeof(int));
    cudaMalloc(&fd, cap * sizeof(float));
    cudaMalloc(&fid_alt, cap * sizeof(int));
    cudaMalloc(&fd_alt, cap * sizeof(float));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return (int)e;

    cudaStream_t s;
    cudaStreamCreate(&s);
    run_gpu_batch_logic(idx, queries, probe_ids, probe_dists, tables, fid, fd, fid_alt, fd_alt, cap,
                        counts, offs, atomic, top_ids, top_dists, top_counts, bs, top_m, rerank_m,
                        final_k, prune_ratio, cutoffs, thr, coffs, s, nullptr, p1_lists, limit_k,
                        threshold_coeff);
    if (out_candidate_counts)
        cudaMemcpyAsync(out_candidate_counts, atomic, bs * sizeof(int), cudaMemcpyDeviceToDevice, s);
    e = cudaStreamSynchronize(s);
    cudaStreamDestroy(s);
    cudaFree(tables); cudaFree(counts); cudaFree(offs); cudaFree(atomic); cudaFree(coffs);
    cudaFree(cutoffs); cudaFree(thr); cudaFree(fid); cudaFree(fd); cudaFree(fid_alt); cudaFree(fd_alt);
    if (e == cudaSuccess) e = cudaGetLastError();
    return (int)e;
}

extern "C" int ref_run_rerank(float* queries, int* top_ids, int* top_counts, float* base,
                              int* final_ids, float* final_dists, int bs, int rerank_m, int final_k,
                              int total_vecs, int mini_batch, float eps, int beta) {
    int* stable = nullptr;
    bool* fin = nullptr;
    cudaMalloc(&stable, bs * sizeof(int));
    cudaMalloc(&fin, bs * sizeof(bool));
    cudaStream_t s;
    cudaStreamCreate(&s);
    run_gpu_rerank(queries, top_ids, top_counts, base, final_ids, final_dists, stable, fin, bs,
                   rerank_m, final_k, total_vecs, mini_batch, eps, beta, s);
    cudaError_t e = cudaStreamSynchronize(s);
    cudaStreamDestroy(s);
    cudaFree(stable);
    cudaFree(fin);
    if (e == cudaSuccess) e = cudaGetLastError();
    return (int)e;
}
