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

/* ---- timing context: the caller-owned buffers of SearchPipeline's BatchCtx
 * (search_pipeline.cu:179-211), allocated once for batches of up to `bs`
 * queries with up to `top_m` probes, so that repeated searches time only
 * what the reference runs per batch: run_gpu_batch_logic (with its two host
 * waits) followed by run_gpu_rerank, on the context's stream.  The
 * reference's function-static scratch (gpu_global.cu:699-700) is shared by
 * every stream, so contexts must not run concurrently. */
struct RefCtx {
    int bs = 0, top_m = 0, rerank_m = 0, final_k = 0, p1 = 1;
    cudaStream_t s = nullptr;
    float* tables = nullptr;
    int *counts = nullptr, *offs = nullptr, *atomic = nullptr, *coffs = nullptr;
    float *cutoffs = nullptr, *thr = nullptr;
    int *fid = nullptr, *fid_alt = nullptr;
    float *fd = nullptr, *fd_alt = nullptr;
    size_t cap = 0;
    uint32_t* probes = nullptr;  // per-call copy: the prune step rewrites the probe list in place
    int *top_ids = nullptr, *top_counts = nullptr, *stable = nullptr;
    float* top_dists = nullptr;
    bool* fin = nullptr;
};

extern "C" void ref_ctx_destroy(void* h) {
    RefCtx* c = static_cast<RefCtx*>(h);
    if (!c) return;
    if (c->s) cudaStreamSynchronize(c->s);
    cudaFree(c->tables); cudaFree(c->counts); cudaFree(c->offs); cudaFree(c->atomic); cudaFree(c->coffs);
    cudaFree(c->cutoffs); cudaFree(c->thr); cudaFree(c->fid); cudaFree(c->fd); cudaFree(c->fid_alt);
    cudaFree(c->fd_alt); cudaFree(c->probes); cudaFree(c->top_ids); cudaFree(c->top_dists);
    cudaFree(c->top_counts); cudaFree(c->stable); cudaFree(c->fin);
    if (c->s) cudaStreamDestroy(c->s);
    delete c;
}

/* Returns the context, or null when an allocation fails. */
extern "C" void* ref_ctx_create(int bs, int top_m, int rerank_m, int final_k, int p1_lists) {
    RefCtx* c = new RefCtx;
    c->bs = bs; c->top_m = top_m; c->rerank_m = rerank_m; c->final_k = final_k;
    c->p1 = p1_lists > 0 ? p1_lists : 1;
    c->cap = (size_t)bs * 2000;  // SearchPipeline's initial pool (search_pipeline.cu:166)
    bool ok = cudaStreamCreateWithFlags(&c->s, cudaStreamNonBlocking) == cudaSuccess;
    ok = ok && cudaMalloc(&c->tables, (size_t)bs * top_m * PQ_M * PQ_K * sizeof(float)) == cudaSuccess;
    ok = ok && cudaMalloc(&c->counts, bs * sizeof(int)) == cudaSuccess;
    ok = ok && cudaMalloc(&c->offs, (bs + 1) * sizeof(int)) == cudaSuccess;
    ok = ok && cudaMalloc(&c->atomic, bs * sizeof(int)) == cudaSuccess;
    ok = ok && cudaMalloc(&c->coffs, (bs + 1) * sizeof(int)) == cudaSuccess;
    ok = ok && cudaMalloc(&c->cutoffs, (size_t)bs * c->p1 * sizeof(float)) == cudaSuccess;
    ok = ok && cudaMalloc(&c->thr, bs * sizeof(float)) == cudaSuccess;
    ok = ok && cudaMalloc(&c->fid, c->cap * sizeof(int)) == cudaSuccess;
    ok = ok && cudaMalloc(&c->fd, c->cap * sizeof(float)) == cudaSuccess;
    ok = ok && cudaMalloc(&c->fid_alt, c->cap * sizeof(int)) == cudaSuccess;
    ok = ok && cudaMalloc(&c->fd_alt, c->cap * sizeof(float)) == cudaSuccess;
    ok = ok && cudaMalloc(&c->probes, (size_t)bs * top_m * sizeof(uint32_t)) == cudaSuccess;
    // zeroed like SearchPipeline's cudaMalloc'd top arrays on a fresh device
    ok = ok && cudaMalloc(&c->top_ids, (size_t)bs * rerank_m * sizeof(int)) == cudaSuccess;
    ok = ok && cudaMalloc(&c->top_dists, (size_t)bs * rerank_m * sizeof(float)) == cudaSuccess;
    ok = ok && cudaMalloc(&c->top_counts, bs * sizeof(int)) == cudaSuccess;
    ok = ok && cudaMalloc(&c->stable, bs * sizeof(int)) == cudaSuccess;
    ok = ok && cudaMalloc(&c->fin, bs * sizeof(bool)) == cudaSuccess;
    ok = ok && cudaMemset(c->top_ids, 0, (size_t)bs * rerank_m * sizeof(int)) == cudaSuccess;
    ok = ok && cudaMemset(c->top_dists, 0, (size_t)bs * rerank_m * sizeof(float)) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        ref_ctx_destroy(c);
        return nullptr;
    }
    return c;
}

extern "C" void* ref_ctx_stream(void* h) { return static_cast<RefCtx*>(h)->s; }

/* One reference batch: copy the probe list, run_gpu_batch_logic, then
 * run_gpu_rerank into final_ids/final_dists [nq][final_k] (device).  nq <=
 * the context's bs, top_m <= its top_m.  Returns a CUDA error code (0 = ok;
 * -1 = a shape beyond the context). */
extern "C" int ref_ctx_search(void* h, const float* codebook, const int* offsets, const uint8_t* codes,
                              const int* vec_ids, const float* centroids, int nlist, const float* base,
                              int total_vecs, float* queries, const uint32_t* probe_ids, float* probe_dists,
                              int nq, int top_m, float prune_ratio, int p1_lists, int limit_k,
                              float threshold_coeff, int mini_batch, float eps, int beta, int* final_ids,
                              float* final_dists, int* out_candidate_counts) {
    RefCtx* c = static_cast<RefCtx*>(h);
    if (!c || nq > c->bs || top_m > c->top_m || (p1_lists > 0 ? p1_lists : 1) > c->p1) return -1;
    IVFIndexGPU idx;
    idx.d_pq_codebook = const_cast<float*>(codebook);
    idx.d_cluster_offsets = const_cast<int*>(offsets);
    idx.d_all_pq_codes = const_cast<uint8_t*>(codes);
    idx.d_all_vector_ids = const_cast<int*>(vec_ids);
    idx.d_centroids = const_cast<float*>(centroids);
    idx.num_clusters = nlist;
    cudaMemcpyAsync(c->probes, probe_ids, (size_t)nq * top_m * sizeof(uint32_t), cudaMemcpyDeviceToDevice, c->s);
    run_gpu_batch_logic(idx, queries, c->probes, probe_dists, c->tables, c->fid, c->fd, c->fid_alt, c->fd_alt,
                        c->cap, c->counts, c->offs, c->atomic, c->top_ids, c->top_dists, c->top_counts, nq,
                        top_m, c->rerank_m, c->final_k, prune_ratio, c->cutoffs, c->thr, c->coffs, c->s, nullptr,
                        p1_lists, limit_k, threshold_coeff);
    if (out_candidate_counts)
        cudaMemcpyAsync(out_candidate_counts, c->atomic, nq * sizeof(int), cudaMemcpyDeviceToDevice, c->s);
    run_gpu_rerank(queries, c->top_ids, c->top_counts, const_cast<float*>(base), final_ids, final_dists, c->stable,
                   c->fin, nq, c->rerank_m, c->final_k, total_vecs, mini_batch, eps, beta, c->s);
    return (int)cudaGetLastError();
}
