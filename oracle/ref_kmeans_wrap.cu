/*
 * ref_kmeans_wrap.cu -- TEST INFRASTRUCTURE ONLY.
 *
 * Compiles the reference's GPU k-means and PQ encoder (kmeans_gpu.cuh,
 * included by path through REF_SRC; cuBLAS SGEMM for the assignment) behind a
 * plain C ABI, so the GPU tests can compare the product's assignment, centroid
 * update and encoder with the reference's own on the same data.  All pointers
 * are host pointers, as in the reference's functions.  The reference exits the
 * process on a CUDA error (its CUDA_CHECK).
 */
#include <vector>

#include REF_SRC

/* run_kmeans_gpu (kmeans_gpu.cuh:234-324): strided MT19937(42) seeding, then
 * max_iter Lloyd steps; centroids_out [k][dim]. */
extern "C" int ref_run_kmeans(const float* data, int n, int dim, int k, int max_iter, float* centroids_out) {
    std::vector<float> c;
    run_kmeans_gpu(data, n, dim, k, c, max_iter);
    std::copy(c.begin(), c.end(), centroids_out);
    return 0;
}

/* gpu_assign_to_centroids (kmeans_gpu.cuh:367-394) */
extern "C" int ref_assign(const float* data, const float* centroids, int n, int dim, int k, int* out) {
    std::vector<int> a;
    gpu_assign_to_centroids(data, centroids, n, dim, k, a);
    std::copy(a.begin(), a.end(), out);
    return 0;
}

/* encode_residuals_to_pq_gpu (kmeans_gpu.cuh:450-508) */
extern "C" int ref_encode(const float* data, int n, int dim, const int* ids, const float* centroids, int ncent,
                          const float* codebook, int pq_m, unsigned char* codes) {
    std::vector<int> vid(ids, ids + n);
    std::vector<float> cen(centroids, centroids + (size_t)ncent * dim);
    std::vector<float> cb(codebook, codebook + (size_t)pq_m * 256 * (dim / pq_m));
    encode_residuals_to_pq_gpu(data, n, dim, vid, cen, cb, codes, pq_m, 256, dim / pq_m);
    return 0;
}

/* releases the reference's process-global k-means context (kmeans_gpu.cuh:192) */
extern "C" void ref_kmeans_cleanup(void) { cleanup_kmeans_gpu(); }
