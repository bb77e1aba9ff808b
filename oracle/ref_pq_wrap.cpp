/*
 * ref_pq_wrap.cpp -- TEST INFRASTRUCTURE ONLY.
 *
 * Compiles the reference's CPU residual-PQ trainer and encoder (pq_utils.h,
 * included by path through REF_SRC) behind a C ABI, so tests can compare the
 * product's codebooks with the reference's own on the same data.
 */
#include "ref_defs.h"
#include REF_SRC

#include <cstring>

extern "C" int ref_pq_dim(void) { return DIM; }
extern "C" int ref_pq_m(void) { return PQ_M; }

/* pq_utils.h:77-138 */
extern "C" int ref_pq_train(const float* data, int n, const int* vec_cluster_ids,
                            const float* clusters, int nclusters, int sample_size, int max_iter,
                            float* codebook_out) {
    std::vector<int> ids(vec_cluster_ids, vec_cluster_ids + n);
    std::vector<float> cl(clusters, clusters + (size_t)nclusters * DIM);
    std::vector<float> cb;
    train_residual_pq_codebooks(reinterpret_cast<const point_t<float>*>(data), n, ids, cl, cb,
                                sample_size, max_iter);
    std::memcpy(codebook_out, cb.data(), cb.size() * sizeof(float));
    return 0;
}

/* pq_utils.h:141-174 */
extern "C" int ref_pq_encode(const float* data, int n, const int* vec_cluster_ids,
                             const float* clusters, int nclusters, const float* codebook,
                             uint8_t* codes) {
    std::vector<int> ids(vec_cluster_ids, vec_cluster_ids + n);
    std::vector<float> cl(clusters, clusters + (size_t)nclusters * DIM);
    std::vector<float> cb(codebook, codebook + (size_t)PQ_M * PQ_K * PQ_SUB_DIM);
    encode_residuals_to_pq(reinterpret_cast<const point_t<float>*>(data), n, ids, cl, cb, codes);
    return 0;
}

/* std::shuffle of 0..n-1 with std::mt19937(seed), the draw pq_utils.h:24-26
 * and :90-93 make, from this compiler's standard library: pins the oracle's
 * restatement of it. */
extern "C" void ref_std_shuffle(int n, unsigned seed, int* out) {
    std::vector<int> v(n);
    std::iota(v.begin(), v.end(), 0);
    std::mt19937 rng(seed);
    std::shuffle(v.begin(), v.end(), rng);
    std::memcpy(out, v.data(), (size_t)n * sizeof(int));
}
