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
