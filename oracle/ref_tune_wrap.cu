/*
 * ref_tune_wrap.cu -- TEST INFRASTRUCTURE ONLY.
 *
 * Compiles the reference's tuner (tune_parameters.cu, included by path through
 * REF_SRC) and exposes, behind a plain C ABI:
 *   ref_elbow / ref_percentile_int  its host statistics (find_elbow_point,
 *                                   compute_percentile_int), callable on a CPU;
 *   ref_tune_sample                 the sample rows its tuner draws for a seed;
 *   ref_tune                        tune_search_parameters itself (needs a GPU).
 * The reference seeds its sampler from std::random_device; here that name is
 * bound to a generator returning a fixed seed so that runs repeat.  Its CAGRA
 * header (unused by the tuner, and needing RAFT) is skipped by defining its
 * include guard, and its main() is renamed.
 */
#include "ref_defs.h"

#include <cstring>
#include <iomanip>
#include <random>

static unsigned g_ref_tune_seed = 0;
namespace std {
struct fg_ref_seeded_device {
    unsigned operator()() { return g_ref_tune_seed; }
};
}  // namespace std

#define CAGRA_ADAPTER_CUH
#define random_device fg_ref_seeded_device
#define main ref_tune_main
#include REF_SRC
#undef main
#undef random_device

extern "C" int ref_elbow(const int* hits, int n, int total, float* coverage) {
    std::vector<int> h(hits, hits + n);
    ElbowAnalysisResult r = find_elbow_point(h, total);
    *coverage = r.coverage_at_elbow;
    return r.elbow_point;
}

extern "C" int ref_percentile_int(const int* data, int n, float p) {
    std::vector<int> v(data, data + n);
    return compute_percentile_int(v, p);
}

extern "C" void ref_tune_sample(unsigned seed, int n_base, int n_samples, int* out) {
    std::mt19937 gen(seed);
    std::uniform_int_distribution<> dis(0, n_base - 1);
    for (int i = 0; i < n_samples; ++i) out[i] = dis(gen);
}

/* out_i = {top_m, p1_lists, limit_k, n_cluster_ranks, n_pq_ranks, n_ratios};
 * cluster_ranks / pq_ranks / exact_ranks hold n_samples*final_k entries at
 * most, ratios n_samples, all in the reference's push order. */
extern "C" int ref_tune(const float* base, int n_base, const float* centroids, int n_clusters, const int* offsets,
                        const int* ids, const uint8_t* codes, const float* codebook, int n_samples, int final_k,
                        unsigned seed, int* out_i, float* out_coeff, int* cluster_ranks, int* pq_ranks,
                        int* exact_ranks, float* ratios) {
    g_ref_tune_seed = seed;
    TuneConfig cfg;
    cfg.n_samples = n_samples;
    cfg.final_k = final_k;
    TuneResults r = tune_search_parameters(base, n_base, centroids, n_clusters, offsets, ids, codes, codebook, cfg);
    out_i[0] = r.recommended_top_m;
    out_i[1] = r.recommended_p1_lists;
    out_i[2] = r.recommended_limit_k;
    out_i[3] = (int)r.cluster_ranks.size();
    out_i[4] = (int)r.pq_ranks.size();
    out_i[5] = (int)r.pq_ratios.size();
    *out_coeff = r.threshold_coeff;
    std::memcpy(cluster_ranks, r.cluster_ranks.data(), r.cluster_ranks.size() * sizeof(int));
    std::memcpy(pq_ranks, r.pq_ranks.data(), r.pq_ranks.size() * sizeof(int));
    std::memcpy(exact_ranks, r.exact_ranks.data(), r.exact_ranks.size() * sizeof(int));
    std::memcpy(ratios, r.pq_ratios.data(), r.pq_ratios.size() * sizeof(float));
    return cudaGetLastError() == cudaSuccess ? 0 : 1;
}
