// capi.cu -- the extern "C" entry points declared in include/fusiongpu.h.
#include <algorithm>
#include <cstdarg>
#include <map>
#include <mutex>
#include <string>

#include "fg_common.cuh"

namespace fg {

static thread_local std::string g_err;

void set_error(const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
}

int fail(int status, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return status;
}

int check_launch(const char* what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(FG_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
    return FG_OK;
}

namespace {
std::mutex g_attr_mu;
std::map<std::pair<int, int>, int> g_attr;           // (device, attribute) -> value
std::map<std::pair<int, const void*>, int> g_smem;   // (device, function) -> granted bytes
}  // namespace

int device_attr(cudaDeviceAttr attr) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    std::lock_guard<std::mutex> lk(g_attr_mu);
    const auto key = std::make_pair(dev, (int)attr);
    auto it = g_attr.find(key);
    if (it != g_attr.end()) return it->second;
    int v = 0;
    if (cudaDeviceGetAttribute(&v, attr, dev) != cudaSuccess) return 0;
    g_attr[key] = v;
    return v;
}

cudaError_t ensure_smem(const void* func, int bytes) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lk(g_attr_mu);
    int& granted = g_smem[std::make_pair(dev, func)];
    if (bytes <= granted) return cudaSuccess;
    e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess) granted = bytes;
    return e;
}

// implemented in the kernel files
int batch_logic(const fg_ivfpq_view*, const float*, int, const uint32_t*, const float*, const fg_search_params*,
                int32_t*, float*, int32_t*, int32_t*, cudaStream_t, bool write_pad, int* work_counter = nullptr,
                void* ws = nullptr, size_t ws_bytes = 0);
size_t batch_logic_workspace(const fg_ivfpq_view* ix, const fg_search_params* p, int nq);
int rerank(const float*, int, int, const int32_t*, const int32_t*, const void*, int, long long,
           const fg_search_params*, int32_t*, float*, cudaStream_t);
int knn_like(const float* Y, long long ny, int dim, const float* Q, long long nq, int k, int32_t* out_i,
             float* out_v, void* ws, size_t ws_bytes, cudaStream_t s, int metric = FG_METRIC_L2);
size_t knn_like_workspace(long long nq, int ncols, int k);
int l2_argmin(const float* X, long long nx, const float* Y, int ny, int dim, int32_t* amin, cudaStream_t s);
int kmeans_init(const float* data, int64_t n, int dim, int k, uint32_t seed, float* centroids, int64_t* d_rows,
                cudaStream_t s);
size_t sort_workspace(int64_t n, int k);
int sort_by_list(const int32_t* assign, int64_t n, int k, int32_t* order, int32_t* offsets, void* ws,
                 size_t ws_bytes, cudaStream_t s);
int kmeans_update(const float* data, int dim, const int32_t* order, const int32_t* offsets, int k, float* centroids,
                  cudaStream_t s);
size_t kmeans_workspace(int64_t n, int dim, int k);
int kmeans(const float* data, int64_t n, int dim, int k, int iters, uint32_t seed, float* centroids, void* ws,
           size_t ws_bytes, cudaStream_t s);
size_t pq_train_workspace(int64_t n, int dim, int pq_m, int sample);
int pq_train(const float* data, int64_t n, int dim, const int32_t* assign, const float* centroids, int pq_m,
             int sample, int iters, float* codebook, void* ws, size_t ws_bytes, cudaStream_t s);
int pq_encode(const float* data, int64_t n, int dim, const int32_t* assign, const float* centroids,
              const float* codebook, int pq_m, uint8_t* codes, cudaStream_t s);
int gather_lists(const uint8_t* codes, int64_t n, int pq_m, const int32_t* order, uint8_t* out_codes,
                 int32_t* out_ids, cudaStream_t s);
size_t assign_workspace(long long n, int k, int dim);
int assign_auto(const float* X, long long n, int dim, const float* C, int k, int32_t* out, void* ws, size_t ws_bytes,
                cudaStream_t s);
int probe_budget(const int32_t* list_offsets, int nlist, const uint32_t* probe_ids, const float* probe_dists, int nq,
                 int top_m, float prune_ratio, int32_t* counts, int32_t* offsets, cudaStream_t s);
int rebalance(const float* data, int64_t n, int dim, const int32_t* assign, const float* centroids, int k, int iters,
              uint32_t seed, int32_t* out_assign, float* out_centroids, int cap, int32_t* out_nlist, cudaStream_t s);
bool coarse_tc_supported(int dim, int P);
size_t coarse_tc_workspace(long long nq, int nlist, int dim, int P);
int coarse_tc(const float* centroids, int nlist, int dim, const float* queries, long long nq, int P,
              uint32_t* out_ids, float* out_d, void* ws, size_t ws_bytes, cudaStream_t s, int* n_fallback_host);

// Coarse quantizer dispatch: tensor cores with exact rescoring when the shape
// fits (3*dim <= 384), else exact CUDA-core tiles.
static size_t coarse_workspace(long long nq, int nlist, int dim, int P) {
    size_t b = knn_like_workspace(std::max(nq, 1ll), nlist, P);
    if (coarse_tc_supported(dim, P)) b = std::max(b, coarse_tc_workspace(std::max(nq, 1ll), nlist, dim, P));
    return b;
}

static int coarse(const float* centroids, int nlist, int dim, const float* queries, long long nq, int P,
                  uint32_t* out_ids, float* out_d, void* ws, size_t ws_bytes, cudaStream_t s) {
    if (coarse_tc_supported(dim, P))
        return coarse_tc(centroids, nlist, dim, queries, nq, P, out_ids, out_d, ws, ws_bytes, s, nullptr);
    return knn_like(centroids, nlist, dim, queries, nq, P, reinterpret_cast<int32_t*>(out_ids), out_d, ws,
                    ws_bytes, s);
}

static cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

static int need_ws(void* ws, size_t have, size_t need) {
    if (need == 0) return FG_OK;
    if (!ws) return fail(FG_ERR_WORKSPACE, "workspace is NULL (%zu bytes needed)", need);
    if (!aligned(ws, 256)) return fail(FG_ERR_WORKSPACE, "workspace must be 256-byte aligned");
    if (have < need) return fail(FG_ERR_WORKSPACE, "workspace of %zu bytes < %zu needed", have, need);
    return FG_OK;
}

struct SearchWs {
    uint32_t* pids;
    float* pd;
    int32_t* tid;
    float* td;
    int32_t* tc;
    void* coarse;
    size_t coarse_bytes;
};

static size_t search_fixed_bytes(int nq, const fg_search_params* p) {
    const size_t P = (size_t)p->top_m, R = (size_t)p->rerank_m;
    return round_up((size_t)nq * P * 4, 256) * 2 + round_up((size_t)nq * R * 4, 256) * 2 +
           round_up((size_t)nq * 4, 256) + 256;  // + the scan's query counter
}

}  // namespace fg

using namespace fg;

extern "C" {

const char* fg_version(void) { return "fusiongpu_b200 0.1.0 (sm_100a)"; }

const char* fg_last_error(void) { return g_err.c_str(); }

void fg_search_params_default(fg_search_params* p) {
    if (!p) return;
    p->top_m = 20;
    p->p1_lists = 12;
    p->limit_k = 50;
    p->threshold_coeff = 1.0f;
    p->prune_ratio = 100.0f;
    p->rerank_m = 10000;
    p->final_k = 10;
    p->mini_batch = 128;
    p->epsilon = 0.1f;
    p->beta = 2;
    p->ref_compat = 1;
}

int fg_coarse_workspace_size(int32_t nlist, int32_t dim, int32_t nq, int32_t top_m, size_t* bytes) {
    FG_REQUIRE(bytes, "null bytes");
    FG_REQUIRE(nlist >= 1 && dim >= 1 && nq >= 0 && top_m >= 1 && top_m <= nlist, "bad coarse shape");
    *bytes = coarse_workspace(std::max(nq, 1), nlist, dim, top_m);
    return FG_OK;
}

int fg_coarse_search(const float* centroids, int32_t nlist, int32_t dim, const float* queries, int32_t nq,
                     int32_t top_m, uint32_t* out_ids, float* out_dists, void* ws, size_t ws_bytes,
                     void* stream) {
    FG_REQUIRE(nlist >= 1 && dim >= 1 && nq >= 0, "bad coarse shape");
    FG_REQUIRE(top_m >= 1 && top_m <= nlist && top_m <= 4096, "top_m %d outside [1, min(nlist, 4096)]", top_m);
    if (nq == 0) return FG_OK;
    FG_REQUIRE(centroids && queries && out_ids && out_dists, "null buffer");
    int rc = need_ws(ws, ws_bytes, 1024);
    if (rc) return rc;
    return coarse(centroids, nlist, dim, queries, nq, top_m, out_ids, out_dists, ws, ws_bytes, as_stream(stream));
}

int fg_coarse_search_simt(const float* centroids, int32_t nlist, int32_t dim, const float* queries, int32_t nq,
                          int32_t top_m, uint32_t* out_ids, float* out_dists, void* ws, size_t ws_bytes,
                          void* stream) {
    FG_REQUIRE(nlist >= 1 && dim >= 1 && nq >= 0, "bad coarse shape");
    FG_REQUIRE(top_m >= 1 && top_m <= nlist && top_m <= 4096, "top_m %d outside [1, min(nlist, 4096)]", top_m);
    if (nq == 0) return FG_OK;
    FG_REQUIRE(centroids && queries && out_ids && out_dists, "null buffer");
    int rc = need_ws(ws, ws_bytes, 1024);
    if (rc) return rc;
    return knn_like(centroids, nlist, dim, queries, nq, top_m, reinterpret_cast<int32_t*>(out_ids), out_dists, ws,
                    ws_bytes, as_stream(stream));
}

int fg_coarse_search_tc(const float* centroids, int32_t nlist, int32_t dim, const float* queries, int32_t nq,
                        int32_t top_m, uint32_t* out_ids, float* out_dists, void* ws, size_t ws_bytes,
                        int32_t* n_fallback, void* stream) {
    FG_REQUIRE(nlist >= 1 && dim >= 1 && nq >= 0, "bad coarse shape");
    FG_REQUIRE(top_m >= 1 && top_m <= nlist && top_m <= 4096, "top_m %d outside [1, min(nlist, 4096)]", top_m);
    if (!coarse_tc_supported(dim, top_m))
        return fail(FG_ERR_UNSUPPORTED, "tensor-core coarse path needs 3*dim <= 384 and top_m <= 256");
    if (nq == 0) return FG_OK;
    FG_REQUIRE(centroids && queries && out_ids && out_dists, "null buffer");
    int rc = need_ws(ws, ws_bytes, coarse_tc_workspace(nq, nlist, dim, top_m));
    if (rc) return rc;
    return coarse_tc(centroids, nlist, dim, queries, nq, top_m, out_ids, out_dists, ws, ws_bytes, as_stream(stream),
                     n_fallback);
}

int fg_batch_logic(const fg_ivfpq_view* index, const float* queries, int32_t nq, const uint32_t* probe_ids,
                   const float* probe_dists, const fg_search_params* params, int32_t* top_ids, float* top_dists,
                   int32_t* top_counts, int32_t* candidate_counts, void* stream) {
    return batch_logic(index, queries, nq, probe_ids, probe_dists, params, top_ids, top_dists, top_counts,
                       candidate_counts, as_stream(stream), true);
}

int fg_batch_logic_workspace_size(const fg_ivfpq_view* index, const fg_search_params* params, int32_t nq,
                                  size_t* bytes) {
    FG_REQUIRE(index && params && bytes && nq >= 0, "bad arguments");
    *bytes = batch_logic_workspace(index, params, nq);
    return FG_OK;
}

int fg_batch_logic_ws(const fg_ivfpq_view* index, const float* queries, int32_t nq, const uint32_t* probe_ids,
                      const float* probe_dists, const fg_search_params* params, int32_t* top_ids, float* top_dists,
                      int32_t* top_counts, int32_t* candidate_counts, void* ws, size_t ws_bytes, void* stream) {
    FG_REQUIRE(index && params, "null index or params");
    int rc = need_ws(ws, ws_bytes, batch_logic_workspace(index, params, nq));
    if (rc) return rc;
    return batch_logic(index, queries, nq, probe_ids, probe_dists, params, top_ids, top_dists, top_counts,
                       candidate_counts, as_stream(stream), true, nullptr, ws, ws_bytes);
}

int fg_probe_budget(const int32_t* list_offsets, int32_t nlist, const uint32_t* probe_ids, const float* probe_dists,
                    int32_t nq, int32_t top_m, float prune_ratio, int32_t* counts, int32_t* offsets, void* stream) {
    return probe_budget(list_offsets, nlist, probe_ids, probe_dists, nq, top_m, prune_ratio, counts, offsets,
                        as_stream(stream));
}

int fg_rerank(const float* queries, int32_t nq, int32_t dim, const int32_t* top_ids, const int32_t* top_counts,
              const float* base, int64_t nbase, const fg_search_params* params, int32_t* out_ids, float* out_dists,
              void* stream) {
    return rerank(queries, nq, dim, top_ids, top_counts, base, 0, nbase, params, out_ids, out_dists,
                  as_stream(stream));
}

int fg_rerank_u8(const float* queries, int32_t nq, int32_t dim, const int32_t* top_ids, const int32_t* top_counts,
                 const uint8_t* base, int64_t nbase, const fg_search_params* params, int32_t* out_ids,
                 float* out_dists, void* stream) {
    return rerank(queries, nq, dim, top_ids, top_counts, base, 1, nbase, params, out_ids, out_dists,
                  as_stream(stream));
}

int fg_search_workspace_size(const fg_ivfpq_view* index, const fg_search_params* params, int32_t nq,
                             size_t* bytes) {
    FG_REQUIRE(index && params && bytes, "null argument");
    FG_REQUIRE(nq >= 0 && params->top_m >= 1 && params->top_m <= index->nlist && params->rerank_m >= 1,
               "bad search shape");
    *bytes = search_fixed_bytes(std::max(nq, 1), params) +
             std::max(coarse_workspace(std::max(nq, 1), index->nlist, index->dim, params->top_m),
                      batch_logic_workspace(index, params, std::max(nq, 1))) + 1024;
    return FG_OK;
}

static int search_any(const fg_ivfpq_view* index, const void* base, int base_u8, int64_t nbase, const float* queries,
                      int32_t nq, const fg_search_params* params, int32_t* out_ids, float* out_dists, void* ws,
                      size_t ws_bytes, void* stream) {
    FG_REQUIRE(index && params, "null index or params");
    FG_REQUIRE(nq >= 0, "nq < 0");
    if (nq == 0) return FG_OK;
    FG_REQUIRE(params->top_m >= 1 && params->top_m <= index->nlist, "top_m %d outside [1, nlist=%d]",
               params->top_m, index->nlist);
    int rc = need_ws(ws, ws_bytes, search_fixed_bytes(nq, params) + 1024);
    if (rc) return rc;
    cudaStream_t s = as_stream(stream);
    const size_t P = params->top_m, R = params->rerank_m;
    Carve cv(ws, ws_bytes);
    uint32_t* pids = cv.take<uint32_t>((size_t)nq * P);
    float* pd = cv.take<float>((size_t)nq * P);
    int32_t* tid = cv.take<int32_t>((size_t)nq * R);
    float* td = cv.take<float>((size_t)nq * R);
    int32_t* tc = cv.take<int32_t>((size_t)nq);
    int* qctr = cv.take<int>(4);
    const size_t used = round_up(cv.used, 256);
    if (!cv.ok() || used >= ws_bytes) return fail(FG_ERR_WORKSPACE, "search workspace too small");
    rc = coarse(index->centroids, index->nlist, index->dim, queries, nq, params->top_m, pids, pd,
                static_cast<char*>(ws) + used, ws_bytes - used, s);
    if (rc) return rc;
    // the rerank reads only the first top_counts[q] entries: skip the padding.
    // The coarse scratch is dead once the probes exist: the split scan reuses it.
    FG_CUDA_TRY(cudaMemsetAsync(qctr, 0, sizeof(int), s));
    rc = batch_logic(index, queries, nq, pids, pd, params, tid, td, tc, nullptr, s, false, qctr,
                     static_cast<char*>(ws) + used, ws_bytes - used);
    if (rc) return rc;
    return rerank(queries, nq, index->dim, tid, tc, base, base_u8, nbase, params, out_ids, out_dists, s);
}

int fg_search(const fg_ivfpq_view* index, const float* base, int64_t nbase, const float* queries, int32_t nq,
              const fg_search_params* params, int32_t* out_ids, float* out_dists, void* ws, size_t ws_bytes,
              void* stream) {
    return search_any(index, base, 0, nbase, queries, nq, params, out_ids, out_dists, ws, ws_bytes, stream);
}

int fg_search_u8(const fg_ivfpq_view* index, const uint8_t* base, int64_t nbase, const float* queries, int32_t nq,
                 const fg_search_params* params, int32_t* out_ids, float* out_dists, void* ws, size_t ws_bytes,
                 void* stream) {
    return search_any(index, base, 1, nbase, queries, nq, params, out_ids, out_dists, ws, ws_bytes, stream);
}

int fg_host_memory_mapped(const void* p, int32_t* mapped) {
    FG_REQUIRE(mapped, "null output");
    *mapped = 0;
    if (!p) return FG_OK;
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        (void)cudaGetLastError();  // an unknown pointer is not mapped
        return FG_OK;
    }
    *mapped = (at.type == cudaMemoryTypeHost && at.devicePointer == p) ? 1 : 0;
    return FG_OK;
}

int fg_kmeans_init(const float* data, int64_t n, int32_t dim, int32_t k, uint32_t seed, float* centroids,
                   void* ws, size_t ws_bytes, void* stream) {
    FG_REQUIRE(data && centroids && n >= 1 && dim >= 1 && k >= 1, "bad k-means init arguments");
    int rc = need_ws(ws, ws_bytes, (size_t)k * 8);
    if (rc) return rc;
    rc = kmeans_init(data, n, dim, k, seed, centroids, static_cast<int64_t*>(ws), as_stream(stream));
    return rc;
}

int fg_assign_workspace_size(int64_t n, int32_t dim, int32_t k, size_t* bytes) {
    FG_REQUIRE(bytes && n >= 0 && dim >= 1 && k >= 1, "bad arguments");
    *bytes = assign_workspace(n, k, dim);
    return FG_OK;
}

int fg_assign(const float* data, int64_t n, int32_t dim, const float* centroids, int32_t k, int32_t* out_assign,
              void* ws, size_t ws_bytes, void* stream) {
    FG_REQUIRE(n >= 0 && dim >= 1 && k >= 1, "bad assign shape");
    if (n == 0) return FG_OK;
    FG_REQUIRE(data && centroids && out_assign, "null buffer");
    cudaStream_t s = as_stream(stream);
    const size_t wb = assign_workspace(n, k, dim);
    if (!wb) return l2_argmin(data, n, centroids, k, dim, out_assign, s);
    int rc = need_ws(ws, ws_bytes, wb);
    if (rc) return rc;
    return assign_auto(data, n, dim, centroids, k, out_assign, ws, ws_bytes, s);
}

int fg_sort_by_list_workspace_size(int64_t n, int32_t k, size_t* bytes) {
    FG_REQUIRE(bytes && n >= 0 && k >= 1, "bad arguments");
    *bytes = sort_workspace(n, k);
    return FG_OK;
}

int fg_sort_by_list(const int32_t* assign, int64_t n, int32_t k, int32_t* order, int32_t* offsets, void* ws,
                    size_t ws_bytes, void* stream) {
    FG_REQUIRE(order && offsets && (assign || n == 0), "null buffer");
    int rc = need_ws(ws, ws_bytes, sort_workspace(n, k));
    if (rc) return rc;
    return sort_by_list(assign, n, k, order, offsets, ws, ws_bytes, as_stream(stream));
}

int fg_kmeans_update(const float* data, int32_t dim, const int32_t* order, const int32_t* offsets, int32_t k,
                     float* centroids, void* stream) {
    FG_REQUIRE(data && order && offsets && centroids && dim >= 1 && k >= 1, "bad arguments");
    return kmeans_update(data, dim, order, offsets, k, centroids, as_stream(stream));
}

int fg_kmeans_workspace_size(int64_t n, int32_t dim, int32_t k, size_t* bytes) {
    FG_REQUIRE(bytes && n >= 1 && dim >= 1 && k >= 1, "bad arguments");
    *bytes = kmeans_workspace(n, dim, k);
    return FG_OK;
}

int fg_kmeans(const float* data, int64_t n, int32_t dim, int32_t k, int32_t iters, uint32_t seed, float* centroids,
              void* ws, size_t ws_bytes, void* stream) {
    FG_REQUIRE(data && centroids && n >= k && k >= 1 && iters >= 0, "bad k-means arguments");
    int rc = need_ws(ws, ws_bytes, kmeans_workspace(n, dim, k));
    if (rc) return rc;
    return kmeans(data, n, dim, k, iters, seed, centroids, ws, ws_bytes, as_stream(stream));
}

int fg_pq_train_workspace_size(int64_t n, int32_t dim, int32_t pq_m, int32_t sample, size_t* bytes) {
    FG_REQUIRE(bytes && n >= 1 && pq_m >= 1 && sample >= 1, "bad arguments");
    *bytes = pq_train_workspace(n, dim, pq_m, sample);
    return FG_OK;
}

int fg_pq_train(const float* data, int64_t n, int32_t dim, const int32_t* assign, const float* centroids,
                int32_t pq_m, int32_t sample, int32_t iters, float* codebook, void* ws, size_t ws_bytes,
                void* stream) {
    FG_REQUIRE(data && assign && centroids && codebook, "null buffer");
    int rc = need_ws(ws, ws_bytes, pq_train_workspace(n, dim, pq_m, sample));
    if (rc) return rc;
    return pq_train(data, n, dim, assign, centroids, pq_m, sample, iters, codebook, ws, ws_bytes, as_stream(stream));
}

int fg_pq_encode(const float* data, int64_t n, int32_t dim, const int32_t* assign, const float* centroids,
                 const float* codebook, int32_t pq_m, uint8_t* codes, void* stream) {
    FG_REQUIRE(data && assign && centroids && codebook && codes, "null buffer");
    return pq_encode(data, n, dim, assign, centroids, codebook, pq_m, codes, as_stream(stream));
}

int fg_gather_lists(const uint8_t* codes, int64_t n, int32_t pq_m, const int32_t* order, uint8_t* out_codes,
                    int32_t* out_ids, void* stream) {
    FG_REQUIRE(codes && order && out_codes && out_ids && pq_m >= 1, "bad arguments");
    return gather_lists(codes, n, pq_m, order, out_codes, out_ids, as_stream(stream));
}

int fg_rebalance(const float* data, int64_t n, int32_t dim, const int32_t* assign, const float* centroids,
                 int32_t k, int32_t iters, uint32_t seed, int32_t* out_assign, float* out_centroids, int32_t cap,
                 int32_t* out_nlist, void* stream) {
    return rebalance(data, n, dim, assign, centroids, k, iters, seed, out_assign, out_centroids, cap, out_nlist,
                     as_stream(stream));
}

int fg_knn_workspace_size(int64_t nbase, int32_t dim, int32_t nq, int32_t k, size_t* bytes) {
    FG_REQUIRE(bytes && nbase >= 1 && dim >= 1 && nq >= 0 && k >= 1 && k <= nbase, "bad arguments");
    FG_REQUIRE(nbase <= 0x7fffffffll, "nbase too large");
    *bytes = knn_like_workspace(std::max(nq, 1), (int)nbase, k);
    return FG_OK;
}

int fg_knn(const float* base, int64_t nbase, int32_t dim, const float* queries, int32_t nq, int32_t k, int32_t metric,
           int32_t* out_ids, float* out_dists, void* ws, size_t ws_bytes, void* stream) {
    FG_REQUIRE(nbase >= 1 && nbase <= 0x7fffffffll && dim >= 1 && nq >= 0 && k >= 1 && k <= nbase && k <= 4096,
               "bad knn arguments");
    FG_REQUIRE(metric == FG_METRIC_L2 || metric == FG_METRIC_IP, "unknown metric %d", metric);
    if (nq == 0) return FG_OK;
    FG_REQUIRE(base && queries && out_ids && out_dists, "null buffer");
    int rc = need_ws(ws, ws_bytes, 1024);
    if (rc) return rc;
    return knn_like(base, nbase, dim, queries, nq, k, out_ids, out_dists, ws, ws_bytes, as_stream(stream), metric);
}

int fg_knn_exact(const float* base, int64_t nbase, int32_t dim, const float* queries, int32_t nq, int32_t k,
                 int32_t* out_ids, float* out_dists, void* ws, size_t ws_bytes, void* stream) {
    return fg_knn(base, nbase, dim, queries, nq, k, FG_METRIC_L2, out_ids, out_dists, ws, ws_bytes, stream);
}

}  // extern "C"
