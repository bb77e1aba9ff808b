// noalloc.cu -- a coarse search that allocates nothing and takes no workspace.
//
// Some callers cannot hand this library device memory at call time:
//   * plugins hosted inside another runtime that owns every device pool and
//     forbids its plugins from calling the CUDA allocator;
//   * latency-critical serving loops that must never hit cudaMalloc/cudaFree,
//     which can synchronise the whole device.
// fg_coarse_search_noalloc serves them: it runs the exact CUDA-core coarse
// search (the same kernels as fg_coarse_search_simt) with its scratch in a
// 16 MiB array that lives in the library's device image.  Every GPU that loads
// the library holds that array until the process exits.
//
// The array's name is only a host-side handle: host code must never pass it
// to a kernel.  Its device address is resolved with cudaGetSymbolAddress once
// per device, the first time the entry point runs with that device current,
// and cached for the life of the process; make that first call before any
// stream capture.  cudaDeviceReset unloads the library's device image, so a
// process that resets a device must not call this entry point there again:
// the cached address would point at the old image.
//
// All calls on one device share the array.  Calls whose GPU work overlaps
// (different streams, or different host threads) race on it and may return
// wrong results: serialise them.  Nothing in the array needs to start at zero:
// each call writes every scratch element before reading it (distance rows,
// then the selection stage buffers), so the contents left by the previous
// call are never used.
#include <mutex>

#include "fg_common.cuh"

namespace fg {

int knn_like(const float* Y, long long ny, int dim, const float* Q, long long nq, int k, int32_t* out_i,
             float* out_v, void* ws, size_t ws_bytes, cudaStream_t s, int metric = FG_METRIC_L2);

constexpr size_t kNoAllocScratchBytes = 16u << 20;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[kNoAllocMaxDevices];

// Device address of g_noalloc_scratch on the current device (resolved once).
static int noalloc_scratch(void** out) {
    int dev = 0;
    FG_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kNoAllocMaxDevices)
        return fail(FG_ERR_UNSUPPORTED, "device %d beyond the %d devices the scratch table covers", dev,
                    kNoAllocMaxDevices);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || p == nullptr)
            return fail(FG_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
        g_noalloc_ptr[dev] = p;
    }
    *out = g_noalloc_ptr[dev];
    return FG_OK;
}

// Scratch one query row of the exact path needs: its distance row plus, past
// one 8192-column select segment, the stage-1 winners (values and ids).
static size_t noalloc_row_bytes(int nlist, int top_m) {
    const int nseg = (nlist + 8191) / 8192;
    return (size_t)nlist * 4 + (nseg > 1 ? (size_t)nseg * top_m * 8 : 0);
}

}  // namespace fg

using namespace fg;

extern "C" int fg_coarse_search_noalloc(const float* centroids, int32_t nlist, int32_t dim, const float* queries,
                                        int32_t nq, int32_t top_m, uint32_t* out_ids, float* out_dists,
                                        void* stream) {
    FG_REQUIRE(nlist >= 1 && dim >= 1 && nq >= 0, "bad coarse shape");
    FG_REQUIRE(top_m >= 1 && top_m <= nlist && top_m <= 4096, "top_m %d outside [1, min(nlist, 4096)]", top_m);
    const size_t row = noalloc_row_bytes(nlist, top_m);
    FG_REQUIRE(row + 2048 <= kNoAllocScratchBytes,
               "nlist=%d, top_m=%d needs %zu scratch bytes per query; the allocation-free path has %zu",
               nlist, top_m, row + 2048, kNoAllocScratchBytes);
    if (nq == 0) return FG_OK;
    FG_REQUIRE(centroids && queries && out_ids && out_dists, "null buffer");
    void* scratch = nullptr;
    int rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    return knn_like(centroids, nlist, dim, queries, nq, top_m, reinterpret_cast<int32_t*>(out_ids), out_dists,
                    scratch, kNoAllocScratchBytes, static_cast<cudaStream_t>(stream));
}
