// fg_build_global -- the reference's build_global executable (build_global.cu:21-258)
// on this library's C ABI: k-means, assignment, list rebalancing, residual PQ
// training, encoding and list assembly, all on the GPU, writing the same
// ivf_data.bin / global_pq_codebook.bin / cluster_distribution.csv.
//
//   fg_build_global <base.fvecs|.bvecs> [--nlist 2048] [--pq_m 32] [--out ../res]
//       [--kmeans_iters 20] [--split_iters 15] [--pq_sample 50000] [--pq_iters 8]
//       [--max_n N] [--no-rebalance]
//
// No CAGRA graph over the centroids is built: the coarse quantizer searches
// the centroids exactly.  The build is deterministic (same files every run).
#include <chrono>
#include <fstream>
#include <iostream>

#include "fg_host.hpp"

using namespace fghost;

namespace {

double now_ms() {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

template <class F>
void stage(const char* name, F&& f) {
    const double t0 = now_ms();
    f();
    check_cuda(cudaDeviceSynchronize(), name);
    std::cout << "  " << name << ": " << (now_ms() - t0) << " ms" << std::endl;
}

}  // namespace

int main(int argc, char** argv) {
    Args a(argc, argv, {"--no-rebalance"});
    if (a.pos.size() != 1) {
        std::cerr << "Usage: fg_build_global <base.fvecs|.bvecs> [--nlist 2048] [--pq_m 32] [--out ../res]\n"
                     "       [--kmeans_iters 20] [--split_iters 15] [--pq_sample 50000] [--pq_iters 8]\n"
                     "       [--max_n N] [--no-rebalance]\n";
        return 1;
    }
    const int k = a.geti({"--nlist", "-k"}, 2048);
    const int pq_m = a.geti({"--pq_m", "-M"}, 32);
    const std::string out = a.gets({"--out", "-o"}, "../res");
    const int km_iters = a.geti({"--kmeans_iters"}, 20);
    const int split_iters = a.geti({"--split_iters"}, 15);
    const int pq_sample = a.geti({"--pq_sample"}, 50000);
    const int pq_iters = a.geti({"--pq_iters"}, 8);
    const int64_t max_n = a.geti({"--max_n"}, -1);
    const uint32_t seed = 42;

    std::vector<float> host;
    int dim = 0;
    const int64_t n = read_base(a.pos[0], host, dim, max_n);
    std::cout << "Loaded " << n << " vectors of dimension " << dim << "." << std::endl;
    if (dim % pq_m) die("dimension is not a multiple of --pq_m");
    if (n < k) die("fewer vectors than --nlist");

    DevBuf<float> x((size_t)n * dim), cen((size_t)k * dim);
    DevBuf<int32_t> as((size_t)n);
    x.upload(host.data(), host.size());
    size_t wsb = 0;
    check(fg_kmeans_workspace_size(n, dim, k, &wsb), "fg_kmeans_workspace_size");
    DevBuf<uint8_t> ws(wsb);

    std::cout << "Training " << k << " initial centroids (GPU)..." << std::endl;
    stage("k-means", [&] { check(fg_kmeans(x.p, n, dim, k, km_iters, seed, cen.p, ws.p, wsb, nullptr), "fg_kmeans"); });
    size_t awb = 0;
    check(fg_assign_workspace_size(n, dim, k, &awb), "fg_assign_workspace_size");
    DevBuf<uint8_t> aws(awb ? awb : 256);
    stage("assign", [&] { check(fg_assign(x.p, n, dim, cen.p, k, as.p, aws.p, awb, nullptr), "fg_assign"); });

    int nlist = k;
    DevBuf<float> fcen;
    if (!a.has("--no-rebalance")) {
        std::cout << "--- Recursive rebalancing (FIFO queue) ---" << std::endl;
        int cap = (int)std::min<int64_t>(n, 4ll * k);
        int32_t got = 0;
        stage("rebalance", [&] {
            for (;;) {
                fcen.resize((size_t)cap * dim);
                const int rc = fg_rebalance(x.p, n, dim, as.p, cen.p, k, split_iters, seed, as.p, fcen.p, cap, &got,
                                            nullptr);
                if (rc == FG_ERR_WORKSPACE && got > cap) {
                    cap = got;
                    continue;
                }
                check(rc, "fg_rebalance");
                break;
            }
        });
        nlist = got;
        std::cout << "Cluster Count: " << k << " -> " << nlist << std::endl;
    } else {
        fcen.resize((size_t)k * dim);
        check_cuda(cudaMemcpy(fcen.p, cen.p, (size_t)k * dim * 4, cudaMemcpyDeviceToDevice), "copy");
    }

    HostIndex h;
    h.dim = dim;
    h.pq_m = pq_m;
    h.nlist = nlist;
    h.total = (int)n;

    // list sizes for cluster_distribution.csv
    DevBuf<int32_t> order((size_t)n), offs((size_t)nlist + 1);
    size_t swsb = 0;
    check(fg_sort_by_list_workspace_size(n, nlist, &swsb), "fg_sort_by_list_workspace_size");
    DevBuf<uint8_t> sws(swsb);
    stage("sort by list",
          [&] { check(fg_sort_by_list(as.p, n, nlist, order.p, offs.p, sws.p, swsb, nullptr), "fg_sort_by_list"); });
    h.offsets.resize((size_t)nlist + 1);
    offs.download(h.offsets.data(), h.offsets.size());
    check_cuda(cudaDeviceSynchronize(), "download offsets");
    {
        std::ofstream csv("cluster_distribution.csv");
        csv << "cluster_id,count\n";
        for (int c = 0; c < nlist; ++c) csv << c << "," << (h.offsets[c + 1] - h.offsets[c]) << "\n";
    }

    std::cout << "Training residual global PQ..." << std::endl;
    const int sd = dim / pq_m;
    DevBuf<float> cb((size_t)pq_m * 256 * sd);
    size_t pwsb = 0;
    check(fg_pq_train_workspace_size(n, dim, pq_m, pq_sample, &pwsb), "fg_pq_train_workspace_size");
    DevBuf<uint8_t> pws(pwsb);
    stage("pq train", [&] {
        check(fg_pq_train(x.p, n, dim, as.p, fcen.p, pq_m, pq_sample, pq_iters, cb.p, pws.p, pwsb, nullptr),
              "fg_pq_train");
    });
    DevBuf<uint8_t> codes((size_t)n * pq_m), lcodes((size_t)n * pq_m);
    DevBuf<int32_t> lids((size_t)n);
    stage("pq encode",
          [&] { check(fg_pq_encode(x.p, n, dim, as.p, fcen.p, cb.p, pq_m, codes.p, nullptr), "fg_pq_encode"); });
    stage("gather lists",
          [&] { check(fg_gather_lists(codes.p, n, pq_m, order.p, lcodes.p, lids.p, nullptr), "fg_gather_lists"); });

    h.ids.resize((size_t)n);
    h.codes.resize((size_t)n * pq_m);
    h.centroids.resize((size_t)nlist * dim);
    h.codebook.resize(cb.n);
    lids.download(h.ids.data(), h.ids.size());
    lcodes.download(h.codes.data(), h.codes.size());
    fcen.download(h.centroids.data(), h.centroids.size());
    cb.download(h.codebook.data(), h.codebook.size());
    check_cuda(cudaDeviceSynchronize(), "download index");
    save_index(out, h);
    std::cout << "Wrote " << out << "/ivf_data.bin (" << nlist << " lists) and " << out
              << "/global_pq_codebook.bin.\nBuild complete." << std::endl;
    return 0;
}
