// Test program: a caller written against the reference's C++ entry points
// (the way search_pipeline.cu:341-361 and build_global.cu:41-213 call them),
// compiled against include/fusiongpu_compat.hpp instead of gpu_global.cu and
// kmeans_gpu.cuh.  DIM and PQ_M come from -D flags as in the reference.
//
//   compat_search <index_dir> <queries.fvecs> <base.fvecs> <out_prefix> top_m rerank_m final_k
//       -> <out_prefix>.ids.ivecs, <out_prefix>.dists.fvecs (final results)
//   compat_search --kmeans <data.fvecs> k iters <out.fvecs>
//       -> run_kmeans_gpu centroids, then gpu_assign_to_centroids in <out>.assign.ivecs
#define FG_COMPAT_IMPLEMENTATION
#include "fusiongpu_compat.hpp"

#include <cstdlib>
#include <iostream>
#include <string>

#include "fg_host.hpp"

using namespace fghost;

static int kmeans_mode(int argc, char** argv) {
    if (argc != 6) return 2;
    std::vector<float> x;
    int d = 0;
    const int64_t n = read_vecs(argv[2], x, d);
    if (d != DIM) die("dimension differs from DIM");
    const int k = std::atoi(argv[3]), iters = std::atoi(argv[4]);
    std::vector<float> cen;
    run_kmeans_gpu(x.data(), (int)n, DIM, k, cen, iters);
    if (fg_compat_last_status() != 0) return 3;
    std::vector<int> as;
    gpu_assign_to_centroids(x.data(), cen.data(), (int)n, DIM, k, as);
    if (fg_compat_last_status() != 0) return 3;
    const std::string out = argv[5];
    write_vecs(out, cen.data(), k, DIM);
    write_vecs(out + ".assign.ivecs", as.data(), 1, (int)n);
    return 0;
}

int main(int argc, char** argv) {
    if (argc > 1 && std::string(argv[1]) == "--kmeans") return kmeans_mode(argc, argv);
    if (argc != 8) {
        std::cerr << "usage: compat_search <index_dir> <queries> <base> <out_prefix> top_m rerank_m final_k\n";
        return 2;
    }
    const int top_m = std::atoi(argv[5]), rerank_m = std::atoi(argv[6]), final_k = std::atoi(argv[7]);
    std::vector<float> q, base;
    int d = 0, d2 = 0;
    const int64_t nq = read_vecs(argv[2], q, d);
    const int64_t nbase = read_vecs(argv[3], base, d2);
    if (d != DIM || d2 != DIM) die("dimension differs from DIM");
    HostIndex h = load_index(argv[1], DIM, PQ_M);
    DevIndex di;
    di.upload(h, nullptr);
    IVFIndexGPU idx;
    idx.d_pq_codebook = di.codebook.p;
    idx.d_cluster_offsets = di.offsets.p;
    idx.d_all_pq_codes = di.codes.p;
    idx.d_all_vector_ids = di.ids.p;
    idx.d_centroids = di.centroids.p;
    idx.num_clusters = h.nlist;

    const int bs = (int)nq;
    DevBuf<float> dq(q.size()), db(base.size()), pd((size_t)bs * top_m), top_d((size_t)bs * rerank_m),
        fd((size_t)bs * final_k), tables(16), cut(16), thr(16);
    DevBuf<uint32_t> pid((size_t)bs * top_m);
    DevBuf<int> cnt(bs), off(bs + 1), atom(bs), top_i((size_t)bs * rerank_m), top_c(bs), fi((size_t)bs * final_k),
        coff(bs + 1), stable(bs);
    DevBuf<bool> fin(bs);
    dq.upload(q.data(), q.size());
    db.upload(base.data(), base.size());
    cudaMemset(top_i.p, 0, top_i.n * sizeof(int));
    cudaMemset(top_d.p, 0, top_d.n * sizeof(float));
    size_t wsb = 0;
    check(fg_coarse_workspace_size(h.nlist, DIM, bs, top_m, &wsb), "fg_coarse_workspace_size");
    DevBuf<uint8_t> ws(wsb);
    cudaStream_t s;
    cudaStreamCreate(&s);
    check(fg_coarse_search(di.centroids.p, h.nlist, DIM, dq.p, bs, top_m, pid.p, pd.p, ws.p, wsb, s),
          "fg_coarse_search");
    // the pools the reference passes by reference (and may reallocate)
    int *flat_i = nullptr, *flat_i2 = nullptr;
    float *flat_d = nullptr, *flat_d2 = nullptr;
    size_t pool_cap = 0;
    run_gpu_batch_logic(idx, dq.p, pid.p, pd.p, tables.p, flat_i, flat_d, flat_i2, flat_d2, pool_cap, cnt.p, off.p,
                        atom.p, top_i.p, top_d.p, top_c.p, bs, top_m, rerank_m, final_k, 100.0f, cut.p, thr.p, coff.p, s,
                        nullptr, 12, 50, 1.0f);
    if (fg_compat_last_status() != 0) return 3;
    run_gpu_rerank(dq.p, top_i.p, top_c.p, db.p, fi.p, fd.p, stable.p, fin.p, bs, rerank_m, final_k, (int)nbase, 128,
                   0.1f, 2, s);
    if (fg_compat_last_status() != 0) return 3;
    check_cuda(cudaStreamSynchronize(s), "search");
    std::vector<int> hi((size_t)bs * final_k);
    std::vector<float> hd((size_t)bs * final_k);
    fi.download(hi.data(), hi.size());
    fd.download(hd.data(), hd.size());
    const std::string out = argv[4];
    write_vecs(out + ".ids.ivecs", hi.data(), bs, final_k);
    write_vecs(out + ".dists.fvecs", hd.data(), bs, final_k);
    std::cout << "ok " << bs << " queries" << std::endl;
    return 0;
}
