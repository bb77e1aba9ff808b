// fg_tune_parameters -- the reference's tune_parameters executable
// (tune_parameters.cu:1122-1224) on this library's C ABI, plus a sweep.
//
//   fg_tune_parameters <base.fvecs|.bvecs> [-n 1000] [-k 10] [-o search_config.txt]
//       [--res ../res] [--pq_m 32] [--seed 42] [--sweep] [--target 0.95]
//       [--queries q.fvecs --gt gt.ivecs]
//
// Samples -n base vectors as queries (MT19937(seed) output modulo the base
// size), finds their exact -k nearest neighbours on the GPU (fg_knn_exact),
// and derives the reference's four recommendations with fg_tune; writes them
// with the reference's keys.  --sweep then measures recall@k and device-timed
// throughput of the full search over a grid of nprobe (top_m) and rerank
// depth around the recommendation, on the sample or on --queries/--gt, and
// prints the fastest point that reaches --target recall.
#include <cmath>
#include <fstream>
#include <iomanip>
#include <iostream>
#include <random>
#include <set>

#include "fg_host.hpp"

using namespace fghost;

int main(int argc, char** argv) {
    Args a(argc, argv, {"--sweep"});
    if (a.pos.size() != 1) {
        std::cerr << "Usage: fg_tune_parameters <base.fvecs|.bvecs> [-n 1000] [-k 10] [-o search_config.txt]\n"
                     "       [--res ../res] [--pq_m 32] [--seed 42] [--sweep] [--target 0.95]\n"
                     "       [--queries q.fvecs --gt gt.ivecs]\n";
        return 1;
    }
    const int ns = a.geti({"-n"}, 1000);
    const int k = a.geti({"-k"}, 10);
    const std::string out = a.gets({"-o"}, "search_config.txt");
    const std::string res = a.gets({"--res"}, "../res");
    const int pq_m = a.geti({"--pq_m"}, 32);
    const uint32_t seed = (uint32_t)a.geti({"--seed"}, 42);
    if (ns < 1 || k < 1) die("-n and -k must be positive");

    std::vector<float> base;
    int dim = 0;
    const int64_t nbase = read_base(a.pos[0], base, dim);
    HostIndex h = load_index(res, dim, pq_m);
    std::cout << "Base: " << nbase << " x " << dim << "; index: " << h.nlist << " lists, pq_m " << pq_m << std::endl;

    cudaStream_t s;
    check_cuda(cudaStreamCreate(&s), "cudaStreamCreate");
    DevIndex idx;
    idx.upload(h, s);
    DevBuf<float> d_base((size_t)nbase * dim);
    d_base.upload(base.data(), base.size(), s);

    // sample queries: base rows MT19937(seed)() % nbase
    std::mt19937 gen(seed);
    std::vector<float> hq((size_t)ns * dim);
    for (int i = 0; i < ns; ++i) {
        const int64_t r = (int64_t)(gen() % (uint32_t)nbase);
        std::copy(base.begin() + (size_t)r * dim, base.begin() + (size_t)(r + 1) * dim, hq.begin() + (size_t)i * dim);
    }
    DevBuf<float> dq(hq.size());
    dq.upload(hq.data(), hq.size(), s);
    DevBuf<int32_t> gt((size_t)ns * k);
    DevBuf<float> gd((size_t)ns * k);
    size_t wsb = 0;
    check(fg_knn_workspace_size(nbase, dim, ns, k, &wsb), "fg_knn_workspace_size");
    {
        DevBuf<uint8_t> ws(wsb);
        check(fg_knn_exact(d_base.p, nbase, dim, dq.p, ns, k, gt.p, gd.p, ws.p, wsb, s), "fg_knn_exact");
        check_cuda(cudaStreamSynchronize(s), "ground truth");
    }

    fg_tune_result r{};
    std::vector<int32_t> cr((size_t)ns * k), pr((size_t)ns * k), er((size_t)ns * k);
    std::vector<float> ratios((size_t)ns);
    check(fg_tune(&idx.view, d_base.p, nbase, dq.p, ns, gt.p, k, &r, cr.data(), pr.data(), er.data(), ratios.data(),
                  s),
          "fg_tune");

    auto mean = [](const std::vector<int32_t>& v) {
        double sum = 0;
        int64_t n = 0;
        for (int32_t x : v)
            if (x > 0) sum += x, ++n;
        return n ? sum / n : 0.0;
    };
    std::cout << "\n========== tuning results ==========\n"
              << "  sample queries x k:       " << ns << " x " << k << "\n"
              << "  neighbours in a list:     " << r.n_ranked << "\n"
              << "  mean coarse rank:         " << mean(cr) << "\n"
              << "  mean PQ rank in list:     " << mean(pr) << "\n"
              << "  mean exact rank in list:  " << mean(er) << "\n"
              << "  RECOMMENDED_TOP_M (P99.5 of coarse ranks):   " << r.top_m << "\n"
              << "  RECOMMENDED_P1_LISTS (elbow, coverage " << std::fixed << std::setprecision(1)
              << r.coverage_at_elbow * 100 << "%): " << r.p1_lists << "\n"
              << "  RECOMMENDED_LIMIT_K (max PQ rank in P1 lists, " << r.n_in_p1 << " neighbours): " << r.limit_k
              << "\n"
              << "  THRESHOLD_COEFF (max of " << r.n_ratios << " ratios): " << std::setprecision(3)
              << r.threshold_coeff << "\n====================================" << std::endl;
    {
        std::ofstream f(out);
        if (!f) die("cannot write " + out);
        f << "# search parameters recommended by fg_tune_parameters\n"
          << "RECOMMENDED_TOP_M=" << r.top_m << "\n"
          << "RECOMMENDED_P1_LISTS=" << r.p1_lists << "\n"
          << "RECOMMENDED_LIMIT_K=" << r.limit_k << "\n"
          << "THRESHOLD_COEFF=" << std::fixed << std::setprecision(3) << r.threshold_coeff << "\n";
    }
    std::cout << "Wrote " << out << std::endl;
    std::cout << std::defaultfloat << std::setprecision(6);
    std::cout << "TUNE top_m=" << r.top_m << " p1_lists=" << r.p1_lists << " limit_k=" << r.limit_k
              << " threshold_coeff=" << r.threshold_coeff << std::endl;

    if (!a.has("--sweep")) return 0;

    // sweep: the sample (or the given queries) with its ground truth
    std::vector<int32_t> hgt;
    int gt_k = k;
    int64_t nq = ns;
    DevBuf<float> sq;
    const float* qptr = dq.p;
    const std::string qpath = a.gets({"--queries"}, ""), gpath = a.gets({"--gt"}, "");
    if (!qpath.empty()) {
        if (gpath.empty()) die("--queries needs --gt");
        std::vector<float> q2;
        int d2 = 0;
        nq = read_base(qpath, q2, d2);
        if (d2 != dim) die("query dimension differs from the base");
        sq.resize(q2.size());
        sq.upload(q2.data(), q2.size(), s);
        qptr = sq.p;
        if (read_vecs(gpath, hgt, gt_k) < nq) die("ground truth has fewer rows than queries");
    } else {
        hgt.resize((size_t)ns * k);
        gt.download(hgt.data(), hgt.size(), s);
        check_cuda(cudaStreamSynchronize(s), "download ground truth");
    }
    const float target = a.getf({"--target"}, 0.95f);
    const int rk = std::min(10, k);
    std::set<int> tms;
    for (int f : {1, 2, 4, 8}) {
        tms.insert(std::max(1, std::min(h.nlist, r.top_m * f / 4)));
        tms.insert(std::max(1, std::min(h.nlist, r.top_m * f)));
    }
    const int rms[] = {std::max(k, 50), 100, 200, 500, 1000};
    fg_search_params p;
    fg_search_params_default(&p);
    p.final_k = k;
    p.limit_k = std::max(1, std::min(r.limit_k, 1024));
    p.threshold_coeff = r.threshold_coeff;
    p.ref_compat = 0;
    DevBuf<int32_t> oi((size_t)nq * k);
    DevBuf<float> od((size_t)nq * k);
    std::vector<int32_t> hi((size_t)nq * k);
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    std::cout << "\n  top_m  rerank_m  recall@" << rk << "        QPS" << std::endl;
    double best_qps = -1;
    int best_tm = 0, best_rm = 0;
    for (int tm : tms) {
        for (int rm : rms) {
            if (rm < k) continue;
            p.top_m = tm;
            p.p1_lists = std::min(r.p1_lists, tm);
            p.rerank_m = rm;
            size_t b = 0;
            if (fg_search_workspace_size(&idx.view, &p, (int32_t)nq, &b) != FG_OK) continue;
            DevBuf<uint8_t> ws(b);
            if (fg_search(&idx.view, d_base.p, nbase, qptr, (int32_t)nq, &p, oi.p, od.p, ws.p, b, s) != FG_OK) {
                std::cout << std::setw(7) << tm << std::setw(10) << rm << "  unsupported: " << fg_last_error()
                          << std::endl;
                continue;
            }
            oi.download(hi.data(), hi.size(), s);
            check_cuda(cudaStreamSynchronize(s), "search");
            const double rec = recall_at(hi, k, hgt, gt_k, nq, rk);
            const int reps = 3;
            cudaEventRecord(e0, s);
            for (int i = 0; i < reps; ++i)
                check(fg_search(&idx.view, d_base.p, nbase, qptr, (int32_t)nq, &p, oi.p, od.p, ws.p, b, s),
                      "fg_search");
            cudaEventRecord(e1, s);
            check_cuda(cudaEventSynchronize(e1), "timing");
            float ms = 0;
            cudaEventElapsedTime(&ms, e0, e1);
            const double qps = nq / (ms / reps / 1e3);
            std::cout << std::setw(7) << tm << std::setw(10) << rm << std::setw(12) << std::setprecision(4) << rec
                      << std::setw(12) << std::setprecision(6) << qps << std::endl;
            if (rec >= target && qps > best_qps) {
                best_qps = qps;
                best_tm = tm;
                best_rm = rm;
            }
        }
    }
    if (best_qps > 0)
        std::cout << "SWEEP best top_m=" << best_tm << " rerank_m=" << best_rm << " qps=" << best_qps
                  << " at recall@" << rk << " >= " << target << std::endl;
    else
        std::cout << "SWEEP no grid point reached recall@" << rk << " >= " << target << std::endl;
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaStreamDestroy(s);
    return 0;
}
