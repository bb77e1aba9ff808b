// fg_search_pipeline -- the reference's search_pipeline executable
// (search_pipeline.cu:49-647) on this library's C ABI.
//
//   fg_search_pipeline <base> <query> [gt] [-b 128] [-m 20] [-r 10000] [-mb 128]
//       [-e 0.1] [--beta 2] [-p 100] [-s 2] [-k 10] [--p1_lists 12] [--limit_k 50]
//       [--threshold_coeff 1.0] [--res ../res] [--pq_m 32] [--intended] [--fused]
//       [--graph] [--out results.ivecs] [--repeat 1]
//
// Queries are cut into batches and handed round-robin to `-s` stream
// contexts; each batch runs H2D copy -> coarse search -> candidate generation
// -> rerank -> D2H copy on its own stream, and a collector thread waits for
// each batch and reads its per-stage CUDA-event times, as the reference's
// pipeline does.  Nothing in a batch blocks the submitting thread: the C ABI
// calls are asynchronous and need no host round trip.
//
// By default the search reproduces the reference's results (ref_compat: the
// 128-lane gather and the other quirks of gpu_global.cu); --intended uses the
// full rerank depth.  --fused issues one fg_search call per batch instead of
// the three stage calls (no per-stage times then).  --graph captures a full
// batch (H2D copy, the search, D2H copy) once per stream context as a CUDA
// graph and replays it (partial batches run eagerly; no per-stage times).
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <iomanip>
#include <iostream>
#include <mutex>
#include <queue>
#include <thread>

#include "fg_host.hpp"

using namespace fghost;

namespace {

struct StageTimes {
    double h2d = 0, coarse = 0, batch = 0, rerank = 0, d2h = 0, e2e = 0;
    int64_t batches = 0, candidates = 0;
};

struct Ctx {
    cudaStream_t s = nullptr;
    float* h_q = nullptr;
    int32_t* h_ids = nullptr;
    int32_t* h_cand = nullptr;
    DevBuf<float> q, pd, top_d, fd;
    DevBuf<uint32_t> pid;
    DevBuf<int32_t> top_i, top_c, cand, fi;
    DevBuf<uint8_t> ws;
    size_t ws_bytes = 0;
    cudaEvent_t e[7];  // h2d start/end, coarse end, batch end, rerank end, d2h end (= done), spare
    cudaGraphExec_t graph = nullptr;  // a captured full batch (--graph)
    int n = 0;
    int64_t offset = 0;
    bool busy = false;
    std::mutex m;
    std::condition_variable cv;
};

class SearchPipeline {
   public:
    SearchPipeline(const DevIndex& idx, const float* d_base, int64_t nbase, const fg_search_params& p, int batch,
                   int nstreams, int64_t nq, bool fused, bool graph)
        : idx_(idx),
          base_(d_base),
          nbase_(nbase),
          p_(p),
          batch_(batch),
          fused_(fused),
          use_graph_(graph),
          results_((size_t)nq * p.final_k) {
        const int dim = idx.view.dim;
        for (int i = 0; i < nstreams; ++i) {
            auto c = std::make_unique<Ctx>();
            check_cuda(cudaStreamCreateWithFlags(&c->s, cudaStreamNonBlocking), "cudaStreamCreate");
            check_cuda(cudaMallocHost(&c->h_q, (size_t)batch * dim * 4), "cudaMallocHost");
            check_cuda(cudaMallocHost(&c->h_ids, (size_t)batch * p.final_k * 4), "cudaMallocHost");
            check_cuda(cudaMallocHost(&c->h_cand, (size_t)batch * 4), "cudaMallocHost");
            c->q.resize((size_t)batch * dim);
            c->fi.resize((size_t)batch * p.final_k);
            c->fd.resize((size_t)batch * p.final_k);
            c->cand.resize((size_t)batch);
            if (fused) {
                check(fg_search_workspace_size(&idx.view, &p, batch, &c->ws_bytes), "fg_search_workspace_size");
            } else {
                check(fg_coarse_workspace_size(idx.view.nlist, dim, batch, p.top_m, &c->ws_bytes),
                      "fg_coarse_workspace_size");
                c->pid.resize((size_t)batch * p.top_m);
                c->pd.resize((size_t)batch * p.top_m);
                c->top_i.resize((size_t)batch * p.rerank_m);
                c->top_d.resize((size_t)batch * p.rerank_m);
                c->top_c.resize((size_t)batch);
            }
            c->ws.resize(c->ws_bytes);
            for (cudaEvent_t& ev : c->e) check_cuda(cudaEventCreate(&ev), "cudaEventCreate");
            ctx_.push_back(std::move(c));
        }
        worker_ = std::thread([this] { collect(); });
    }

    ~SearchPipeline() {
        {
            std::lock_guard<std::mutex> lk(qm_);
            running_ = false;
        }
        qcv_.notify_all();
        worker_.join();
        for (auto& c : ctx_) {
            if (c->graph) cudaGraphExecDestroy(c->graph);
            for (cudaEvent_t ev : c->e) cudaEventDestroy(ev);
            cudaFreeHost(c->h_q);
            cudaFreeHost(c->h_ids);
            cudaFreeHost(c->h_cand);
            cudaStreamDestroy(c->s);
        }
    }

    void submit(const float* queries, int n, int64_t offset) {
        Ctx& c = *ctx_[next_];
        next_ = (next_ + 1) % ctx_.size();
        {
            std::unique_lock<std::mutex> lk(c.m);
            c.cv.wait(lk, [&] { return !c.busy; });
            c.busy = true;
        }
        const int dim = idx_.view.dim;
        c.n = n;
        c.offset = offset;
        std::memcpy(c.h_q, queries, (size_t)n * dim * 4);
        if (use_graph_ && n == batch_) {
            if (!c.graph) {
                // the whole batch as one graph: H2D, the search, D2H
                cudaGraph_t g;
                check_cuda(cudaStreamBeginCapture(c.s, cudaStreamCaptureModeThreadLocal), "begin capture");
                enqueue(c, n);
                check_cuda(cudaStreamEndCapture(c.s, &g), "end capture");
                check_cuda(cudaGraphInstantiate(&c.graph, g, 0), "graph instantiate");
                cudaGraphDestroy(g);
            }
            cudaEventRecord(c.e[0], c.s);
            for (int i = 1; i < 5; ++i) cudaEventRecord(c.e[i], c.s);
            check_cuda(cudaGraphLaunch(c.graph, c.s), "graph launch");
            cudaEventRecord(c.e[5], c.s);
        } else {
            cudaEventRecord(c.e[0], c.s);
            enqueue(c, n, true);
            cudaEventRecord(c.e[5], c.s);
        }
        {
            std::lock_guard<std::mutex> lk(qm_);
            work_.push(&c);
            ++pending_;
        }
        qcv_.notify_all();
    }

    // H2D copy, search, D2H copy of one batch on the context's stream; with
    // `events`, the stage boundaries are recorded (not inside a capture)
    void enqueue(Ctx& c, int n, bool events = false) {
        const int dim = idx_.view.dim, k = p_.final_k;
        check_cuda(cudaMemcpyAsync(c.q.p, c.h_q, (size_t)n * dim * 4, cudaMemcpyHostToDevice, c.s), "H2D");
        if (events) cudaEventRecord(c.e[1], c.s);
        if (fused_) {
            check(fg_search(&idx_.view, base_, nbase_, c.q.p, n, &p_, c.fi.p, c.fd.p, c.ws.p, c.ws_bytes, c.s),
                  "fg_search");
            if (events) {
                cudaEventRecord(c.e[2], c.s);
                cudaEventRecord(c.e[3], c.s);
            }
        } else {
            check(fg_coarse_search(idx_.view.centroids, idx_.view.nlist, dim, c.q.p, n, p_.top_m, c.pid.p, c.pd.p,
                                   c.ws.p, c.ws_bytes, c.s),
                  "fg_coarse_search");
            if (events) cudaEventRecord(c.e[2], c.s);
            check(fg_batch_logic(&idx_.view, c.q.p, n, c.pid.p, c.pd.p, &p_, c.top_i.p, c.top_d.p, c.top_c.p,
                                 c.cand.p, c.s),
                  "fg_batch_logic");
            if (events) cudaEventRecord(c.e[3], c.s);
            check(fg_rerank(c.q.p, n, dim, c.top_i.p, c.top_c.p, base_, nbase_, &p_, c.fi.p, c.fd.p, c.s),
                  "fg_rerank");
        }
        if (events) cudaEventRecord(c.e[4], c.s);
        check_cuda(cudaMemcpyAsync(c.h_ids, c.fi.p, (size_t)n * k * 4, cudaMemcpyDeviceToHost, c.s), "D2H");
        if (!fused_)
            check_cuda(cudaMemcpyAsync(c.h_cand, c.cand.p, (size_t)n * 4, cudaMemcpyDeviceToHost, c.s), "D2H");
    }

    void wait_all() {
        std::unique_lock<std::mutex> lk(qm_);
        qcv_.wait(lk, [&] { return pending_ == 0; });
    }

    void reset_times() {
        std::lock_guard<std::mutex> lk(qm_);
        t_ = StageTimes{};
    }
    StageTimes times() {
        std::lock_guard<std::mutex> lk(qm_);
        return t_;
    }
    const std::vector<int32_t>& results() const { return results_; }

   private:
    void collect() {
        for (;;) {
            Ctx* c = nullptr;
            {
                std::unique_lock<std::mutex> lk(qm_);
                qcv_.wait(lk, [&] { return !work_.empty() || !running_; });
                if (work_.empty()) return;
                c = work_.front();
                work_.pop();
            }
            check_cuda(cudaEventSynchronize(c->e[5]), "batch");
            float h2d = 0, co = 0, ba = 0, re = 0, d2h = 0, e2e = 0;
            cudaEventElapsedTime(&h2d, c->e[0], c->e[1]);
            cudaEventElapsedTime(&co, c->e[1], c->e[2]);
            cudaEventElapsedTime(&ba, c->e[2], c->e[3]);
            cudaEventElapsedTime(&re, c->e[3], c->e[4]);
            cudaEventElapsedTime(&d2h, c->e[4], c->e[5]);
            cudaEventElapsedTime(&e2e, c->e[0], c->e[5]);
            const int k = p_.final_k;
            std::memcpy(results_.data() + (size_t)c->offset * k, c->h_ids, (size_t)c->n * k * 4);
            int64_t cand = 0;
            if (!fused_)
                for (int i = 0; i < c->n; ++i) cand += c->h_cand[i];
            {
                std::lock_guard<std::mutex> lk(qm_);
                t_.h2d += h2d;
                t_.coarse += co;
                t_.batch += ba;
                t_.rerank += re;
                t_.d2h += d2h;
                t_.e2e += e2e;
                t_.candidates += cand;
                ++t_.batches;
                --pending_;
            }
            {
                std::lock_guard<std::mutex> lk(c->m);
                c->busy = false;
            }
            c->cv.notify_all();
            qcv_.notify_all();
        }
    }

    const DevIndex& idx_;
    const float* base_;
    int64_t nbase_;
    fg_search_params p_;
    int batch_;
    bool fused_;
    bool use_graph_;
    std::vector<std::unique_ptr<Ctx>> ctx_;
    size_t next_ = 0;
    std::vector<int32_t> results_;
    std::thread worker_;
    std::mutex qm_;
    std::condition_variable qcv_;
    std::queue<Ctx*> work_;
    int64_t pending_ = 0;
    bool running_ = true;
    StageTimes t_;
};

}  // namespace

int main(int argc, char** argv) {
    Args a(argc, argv, {"--intended", "--fused", "--graph"});
    if (a.pos.size() < 2) {
        std::cerr << "Usage: fg_search_pipeline <base> <query> [gt] [-b 128] [-m 20] [-r 10000] [-mb 128] [-e 0.1]\n"
                     "       [--beta 2] [-p 100] [-s 2] [-k 10] [--p1_lists 12] [--limit_k 50]\n"
                     "       [--threshold_coeff 1.0] [--res ../res] [--pq_m 32] [--intended] [--fused]\n"
                     "       [--graph] [--out results.ivecs] [--repeat 1]\n";
        return 1;
    }
    fg_search_params p;
    fg_search_params_default(&p);
    const int batch = a.geti({"-b", "--batch_size"}, 128);
    p.top_m = a.geti({"-m", "--top_m"}, 20);
    p.rerank_m = a.geti({"-r", "--rerank_m"}, 10000);
    p.mini_batch = a.geti({"-mb", "--mini_batch"}, 128);
    p.epsilon = a.getf({"-e", "--epsilon"}, 0.1f);
    p.beta = a.geti({"--beta"}, 2);
    p.prune_ratio = a.getf({"-p", "--prune"}, 100.0f);
    const int nstreams = a.geti({"-s", "--streams"}, 2);
    p.final_k = a.geti({"-k", "--topk"}, 10);
    p.p1_lists = a.geti({"--p1_lists"}, 12);
    p.limit_k = a.geti({"--limit_k"}, 50);
    p.threshold_coeff = a.getf({"--threshold_coeff"}, 1.0f);
    p.ref_compat = a.has("--intended") ? 0 : 1;
    const std::string res = a.gets({"--res"}, "../res");
    const int pq_m = a.geti({"--pq_m"}, 32);
    const int repeat = std::max(1, a.geti({"--repeat"}, 1));
    const bool fused = a.has("--fused");
    const bool graph = a.has("--graph");
    if (batch < 1 || nstreams < 1) die("batch size and stream count must be positive");

    std::vector<float> base, queries;
    int dim = 0, qdim = 0;
    const int64_t nbase = read_base(a.pos[0], base, dim);
    const int64_t nq = read_base(a.pos[1], queries, qdim);
    if (qdim != dim) die("query and base dimensions differ");
    HostIndex h = load_index(res, dim, pq_m);

    cudaStream_t init;
    check_cuda(cudaStreamCreate(&init), "cudaStreamCreate");
    DevIndex idx;
    idx.upload(h, init);
    DevBuf<float> d_base((size_t)nbase * dim);
    d_base.upload(base.data(), base.size(), init);
    check_cuda(cudaStreamSynchronize(init), "index upload");
    cudaStreamDestroy(init);
    std::cout << "Index: " << h.nlist << " lists, " << h.total << " vectors, dim " << dim << ", pq_m " << pq_m
              << (p.ref_compat ? " (reference-compatible search)" : " (intended search)") << std::endl;

    double elapsed_ms = 0;
    StageTimes t;
    std::vector<int32_t> results;
    {
        SearchPipeline pipe(idx, d_base.p, nbase, p, batch, nstreams, nq, fused, graph);
        // warm-up: one batch per stream context
        for (int i = 0; i < nstreams; ++i) pipe.submit(queries.data(), (int)std::min<int64_t>(nq, batch), 0);
        pipe.wait_all();
        pipe.reset_times();
        const auto t0 = std::chrono::steady_clock::now();
        for (int r = 0; r < repeat; ++r)
            for (int64_t s = 0; s < nq; s += batch)
                pipe.submit(queries.data() + (size_t)s * dim, (int)std::min<int64_t>(batch, nq - s), s);
        pipe.wait_all();
        elapsed_ms = std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
        t = pipe.times();
        results = pipe.results();
    }
    const double qps = (double)nq * repeat / (elapsed_ms / 1000.0);
    std::cout << "\nTotal time: " << elapsed_ms << " ms, QPS: " << qps << std::endl;
    const double nb = t.batches ? (double)t.batches : 1.0;
    std::cout << std::fixed << std::setprecision(3) << "\n=========== Per-batch stage times (avg, ms) ===========\n"
              << "  H2D copy:      " << t.h2d / nb << "\n"
              << "  Coarse search: " << t.coarse / nb << "\n"
              << "  Candidates:    " << t.batch / nb << (fused ? "  (fused: whole search above)" : "")
              << (graph ? "  (graph replays: stages not timed separately)" : "") << "\n"
              << "  Rerank:        " << t.rerank / nb << "\n"
              << "  D2H copy:      " << t.d2h / nb << "\n"
              << "  E2E per batch: " << t.e2e / nb << "\n"
              << "  batches:       " << t.batches << "\n";
    if (!fused) std::cout << "  candidates per query: " << (double)t.candidates / ((double)nq * repeat) << "\n";
    std::cout << "======================================================" << std::endl;
    const std::string out = a.gets({"--out"}, "");
    if (!out.empty()) write_vecs(out, results.data(), nq, p.final_k);
    std::cout << std::defaultfloat << std::setprecision(6);
    if (a.pos.size() >= 3) {
        std::vector<int32_t> gt;
        int gt_k = 0;
        const int64_t ngt = read_vecs(a.pos[2], gt, gt_k);
        if (ngt < nq) die("ground truth has fewer rows than queries");
        const double r1 = recall_at(results, p.final_k, gt, gt_k, nq, 1);
        const double r10 = recall_at(results, p.final_k, gt, gt_k, nq, std::min(10, p.final_k));
        std::cout << "Recall@1: " << r1 * 100 << "%, Recall@10: " << r10 * 100 << "%" << std::endl;
        std::cout << "RESULT qps=" << qps << " recall1=" << r1 << " recall10=" << r10 << std::endl;
    } else {
        std::cout << "RESULT qps=" << qps << std::endl;
    }
    return 0;
}
