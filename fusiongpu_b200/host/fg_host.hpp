// fg_host.hpp -- host-side helpers shared by the C++ programs that mirror the
// reference's executables (build_global, search_pipeline, tune_parameters):
// the .fvecs/.ivecs/.bvecs readers and writers (utils.h:21-96), the
// ivf_data.bin / global_pq_codebook.bin layout (build_global.cu:242-252,
// search_pipeline.cu:481-529), a device buffer, and status checks.
//
// The dimension is read from the files instead of a compile-time DIM, and
// PQ_M is a command-line option: one binary serves every configuration.
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <string>
#include <vector>

#include "fusiongpu.h"

namespace fghost {

[[noreturn]] inline void die(const std::string& msg) {
    std::fprintf(stderr, "error: %s\n", msg.c_str());
    std::exit(1);
}

inline void check(int rc, const char* what) {
    if (rc != FG_OK) die(std::string(what) + ": " + fg_last_error());
}

inline void check_cuda(cudaError_t e, const char* what) {
    if (e != cudaSuccess) die(std::string(what) + ": " + cudaGetErrorString(e));
}

// A vector file: n records of [int32 d][d elements of T].  Every record must
// have the same d (the reference checks the first against DIM).
template <class T>
int64_t read_vecs(const std::string& path, std::vector<T>& out, int& d, int64_t max_n = -1) {
    std::ifstream f(path, std::ios::binary);
    if (!f) die("cannot open " + path);
    int32_t d0 = 0;
    if (!f.read(reinterpret_cast<char*>(&d0), 4) || d0 <= 0) die("bad header in " + path);
    f.seekg(0, std::ios::end);
    const int64_t bytes = f.tellg();
    const int64_t rec = 4 + (int64_t)d0 * (int64_t)sizeof(T);
    if (bytes % rec) die(path + ": size is not a whole number of records");
    int64_t n = bytes / rec;
    if (max_n >= 0 && n > max_n) n = max_n;
    f.seekg(0, std::ios::beg);
    out.resize((size_t)n * d0);
    for (int64_t i = 0; i < n; ++i) {
        int32_t di = 0;
        f.read(reinterpret_cast<char*>(&di), 4);
        if (di != d0) die(path + ": records of different dimensions");
        f.read(reinterpret_cast<char*>(out.data() + (size_t)i * d0), (std::streamsize)d0 * sizeof(T));
    }
    if (!f) die("short read in " + path);
    d = d0;
    return n;
}

// Base vectors as float: .fvecs as is, .bvecs (uint8) widened.
inline int64_t read_base(const std::string& path, std::vector<float>& out, int& d, int64_t max_n = -1) {
    if (path.size() > 6 && path.compare(path.size() - 6, 6, ".bvecs") == 0) {
        std::vector<uint8_t> b;
        const int64_t n = read_vecs(path, b, d, max_n);
        out.resize(b.size());
        for (size_t i = 0; i < b.size(); ++i) out[i] = (float)b[i];
        return n;
    }
    return read_vecs(path, out, d, max_n);
}

template <class T>
void write_vecs(const std::string& path, const T* x, int64_t n, int d) {
    std::ofstream f(path, std::ios::binary);
    if (!f) die("cannot write " + path);
    for (int64_t i = 0; i < n; ++i) {
        const int32_t dd = d;
        f.write(reinterpret_cast<const char*>(&dd), 4);
        f.write(reinterpret_cast<const char*>(x + (size_t)i * d), (std::streamsize)d * sizeof(T));
    }
}

// The index files: ivf_data.bin = [int32 total][int32 nlist][int32 offsets
// [nlist+1]][int32 ids [total]][uint8 codes [total][pq_m]][float centroids
// [nlist][dim]]; global_pq_codebook.bin = float [pq_m][256][dim/pq_m].
struct HostIndex {
    int dim = 0, pq_m = 0, nlist = 0, total = 0;
    std::vector<int32_t> offsets, ids;
    std::vector<uint8_t> codes;
    std::vector<float> centroids, codebook;
};

inline void save_index(const std::string& dir, const HostIndex& h) {
    {
        std::ofstream f(dir + "/ivf_data.bin", std::ios::binary);
        if (!f) die("cannot write " + dir + "/ivf_data.bin");
        f.write(reinterpret_cast<const char*>(&h.total), 4);
        f.write(reinterpret_cast<const char*>(&h.nlist), 4);
        f.write(reinterpret_cast<const char*>(h.offsets.data()), (std::streamsize)h.offsets.size() * 4);
        f.write(reinterpret_cast<const char*>(h.ids.data()), (std::streamsize)h.ids.size() * 4);
        f.write(reinterpret_cast<const char*>(h.codes.data()), (std::streamsize)h.codes.size());
        f.write(reinterpret_cast<const char*>(h.centroids.data()), (std::streamsize)h.centroids.size() * 4);
    }
    std::ofstream f(dir + "/global_pq_codebook.bin", std::ios::binary);
    if (!f) die("cannot write " + dir + "/global_pq_codebook.bin");
    f.write(reinterpret_cast<const char*>(h.codebook.data()), (std::streamsize)h.codebook.size() * 4);
}

inline HostIndex load_index(const std::string& dir, int dim, int pq_m) {
    HostIndex h;
    h.dim = dim;
    h.pq_m = pq_m;
    std::ifstream f(dir + "/ivf_data.bin", std::ios::binary);
    if (!f) die("cannot open " + dir + "/ivf_data.bin");
    f.read(reinterpret_cast<char*>(&h.total), 4);
    f.read(reinterpret_cast<char*>(&h.nlist), 4);
    if (!f || h.total < 0 || h.nlist < 1) die("bad ivf_data.bin header");
    h.offsets.resize((size_t)h.nlist + 1);
    h.ids.resize((size_t)h.total);
    h.codes.resize((size_t)h.total * pq_m);
    h.centroids.resize((size_t)h.nlist * dim);
    f.read(reinterpret_cast<char*>(h.offsets.data()), (std::streamsize)h.offsets.size() * 4);
    f.read(reinterpret_cast<char*>(h.ids.data()), (std::streamsize)h.ids.size() * 4);
    f.read(reinterpret_cast<char*>(h.codes.data()), (std::streamsize)h.codes.size());
    f.read(reinterpret_cast<char*>(h.centroids.data()), (std::streamsize)h.centroids.size() * 4);
    if (!f) die("ivf_data.bin is shorter than its header says (wrong --pq_m or dimension?)");
    f.peek();
    if (!f.eof()) die("ivf_data.bin is longer than its header says (wrong --pq_m or dimension?)");
    if (h.offsets[0] != 0 || h.offsets[h.nlist] != h.total) die("ivf_data.bin: offsets do not cover the lists");
    std::ifstream g(dir + "/global_pq_codebook.bin", std::ios::binary | std::ios::ate);
    if (!g) die("cannot open " + dir + "/global_pq_codebook.bin");
    const size_t want = (size_t)pq_m * 256 * (dim / pq_m) * 4;
    if ((size_t)g.tellg() != want) die("global_pq_codebook.bin does not hold pq_m x 256 x dim/pq_m floats");
    g.seekg(0);
    h.codebook.resize(want / 4);
    g.read(reinterpret_cast<char*>(h.codebook.data()), (std::streamsize)want);
    return h;
}

template <class T>
struct DevBuf {
    T* p = nullptr;
    size_t n = 0;
    DevBuf() = default;
    explicit DevBuf(size_t count) { resize(count); }
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    ~DevBuf() {
        if (p) cudaFree(p);
    }
    void resize(size_t count) {
        if (p) cudaFree(p);
        p = nullptr;
        n = count;
        if (count) check_cuda(cudaMalloc(&p, count * sizeof(T)), "cudaMalloc");
    }
    void upload(const T* src, size_t count, cudaStream_t s = nullptr) {
        check_cuda(cudaMemcpyAsync(p, src, count * sizeof(T), cudaMemcpyHostToDevice, s), "H2D copy");
    }
    void download(T* dst, size_t count, cudaStream_t s = nullptr) const {
        check_cuda(cudaMemcpyAsync(dst, p, count * sizeof(T), cudaMemcpyDeviceToHost, s), "D2H copy");
    }
};

// A device copy of an index with the view the C ABI takes.
struct DevIndex {
    DevBuf<float> codebook, centroids;
    DevBuf<int32_t> offsets, ids;
    DevBuf<uint8_t> codes;
    fg_ivfpq_view view{};

    void upload(const HostIndex& h, cudaStream_t s) {
        codebook.resize(h.codebook.size());
        codebook.upload(h.codebook.data(), h.codebook.size(), s);
        centroids.resize(h.centroids.size());
        centroids.upload(h.centroids.data(), h.centroids.size(), s);
        offsets.resize(h.offsets.size());
        offsets.upload(h.offsets.data(), h.offsets.size(), s);
        ids.resize(std::max<size_t>(1, h.ids.size()));
        ids.upload(h.ids.data(), h.ids.size(), s);
        codes.resize(std::max<size_t>(16, h.codes.size()));
        codes.upload(h.codes.data(), h.codes.size(), s);
        int lmax = 0;
        for (int c = 0; c < h.nlist; ++c) lmax = std::max(lmax, h.offsets[c + 1] - h.offsets[c]);
        view = fg_ivfpq_view{codebook.p, offsets.p, codes.p, ids.p, centroids.p, h.nlist, h.dim, h.pq_m, h.total, lmax};
    }
};

// Command-line scan in the reference's style: flags with one value each,
// positional arguments in order.
struct Args {
    std::vector<std::string> pos;
    std::vector<std::pair<std::string, std::string>> kv;
    std::vector<std::string> flags;

    Args(int argc, char** argv, const std::vector<std::string>& switches) {
        for (int i = 1; i < argc; ++i) {
            std::string a = argv[i];
            if (a.size() > 1 && a[0] == '-' && !(a[1] >= '0' && a[1] <= '9')) {
                bool sw = false;
                for (const auto& s : switches) sw |= (s == a);
                if (sw) {
                    flags.push_back(a);
                } else if (i + 1 < argc) {
                    kv.emplace_back(a, argv[++i]);
                } else {
                    die("option " + a + " needs a value");
                }
            } else {
                pos.push_back(a);
            }
        }
    }
    bool has(const std::string& name) const {
        for (const auto& f : flags)
            if (f == name) return true;
        return false;
    }
    const char* get(std::initializer_list<const char*> names) const {
        const char* v = nullptr;
        for (const auto& p : kv)
            for (const char* nm : names)
                if (p.first == nm) v = p.second.c_str();
        return v;
    }
    int geti(std::initializer_list<const char*> names, int def) const {
        const char* v = get(names);
        return v ? std::atoi(v) : def;
    }
    float getf(std::initializer_list<const char*> names, float def) const {
        const char* v = get(names);
        return v ? (float)std::atof(v) : def;
    }
    std::string gets(std::initializer_list<const char*> names, const std::string& def) const {
        const char* v = get(names);
        return v ? std::string(v) : def;
    }
};

// recall@k as the reference counts it (search_pipeline.cu:530-556): hits of
// the first k distinct returned ids in the query's gt_k ground-truth ids,
// over nq * k.
inline double recall_at(const std::vector<int32_t>& res, int res_k, const std::vector<int32_t>& gt, int gt_k,
                        int64_t nq, int k) {
    int64_t hits = 0;
    std::vector<int32_t> seen;
    for (int64_t q = 0; q < nq; ++q) {
        seen.clear();
        const int32_t* g = gt.data() + (size_t)q * gt_k;
        const int ck = std::min(k, res_k);
        for (int j = 0; j < ck; ++j) {
            const int32_t id = res[(size_t)q * res_k + j];
            bool dup = false;
            for (int32_t s : seen) dup |= (s == id);
            if (dup) continue;
            seen.push_back(id);
            for (int t = 0; t < gt_k; ++t)
                if (g[t] == id) {
                    ++hits;
                    break;
                }
        }
    }
    return nq ? (double)hits / ((double)nq * k) : 0.0;
}

}  // namespace fghost
