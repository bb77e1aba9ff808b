// build.cu -- index build on the GPU: k-means (assign + ordered update),
// stable sort of points by list, residual PQ training and encoding, list
// assembly.  Replaces kmeans_gpu.cuh:37-116,197-324,403-508, pq_utils.h:17-138
// and build_global.cu:226-240.
//
// The centroid update never adds floats atomically: points are first put in
// list order (a stable counting sort: per-chunk histograms with integer
// atomics, a deterministic scan, and a warp-per-chunk scatter that keeps
// point order), then one warp per cluster sums its members in point order in
// double and rounds once.  Results are therefore reproducible run to run and
// equal to the CPU oracle's.
#include <algorithm>
#include <cmath>
#include <deque>
#include <vector>

#include "fg_common.cuh"

namespace fg {

int l2_argmin(const float* X, long long nx, const float* Y, int ny, int dim, int32_t* amin, cudaStream_t s);
bool coarse_tc_supported(int dim, int P);
size_t assign_tc_workspace(long long n, int k, int dim);
int assign_tc(const float* X, long long n, int dim, const float* C, int k, int32_t* out, void* ws, size_t ws_bytes,
              cudaStream_t s);

// Nearest centroid of every point: the tensor-core path for dim <= 128 when the
// workspace holds it, else the exact CUDA-core tiles (identical results).
bool assign_on_tc(long long n, int k, int dim) { return coarse_tc_supported(dim, 1) && k >= 64 && n >= 4096; }

size_t assign_workspace(long long n, int k, int dim) {
    return assign_on_tc(n, k, dim) ? assign_tc_workspace(n, k, dim) : 0;
}

int assign_auto(const float* X, long long n, int dim, const float* C, int k, int32_t* out, void* ws, size_t ws_bytes,
                cudaStream_t s) {
    if (assign_on_tc(n, k, dim) && ws && ws_bytes >= assign_tc_workspace(n, k, dim))
        return assign_tc(X, n, dim, C, k, out, ws, ws_bytes, s);
    return l2_argmin(X, n, C, k, dim, out, s);
}

// ---- MT19937 on the host (seeding only; k or `sample` draws) -------------------

struct Mt19937 {
    uint32_t mt[624];
    int i = 624;
    explicit Mt19937(uint32_t seed) {
        mt[0] = seed;
        for (int j = 1; j < 624; ++j) mt[j] = 1812433253u * (mt[j - 1] ^ (mt[j - 1] >> 30)) + (uint32_t)j;
    }
    uint32_t next() {
        if (i >= 624) {
            for (int k = 0; k < 624; ++k) {
                uint32_t y = (mt[k] & 0x80000000u) | (mt[(k + 1) % 624] & 0x7fffffffu);
                mt[k] = mt[(k + 397) % 624] ^ (y >> 1) ^ ((y & 1u) ? 0x9908b0dfu : 0u);
            }
            i = 0;
        }
        uint32_t y = mt[i++];
        y ^= y >> 11;
        y ^= (y << 7) & 0x9d2c5680u;
        y ^= (y << 15) & 0xefc60000u;
        y ^= y >> 18;
        return y;
    }
};

// Row i = (i*stride + r_i % stride) % n, stride = max(1, n/k).
static void strided_rows(int64_t n, int k, uint32_t seed, std::vector<int64_t>& rows) {
    Mt19937 g(seed);
    const int64_t stride = std::max<int64_t>(1, n / k);
    rows.resize(k);
    for (int i = 0; i < k; ++i) rows[i] = ((int64_t)i * stride + (int64_t)(g.next() % (uint32_t)stride)) % n;
}

__global__ void gather_rows_kernel(const float* __restrict__ data, int dim, const int64_t* __restrict__ rows,
                                   int k, float* __restrict__ out) {
    const int i = blockIdx.x;
    if (i >= k) return;
    const float* src = data + (size_t)rows[i] * dim;
    for (int t = threadIdx.x; t < dim; t += blockDim.x) out[(size_t)i * dim + t] = src[t];
}

// Uniform integer in [0, range) from a 32-bit MT19937 by multiply-shift with
// rejection (D. Lemire, "Fast Random Integer Generation in an Interval", ACM
// TOMACS 29(1), 2019) -- how GCC's uniform_int_distribution bounds a 32-bit
// generator.
static uint32_t mt_below(Mt19937& g, uint32_t range) {
    uint64_t prod = (uint64_t)g.next() * range;
    uint32_t low = (uint32_t)prod;
    if (low < range) {
        const uint32_t thr = (0u - range) % range;
        while (low < thr) {
            prod = (uint64_t)g.next() * range;
            low = (uint32_t)prod;
        }
    }
    return (uint32_t)(prod >> 32);
}

// v = a permutation of 0..n-1: std::shuffle(iota, MT19937(seed)) as GCC's
// standard library performs it, the draw the reference's PQ trainer makes
// (pq_utils.h:24-26, :90-93).  Fisher-Yates: element i swaps with a uniform
// position in [0, i]; while the generator's range covers n*n, one draw in
// [0, (i+1)(i+2)) gives the positions of elements i and i+1 (quotient and
// remainder by i+2), after one draw in [0, 1] for element 1 when n is even.
static void std_shuffle_iota(int64_t n, uint32_t seed, std::vector<int32_t>& v) {
    v.resize(n);
    for (int64_t i = 0; i < n; ++i) v[i] = (int32_t)i;
    if (n <= 1) return;
    Mt19937 g(seed);
    if (0xffffffffull / (uint64_t)n >= (uint64_t)n) {
        int64_t i = 1;
        if (n % 2 == 0) {
            std::swap(v[1], v[mt_below(g, 2u)]);
            i = 2;
        }
        for (; i < n; i += 2) {
            const uint64_t b1 = (uint64_t)i + 2;
            const uint32_t x = mt_below(g, (uint32_t)(((uint64_t)i + 1) * b1));
            std::swap(v[i], v[x / b1]);
            std::swap(v[i + 1], v[x % b1]);
        }
        return;
    }
    for (int64_t i = 1; i < n; ++i) std::swap(v[i], v[mt_below(g, (uint32_t)(i + 1))]);
}

static int upload_rows(const std::vector<int64_t>& rows, int64_t* d_rows, cudaStream_t s) {
    // pageable source: cudaMemcpyAsync stages it before returning
    FG_CUDA_TRY(cudaMemcpyAsync(d_rows, rows.data(), rows.size() * sizeof(int64_t), cudaMemcpyHostToDevice, s));
    return FG_OK;
}

int kmeans_init(const float* data, int64_t n, int dim, int k, uint32_t seed, float* centroids, int64_t* d_rows,
                cudaStream_t s) {
    std::vector<int64_t> rows;
    strided_rows(n, k, seed, rows);
    int rc = upload_rows(rows, d_rows, s);
    if (rc) return rc;
    gather_rows_kernel<<<k, 128, 0, s>>>(data, dim, d_rows, k, centroids);
    rc = check_launch("gather_rows_kernel");
    if (rc) return rc;
    // `rows` must outlive the staged copy: the pageable copy has been staged on return
    return FG_OK;
}

// ---- stable counting sort of point ids by list --------------------------------

struct SortPlan {
    int64_t n;
    int k;
    int nchunk;
    int64_t chunk;
};

static SortPlan sort_plan(int64_t n, int k) {
    SortPlan p;
    p.n = n;
    p.k = k;
    int64_t want = std::max<int64_t>(1, (n + 4095) / 4096);
    const int64_t cap = std::max<int64_t>(1, (64ll << 20) / std::max(1, k));  // <= 256 MB of counters
    p.nchunk = (int)std::min<int64_t>({want, cap, 65535});
    p.chunk = (n + p.nchunk - 1) / p.nchunk;
    return p;
}

size_t sort_workspace(int64_t n, int k) {
    SortPlan p = sort_plan(n, k);
    return round_up((size_t)p.nchunk * k * sizeof(int32_t), 256) + 256;
}

__global__ void chunk_hist_kernel(const int32_t* __restrict__ assign, int64_t n, int64_t chunk, int k,
                                  int32_t* __restrict__ hist) {
    const int b = blockIdx.x;
    const int64_t s = (int64_t)b * chunk, e = min(n, s + chunk);
    int32_t* row = hist + (size_t)b * k;
    for (int64_t i = s + threadIdx.x; i < e; i += blockDim.x) {
        const int c = assign[i];
        if (c >= 0 && c < k) atomicAdd(row + c, 1);
    }
}

// offsets[c] = sum of earlier clusters; hist[b][c] becomes the first output
// position of chunk b's members of cluster c.
__global__ void chunk_scan_kernel(int32_t* __restrict__ hist, int nchunk, int k, int32_t* __restrict__ offsets) {
    __shared__ int warp[32];
    __shared__ int carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int c0 = 0; c0 < k; c0 += 1024) {
        const int c = c0 + threadIdx.x;
        int tot = 0;
        if (c < k)
            for (int b = 0; b < nchunk; ++b) tot += hist[(size_t)b * k + c];
        int all;
        const int pre = block_exclusive_scan<1024>(tot, warp, all);
        const int base = carry + pre;
        if (c < k) {
            offsets[c] = base;
            int run = base;
            for (int b = 0; b < nchunk; ++b) {
                const int h = hist[(size_t)b * k + c];
                hist[(size_t)b * k + c] = run;
                run += h;
            }
        }
        __syncthreads();
        if (threadIdx.x == 0) carry += all;
        __syncthreads();
    }
    if (threadIdx.x == 0) offsets[k] = carry;
}

// One warp per chunk walks its points in order, 32 at a time.
__global__ void chunk_scatter_kernel(const int32_t* __restrict__ assign, int64_t n, int64_t chunk, int k,
                                     int32_t* __restrict__ cursor, int nchunk, int32_t* __restrict__ order) {
    const int warp_id = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp_id >= nchunk) return;
    const int64_t s = (int64_t)warp_id * chunk, e = min(n, s + chunk);
    int32_t* row = cursor + (size_t)warp_id * k;
    for (int64_t i0 = s; i0 < e; i0 += 32) {
        const int64_t i = i0 + lane;
        const bool in = i < e;
        const unsigned act = __ballot_sync(0xffffffffu, in);
        int c = in ? assign[i] : -1;
        if (c < 0 || c >= k) c = -1;
        const unsigned peers = __match_any_sync(0xffffffffu, c);
        const int rank = __popc(peers & ((1u << lane) - 1u));
        int pos = 0;
        if (in && c >= 0) pos = row[c] + rank;
        __syncwarp();
        if (in && c >= 0) {
            order[pos] = (int32_t)i;
            if (rank == 0) row[c] += __popc(peers & act);
        }
        __syncwarp();
    }
}

int sort_by_list(const int32_t* assign, int64_t n, int k, int32_t* order, int32_t* offsets, void* ws,
                 size_t ws_bytes, cudaStream_t s) {
    FG_REQUIRE(n >= 0 && n <= 0x7fffffffll && k >= 1, "bad n/k");
    SortPlan p = sort_plan(n, k);
    Carve cv(ws, ws_bytes);
    int32_t* hist = cv.take<int32_t>((size_t)p.nchunk * k);
    if (!cv.ok()) return fail(FG_ERR_WORKSPACE, "sort_by_list workspace too small (%zu < %zu)", ws_bytes,
                              sort_workspace(n, k));
    FG_CUDA_TRY(cudaMemsetAsync(hist, 0, (size_t)p.nchunk * k * sizeof(int32_t), s));
    if (n > 0) {
        chunk_hist_kernel<<<p.nchunk, 256, 0, s>>>(assign, n, p.chunk, k, hist);
        int rc = check_launch("chunk_hist_kernel");
        if (rc) return rc;
    }
    chunk_scan_kernel<<<1, 1024, 0, s>>>(hist, p.nchunk, k, offsets);
    int rc = check_launch("chunk_scan_kernel");
    if (rc) return rc;
    if (n > 0) {
        const int warps_per_block = 4;
        chunk_scatter_kernel<<<(p.nchunk + warps_per_block - 1) / warps_per_block, 32 * warps_per_block, 0, s>>>(
            assign, n, p.chunk, k, hist, p.nchunk, order);
        rc = check_launch("chunk_scatter_kernel");
    }
    return rc;
}

// ---- centroid update: warp per cluster, members in point order, double sums ---

__global__ void kmeans_update_kernel(const float* __restrict__ data, int dim, const int32_t* __restrict__ order,
                                     const int32_t* __restrict__ offsets, int k, float* __restrict__ centroids) {
    const int c = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (c >= k) return;
    const int s = offsets[c], e = offsets[c + 1];
    if (e <= s) return;  // empty: keep the previous centroid
    for (int d0 = 0; d0 < dim; d0 += 128) {
        double acc[4] = {0.0, 0.0, 0.0, 0.0};
        for (int m = s; m < e; ++m) {
            const float* x = data + (size_t)order[m] * dim;
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const int j = d0 + lane + 32 * t;
                if (j < dim) acc[t] += (double)x[j];
            }
        }
        const double cnt = (double)(e - s);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int j = d0 + lane + 32 * t;
            if (j < dim) centroids[(size_t)c * dim + j] = (float)(acc[t] / cnt);
        }
    }
}

int kmeans_update(const float* data, int dim, const int32_t* order, const int32_t* offsets, int k, float* centroids,
                  cudaStream_t s) {
    const int wpb = 8;
    kmeans_update_kernel<<<(k + wpb - 1) / wpb, 32 * wpb, 0, s>>>(data, dim, order, offsets, k, centroids);
    return check_launch("kmeans_update_kernel");
}

size_t kmeans_workspace(int64_t n, int dim, int k) {
    return round_up((size_t)n * 4, 256) * 2 + round_up((size_t)(k + 1) * 4, 256) + round_up((size_t)k * 8, 256) +
           std::max(sort_workspace(n, k), assign_workspace(n, k, dim)) + 1024;
}

int kmeans(const float* data, int64_t n, int dim, int k, int iters, uint32_t seed, float* centroids, void* ws,
           size_t ws_bytes, cudaStream_t s) {
    FG_REQUIRE(n >= 1 && n <= 0x7fffffffll && dim >= 1 && k >= 1, "bad k-means shape");
    Carve cv(ws, ws_bytes);
    int32_t* as = cv.take<int32_t>((size_t)n);
    int32_t* order = cv.take<int32_t>((size_t)n);
    int32_t* offs = cv.take<int32_t>((size_t)k + 1);
    int64_t* rows = cv.take<int64_t>((size_t)k);
    const size_t used = round_up(cv.used, 256);
    if (!cv.ok() || used > ws_bytes) return fail(FG_ERR_WORKSPACE, "k-means workspace too small");
    void* sws = static_cast<char*>(ws) + used;
    const size_t sws_bytes = ws_bytes - used;
    int rc = kmeans_init(data, n, dim, k, seed, centroids, rows, s);
    for (int it = 0; it < iters && !rc; ++it) {
        rc = assign_auto(data, n, dim, centroids, k, as, sws, sws_bytes, s);
        if (!rc) rc = sort_by_list(as, n, k, order, offs, sws, sws_bytes, s);
        if (!rc) rc = kmeans_update(data, dim, order, offs, k, centroids, s);
    }
    if (!rc) {
        // the host row list behind the staged copy is gone; make sure the copy finished
        FG_CUDA_TRY(cudaStreamSynchronize(s));
    }
    return rc;
}

// ---- residual PQ training ----------------------------------------------------

// res[i][j] = data[row_i][j] - centroids[assign[row_i]][j]
__global__ void gather_residuals_kernel(const float* __restrict__ data, int dim, const int32_t* __restrict__ assign,
                                        const float* __restrict__ centroids, const int64_t* __restrict__ rows,
                                        int64_t S, float* __restrict__ res) {
    const int64_t i = blockIdx.x;
    if (i >= S) return;
    const int64_t r = rows[i];
    const float* x = data + (size_t)r * dim;
    const float* c = centroids + (size_t)assign[r] * dim;
    for (int t = threadIdx.x; t < dim; t += blockDim.x) res[(size_t)i * dim + t] = x[t] - c[t];
}

// subspace m, codeword kc <- res[row][m*sd .. +sd)
__global__ void pq_init_kernel(const float* __restrict__ res, int dim, int sd, const int64_t* __restrict__ rows,
                               int pq_m, float* __restrict__ codebook) {
    const int m = blockIdx.x;
    for (int kc = threadIdx.x; kc < 256; kc += blockDim.x) {
        const int64_t r = rows[(size_t)m * 256 + kc];
        for (int t = 0; t < sd; ++t)
            codebook[((size_t)m * 256 + kc) * sd + t] = res[(size_t)r * dim + m * sd + t];
    }
}

// assign[m][i] = nearest codeword of subspace m (exact, first minimum)
__global__ void pq_assign_kernel(const float* __restrict__ res, int64_t S, int dim, int sd,
                                 const float* __restrict__ codebook, int32_t* __restrict__ assign) {
    extern __shared__ float scb[];  // [256][sd]
    const int m = blockIdx.y;
    for (int t = threadIdx.x; t < 256 * sd; t += blockDim.x) scb[t] = codebook[(size_t)m * 256 * sd + t];
    __syncthreads();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= S) return;
    float x[16];
    for (int t = 0; t < sd; ++t) x[t] = res[(size_t)i * dim + m * sd + t];
    float best = FLT_MAX;
    int bk = 0;
    for (int kc = 0; kc < 256; ++kc) {
        float d = 0.0f;
        for (int t = 0; t < sd; ++t) {
            // `d += diff * diff` with two roundings, as the reference trainer
            // computes it (pq_utils.h:44-47; built without FMA contraction)
            const float df = x[t] - scb[kc * sd + t];
            d = __fadd_rn(d, __fmul_rn(df, df));
        }
        if (d < best) {
            best = d;
            bk = kc;
        }
    }
    assign[(size_t)m * S + i] = m * 256 + bk;
}

// one thread per (subspace, codeword, component); members in sample order
__global__ void pq_update_kernel(const float* __restrict__ res, int64_t S, int dim, int sd, int pq_m,
                                 const int32_t* __restrict__ order, const int32_t* __restrict__ offsets,
                                 float* __restrict__ codebook) {
    const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= (int64_t)pq_m * 256 * sd) return;
    const int t = (int)(g % sd);
    const int key = (int)(g / sd);  // m*256 + kc
    const int m = key / 256;
    const int s = offsets[key], e = offsets[key + 1];
    if (e <= s) return;
    double acc = 0.0;
    for (int u = s; u < e; ++u) {
        const int64_t i = order[u] - (int64_t)m * S;
        acc += (double)res[(size_t)i * dim + m * sd + t];
    }
    codebook[(size_t)key * sd + t] = (float)(acc / (double)(e - s));
}

size_t pq_train_workspace(int64_t n, int dim, int pq_m, int sample) {
    const int64_t S = std::min<int64_t>(sample, n);
    const int64_t items = S * pq_m;
    return round_up((size_t)S * dim * 4, 256) + round_up((size_t)std::max<int64_t>(S, (int64_t)pq_m * 256) * 8, 256) +
           round_up((size_t)items * 4, 256) * 2 + round_up(((size_t)pq_m * 256 + 1) * 4, 256) +
           sort_workspace(items, pq_m * 256) + 2048;
}

int pq_train(const float* data, int64_t n, int dim, const int32_t* assign, const float* centroids, int pq_m,
             int sample, int iters, float* codebook, void* ws, size_t ws_bytes, cudaStream_t s) {
    FG_REQUIRE(pq_m >= 1 && dim % pq_m == 0, "dim %d not divisible by pq_m %d", dim, pq_m);
    const int sd = dim / pq_m;
    FG_REQUIRE(sd <= 16, "sub_dim %d > 16", sd);
    const int64_t S = std::min<int64_t>(sample, n);
    FG_REQUIRE(S >= 256, "need at least 256 training vectors, have %lld", (long long)S);
    FG_REQUIRE(S * pq_m <= 0x7fffffffll, "sample * pq_m too large");
    Carve cv(ws, ws_bytes);
    float* res = cv.take<float>((size_t)S * dim);
    int64_t* rows = cv.take<int64_t>((size_t)std::max<int64_t>(S, (int64_t)pq_m * 256));
    int32_t* as = cv.take<int32_t>((size_t)S * pq_m);
    int32_t* order = cv.take<int32_t>((size_t)S * pq_m);
    int32_t* offs = cv.take<int32_t>((size_t)pq_m * 256 + 1);
    const size_t used = round_up(cv.used, 256);
    if (!cv.ok() || used > ws_bytes) return fail(FG_ERR_WORKSPACE, "pq_train workspace too small");
    void* sws = static_cast<char*>(ws) + used;
    const size_t sws_bytes = ws_bytes - used;

    // the sample: the first S rows of std::shuffle(0..n-1, MT19937(12345)),
    // residuals in that order (pq_utils.h:88-104)
    FG_REQUIRE(n <= 0x7fffffffll, "pq_train samples from at most 2^31 - 1 rows");
    std::vector<int64_t> hrows;
    {
        std::vector<int32_t> perm;
        std_shuffle_iota(n, 12345u, perm);
        hrows.assign(perm.begin(), perm.begin() + S);
    }
    int rc = upload_rows(hrows, rows, s);
    if (rc) return rc;
    gather_residuals_kernel<<<(unsigned)S, 128, 0, s>>>(data, dim, assign, centroids, rows, S, res);
    if ((rc = check_launch("gather_residuals_kernel"))) return rc;
    FG_CUDA_TRY(cudaStreamSynchronize(s));  // before the host row list is reused

    // subspace m starts from the sample rows at the first 256 positions of
    // std::shuffle(0..S-1, MT19937(1234 + m)) (pq_utils.h:20-31)
    std::vector<int64_t> init((size_t)pq_m * 256);
    for (int m = 0; m < pq_m; ++m) {
        std::vector<int32_t> r;
        std_shuffle_iota(S, 1234u + (uint32_t)m, r);
        std::copy(r.begin(), r.begin() + 256, init.begin() + (size_t)m * 256);
    }
    if ((rc = upload_rows(init, rows, s))) return rc;
    pq_init_kernel<<<pq_m, 256, 0, s>>>(res, dim, sd, rows, pq_m, codebook);
    if ((rc = check_launch("pq_init_kernel"))) return rc;
    for (int it = 0; it < iters; ++it) {
        dim3 grid((unsigned)((S + 255) / 256), pq_m);
        pq_assign_kernel<<<grid, 256, 256 * sd * sizeof(float), s>>>(res, S, dim, sd, codebook, as);
        if ((rc = check_launch("pq_assign_kernel"))) return rc;
        if ((rc = sort_by_list(as, S * pq_m, pq_m * 256, order, offs, sws, sws_bytes, s))) return rc;
        const int64_t th = (int64_t)pq_m * 256 * sd;
        pq_update_kernel<<<(unsigned)((th + 255) / 256), 256, 0, s>>>(res, S, dim, sd, pq_m, order, offs, codebook);
        if ((rc = check_launch("pq_update_kernel"))) return rc;
    }
    FG_CUDA_TRY(cudaStreamSynchronize(s));
    return FG_OK;
}

// ---- PQ encode ---------------------------------------------------------------------

__global__ void pq_encode_kernel(const float* __restrict__ data, int64_t n, int dim, int sd,
                                 const int32_t* __restrict__ assign, const float* __restrict__ centroids,
                                 const float* __restrict__ codebook, int pq_m, uint8_t* __restrict__ codes) {
    extern __shared__ float scb[];  // [256][sd] of subspace m
    const int m = blockIdx.y;
    for (int t = threadIdx.x; t < 256 * sd; t += blockDim.x) scb[t] = codebook[(size_t)m * 256 * sd + t];
    __syncthreads();
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float* x = data + (size_t)i * dim + m * sd;
    const float* c = centroids + (size_t)assign[i] * dim + m * sd;
    float r[16];
    for (int t = 0; t < sd; ++t) r[t] = x[t] - c[t];
    float best = FLT_MAX;
    int bk = 0;
    for (int kc = 0; kc < 256; ++kc) {
        float d = 0.0f;
        for (int t = 0; t < sd; ++t) {
            const float df = r[t] - scb[kc * sd + t];
            d = fmaf(df, df, d);
        }
        if (d < best) {
            best = d;
            bk = kc;
        }
    }
    codes[(size_t)i * pq_m + m] = (uint8_t)bk;
}

int pq_encode(const float* data, int64_t n, int dim, const int32_t* assign, const float* centroids,
              const float* codebook, int pq_m, uint8_t* codes, cudaStream_t s) {
    FG_REQUIRE(pq_m >= 1 && dim % pq_m == 0, "dim %d not divisible by pq_m %d", dim, pq_m);
    const int sd = dim / pq_m;
    FG_REQUIRE(sd <= 16, "sub_dim %d > 16", sd);
    if (n == 0) return FG_OK;
    dim3 grid((unsigned)((n + 255) / 256), pq_m);
    pq_encode_kernel<<<grid, 256, 256 * sd * sizeof(float), s>>>(data, n, dim, sd, assign, centroids, codebook,
                                                                  pq_m, codes);
    return check_launch("pq_encode_kernel");
}

__global__ void gather_lists_kernel(const uint8_t* __restrict__ codes, int64_t n, int pq_m,
                                    const int32_t* __restrict__ order, uint8_t* __restrict__ out_codes,
                                    int32_t* __restrict__ out_ids) {
    const int64_t r = blockIdx.x;
    if (r >= n) return;
    const int32_t src = order[r];
    if (threadIdx.x == 0) out_ids[r] = src;
    for (int t = threadIdx.x; t < pq_m; t += blockDim.x) out_codes[(size_t)r * pq_m + t] = codes[(size_t)src * pq_m + t];
}

int gather_lists(const uint8_t* codes, int64_t n, int pq_m, const int32_t* order, uint8_t* out_codes,
                 int32_t* out_ids, cudaStream_t s) {
    if (n == 0) return FG_OK;
    gather_lists_kernel<<<(unsigned)n, 64, 0, s>>>(codes, n, pq_m, order, out_codes, out_ids);
    return check_launch("gather_lists_kernel");
}

// ---- list rebalancing (build_global.cu:62-169) --------------------------------
//
// Oversized lists are split by a local k-means until every list holds at most
// twice the mean.  The control flow is the reference's FIFO work queue and
// runs on the host; each split gathers the list's rows on the device, runs
// k-means (sub_k centroids, `iters` Lloyd steps, the same strided seeding) and
// the exact assignment there.  Lists are kept with ids ascending, so the
// result is a pure function of the inputs.

namespace {

struct DevMem {
    void* p = nullptr;
    ~DevMem() {
        if (p) cudaFree(p);
    }
    int alloc(size_t bytes) {
        if (p) cudaFree(p);
        p = nullptr;
        if (bytes && cudaMalloc(&p, bytes) != cudaSuccess)
            return fail(FG_ERR_CUDA, "cudaMalloc of %zu bytes failed", bytes);
        return FG_OK;
    }
};

struct Bucket {
    std::vector<int32_t> ids;  // ascending point ids
    std::vector<float> centroid;
};

}  // namespace

int rebalance(const float* data, int64_t n, int dim, const int32_t* assign, const float* centroids, int k, int iters,
              uint32_t seed, int32_t* out_assign, float* out_centroids, int cap, int32_t* out_nlist,
              cudaStream_t s) {
    FG_REQUIRE(n >= 1 && n <= 0x7fffffffll && dim >= 1 && k >= 1 && iters >= 0 && cap >= 0, "bad rebalance shape");
    FG_REQUIRE(data && assign && centroids && out_assign && out_nlist && (out_centroids || cap == 0),
               "null buffer");
    std::vector<int32_t> a((size_t)n);
    std::vector<float> cen((size_t)k * dim);
    FG_CUDA_TRY(cudaMemcpyAsync(a.data(), assign, (size_t)n * 4, cudaMemcpyDeviceToHost, s));
    FG_CUDA_TRY(cudaMemcpyAsync(cen.data(), centroids, cen.size() * 4, cudaMemcpyDeviceToHost, s));
    FG_CUDA_TRY(cudaStreamSynchronize(s));

    std::vector<int64_t> count((size_t)k, 0);
    for (int64_t i = 0; i < n; ++i) {
        FG_REQUIRE(a[i] >= 0 && a[i] < k, "assignment %d of point %lld outside [0, %d)", a[i], (long long)i, k);
        ++count[a[i]];
    }
    const double avg = (double)n / k;
    const size_t split_above = (size_t)(avg * 2);
    const size_t min_split = 32;

    std::deque<Bucket> queue;
    {
        std::vector<Bucket> init((size_t)k);
        for (int c = 0; c < k; ++c) init[c].ids.reserve((size_t)count[c]);
        for (int64_t i = 0; i < n; ++i) init[a[i]].ids.push_back((int32_t)i);
        for (int c = 0; c < k; ++c) {
            if (init[c].ids.empty()) continue;
            init[c].centroid.assign(cen.begin() + (size_t)c * dim, cen.begin() + (size_t)(c + 1) * dim);
            queue.push_back(std::move(init[c]));
        }
    }

    // device scratch sized for the largest list that can be split (children
    // are never larger than their parent)
    size_t big = 0;
    for (const Bucket& b : queue) big = std::max(big, b.ids.size());
    const int big_k = (int)std::max<int64_t>(2, (int64_t)std::ceil((double)big / avg));
    DevMem d_rows, d_sub, d_cen, d_as, d_ws;
    bool have_scratch = false;
    std::vector<int64_t> rows;
    std::vector<int32_t> sub_as;
    std::vector<float> sub_cen;

    std::vector<Bucket> done;
    int rc = FG_OK;
    while (!queue.empty() && rc == FG_OK) {
        Bucket b = std::move(queue.front());
        queue.pop_front();
        const size_t sz = b.ids.size();
        if (sz <= split_above || sz < min_split) {
            done.push_back(std::move(b));
            continue;
        }
        int sub_k = (int)std::ceil((double)sz / avg);
        if (sub_k < 2) sub_k = 2;
        if (sub_k > (int)sz / 2) sub_k = (int)sz / 2;
        if (!have_scratch) {
            if ((rc = d_rows.alloc(big * 8)) || (rc = d_sub.alloc(big * dim * 4)) ||
                (rc = d_cen.alloc((size_t)big_k * dim * 4)) || (rc = d_as.alloc(big * 4)) ||
                (rc = d_ws.alloc(kmeans_workspace((int64_t)big, dim, big_k))))
                break;
            have_scratch = true;
        }
        rows.assign(b.ids.begin(), b.ids.end());
        if ((rc = upload_rows(rows, static_cast<int64_t*>(d_rows.p), s))) break;
        gather_rows_kernel<<<(unsigned)sz, 128, 0, s>>>(data, dim, static_cast<int64_t*>(d_rows.p), (int)sz,
                                                        static_cast<float*>(d_sub.p));
        if ((rc = check_launch("gather_rows_kernel"))) break;
        float* sc = static_cast<float*>(d_cen.p);
        if ((rc = kmeans(static_cast<float*>(d_sub.p), (int64_t)sz, dim, sub_k, iters, seed, sc, d_ws.p,
                         kmeans_workspace((int64_t)big, dim, big_k), s)))
            break;
        if ((rc = l2_argmin(static_cast<float*>(d_sub.p), (long long)sz, sc, sub_k, dim,
                            static_cast<int32_t*>(d_as.p), s)))
            break;
        sub_as.resize(sz);
        sub_cen.resize((size_t)sub_k * dim);
        FG_CUDA_TRY(cudaMemcpyAsync(sub_as.data(), d_as.p, sz * 4, cudaMemcpyDeviceToHost, s));
        FG_CUDA_TRY(cudaMemcpyAsync(sub_cen.data(), sc, sub_cen.size() * 4, cudaMemcpyDeviceToHost, s));
        FG_CUDA_TRY(cudaStreamSynchronize(s));
        std::vector<Bucket> kids((size_t)sub_k);
        for (size_t i = 0; i < sz; ++i) kids[sub_as[i]].ids.push_back(b.ids[i]);
        int nonempty = 0;
        for (const Bucket& kb : kids) nonempty += kb.ids.empty() ? 0 : 1;
        for (int c = 0; c < sub_k; ++c) {
            if (kids[c].ids.empty()) continue;
            kids[c].centroid.assign(sub_cen.begin() + (size_t)c * dim, sub_cen.begin() + (size_t)(c + 1) * dim);
            // a split that leaves every point in one child would repeat forever
            // (all points equal); that child is final
            if (nonempty == 1)
                done.push_back(std::move(kids[c]));
            else
                queue.push_back(std::move(kids[c]));
        }
    }
    if (rc) return rc;

    const int nl = (int)done.size();
    *out_nlist = nl;
    if (nl > cap) return fail(FG_ERR_WORKSPACE, "rebalancing made %d lists; out_centroids holds %d", nl, cap);
    std::vector<int32_t> na((size_t)n);
    std::vector<float> nc((size_t)nl * dim);
    for (int c = 0; c < nl; ++c) {
        for (int32_t id : done[c].ids) na[id] = c;
        std::copy(done[c].centroid.begin(), done[c].centroid.end(), nc.begin() + (size_t)c * dim);
    }
    FG_CUDA_TRY(cudaMemcpyAsync(out_assign, na.data(), (size_t)n * 4, cudaMemcpyHostToDevice, s));
    FG_CUDA_TRY(cudaMemcpyAsync(out_centroids, nc.data(), nc.size() * 4, cudaMemcpyHostToDevice, s));
    FG_CUDA_TRY(cudaStreamSynchronize(s));
    return FG_OK;
}

}  // namespace fg
