// graph.cu -- fixed-degree k-NN graph index: build and CAGRA-style traversal.
//
// The reference searches a CAGRA graph only over its centroids, through cuVS
// (cagra_adapter.cuh:10-68, library code absent here).  This is the graph
// index of the C4 configuration (1M x 768 fp16, inner product, degree 64,
// itopk 128, search width 4), built and searched by our own kernels after the
// published CAGRA design (Ootomo et al., ICDE 2024):
//
// build   1. IVF partition: k-means (L2) + exact assignment, lists sorted by id.
//         2. Initial k-NN graph of degree I from IVF candidates: the
//            neighbours of a point are searched exactly (metric distance, fmaf
//            in dimension order) among the members of its list's P nearest
//            lists; ties by id; the point itself is dropped.
//         3. Rank-based pruning: for neighbour v_i (rank i) of u, count the
//            detours u -> v_j -> v_i with j < i and rank(v_i in N(v_j)) < i;
//            keep the D neighbours with the fewest detours (ties by rank).
//         4. Reverse edges: v collects every u whose pruned list holds v, in
//            (rank of v in u's list, u) order.
//         5. Final list: the first D/2 pruned neighbours, then up to D/2
//            reverse neighbours not yet present, then the remaining pruned
//            neighbours, deduplicated; -1 pads a short list.
//
// search  One CTA per query.  An internal top list of `itopk` (distance, id)
//         entries with explored flags; each iteration takes the first
//         `search_width` unexplored entries as parents, gathers their D
//         neighbours, drops those already visited (4096-slot open-addressing
//         hash in shared memory, reset to the current top list when half full),
//         computes the new distances (one warp per vector, 16-byte loads,
//         fixed reduction order), sorts them and merges them into the top
//         list (merge path).  Starts from search_width*D pseudo-random nodes
//         and stops when no unexplored entry is left or after max_iterations.
#include <cuda_fp16.h>

#include <algorithm>
#include <vector>

#include "fg_common.cuh"

namespace fg {

int sort_by_list(const int32_t* assign, int64_t n, int k, int32_t* order, int32_t* offsets, void* ws, size_t ws_bytes,
                 cudaStream_t s);
size_t sort_workspace(int64_t n, int k);
size_t kmeans_workspace(int64_t n, int dim, int k);
int kmeans(const float* data, int64_t n, int dim, int k, int iters, uint32_t seed, float* centroids, void* ws,
           size_t ws_bytes, cudaStream_t s);
int l2_argmin(const float* X, long long nx, const float* Y, int ny, int dim, int32_t* amin, cudaStream_t s);
int knn_like(const float* Y, long long ny, int dim, const float* Q, long long nq, int k, int32_t* out_i, float* out_v,
             void* ws, size_t ws_bytes, cudaStream_t s, int metric);
size_t knn_like_workspace(long long nq, int ncols, int k);

namespace {

struct DevMem {
    void* p = nullptr;
    size_t bytes = 0;
    ~DevMem() {
        if (p) cudaFree(p);
    }
    int alloc(size_t b) {
        if (b <= bytes && p) return FG_OK;
        if (p) cudaFree(p);
        p = nullptr;
        bytes = 0;
        if (b && cudaMalloc(&p, b) != cudaSuccess) return fail(FG_ERR_CUDA, "cudaMalloc of %zu bytes failed", b);
        bytes = b;
        return FG_OK;
    }
    template <class T>
    T* as() const {
        return static_cast<T*>(p);
    }
};

}  // namespace

// ============================== build ==========================================

__global__ void half_to_float_kernel(const __half* __restrict__ in, long long n, float* __restrict__ out) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __half2float(in[i]);
}

__global__ void gather_rows32_kernel(const float* __restrict__ X, int dim, const int32_t* __restrict__ rows, int nr,
                                     float* __restrict__ out) {
    const int r = blockIdx.x;
    if (r >= nr) return;
    const float* src = X + (size_t)rows[r] * dim;
    for (int t = threadIdx.x; t < dim; t += blockDim.x) out[(size_t)r * dim + t] = src[t];
}

// Column indices of the k-NN over a list's candidates -> global ids, the
// member itself dropped, first I kept (-1 padded).
__global__ void knn_rows_kernel(const int32_t* __restrict__ col, int kk, const int32_t* __restrict__ cand,
                                const int32_t* __restrict__ members, int nm, int I, int32_t* __restrict__ g0) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= nm) return;
    const int32_t self = members[r];
    int32_t* out = g0 + (size_t)self * I;
    int o = 0;
    for (int j = 0; j < kk && o < I; ++j) {
        const int32_t c = col[(size_t)r * kk + j];
        if (c < 0) continue;
        const int32_t id = cand[c];
        if (id == self) continue;
        out[o++] = id;
    }
    for (; o < I; ++o) out[o] = -1;
}

// Rank-based pruning of one node per CTA (blockDim = I rounded up to 32).
// CTAs take the nodes in IVF list order, so that the neighbour lists they
// read are shared by the CTAs running beside them (L2 reuse).
__global__ void prune_kernel(const int32_t* __restrict__ g0, const int32_t* __restrict__ node_order, long long n, int I,
                             int D, int32_t* __restrict__ pruned) {
    extern __shared__ __align__(16) int32_t gsm[];
    int32_t* nb = gsm;                 // [I]
    int32_t* wl = nb + I;              // [I]
    uint32_t* key = reinterpret_cast<uint32_t*>(wl + I);  // [next_pow2(I)]
    const long long u = node_order[blockIdx.x];
    const int i = threadIdx.x;
    const int ipow = next_pow2(I);
    if (i < I) nb[i] = g0[u * I + i];
    __syncthreads();
    const int32_t vi = i < I ? nb[i] : -1;
    int cnt = 0;
    for (int j = 0; j < I; ++j) {
        const int32_t w = nb[j];
        if (w < 0 || w >= n) continue;  // uniform: nb is shared
        __syncthreads();
        if (i < I) wl[i] = g0[(long long)w * I + i];
        __syncthreads();
        if (i > j && i < I && vi >= 0) {
            for (int x = 0; x < i; ++x)
                if (wl[x] == vi) {
                    ++cnt;
                    break;
                }
        }
    }
    __syncthreads();
    for (int t = i; t < ipow; t += blockDim.x) {
        uint32_t k = 0xffffffffu;
        if (t < I) k = nb[t] >= 0 ? ((uint32_t)min(cnt, 0xffff) << 16) | (uint32_t)t : (0xffffu << 16) | (uint32_t)t;
        if (t == i) key[t] = k;
        else if (t >= I) key[t] = 0xffffffffu;
    }
    __syncthreads();
    // bitonic sort of ipow keys by (detours, rank)
    for (int k2 = 2; k2 <= ipow; k2 <<= 1)
        for (int j2 = k2 >> 1; j2 > 0; j2 >>= 1) {
            for (int t = i; t < ipow; t += blockDim.x) {
                const int o = t ^ j2;
                if (o > t) {
                    const uint32_t a = key[t], b = key[o];
                    if ((a > b) == ((t & k2) == 0)) {
                        key[t] = b;
                        key[o] = a;
                    }
                }
            }
            __syncthreads();
        }
    for (int r = i; r < D; r += blockDim.x) {
        const uint32_t k = key[r];
        pruned[u * D + r] = (r < I && k != 0xffffffffu) ? nb[k & 0xffffu] : -1;
    }
}

// Entry node of each IVF list: the member nearest its centroid by the metric
// (fmaf in dimension order, ties by id); -1 for an empty list.  One warp per list.
__global__ void medoid_kernel(const float* __restrict__ X, int dim, const float* __restrict__ cen,
                              const int32_t* __restrict__ order, const int32_t* __restrict__ off, int L, int metric,
                              int32_t* __restrict__ entry) {
    const int c = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (c >= L) return;
    const float* y = cen + (size_t)c * dim;
    float best = FLT_MAX;
    int32_t bid = -1;
    for (int r = off[c] + lane; r < off[c + 1]; r += 32) {
        const int32_t id = order[r];
        const float* x = X + (size_t)id * dim;
        float acc = 0.0f;
        for (int j = 0; j < dim; ++j) {
            if (metric == FG_METRIC_IP) {
                acc = fmaf(x[j], y[j], acc);
            } else {
                const float df = x[j] - y[j];
                acc = fmaf(df, df, acc);
            }
        }
        const float d = metric == FG_METRIC_IP ? -acc : acc;
        if (d < best || (d == best && (bid < 0 || id < bid))) {
            best = d;
            bid = id;
        }
    }
    for (int o = 16; o; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int32_t oi = __shfl_xor_sync(0xffffffffu, bid, o);
        if (oi >= 0 && (bid < 0 || ob < best || (ob == best && oi < bid))) {
            best = ob;
            bid = oi;
        }
    }
    if (lane == 0) entry[c] = bid;
}

// edge e = i*n + u carries u -> pruned[u][i]; bucket n collects invalid edges
__global__ void edge_targets_kernel(const int32_t* __restrict__ pruned, long long n, int D, int32_t* __restrict__ tgt) {
    const long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= n * D) return;
    const int i = (int)(e / n);
    const long long u = e % n;
    const int32_t v = pruned[u * D + i];
    tgt[e] = (v >= 0 && v < n) ? v : (int32_t)n;
}

__device__ __forceinline__ bool has_id(const int32_t* row, int cnt, int32_t v) {
    for (int x = 0; x < cnt; ++x)
        if (row[x] == v) return true;
    return false;
}

__global__ void merge_graph_kernel(const int32_t* __restrict__ pruned, const int32_t* __restrict__ order,
                                   const int32_t* __restrict__ roff, long long n, int D, int32_t* __restrict__ graph) {
    const long long u = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (u >= n) return;
    int32_t* out = graph + u * D;
    const int32_t* pu = pruned + u * D;
    const int half = D / 2;
    int cnt = 0;
    for (int r = 0; r < half; ++r) {
        const int32_t v = pu[r];
        if (v >= 0 && !has_id(out, cnt, v)) out[cnt++] = v;
    }
    int taken = 0;
    for (int32_t e = roff[u]; e < roff[u + 1] && taken < D - half && cnt < D; ++e) {
        const int32_t src = (int32_t)((long long)order[e] % n);
        if (!has_id(out, cnt, src)) {
            out[cnt++] = src;
            ++taken;
        }
    }
    for (int r = half; r < D && cnt < D; ++r) {
        const int32_t v = pu[r];
        if (v >= 0 && !has_id(out, cnt, v)) out[cnt++] = v;
    }
    for (; cnt < D; ++cnt) out[cnt] = -1;
}

int graph_build(const void* data, int dtype, long long n, int dim, const fg_graph_build_params* p, int32_t* graph,
                float* entry_centroids, int32_t* entry_nodes, cudaStream_t s) {
    FG_REQUIRE(data && p && graph, "null argument");
    FG_REQUIRE(dtype == FG_DTYPE_F32 || dtype == FG_DTYPE_F16, "unknown dtype %d", dtype);
    FG_REQUIRE(p->metric == FG_METRIC_L2 || p->metric == FG_METRIC_IP, "unknown metric %d", p->metric);
    const int D = p->graph_degree, I = p->intermediate_degree, L = p->nlist, P = p->probe_lists;
    FG_REQUIRE(n >= 2 && n <= 0x3fffffffll && dim >= 1, "bad graph shape");
    FG_REQUIRE(D >= 2 && D % 2 == 0 && I >= D && I <= 1024, "need 2 <= degree (even) <= intermediate_degree <= 1024");
    FG_REQUIRE(L >= 1 && L <= n && P >= 1 && P <= L && p->kmeans_iters >= 0, "bad IVF parameters");
    FG_REQUIRE((long long)D * n <= 0x7fffffffll, "n * degree exceeds 2^31");
    int rc = FG_OK;
    DevMem xf, cen, as, order, offs, ws, cnn, cnd, cbuf, qbuf, mem, col, val, g0, pr, tgt, rord, roff;

    // fp32 view of the data
    const float* X = static_cast<const float*>(data);
    if (dtype == FG_DTYPE_F16) {
        if ((rc = xf.alloc((size_t)n * dim * 4))) return rc;
        const long long tot = n * dim;
        half_to_float_kernel<<<(unsigned)((tot + 255) / 256), 256, 0, s>>>(static_cast<const __half*>(data), tot,
                                                                          xf.as<float>());
        if ((rc = check_launch("half_to_float_kernel"))) return rc;
        X = xf.as<float>();
    }
    // 1. IVF partition
    const size_t wk = std::max(kmeans_workspace(n, dim, L), sort_workspace(n, L));
    if ((rc = cen.alloc((size_t)L * dim * 4)) || (rc = as.alloc((size_t)n * 4)) || (rc = order.alloc((size_t)n * 4)) ||
        (rc = offs.alloc((size_t)(L + 1) * 4)) || (rc = ws.alloc(wk)))
        return rc;
    if ((rc = kmeans(X, n, dim, L, p->kmeans_iters, p->seed, cen.as<float>(), ws.p, wk, s))) return rc;
    if ((rc = l2_argmin(X, n, cen.as<float>(), L, dim, as.as<int32_t>(), s))) return rc;
    if ((rc = sort_by_list(as.as<int32_t>(), n, L, order.as<int32_t>(), offs.as<int32_t>(), ws.p, wk, s))) return rc;
    // nearest lists of every list (L2 between centroids)
    const size_t wc = knn_like_workspace(L, L, P);
    if ((rc = cnn.alloc((size_t)L * P * 4)) || (rc = cnd.alloc((size_t)L * P * 4)) || (rc = ws.alloc(std::max(wk, wc))))
        return rc;
    if ((rc = knn_like(cen.as<float>(), L, dim, cen.as<float>(), L, P, cnn.as<int32_t>(), cnd.as<float>(), ws.p,
                       ws.bytes, s, FG_METRIC_L2)))
        return rc;
    std::vector<int32_t> h_order((size_t)n), h_off((size_t)L + 1), h_nn((size_t)L * P);
    FG_CUDA_TRY(cudaMemcpyAsync(h_order.data(), order.p, (size_t)n * 4, cudaMemcpyDeviceToHost, s));
    FG_CUDA_TRY(cudaMemcpyAsync(h_off.data(), offs.p, h_off.size() * 4, cudaMemcpyDeviceToHost, s));
    FG_CUDA_TRY(cudaMemcpyAsync(h_nn.data(), cnn.p, h_nn.size() * 4, cudaMemcpyDeviceToHost, s));
    FG_CUDA_TRY(cudaStreamSynchronize(s));

    // 2. initial k-NN graph from each list's candidate lists
    std::vector<std::vector<int32_t>> cands((size_t)L);
    size_t max_c = 0, max_m = 0;
    for (int c = 0; c < L; ++c) {
        std::vector<int> lists{c};
        for (int j = 0; j < P && (int)lists.size() < P; ++j)
            if (h_nn[(size_t)c * P + j] != c) lists.push_back(h_nn[(size_t)c * P + j]);
        std::vector<int32_t>& cc = cands[c];
        for (int l : lists) cc.insert(cc.end(), h_order.begin() + h_off[l], h_order.begin() + h_off[l + 1]);
        std::sort(cc.begin(), cc.end());
        max_c = std::max(max_c, cc.size());
        max_m = std::max(max_m, (size_t)(h_off[c + 1] - h_off[c]));
    }
    const int kk_max = (int)std::min<size_t>(max_c, (size_t)I + 1);
    const size_t wn = knn_like_workspace((long long)max_m, (int)max_c, kk_max);
    if ((rc = g0.alloc((size_t)n * I * 4)) || (rc = cbuf.alloc(max_c * dim * 4)) || (rc = qbuf.alloc(max_m * dim * 4)) ||
        (rc = cnd.alloc(max_c * 4)) || (rc = mem.alloc(max_m * 4)) || (rc = col.alloc(max_m * kk_max * 4)) ||
        (rc = val.alloc(max_m * kk_max * 4)) || (rc = ws.alloc(std::max({wk, wc, wn}))))
        return rc;
    FG_CUDA_TRY(cudaMemsetAsync(g0.p, 0xff, (size_t)n * I * 4, s));
    for (int c = 0; c < L; ++c) {
        const int nm = h_off[c + 1] - h_off[c];
        const int nc = (int)cands[c].size();
        if (nm == 0) continue;
        const int kk = std::min(nc, I + 1);
        FG_CUDA_TRY(cudaMemcpyAsync(cnd.p, cands[c].data(), (size_t)nc * 4, cudaMemcpyHostToDevice, s));
        FG_CUDA_TRY(cudaMemcpyAsync(mem.p, h_order.data() + h_off[c], (size_t)nm * 4, cudaMemcpyHostToDevice, s));
        gather_rows32_kernel<<<nc, 128, 0, s>>>(X, dim, cnd.as<int32_t>(), nc, cbuf.as<float>());
        gather_rows32_kernel<<<nm, 128, 0, s>>>(X, dim, mem.as<int32_t>(), nm, qbuf.as<float>());
        if ((rc = check_launch("gather_rows32_kernel"))) return rc;
        if ((rc = knn_like(cbuf.as<float>(), nc, dim, qbuf.as<float>(), nm, kk, col.as<int32_t>(), val.as<float>(),
                           ws.p, ws.bytes, s, p->metric)))
            return rc;
        knn_rows_kernel<<<(nm + 127) / 128, 128, 0, s>>>(col.as<int32_t>(), kk, cnd.as<int32_t>(), mem.as<int32_t>(),
                                                          nm, I, g0.as<int32_t>());
        if ((rc = check_launch("knn_rows_kernel"))) return rc;
        // the pageable sources of the next copies are staged before return; the
        // device buffers are reused in stream order
    }
    // 3. pruning
    if ((rc = pr.alloc((size_t)n * D * 4))) return rc;
    {
        const int nt = (I + 31) / 32 * 32;
        const size_t sm = (size_t)I * 8 + (size_t)next_pow2(I) * 4;
        FG_CUDA_TRY(ensure_smem(reinterpret_cast<const void*>(&prune_kernel), (int)sm));
        prune_kernel<<<(unsigned)n, nt, sm, s>>>(g0.as<int32_t>(), order.as<int32_t>(), n, I, D, pr.as<int32_t>());
        if ((rc = check_launch("prune_kernel"))) return rc;
    }
    // 4. reverse edges: stable sort of edges (i-major, then u) by target
    const long long ne = n * D;
    const size_t ws4 = sort_workspace(ne, (int)n + 1);
    if ((rc = tgt.alloc((size_t)ne * 4)) || (rc = rord.alloc((size_t)ne * 4)) || (rc = roff.alloc((size_t)(n + 2) * 4)) ||
        (rc = ws.alloc(std::max({wk, wc, wn, ws4}))))
        return rc;
    edge_targets_kernel<<<(unsigned)((ne + 255) / 256), 256, 0, s>>>(pr.as<int32_t>(), n, D, tgt.as<int32_t>());
    if ((rc = check_launch("edge_targets_kernel"))) return rc;
    if ((rc = sort_by_list(tgt.as<int32_t>(), ne, (int)n + 1, rord.as<int32_t>(), roff.as<int32_t>(), ws.p, ws.bytes,
                           s)))
        return rc;
    // 5. final lists
    merge_graph_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(pr.as<int32_t>(), rord.as<int32_t>(),
                                                                    roff.as<int32_t>(), n, D, graph);
    if ((rc = check_launch("merge_graph_kernel"))) return rc;
    // entry points for the search: the IVF centroids and each list's medoid
    if (entry_centroids)
        FG_CUDA_TRY(cudaMemcpyAsync(entry_centroids, cen.p, (size_t)L * dim * 4, cudaMemcpyDeviceToDevice, s));
    if (entry_nodes) {
        medoid_kernel<<<(L + 3) / 4, 128, 0, s>>>(X, dim, cen.as<float>(), order.as<int32_t>(), offs.as<int32_t>(), L,
                                                   p->metric, entry_nodes);
        if ((rc = check_launch("medoid_kernel"))) return rc;
    }
    FG_CUDA_TRY(cudaStreamSynchronize(s));
    return FG_OK;
}

// ============================== search =========================================

#ifndef FG_GS_NT
#define FG_GS_NT 128
#endif
#ifndef FG_GS_HASH_BITS
#define FG_GS_HASH_BITS 12
#endif
#ifndef FG_GS_CHUNKS
#define FG_GS_CHUNKS 2
#endif
constexpr int GS_NT = FG_GS_NT;
constexpr int GS_WARPS = GS_NT / 32;
constexpr int GS_HASH_BITS = FG_GS_HASH_BITS;  // 4096 slots (16 KB), reset at half load
constexpr int GS_HASH = 1 << GS_HASH_BITS;
constexpr uint32_t GS_EMPTY = 0xffffffffu;
constexpr int GS_UNROLL = 4;         // vectors in flight per warp
constexpr int GS_CHUNKS = FG_GS_CHUNKS;  // 16-byte chunks per lane and vector loaded per round

// murmur3's 32-bit finaliser (a published mixing function)
__host__ __device__ __forceinline__ uint32_t mix32(uint32_t h) {
    h ^= h >> 16;
    h *= 0x85ebca6bu;
    h ^= h >> 13;
    h *= 0xc2b2ae35u;
    h ^= h >> 16;
    return h;
}

// the s-th starting node of query q
__host__ __device__ __forceinline__ uint32_t seed_node(uint32_t seed, long long q, int s, int S, long long n) {
    const uint32_t x = mix32(seed ^ mix32((uint32_t)(q * S + s) * 0x9e3779b9u + 0x7f4a7c15u));
    return (uint32_t)((unsigned long long)x % (unsigned long long)n);
}

struct GraphSearchArgs {
    const void* data;
    long long n;
    int dim;
    const int32_t* graph;
    int degree;
    const void* queries;
    int nq;
    int itopk, width, max_iter, k;
    uint32_t seed;
    const int32_t* entry_nodes;   // [n_entries]
    const int32_t* query_entry;   // [nq][entry_probes]: nearest entry lists per query, or null
    int entry_probes;
    int32_t* out_ids;
    float* out_d;
    unsigned long long* counters;
};

template <class T>
struct Chunk;
template <>
struct Chunk<__half> {
    static constexpr int E = 8;  // elements per 16-byte chunk
};
template <>
struct Chunk<float> {
    static constexpr int E = 4;
};

template <class T>
__device__ __forceinline__ void chunk_to_float(const uint4& v, float* f) {
    if constexpr (sizeof(T) == 2) {
        const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 x = __half22float2(h[e]);
            f[2 * e] = x.x;
            f[2 * e + 1] = x.y;
        }
    } else {
        f[0] = __uint_as_float(v.x);
        f[1] = __uint_as_float(v.y);
        f[2] = __uint_as_float(v.z);
        f[3] = __uint_as_float(v.w);
    }
}

// Distance of up to GS_UNROLL vectors to the query, one warp: lane l takes the
// 16-byte chunks l, l+32, ... in order, fmaf per element, then an xor
// butterfly (16, 8, 4, 2, 1).
template <class T, int METRIC>
__device__ __forceinline__ void warp_dist(const T* __restrict__ data, long long n, int dim, const float* qv,
                                          const int32_t* ids, int cnt, float* out, unsigned long long* bad) {
    constexpr int E = Chunk<T>::E;
    const int lane = threadIdx.x & 31;
    const int nch = dim / E;
    // row pointers: every address stays inside the data array (row 0 stands
    // in for an unused or out-of-range id, whose result is discarded)
    const uint4* row[GS_UNROLL];
#pragma unroll
    for (int u = 0; u < GS_UNROLL; ++u) {
        long long id = u < cnt ? ids[u] : 0;
        if (id < 0 || id >= n) {
            if (lane == 0) atomicAdd(bad, 1ull);
            id = 0;
        }
        row[u] = reinterpret_cast<const uint4*>(data + (size_t)id * dim);
    }
    float acc[GS_UNROLL];
#pragma unroll
    for (int u = 0; u < GS_UNROLL; ++u) acc[u] = 0.0f;
    for (int c0 = 0; c0 < nch; c0 += 32 * GS_CHUNKS) {
        uint4 v[GS_UNROLL][GS_CHUNKS];
#pragma unroll
        for (int u = 0; u < GS_UNROLL; ++u)
#pragma unroll
            for (int h = 0; h < GS_CHUNKS; ++h) {
                const int c = c0 + h * 32 + lane;
                v[u][h] = __ldg(row[u] + (c < nch ? c : 0));
            }
#pragma unroll
        for (int h = 0; h < GS_CHUNKS; ++h) {
            const int c = c0 + h * 32 + lane;
            if (c >= nch) continue;
            // the query chunk, stored lane-interleaved (qv_index): the 32 lanes'
            // float4 reads of one step are consecutive, so conflict-free
            float q[E];
            const float4* q4 = reinterpret_cast<const float4*>(qv) + (size_t)(c >> 5) * (E / 4) * 32 + lane;
#pragma unroll
            for (int e4 = 0; e4 < E / 4; ++e4) {
                const float4 t = q4[e4 * 32];
                q[4 * e4] = t.x;
                q[4 * e4 + 1] = t.y;
                q[4 * e4 + 2] = t.z;
                q[4 * e4 + 3] = t.w;
            }
#pragma unroll
            for (int u = 0; u < GS_UNROLL; ++u) {
                float f[E];
                chunk_to_float<T>(v[u][h], f);
#pragma unroll
                for (int e = 0; e < E; ++e) {
                    if (METRIC == FG_METRIC_IP) {
                        acc[u] = fmaf(f[e], q[e], acc[u]);
                    } else {
                        const float df = f[e] - q[e];
                        acc[u] = fmaf(df, df, acc[u]);
                    }
                }
            }
        }
    }
#pragma unroll
    for (int u = 0; u < GS_UNROLL; ++u) {
        float a = acc[u];
#pragma unroll
        for (int o = 16; o; o >>= 1) a = a + __shfl_xor_sync(0xffffffffu, a, o);
        out[u] = METRIC == FG_METRIC_IP ? -a : a;
    }
}

// Position of query element j in shared memory: element e of the 16-byte
// chunk c (E elements per chunk) goes to float4 ((c / 32) * E/4 + e / 4) * 32
// + c % 32, lane (c % 32) of warp_dist's reads of that step.  The layout
// spans round_up(dim, 256) floats at most.
template <int E>
__host__ __device__ __forceinline__ int qv_index(int j) {
    const int c = j / E, e = j % E;
    return (((c >> 5) * (E / 4) + e / 4) * 32 + (c & 31)) * 4 + (e & 3);
}

struct GsShared {
    int ntop;    // valid entries in the top list
    int hcount;  // occupied hash slots
    int pad[2];
    unsigned long long evals, expanded, bad;  // bad: index checks that failed (access skipped)
};

// 0 = automatic: twice the iterations needed to expand a full top list, plus 10
__host__ __device__ inline int graph_auto_iterations(int itopk, int width) {
    return 2 * ((itopk + width - 1) / width) + 10;
}

// byte offsets of the search kernel's shared memory
struct GsLayout {
    int qv, hash, top, top2, cand, expl, expl2, nid, slot, parents, swarp, sh, total;
};

__host__ __device__ inline GsLayout gs_layout(int dim, int itopk, int width, int degree) {
    GsLayout L;
    int o = 0;
    auto take = [&](int bytes) {
        const int r = o;
        o += (bytes + 15) / 16 * 16;
        return r;
    };
    const int WD = width * degree;
    L.qv = take((dim + 255) / 256 * 256 * 4);
    L.hash = take(GS_HASH * 4);
    L.top = take(itopk * 8);
    L.top2 = take(itopk * 8);
    L.cand = take(next_pow2(WD) * 8);
    L.expl = take(itopk);
    L.expl2 = take(itopk);
    L.nid = take(WD * 4);
    L.slot = take(WD * 4);
    L.parents = take(width * 4);
    L.swarp = take((GS_WARPS + 2) * 4);
    L.sh = take((int)sizeof(GsShared));
    L.total = o;
    return L;
}

template <class T, int METRIC>
__global__ void __launch_bounds__(GS_NT) graph_search_kernel(const GraphSearchArgs a) {
    extern __shared__ __align__(16) unsigned char gs_raw[];
    const int dim = a.dim, D = a.degree, W = a.width, IT = a.itopk;
    const int WD = W * D;
    const int cpow = next_pow2(WD);
    const GsLayout L = gs_layout(dim, IT, W, D);
    float* qv = reinterpret_cast<float*>(gs_raw + L.qv);
    uint32_t* hash = reinterpret_cast<uint32_t*>(gs_raw + L.hash);
    unsigned long long* top = reinterpret_cast<unsigned long long*>(gs_raw + L.top);
    unsigned long long* top2 = reinterpret_cast<unsigned long long*>(gs_raw + L.top2);
    unsigned long long* cand = reinterpret_cast<unsigned long long*>(gs_raw + L.cand);
    uint8_t* expl = gs_raw + L.expl;
    uint8_t* expl2 = gs_raw + L.expl2;
    int32_t* nid = reinterpret_cast<int32_t*>(gs_raw + L.nid);       // fresh nodes of this iteration
    int32_t* slot = reinterpret_cast<int32_t*>(gs_raw + L.slot);     // candidate slots of this iteration
    int32_t* parents = reinterpret_cast<int32_t*>(gs_raw + L.parents);
    int* swarp = reinterpret_cast<int*>(gs_raw + L.swarp);
    GsShared* sh = reinterpret_cast<GsShared*>(gs_raw + L.sh);

    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const long long q = blockIdx.x;
    const T* data = static_cast<const T*>(a.data);
    const T* qsrc = static_cast<const T*>(a.queries) + (size_t)q * dim;
    for (int j = tid; j < dim; j += GS_NT) {
        if constexpr (sizeof(T) == 2)
            qv[qv_index<Chunk<T>::E>(j)] = __half2float(qsrc[j]);
        else
            qv[qv_index<Chunk<T>::E>(j)] = qsrc[j];
    }
    for (int j = tid; j < GS_HASH; j += GS_NT) hash[j] = GS_EMPTY;
    for (int j = tid; j < IT; j += GS_NT) {
        top[j] = ~0ull;
        expl[j] = 0;
    }
    if (tid == 0) {
        sh->ntop = 0;
        sh->hcount = 0;
        sh->evals = 0;
        sh->expanded = 0;
        sh->bad = 0;
    }
    __syncthreads();

    for (int iter = -1; iter < a.max_iter; ++iter) {
        // ---- candidate slots: random nodes first, then the parents' neighbours
        if (iter < 0) {
            // entry lists (the query's nearest IVF lists, selected before the
            // launch): their medoids take slots 0..S-1, pseudo-random nodes the rest
            int S = 0;
            if (a.query_entry) {
                S = min(a.entry_probes, WD);
                for (int t = tid; t < S; t += GS_NT) {
                    const int32_t c = a.query_entry[(size_t)q * a.entry_probes + t];
                    slot[t] = c >= 0 ? a.entry_nodes[c] : -1;
                }
            }
            for (int t = S + tid; t < WD; t += GS_NT) slot[t] = (int32_t)seed_node(a.seed, q, t, WD, a.n);
        } else {
            // parents: the first W unexplored valid entries of the top list
            int base = 0;
            for (int t0 = 0; t0 < IT; t0 += GS_NT) {
                const int t = t0 + tid;
                const int f = (t < IT && t < sh->ntop && !expl[t]) ? 1 : 0;
                int tot;
                const int pre = block_exclusive_scan<GS_NT>(f, swarp, tot);
                if (f && base + pre < W) {
                    parents[base + pre] = (int32_t)(top[t] & 0xffffffffu);
                    expl[t] = 1;
                }
                base += tot;
            }
            const int np = base < W ? base : W;
            if (np == 0) break;  // uniform: every thread computed the same base
            if (tid == 0) sh->expanded += np;
            // hash reset at half load: keep exactly the top list
            if (sh->hcount > GS_HASH / 2) {
                __syncthreads();
                for (int j = tid; j < GS_HASH; j += GS_NT) hash[j] = GS_EMPTY;
                __syncthreads();
                if (tid == 0) sh->hcount = 0;
                __syncthreads();
                for (int t = tid; t < sh->ntop; t += GS_NT) {
                    const uint32_t v = (uint32_t)(top[t] & 0xffffffffu);
                    uint32_t h = mix32(v) & (GS_HASH - 1);
                    for (int pr = 0; pr < GS_HASH; ++pr) {
                        const uint32_t old = atomicCAS(&hash[h], GS_EMPTY, v);
                        if (old == GS_EMPTY || old == v) break;
                        h = (h + 1) & (GS_HASH - 1);
                    }
                }
                __syncthreads();
                if (tid == 0) sh->hcount = sh->ntop;
            }
            __syncthreads();
            for (int t = tid; t < WD; t += GS_NT) {
                const int pi = t / D;
                int32_t v = -1;
                if (pi < np) {
                    const int32_t par = parents[pi];
                    if (par >= 0 && par < a.n)
                        v = a.graph[(size_t)par * D + (t - pi * D)];
                    else
                        atomicAdd(&sh->bad, 1ull);
                }
                slot[t] = v;
            }
        }
        __syncthreads();
        // ---- visited filter: insert into the hash; the inserting thread owns the node
        for (int t = tid; t < WD; t += GS_NT) {
            const int32_t v = slot[t];
            bool fresh = false;
            if (v >= 0 && v < a.n) {
                uint32_t h = mix32((uint32_t)v) & (GS_HASH - 1);
                for (int pr = 0; pr < GS_HASH; ++pr) {
                    const uint32_t old = atomicCAS(&hash[h], GS_EMPTY, (uint32_t)v);
                    if (old == GS_EMPTY) {
                        fresh = true;
                        break;
                    }
                    if (old == (uint32_t)v) break;
                    h = (h + 1) & (GS_HASH - 1);
                }
            }
            slot[t] = fresh ? v : -1;
        }
        __syncthreads();
        // compact the fresh nodes (slot order)
        int m = 0;
        for (int t0 = 0; t0 < WD; t0 += GS_NT) {
            const int t = t0 + tid;
            const int f = (t < WD && slot[t] >= 0) ? 1 : 0;
            int tot;
            const int pre = block_exclusive_scan<GS_NT>(f, swarp, tot);
            if (f) {
                if (m + pre < WD)
                    nid[m + pre] = slot[t];
                else
                    atomicAdd(&sh->bad, 1ull);
            }
            m += tot;
        }
        if (m > WD) m = WD;
        if (tid == 0) {
            sh->hcount += m;
            sh->evals += m;
        }
        __syncthreads();  // nid[] is written after the scan by other warps
        // ---- distances: warp w takes fresh nodes w*U.. in strides of WARPS*U
        for (int b = wid * GS_UNROLL; b < m; b += GS_WARPS * GS_UNROLL) {
            const int cnt = min(GS_UNROLL, m - b);
            float d[GS_UNROLL];
            warp_dist<T, METRIC>(data, a.n, dim, qv, nid + b, cnt, d, &sh->bad);
            if (lane < cnt) {
                float dd = d[0];
#pragma unroll
                for (int u = 1; u < GS_UNROLL; ++u)
                    if (lane == u) dd = d[u];
                cand[b + lane] = ((unsigned long long)f2key(dd) << 32) | (uint32_t)nid[b + lane];
            }
        }
        // sort the fresh candidates only (padded to a power of two): one warp
        // without block barriers when they fit in 32
        const int mpow = next_pow2(m > 0 ? m : 1);
        for (int t = m + tid; t < mpow; t += GS_NT) cand[t] = ~0ull;
        __syncthreads();
        if (mpow <= 32) {
            if (wid == 0) warp_bitonic_sort(cand, mpow);
            __syncthreads();
        } else {
            block_bitonic_sort<GS_NT>(cand, mpow);
        }
        // ---- merge path: top (ntop sorted) with cand (m sorted) -> first IT
        const int na = sh->ntop, nb = m;
        const int nout = min(IT, na + nb);
        for (int r = tid; r < IT; r += GS_NT) {
            if (r >= nout) {
                top2[r] = ~0ull;
                expl2[r] = 0;
                continue;
            }
            // co-rank: i from top, r - i from cand, A[i-1] < B[r-i] and B[r-i-1] < A[i]
            int lo = max(0, r - nb), hi = min(r, na);
            while (lo < hi) {
                const int i = (lo + hi) >> 1;
                if (top[i] < cand[r - i - 1])
                    lo = i + 1;
                else
                    hi = i;
            }
            const int i = lo, j = r - i;
            // reads: top[i] only for i < na, cand[j] only for j < nb (<= cpow)
            if (i > na || j < 0 || (i == na && j >= nb) || (j < nb && j >= cpow)) {
                atomicAdd(&sh->bad, 1ull);
                top2[r] = ~0ull;
                expl2[r] = 0;
                continue;
            }
            const bool take_a = i < na && (j >= nb || top[i] < cand[j]);
            top2[r] = take_a ? top[i] : cand[j];
            expl2[r] = take_a ? expl[i] : 0;
        }
        __syncthreads();
        for (int r = tid; r < IT; r += GS_NT) {
            top[r] = top2[r];
            expl[r] = expl2[r];
        }
        if (tid == 0) sh->ntop = nout;
        __syncthreads();
    }
    for (int r = tid; r < a.k; r += GS_NT) {
        const unsigned long long e = r < IT ? top[r] : ~0ull;
        const bool ok = e != ~0ull;
        a.out_ids[(size_t)q * a.k + r] = ok ? (int32_t)(e & 0xffffffffu) : -1;
        a.out_d[(size_t)q * a.k + r] = ok ? key2f((uint32_t)(e >> 32)) : FLT_MAX;
    }
    if (tid == 0 && a.counters) {
        atomicAdd(&a.counters[0], sh->evals);
        atomicAdd(&a.counters[1], sh->expanded);
        atomicAdd(&a.counters[2], sh->bad);
    }
}

size_t graph_search_smem(int dim, int itopk, int width, int degree) {
    return (size_t)gs_layout(dim, itopk, width, degree).total;
}

// scratch of the entry selection: fp32 queries (when the vectors are fp16),
// the per-query entry lists and their distances, and the k-NN workspace
size_t graph_search_workspace(int dtype, int dim, int nq, int n_entries, int probes) {
    if (probes <= 0 || nq <= 0) return 0;
    size_t b = 0;
    if (dtype == FG_DTYPE_F16) b += round_up((size_t)nq * dim * 4, 256);
    b += round_up((size_t)nq * probes * 4, 256) * 2;
    b += knn_like_workspace(nq, n_entries, probes);
    return b + 1024;
}

int graph_search(const void* data, int dtype, long long n, int dim, const int32_t* graph, int degree,
                 const float* entry_cen, const int32_t* entry_nodes, int n_entries, const void* queries, int nq,
                 const fg_graph_search_params* p, int32_t* out_ids, float* out_d, unsigned long long* counters,
                 void* ws, size_t ws_bytes, cudaStream_t s) {
    FG_REQUIRE(p, "null params");
    FG_REQUIRE(dtype == FG_DTYPE_F32 || dtype == FG_DTYPE_F16, "unknown dtype %d", dtype);
    FG_REQUIRE(p->metric == FG_METRIC_L2 || p->metric == FG_METRIC_IP, "unknown metric %d", p->metric);
    FG_REQUIRE(n >= 1 && n <= 0x7fffffffll && nq >= 0 && degree >= 1, "bad graph shape");
    const int E = dtype == FG_DTYPE_F16 ? 8 : 4;
    FG_REQUIRE(dim >= E && dim % E == 0 && dim <= 4096, "dim must be a multiple of %d (16-byte rows), <= 4096", E);
    FG_REQUIRE(p->itopk >= 1 && p->itopk <= 1024, "itopk %d outside [1, 1024]", p->itopk);
    FG_REQUIRE(p->search_width >= 1 && p->search_width * degree <= 2048, "search_width * degree must be <= 2048");
    FG_REQUIRE(p->k >= 1 && p->k <= p->itopk, "k must be in [1, itopk]");
    FG_REQUIRE(p->max_iterations >= 0, "max_iterations < 0");
    FG_REQUIRE(p->entry_probes >= 0, "entry_probes < 0");
    FG_REQUIRE(p->entry_probes <= 4096, "entry_probes %d above 4096", p->entry_probes);
    FG_REQUIRE(p->entry_probes == 0 || (entry_cen && entry_nodes && n_entries >= 1),
               "entry_probes needs the entry centroids and nodes of the build");
    if (nq == 0) return FG_OK;
    FG_REQUIRE(data && graph && queries && out_ids && out_d, "null buffer");
    FG_REQUIRE(((uintptr_t)data & 15) == 0 && ((uintptr_t)queries & 15) == 0, "data and queries must be 16-byte aligned");
    GraphSearchArgs a;
    a.data = data;
    a.n = n;
    a.dim = dim;
    a.graph = graph;
    a.degree = degree;
    a.queries = queries;
    a.nq = nq;
    a.itopk = p->itopk;
    a.width = p->search_width;
    a.max_iter = p->max_iterations ? p->max_iterations : graph_auto_iterations(p->itopk, p->search_width);
    a.k = p->k;
    a.seed = p->seed;
    a.out_ids = out_ids;
    a.out_d = out_d;
    a.counters = counters;
    a.entry_nodes = entry_nodes;
    a.query_entry = nullptr;
    a.entry_probes = p->entry_probes;
    if (p->entry_probes > 0) {
        // the S nearest entry lists of every query: exact metric distances to
        // the entry centroids (fmaf in dimension order), ties by list id
        const int S = std::min(p->entry_probes, n_entries);
        a.entry_probes = S;
        const size_t need = graph_search_workspace(dtype, dim, nq, n_entries, S);
        FG_REQUIRE(ws && ws_bytes >= need, "graph search workspace: %zu bytes needed, %zu given", need, ws_bytes);
        Carve cv(ws, ws_bytes);
        const float* q32 = static_cast<const float*>(queries);
        if (dtype == FG_DTYPE_F16) {
            float* t = cv.take<float>((size_t)nq * dim);
            const long long tot = (long long)nq * dim;
            half_to_float_kernel<<<(unsigned)((tot + 255) / 256), 256, 0, s>>>(static_cast<const __half*>(queries),
                                                                              tot, t);
            int rc = check_launch("half_to_float_kernel");
            if (rc) return rc;
            q32 = t;
        }
        int32_t* qe = cv.take<int32_t>((size_t)nq * S);
        float* qd = cv.take<float>((size_t)nq * S);
        const size_t used = round_up(cv.used, 256);
        if (!cv.ok() || used > ws_bytes) return fail(FG_ERR_WORKSPACE, "graph search workspace too small");
        int rc = knn_like(entry_cen, n_entries, dim, q32, nq, S, qe, qd, static_cast<char*>(ws) + used,
                          ws_bytes - used, s, p->metric);
        if (rc) return rc;
        a.query_entry = qe;
    }
    const size_t sm = graph_search_smem(dim, p->itopk, p->search_width, degree);
    int dev = 0, smem_max = 0;
    FG_CUDA_TRY(cudaGetDevice(&dev));
    FG_CUDA_TRY(cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    FG_REQUIRE(sm <= (size_t)smem_max, "graph search needs %zu bytes of shared memory", sm);
    void (*k)(const GraphSearchArgs) = nullptr;
    if (dtype == FG_DTYPE_F16)
        k = p->metric == FG_METRIC_IP ? graph_search_kernel<__half, FG_METRIC_IP> : graph_search_kernel<__half, FG_METRIC_L2>;
    else
        k = p->metric == FG_METRIC_IP ? graph_search_kernel<float, FG_METRIC_IP> : graph_search_kernel<float, FG_METRIC_L2>;
    FG_CUDA_TRY(ensure_smem(reinterpret_cast<const void*>(k), (int)sm));
    k<<<nq, GS_NT, sm, s>>>(a);
    return check_launch("graph_search_kernel");
}

}  // namespace fg

extern "C" int fg_graph_build(const void* data, int32_t dtype, int64_t n, int32_t dim,
                              const fg_graph_build_params* params, int32_t* graph, float* entry_centroids,
                              int32_t* entry_nodes, void* stream) {
    return fg::graph_build(data, dtype, n, dim, params, graph, entry_centroids, entry_nodes,
                           static_cast<cudaStream_t>(stream));
}

extern "C" int fg_graph_search_workspace_size(int32_t dtype, int32_t dim, int32_t nq, int32_t n_entries,
                                              const fg_graph_search_params* params, size_t* bytes) {
    if (!params || !bytes) return fg::fail(FG_ERR_INVALID_ARG, "null argument");
    *bytes = fg::graph_search_workspace(dtype, dim, nq, n_entries, std::min(params->entry_probes, n_entries));
    return FG_OK;
}

extern "C" int fg_graph_search(const void* data, int32_t dtype, int64_t n, int32_t dim, const int32_t* graph,
                               int32_t degree, const float* entry_centroids, const int32_t* entry_nodes,
                               int32_t n_entries, const void* queries, int32_t nq,
                               const fg_graph_search_params* params, int32_t* out_ids, float* out_dists,
                               uint64_t* counters, void* workspace, size_t workspace_bytes, void* stream) {
    return fg::graph_search(data, dtype, n, dim, graph, degree, entry_centroids, entry_nodes, n_entries, queries, nq,
                            params, out_ids, out_dists, reinterpret_cast<unsigned long long*>(counters), workspace,
                            workspace_bytes, static_cast<cudaStream_t>(stream));
}
