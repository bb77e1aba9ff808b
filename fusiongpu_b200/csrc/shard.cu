// shard.cu -- the exchange step of a list-sharded search across GPUs.
//
// Each GPU searches only the inverted lists it owns and returns its local
// top-k per query (ascending by distance).  After one all-gather the per-GPU
// lists sit side by side as [nshards][nq][k]; merge_topk_kernel keeps the k
// smallest of the nshards*k candidates per query by (distance, global id).
// The reference is single-GPU (search_pipeline.cu:560 cudaSetDevice(0)); this
// is the sharded deployment of its search.
#include <algorithm>

#include "fg_common.cuh"

namespace fg {

constexpr int MG_WARPS = 4;  // queries per CTA, one warp each

__global__ void __launch_bounds__(MG_WARPS * 32)
    merge_topk_kernel(const float* __restrict__ dists, const int32_t* __restrict__ ids, int nshards, int nq, int k,
                      int npow, int32_t* __restrict__ out_ids, float* __restrict__ out_d) {
    extern __shared__ __align__(16) unsigned long long keys[];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * MG_WARPS + w;
    if (q >= nq) return;
    unsigned long long* s = keys + (size_t)w * npow;
    const int n = nshards * k;
    for (int i = lane; i < npow; i += 32) {
        unsigned long long key = ~0ull;
        if (i < n) {
            const int sh = i / k, j = i % k;
            const size_t o = ((size_t)sh * nq + q) * k + j;
            const int32_t id = ids[o];
            // padding (-1) sorts after every real id at equal distance
            key = ((unsigned long long)f2key(dists[o]) << 32) | (uint32_t)id;
        }
        s[i] = key;
    }
    __syncwarp();
    warp_bitonic_sort(s, npow);
    for (int j = lane; j < k; j += 32) {
        const unsigned long long e = s[j];
        out_ids[(size_t)q * k + j] = (int32_t)(uint32_t)(e & 0xffffffffu);
        out_d[(size_t)q * k + j] = key2f((uint32_t)(e >> 32));
    }
}

// The same selection over packed keys: one all-gather of [nshards][nq][k]
// 64-bit keys (distance key << 32 | global id) replaces two of the distances
// and the ids.  Each shard's row arrives sorted ascending (pack_sort_kernel),
// so a warp merges the nshards rows of its query pairwise in ceil(log2
// nshards) rounds, keeping the first k of each merge: a key's place in the
// merge of A and B is its index plus the number of keys of the other row
// before it (B keys strictly less than an A key, A keys less or equal to a B
// key), found by binary search -- O(k log k) per round instead of a bitonic
// sort of all nshards * k keys.
__global__ void merge_keys_kernel(const unsigned long long* __restrict__ in, int nshards, int nq, int k, int wpc,
                                  int32_t* __restrict__ out_ids, float* __restrict__ out_d) {
    extern __shared__ __align__(16) unsigned long long keys[];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * wpc + w;
    if (q >= nq) return;
    const int n = nshards * k;
    unsigned long long* cur = keys + (size_t)w * 2 * n;
    unsigned long long* nxt = cur + n;
    for (int i = lane; i < n; i += 32) {
        const int sh = i / k, j = i - sh * k;
        cur[i] = in[((size_t)sh * nq + q) * k + j];
    }
    __syncwarp();
    int nl = nshards;
    while (nl > 1) {
        const int pairs = nl >> 1;
        for (int pr = 0; pr < pairs; ++pr) {
            const unsigned long long* A = cur + (size_t)(2 * pr) * k;
            const unsigned long long* B = A + k;
            unsigned long long* O = nxt + (size_t)pr * k;
            for (int i = lane; i < k; i += 32) {
                const unsigned long long a = A[i], b = B[i];
                int lo = 0, hi = k;
                while (lo < hi) {
                    const int m = (lo + hi) >> 1;
                    if (B[m] < a) lo = m + 1; else hi = m;
                }
                if (i + lo < k) O[i + lo] = a;
                lo = 0;
                hi = k;
                while (lo < hi) {
                    const int m = (lo + hi) >> 1;
                    if (A[m] <= b) lo = m + 1; else hi = m;
                }
                if (i + lo < k) O[i + lo] = b;
            }
        }
        if (nl & 1)
            for (int i = lane; i < k; i += 32) nxt[(size_t)pairs * k + i] = cur[(size_t)(nl - 1) * k + i];
        __syncwarp();
        unsigned long long* t = cur;
        cur = nxt;
        nxt = t;
        nl = pairs + (nl & 1);
    }
    for (int j = lane; j < k; j += 32) {
        const unsigned long long e = cur[j];
        out_ids[(size_t)q * k + j] = (int32_t)(uint32_t)(e & 0xffffffffu);
        out_d[(size_t)q * k + j] = key2f((uint32_t)(e >> 32));
    }
}

// Row q of keys = its k entries f2key(d) << 32 | global id, sorted ascending,
// the global id being map[id] (the id itself without a map; -1, which sorts
// last, for an id outside the map).  One warp per row.
__global__ void __launch_bounds__(MG_WARPS * 32)
    pack_sort_kernel(const int32_t* __restrict__ ids, const float* __restrict__ d, int nq, int k, int npow,
                     const int32_t* __restrict__ map, long long nmap, unsigned long long* __restrict__ out) {
    extern __shared__ __align__(16) unsigned long long keys[];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * MG_WARPS + w;
    if (q >= nq) return;
    unsigned long long* s = keys + (size_t)w * npow;
    for (int i = lane; i < npow; i += 32) {
        unsigned long long key = ~0ull;
        if (i < k) {
            const size_t o = (size_t)q * k + i;
            int32_t v = ids[o];
            if (map) v = (v >= 0 && v < nmap) ? map[v] : -1;
            key = ((unsigned long long)f2key(d[o]) << 32) | (uint32_t)v;
        }
        s[i] = key;
    }
    __syncwarp();
    warp_bitonic_sort(s, npow);
    for (int i = lane; i < k; i += 32) out[(size_t)q * k + i] = s[i];
}

__global__ void map_ids_kernel(const int32_t* __restrict__ in, long long n, const int32_t* __restrict__ map,
                               long long nmap, int32_t* __restrict__ out) {
    const long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int32_t v = in[i];
    out[i] = (v >= 0 && v < nmap) ? map[v] : -1;
}

int merge_topk(const float* dists, const int32_t* ids, int nshards, int nq, int k, int32_t* out_ids, float* out_d,
               cudaStream_t s) {
    FG_REQUIRE(nshards >= 1 && nq >= 0 && k >= 1, "bad merge shape");
    if (nq == 0) return FG_OK;
    FG_REQUIRE(dists && ids && out_ids && out_d, "null buffer");
    const int npow = next_pow2(nshards * k);
    FG_REQUIRE(npow <= 4096, "nshards * k = %d exceeds 4096", nshards * k);
    const size_t smem = (size_t)MG_WARPS * npow * 8;
    FG_CUDA_TRY(ensure_smem(reinterpret_cast<const void*>(&merge_topk_kernel), (int)smem));
    merge_topk_kernel<<<(nq + MG_WARPS - 1) / MG_WARPS, MG_WARPS * 32, smem, s>>>(dists, ids, nshards, nq, k, npow,
                                                                                out_ids, out_d);
    return check_launch("merge_topk_kernel");
}

int merge_keys(const unsigned long long* in, int nshards, int nq, int k, int32_t* out_ids, float* out_d,
               cudaStream_t s) {
    FG_REQUIRE(nshards >= 1 && nq >= 0 && k >= 1, "bad merge shape");
    if (nq == 0) return FG_OK;
    FG_REQUIRE(in && out_ids && out_d, "null buffer");
    FG_REQUIRE(nshards * k <= 4096, "nshards * k = %d exceeds 4096", nshards * k);
    const size_t per_warp = (size_t)2 * nshards * k * 8;
    const int wpc = (int)std::max<size_t>(1, std::min<size_t>(4, (200u << 10) / per_warp));
    const size_t smem = per_warp * wpc;
    FG_CUDA_TRY(ensure_smem(reinterpret_cast<const void*>(&merge_keys_kernel), (int)smem));
    merge_keys_kernel<<<(nq + wpc - 1) / wpc, wpc * 32, smem, s>>>(in, nshards, nq, k, wpc, out_ids, out_d);
    return check_launch("merge_keys_kernel");
}

int pack_topk(const int32_t* ids, const float* d, int nq, int k, const int32_t* map, long long nmap,
              unsigned long long* out, cudaStream_t s) {
    FG_REQUIRE(nq >= 0 && k >= 1 && nmap >= 0, "bad sizes");
    FG_REQUIRE(k <= 4096, "k = %d exceeds 4096", k);
    if (nq == 0) return FG_OK;
    FG_REQUIRE(ids && d && out && (map || nmap == 0), "null buffer");
    const int npow = next_pow2(k);
    const size_t smem = (size_t)MG_WARPS * npow * 8;
    FG_CUDA_TRY(ensure_smem(reinterpret_cast<const void*>(&pack_sort_kernel), (int)smem));
    pack_sort_kernel<<<(nq + MG_WARPS - 1) / MG_WARPS, MG_WARPS * 32, smem, s>>>(ids, d, nq, k, npow, map, nmap,
                                                                                out);
    return check_launch("pack_sort_kernel");
}

int map_ids(const int32_t* in, long long n, const int32_t* map, long long nmap, int32_t* out, cudaStream_t s) {
    FG_REQUIRE(n >= 0 && nmap >= 0, "bad sizes");
    if (n == 0) return FG_OK;
    FG_REQUIRE(in && out && (map || nmap == 0), "null buffer");
    map_ids_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(in, n, map, nmap, out);
    return check_launch("map_ids_kernel");
}

}  // namespace fg

extern "C" int fg_merge_topk(const float* dists, const int32_t* ids, int32_t nshards, int32_t nq, int32_t k,
                             int32_t* out_ids, float* out_dists, void* stream) {
    return fg::merge_topk(dists, ids, nshards, nq, k, out_ids, out_dists, static_cast<cudaStream_t>(stream));
}

extern "C" int fg_map_ids(const int32_t* in, int64_t n, const int32_t* map, int64_t nmap, int32_t* out,
                          void* stream) {
    return fg::map_ids(in, n, map, nmap, out, static_cast<cudaStream_t>(stream));
}

extern "C" int fg_pack_topk(const int32_t* ids, const float* dists, int32_t nq, int32_t k, const int32_t* map,
                            int64_t nmap, uint64_t* keys, void* stream) {
    return fg::pack_topk(ids, dists, nq, k, map, nmap, reinterpret_cast<unsigned long long*>(keys),
                         static_cast<cudaStream_t>(stream));
}

extern "C" int fg_merge_topk_keys(const uint64_t* keys, int32_t nshards, int32_t nq, int32_t k, int32_t* out_ids,
                                  float* out_dists, void* stream) {
    return fg::merge_keys(reinterpret_cast<const unsigned long long*>(keys), nshards, nq, k, out_ids, out_dists,
                          static_cast<cudaStream_t>(stream));
}
