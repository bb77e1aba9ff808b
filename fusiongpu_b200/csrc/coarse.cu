// coarse.cu -- exact squared-L2 tiles and per-row top-k selection.
//
// Used by the coarse quantizer (replaces cuVS CAGRA search over centroids,
// cagra_adapter.cuh:38-68), by k-means assignment (replaces the SGEMM +
// argmin of kmeans_gpu.cuh:197-229) and by exact k-NN ground truth.
//
// Distances are sum_j fmaf(x_j - y_j, x_j - y_j, acc) in dimension order, the
// same arithmetic the oracle uses, so rankings match it exactly (ties broken
// by the lower column index).  The inner-product metric (graph build and its
// ground truth) uses -(sum_j fmaf(x_j, y_j, acc)) so that smaller is nearer.
#include <algorithm>

#include "fg_common.cuh"

namespace fg {

__host__ __device__ inline int round_up_dev(int x) { return (x + 15) / 16 * 16; }

constexpr int L2_T = 64;       // rows of X and of Y per tile
constexpr int L2_DC = 32;      // dimensions per shared-memory chunk
constexpr int L2_LD = L2_T + 4;
constexpr int L2_NT = 256;

// Nearest Y row of each X row: each CTA owns 64 rows of X and sweeps all of Y
// in 64-row tiles (256 threads, 4 x 4 pairs each), keeping per thread the
// smallest distance and, on ties, the lowest Y index; writes amin[x].
__global__ void __launch_bounds__(L2_NT) l2_argmin_kernel(const float* __restrict__ X, long long nx,
                                                          const float* __restrict__ Y, int ny, int dim,
                                                          int32_t* __restrict__ amin) {
    __shared__ __align__(16) float sX[L2_DC][L2_LD];
    __shared__ __align__(16) float sY[L2_DC][L2_LD];
    __shared__ float rd[L2_T][17];
    __shared__ int ri[L2_T][17];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const long long x0 = (long long)blockIdx.x * L2_T;
    const int nyt = (ny + L2_T - 1) / L2_T;
    float best[4];
    int bidx[4];
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        best[a] = FLT_MAX;
        bidx[a] = 0x7fffffff;
    }
    for (int yt = 0; yt < nyt; ++yt) {
        const int y0 = yt * L2_T;
        float acc[4][4];
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) acc[a][b] = 0.0f;
        for (int d0 = 0; d0 < dim; d0 += L2_DC) {
            // 64 rows x 32 dims of each operand, transposed into shared memory
            for (int f = tid; f < L2_T * L2_DC; f += L2_NT) {
                const int r = f / L2_DC, c = f % L2_DC;
                const int dj = d0 + c;
                const long long xr = x0 + r;
                const int yr = y0 + r;
                sX[c][r] = (xr < nx && dj < dim) ? X[xr * dim + dj] : 0.0f;
                sY[c][r] = (yr < ny && dj < dim) ? Y[(long long)yr * dim + dj] : 0.0f;
            }
            __syncthreads();
            const int dn = min(L2_DC, dim - d0);
            for (int j = 0; j < dn; ++j) {
                const float4 xv = *reinterpret_cast<const float4*>(&sX[j][tx * 4]);
                const float4 yv = *reinterpret_cast<const float4*>(&sY[j][ty * 4]);
                const float xa[4] = {xv.x, xv.y, xv.z, xv.w};
                const float yb[4] = {yv.x, yv.y, yv.z, yv.w};
#pragma unroll
                for (int a = 0; a < 4; ++a)
#pragma unroll
                    for (int b = 0; b < 4; ++b) {
                        const float df = xa[a] - yb[b];
                        acc[a][b] = fmaf(df, df, acc[a][b]);
                    }
            }
            __syncthreads();
        }
#pragma unroll
        for (int a = 0; a < 4; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b) {
                const int yr = y0 + ty * 4 + b;
                if (yr < ny && acc[a][b] < best[a]) {
                    best[a] = acc[a][b];
                    bidx[a] = yr;
                }
            }
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        rd[tx * 4 + a][ty] = best[a];
        ri[tx * 4 + a][ty] = bidx[a];
    }
    __syncthreads();
    if (tid < L2_T) {
        float bd = rd[tid][0];
        int bi = ri[tid][0];
        for (int t = 1; t < 16; ++t) {
            const float d = rd[tid][t];
            const int i = ri[tid][t];
            if (d < bd || (d == bd && i < bi)) {
                bd = d;
                bi = i;
            }
        }
        const long long xr = x0 + tid;
        if (xr < nx) amin[xr] = (bi == 0x7fffffff) ? 0 : bi;
    }
}

constexpr int TK_NT = 512;
constexpr int TK_SEG = 8192;          // columns per stage-1 segment (32 KB of keys), at least
constexpr int TK_STAGE_MAX = 32768;   // candidates stage 2 selects from, at most

// Stage-1 segment length: TK_SEG, or longer when the per-segment winners of a
// very wide row (100M columns) would not fit stage 2.
static int topk_seg_len(int ncols, int k) {
    if (ncols <= TK_SEG) return ncols;
    const long long nseg_max = std::max(1, TK_STAGE_MAX / std::max(k, 1));
    const long long need = (ncols + nseg_max - 1) / nseg_max;  // ceil(ncols / seg) <= nseg_max
    const long long seg = std::max<long long>(TK_SEG, (need + 3) / 4 * 4);
    return (int)std::min<long long>(seg, ncols);
}

static int topk_nseg(int ncols, int k) {
    const int seg = topk_seg_len(ncols, k);
    return (ncols + seg - 1) / seg;
}

// Top-k (ascending by value, ties by column/position) of one segment of one
// row.  Input value v[row][c0 + i] with row stride ldv; optional payload
// pay[row][c0 + i] (default: the column index).  Writes kk = min(k, len)
// sorted (index, value) pairs at out_i/out_v + row*out_ld + seg*k, padding
// up to k with (-1, FLT_MAX).
__global__ void __launch_bounds__(TK_NT) topk_segment_kernel(const float* __restrict__ v, long long ldv,
                                                             int ncols, int seg_len,
                                                             const int32_t* __restrict__ pay, int k,
                                                             int32_t* __restrict__ out_i,
                                                             float* __restrict__ out_v, long long out_ld) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ uint32_t hist[256];
    __shared__ uint32_t sb[2];
    __shared__ int warp[TK_NT / 32];
    const long long row = blockIdx.x;
    const int seg = blockIdx.y;
    const int c0 = seg * seg_len;
    const int len = min(seg_len, ncols - c0);
    const int kk = min(k, len);
    const int kpow = next_pow2(kk);
    uint32_t* keys = reinterpret_cast<uint32_t*>(smem);
    unsigned long long* sortb = reinterpret_cast<unsigned long long*>(smem + round_up_dev(seg_len * 4));
    const float* vr = v + row * ldv + c0;
    for (int i = threadIdx.x; i < len; i += TK_NT) keys[i] = f2key(vr[i]);
    __syncthreads();
    uint32_t kth;
    int n_less;
    block_radix_select<TK_NT>(keys, len, kk, hist, sb, kth, n_less);
    const int need_eq = kk - n_less;
    int eq_base = 0, out_base = 0;
    for (int r0 = 0; r0 < len; r0 += TK_NT) {
        const int i = r0 + threadIdx.x;
        const bool in = i < len;
        const uint32_t key = in ? keys[i] : 0xffffffffu;
        const int is_eq = (in && key == kth) ? 1 : 0;
        int eq_tot, s_tot;
        const int eq_pre = block_exclusive_scan<TK_NT>(is_eq, warp, eq_tot);
        const bool sel = in && (key < kth || (is_eq && eq_base + eq_pre < need_eq));
        eq_base += eq_tot;
        const int s_pre = block_exclusive_scan<TK_NT>(sel ? 1 : 0, warp, s_tot);
        if (sel) sortb[out_base + s_pre] = ((unsigned long long)key << 32) | (unsigned)i;
        out_base += s_tot;
    }
    for (int i = kk + threadIdx.x; i < kpow; i += TK_NT) sortb[i] = ~0ull;
    __syncthreads();
    block_bitonic_sort<TK_NT>(sortb, kpow);
    const long long ob = row * out_ld + (long long)seg * k;
    for (int r = threadIdx.x; r < k; r += TK_NT) {
        if (r < kk) {
            const unsigned long long e = sortb[r];
            const int li = (int)(e & 0xffffffffu);
            out_i[ob + r] = pay ? pay[row * ldv + c0 + li] : c0 + li;
            out_v[ob + r] = key2f((uint32_t)(e >> 32));
        } else {
            out_i[ob + r] = -1;
            out_v[ob + r] = FLT_MAX;
        }
    }
}

// Per-row top-k of a [rows][ncols] matrix with row stride ldv.  When ncols
// exceeds one segment, stage 1 writes the per-segment winners to `stage`
// ([rows][nseg*k] values + ids) and stage 2 selects from those.
int rows_topk(const float* v, long long ldv, long long rows, int ncols, int k, int32_t* out_i,
              float* out_v, long long out_ld, float* stage_v, int32_t* stage_i, cudaStream_t s) {
    if (rows <= 0) return FG_OK;
    const int nseg = topk_nseg(ncols, k);
    const int seg_len = nseg == 1 ? ncols : topk_seg_len(ncols, k);
    auto smem_for = [&](int len, int kk) { return round_up_dev(len * 4) + next_pow2(kk) * 8; };
    if (nseg == 1) {
        const int sm = smem_for(seg_len, k);
        FG_CUDA_TRY(ensure_smem(reinterpret_cast<const void*>(&topk_segment_kernel), sm));
        topk_segment_kernel<<<dim3((unsigned)rows, 1), TK_NT, sm, s>>>(v, ldv, ncols, seg_len, nullptr, k,
                                                                      out_i, out_v, out_ld);
        return check_launch("topk_segment_kernel");
    }
    const long long sld = (long long)nseg * k;
    int sm = smem_for(seg_len, k);
    int dev = 0, smem_max = 0;
    FG_CUDA_TRY(cudaGetDevice(&dev));
    FG_CUDA_TRY(cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    if (sm > smem_max || sld > TK_STAGE_MAX)
        return fail(FG_ERR_UNSUPPORTED, "top-%d of %d columns per row is beyond the two-stage select", k, ncols);
    FG_CUDA_TRY(ensure_smem(reinterpret_cast<const void*>(&topk_segment_kernel), std::max(sm, smem_for((int)sld, k))));
    topk_segment_kernel<<<dim3((unsigned)rows, nseg), TK_NT, sm, s>>>(v, ldv, ncols, seg_len, nullptr, k,
                                                                     stage_i, stage_v, sld);
    int rc = check_launch("topk_segment_kernel(stage 1)");
    if (rc) return rc;
    if (sld > TK_STAGE_MAX) return fail(FG_ERR_UNSUPPORTED, "top-k stage 2 of %lld candidates", sld);
    sm = smem_for((int)sld, k);
    topk_segment_kernel<<<dim3((unsigned)rows, 1), TK_NT, sm, s>>>(stage_v, sld, (int)sld, (int)sld, stage_i,
                                                                   k, out_i, out_v, out_ld);
    return check_launch("topk_segment_kernel(stage 2)");
}

size_t rows_topk_stage_bytes(long long rows, int ncols, int k) {
    const int nseg = topk_nseg(ncols, k);
    if (nseg == 1) return 0;
    return round_up((size_t)rows * nseg * k * 4, 256) * 2;
}

// The distance matrix with 128 x 128 tiles: 256 threads, each 8 X rows x 8 Y
// rows, 16 dimensions per shared-memory chunk, so that one dimension step is
// four 16-byte shared loads for 64 fmaf.  Every pair still accumulates
// fmaf(.., .., acc) over the dimensions in increasing order, so the values
// are the oracle's sum_j fmaf(...) in dimension order bit for bit.
constexpr int MT_T = 128;
constexpr int MT_DC = 16;
constexpr int MT_LD = MT_T + 4;

// 4-byte global -> shared copy that completes asynchronously; `bytes` 0 writes
// a zero without reading (the source address is then not dereferenced).
__device__ __forceinline__ void cp_async4(float* dst, const float* src, int bytes) {
    const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(d), "l"(src), "r"(bytes) : "memory");
}

template <int METRIC>
__global__ void __launch_bounds__(L2_NT) l2_matrix128_kernel(const float* __restrict__ X, long long nx,
                                                             const float* __restrict__ Y, int ny, int dim,
                                                             float* __restrict__ D, long long ldd) {
    // two chunk buffers: the next 16 dimensions are copied in while this
    // chunk's fmaf run
    __shared__ __align__(16) float sX[2][MT_DC][MT_LD];
    __shared__ __align__(16) float sY[2][MT_DC][MT_LD];
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const long long x0 = (long long)blockIdx.y * MT_T;
    const int y0 = blockIdx.x * MT_T;
    // 128 rows x 16 dimensions of each operand, transposed into buffer b
    auto stage = [&](int b, int d0) {
#pragma unroll 4
        for (int f = tid; f < MT_T * MT_DC; f += L2_NT) {
            const int r = f / MT_DC, c = f % MT_DC;
            const int dj = d0 + c;
            const long long xr = x0 + r;
            const int yr = y0 + r;
            const bool xin = xr < nx && dj < dim, yin = yr < ny && dj < dim;
            cp_async4(&sX[b][c][r], xin ? X + xr * dim + dj : X, xin ? 4 : 0);
            cp_async4(&sY[b][c][r], yin ? Y + (long long)yr * dim + dj : Y, yin ? 4 : 0);
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
    };
    float acc[8][8];
#pragma unroll
    for (int a = 0; a < 8; ++a)
#pragma unroll
        for (int b = 0; b < 8; ++b) acc[a][b] = 0.0f;
    stage(0, 0);
    int buf = 0;
    for (int d0 = 0; d0 < dim; d0 += MT_DC) {
        if (d0 + MT_DC < dim) {
            stage(buf ^ 1, d0 + MT_DC);
            asm volatile("cp.async.wait_group 1;" ::: "memory");
        } else {
            asm volatile("cp.async.wait_group 0;" ::: "memory");
        }
        __syncthreads();
        const int dn = min(MT_DC, dim - d0);
        for (int j = 0; j < dn; ++j) {
            const float4 xa0 = *reinterpret_cast<const float4*>(&sX[buf][j][tx * 8]);
            const float4 xa1 = *reinterpret_cast<const float4*>(&sX[buf][j][tx * 8 + 4]);
            const float4 yb0 = *reinterpret_cast<const float4*>(&sY[buf][j][ty * 8]);
            const float4 yb1 = *reinterpret_cast<const float4*>(&sY[buf][j][ty * 8 + 4]);
            const float xa[8] = {xa0.x, xa0.y, xa0.z, xa0.w, xa1.x, xa1.y, xa1.z, xa1.w};
            const float yb[8] = {yb0.x, yb0.y, yb0.z, yb0.w, yb1.x, yb1.y, yb1.z, yb1.w};
#pragma unroll
            for (int a = 0; a < 8; ++a)
#pragma unroll
                for (int b = 0; b < 8; ++b) {
                    if (METRIC == FG_METRIC_IP) {
                        acc[a][b] = fmaf(xa[a], yb[b], acc[a][b]);
                    } else {
                        const float df = xa[a] - yb[b];
                        acc[a][b] = fmaf(df, df, acc[a][b]);
                    }
                }
        }
        __syncthreads();  // buffer buf is refilled two chunks from now
        buf ^= 1;
    }
#pragma unroll
    for (int a = 0; a < 8; ++a) {
        const long long xr = x0 + tx * 8 + a;
        if (xr >= nx) continue;
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            const int yr = y0 + ty * 8 + b;
            if (yr < ny) D[xr * ldd + yr] = (METRIC == FG_METRIC_IP) ? -acc[a][b] : acc[a][b];
        }
    }
}

int l2_matrix(const float* X, long long nx, const float* Y, int ny, int dim, float* D, long long ldd,
              cudaStream_t s, int metric = FG_METRIC_L2) {
    if (nx <= 0 || ny <= 0) return FG_OK;
    const int nyt = (ny + MT_T - 1) / MT_T;
    // at most 65535 X tiles per launch (grid.y)
    const long long xrows = 65535ll * MT_T;
    for (long long r0 = 0; r0 < nx; r0 += xrows) {
        const long long nr = std::min(xrows, nx - r0);
        dim3 grid((unsigned)nyt, (unsigned)((nr + MT_T - 1) / MT_T));
        if (metric == FG_METRIC_IP)
            l2_matrix128_kernel<FG_METRIC_IP><<<grid, L2_NT, 0, s>>>(X + r0 * dim, nr, Y, ny, dim, D + r0 * ldd, ldd);
        else
            l2_matrix128_kernel<FG_METRIC_L2><<<grid, L2_NT, 0, s>>>(X + r0 * dim, nr, Y, ny, dim, D + r0 * ldd, ldd);
        const int rc = check_launch("l2_matrix128_kernel");
        if (rc) return rc;
    }
    return FG_OK;
}

int l2_argmin(const float* X, long long nx, const float* Y, int ny, int dim, int32_t* amin,
              cudaStream_t s) {
    if (nx <= 0) return FG_OK;
    dim3 grid((unsigned)((nx + L2_T - 1) / L2_T), 1);
    l2_argmin_kernel<<<grid, L2_NT, 0, s>>>(X, nx, Y, ny, dim, amin);
    return check_launch("l2_argmin_kernel");
}

// ---- coarse search and exact k-NN (row chunks through a workspace matrix) ----

static long long chunk_rows(size_t ws_bytes, long long nrows, int ncols, int k) {
    // matrix [r][ncols] + stage buffers [r][nseg*k] x2
    const int nseg = topk_nseg(ncols, k);
    const size_t per_row = (size_t)ncols * 4 + (nseg > 1 ? (size_t)nseg * k * 8 : 0);
    if (ws_bytes < 1024) return 0;
    long long r = (long long)((ws_bytes - 1024) / per_row);
    if (r > nrows) r = nrows;
    return r;
}

size_t knn_like_workspace(long long nq, int ncols, int k) {
    const long long want = std::min<long long>(nq, std::max<long long>(64, (256ll << 20) / ((long long)ncols * 4)));
    const int nseg = topk_nseg(ncols, k);
    size_t b = round_up((size_t)want * ncols * 4, 256);
    if (nseg > 1) b += round_up((size_t)want * nseg * k * 4, 256) * 2;
    return b + 1024;
}

int knn_like(const float* Y, long long ny, int dim, const float* Q, long long nq, int k, int32_t* out_i,
             float* out_v, void* ws, size_t ws_bytes, cudaStream_t s, int metric) {
    FG_REQUIRE(ny <= 0x7fffffffll, "too many columns");
    const int ncols = (int)ny;
    long long rows = chunk_rows(ws_bytes, nq, ncols, k);
    if (rows < 1) return fail(FG_ERR_WORKSPACE, "workspace of %zu bytes holds no row of %d distances",
                              ws_bytes, ncols);
    const int nseg = topk_nseg(ncols, k);
    for (long long q0 = 0; q0 < nq; q0 += rows) {
        const long long r = std::min(rows, nq - q0);
        Carve cv(ws, ws_bytes);
        float* D = cv.take<float>((size_t)r * ncols);
        float* sv = nseg > 1 ? cv.take<float>((size_t)r * nseg * k) : nullptr;
        int32_t* si = nseg > 1 ? cv.take<int32_t>((size_t)r * nseg * k) : nullptr;
        if (!cv.ok()) return fail(FG_ERR_WORKSPACE, "workspace too small");
        int rc = l2_matrix(Q + q0 * dim, r, Y, ncols, dim, D, ncols, s, metric);
        if (rc) return rc;
        rc = rows_topk(D, ncols, r, ncols, k, out_i + q0 * k, out_v + q0 * k, k, sv, si, s);
        if (rc) return rc;
    }
    return FG_OK;
}

}  // namespace fg
