// bf_kernels.cu -- exact brute-force scan (BruteForceIndex::scan_range /
// search_parallel, forge-db src/index/brute_force.rs:105-214).
//
// Each block takes a tile of QT queries (shared memory) and a chunk of rows;
// every thread scores one row against the QT queries per step, computing the
// metric of DistanceMetric::compute (distance/mod.rs:40-48) in the AVX2
// order, so distances are bit-identical to the reference.  Each warp keeps a
// WarpTopK per query; the block's warps merge at the end and write a partial
// top-k per (row chunk, query), which merge_lists_kernel folds together.
// Grid x runs over query tiles so that the blocks of one row chunk are
// resident together and read that chunk from L2, not HBM.
#include <algorithm>

#include "fdb_device.cuh"
#include "fdb_internal.h"
#include "fdb_kernels.h"

namespace fdb {

constexpr int BF_THREADS = 128;
constexpr int BF_WARPS = BF_THREADS / 32;

__global__ void row_norms_kernel(const float* __restrict__ x, size_t n, int dim,
                                 float* __restrict__ out) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = dot_exact(x + i * dim, x + i * dim, dim);
}

void launch_row_norms(cudaStream_t s, const float* x, size_t n, int dim, float* norms) {
    if (n == 0) return;
    row_norms_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(x, n, dim, norms);
    FDB_LAUNCH_CHECK();
}

template <int METRIC>
__device__ __forceinline__ void bf_acc(float& acc, float q, float x) {
    if (METRIC == EUCLIDEAN || METRIC == EUCLIDEAN_SQUARED) {
        float d = __fsub_rn(q, x);
        acc = __fmaf_rn(d, d, acc);
    } else if (METRIC == DOT_PRODUCT || METRIC == COSINE) {
        acc = __fmaf_rn(q, x, acc);
    } else {
        acc = __fadd_rn(acc, fabsf(__fsub_rn(q, x)));
    }
}

template <int METRIC>
__device__ __forceinline__ float bf_tail(float t, float q, float x) {
    if (METRIC == EUCLIDEAN || METRIC == EUCLIDEAN_SQUARED) {
        float d = __fsub_rn(q, x);
        return __fadd_rn(t, __fmul_rn(d, d));
    } else if (METRIC == DOT_PRODUCT || METRIC == COSINE) {
        return __fadd_rn(t, __fmul_rn(q, x));
    } else {
        return __fadd_rn(t, fabsf(__fsub_rn(q, x)));
    }
}

template <int METRIC>
__device__ __forceinline__ float bf_final(float t, float qn, float xn) {
    if (METRIC == EUCLIDEAN) return __fsqrt_rn(t);
    if (METRIC == DOT_PRODUCT) return -t;
    if (METRIC == COSINE) return cosine_from(t, qn, xn);
    return t;
}

template <int P, int QT, int METRIC>
__global__ void __launch_bounds__(BF_THREADS)
    bf_scan_kernel(const float* __restrict__ Q, int nq, const float* __restrict__ qnorm,
                   const float* __restrict__ X, size_t n, int dim,
                   const float* __restrict__ xnorm, size_t chunk_rows, uint64_t tag_base, int k,
                   uint64_t* __restrict__ part) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int dim_pad = (dim + 3) & ~3;
    float* sq = reinterpret_cast<float*>(smem);
    uint64_t* wbuf = reinterpret_cast<uint64_t*>(sq + QT * dim_pad);
    uint64_t* lists = wbuf + QT * BF_WARPS * 64;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q0 = blockIdx.x * QT;
    const int nqt = min(QT, nq - q0);
    const size_t r0 = (size_t)blockIdx.y * chunk_rows;
    const size_t r1 = min(n, r0 + chunk_rows);
    for (int e = threadIdx.x; e < QT * dim_pad; e += BF_THREADS) {
        int qi = e / dim_pad, j = e - qi * dim_pad;
        sq[e] = (qi < nqt && j < dim) ? Q[(size_t)(q0 + qi) * dim + j] : 0.0f;
    }
    __syncthreads();
    float qn[QT];
#pragma unroll
    for (int a = 0; a < QT; ++a) qn[a] = (METRIC == COSINE && a < nqt) ? qnorm[q0 + a] : 0.0f;

    WarpTopK<P> tk[QT];
#pragma unroll
    for (int a = 0; a < QT; ++a) tk[a].init(k, wbuf + (a * BF_WARPS + warp) * 64);

    const int full = dim & ~7;
    const bool vec = (dim & 3) == 0;
    for (size_t base = r0 + (size_t)warp * 32; base < r1; base += (size_t)BF_WARPS * 32) {
        const size_t row = base + lane;
        const bool valid = row < r1;
        const float* xr = X + (valid ? row : r0) * dim;
        float acc[QT][8];
#pragma unroll
        for (int a = 0; a < QT; ++a)
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[a][j] = 0.0f;
        for (int g = 0; g < full; g += 8) {
            float xv[8];
            if (vec) {
                float4 u = __ldg(reinterpret_cast<const float4*>(xr + g));
                float4 v = __ldg(reinterpret_cast<const float4*>(xr + g + 4));
                xv[0] = u.x; xv[1] = u.y; xv[2] = u.z; xv[3] = u.w;
                xv[4] = v.x; xv[5] = v.y; xv[6] = v.z; xv[7] = v.w;
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) xv[j] = __ldg(xr + g + j);
            }
#pragma unroll
            for (int a = 0; a < QT; ++a) {
                const float* qa = sq + a * dim_pad + g;
#pragma unroll
                for (int j = 0; j < 8; ++j) bf_acc<METRIC>(acc[a][j], qa[j], xv[j]);
            }
        }
        const float xn = (METRIC == COSINE && valid) ? xnorm[row] : 0.0f;
#pragma unroll
        for (int a = 0; a < QT; ++a) {
            float t = lane_sum(acc[a]);
            for (int g = full; g < dim; ++g) t = bf_tail<METRIC>(t, sq[a * dim_pad + g], __ldg(xr + g));
            float d = bf_final<METRIC>(t, qn[a], xn);
            tk[a].add(make_key(d, (uint32_t)(tag_base + row)), valid && a < nqt);
        }
    }
#pragma unroll
    for (int a = 0; a < QT; ++a) {
        tk[a].flush();
        tk[a].store(lists + (size_t)(a * BF_WARPS + warp) * k);
    }
    __syncthreads();
    // Warp w folds the BF_WARPS lists of queries w, w + BF_WARPS, ...
    for (int a = warp; a < nqt; a += BF_WARPS) {
        WarpTopK<P> m;
        m.init(k, wbuf + (a * BF_WARPS + warp) * 64);
        for (int w = 0; w < BF_WARPS; ++w) m.ingest(lists + (size_t)(a * BF_WARPS + w) * k, k);
        m.store(part + ((size_t)blockIdx.y * nq + q0 + a) * k);
    }
}

static size_t bf_chunk_rows(size_t n, int nq, int qt, int sm_count) {
    size_t tiles = (size_t)((nq + qt - 1) / qt);
    size_t target = (size_t)sm_count * 6;
    size_t chunks = std::max<size_t>(1, (target + tiles - 1) / tiles);
    size_t rows = (n + chunks - 1) / chunks;
    rows = std::max<size_t>(rows, 512);
    rows = std::min<size_t>(rows, 65536);
    rows = (rows + 127) / 128 * 128;
    return rows;
}

static int bf_qt(int k) { return k <= 64 ? 8 : 4; }

size_t bf_part_size(size_t n, int nq, int k, int sm_count) {
    size_t rows = bf_chunk_rows(n, nq, bf_qt(k), sm_count);
    size_t chunks = std::max<size_t>(1, (n + rows - 1) / rows);
    return chunks * (size_t)nq * k;
}

template <int P, int QT, int METRIC>
static void bf_launch_t(cudaStream_t s, const float* Q, int nq, const float* qnorm,
                        const float* X, size_t n, int dim, const float* xnorm, size_t rows,
                        size_t chunks, uint64_t tag_base, int k, uint64_t* part) {
    const int dim_pad = (dim + 3) & ~3;
    size_t smem = (size_t)QT * dim_pad * sizeof(float) + (size_t)QT * BF_WARPS * 64 * 8 +
                  (size_t)QT * BF_WARPS * k * 8;
    FDB_REQUIRE(smem <= 227 * 1024, FDB_ERR_UNSUPPORTED, "dimension too large for brute force");
    auto kern = bf_scan_kernel<P, QT, METRIC>;
    if (smem > 48 * 1024)
        FDB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid((unsigned)((nq + QT - 1) / QT), (unsigned)chunks);
    kern<<<grid, BF_THREADS, smem, s>>>(Q, nq, qnorm, X, n, dim, xnorm, rows, tag_base, k, part);
    FDB_LAUNCH_CHECK();
}

template <int P, int QT>
static void bf_launch_m(int metric, cudaStream_t s, const float* Q, int nq, const float* qnorm,
                        const float* X, size_t n, int dim, const float* xnorm, size_t rows,
                        size_t chunks, uint64_t tag_base, int k, uint64_t* part) {
    switch (metric) {
        case EUCLIDEAN: bf_launch_t<P, QT, EUCLIDEAN>(s, Q, nq, qnorm, X, n, dim, xnorm, rows, chunks, tag_base, k, part); break;
        case EUCLIDEAN_SQUARED: bf_launch_t<P, QT, EUCLIDEAN_SQUARED>(s, Q, nq, qnorm, X, n, dim, xnorm, rows, chunks, tag_base, k, part); break;
        case COSINE: bf_launch_t<P, QT, COSINE>(s, Q, nq, qnorm, X, n, dim, xnorm, rows, chunks, tag_base, k, part); break;
        case DOT_PRODUCT: bf_launch_t<P, QT, DOT_PRODUCT>(s, Q, nq, qnorm, X, n, dim, xnorm, rows, chunks, tag_base, k, part); break;
        default: bf_launch_t<P, QT, MANHATTAN>(s, Q, nq, qnorm, X, n, dim, xnorm, rows, chunks, tag_base, k, part); break;
    }
}

int launch_bf_scan(cudaStream_t s, int metric, const float* Q, int nq, const float* qnorm,
                   const float* X, size_t n, int dim, const float* xnorm, uint64_t tag_base,
                   int k, int sm_count, uint64_t* part, size_t part_capacity) {
    FDB_REQUIRE(k >= 1 && k <= FDB_MAX_K, FDB_ERR_UNSUPPORTED, "k out of range");
    const int qt = bf_qt(k);
    size_t rows = bf_chunk_rows(n, nq, qt, sm_count);
    size_t chunks = std::max<size_t>(1, (n + rows - 1) / rows);
    FDB_REQUIRE(chunks * (size_t)nq * k <= part_capacity, FDB_ERR_INVALID_ARG,
                "partial top-k buffer too small");
    if (k <= 32) bf_launch_m<1, 8>(metric, s, Q, nq, qnorm, X, n, dim, xnorm, rows, chunks, tag_base, k, part);
    else if (k <= 64) bf_launch_m<2, 8>(metric, s, Q, nq, qnorm, X, n, dim, xnorm, rows, chunks, tag_base, k, part);
    else if (k <= 128) bf_launch_m<4, 4>(metric, s, Q, nq, qnorm, X, n, dim, xnorm, rows, chunks, tag_base, k, part);
    else bf_launch_m<8, 4>(metric, s, Q, nq, qnorm, X, n, dim, xnorm, rows, chunks, tag_base, k, part);
    return (int)chunks;
}

}  // namespace fdb
