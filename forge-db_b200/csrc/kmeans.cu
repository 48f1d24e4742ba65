// kmeans.cu -- Lloyd k-means on the device with the reference's exact
// arithmetic (forge-db src/kmeans.rs:45-193, 200-329):
//   assign : first-minimum argmin of the AVX2-order L2^2   (kmeans.rs:257-270)
//   update : per-cluster serial sum in point order, / count as f32, empty
//            clusters keep their centroid                   (kmeans.rs:276-314)
//   change : ordered sum of L2^2(old, new) / k, stop below 1e-3
//                                                            (kmeans.rs:320-329)
// The ordered update is what makes bit-exactness possible on a GPU: points
// are first grouped by cluster with a stable radix sort (ties keep point
// order), then one thread per (cluster, dimension) adds its points serially.
// No floating-point atomics or tree reductions are used anywhere.
//
// Several independent problems (the M subspaces of PQ training) run in one
// launch; each has its own convergence flag, as each subspace's KMeans in
// the reference stops on its own (pq.rs:71-87).
#include <cub/cub.cuh>

#include <algorithm>
#include <cfloat>

#include "fdb_device.cuh"
#include "fdb_internal.h"
#include "fdb_kernels.h"

namespace fdb {

constexpr float CONVERGENCE_THRESHOLD = 0.001f;  // constants.rs:29
constexpr int ASSIGN_THREADS = 128;
constexpr int ASSIGN_CB = 4;  // centroids sharing one load of a point's coordinates

// ---------------------------------------------------------------------------
// assign
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(ASSIGN_THREADS)
    assign_kernel(const float* __restrict__ x, size_t n, int dim, int ld,
                  const float* __restrict__ cent, int k, int tc, uint32_t* __restrict__ out,
                  const int* __restrict__ active) {
    const int s = blockIdx.y;
    if (active && !active[s]) return;
    extern __shared__ float sc[];  // tc rows of `dim`
    const float* cs = cent + (size_t)s * k * dim;
    const size_t i = (size_t)blockIdx.x * ASSIGN_THREADS + threadIdx.x;
    const bool live = i < n;
    const float* xr = x + (live ? i : 0) * (size_t)ld + (size_t)s * dim;
    const int full = dim & ~7;
    float best = 0.0f;
    uint32_t bi = 0;
    for (int t0 = 0; t0 < k; t0 += tc) {
        const int nt = min(tc, k - t0);
        __syncthreads();
        for (int e = threadIdx.x; e < nt * dim; e += ASSIGN_THREADS)
            sc[e] = cs[(size_t)t0 * dim + e];
        __syncthreads();
        if (!live) continue;
        for (int c0 = 0; c0 < nt; c0 += ASSIGN_CB) {
            float acc[ASSIGN_CB][8];
#pragma unroll
            for (int b = 0; b < ASSIGN_CB; ++b)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[b][j] = 0.0f;
            for (int g = 0; g < full; g += 8) {
                float xv[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) xv[j] = __ldg(xr + g + j);
#pragma unroll
                for (int b = 0; b < ASSIGN_CB; ++b) {
                    const float* cr = sc + (c0 + b) * dim + g;  // rows past nt are unused
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        float d = __fsub_rn(xv[j], cr[j]);
                        acc[b][j] = __fmaf_rn(d, d, acc[b][j]);
                    }
                }
            }
#pragma unroll
            for (int b = 0; b < ASSIGN_CB; ++b) {
                if (c0 + b >= nt) break;
                float t = lane_sum(acc[b]);
                const float* cr = sc + (c0 + b) * dim;
                for (int g = full; g < dim; ++g) {
                    float d = __fsub_rn(__ldg(xr + g), cr[g]);
                    t = __fadd_rn(t, __fmul_rn(d, d));
                }
                const int c = t0 + c0 + b;
                // min_by keeps the running minimum unless it compares Greater.
                if (c == 0 || best > t) {
                    best = t;
                    bi = (uint32_t)c;
                }
            }
        }
    }
    if (live) out[(size_t)s * n + i] = bi;
}

static int assign_tile(int dim, int k, size_t* smem) {
    int tc = (32768 / (dim * 4)) / ASSIGN_CB * ASSIGN_CB;
    tc = std::max(tc, ASSIGN_CB);
    int kr = (k + ASSIGN_CB - 1) / ASSIGN_CB * ASSIGN_CB;
    tc = std::min(tc, kr);
    *smem = (size_t)tc * dim * sizeof(float);
    return tc;
}

static void launch_assign_multi(cudaStream_t s, const float* x, size_t n, int dim, int ld,
                                int nsub, const float* cent, int k, uint32_t* out,
                                const int* active) {
    if (n == 0) return;
    size_t smem = 0;
    int tc = assign_tile(dim, k, &smem);
    FDB_REQUIRE(smem <= 227 * 1024, FDB_ERR_UNSUPPORTED, "dimension too large for assign");
    if (smem > 48 * 1024)
        FDB_CUDA(cudaFuncSetAttribute(assign_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem));
    dim3 grid((unsigned)((n + ASSIGN_THREADS - 1) / ASSIGN_THREADS), (unsigned)nsub);
    assign_kernel<<<grid, ASSIGN_THREADS, smem, s>>>(x, n, dim, ld, cent, k, tc, out, active);
    FDB_LAUNCH_CHECK();
}

// ---------------------------------------------------------------------------
// register-tiled assignment (one problem, large n x k)
// ---------------------------------------------------------------------------
// A block covers AT_Q points x AT_C centroids; a thread AT_TQ x AT_TC pairs.
// The distance is l2sq_exact's: eight lane accumulators over i = j (mod 8),
// summed left to right, then the unfused scalar tail.  The block runs the
// lanes in turn, staging only dims i = j (mod 8) of both tiles (transposed) in
// shared memory, so a pair needs two registers and the result is
// bit-identical.  Each block reduces, per point, the first minimum of its
// centroids into a 64-bit key (orderable distance, centroid index) and folds
// it into best[p] with one atomicMin: smaller distance first, then the
// smaller index -- the first minimum over all centroids, as Iterator::min_by.
constexpr int AT_Q = 128, AT_C = 128, AT_TQ = 4, AT_TC = 8;
constexpr int AT_THREADS = (AT_Q / AT_TQ) * (AT_C / AT_TC);  // 512

__global__ void __launch_bounds__(AT_THREADS)
    assign_tiled_kernel(const float* __restrict__ XT, size_t n, size_t n_pad, int dim,
                        const float* __restrict__ CT, int k, int k_pad,
                        unsigned long long* __restrict__ best) {
    extern __shared__ __align__(16) float at_smem[];
    const int G = dim >> 3;  // full groups of eight
    float* qs = at_smem;                 // [G][AT_Q]
    float* cs = qs + (size_t)G * AT_Q;   // [G][AT_C]
    unsigned long long* red = reinterpret_cast<unsigned long long*>(cs + (size_t)G * AT_C);
    const size_t p0 = (size_t)blockIdx.x * AT_Q;
    const int c0 = blockIdx.y * AT_C;
    const int tq = threadIdx.x & 31;  // point group (4 points)
    const int tc = threadIdx.x >> 5;  // centroid group (8 centroids)
    const float* qb = qs + tq * AT_TQ;
    const float* cb = cs + tc * AT_TC;
    float t[AT_TQ][AT_TC];
#pragma unroll 1
    for (int j = 0; j < 8; ++j) {
        __syncthreads();
        for (int e = threadIdx.x; e < G * (AT_Q / 4); e += AT_THREADS) {
            const int g = e / (AT_Q / 4), v = e - g * (AT_Q / 4);
            reinterpret_cast<float4*>(qs + (size_t)g * AT_Q)[v] = __ldg(
                reinterpret_cast<const float4*>(XT + (size_t)(8 * g + j) * n_pad + p0) + v);
        }
        for (int e = threadIdx.x; e < G * (AT_C / 4); e += AT_THREADS) {
            const int g = e / (AT_C / 4), v = e - g * (AT_C / 4);
            reinterpret_cast<float4*>(cs + (size_t)g * AT_C)[v] = __ldg(
                reinterpret_cast<const float4*>(CT + (size_t)(8 * g + j) * k_pad + c0) + v);
        }
        __syncthreads();
        float acc[AT_TQ][AT_TC];
#pragma unroll
        for (int a = 0; a < AT_TQ; ++a)
#pragma unroll
            for (int b = 0; b < AT_TC; ++b) acc[a][b] = 0.0f;
#pragma unroll 4
        for (int g = 0; g < G; ++g) {
            const float4 qv = *reinterpret_cast<const float4*>(qb + (size_t)g * AT_Q);
            const float4 c0v = *reinterpret_cast<const float4*>(cb + (size_t)g * AT_C);
            const float4 c1v = *reinterpret_cast<const float4*>(cb + (size_t)g * AT_C + 4);
            const float qa[AT_TQ] = {qv.x, qv.y, qv.z, qv.w};
            const float ca[AT_TC] = {c0v.x, c0v.y, c0v.z, c0v.w, c1v.x, c1v.y, c1v.z, c1v.w};
#pragma unroll
            for (int a = 0; a < AT_TQ; ++a)
#pragma unroll
                for (int b = 0; b < AT_TC; ++b) {
                    const float d = __fsub_rn(qa[a], ca[b]);
                    acc[a][b] = __fmaf_rn(d, d, acc[a][b]);
                }
        }
#pragma unroll
        for (int a = 0; a < AT_TQ; ++a)
#pragma unroll
            for (int b = 0; b < AT_TC; ++b) t[a][b] = j == 0 ? acc[a][b] : __fadd_rn(t[a][b], acc[a][b]);
    }
    for (int i = 8 * G; i < dim; ++i) {  // unfused scalar tail
#pragma unroll
        for (int a = 0; a < AT_TQ; ++a) {
            const float xq = __ldg(XT + (size_t)i * n_pad + p0 + tq * AT_TQ + a);
#pragma unroll
            for (int b = 0; b < AT_TC; ++b) {
                const float d = __fsub_rn(xq, __ldg(CT + (size_t)i * k_pad + c0 + tc * AT_TC + b));
                t[a][b] = __fadd_rn(t[a][b], __fmul_rn(d, d));
            }
        }
    }
#pragma unroll
    for (int a = 0; a < AT_TQ; ++a) {
        unsigned long long key = ~0ull;
#pragma unroll
        for (int b = 0; b < AT_TC; ++b) {
            const int l = c0 + tc * AT_TC + b;
            if (l < k) {
                const unsigned long long kk = make_key(t[a][b], (uint32_t)l);
                key = kk < key ? kk : key;
            }
        }
        red[(size_t)tc * AT_Q + tq * AT_TQ + a] = key;
    }
    __syncthreads();
    if (threadIdx.x < AT_Q) {
        const size_t p = p0 + threadIdx.x;
        if (p < n) {
            unsigned long long key = ~0ull;
            for (int r = 0; r < AT_C / AT_TC; ++r) {
                const unsigned long long kk = red[(size_t)r * AT_Q + threadIdx.x];
                key = kk < key ? kk : key;
            }
            atomicMin(best + p, key);
        }
    }
}

__global__ void key_index_kernel(const unsigned long long* __restrict__ best, size_t n,
                                 uint32_t* __restrict__ out) {
    const size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t < n) out[t] = (uint32_t)best[t];
}

// out[p] = first-minimum centroid of point p, from the transposed operands
// XT [dim][n_pad] (n_pad a multiple of 128) and CT [dim][k_pad] (k_pad a
// multiple of 128).  best: scratch of n keys.
void launch_assign_tiled(cudaStream_t s, const float* XT, size_t n, size_t n_pad, int dim,
                         const float* CT, int k, int k_pad, unsigned long long* best,
                         uint32_t* out) {
    if (n == 0) return;
    FDB_REQUIRE(n_pad % AT_Q == 0 && k_pad % AT_C == 0, FDB_ERR_UNSUPPORTED, "bad padding");
    const size_t smem = (size_t)(dim >> 3) * (AT_Q + AT_C) * sizeof(float) +
                        (size_t)(AT_C / AT_TC) * AT_Q * sizeof(unsigned long long);
    FDB_REQUIRE(smem <= 227 * 1024, FDB_ERR_UNSUPPORTED, "dimension too large for tiled assign");
    if (smem > 48 * 1024)
        FDB_CUDA(cudaFuncSetAttribute(assign_tiled_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    FDB_CUDA(cudaMemsetAsync(best, 0xff, n * sizeof(unsigned long long), s));
    dim3 grid((unsigned)(n_pad / AT_Q), (unsigned)(k_pad / AT_C));
    assign_tiled_kernel<<<grid, AT_THREADS, smem, s>>>(XT, n, n_pad, dim, CT, k, k_pad, best);
    FDB_LAUNCH_CHECK();
    key_index_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(best, n, out);
    FDB_LAUNCH_CHECK();
}

// The tiled kernel pays off for many points and centroids of 16+ dimensions
// (and its dim/8 rows of both tiles must fit in shared memory).
static bool assign_tiled_ok(size_t n, int dim, int k) {
    return n >= 4096 && k >= 64 && dim >= 16 && (size_t)(dim >> 3) * (AT_Q + AT_C) * 4 +
                                                       16 * AT_Q * 8 <= 200 * 1024;
}

// Transposed, zero-padded copies of the points (once) and the centroids.
struct AssignTiled {
    DevBuf<float> XT, CT;
    DevBuf<unsigned long long> best;
    size_t n_pad = 0;
    int k_pad = 0;
    void prepare_points(cudaStream_t s, const float* x, size_t n, int dim) {
        n_pad = (n + AT_Q - 1) / AT_Q * AT_Q;
        XT.alloc(n_pad * dim);
        launch_transpose_pad(s, x, (int)n, dim, (int)n_pad, XT.p);
        best.alloc(n);
    }
    void run(cudaStream_t s, size_t n, int dim, const float* cent, int k, uint32_t* out) {
        k_pad = (k + AT_C - 1) / AT_C * AT_C;
        CT.ensure((size_t)k_pad * dim);
        launch_transpose_pad(s, cent, k, dim, k_pad, CT.p);
        launch_assign_tiled(s, XT.p, n, n_pad, dim, CT.p, k, k_pad, best.p, out);
    }
};

void launch_assign(cudaStream_t s, const float* x, size_t n, int dim, int ld, const float* cent,
                   int k, uint32_t* out) {
    if (ld == dim && assign_tiled_ok(n, dim, k) && n < (1ull << 31)) {
        AssignTiled at;
        at.prepare_points(s, x, n, dim);
        at.run(s, n, dim, cent, k, out);
        FDB_CUDA(cudaStreamSynchronize(s));  // scratch is released on return
        return;
    }
    launch_assign_multi(s, x, n, dim, ld, 1, cent, k, out, nullptr);
}

// ---------------------------------------------------------------------------
// stable grouping
// ---------------------------------------------------------------------------
__global__ void make_group_keys(const uint32_t* __restrict__ assign, size_t n, int nsub, int k,
                                uint32_t* __restrict__ keys, uint32_t* __restrict__ vals,
                                uint32_t* __restrict__ counts) {
    size_t total = n * nsub;
    for (size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (size_t)gridDim.x * blockDim.x) {
        uint32_t s = (uint32_t)(t / n);
        uint32_t key = s * (uint32_t)k + assign[t];
        keys[t] = key;
        vals[t] = (uint32_t)(t - (size_t)s * n);
        atomicAdd(&counts[key], 1u);  // integer: order-independent
    }
}

static int bits_for(uint32_t v) {
    int b = 1;
    while (b < 32 && (1ull << b) <= v) ++b;
    return b;
}

// Groups `nsub` problems of n assignments (layout [nsub][n]) by (problem,
// cluster); perm[p] is the within-problem point index at group position p
// and offsets[nsub*k + 1] delimit the groups.  Stable: the radix sort keeps
// point order among equal keys, so each group lists its points ascending.
static void group_multi(cudaStream_t s, const uint32_t* assign, size_t n, int nsub, int k,
                        uint32_t* perm, uint64_t* offsets) {
    const size_t total = n * (size_t)nsub;
    const uint32_t nkeys = (uint32_t)nsub * (uint32_t)k;
    DevBuf<uint32_t> keys(total), keys_out(total), vals(total), counts(nkeys + 1);
    FDB_CUDA(cudaMemsetAsync(counts.p, 0, counts.bytes(), s));
    unsigned grid = (unsigned)std::min<size_t>((total + 255) / 256, 148 * 16);
    make_group_keys<<<grid, 256, 0, s>>>(assign, n, nsub, k, keys.p, vals.p, counts.p);
    FDB_LAUNCH_CHECK();
    size_t tmp_sort = 0, tmp_scan = 0;
    const int end_bit = bits_for(nkeys);
    FDB_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, tmp_sort, keys.p, keys_out.p, vals.p, perm,
                                             total, 0, end_bit, s));
    FDB_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, tmp_scan, counts.p, offsets,
                                           (size_t)nkeys + 1, s));
    DevBuf<uint8_t> tmp(std::max(tmp_sort, tmp_scan));
    FDB_CUDA(cub::DeviceRadixSort::SortPairs(tmp.p, tmp_sort, keys.p, keys_out.p, vals.p, perm,
                                             total, 0, end_bit, s));
    FDB_CUDA(cub::DeviceScan::ExclusiveSum(tmp.p, tmp_scan, counts.p, offsets,
                                           (size_t)nkeys + 1, s));
    // The buffers above are released when this returns; keep the stream
    // ordered with respect to their reuse.
    FDB_CUDA(cudaStreamSynchronize(s));
}

void group_by_assignment(Ctx& ctx, const uint32_t* assign, size_t n, int k, uint32_t* perm,
                         uint64_t* offsets) {
    group_multi(ctx.stream, assign, n, 1, k, perm, offsets);
}

// ---------------------------------------------------------------------------
// update and change
// ---------------------------------------------------------------------------
__global__ void update_kernel(const float* __restrict__ x, size_t n, int dim, int ld, int nsub,
                              int k, const uint32_t* __restrict__ perm,
                              const uint64_t* __restrict__ offs, const float* __restrict__ old,
                              float* __restrict__ neu, const int* __restrict__ active) {
    const size_t total = (size_t)nsub * k * dim;
    const size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= total) return;
    const size_t per = (size_t)k * dim;
    const int s = (int)(t / per);
    const size_t rem = t - (size_t)s * per;
    const int c = (int)(rem / dim);
    const int j = (int)(rem - (size_t)c * dim);
    const float ov = old[t];
    if (active && !active[s]) { neu[t] = ov; return; }
    const uint64_t beg = offs[(size_t)s * k + c], end = offs[(size_t)s * k + c + 1];
    if (beg == end) { neu[t] = ov; return; }  // empty cluster keeps its centroid
    const uint32_t* pp = perm + (size_t)s * n;
    // perm positions are global across problems: group p of problem s lies
    // in [s*n, (s+1)*n) of the sorted order.
    float sum = 0.0f;
    const float* col = x + (size_t)s * dim + j;
    for (uint64_t p = beg; p < end; ++p) {
        uint32_t i = pp[p - (uint64_t)s * n];
        sum = __fadd_rn(sum, __ldg(col + (size_t)i * ld));
    }
    neu[t] = __fdiv_rn(sum, __ull2float_rn(end - beg));
}

__global__ void change_dist_kernel(const float* __restrict__ old, const float* __restrict__ neu,
                                   int nsub, int k, int dim, float* __restrict__ dc,
                                   const int* __restrict__ active) {
    int t = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= nsub * k) return;
    int s = t / k;
    if (active && !active[s]) return;
    dc[t] = l2sq_exact(old + (size_t)t * dim, neu + (size_t)t * dim, dim);
}

__global__ void change_sum_kernel(const float* __restrict__ dc, int nsub, int k,
                                  float* __restrict__ change, const int* __restrict__ active) {
    int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s >= nsub) return;
    if (active && !active[s]) { change[s] = 0.0f; return; }
    float total = 0.0f;
    for (int c = 0; c < k; ++c) total = __fadd_rn(total, dc[(size_t)s * k + c]);
    change[s] = __fdiv_rn(total, (float)k);
}

// ever[g] |= group g is non-empty, for the problems still iterating.
__global__ void nonempty_kernel(const uint64_t* __restrict__ offs, int nsub, int k,
                                const int* __restrict__ active, uint8_t* __restrict__ ever) {
    const int g = blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= nsub * k || !active[g / k]) return;
    if (offs[g + 1] > offs[g]) ever[g] = 1;
}

void kmeans_run(Ctx& ctx, const KMeansProblem& pb, float* cent, int* iters_out,
                uint8_t* ever_out) {
    cudaStream_t s = ctx.stream;
    const size_t n = pb.n;
    const int nsub = pb.nsub, k = pb.k, dim = pb.dim;
    const size_t csz = (size_t)nsub * k * dim;
    DevBuf<float> neu(csz), dc((size_t)nsub * k), change(nsub);
    DevBuf<uint32_t> assign(n * nsub), perm(n * nsub);
    DevBuf<uint64_t> offs((size_t)nsub * k + 1);
    DevBuf<int> d_active(nsub);
    DevBuf<uint8_t> ever;
    if (ever_out) {
        ever.alloc((size_t)nsub * k);
        FDB_CUDA(cudaMemsetAsync(ever.p, 0, ever.bytes(), s));
    }
    std::vector<int> active(nsub, 1);
    std::vector<float> h_change(nsub);
    for (int q = 0; q < nsub; ++q) iters_out[q] = 0;
    // one large problem: register-tiled assignment over a transposed copy
    AssignTiled at;
    const bool tiled = nsub == 1 && pb.ld == dim && assign_tiled_ok(n, dim, k) &&
                       n < (1ull << 31);
    if (tiled) at.prepare_points(s, pb.x, n, dim);
    for (int it = 0; it < pb.max_iters; ++it) {
        bool any = false;
        for (int q = 0; q < nsub; ++q) any |= active[q] != 0;
        if (!any) break;
        FDB_CUDA(cudaMemcpyAsync(d_active.p, active.data(), nsub * sizeof(int),
                                 cudaMemcpyHostToDevice, s));
        if (tiled) at.run(s, n, dim, cent, k, assign.p);
        else launch_assign_multi(s, pb.x, n, dim, pb.ld, nsub, cent, k, assign.p, d_active.p);
        group_multi(s, assign.p, n, nsub, k, perm.p, offs.p);
        if (ever_out) {
            nonempty_kernel<<<(nsub * k + 255) / 256, 256, 0, s>>>(offs.p, nsub, k, d_active.p,
                                                                   ever.p);
            FDB_LAUNCH_CHECK();
        }
        unsigned g = (unsigned)((csz + 255) / 256);
        update_kernel<<<g, 256, 0, s>>>(pb.x, n, dim, pb.ld, nsub, k, perm.p, offs.p, cent, neu.p,
                                        d_active.p);
        FDB_LAUNCH_CHECK();
        change_dist_kernel<<<(nsub * k + 255) / 256, 256, 0, s>>>(cent, neu.p, nsub, k, dim, dc.p,
                                                                  d_active.p);
        FDB_LAUNCH_CHECK();
        change_sum_kernel<<<(nsub + 127) / 128, 128, 0, s>>>(dc.p, nsub, k, change.p, d_active.p);
        FDB_LAUNCH_CHECK();
        FDB_CUDA(cudaMemcpyAsync(cent, neu.p, csz * sizeof(float), cudaMemcpyDeviceToDevice, s));
        FDB_CUDA(cudaMemcpyAsync(h_change.data(), change.p, nsub * sizeof(float),
                                 cudaMemcpyDeviceToHost, s));
        FDB_CUDA(cudaStreamSynchronize(s));
        for (int q = 0; q < nsub; ++q) {
            if (!active[q]) continue;
            iters_out[q]++;
            if (h_change[q] < CONVERGENCE_THRESHOLD) active[q] = 0;
        }
    }
    if (ever_out) {
        FDB_CUDA(cudaMemcpyAsync(ever_out, ever.p, ever.bytes(), cudaMemcpyDeviceToHost, s));
        FDB_CUDA(cudaStreamSynchronize(s));
    }
}

// ---------------------------------------------------------------------------
// k-means++ (k <= 64), src/kmeans.rs:106-141 (fit_raw) / :200-252 (fit)
// ---------------------------------------------------------------------------
__global__ void fill_kernel(float* p, size_t n, float v) {
    size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t < n) p[t] = v;
}

__global__ void kpp_update_kernel(const float* __restrict__ x, size_t n, int dim,
                                  const float* __restrict__ c, float* __restrict__ mind) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float d = l2sq_exact(x + i * dim, c, dim);
    mind[i] = fminf(mind[i], d);  // fold(f32::MAX, f32::min)
}

// Sequential total and subtract-walk, exactly as the reference: one thread.
__global__ void kpp_pick_kernel(const float* __restrict__ mind, size_t n, float u,
                                uint32_t fallback, const float* __restrict__ x, int dim,
                                float* __restrict__ out_row, uint32_t* __restrict__ pick_out) {
    __shared__ uint32_t sel;
    if (threadIdx.x == 0) {
        float total = 0.0f;
        for (size_t i = 0; i < n; ++i) total = __fadd_rn(total, mind[i]);
        uint32_t pick;
        if (total == 0.0f) {
            pick = fallback;
        } else {
            float r = __fmul_rn(u, total);  // gen_range(0.0..total) = u * total + 0
            pick = (uint32_t)(n - 1);
            for (size_t i = 0; i < n; ++i) {
                r = __fsub_rn(r, mind[i]);
                if (r <= 0.0f) { pick = (uint32_t)i; break; }
            }
        }
        sel = pick;
        *pick_out = pick;
    }
    __syncthreads();
    for (int j = threadIdx.x; j < dim; j += blockDim.x) out_row[j] = x[(size_t)sel * dim + j];
}

void kmeans_pp_init(Ctx& ctx, const float* x, size_t n, int dim, int k,
                    const uint32_t* init_idx, const float* kpp_u, float* cent,
                    uint32_t* picks_out) {
    cudaStream_t s = ctx.stream;
    FDB_REQUIRE(init_idx[0] < n, FDB_ERR_INVALID_ARG, "k-means++ first pick out of range");
    FDB_CUDA(cudaMemcpyAsync(cent, x + (size_t)init_idx[0] * dim, dim * sizeof(float),
                             cudaMemcpyDeviceToDevice, s));
    DevBuf<float> mind(n);
    DevBuf<uint32_t> picks((size_t)k);
    fill_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(mind.p, n, FLT_MAX);
    FDB_LAUNCH_CHECK();
    for (int c = 1; c < k; ++c) {
        FDB_REQUIRE(init_idx[c] < n, FDB_ERR_INVALID_ARG, "k-means++ fallback pick out of range");
        kpp_update_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
            x, n, dim, cent + (size_t)(c - 1) * dim, mind.p);
        FDB_LAUNCH_CHECK();
        kpp_pick_kernel<<<1, 128, 0, s>>>(mind.p, n, kpp_u[c], init_idx[c], x, dim,
                                          cent + (size_t)c * dim, picks.p + c);
        FDB_LAUNCH_CHECK();
    }
    if (picks_out) {
        picks_out[0] = init_idx[0];
        if (k > 1)
            FDB_CUDA(cudaMemcpyAsync(picks_out + 1, picks.p + 1, (size_t)(k - 1) * 4,
                                     cudaMemcpyDeviceToHost, s));
    }
    FDB_CUDA(cudaStreamSynchronize(s));
}

}  // namespace fdb
