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

void launch_assign(cudaStream_t s, const float* x, size_t n, int dim, int ld, const float* cent,
                   int k, uint32_t* out) {
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

void kmeans_run(Ctx& ctx, const KMeansProblem& pb, float* cent, int* iters_out) {
    cudaStream_t s = ctx.stream;
    const size_t n = pb.n;
    const int nsub = pb.nsub, k = pb.k, dim = pb.dim;
    const size_t csz = (size_t)nsub * k * dim;
    DevBuf<float> neu(csz), dc((size_t)nsub * k), change(nsub);
    DevBuf<uint32_t> assign(n * nsub), perm(n * nsub);
    DevBuf<uint64_t> offs((size_t)nsub * k + 1);
    DevBuf<int> d_active(nsub);
    std::vector<int> active(nsub, 1);
    std::vector<float> h_change(nsub);
    for (int q = 0; q < nsub; ++q) iters_out[q] = 0;
    for (int it = 0; it < pb.max_iters; ++it) {
        bool any = false;
        for (int q = 0; q < nsub; ++q) any |= active[q] != 0;
        if (!any) break;
        FDB_CUDA(cudaMemcpyAsync(d_active.p, active.data(), nsub * sizeof(int),
                                 cudaMemcpyHostToDevice, s));
        launch_assign_multi(s, pb.x, n, dim, pb.ld, nsub, cent, k, assign.p, d_active.p);
        group_multi(s, assign.p, n, nsub, k, perm.p, offs.p);
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
                                float* __restrict__ out_row) {
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
    }
    __syncthreads();
    for (int j = threadIdx.x; j < dim; j += blockDim.x) out_row[j] = x[(size_t)sel * dim + j];
}

void kmeans_pp_init(Ctx& ctx, const float* x, size_t n, int dim, int k,
                    const uint32_t* init_idx, const float* kpp_u, float* cent) {
    cudaStream_t s = ctx.stream;
    FDB_REQUIRE(init_idx[0] < n, FDB_ERR_INVALID_ARG, "k-means++ first pick out of range");
    FDB_CUDA(cudaMemcpyAsync(cent, x + (size_t)init_idx[0] * dim, dim * sizeof(float),
                             cudaMemcpyDeviceToDevice, s));
    DevBuf<float> mind(n);
    fill_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(mind.p, n, FLT_MAX);
    FDB_LAUNCH_CHECK();
    for (int c = 1; c < k; ++c) {
        FDB_REQUIRE(init_idx[c] < n, FDB_ERR_INVALID_ARG, "k-means++ fallback pick out of range");
        kpp_update_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(
            x, n, dim, cent + (size_t)(c - 1) * dim, mind.p);
        FDB_LAUNCH_CHECK();
        kpp_pick_kernel<<<1, 128, 0, s>>>(mind.p, n, kpp_u[c], init_idx[c], x, dim,
                                          cent + (size_t)c * dim);
        FDB_LAUNCH_CHECK();
    }
    FDB_CUDA(cudaStreamSynchronize(s));
}

}  // namespace fdb
