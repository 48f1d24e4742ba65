// distances.cu -- row-pair distances (DistanceMetric::compute,
// forge-db src/distance/mod.rs:40-48) and row gathers.
#include "fdb_device.cuh"
#include "fdb_internal.h"

namespace fdb {

__global__ void pairwise_kernel(int metric, const float* __restrict__ a,
                                const float* __restrict__ b, size_t n, int dim,
                                float* __restrict__ out) {
    size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float* x = a + i * dim;
    const float* y = b + i * dim;
    float r;
    switch (metric) {
        case EUCLIDEAN: r = __fsqrt_rn(l2sq_exact(x, y, dim)); break;
        case EUCLIDEAN_SQUARED: r = l2sq_exact(x, y, dim); break;
        case COSINE:
            r = cosine_from(dot_exact(x, y, dim), dot_exact(x, x, dim), dot_exact(y, y, dim));
            break;
        case DOT_PRODUCT: r = -dot_exact(x, y, dim); break;
        default: r = l1_exact(x, y, dim); break;
    }
    out[i] = r;
}

void launch_pairwise(cudaStream_t s, int metric, const float* a, const float* b, size_t n,
                     int dim, float* out) {
    if (n == 0) return;
    unsigned grid = (unsigned)((n + 255) / 256);
    pairwise_kernel<<<grid, 256, 0, s>>>(metric, a, b, n, dim, out);
    FDB_LAUNCH_CHECK();
}

__global__ void gather_rows_kernel(const float* __restrict__ x, size_t dim,
                                   const uint32_t* __restrict__ idx, size_t count,
                                   float* __restrict__ out) {
    size_t total = count * dim;
    for (size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (size_t)gridDim.x * blockDim.x) {
        size_t r = t / dim, c = t - r * dim;
        out[t] = x[(size_t)idx[r] * dim + c];
    }
}

void launch_gather_rows(cudaStream_t s, const float* x, size_t dim, const uint32_t* idx,
                        size_t count, float* out) {
    if (count == 0) return;
    size_t total = count * dim;
    unsigned grid = (unsigned)std::min<size_t>((total + 255) / 256, 148 * 32);
    gather_rows_kernel<<<grid, 256, 0, s>>>(x, dim, idx, count, out);
    FDB_LAUNCH_CHECK();
}

}  // namespace fdb
