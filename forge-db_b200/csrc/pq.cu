// pq.cu -- product-quantizer kernels (forge-db src/pq.rs:55-189):
//   codebook training  = M independent k-means(256, iters) runs over the
//                        sub-columns, batched into one set of launches
//                        (ProductQuantizer::try_train, pq.rs:55-95);
//   encode             = per-subspace first-minimum argmin of the AVX2-order
//                        L2^2, fused with the IVF residual (pq.rs:114-139,
//                        ivf_pq.rs:450-478);
//   lookup tables      = build_lookup_table_flat (pq.rs:175-189).
#include <algorithm>

#include "fdb_device.cuh"
#include "fdb_internal.h"

namespace fdb {

constexpr int ENC_THREADS = 128;

// One block of 128 points x one subspace.  The subspace's 256 codewords sit
// in shared memory; each thread's residual row sits there too (stride sub+1
// keeps the per-thread rows on distinct banks).
__global__ void __launch_bounds__(ENC_THREADS)
    pq_encode_kernel(const float* __restrict__ x, size_t n, int dim,
                     const float* __restrict__ cents, const uint32_t* __restrict__ assign,
                     const float* __restrict__ cb, int m, const uint32_t* __restrict__ slot,
                     uint8_t* __restrict__ codes) {
    const int s = blockIdx.y;
    const int sub = dim / m;
    extern __shared__ float sm[];
    float* scb = sm;
    float* sr = sm + KSUB * sub;
    for (int e = threadIdx.x; e < KSUB * sub; e += ENC_THREADS) scb[e] = cb[(size_t)s * KSUB * sub + e];
    const size_t i = (size_t)blockIdx.x * ENC_THREADS + threadIdx.x;
    const bool live = i < n;
    float* r = sr + threadIdx.x * (sub + 1);
    if (live) {
        const float* xr = x + i * dim + (size_t)s * sub;
        if (cents) {
            const float* cr = cents + (size_t)assign[i] * dim + (size_t)s * sub;
            for (int j = 0; j < sub; ++j) r[j] = __fsub_rn(xr[j], cr[j]);  // residual v - c
        } else {
            for (int j = 0; j < sub; ++j) r[j] = xr[j];
        }
    }
    __syncthreads();
    if (!live) return;
    float best = 0.0f;
    int bi = 0;
    for (int c = 0; c < KSUB; ++c) {
        float t = l2sq_exact(r, scb + c * sub, sub);
        if (c == 0 || best > t) { best = t; bi = c; }
    }
    codes[(slot ? (size_t)slot[i] : i) * m + s] = (uint8_t)bi;
}

void launch_pq_encode(cudaStream_t s, const float* x, size_t n, int dim, const float* cents,
                      const uint32_t* assign, const float* cb, int m, const uint32_t* slot,
                      uint8_t* codes) {
    if (n == 0) return;
    const int sub = dim / m;
    size_t smem = ((size_t)KSUB * sub + (size_t)ENC_THREADS * (sub + 1)) * sizeof(float);
    FDB_REQUIRE(smem <= 227 * 1024, FDB_ERR_UNSUPPORTED, "subvector too long for the encoder");
    if (smem > 48 * 1024)
        FDB_CUDA(cudaFuncSetAttribute(pq_encode_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid((unsigned)((n + ENC_THREADS - 1) / ENC_THREADS), (unsigned)m);
    pq_encode_kernel<<<grid, ENC_THREADS, smem, s>>>(x, n, dim, cents, assign, cb, m, slot, codes);
    FDB_LAUNCH_CHECK();
}

__global__ void lut_kernel(const float* __restrict__ cb, int m, int dim,
                           const float* __restrict__ q, size_t nq, float* __restrict__ lut) {
    const size_t per = (size_t)m * KSUB;
    const size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= per * nq) return;
    const size_t qi = t / per;
    const int e = (int)(t - qi * per);
    const int sub = dim / m;
    const int s = e / KSUB;
    lut[t] = l2sq_exact(q + qi * dim + (size_t)s * sub, cb + (size_t)e * sub, sub);
}

void launch_lut(cudaStream_t s, const float* cb, int m, int dim, const float* q, size_t nq,
                float* lut) {
    size_t total = (size_t)m * KSUB * nq;
    if (total == 0) return;
    lut_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(cb, m, dim, q, nq, lut);
    FDB_LAUNCH_CHECK();
}

// Initial codewords: codebook[s][c] = sub-columns of row init_idx[s*256+c].
__global__ void pq_init_kernel(const float* __restrict__ x, int dim, int m,
                               const uint32_t* __restrict__ idx, float* __restrict__ cb) {
    const int sub = dim / m;
    const size_t total = (size_t)m * KSUB * sub;
    const size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= total) return;
    const size_t e = t / sub;  // s*256 + c
    const int j = (int)(t - e * sub);
    const int s = (int)(e / KSUB);
    cb[t] = x[(size_t)idx[e] * dim + (size_t)s * sub + j];
}

// ProductQuantizer::try_train on device rows x[n][dim].
void pq_train_dev(Ctx& ctx, const float* x, size_t n, int dim, int m, int iters,
                  const uint32_t* init_idx_host, float* cb, int* iters_out, uint8_t* ever_out) {
    cudaStream_t s = ctx.stream;
    const size_t ni = (size_t)m * KSUB;
    for (size_t e = 0; e < ni; ++e)
        FDB_REQUIRE(init_idx_host[e] < n, FDB_ERR_INVALID_ARG, "PQ init index out of range");
    DevBuf<uint32_t> d_idx(ni);
    FDB_CUDA(cudaMemcpyAsync(d_idx.p, init_idx_host, ni * sizeof(uint32_t),
                             cudaMemcpyHostToDevice, s));
    const int sub = dim / m;
    size_t total = ni * sub;
    pq_init_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(x, dim, m, d_idx.p, cb);
    FDB_LAUNCH_CHECK();
    KMeansProblem pb{x, n, sub, dim, m, KSUB, iters};
    kmeans_run(ctx, pb, cb, iters_out, ever_out);
}

}  // namespace fdb
