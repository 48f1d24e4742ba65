// ivfpq_kernels.cu -- the IVF-PQ search kernels.
//
//   coarse_dist_kernel : L2^2 of each query to every IVF centroid, AVX2 order
//                        (find_nearest_partitions, ivf_pq.rs:538-553, and
//                        the inline copy in batch_search, :865-888).
//   select_kernel      : the nprobe nearest lists per query, by (distance,
//                        list) -- one warp per query, WarpTopK.
//   scan_kernel        : per (query, probed list): residual q - c_l, the
//                        M x 256 LUT in shared memory (pq.rs:175-189), then a
//                        streaming scan of the list's codes with 128-bit
//                        loads, LUT gathers in the reference's ADC order
//                        (pq.rs:218-245 or 435-485) and a per-warp top-k;
//                        warps merge at the end of the query.
//   merge_lists_kernel : top-k of several sorted top-k lists per query (the
//                        cross-device merge after ncclAllGather, and the
//                        row-chunk merge of brute force).
//   finalize_kernel    : keys -> (id, distance), padding, counts.
#include "fdb_device.cuh"
#include "fdb_internal.h"
#include "fdb_kernels.h"

namespace fdb {

// ---------------------------------------------------------------------------
// coarse distances
// ---------------------------------------------------------------------------
constexpr int COARSE_QT = 8;
constexpr int COARSE_THREADS = 256;

__global__ void __launch_bounds__(COARSE_THREADS)
    coarse_dist_kernel(const float* __restrict__ Q, int nq, int dim,
                       const float* __restrict__ cents, int nlist, float* __restrict__ D) {
    extern __shared__ float sq[];  // COARSE_QT x dim
    const int q0 = blockIdx.y * COARSE_QT;
    const int nqt = min(COARSE_QT, nq - q0);
    for (int e = threadIdx.x; e < COARSE_QT * dim; e += COARSE_THREADS) {
        int qi = e / dim;
        sq[e] = qi < nqt ? Q[(size_t)q0 * dim + e] : 0.0f;
    }
    __syncthreads();
    const int l = blockIdx.x * COARSE_THREADS + threadIdx.x;
    if (l >= nlist) return;
    const float* cr = cents + (size_t)l * dim;
    float acc[COARSE_QT][8];
#pragma unroll
    for (int a = 0; a < COARSE_QT; ++a)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[a][j] = 0.0f;
    const int full = dim & ~7;
    for (int g = 0; g < full; g += 8) {
        float cv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) cv[j] = __ldg(cr + g + j);
#pragma unroll
        for (int a = 0; a < COARSE_QT; ++a) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float d = __fsub_rn(sq[a * dim + g + j], cv[j]);
                acc[a][j] = __fmaf_rn(d, d, acc[a][j]);
            }
        }
    }
#pragma unroll
    for (int a = 0; a < COARSE_QT; ++a) {
        if (a >= nqt) break;
        float t = lane_sum(acc[a]);
        for (int g = full; g < dim; ++g) {
            float d = __fsub_rn(sq[a * dim + g], __ldg(cr + g));
            t = __fadd_rn(t, __fmul_rn(d, d));
        }
        D[(size_t)(q0 + a) * nlist + l] = t;
    }
}

void launch_coarse_dist(cudaStream_t s, const float* Q, int nq, int dim, const float* cents,
                        int nlist, float* D) {
    if (nq == 0) return;
    size_t smem = (size_t)COARSE_QT * dim * sizeof(float);
    FDB_REQUIRE(smem <= 227 * 1024, FDB_ERR_UNSUPPORTED, "dimension too large");
    if (smem > 48 * 1024)
        FDB_CUDA(cudaFuncSetAttribute(coarse_dist_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid((nlist + COARSE_THREADS - 1) / COARSE_THREADS, (nq + COARSE_QT - 1) / COARSE_QT);
    coarse_dist_kernel<<<grid, COARSE_THREADS, smem, s>>>(Q, nq, dim, cents, nlist, D);
    FDB_LAUNCH_CHECK();
}

// Register-tiled coarse distances for dim <= 256.  A block covers CT_Q queries
// x CT_C centroids with both tiles transposed in shared memory ([dim][..]);
// a thread owns CT_TQ x CT_TC pairs.  The AVX2 order of l2sq_exact (eight
// lane accumulators over i = j (mod 8), then a left-to-right lane sum, then
// the unfused scalar tail) is kept by running the lanes in the outer loop:
// lane j's accumulator is complete before it is added to the running sum, so
// only two registers per pair are live and every result is bit-identical.
constexpr int CT_Q = 32, CT_C = 128, CT_TQ = 4, CT_TC = 8;
constexpr int CT_THREADS = (CT_Q / CT_TQ) * (CT_C / CT_TC);  // 128
constexpr int CT_MAX_DIM = 256;

// out[i][q] = x[q][i] for q < n, 0 for n <= q < npad.
__global__ void transpose_pad_kernel(const float* __restrict__ x, int n, int dim, int npad,
                                     float* __restrict__ out) {
    __shared__ float tile[32][33];
    const int q0 = blockIdx.x * 32, i0 = blockIdx.y * 32;
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int q = q0 + r, i = i0 + threadIdx.x;
        tile[r][threadIdx.x] = (q < n && i < dim) ? x[(size_t)q * dim + i] : 0.0f;
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int i = i0 + r, q = q0 + threadIdx.x;
        if (i < dim && q < npad) out[(size_t)i * npad + q] = tile[threadIdx.x][r];
    }
}

// Shared memory holds one lane's rows at a time: for lane j the rows
// i = j, j + 8, ... (< full) of both tiles (then the tail rows), so a block
// needs (full / 8) x (CT_Q + CT_C) floats and many blocks fit on an SM.
__global__ void __launch_bounds__(CT_THREADS)
    coarse_tiled_kernel(const float* __restrict__ QT, int nq, int nq_pad, int dim,
                        const float* __restrict__ CT, int nlist, int nlist_pad,
                        float* __restrict__ D) {
    extern __shared__ __align__(16) float ct_smem[];
    const int full = dim & ~7, rows = max(full / 8, dim - full);
    float* qs = ct_smem;              // [rows][CT_Q]
    float* cs = qs + rows * CT_Q;     // [rows][CT_C]
    const int q0 = blockIdx.y * CT_Q, c0 = blockIdx.x * CT_C;
    const int tq = threadIdx.x & (CT_Q / CT_TQ - 1);  // 0..7
    const int tc = threadIdx.x / (CT_Q / CT_TQ);      // 0..15
    const float* qb = qs + tq * CT_TQ;
    const float* cb = cs + tc * CT_TC;
    // rows i0, i0 + step, ... (nr of them) of both tiles into shared memory
    auto stage = [&](int i0, int step, int nr) {
        __syncthreads();  // the previous stage is no longer read
        for (int e = threadIdx.x; e < nr * (CT_Q / 4); e += CT_THREADS) {
            const int r = e / (CT_Q / 4), v = e - r * (CT_Q / 4);
            reinterpret_cast<float4*>(qs + r * CT_Q)[v] = __ldg(
                reinterpret_cast<const float4*>(QT + (size_t)(i0 + r * step) * nq_pad + q0) + v);
        }
        for (int e = threadIdx.x; e < nr * (CT_C / 4); e += CT_THREADS) {
            const int r = e / (CT_C / 4), v = e - r * (CT_C / 4);
            reinterpret_cast<float4*>(cs + r * CT_C)[v] = __ldg(
                reinterpret_cast<const float4*>(CT + (size_t)(i0 + r * step) * nlist_pad + c0) + v);
        }
        __syncthreads();
    };
    float t[CT_TQ][CT_TC];
    const int nr = full / 8;
#pragma unroll 1
    for (int j = 0; j < 8; ++j) {
        float acc[CT_TQ][CT_TC];
#pragma unroll
        for (int a = 0; a < CT_TQ; ++a)
#pragma unroll
            for (int b = 0; b < CT_TC; ++b) acc[a][b] = 0.0f;
        if (nr > 0) stage(j, 8, nr);
        // packed pairs of centroids: sub.rn.f32x2 / fma.rn.f32x2 perform two
        // independent round-to-nearest operations, the same results as the
        // scalar __fsub_rn / __fmaf_rn, in half the instructions
        uint64_t* acc2 = reinterpret_cast<uint64_t*>(&acc[0][0]);
#pragma unroll 4
        for (int r = 0; r < nr; ++r) {  // element i = j + 8 r
            const float4 qv = *reinterpret_cast<const float4*>(qb + r * CT_Q);
            const ulonglong2 c01 = *reinterpret_cast<const ulonglong2*>(cb + r * CT_C);
            const ulonglong2 c23 = *reinterpret_cast<const ulonglong2*>(cb + r * CT_C + 4);
            const uint64_t cpair[CT_TC / 2] = {c01.x, c01.y, c23.x, c23.y};
            const float qa[CT_TQ] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
            for (int a = 0; a < CT_TQ; ++a) {
                const uint32_t qb32 = __float_as_uint(qa[a]);
                const uint64_t qq = ((uint64_t)qb32 << 32) | qb32;
#pragma unroll
                for (int b2 = 0; b2 < CT_TC / 2; ++b2) {
                    uint64_t d;
                    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(qq), "l"(cpair[b2]));
                    uint64_t& ac = acc2[a * (CT_TC / 2) + b2];
                    asm("fma.rn.f32x2 %0, %1, %1, %0;" : "+l"(ac) : "l"(d));
                }
            }
        }
#pragma unroll
        for (int a = 0; a < CT_TQ; ++a)
#pragma unroll
            for (int b = 0; b < CT_TC; ++b) t[a][b] = j == 0 ? acc[a][b] : __fadd_rn(t[a][b], acc[a][b]);
    }
    if (dim > full) {
        stage(full, 1, dim - full);
        for (int r = 0; r < dim - full; ++r) {
#pragma unroll
            for (int a = 0; a < CT_TQ; ++a)
#pragma unroll
                for (int b = 0; b < CT_TC; ++b) {
                    const float d = __fsub_rn(qb[r * CT_Q + a], cb[r * CT_C + b]);
                    t[a][b] = __fadd_rn(t[a][b], __fmul_rn(d, d));
                }
        }
    }
#pragma unroll
    for (int a = 0; a < CT_TQ; ++a) {
        const int q = q0 + tq * CT_TQ + a;
        if (q >= nq) continue;
        float* row = D + (size_t)q * nlist;
#pragma unroll
        for (int b = 0; b < CT_TC; ++b) {
            const int l = c0 + tc * CT_TC + b;
            if (l < nlist) row[l] = t[a][b];
        }
    }
}

void launch_transpose_pad(cudaStream_t s, const float* x, int n, int dim, int npad, float* out) {
    if (npad == 0 || dim == 0) return;
    dim3 grid((unsigned)((npad + 31) / 32), (unsigned)((dim + 31) / 32));
    transpose_pad_kernel<<<grid, dim3(32, 8), 0, s>>>(x, n, dim, npad, out);
    FDB_LAUNCH_CHECK();
}

void launch_coarse_tiled(cudaStream_t s, const float* QT, int nq, int nq_pad, int dim,
                         const float* CT, int nlist, int nlist_pad, float* D) {
    if (nq == 0) return;
    FDB_REQUIRE(dim <= CT_MAX_DIM && nq_pad % CT_Q == 0 && nlist_pad % CT_C == 0,
                FDB_ERR_UNSUPPORTED, "coarse tiling: bad shape");
    const int full = dim & ~7, rows = std::max(full / 8, dim - full);
    const size_t smem = (size_t)std::max(rows, 1) * (CT_Q + CT_C) * sizeof(float);
    if (smem > 48 * 1024)
        FDB_CUDA(cudaFuncSetAttribute(coarse_tiled_kernel,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    dim3 grid((unsigned)(nlist_pad / CT_C), (unsigned)(nq_pad / CT_Q));
    coarse_tiled_kernel<<<grid, CT_THREADS, smem, s>>>(QT, nq, nq_pad, dim, CT, nlist, nlist_pad,
                                                        D);
    FDB_LAUNCH_CHECK();
}

// ---------------------------------------------------------------------------
// probe selection
// ---------------------------------------------------------------------------
constexpr int SEL_WARPS = 8;

template <int P>
__global__ void __launch_bounds__(SEL_WARPS * 32)
    select_kernel(const float* __restrict__ D, int nq, int nlist, int take,
                  uint32_t* __restrict__ probes, float* __restrict__ pdist) {
    __shared__ uint64_t buf[SEL_WARPS * 64];
    __shared__ unsigned hist[SEL_WARPS * 256];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * SEL_WARPS + warp;
    if (q >= nq) return;  // whole warp leaves together
    WarpTopK<P> tk;
    tk.init(take, buf + warp * 64);
    const float* row = D + (size_t)q * nlist;
    // the row's keys, eight loads in flight per lane
    auto visit = [&](auto&& f) {
        for (int base = 0; base < nlist; base += 32 * 8) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int l = base + u * 32 + lane;
                v[u] = l < nlist ? row[l] : 0.0f;
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int l = base + u * 32 + lane;
                const bool valid = l < nlist;
                f(valid ? make_key(v[u], (uint32_t)l) : KEY_NONE, valid);
            }
        }
    };
    // only the bins that hold the take smallest keys are offered
    const KeyBins kb = warp_key_bins(visit, take, hist + warp * 256);
    visit([&](uint64_t key, bool valid) { tk.add(key, valid && kb.keep(key)); });
    tk.flush();
#pragma unroll
    for (int e = 0; e < P; ++e) {
        int i = e * 32 + lane;
        if (i < take) {
            probes[(size_t)q * take + i] = key_tag(tk.L[e]);
            if (pdist) pdist[(size_t)q * take + i] = key_dist(tk.L[e]);
        }
    }
}

// More than FDB_MAX_K probes: one block per query sorts all (distance, list)
// keys with a bitonic network in shared memory.
__global__ void select_sort_kernel(const float* __restrict__ D, int nq, int nlist, int npow2,
                                   int take, uint32_t* __restrict__ probes,
                                   float* __restrict__ pdist) {
    extern __shared__ uint64_t keys[];
    const int q = blockIdx.x;
    for (int i = threadIdx.x; i < npow2; i += blockDim.x)
        keys[i] = i < nlist ? make_key(D[(size_t)q * nlist + i], (uint32_t)i) : KEY_NONE;
    __syncthreads();
    for (int size = 2; size <= npow2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < npow2; i += blockDim.x) {
                int j = i ^ stride;
                if (j > i) {
                    bool up = (i & size) == 0;
                    uint64_t a = keys[i], b = keys[j];
                    if ((a > b) == up) { keys[i] = b; keys[j] = a; }
                }
            }
            __syncthreads();
        }
    }
    for (int i = threadIdx.x; i < take; i += blockDim.x) {
        probes[(size_t)q * take + i] = key_tag(keys[i]);
        if (pdist) pdist[(size_t)q * take + i] = key_dist(keys[i]);
    }
}

void launch_select(cudaStream_t s, const float* D, int nq, int nlist, int take,
                   uint32_t* probes, float* pdist) {
    if (nq == 0 || take == 0) return;
    unsigned grid = (nq + SEL_WARPS - 1) / SEL_WARPS;
    if (take <= 32) select_kernel<1><<<grid, SEL_WARPS * 32, 0, s>>>(D, nq, nlist, take, probes, pdist);
    else if (take <= 64) select_kernel<2><<<grid, SEL_WARPS * 32, 0, s>>>(D, nq, nlist, take, probes, pdist);
    else if (take <= 128) select_kernel<4><<<grid, SEL_WARPS * 32, 0, s>>>(D, nq, nlist, take, probes, pdist);
    else if (take <= 256) select_kernel<8><<<grid, SEL_WARPS * 32, 0, s>>>(D, nq, nlist, take, probes, pdist);
    else {
        int npow2 = 1;
        while (npow2 < nlist) npow2 <<= 1;
        size_t smem = (size_t)npow2 * sizeof(uint64_t);
        FDB_REQUIRE(smem <= 200 * 1024, FDB_ERR_UNSUPPORTED,
                    "more than 256 probes supported up to 16384 lists");
        if (smem > 48 * 1024)
            FDB_CUDA(cudaFuncSetAttribute(select_sort_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        select_sort_kernel<<<nq, 512, smem, s>>>(D, nq, nlist, npow2, take, probes, pdist);
    }
    FDB_LAUNCH_CHECK();
}

// ---------------------------------------------------------------------------
// LUT + scan
// ---------------------------------------------------------------------------
constexpr int SCAN_THREADS = 256;
constexpr int SCAN_WARPS = SCAN_THREADS / 32;

// One LUT entry: L2^2 of the residual sub-vector (shared memory) and a
// codeword (global, read through the read-only cache), AVX2 order.
__device__ __forceinline__ float lut_entry(const float* __restrict__ r,
                                           const float* __restrict__ cw, int sub) {
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
    int i = 0;
    if ((sub & 3) == 0) {
        for (; i + 8 <= sub; i += 8) {
            float4 u = __ldg(reinterpret_cast<const float4*>(cw + i));
            float4 v = __ldg(reinterpret_cast<const float4*>(cw + i + 4));
            float c[8] = {u.x, u.y, u.z, u.w, v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float d = __fsub_rn(r[i + j], c[j]);
                acc[j] = __fmaf_rn(d, d, acc[j]);
            }
        }
    } else {
        for (; i + 8 <= sub; i += 8) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float d = __fsub_rn(r[i + j], __ldg(cw + i + j));
                acc[j] = __fmaf_rn(d, d, acc[j]);
            }
        }
    }
    float t = lane_sum(acc);
    for (; i < sub; ++i) {
        float d = __fsub_rn(r[i], __ldg(cw + i));
        t = __fadd_rn(t, __fmul_rn(d, d));
    }
    return t;
}

// Code bytes: MB > 0 is the compile-time code length (a multiple of 8, read
// with 64/128-bit loads); MB == 0 reads m bytes one by one.
template <int ORDER, int MB>
__device__ __forceinline__ float adc_code(const float* __restrict__ lut,
                                          const uint8_t* __restrict__ code, int m) {
    if constexpr (MB > 0) {
        constexpr int NW = MB / 4;
        uint32_t w[NW];
        if constexpr (MB % 16 == 0) {
#pragma unroll
            for (int v = 0; v < MB / 16; ++v) {
                uint4 u = __ldg(reinterpret_cast<const uint4*>(code) + v);
                w[4 * v] = u.x; w[4 * v + 1] = u.y; w[4 * v + 2] = u.z; w[4 * v + 3] = u.w;
            }
        } else {
#pragma unroll
            for (int v = 0; v < MB / 8; ++v) {
                uint2 u = __ldg(reinterpret_cast<const uint2*>(code) + v);
                w[2 * v] = u.x; w[2 * v + 1] = u.y;
            }
        }
        auto lk = [&](int i) -> float {
            return lut[i * KSUB + ((w[i >> 2] >> ((i & 3) * 8)) & 0xffu)];
        };
        return adc_order<ORDER>(lk, MB);
    } else {
        auto lk = [&](int i) -> float { return lut[i * KSUB + __ldg(code + i)]; };
        return adc_order<ORDER>(lk, m);
    }
}

// Shared memory of one scan block:
//   lut   [m*256]  f32   the (query, list) table
//   ctab  [m*256]  f32   table mode only: <q_s, b_sj> for this block's query
//   resid [dim_pad] f32  exact mode: q - c_l
//   aterm [m_pad]  f32   table mode: ||q_s - c_ls||^2
//   wbuf  [warps*64] u64 WarpTopK candidate buffers
//   lists [warps*k]  u64 per-warp results for the end-of-query merge
//
// TABLES == false: every LUT entry is L2^2(q_s - c_ls, b_sj) in the AVX2
//   order -- the reference's value, bit for bit.
// TABLES == true: LUT entry = ||q_s - c_ls||^2 + (||b_sj||^2 + 2<c_ls,b_sj>)
//   - 2<q_s,b_sj>, the middle term precomputed per list at build time and the
//   last computed once per query: the same real number with different
//   rounding.  The block then keeps a shortlist of a.k >= 2k candidates that
//   rescore_kernel re-ranks with exact distances and certifies.
template <int P, int ORDER, int MB, bool TABLES>
__global__ void __launch_bounds__(SCAN_THREADS) scan_kernel(ScanParams a) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int m = MB > 0 ? MB : a.m;
    const int L = m * KSUB;
    const int dim_pad = (a.dim + 3) & ~3;
    const int m_pad = (m + 3) & ~3;
    float* lut = reinterpret_cast<float*>(smem);
    float* ctab = lut + L;
    float* resid = ctab + (TABLES ? L : 0);
    float* aterm = resid + dim_pad;
    uint64_t* wbuf = reinterpret_cast<uint64_t*>(aterm + m_pad);
    uint64_t* lists = wbuf + SCAN_WARPS * 64;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int sub = a.dim / m;
    int nq = a.nq;
    if (a.nq_dev) {
        const uint32_t total = *a.nq_dev;
        nq = total > a.nq_dev_base ? (int)min((uint32_t)a.nq, total - a.nq_dev_base) : 0;
    }
    for (int qi = blockIdx.x; qi < nq; qi += gridDim.x) {
        const int q = a.qidx ? (int)a.qidx[qi] : qi;
        const float* qv = a.Q + (size_t)q * a.dim;
        if (TABLES) {
            __syncthreads();  // the previous query's ctab is no longer read
            for (int e = threadIdx.x; e < L; e += SCAN_THREADS) {
                const float* qs = qv + (e >> 8) * sub;
                const float* b = a.cb + (size_t)e * sub;
                float t = 0.0f;
                for (int i = 0; i < sub; ++i) t = __fmaf_rn(__ldg(qs + i), __ldg(b + i), t);
                ctab[e] = t;
            }
        }
        WarpTopK<P> tk;
        tk.init(a.k, wbuf + warp * 64);
        unsigned long long nscan = 0, nl = 0;
        const uint32_t* pl = a.probe_list ? a.probe_list + (size_t)qi * a.nprobe
                                          : a.probes + (size_t)q * a.nprobe;
        const int npq = (a.probe_list && a.probe_cnt) ? (int)a.probe_cnt[qi] : a.nprobe;
        for (int p = 0; p < npq; ++p) {
            const uint32_t l = pl[p];
            const uint64_t beg = a.offs[l], end = a.ends[l];
            if (beg == end) continue;  // empty, or held by another device
            __syncthreads();           // previous list's LUT no longer in use
            const float* cl = a.cents + (size_t)l * a.dim;
            if (TABLES) {
                if (threadIdx.x < m) {
                    const int s = threadIdx.x;
                    float t = 0.0f;
                    for (int i = 0; i < sub; ++i) {
                        float d = __fsub_rn(__ldg(qv + s * sub + i), __ldg(cl + s * sub + i));
                        t = __fmaf_rn(d, d, t);
                    }
                    aterm[s] = t;
                }
                __syncthreads();
                const float4* B4 = reinterpret_cast<const float4*>(a.btab + (size_t)l * L);
                const float4* C4 = reinterpret_cast<const float4*>(ctab);
                float4* T4 = reinterpret_cast<float4*>(lut);
                for (int e4 = threadIdx.x; e4 < L / 4; e4 += SCAN_THREADS) {
                    const float A = aterm[e4 >> 6];
                    const float4 b = __ldg(B4 + e4);
                    const float4 c = C4[e4];
                    float4 r;
                    r.x = __fmaf_rn(-2.0f, c.x, __fadd_rn(A, b.x));
                    r.y = __fmaf_rn(-2.0f, c.y, __fadd_rn(A, b.y));
                    r.z = __fmaf_rn(-2.0f, c.z, __fadd_rn(A, b.z));
                    r.w = __fmaf_rn(-2.0f, c.w, __fadd_rn(A, b.w));
                    T4[e4] = r;
                }
            } else {
                for (int d = threadIdx.x; d < a.dim; d += SCAN_THREADS)
                    resid[d] = __fsub_rn(qv[d], cl[d]);  // q - c (ivf_pq.rs:926-938)
                __syncthreads();
                for (int e = threadIdx.x; e < L; e += SCAN_THREADS)
                    lut[e] = lut_entry(resid + (e >> 8) * sub, a.cb + (size_t)e * sub, sub);
            }
            __syncthreads();
            // Scan: each lane scores two codes per step; out-of-range lanes
            // read the list's first code (always present) and are masked.
            const uint32_t len = (uint32_t)(end - beg);
            const uint8_t* lc = a.codes + beg * (uint64_t)m;
            const uint32_t tag0 = (uint32_t)beg;
            for (uint32_t b = (uint32_t)warp * 64u; b < len; b += SCAN_WARPS * 64u) {
                const uint32_t i0 = b + lane, i1 = i0 + 32u;
                bool v0 = i0 < len, v1 = i1 < len;
                if (a.skip) {
                    const uint32_t r0 = tag0 + i0, r1 = tag0 + i1;
                    v0 = v0 && !((__ldg(a.skip + (r0 >> 5)) >> (r0 & 31)) & 1u);
                    v1 = v1 && !((__ldg(a.skip + (r1 >> 5)) >> (r1 & 31)) & 1u);
                }
                const float d0 = adc_code<ORDER, MB>(lut, lc + (size_t)(v0 ? i0 : 0u) * m, m);
                const float d1 = adc_code<ORDER, MB>(lut, lc + (size_t)(v1 ? i1 : 0u) * m, m);
                tk.add(make_key(d0, tag0 + i0), v0);
                tk.add(make_key(d1, tag0 + i1), v1);
            }
            nscan += len;
            ++nl;
        }
        tk.flush();
        tk.store(lists + warp * a.k);
        __syncthreads();
        if (warp == 0) {
            block_merge_warp0(tk, lists, SCAN_WARPS);
            uint64_t* orow = a.out_keys + (size_t)(a.out_by_block ? qi : q) * a.k;
            if (a.seed) tk.ingest(orow, a.k);
            tk.store(orow);
        }
        if (threadIdx.x == 0 && a.stat) {
            atomicAdd(&a.stat[0], nl);
            atomicAdd(&a.stat[1], nscan);
        }
        __syncthreads();
    }
}

template <int P, int ORDER, int MB, bool TABLES>
static void launch_scan_t(cudaStream_t s, const ScanParams& a, int grid) {
    const int m = a.m;
    size_t smem = (size_t)m * KSUB * sizeof(float) * (TABLES ? 2 : 1) +
                  (size_t)((a.dim + 3) & ~3) * sizeof(float) +
                  (size_t)((m + 3) & ~3) * sizeof(float) +
                  (size_t)SCAN_WARPS * 64 * sizeof(uint64_t) +
                  (size_t)SCAN_WARPS * a.k * sizeof(uint64_t);
    FDB_REQUIRE(smem <= 227 * 1024, FDB_ERR_UNSUPPORTED, "LUT does not fit in shared memory");
    auto kern = scan_kernel<P, ORDER, MB, TABLES>;
    if (smem > 48 * 1024)
        FDB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem));
    kern<<<grid, SCAN_THREADS, smem, s>>>(a);
    FDB_LAUNCH_CHECK();
}

template <int P, int ORDER, bool TABLES>
static void launch_scan_m(cudaStream_t s, const ScanParams& a, int grid) {
    switch (a.m) {
        case 8: launch_scan_t<P, ORDER, 8, TABLES>(s, a, grid); break;
        case 16: launch_scan_t<P, ORDER, 16, TABLES>(s, a, grid); break;
        case 32: launch_scan_t<P, ORDER, 32, TABLES>(s, a, grid); break;
        case 48: launch_scan_t<P, ORDER, 48, TABLES>(s, a, grid); break;
        default: launch_scan_t<P, ORDER, 0, TABLES>(s, a, grid); break;
    }
}

template <int ORDER, bool TABLES>
static void launch_scan_o(cudaStream_t s, const ScanParams& a, int grid) {
    if (a.k <= 32) launch_scan_m<1, ORDER, TABLES>(s, a, grid);
    else if (a.k <= 64) launch_scan_m<2, ORDER, TABLES>(s, a, grid);
    else if (a.k <= 128) launch_scan_m<4, ORDER, TABLES>(s, a, grid);
    else launch_scan_m<8, ORDER, TABLES>(s, a, grid);
}

void launch_scan(cudaStream_t s, const ScanParams& a, int order) {
    if (a.nq == 0) return;
    FDB_REQUIRE(a.k >= 1 && a.k <= FDB_MAX_K, FDB_ERR_UNSUPPORTED, "k out of range");
    const bool tables = a.btab != nullptr;
    const int grid = a.grid_cap > 0 ? std::min(a.nq, a.grid_cap) : a.nq;
    if (order == ORDER_LANE8) {
        if (tables) launch_scan_o<ORDER_LANE8, true>(s, a, grid);
        else launch_scan_o<ORDER_LANE8, false>(s, a, grid);
    } else {
        if (tables) launch_scan_o<ORDER_FAST4, true>(s, a, grid);
        else launch_scan_o<ORDER_FAST4, false>(s, a, grid);
    }
}

// ---------------------------------------------------------------------------
// exact rescoring and certification of a table-mode shortlist
// ---------------------------------------------------------------------------
constexpr int RESCORE_WARPS = 8;

// One warp per query.  The shortlist (a.kp approximate keys, ascending) is
// rescored exactly and the k best exact keys are kept.  Certification: every
// approximate distance is within E of the exact one (E is a worst-case bound
// of the rounding of both computations), so if (exact k-th distance) + E is
// below the approximate distance of the last shortlisted candidate, no code
// outside the shortlist can belong to the exact top-k.  Queries that fail the
// test are listed for an exact re-scan.
template <int P, int ORDER>
__global__ void __launch_bounds__(RESCORE_WARPS * 32) rescore_kernel(RescoreParams r) {
    __shared__ uint64_t buf[RESCORE_WARPS * 64];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * RESCORE_WARPS + warp;
    if (q >= r.nq) return;  // whole warp
    const int m = r.m, sub = r.dim / m;
    const float* qv = r.Q + (size_t)q * r.dim;
    const uint64_t* ak = r.approx + (size_t)q * r.kp;
    WarpTopK<P> tk;
    tk.init(r.k, buf + warp * 64);
    for (int base = 0; base < r.kp; base += 32) {
        const int i = base + lane;
        const uint64_t key = i < r.kp ? ak[i] : KEY_NONE;
        uint64_t ek = KEY_NONE;
        if (key != KEY_NONE) {
            const uint32_t pos = key_tag(key);
            int lo = 0, hi = r.nlist;  // the list l with offs[l] <= pos < offs[l+1]
            while (lo < hi) {
                int mid = (lo + hi) >> 1;
                if (r.offs_full[mid + 1] <= pos) lo = mid + 1; else hi = mid;
            }
            const float d = exact_adc<ORDER>(qv, r.cents + (size_t)lo * r.dim, r.cb,
                                             r.codes + (size_t)pos * m, m, sub);
            ek = make_key(d, pos);
        }
        if (__any_sync(0xffffffffu, ek != KEY_NONE)) tk.merge32(ek);
    }
    tk.store(r.out_keys + (size_t)q * r.k);
    // error bound: E = (32 + 4m) u sum_s (|q_s| + cmax_s + bmax_s)^2, u = 2^-24
    double part = 0.0;
    for (int s = lane; s < m; s += 32) {
        double qn = 0.0;
        for (int i = 0; i < sub; ++i) {
            double x = qv[s * sub + i];
            qn += x * x;
        }
        double t = sqrt(qn) + (double)r.cmax[s] + (double)r.bmax[s];
        part += t * t;
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    const double E = (32.0 + 4.0 * m) * 5.9604644775390625e-8 * part * 1.01;
    const uint64_t last = ak[r.kp - 1];
    bool cert = true;
    if (last != KEY_NONE) {
        // the shortlist is full; tk.thr is the exact k-th key
        const double dk = (double)key_dist(tk.thr);
        const double tau = (double)key_dist(last);
        cert = (tk.thr != KEY_NONE) && (dk + E < tau);
    }
    if (!cert && lane == 0) {
        const uint32_t idx = atomicAdd(r.flag_count, 1u);
        r.flag_list[idx] = (uint32_t)q;
    }
}

void launch_rescore(cudaStream_t s, const RescoreParams& r, int order) {
    if (r.nq == 0) return;
    unsigned grid = (unsigned)((r.nq + RESCORE_WARPS - 1) / RESCORE_WARPS);
    const int T = RESCORE_WARPS * 32;
#define FDB_RESCORE(PP)                                                                    \
    do {                                                                                   \
        if (order == ORDER_LANE8) rescore_kernel<PP, ORDER_LANE8><<<grid, T, 0, s>>>(r);   \
        else rescore_kernel<PP, ORDER_FAST4><<<grid, T, 0, s>>>(r);                        \
    } while (0)
    if (r.k <= 32) FDB_RESCORE(1);
    else if (r.k <= 64) FDB_RESCORE(2);
    else FDB_RESCORE(4);
#undef FDB_RESCORE
    FDB_LAUNCH_CHECK();
}

// Per-list table of the table mode: btab[l][s][j] = ||b_sj||^2 + 2<c_ls, b_sj>.
__global__ void ivf_tables_kernel(const float* __restrict__ cents, const float* __restrict__ cb,
                                  int nlist, int m, int dim, float* __restrict__ btab) {
    const size_t L = (size_t)m * KSUB;
    const size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= (size_t)nlist * L) return;
    const size_t l = t / L;
    const int e = (int)(t - l * L);
    const int sub = dim / m;
    const int s = e >> 8;
    const float* b = cb + (size_t)e * sub;
    const float* c = cents + l * dim + (size_t)s * sub;
    float v = 0.0f;
    for (int i = 0; i < sub; ++i) v = __fmaf_rn(b[i], __fmaf_rn(2.0f, c[i], b[i]), v);
    btab[t] = v;
}

void launch_ivf_tables(cudaStream_t s, const float* cents, const float* cb, int nlist, int m,
                       int dim, float* btab) {
    size_t total = (size_t)nlist * m * KSUB;
    if (total == 0) return;
    ivf_tables_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(cents, cb, nlist, m, dim,
                                                                      btab);
    FDB_LAUNCH_CHECK();
}

// ---------------------------------------------------------------------------
// merging sorted top-k lists
// ---------------------------------------------------------------------------
constexpr int MERGE_WARPS = 8;

template <int P>
__global__ void __launch_bounds__(MERGE_WARPS * 32)
    merge_lists_kernel(const uint64_t* __restrict__ lists, int nlists, size_t list_stride,
                       size_t nq, int k, uint64_t* __restrict__ out) {
    __shared__ uint64_t buf[MERGE_WARPS * 64];
    const int warp = threadIdx.x >> 5;
    const size_t q = (size_t)blockIdx.x * MERGE_WARPS + warp;
    if (q >= nq) return;
    WarpTopK<P> tk;
    tk.init(k, buf + warp * 64);
    for (int r = 0; r < nlists; ++r) tk.ingest(lists + (size_t)r * list_stride + q * k, k);
    tk.store(out + q * k);
}

void launch_merge_lists(cudaStream_t s, const uint64_t* lists, int nlists, size_t list_stride,
                        size_t nq, int k, uint64_t* out) {
    if (nq == 0) return;
    unsigned grid = (unsigned)((nq + MERGE_WARPS - 1) / MERGE_WARPS);
    if (k <= 32) merge_lists_kernel<1><<<grid, MERGE_WARPS * 32, 0, s>>>(lists, nlists, list_stride, nq, k, out);
    else if (k <= 64) merge_lists_kernel<2><<<grid, MERGE_WARPS * 32, 0, s>>>(lists, nlists, list_stride, nq, k, out);
    else if (k <= 128) merge_lists_kernel<4><<<grid, MERGE_WARPS * 32, 0, s>>>(lists, nlists, list_stride, nq, k, out);
    else merge_lists_kernel<8><<<grid, MERGE_WARPS * 32, 0, s>>>(lists, nlists, list_stride, nq, k, out);
    FDB_LAUNCH_CHECK();
}

// After a cross-device merge: find each winning key in the gathered lists
// (each sorted ascending) and take the id stored beside it.
__global__ void lookup_gathered_ids(const uint64_t* __restrict__ keys,
                                    const uint64_t* __restrict__ gkeys,
                                    const uint64_t* __restrict__ gids, int world,
                                    size_t list_stride, size_t nq, int k,
                                    uint64_t* __restrict__ ids) {
    const size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= nq * k) return;
    const size_t q = t / k;
    const uint64_t key = keys[t];
    uint64_t id = ~0ull;
    if (key != KEY_NONE) {
        for (int r = 0; r < world; ++r) {
            const uint64_t* L = gkeys + (size_t)r * list_stride + q * k;
            int lo = 0, hi = k;
            while (lo < hi) {
                int mid = (lo + hi) >> 1;
                if (L[mid] < key) lo = mid + 1; else hi = mid;
            }
            if (lo < k && L[lo] == key) {
                id = gids[(size_t)r * list_stride + q * k + lo];
                break;
            }
        }
    }
    ids[t] = id;
}

void launch_lookup_gathered(cudaStream_t s, const uint64_t* keys, const uint64_t* gkeys,
                            const uint64_t* gids, int world, size_t list_stride, size_t nq, int k,
                            uint64_t* ids) {
    size_t total = nq * (size_t)k;
    if (total == 0) return;
    lookup_gathered_ids<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(keys, gkeys, gids, world,
                                                                        list_stride, nq, k, ids);
    FDB_LAUNCH_CHECK();
}

// keys -> ids through a row-id table (tag - tag_base indexes row_ids).
__global__ void keys_to_ids_kernel(const uint64_t* __restrict__ keys, size_t total,
                                   const uint64_t* __restrict__ row_ids, uint64_t tag_base,
                                   uint64_t* __restrict__ ids) {
    const size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= total) return;
    const uint64_t key = keys[t];
    ids[t] = key == KEY_NONE ? ~0ull : row_ids[(uint64_t)key_tag(key) - tag_base];
}

void launch_keys_to_ids(cudaStream_t s, const uint64_t* keys, size_t total,
                        const uint64_t* row_ids, uint64_t tag_base, uint64_t* ids) {
    if (total == 0) return;
    keys_to_ids_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(keys, total, row_ids,
                                                                       tag_base, ids);
    FDB_LAUNCH_CHECK();
}

// keys (+ ids) -> caller's ids / distances / counts, UINT64_MAX / +inf padding.
__global__ void finalize_kernel(const uint64_t* __restrict__ keys,
                                const uint64_t* __restrict__ ids_in, size_t nq, int k,
                                uint64_t* __restrict__ ids, float* __restrict__ dists,
                                uint32_t* __restrict__ counts) {
    const size_t q = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= nq) return;
    uint32_t cnt = 0;
    for (int i = 0; i < k; ++i) {
        const uint64_t key = keys[q * k + i];
        const bool ok = key != KEY_NONE;
        ids[q * k + i] = ok ? ids_in[q * k + i] : ~0ull;
        dists[q * k + i] = ok ? key_dist(key) : __int_as_float(0x7f800000);
        cnt += ok;
    }
    if (counts) counts[q] = cnt;
}

void launch_finalize(cudaStream_t s, const uint64_t* keys, const uint64_t* ids_in, size_t nq,
                     int k, uint64_t* ids, float* dists, uint32_t* counts) {
    if (nq == 0) return;
    finalize_kernel<<<(unsigned)((nq + 127) / 128), 128, 0, s>>>(keys, ids_in, nq, k, ids, dists,
                                                                 counts);
    FDB_LAUNCH_CHECK();
}

}  // namespace fdb
