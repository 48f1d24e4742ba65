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

// ---------------------------------------------------------------------------
// probe selection
// ---------------------------------------------------------------------------
constexpr int SEL_WARPS = 8;

template <int P>
__global__ void __launch_bounds__(SEL_WARPS * 32)
    select_kernel(const float* __restrict__ D, int nq, int nlist, int take,
                  uint32_t* __restrict__ probes) {
    __shared__ uint64_t buf[SEL_WARPS * 64];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * SEL_WARPS + warp;
    if (q >= nq) return;  // whole warp leaves together
    WarpTopK<P> tk;
    tk.init(take, buf + warp * 64);
    const float* row = D + (size_t)q * nlist;
    for (int base = 0; base < nlist; base += 32) {
        int l = base + lane;
        bool valid = l < nlist;
        uint64_t key = valid ? make_key(row[l], (uint32_t)l) : KEY_NONE;
        tk.add(key, valid);
    }
    tk.flush();
#pragma unroll
    for (int e = 0; e < P; ++e) {
        int i = e * 32 + lane;
        if (i < take) probes[(size_t)q * take + i] = key_tag(tk.L[e]);
    }
}

// More than FDB_MAX_K probes: one block per query sorts all (distance, list)
// keys with a bitonic network in shared memory.
__global__ void select_sort_kernel(const float* __restrict__ D, int nq, int nlist, int npow2,
                                   int take, uint32_t* __restrict__ probes) {
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
    for (int i = threadIdx.x; i < take; i += blockDim.x)
        probes[(size_t)q * take + i] = key_tag(keys[i]);
}

void launch_select(cudaStream_t s, const float* D, int nq, int nlist, int take,
                   uint32_t* probes) {
    if (nq == 0 || take == 0) return;
    unsigned grid = (nq + SEL_WARPS - 1) / SEL_WARPS;
    if (take <= 32) select_kernel<1><<<grid, SEL_WARPS * 32, 0, s>>>(D, nq, nlist, take, probes);
    else if (take <= 64) select_kernel<2><<<grid, SEL_WARPS * 32, 0, s>>>(D, nq, nlist, take, probes);
    else if (take <= 128) select_kernel<4><<<grid, SEL_WARPS * 32, 0, s>>>(D, nq, nlist, take, probes);
    else if (take <= 256) select_kernel<8><<<grid, SEL_WARPS * 32, 0, s>>>(D, nq, nlist, take, probes);
    else {
        int npow2 = 1;
        while (npow2 < nlist) npow2 <<= 1;
        size_t smem = (size_t)npow2 * sizeof(uint64_t);
        FDB_REQUIRE(smem <= 200 * 1024, FDB_ERR_UNSUPPORTED,
                    "nprobe > 256 supported up to 25600 lists");
        if (smem > 48 * 1024)
            FDB_CUDA(cudaFuncSetAttribute(select_sort_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        select_sort_kernel<<<nq, 512, smem, s>>>(D, nq, nlist, npow2, take, probes);
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

// ADC of one code in the requested order; `lk(i)` returns LUT[i][code[i]].
template <int ORDER, class F>
__device__ __forceinline__ float adc_order(F lk, int m) {
    if (ORDER == ORDER_LANE8) {
        const int full = m & ~7;
        float total = 0.0f;
        if (full > 0) {
            float acc[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] = lk(j);
            for (int i = 8; i < full; i += 8) {
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[j] = __fadd_rn(acc[j], lk(i + j));
            }
            total = lane_sum(acc);
        }
        for (int i = full; i < m; ++i) total = __fadd_rn(total, lk(i));
        return total;
    } else {
        float sum = 0.0f;
        int i = 0;
        for (; i + 4 <= m; i += 4) {
            float g = __fadd_rn(__fadd_rn(__fadd_rn(lk(i), lk(i + 1)), lk(i + 2)), lk(i + 3));
            sum = __fadd_rn(sum, g);
        }
        for (; i < m; ++i) sum = __fadd_rn(sum, lk(i));
        return sum;
    }
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

template <int P, int ORDER, int MB>
__global__ void __launch_bounds__(SCAN_THREADS) scan_kernel(ScanParams a) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int m = MB > 0 ? MB : a.m;
    float* lut = reinterpret_cast<float*>(smem);
    float* resid = lut + m * KSUB;
    const int dim_pad = (a.dim + 3) & ~3;
    uint64_t* wbuf = reinterpret_cast<uint64_t*>(resid + dim_pad);
    uint64_t* lists = wbuf + SCAN_WARPS * 64;
    const int warp = threadIdx.x >> 5;
    const int sub = a.dim / m;
    for (int q = blockIdx.x; q < a.nq; q += gridDim.x) {
        WarpTopK<P> tk;
        tk.init(a.k, wbuf + warp * 64);
        const float* qv = a.Q + (size_t)q * a.dim;
        unsigned long long nscan = 0, nl = 0;
        for (int p = 0; p < a.nprobe; ++p) {
            const uint32_t l = a.probes[(size_t)q * a.nprobe + p];
            const uint64_t beg = a.offs[l], end = a.ends[l];
            if (beg == end) continue;  // empty, or held by another device
            __syncthreads();           // previous list's LUT no longer in use
            const float* cl = a.cents + (size_t)l * a.dim;
            for (int d = threadIdx.x; d < a.dim; d += SCAN_THREADS)
                resid[d] = __fsub_rn(qv[d], cl[d]);  // q - c (ivf_pq.rs:926-938)
            __syncthreads();
            for (int e = threadIdx.x; e < m * KSUB; e += SCAN_THREADS) {
                const int s = e >> 8;
                lut[e] = lut_entry(resid + s * sub, a.cb + (size_t)e * sub, sub);
            }
            __syncthreads();
            for (uint64_t base = beg + (uint64_t)warp * 32; base < end;
                 base += (uint64_t)SCAN_WARPS * 32) {
                const uint64_t pos = base + (threadIdx.x & 31);
                const bool valid = pos < end;
                float dist = 0.0f;
                if (valid) dist = adc_code<ORDER, MB>(lut, a.codes + pos * m, m);
                tk.add(make_key(dist, (uint32_t)pos), valid);
            }
            nscan += end - beg;
            ++nl;
        }
        tk.flush();
        tk.store(lists + warp * a.k);
        __syncthreads();
        if (warp == 0) {
            block_merge_warp0(tk, lists, SCAN_WARPS);
            tk.store(a.out_keys + (size_t)q * a.k);
        }
        if (threadIdx.x == 0 && a.stat) {
            atomicAdd(&a.stat[0], nl);
            atomicAdd(&a.stat[1], nscan);
        }
        __syncthreads();
    }
}

template <int P, int ORDER, int MB>
static void launch_scan_t(cudaStream_t s, const ScanParams& a, int grid) {
    const int m = a.m;
    size_t smem = (size_t)m * KSUB * sizeof(float) + (size_t)((a.dim + 3) & ~3) * sizeof(float) +
                  (size_t)SCAN_WARPS * 64 * sizeof(uint64_t) +
                  (size_t)SCAN_WARPS * a.k * sizeof(uint64_t);
    FDB_REQUIRE(smem <= 227 * 1024, FDB_ERR_UNSUPPORTED, "LUT does not fit in shared memory");
    auto kern = scan_kernel<P, ORDER, MB>;
    if (smem > 48 * 1024)
        FDB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem));
    kern<<<grid, SCAN_THREADS, smem, s>>>(a);
    FDB_LAUNCH_CHECK();
}

template <int P, int ORDER>
static void launch_scan_m(cudaStream_t s, const ScanParams& a, int grid) {
    switch (a.m) {
        case 8: launch_scan_t<P, ORDER, 8>(s, a, grid); break;
        case 16: launch_scan_t<P, ORDER, 16>(s, a, grid); break;
        case 32: launch_scan_t<P, ORDER, 32>(s, a, grid); break;
        case 48: launch_scan_t<P, ORDER, 48>(s, a, grid); break;
        default: launch_scan_t<P, ORDER, 0>(s, a, grid); break;
    }
}

template <int ORDER>
static void launch_scan_o(cudaStream_t s, const ScanParams& a, int grid) {
    if (a.k <= 32) launch_scan_m<1, ORDER>(s, a, grid);
    else if (a.k <= 64) launch_scan_m<2, ORDER>(s, a, grid);
    else if (a.k <= 128) launch_scan_m<4, ORDER>(s, a, grid);
    else launch_scan_m<8, ORDER>(s, a, grid);
}

void launch_scan(cudaStream_t s, const ScanParams& a, int order) {
    if (a.nq == 0) return;
    FDB_REQUIRE(a.k >= 1 && a.k <= FDB_MAX_K, FDB_ERR_UNSUPPORTED, "k out of range");
    const int grid = a.nq;
    if (order == ORDER_LANE8) launch_scan_o<ORDER_LANE8>(s, a, grid);
    else launch_scan_o<ORDER_FAST4>(s, a, grid);
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
