// coarse_tc.cu -- the coarse quantizer on the tensor cores.
//
// find_nearest_partitions (src/index/ivf_pq.rs:538-553) and its inline copy
// in batch_search (:865-888) pick, per query, the nprobe centroids of
// smallest L2^2 in the AVX2 order of euclidean_distance_squared
// (src/distance/simd.rs:338-366).  Here that is three steps:
//
//   coarse_prep_kernel   : a warp per query -- the query scaled by a power of
//                          two (largest |q_i| in [2^14, 2^15)) and rounded to
//                          fp16, its squared norm, the factor -2 2^-(sa+sb)
//                          that undoes both scalings, and the error bound E_q
//                          of the approximate distances below.
//   coarse_gemm_kernel   : S = Q C^T with tcgen05.mma (fp16 operands staged by
//                          TMA, fp32 accumulators in TMEM); the epilogue writes
//                          d~ = ||q||^2 + ||c||^2 - 2 2^-(sa+sb) s for every
//                          (query, centroid).
//   coarse_refine_kernel : a warp per query -- a value t with at least `take`
//                          entries d~ <= t (binned threshold), then every
//                          centroid with d~ <= t + 2 E_q is rescored with the
//                          reference's exact arithmetic and the take smallest
//                          (distance, list) keys are kept, in order.
//
// Why this selects exactly the reference's probes: |d~ - d| <= E_q for every
// centroid, d the exact (AVX2-order) distance.  The `take` entries with
// d~ <= t have d <= t + E_q, so the take-th smallest exact distance D_k is at
// most t + E_q, and every centroid of the exact top-take has
// d~ <= d + E_q <= D_k + E_q <= t + 2 E_q: it is among the rescored ones.
// The bound: the fp16 roundings of both operands (2^-11 relative each, both
// scaled to the normal range) and the tensor core's fp32 accumulation
// (allowance 2^-13) give C1 ||q|| cmax with C1 = 2 (2^-10 + 2^-13) 1.05;
// the fp32 roundings of the norms and the final fma C2 (||q||^2 + cmax^2),
// C2 = 2^-16; the rounding of the exact distance itself (dim / 8 + 16
// roundings of 2^-24 relative each) C3 (||q|| + cmax)^2.  A query whose
// bound is not finite rescores every centroid.
#include "fdb_device.cuh"
#include "fdb_internal.h"
#include "fdb_kernels.h"
#include "tc_ptx.cuh"

namespace fdb {
namespace ctc {

using namespace tc;

constexpr int THREADS = 384;      // warp 0 TMA, warp 1 MMA, warps 4..11 epilogue
constexpr int EPI_WARP0 = 4;
constexpr int NEPI = 8;           // epilogue warps: 4 TMEM lane quadrants x 2 column halves
constexpr int MAX_TPC = 8;        // centroid tiles (128 each) per block at most
constexpr int REF_WARPS = 8;      // refine: queries per block
constexpr int MAX_DPAD = 256;
constexpr int CAND_CAP = 128;     // refine: candidates rescored from the compact list
constexpr int REG_NLIST = 2048;   // refine: rows held in registers (64 per lane) at most
constexpr int BIG_THREADS = 256;  // refine of longer rows: one block per query
constexpr int BIG_CAND = 1024;    // its compact candidate list
constexpr int MAX_NLIST = 1 << 16;  // the tensor coarse path's largest nlist

struct GemmParams {
    int nq;
    int ntile;          // centroid tiles (nlist_pad / 128)
    int tpc;            // tiles per block (<= MAX_TPC)
    int katoms;         // dpad / 64
    int ldd;            // row stride of D (nlist_pad)
    const float* qn;    // [nq] ||q||^2
    const float* qs2;   // [nq] -2 2^-(sa+sb)
    const float* cn;    // [nlist_pad] ||c||^2 (0 in padding)
    float* D;           // [nq][ldd] approximate distances
    uint32_t* rmin;     // [nq] smallest d~ of each row (orderable bits), preset ~0
    uint32_t* rmax;     // [nq] largest d~ of each row (orderable bits), preset 0
    int* err;
    unsigned long long wait;
};

__global__ void coarse_prep_kernel(const float* __restrict__ Q, int nq, int dim, int dpad,
                                   int sb, float cmax, __half* __restrict__ A,
                                   float* __restrict__ qn, float* __restrict__ qs2,
                                   float* __restrict__ qerr, uint32_t* __restrict__ rmin,
                                   uint32_t* __restrict__ rmax) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (warp >= nq) return;
    const float* q = Q + (size_t)warp * dim;
    float m = 0.0f, ss = 0.0f;
    for (int i = lane; i < dim; i += 32) {
        const float v = q[i];
        m = fmaxf(m, fabsf(v));
        ss = __fmaf_rn(v, v, ss);
    }
    // non-negative floats order like their bit patterns
    m = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(m)));
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    int ex = 0;
    if (m > 0.0f && isfinite(m)) frexpf(m, &ex);  // m in [2^(ex-1), 2^ex)
    const int sa = (m > 0.0f && isfinite(m)) ? 15 - ex : 0;
    __half* arow = A + (size_t)warp * dpad;
    for (int i = lane; i < dpad; i += 32)
        arow[i] = __float2half_rn(i < dim ? ldexpf(q[i], sa) : 0.0f);
    if (lane == 0) {
        const float nrm = sqrtf(ss) * 1.0001f;
        const float C1 = 2.0f * (ldexpf(1.0f, -10) + ldexpf(1.0f, -13)) * 1.05f;
        const float C2 = ldexpf(1.0f, -16);
        const float C3 = ((float)(dim / 8) + 16.0f) * ldexpf(1.0f, -24) * 1.05f;
        const float e = C1 * nrm * cmax + C2 * (ss + cmax * cmax) +
                        C3 * (nrm + cmax) * (nrm + cmax);
        // scalings that leave the normal fp32 range make the estimate unsafe
        const bool ok = isfinite(e) && isfinite(ss) && abs(sa + sb) < 100;
        qn[warp] = ss;
        qs2[warp] = -ldexpf(2.0f, -(sa + sb));
        rmin[warp] = 0xffffffffu;
        rmax[warp] = 0u;
        qerr[warp] = ok ? e * 1.01f : __int_as_float(0x7f800000);
    }
}

// One block: 128 queries x tpc centroid tiles.  Warp 0 loads the query tile
// once and each centroid tile in turn (one B stage) by TMA; warp 1 issues the
// MMAs into two TMEM accumulators; warps 4..11 (a TMEM lane quadrant and a
// column half each) turn scores into d~ and store them through a swizzled
// 32 x 32 staging tile, so every global store writes whole 128-byte lines.
// Each epilogue thread also folds its row's d~ into the row's minimum and
// maximum (orderable bits; atomics once per thread at the end).
__global__ void __launch_bounds__(THREADS, 2)
    coarse_gemm_kernel(const __grid_constant__ CUtensorMap qmap,
                       const __grid_constant__ CUtensorMap cmap, GemmParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t base = smem_u32(smem_raw);
    unsigned char* smem = smem_raw + ((1024 - (base & 1023)) & 1023);  // 1024-byte aligned
    const int KA = p.katoms;
    const uint32_t stage_bytes = (uint32_t)(KA * ATOM_BYTES);
    unsigned char* a_tile = smem;                      // KA atoms
    unsigned char* b_tile = a_tile + KA * ATOM_BYTES;  // KA atoms
    float* cn_s = reinterpret_cast<float*>(b_tile + KA * ATOM_BYTES);  // [MAX_TPC * 128]
    float* stage = cn_s + MAX_TPC * TILE_N;                             // [NEPI][32][32]
    uint64_t* bars = reinterpret_cast<uint64_t*>(stage + NEPI * 32 * 32);
    uint64_t* a_full = bars;       // [1]
    uint64_t* b_full = bars + 1;   // [1]
    uint64_t* b_empty = bars + 2;  // [1]
    uint64_t* t_full = bars + 3;   // [2]
    uint64_t* t_empty = bars + 5;  // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 7);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qb = blockIdx.x;
    const int t0 = blockIdx.y * p.tpc;
    const int count = min(p.tpc, p.ntile - t0);
    // the squared norms of this block's centroids, read by the epilogue
    for (int i = threadIdx.x; i < count * TILE_N; i += THREADS) cn_s[i] = p.cn[t0 * TILE_N + i];

    if (threadIdx.x == 0) {
        mbar_init(a_full, 1);
        mbar_init(b_full, 1);
        mbar_init(b_empty, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(t_full + i, 1);
            mbar_init(t_empty + i, NEPI);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(2 * TILE_N));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    int last_load = -1;  // producer: last tile whose B load was issued
    bool a_issued = false;
    int last_i = -1;  // MMA issuer: last tile committed

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0 && count > 0) {
            mbar_expect_tx(a_full, stage_bytes);
            for (int a = 0; a < KA; ++a)
                tma_load_2d(a_tile + a * ATOM_BYTES, &qmap, a_full, a * KATOM, qb * TILE_M);
            a_issued = true;
            for (int i = 0; i < count; ++i) {
                if (i >= 1 && !mbar_wait(b_empty, (i - 1) & 1, p.err, p.wait)) break;
                mbar_expect_tx(b_full, stage_bytes);
                for (int a = 0; a < KA; ++a)
                    tma_load_2d(b_tile + a * ATOM_BYTES, &cmap, b_full, a * KATOM,
                                (t0 + i) * TILE_N);
                last_load = i;
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0 && count > 0) {
            bool ok = mbar_wait(a_full, 0, p.err, p.wait);
            for (int i = 0; ok && i < count; ++i) {
                const int acc = i & 1, ause = i >> 1;
                if (i >= 2 && !mbar_wait(t_empty + acc, (ause - 1) & 1, p.err, p.wait)) break;
                if (!mbar_wait(b_full, i & 1, p.err, p.wait)) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(acc * TILE_N);
                const uint32_t abase = smem_u32(a_tile);
                const uint32_t bbase = smem_u32(b_tile);
                for (int a = 0; a < KA; ++a) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {  // 4 x K16 per 64-wide atom
                        const uint32_t off = (uint32_t)(a * ATOM_BYTES + kk * 32);
                        umma_f16(d, smem_desc_sw128(abase + off), smem_desc_sw128(bbase + off),
                                 (a | kk) != 0);
                    }
                }
                umma_commit(b_empty);       // the B tile may be refilled once these finish
                umma_commit(t_full + acc);  // accumulator acc is ready for the epilogue
                last_i = i;
            }
        }
    } else if (warp >= EPI_WARP0 && warp < EPI_WARP0 + NEPI) {
        // ---------------- epilogue: one query row, half a tile per thread ----------------
        const int w = warp - EPI_WARP0;
        const int quad = w & 3;  // TMEM lane quadrant = warp % 4
        const int half = w >> 2;
        const int e = quad * 32 + lane;
        const int q = qb * TILE_M + e;
        const bool qok = q < p.nq;
        const float qn = qok ? p.qn[q] : 0.0f;
        const float s2 = qok ? p.qs2[q] : 0.0f;
        const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
        float* st = stage + w * 32 * 32;  // this warp's [32 rows][32 floats], 16-byte swizzle
        const int q0 = qb * TILE_M + quad * 32;  // row of the warp's lane 0
        uint32_t rmin = 0xffffffffu, rmax = 0u;
        for (int i = 0; i < count; ++i) {
            const int acc = i & 1;
            int got = 0;
            if (lane == 0) got = mbar_wait(t_full + acc, (i >> 1) & 1, p.err, p.wait) ? 1 : 0;
            got = __shfl_sync(0xffffffffu, got, 0);
            if (!got) break;
            tc_fence_after();
#pragma unroll 1
            for (int ch = 0; ch < 2; ++ch) {
                uint32_t v[32];
                tmem_ld32(tmem + lane_base + (uint32_t)(acc * TILE_N + half * 64 + ch * 32), v);
                const int cl = i * TILE_N + half * 64 + ch * 32;  // column within the block
                const float4* c4 = reinterpret_cast<const float4*>(cn_s + cl);
                float4* srow = reinterpret_cast<float4*>(st + lane * 32);
#pragma unroll
                for (int g = 0; g < 8; ++g) {
                    const float4 cc = c4[g];
                    float4 o;
                    o.x = __fmaf_rn(s2, __uint_as_float(v[4 * g]), qn + cc.x);
                    o.y = __fmaf_rn(s2, __uint_as_float(v[4 * g + 1]), qn + cc.y);
                    o.z = __fmaf_rn(s2, __uint_as_float(v[4 * g + 2]), qn + cc.z);
                    o.w = __fmaf_rn(s2, __uint_as_float(v[4 * g + 3]), qn + cc.w);
                    rmin = min(rmin, min(min(f2ord(o.x), f2ord(o.y)), min(f2ord(o.z), f2ord(o.w))));
                    rmax = max(rmax, max(max(f2ord(o.x), f2ord(o.y)), max(f2ord(o.z), f2ord(o.w))));
                    srow[g ^ (lane & 7)] = o;
                }
                __syncwarp();
                // lanes 8j..8j+7 store row 4r+j: 128 contiguous bytes per row
                const int col = t0 * TILE_N + cl + 4 * (lane & 7);
#pragma unroll
                for (int r = 0; r < 8; ++r) {
                    const int rr = 4 * r + (lane >> 3);
                    const float4 o = reinterpret_cast<const float4*>(st + rr * 32)[(lane & 7) ^
                                                                                  (rr & 7)];
                    if (q0 + rr < p.nq)
                        *reinterpret_cast<float4*>(p.D + (size_t)(q0 + rr) * p.ldd + col) = o;
                }
                __syncwarp();
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(t_empty + acc);
        }
        if (qok) {
            atomicMin(p.rmin + q, rmin);
            atomicMax(p.rmax + q, rmax);
        }
    }
    // One verdict for the whole block (another block may set the word while
    // this block's threads read it; the barrier inside must not diverge).
    if (__syncthreads_or(*(volatile int*)p.err != 0)) {
        // aborting: let the copies and MMAs this block issued land before exit
        if (warp == 0 && lane == 0) {
            if (a_issued) {
                const unsigned long long c0 = clock64();
                while (!mbar_try(a_full, 0) && clock64() - c0 < WAIT_CYCLES) {
                }
            }
            if (last_load >= 0) {
                const unsigned long long c0 = clock64();
                while (!mbar_try(b_full, last_load & 1) && clock64() - c0 < WAIT_CYCLES) {
                }
            }
        }
        if (warp == 1 && lane == 0 && last_i >= 0) {
            const unsigned long long c0 = clock64();
            while (!mbar_try(t_full + (last_i & 1), (last_i >> 1) & 1) &&
                   clock64() - c0 < WAIT_CYCLES) {
            }
        }
        __syncthreads();
    }
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(2 * TILE_N));
    }
}


// Sorts 64 keys held two per lane (a: entries 0..31, b: 32..63 on input):
// on return a holds the 32 smallest ascending by lane, b the 32 largest.
__device__ __forceinline__ void warp_sort64(uint64_t& a, uint64_t& b, int lane) {
    a = warp_sort32(a, lane);
    b = warp_sort32(b, lane);
    const uint64_t br = __shfl_sync(0xffffffffu, b, 31 - lane);
    uint64_t lo = kmin(a, br), hi = kmax(a, br);  // both bitonic
#pragma unroll
    for (int st = 16; st >= 1; st >>= 1) {
        const uint64_t ol = __shfl_xor_sync(0xffffffffu, lo, st);
        const uint64_t oh = __shfl_xor_sync(0xffffffffu, hi, st);
        const bool upper = (lane & st) != 0;
        lo = upper ? kmax(lo, ol) : kmin(lo, ol);
        hi = upper ? kmax(hi, oh) : kmin(hi, oh);
    }
    a = lo;
    b = hi;
}

// One warp per query; the row of approximate distances is held in registers
// (R per lane, nlist <= 32 R), so the passes over it cost no memory traffic.
// t comes from a 256-bin histogram of the row's distance bits between the
// row's minimum and maximum (from the GEMM): the upper edge of the first bin
// where the running count reaches `take`, rounded up.
template <int R, int P, int DIM>
__global__ void __launch_bounds__(REF_WARPS * 32, 3)
    coarse_refine_kernel(const float* __restrict__ D, int ldd, int nq, int nlist, int take,
                         const float* __restrict__ Q, int dim, const float* __restrict__ cents,
                         const float* __restrict__ qerr, const uint32_t* __restrict__ rmin,
                         const uint32_t* __restrict__ rmax, uint32_t* __restrict__ probes,
                         float* __restrict__ pdist) {
    __shared__ uint64_t buf[REF_WARPS * 64];
    __shared__ unsigned hist[REF_WARPS * 256];
    __shared__ uint32_t cbuf[REF_WARPS * CAND_CAP];
    __shared__ __align__(16) float qsh[REF_WARPS * MAX_DPAD];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * REF_WARPS + warp;
    if (q >= nq) return;  // whole warp leaves together
    const float* row = D + (size_t)q * ldd;
    float v[R];
#pragma unroll
    for (int u = 0; u < R; ++u) {
        const int l = u * 32 + lane;
        v[u] = l < nlist ? row[l] : 0.0f;
    }
    float* qs = qsh + warp * MAX_DPAD;
    for (int i = lane; i < dim; i += 32) qs[i] = Q[(size_t)q * dim + i];
    const float E = qerr[q];
    const uint32_t lo = rmin[q], hi = rmax[q];
    float thr = __int_as_float(0x7f800000);
    if (isfinite(E) && lo <= hi) {
        unsigned* hs = hist + warp * 256;
#pragma unroll
        for (int j = 0; j < 8; ++j) hs[j * 32 + lane] = 0u;
        __syncwarp();
        const float scale = 256.0f / ((float)(hi - lo) + 1.0f);
#pragma unroll
        for (int u = 0; u < R; ++u) {
            const int l = u * 32 + lane;
            if (l < nlist) {
                const float f = (float)(f2ord(v[u]) - lo) * scale;
                atomicAdd(&hs[min(255, (int)f)], 1u);
            }
        }
        __syncwarp();
        // lane owns bins 8 lane .. 8 lane + 7; the first bin where the running
        // count reaches take is bstar
        unsigned c[8], sum = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            c[j] = hs[8 * lane + j];
            sum += c[j];
        }
        unsigned incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        const unsigned reach = __ballot_sync(0xffffffffu, incl >= (unsigned)take);
        int bstar = 255;
        if (reach) {
            const int owner = __ffs(reach) - 1;
            int bs = 255;
            unsigned run = incl - sum;
            bool found = false;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                run += c[j];
                if (!found && run >= (unsigned)take) {
                    bs = 8 * lane + j;
                    found = true;
                }
            }
            bstar = __shfl_sync(0xffffffffu, bs, owner);
        }
        // every key in bins <= bstar has (bits - lo) * scale < bstar + 1 in
        // float arithmetic; the exact bound is widened for both roundings
        uint32_t tb = hi;
        if (bstar < 255) {
            const double w = ((double)bstar + 1.0) / (double)scale * (1.0 + 1e-6) + 2.0;
            tb = (uint32_t)min((double)hi, (double)lo + ceil(w));
        }
        const float t = ord2f(tb);
        thr = t + 2.0f * E;
        thr = thr + fabsf(thr) * ldexpf(1.0f, -22);  // the sum's own rounding
    }
    // candidates d~ <= t + 2 E_q (a NaN distance stays a candidate), compacted
    uint32_t* cb = cbuf + warp * CAND_CAP;
    int nc = 0;
#pragma unroll
    for (int u = 0; u < R; ++u) {
        const int l = u * 32 + lane;
        const bool cand = l < nlist && !(v[u] > thr);
        const unsigned mask = __ballot_sync(0xffffffffu, cand);
        const int pos = nc + __popc(mask & ((1u << lane) - 1u));
        if (cand && pos < CAND_CAP) cb[pos] = (uint32_t)l;
        nc += __popc(mask);
    }
    __syncwarp();
    const bool vec = (dim & 3) == 0;
    if (nc <= 64 && take <= 64) {
        // one pass: each lane rescores the candidates 'lane' and 'lane + 32'
        // (a missing one repeats a present row and is discarded), then the
        // 64 exact keys are sorted across the warp
        const int n0 = min(nc, 32);
        const uint32_t l0 = cb[lane < n0 ? lane : 0];
        uint64_t ka = KEY_NONE, kb = KEY_NONE;
        if (nc <= 32) {
            const float* rows[1] = {cents + (size_t)l0 * dim};
            float d[1];
            l2sq_rows<1, DIM>(qs, rows, dim, vec, d);
            if (lane < n0) ka = make_key(d[0], l0);
        } else {
            const bool has1 = lane + 32 < nc;
            const uint32_t l1 = cb[has1 ? lane + 32 : 0];
            const float* rows[2] = {cents + (size_t)l0 * dim, cents + (size_t)l1 * dim};
            float d[2];
            l2sq_rows<2, DIM>(qs, rows, dim, vec, d);
            ka = make_key(d[0], l0);
            if (has1) kb = make_key(d[1], l1);
        }
        warp_sort64(ka, kb, lane);
        if (lane < take) {
            probes[(size_t)q * take + lane] = key_tag(ka);
            if (pdist) pdist[(size_t)q * take + lane] = key_dist(ka);
        }
        if (lane + 32 < take) {
            probes[(size_t)q * take + lane + 32] = key_tag(kb);
            if (pdist) pdist[(size_t)q * take + lane + 32] = key_dist(kb);
        }
        return;
    }
    WarpTopK<P> tk;
    tk.init(take, buf + warp * 64);
    auto rescore32 = [&](int b0, int count, const uint32_t* list) {
        const bool has = b0 + lane < count;
        const uint32_t l = has ? (list ? list[b0 + lane] : (uint32_t)(b0 + lane)) : 0u;
        const float* rows[1] = {cents + (size_t)l * dim};
        float d[1];
        l2sq_rows<1, DIM>(qs, rows, dim, vec, d);
        tk.add(has ? make_key(d[0], l) : KEY_NONE, has);
    };
    if (nc <= CAND_CAP) {
        for (int b0 = 0; b0 < nc; b0 += 32) rescore32(b0, nc, cb);
    } else {
        // a band too wide for the list (or no usable bound): every centroid
        for (int b0 = 0; b0 < nlist; b0 += 32) rescore32(b0, nlist, nullptr);
    }
    tk.flush();
#pragma unroll
    for (int e = 0; e < P; ++e) {
        const int i = e * 32 + lane;
        if (i < take) {
            probes[(size_t)q * take + i] = key_tag(tk.L[e]);
            if (pdist) pdist[(size_t)q * take + i] = key_dist(tk.L[e]);
        }
    }
}

// Rows longer than REG_NLIST (nlist up to MAX_NLIST): one block per query
// reads its row of approximate distances from D (L2-resident: the GEMM wrote
// the chunk just before) twice -- once into the same 256-bin histogram, once
// to collect the band d~ <= t + 2 E_q -- and rescores the band exactly.  The
// rules are those of coarse_refine_kernel (same threshold arithmetic, same
// keys), so the probes are the same; only the memory the row lives in and
// the number of threads per query differ.
template <int P, int DIM>
__global__ void __launch_bounds__(BIG_THREADS)
    coarse_refine_big_kernel(const float* __restrict__ D, int ldd, int nq, int nlist, int take,
                             const float* __restrict__ Q, int dim,
                             const float* __restrict__ cents, const float* __restrict__ qerr,
                             const uint32_t* __restrict__ rmin, const uint32_t* __restrict__ rmax,
                             uint32_t* __restrict__ probes, float* __restrict__ pdist) {
    __shared__ unsigned hist[256];
    __shared__ uint32_t cand[BIG_CAND];
    __shared__ uint64_t ckey[BIG_CAND];
    __shared__ uint64_t tkbuf[64];
    __shared__ __align__(16) float qs[MAX_DPAD];
    __shared__ unsigned ncand;
    __shared__ int s_bstar;
    const int q = blockIdx.x;
    if (q >= nq) return;  // whole block leaves together
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float* row = D + (size_t)q * ldd;
    for (int i = tid; i < dim; i += BIG_THREADS) qs[i] = Q[(size_t)q * dim + i];
    hist[tid] = 0u;
    if (tid == 0) ncand = 0u;
    __syncthreads();
    const float E = qerr[q];
    const uint32_t lo = rmin[q], hi = rmax[q];
    float thr = __int_as_float(0x7f800000);
    if (isfinite(E) && lo <= hi) {  // block-uniform
        const float scale = 256.0f / ((float)(hi - lo) + 1.0f);
        for (int l = tid; l < nlist; l += BIG_THREADS) {
            const float f = (float)(f2ord(row[l]) - lo) * scale;
            atomicAdd(&hist[min(255, (int)f)], 1u);
        }
        __syncthreads();
        if (warp == 0) {
            // lane owns bins 8 lane .. 8 lane + 7; the first bin where the
            // running count reaches take is bstar
            unsigned c[8], sum = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                c[j] = hist[8 * lane + j];
                sum += c[j];
            }
            unsigned incl = sum;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned t = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += t;
            }
            const unsigned reach = __ballot_sync(0xffffffffu, incl >= (unsigned)take);
            int bstar = 255;
            if (reach) {
                const int owner = __ffs(reach) - 1;
                int bs = 255;
                unsigned run = incl - sum;
                bool found = false;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    run += c[j];
                    if (!found && run >= (unsigned)take) {
                        bs = 8 * lane + j;
                        found = true;
                    }
                }
                bstar = __shfl_sync(0xffffffffu, bs, owner);
            }
            if (lane == 0) s_bstar = bstar;
        }
        __syncthreads();
        const int bstar = s_bstar;
        uint32_t tb = hi;
        if (bstar < 255) {
            const double w = ((double)bstar + 1.0) / (double)scale * (1.0 + 1e-6) + 2.0;
            tb = (uint32_t)min((double)hi, (double)lo + ceil(w));
        }
        const float t = ord2f(tb);
        thr = t + 2.0f * E;
        thr = thr + fabsf(thr) * ldexpf(1.0f, -22);  // the sum's own rounding
    }
    // candidates d~ <= t + 2 E_q (a NaN distance stays a candidate), compacted
    for (int l = tid; l < nlist; l += BIG_THREADS)
        if (!(row[l] > thr)) {
            const unsigned pos = atomicAdd(&ncand, 1u);
            if (pos < (unsigned)BIG_CAND) cand[pos] = (uint32_t)l;
        }
    __syncthreads();
    const unsigned nc = ncand;
    // a band too wide for the list (or no usable bound): every centroid
    const bool all = nc > (unsigned)BIG_CAND;
    const int n = all ? nlist : (int)nc;
    const bool vec = (dim & 3) == 0;
    WarpTopK<P> tk;
    if (warp == 0) tk.init(take, tkbuf);
    for (int b0 = 0; b0 < n; b0 += BIG_CAND) {
        const int cnt = min(BIG_CAND, n - b0);
        for (int i = tid; i < cnt; i += BIG_THREADS) {
            const uint32_t l = all ? (uint32_t)(b0 + i) : cand[i];
            const float* rows[1] = {cents + (size_t)l * dim};
            float d[1];
            l2sq_rows<1, DIM>(qs, rows, dim, vec, d);
            ckey[i] = make_key(d[0], l);
        }
        __syncthreads();
        if (warp == 0)
            for (int i0 = 0; i0 < cnt; i0 += 32) {
                const bool has = i0 + lane < cnt;
                tk.add(has ? ckey[i0 + lane] : KEY_NONE, has);
            }
        __syncthreads();
    }
    if (warp == 0) {
        tk.flush();
#pragma unroll
        for (int e = 0; e < P; ++e) {
            const int i = e * 32 + lane;
            if (i < take) {
                probes[(size_t)q * take + i] = key_tag(tk.L[e]);
                if (pdist) pdist[(size_t)q * take + i] = key_dist(tk.L[e]);
            }
        }
    }
}

}  // namespace ctc

// Centroids for the tensor-core coarse quantizer: fp16 rows scaled by 2^sb
// (largest |c_i| in [2^14, 2^15)), zero-padded to [nlist_pad][dpad], their
// exact squared norms and an upper bound of their norms.
void coarse_tc_prepare(fdb_ivfpq* h) {
    h->c16.release();
    h->c16_norm.release();
    const size_t nlist = h->nlist, dim = h->dim;
    const int dpad = (int)((dim + 63) / 64 * 64);
    if (nlist == 0 || dpad > ctc::MAX_DPAD) return;
    cudaStream_t s = h->ctx->c.stream;
    std::vector<float> cents(nlist * dim);
    FDB_CUDA(cudaMemcpyAsync(cents.data(), h->cents.p, cents.size() * 4, cudaMemcpyDeviceToHost,
                             s));
    FDB_CUDA(cudaStreamSynchronize(s));
    float amax = 0.0f;
    double nmax = 0.0;
    bool finite = true;
    const size_t npad = (nlist + 127) / 128 * 128;
    std::vector<float> norm(npad, 0.0f);
    for (size_t l = 0; l < nlist; ++l) {
        double t = 0.0;
        float t32 = 0.0f;
        for (size_t i = 0; i < dim; ++i) {
            const float x = cents[l * dim + i];
            finite = finite && std::isfinite(x);
            amax = std::max(amax, std::fabs(x));
            t += (double)x * x;
            t32 += x * x;
        }
        norm[l] = t32;
        nmax = std::max(nmax, std::sqrt(t));
    }
    if (!finite) return;  // the SIMT coarse kernel serves such an index
    int ex = 0;
    if (amax > 0.0f) std::frexp(amax, &ex);
    const int sb = amax > 0.0f ? 15 - ex : 0;
    std::vector<__half> c16(npad * dpad, __float2half(0.0f));
    for (size_t l = 0; l < nlist; ++l)
        for (size_t i = 0; i < dim; ++i)
            c16[l * dpad + i] = __float2half_rn(std::ldexp(cents[l * dim + i], sb));
    h->c16.alloc(npad * dpad);
    h->c16_norm.alloc(npad);
    FDB_CUDA(cudaMemcpyAsync(h->c16.p, c16.data(), c16.size() * sizeof(__half),
                             cudaMemcpyHostToDevice, s));
    FDB_CUDA(cudaMemcpyAsync(h->c16_norm.p, norm.data(), npad * 4, cudaMemcpyHostToDevice, s));
    FDB_CUDA(cudaStreamSynchronize(s));
    h->c16_dpad = dpad;
    h->c16_sb = sb;
    h->c16_cmax = (float)(nmax * (1.0 + 1e-6));
    h->c16_npad = (int)npad;
}

bool coarse_tc_eligible(const fdb_ivfpq* h, size_t nq, size_t take) {
    return h->c16.p != nullptr && nq >= 64 && take >= 1 && take <= 256 &&
           take <= h->nlist && h->nlist <= (size_t)ctc::MAX_NLIST;
}

// Probes (ascending (distance, list) keys) and their exact distances for nq
// queries on the device, through the three kernels above.  Queries run in
// chunks whose approximate-distance matrix stays within 96 MB (L2-resident
// between the GEMM and the refinement).
void coarse_tc(fdb_ivfpq* h, const float* dQ, size_t nq, size_t take, uint32_t* probes,
               float* pdist) {
    using namespace ctc;
    Ctx& c = h->ctx->c;
    cudaStream_t s = c.stream;
    const int dpad = h->c16_dpad, npad = h->c16_npad;
    const size_t rows_budget = std::max<size_t>(128, ((size_t)96 << 20) / ((size_t)npad * 4));
    const size_t chunk = std::min(nq, rows_budget / 128 * 128);
    const size_t chunk_pad = (chunk + 127) / 128 * 128;
    h->s_cq16.ensure(chunk_pad * dpad);
    h->s_cqn.ensure(chunk_pad);
    h->s_cqs2.ensure(chunk_pad);
    h->s_cqerr.ensure(chunk_pad);
    h->s_crange.ensure(2 * chunk_pad);
    h->s_cdapprox.ensure(chunk_pad * npad);
    if (chunk_pad > chunk)  // padding rows of the last tile read zeros
        FDB_CUDA(cudaMemsetAsync(h->s_cq16.p + chunk * dpad, 0,
                                 (chunk_pad - chunk) * dpad * sizeof(__half), s));
    const CUtensorMap cm = make_map(h->c16.p, (size_t)npad, dpad);
    int* err = ivf_tc_error_word(h);
    GemmParams p{};
    p.ntile = npad / TILE_N;
    p.katoms = dpad / KATOM;
    p.ldd = npad;
    p.qn = h->s_cqn.p;
    p.qs2 = h->s_cqs2.p;
    p.cn = h->c16_norm.p;
    p.D = h->s_cdapprox.p;
    p.rmin = h->s_crange.p;
    p.rmax = h->s_crange.p + chunk_pad;
    p.err = err;
    p.wait = wait_limit_cycles(c, h->call_wait_cycles);
    // at least 100 KB, so at most two blocks share an SM: each holds 256 of
    // the SM's 512 TMEM columns
    const size_t smem = std::max<size_t>(1024 + 2 * (size_t)p.katoms * ATOM_BYTES +
                                             MAX_TPC * TILE_N * 4 + NEPI * 32 * 32 * 4 + 8 * 8,
                                         100 * 1024);
    FDB_CUDA(cudaFuncSetAttribute(coarse_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)smem));
    for (size_t q0 = 0; q0 < nq; q0 += chunk) {
        const size_t nc = std::min(chunk, nq - q0);
        const float* Qc = dQ + q0 * h->dim;
        coarse_prep_kernel<<<(unsigned)((nc * 32 + 255) / 256), 256, 0, s>>>(
            Qc, (int)nc, (int)h->dim, dpad, h->c16_sb, h->c16_cmax, h->s_cq16.p, h->s_cqn.p,
            h->s_cqs2.p, h->s_cqerr.p, p.rmin, p.rmax);
        FDB_LAUNCH_CHECK();
        const size_t nc_pad = (nc + 127) / 128 * 128;
        const CUtensorMap qm = make_map(h->s_cq16.p, nc_pad, dpad);
        p.nq = (int)nc;
        // tiles per block: about one wave of two blocks per SM
        const size_t qblocks = nc_pad / TILE_M;
        const size_t slots = 2 * (size_t)c.sm_count;
        p.tpc = (int)std::min<size_t>(
            MAX_TPC, std::max<size_t>(1, (qblocks * p.ntile + slots - 1) / slots));
        dim3 grid((unsigned)qblocks, (unsigned)((p.ntile + p.tpc - 1) / p.tpc));
        coarse_gemm_kernel<<<grid, THREADS, smem, s>>>(qm, cm, p);
        FDB_LAUNCH_CHECK();
        const unsigned rgrid = (unsigned)((nc + REF_WARPS - 1) / REF_WARPS);
        uint32_t* pr = probes + q0 * take;
        float* pd = pdist ? pdist + q0 * take : nullptr;
#define FDB_REFINE(RR, PP)                                                                   \
    do {                                                                                     \
        if (h->dim == 128) FDB_REFINE_D(RR, PP, 128);                                        \
        else if (h->dim == 96) FDB_REFINE_D(RR, PP, 96);                                     \
        else FDB_REFINE_D(RR, PP, 0);                                                        \
    } while (0)
#define FDB_REFINE_D(RR, PP, DD)                                                             \
    coarse_refine_kernel<RR, PP, DD><<<rgrid, REF_WARPS * 32, 0, s>>>(                       \
        h->s_cdapprox.p, npad, (int)nc, (int)h->nlist, (int)take, Qc, (int)h->dim, h->cents.p, \
        h->s_cqerr.p, p.rmin, p.rmax, pr, pd)
#define FDB_REFINE_P(RR)                  \
    if (take <= 32) FDB_REFINE(RR, 1);    \
    else if (take <= 64) FDB_REFINE(RR, 2); \
    else if (take <= 128) FDB_REFINE(RR, 4); \
    else FDB_REFINE(RR, 8)
#define FDB_BIG_D(PP, DD)                                                                    \
    coarse_refine_big_kernel<PP, DD><<<(unsigned)nc, BIG_THREADS, 0, s>>>(                   \
        h->s_cdapprox.p, npad, (int)nc, (int)h->nlist, (int)take, Qc, (int)h->dim, h->cents.p, \
        h->s_cqerr.p, p.rmin, p.rmax, pr, pd)
// (run-time dim: the unrolled fixed-dim rescoring needs ~170 registers, which
// would leave one block per SM for the two passes over the row)
#define FDB_BIG(PP) FDB_BIG_D(PP, 0)
        const size_t nl = h->nlist;
        if (nl <= 256) { FDB_REFINE_P(8); }
        else if (nl <= 512) { FDB_REFINE_P(16); }
        else if (nl <= 1024) { FDB_REFINE_P(32); }
        else if (nl <= (size_t)REG_NLIST) { FDB_REFINE_P(64); }
        else if (take <= 32) { FDB_BIG(1); }
        else if (take <= 64) { FDB_BIG(2); }
        else if (take <= 128) { FDB_BIG(4); }
        else { FDB_BIG(8); }
#undef FDB_BIG
#undef FDB_BIG_D
#undef FDB_REFINE_P
#undef FDB_REFINE
#undef FDB_REFINE_D
        FDB_LAUNCH_CHECK();
    }
}

}  // namespace fdb
