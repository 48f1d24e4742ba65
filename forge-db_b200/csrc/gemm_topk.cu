// gemm_topk.cu -- tensor-core (tcgen05) shortlist for brute-force search.
//
// For a block of 128 queries and a chunk of database rows, the kernel forms
// S = Q . X^T with tcgen05.mma (fp16 operands staged in shared memory by TMA
// with 128-byte swizzle, fp32 accumulators in TMEM) and turns every score
// into an approximate metric value:
//     L2^2   : ||q||^2 + ||x||^2 - 2 s
//     dot    : -s
//     cosine : 1 - s / sqrt(||q||^2 ||x||^2)
// Two passes run on the same TMA -> MMA -> TMEM pipeline, with sixteen
// epilogue warps (four per TMEM lane quadrant, each a part of every tile's
// columns) and the tile's column values staged in shared memory by the
// producer:
//   SAMPLE: every S-th 128-row tile only.  Each epilogue thread keeps the 8
//     smallest keys of its row over its 32-column part, sorted in registers
//     (a chunk whose smallest value cannot enter is skipped by one vote); the
//     four parts' lists are the row's 32 entries for the block's row chunk,
//     and the 32nd of their merge over all chunks is a per-query threshold
//     tau that about 32*S rows of the full set pass.
//   FILTER: every tile (256 rows for padded dims <= 128, one N = 256 MMA per
//     K step, else 128).  A score costs half a packed FMA and a third of a
//     three-input minimum; the 8-column groups that may hold a score <= tau
//     are reloaded from TMEM and their hits appended to the block's segment
//     of the query's candidate row, counted with shared-memory atomics.
// select_candidates_kernel then takes the top-kp of each query's candidates
// and bf_rescore_kernel recomputes them exactly in the reference's AVX2
// summation order and certifies the result (see there), so returned
// distances are exact and a bad tau or an overflow only costs a fallback.
//
// Warp roles (640 threads): warp 0 = TMA producer, warp 1 = MMA issuer and
// TMEM owner, warps 4-19 = epilogue.  Every wait on an mbarrier is bounded:
// on timeout the kernel sets an error word, the other warps see it and
// leave, in-flight copies and MMAs are waited for (bounded), TMEM is freed,
// and the host reports FDB_ERR_TIMEOUT.
#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>

#include "fdb_device.cuh"
#include "fdb_internal.h"
#include "fdb_kernels.h"
#include "tc_ptx.cuh"

namespace fdb {
namespace tc {

// Threads per block: both passes run sixteen epilogue warps (four per TMEM
// lane quadrant, one part of each tile's columns apiece) so that the latency
// of each warp's loads and appends is hidden by the others.
constexpr int THREADS_FILTER = 640;
constexpr int EPI_WARP0 = 4;
constexpr int SAMPLE_K = 32;  // sample-pass shortlist per query
constexpr int EPI_SHORTLIST = 0, EPI_FILTER = 1;
constexpr int NCV = 4;        // filter pass: staged column-value slots (one per tile)
constexpr int MAX_STAGES = 6; // B pipeline stages at most
// mbarriers: a_full, b_full/b_empty [MAX_STAGES], t_full/t_empty [4], cv_full/cv_empty [NCV]
constexpr int NBARS = 1 + 2 * MAX_STAGES + 8 + 2 * NCV;

// B pipeline stages: the filter pass keeps more tiles in flight (its shared
// memory holds no candidate buffers); at most ~200 KB in every case.
__host__ __device__ constexpr int b_stages(int katoms, int epi, int bn) {
    return bn == 256 ? (katoms == 1 ? 4 : 2) : (katoms <= 2 ? 4 : (katoms == 3 ? 3 : 2));
}
// The filter pass's B tile height: 256 rows (one N = 256 MMA per K step:
// the A tile is read from shared memory once per 256 rows instead of once
// per 128, which with the TMA writes is what bounds the MMA rate) where the
// stages fit, i.e. padded dim <= 128; else 128.
__host__ __device__ constexpr int filter_bn(int katoms) { return katoms <= 2 ? 256 : 128; }

struct GemmTopkParams {
    int nq;              // queries
    size_t n;            // database rows
    int katoms;          // padded dim / 64
    int metric;
    const float* qnorm;  // [nq] exact squared norms
    const float* colv;   // per-row column values (see column_values), padded to whole tiles
    float colmax;        // L2: largest ||x||^2 (bounds the filter test's rounding)
    size_t rows_per_chunk;
    uint64_t tag_base;   // global index of row 0
    // SAMPLE pass
    int tile_stride;     // process global tiles t with t % tile_stride == 0
    uint64_t* part;      // [chunks][nq][SAMPLE_K], preset to KEY_NONE
    // FILTER pass
    const float* tau_q;  // [nq] admission threshold
    uint64_t* cand;      // [nq][cap] candidate keys
    unsigned* cand_cnt;  // [nq] candidates seen (may exceed cap)
    int seg;             // FILTER: entries of a (query, row chunk) segment of the candidate row
    unsigned* seg_cnt;   // FILTER: [nq][chunks] entries each block found (may exceed seg)
    int cap;
    int* err;            // error word (0 = ok)
    unsigned long long wait;  // limit of each bounded wait, SM clock cycles
};

// Approximate metric families (compile-time, so no per-score branching):
//   MET_L2  : ||q||^2 + ||x||^2 - 2 s   (qv = ||q||^2, cv = ||x||^2)
//   MET_DOT : -s
//   MET_COS : 1 - s / (||q|| ||x||)      (qv = 1/||q||, cv = 1/||x||; a zero
//             norm on either side gives 0, the reference's value)
constexpr int MET_L2 = 0, MET_DOT = 1, MET_COS = 2;

template <int MET>
__device__ __forceinline__ float approx_metric(float s, float qv, float cv) {
    if (MET == MET_DOT) return -s;
    if (MET == MET_COS) return (qv == 0.0f || cv == 0.0f) ? 0.0f : 1.0f - s * (qv * cv);
    return __fmaf_rn(-2.0f, s, qv + cv);
}

// The 32 per-row values of one column chunk (||x||^2 for L2, 1/||x|| for
// cosine), read with eight warp-uniform 128-bit loads.  The arrays are padded
// to whole tiles, so a chunk never reads past their end.
template <int MET>
__device__ __forceinline__ void column_values(const float* colv, size_t row0, float (&cv)[32]) {
    if (MET == MET_DOT) {
#pragma unroll
        for (int j = 0; j < 32; ++j) cv[j] = 0.0f;
        return;
    }
    const float4* p4 = reinterpret_cast<const float4*>(colv + row0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 t = __ldg(p4 + i);
        cv[4 * i] = t.x;
        cv[4 * i + 1] = t.y;
        cv[4 * i + 2] = t.z;
        cv[4 * i + 3] = t.w;
    }
}

// BN: rows of the B tile per MMA (128, or 256 for the filter pass).
template <int EPI, int MET, int BN>
__global__ void __launch_bounds__(THREADS_FILTER, 1)
    gemm_topk_kernel(const __grid_constant__ CUtensorMap qmap,
                     const __grid_constant__ CUtensorMap xmap, GemmTopkParams p) {
    static_assert(BN == 128 || (BN == 256 && EPI == EPI_FILTER), "tile height");
    constexpr int BATOM = BN * 128;  // bytes of one 64-wide K atom of the B tile
    constexpr uint32_t IDESC_BN = (1u << 4) | ((uint32_t)(BN >> 3) << 17) |
                                  ((uint32_t)(TILE_M >> 4) << 24);
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t base = smem_u32(smem_raw);
    unsigned char* smem = smem_raw + ((1024 - (base & 1023)) & 1023);  // 1024-byte aligned
    const int KA = p.katoms;
    const int NSTAGE = b_stages(KA, EPI, BN);
    // TMEM accumulators (BN columns each, 512 columns in all for the filter
    // pass): the MMA runs ahead of the epilogue by NACC - 1 tiles
    constexpr int NACC = 512 / BN;
    // each tile's column values (||x||^2 or 1/||x||) are staged in shared
    // memory by a bulk copy that the producer issues with the tile
    constexpr bool STAGE_CV = MET != MET_DOT;
    unsigned char* a_tile = smem;                                  // KA atoms
    unsigned char* b_tile = a_tile + KA * ATOM_BYTES;              // NSTAGE x KA B atoms
    float* cvbuf = reinterpret_cast<float*>(b_tile + NSTAGE * KA * BATOM);  // [NCV][BN]
    uint64_t* bars = reinterpret_cast<uint64_t*>(cvbuf + NCV * BN);
    uint64_t* a_full = bars + 0;
    uint64_t* b_full = a_full + 1;              // [MAX_STAGES]
    uint64_t* b_empty = b_full + MAX_STAGES;    // [MAX_STAGES]
    uint64_t* t_full = b_empty + MAX_STAGES;    // [4]
    uint64_t* t_empty = t_full + 4;             // [4]
    uint64_t* cv_full = t_empty + 4;            // [NCV]
    uint64_t* cv_empty = cv_full + NCV;         // [NCV]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + NBARS);

    // filter pass: the hits of each query row of this block go to the block's
    // own segment of the query's candidate row, counted here (shared-memory
    // atomics instead of one global atomic per row and group)
    __shared__ unsigned qcnt[TILE_M];
    if (EPI == EPI_FILTER && threadIdx.x < TILE_M) qcnt[threadIdx.x] = 0u;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qb = blockIdx.x;
    const size_t r0 = (size_t)blockIdx.y * p.rows_per_chunk;
    const size_t r1 = min(p.n, r0 + p.rows_per_chunk);
    const int ntiles = r0 < r1 ? (int)((r1 - r0 + BN - 1) / BN) : 0;
    // tiles this block processes: t = first + i * stride, i < count
    const int stride = EPI == EPI_SHORTLIST ? p.tile_stride : 1;
    const int tile0 = (int)(r0 / BN);
    const int first = (stride - tile0 % stride) % stride;
    const int count = ntiles > first ? (ntiles - first + stride - 1) / stride : 0;
    const uint32_t stage_bytes = (uint32_t)(KA * ATOM_BYTES);  // the A tile
    const uint32_t bstage_bytes = (uint32_t)(KA * BATOM);
    const int n_epi_warps = 16;

    if (threadIdx.x == 0) {
        mbar_init(a_full, 1);
        for (int i = 0; i < MAX_STAGES; ++i) {
            mbar_init(b_full + i, 1);
            mbar_init(b_empty + i, 1);
        }
        for (int i = 0; i < 4; ++i) {
            mbar_init(t_full + i, 1);
            mbar_init(t_empty + i, n_epi_warps);
        }
        for (int i = 0; i < NCV; ++i) {
            mbar_init(cv_full + i, 1);
            mbar_init(cv_empty + i, n_epi_warps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(NACC * BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // Last asynchronous operation each role issued, so that an aborting
    // block can wait for it (bounded) before it frees TMEM and exits.
    int last_load[MAX_STAGES];  // producer: last use issued per B stage
    int last_cv[NCV];           // producer: last use issued per column-value slot
    for (int i = 0; i < MAX_STAGES; ++i) last_load[i] = -1;
    for (int i = 0; i < NCV; ++i) last_cv[i] = -1;
    int last_i = -1;                      // MMA issuer: last tile committed

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        if (lane == 0 && count > 0) {
            mbar_expect_tx(a_full, stage_bytes);
            for (int a = 0; a < KA; ++a)
                tma_load_2d(a_tile + a * ATOM_BYTES, &qmap, a_full, a * KATOM, qb * TILE_M);
            for (int i = 0; i < count; ++i) {
                const int s = i % NSTAGE;
                const int use = i / NSTAGE;
                if (i >= NSTAGE && !mbar_wait(b_empty + s, (use - 1) & 1, p.err, p.wait)) break;
                mbar_expect_tx(b_full + s, bstage_bytes);
                const int row = (int)(r0 + (size_t)(first + i * stride) * BN);
                unsigned char* dst = b_tile + s * KA * BATOM;
                // a 256-row atom is two stacked 128-row boxes (the swizzle
                // repeats every 8 rows, so the halves join seamlessly); rows
                // past the end of the rows read as zeros
                for (int a = 0; a < KA; ++a)
#pragma unroll
                    for (int hb = 0; hb < BN / TILE_N; ++hb)
                        tma_load_2d(dst + a * BATOM + hb * ATOM_BYTES, &xmap, b_full + s,
                                    a * KATOM, row + hb * TILE_N);
                last_load[s] = use;
                if (STAGE_CV) {
                    // the tile's BN column values (colv is padded by 256 beyond
                    // its rows; row is a multiple of BN, so the copy is aligned)
                    const int c = i % NCV, cu = i / NCV;
                    if (i >= NCV && !mbar_wait(cv_empty + c, (cu - 1) & 1, p.err, p.wait)) break;
                    mbar_expect_tx(cv_full + c, BN * 4);
                    bulk_load(cvbuf + c * BN, p.colv + row, BN * 4, cv_full + c);
                    last_cv[c] = cu;
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0 && count > 0) {
            bool ok = mbar_wait(a_full, 0, p.err, p.wait);
            for (int i = 0; ok && i < count; ++i) {
                const int s = i % NSTAGE;
                const int use = i / NSTAGE;
                const int b = i % NACC;  // TMEM accumulator buffer
                if (i >= NACC && !mbar_wait(t_empty + b, ((i / NACC) - 1) & 1, p.err, p.wait))
                    break;
                if (!mbar_wait(b_full + s, use & 1, p.err, p.wait)) break;
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)(b * BN);
                const uint32_t abase = smem_u32(a_tile);
                const uint32_t bbase = smem_u32(b_tile + s * KA * BATOM);
                for (int a = 0; a < KA; ++a) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {  // 4 x K16 per 64-wide atom
                        umma_f16_n(d, smem_desc_sw128(abase + (uint32_t)(a * ATOM_BYTES + kk * 32)),
                                   smem_desc_sw128(bbase + (uint32_t)(a * BATOM + kk * 32)),
                                   IDESC_BN, (a | kk) != 0);
                    }
                }
                umma_commit(b_empty + s);  // stage s may be refilled once these MMAs finish
                umma_commit(t_full + b);   // accumulator b is ready for the epilogue
                last_i = i;
            }
        }
    } else if (warp >= EPI_WARP0 && warp < EPI_WARP0 + n_epi_warps) {
        // ---------------- epilogue ----------------
        const int w = warp - EPI_WARP0;
        const int quad = w & 3;            // TMEM lane quadrant = warp % 4
        const int part = w >> 2;           // BN/4-column part of each tile
        const int e = quad * 32 + lane;    // query row in the block
        const int q = qb * TILE_M + e;
        const bool qok = q < p.nq;
        const float qn0 = (qok && p.qnorm) ? p.qnorm[q] : 0.0f;
        const float qn = MET == MET_COS ? (qn0 > 0.0f ? rsqrtf(qn0) : 0.0f) : qn0;
        const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
        const float tau = EPI == EPI_FILTER ? (qok ? p.tau_q[q] : -__int_as_float(0x7f800000))
                                            : __int_as_float(0x7f800000);
        if constexpr (EPI == EPI_FILTER) {
            // Per-lane admission test, one or two instructions per score:
            //   L2 : fma(-2, s, ||x||^2) <= (tau - ||q||^2) + slack
            //   DOT: s >= -tau                              (exact)
            //   COS: s / ||x|| >= (1 - tau) ||q|| - slack, or a zero row
            // The slack covers the different rounding of the rearranged test,
            // so every row whose key distance (approx_metric) is <= tau passes;
            // hits are re-checked with approx_metric before they are appended.
            float tt;
            if (!qok) {
                tt = MET == MET_DOT ? __int_as_float(0x7f800000) : -__int_as_float(0x7f800000);
            } else if (MET == MET_L2) {
                tt = (tau - qn) + ldexpf(2.0f * fabsf(qn) + 2.0f * p.colmax + fabsf(tau), -20);
            } else if (MET == MET_DOT) {
                tt = -tau;
            } else {
                tt = qn == 0.0f ? -__int_as_float(0x7f800000)
                                : ((1.0f - tau) - ldexpf(2.0f + fabsf(tau), -18)) / qn;
            }
            // The test of a 32-column chunk: bit g is set when some row of the
            // warp may admit a row among the chunk's columns 8g..8g+7.  Each
            // group's best test value comes from a short tree (L2: the smallest
            // fma(-2, s, ||x||^2), two per f32x2 instruction; dot and cosine:
            // the negated largest s or s/||x||, zero rows counted as hits) and
            // one vote skips the chunk when no lane can have a hit.
            const float T = MET == MET_L2 ? tt : -tt;
            auto test = [&](const uint32_t(&v)[32], const float* cvs) -> unsigned {
                float m[4];
                if constexpr (MET == MET_L2) {
                    const uint64_t m2 = pack2(__float_as_uint(-2.0f), __float_as_uint(-2.0f));
#pragma unroll
                    for (int g8 = 0; g8 < 4; ++g8) {  // one group at a time: few live values
                        float y[8];
#pragma unroll
                        for (int h2 = 0; h2 < 2; ++h2) {
                            const int i2 = 2 * g8 + h2;
                            const ulonglong2 cc = reinterpret_cast<const ulonglong2*>(cvs)[i2];
                            const uint64_t x01 = fma2(m2, pack2(v[4 * i2], v[4 * i2 + 1]), cc.x);
                            const uint64_t x23 =
                                fma2(m2, pack2(v[4 * i2 + 2], v[4 * i2 + 3]), cc.y);
                            y[4 * h2] = __uint_as_float((uint32_t)x01);
                            y[4 * h2 + 1] = __uint_as_float((uint32_t)(x01 >> 32));
                            y[4 * h2 + 2] = __uint_as_float((uint32_t)x23);
                            y[4 * h2 + 3] = __uint_as_float((uint32_t)(x23 >> 32));
                        }
                        m[g8] = min3f(min3f(y[0], y[1], y[2]), min3f(y[3], y[4], y[5]),
                                      fminf(y[6], y[7]));
                    }
                } else {
#pragma unroll
                    for (int g8 = 0; g8 < 4; ++g8) {
                        float y[8];
#pragma unroll
                        for (int jj = 0; jj < 8; ++jj) {
                            const int j = 8 * g8 + jj;
                            const float sj = __uint_as_float(v[j]);
                            if (MET == MET_DOT) y[jj] = -sj;
                            else
                                y[jj] = cvs[j] == 0.0f ? -__int_as_float(0x7f800000)
                                                       : -(sj * cvs[j]);
                        }
                        m[g8] = min3f(min3f(y[0], y[1], y[2]), min3f(y[3], y[4], y[5]),
                                      fminf(y[6], y[7]));
                    }
                }
                const float mn = fminf(fminf(m[0], m[1]), fminf(m[2], m[3]));
                if (!__any_sync(0xffffffffu, mn <= T)) return 0u;
                unsigned gm = 0;
#pragma unroll
                for (int g8 = 0; g8 < 4; ++g8)
                    gm |= __any_sync(0xffffffffu, m[g8] <= T) ? 1u << g8 : 0u;
                return gm;
            };
            // The groups of gm (bit g: columns 8g..8g+7 of this warp's chunk),
            // reloaded from the accumulator, which is still held: every row
            // whose key distance (approx_metric) is <= tau is appended to the
            // query's candidates, one atomic per group.
            auto admit = [&](unsigned gm, uint32_t tcol, const float* cvs, size_t cbase) {
                const int nvalid = cbase < r1 ? (int)min((size_t)32, r1 - cbase) : 0;
                const uint32_t tag = (uint32_t)(p.tag_base + cbase);
                uint64_t* crow = p.cand + (size_t)q * p.cap + (size_t)blockIdx.y * p.seg;
                while (gm) {
                    const int gi = __ffs(gm) - 1;
                    gm &= gm - 1;
                    uint32_t w8[8];
                    tmem_ld8(tmem + lane_base + tcol + (uint32_t)(gi * 8), w8);
                    float d[8];
                    unsigned hm = 0;
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj) {
                        const int j = gi * 8 + jj;
                        d[jj] = approx_metric<MET>(__uint_as_float(w8[jj]), qn,
                                                   MET == MET_DOT ? 0.0f : cvs[j]);
                        if (qok && j < nvalid && d[jj] <= tau) hm |= 1u << jj;
                    }
                    if (hm == 0) continue;
                    unsigned ix = atomicAdd(qcnt + e, (unsigned)__popc(hm));
#pragma unroll
                    for (int jj = 0; jj < 8; ++jj)
                        if (hm >> jj & 1u) {
                            if (ix < (unsigned)p.seg)
                                crow[ix] = make_key(d[jj], tag + (uint32_t)(gi * 8 + jj));
                            ++ix;
                        }
                }
            };
            for (int i = 0; i < count; ++i) {
                const int b = i % NACC, c = i % NCV;
                int got = 0;
                if (lane == 0)
                    got = mbar_wait(t_full + b, (i / NACC) & 1, p.err, p.wait) &&
                          (!STAGE_CV || mbar_wait(cv_full + c, (i / NCV) & 1, p.err, p.wait));
                got = __shfl_sync(0xffffffffu, got, 0);
                if (!got) break;
                tc_fence_after();
                // this warp's BN/4 columns of the tile, 32 at a time (one copy
                // of the test and slow path: the loop is not unrolled)
#pragma unroll 1
                for (int hc = 0; hc < BN / 128; ++hc) {
                    const int col = part * (BN / 4) + hc * 32;
                    const uint32_t tcol = (uint32_t)(b * BN + col);
                    uint32_t va[32];
                    tmem_ld32_nowait(tmem + lane_base + tcol, va);
                    tmem_wait_regs(va);
                    const float* cvs = cvbuf + c * BN + col;
                    const unsigned gm = test(va, cvs);
                    if (gm) admit(gm, tcol, cvs, r0 + (size_t)i * BN + (size_t)col);
                }
                // done with the accumulator and the staged column values
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(t_empty + b);
                    if (STAGE_CV) mbar_arrive(cv_empty + c);
                }
            }
        } else {
            // Sample pass: each thread keeps the 8 smallest keys of its row over
            // its 32-column part of the sampled tiles, sorted in registers.  The
            // four parts' lists form the chunk's 32 entries for the row; the
            // merged 32nd over all chunks is tau.  That is at least the 32nd of
            // every sampled row (a part may hold more than 8 of the best 32), so
            // at least 32 sampled rows lie at or below it.
            uint64_t top[8];
#pragma unroll
            for (int i2 = 0; i2 < 8; ++i2) top[i2] = KEY_NONE;
            for (int i = 0; i < count; ++i) {
                const int b = i % NACC, cs = i % NCV;
                int got = 0;
                if (lane == 0)
                    got = mbar_wait(t_full + b, (i / NACC) & 1, p.err, p.wait) &&
                          (!STAGE_CV || mbar_wait(cv_full + cs, (i / NCV) & 1, p.err, p.wait));
                got = __shfl_sync(0xffffffffu, got, 0);
                if (!got) break;
                tc_fence_after();
                uint32_t v[32];
                tmem_ld32_nowait(tmem + lane_base + (uint32_t)(b * BN + part * 32), v);
                tmem_wait_regs(v);
                const float* cvs = cvbuf + cs * BN + part * 32;
                float x[32];
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    x[j] = approx_metric<MET>(__uint_as_float(v[j]), qn,
                                              MET == MET_DOT ? 0.0f : cvs[j]);
                // the scores and column values are in registers: release both
                tc_fence_before();
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(t_empty + b);
                    if (STAGE_CV) mbar_arrive(cv_empty + cs);
                }
                const size_t cb = r0 + (size_t)(first + i * stride) * BN + (size_t)part * 32;
                const int nvalid = cb < r1 ? (int)min((size_t)32, r1 - cb) : 0;
                const uint32_t tag0 = (uint32_t)(p.tag_base + cb);
                const float thr = top[7] == KEY_NONE ? __int_as_float(0x7f800000) : key_dist(top[7]);
                float t11[11];
#pragma unroll
                for (int k3 = 0; k3 < 10; ++k3)
                    t11[k3] = min3f(x[3 * k3], x[3 * k3 + 1], x[3 * k3 + 2]);
                t11[10] = fminf(x[30], x[31]);
                const float mn = fminf(min3f(min3f(t11[0], t11[1], t11[2]),
                                             min3f(t11[3], t11[4], t11[5]),
                                             min3f(t11[6], t11[7], t11[8])),
                                       fminf(t11[9], t11[10]));
                if (!__any_sync(0xffffffffu, qok && nvalid > 0 && mn <= thr)) continue;
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    // (NaN fails x <= thr and is never kept)
                    if (!(qok && j < nvalid && x[j] <= thr)) continue;
                    const uint64_t k = make_key(x[j], tag0 + (uint32_t)j);
                    if (k >= top[7]) continue;
                    top[7] = k;
#pragma unroll
                    for (int i2 = 7; i2 > 0; --i2) {
                        const uint64_t lo2 = kmin(top[i2 - 1], top[i2]);
                        const uint64_t hi2 = kmax(top[i2 - 1], top[i2]);
                        top[i2 - 1] = lo2;
                        top[i2] = hi2;
                    }
                }
            }
            if (qok) {
                uint64_t* dst = p.part + ((size_t)blockIdx.y * p.nq + q) * SAMPLE_K + part * 8;
#pragma unroll
                for (int i2 = 0; i2 < 8; ++i2) dst[i2] = top[i2];
            }
        }
    }
    // One verdict for the whole block (another block may set the word while
    // this block's threads read it; the barrier inside must not diverge).
    if (__syncthreads_or(*(volatile int*)p.err != 0)) {
        // aborting: let the copies and MMAs this block issued land before exit
        // (waits on phases that already completed return at once)
        if (warp == 0 && lane == 0) {
            for (int s2 = 0; s2 < NSTAGE; ++s2)
                if (last_load[s2] >= 0) {
                    const unsigned long long t0 = clock64();
                    while (!mbar_try(b_full + s2, last_load[s2] & 1) &&
                           clock64() - t0 < WAIT_CYCLES) {
                    }
                }
            for (int c2 = 0; c2 < NCV; ++c2)
                if (last_cv[c2] >= 0) {
                    const unsigned long long t0 = clock64();
                    while (!mbar_try(cv_full + c2, last_cv[c2] & 1) &&
                           clock64() - t0 < WAIT_CYCLES) {
                    }
                }
        }
        if (warp == 1 && lane == 0 && last_i >= 0) {
            const unsigned long long t0 = clock64();
            while (!mbar_try(t_full + (last_i % NACC), (last_i / NACC) & 1) &&
                   clock64() - t0 < WAIT_CYCLES) {
            }
        }
        __syncthreads();
    }
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(NACC * BN));
    }
    if (EPI == EPI_FILTER && threadIdx.x < TILE_M) {
        // (every epilogue warp is past the block-wide barrier above)
        const int qq = qb * TILE_M + (int)threadIdx.x;
        if (qq < p.nq) p.seg_cnt[(size_t)qq * gridDim.y + blockIdx.y] = qcnt[threadIdx.x];
    }
}

// One warp per query: the filter pass's per-block segments of its candidate
// row moved to the row's front (in block order, a forward copy: a segment's
// destination never passes its source), and the count; a segment that
// overflowed marks the row as overflowing (count cap + 1: never certified).
__global__ void __launch_bounds__(256)
    compact_segments_kernel(uint64_t* __restrict__ cand, const unsigned* __restrict__ seg_cnt,
                            int chunks, int seg, int cap, int nq, unsigned* __restrict__ cnt) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * 8 + warp;
    if (q >= nq) return;
    uint64_t* row = cand + (size_t)q * cap;
    unsigned total = 0;
    bool over = false;
    for (int y = 0; y < chunks; ++y) {
        const unsigned c = seg_cnt[(size_t)q * chunks + y];
        over = over || c > (unsigned)seg;
        const unsigned n = min(c, (unsigned)seg);
        const size_t src = (size_t)y * seg;
        if (src != total)
            for (unsigned i = 0; i < n; i += 32) {
                const uint64_t v = i + lane < n ? row[src + i + lane] : 0;
                __syncwarp();
                if (i + lane < n) row[total + i + lane] = v;
                __syncwarp();
            }
        total += n;
    }
    if (lane == 0) cnt[q] = over ? (unsigned)cap + 1u : total;
}

// Top-kp of each query's candidate keys (one warp per query).
template <int P>
__global__ void __launch_bounds__(256)
    select_candidates_kernel(const uint64_t* __restrict__ cand, const unsigned* __restrict__ cnt,
                             int cap, int nq, int kp, uint64_t* __restrict__ out) {
    const int warp = threadIdx.x >> 5;
    const int q = blockIdx.x * 8 + warp;
    if (q >= nq) return;
    WarpTopK<P> tk;
    tk.init(kp, nullptr);
    const int c = (int)min(cnt[q], (unsigned)cap);
    tk.ingest(cand + (size_t)q * cap, c);
    tk.store(out + (size_t)q * kp);
}

// tau[q] = the 32nd distance of the sample top-32 (+inf if fewer).
__global__ void sample_tau_kernel(const uint64_t* __restrict__ top32, int nq,
                                  float* __restrict__ tau) {
    const int q = blockIdx.x * blockDim.x + threadIdx.x;
    if (q >= nq) return;
    const uint64_t k = top32[(size_t)q * SAMPLE_K + SAMPLE_K - 1];
    tau[q] = k == KEY_NONE ? __int_as_float(0x7f800000) : key_dist(k);
}

}  // namespace tc

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
namespace {

__global__ void to_half_kernel(const float* __restrict__ x, size_t n, int dim, int kpad,
                               __half* __restrict__ out) {
    const size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= n * (size_t)kpad) return;
    const size_t r = t / kpad;
    const int c = (int)(t - r * kpad);
    out[t] = __float2half_rn(c < dim ? x[r * dim + c] : 0.0f);
}

size_t gemm_smem(int katoms, int epi, int bn) {
    const int nstage = tc::b_stages(katoms, epi, bn);
    return 1024 + (size_t)katoms * tc::ATOM_BYTES + (size_t)nstage * katoms * bn * 128 +
           (size_t)tc::NCV * bn * 4 + (tc::NBARS + 1) * 8;
}

// Row chunks: enough blocks for several waves with little tail waste.
int pick_chunks(size_t n, int nq, int sm_count, size_t* rows_per_chunk) {
    const int nqb = (nq + tc::TILE_M - 1) / tc::TILE_M;
    int best_r = 1;
    double best_cost = 1e30;
    const int rmax = (int)std::min<size_t>(
        256, std::max<size_t>(1, (n + tc::TILE_N - 1) / tc::TILE_N / 4));
    for (int r = 1; r <= rmax; ++r) {
        const double ctas = (double)nqb * r;
        const double waves = std::ceil(ctas / sm_count);
        const double cost = waves * (1.0 / r) + 0.001 * r;
        if (cost < best_cost - 1e-12) {
            best_cost = cost;
            best_r = r;
        }
    }
    size_t rows = (n + best_r - 1) / best_r;
    // a multiple of 256 rows: whole filter-pass tiles (and sample-pass tiles)
    rows = (rows + 255) / 256 * 256;
    *rows_per_chunk = rows;
    return (int)((n + rows - 1) / rows);
}

template <int EPI, int MET>
void launch_pass_m(cudaStream_t s, const CUtensorMap& qm, const CUtensorMap& xm, int nq,
                   int chunks, const tc::GemmTopkParams& p) {
    dim3 grid((unsigned)((nq + tc::TILE_M - 1) / tc::TILE_M), (unsigned)chunks);
    const unsigned threads = tc::THREADS_FILTER;
    auto go = [&](auto kernel, int bn) {
        const size_t smem = gemm_smem(p.katoms, EPI, bn);
        FDB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)smem));
        kernel<<<grid, threads, smem, s>>>(qm, xm, p);
    };
    if (EPI == tc::EPI_FILTER && tc::filter_bn(p.katoms) == 256)
        go(tc::gemm_topk_kernel<EPI, MET, (EPI == tc::EPI_FILTER ? 256 : 128)>, 256);
    else
        go(tc::gemm_topk_kernel<EPI, MET, 128>, 128);
    FDB_LAUNCH_CHECK();
}

template <int EPI>
void launch_pass(cudaStream_t s, const CUtensorMap& qm, const CUtensorMap& xm, int nq,
                 int chunks, const tc::GemmTopkParams& p) {
    if (p.metric == DOT_PRODUCT) launch_pass_m<EPI, tc::MET_DOT>(s, qm, xm, nq, chunks, p);
    else if (p.metric == COSINE) launch_pass_m<EPI, tc::MET_COS>(s, qm, xm, nq, chunks, p);
    else launch_pass_m<EPI, tc::MET_L2>(s, qm, xm, nq, chunks, p);
}

}  // namespace

void launch_to_half(cudaStream_t s, const float* x, size_t n, int dim, int kpad, __half* out) {
    size_t total = n * (size_t)kpad;
    if (total == 0) return;
    to_half_kernel<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(x, n, dim, kpad, out);
    FDB_LAUNCH_CHECK();
}

// Sample pass, threshold, filter pass and candidate selection.  Scratch is
// carved from the caller's buffers (sizes from gemm_shortlist_scratch).
void gemm_shortlist(cudaStream_t s, const __half* q16, int nq, const float* qnorm,
                    const __half* x16, size_t n, int kpad, const float* colv, int metric,
                    uint64_t tag_base, int kp, int sm_count, float colmax, GemmScratch& w) {
    FDB_REQUIRE(kpad % tc::KATOM == 0 && kpad <= 256, FDB_ERR_UNSUPPORTED, "bad padded dim");
    FDB_REQUIRE(kp >= 1 && kp <= 256, FDB_ERR_UNSUPPORTED, "shortlist too long");
    CUtensorMap qm = make_map(q16, (size_t)nq, kpad);
    CUtensorMap xm = make_map(x16, n, kpad);
    size_t rows_per_chunk = 0;
    const int chunks = pick_chunks(n, nq, sm_count, &rows_per_chunk);
    // about 32 * stride rows of the full set pass the sample threshold:
    // aim for >= 2 kp of them
    int stride = 1;
    while (tc::SAMPLE_K * stride < 2 * kp) stride <<= 1;
    tc::GemmTopkParams p{};
    p.nq = nq;
    p.n = n;
    p.katoms = kpad / tc::KATOM;
    p.metric = metric;
    p.qnorm = qnorm;
    p.colv = colv;
    p.colmax = colmax;
    p.rows_per_chunk = rows_per_chunk;
    p.tag_base = tag_base;
    p.err = w.err;
    p.wait = w.wait_cycles;
    // --- sample pass ---
    w.part.ensure((size_t)chunks * nq * tc::SAMPLE_K);
    w.top32.ensure((size_t)nq * tc::SAMPLE_K);
    w.tau.ensure(nq);
    FDB_CUDA(cudaMemsetAsync(w.part.p, 0xff, w.part.bytes(), s));
    p.tile_stride = stride;
    p.part = w.part.p;
    launch_pass<tc::EPI_SHORTLIST>(s, qm, xm, nq, chunks, p);
    launch_merge_lists(s, w.part.p, chunks, (size_t)nq * tc::SAMPLE_K, nq, tc::SAMPLE_K,
                       w.top32.p);
    tc::sample_tau_kernel<<<(nq + 255) / 256, 256, 0, s>>>(w.top32.p, nq, w.tau.p);
    FDB_LAUNCH_CHECK();
    // --- filter pass ---
    // each row chunk's block owns a segment of every candidate row
    const int seg = std::max(32, std::max(1024, 16 * kp) / chunks);
    w.cap = seg * chunks;
    w.cand.ensure((size_t)nq * w.cap);
    w.cand_cnt.ensure(nq);
    w.seg_cnt.ensure((size_t)nq * chunks);
    p.seg = seg;
    p.seg_cnt = w.seg_cnt.p;
    p.tile_stride = 1;
    p.tau_q = w.tau.p;
    p.cand = w.cand.p;
    p.cand_cnt = w.cand_cnt.p;
    p.cap = w.cap;
    if (w.filter_ev0) FDB_CUDA(cudaEventRecord(w.filter_ev0, s));
    launch_pass<tc::EPI_FILTER>(s, qm, xm, nq, chunks, p);
    if (w.filter_ev1) FDB_CUDA(cudaEventRecord(w.filter_ev1, s));
    tc::compact_segments_kernel<<<(unsigned)((nq + 7) / 8), 256, 0, s>>>(
        w.cand.p, w.seg_cnt.p, chunks, seg, w.cap, nq, w.cand_cnt.p);
    FDB_LAUNCH_CHECK();
    // --- top-kp of the candidates ---
    w.approx.ensure((size_t)nq * kp);
    const unsigned grid = (unsigned)((nq + 7) / 8);
#define FDB_SEL(PP)                                                                      \
    tc::select_candidates_kernel<PP><<<grid, 256, 0, s>>>(w.cand.p, w.cand_cnt.p, w.cap, nq, \
                                                          kp, w.approx.p)
    if (kp <= 32) FDB_SEL(1);
    else if (kp <= 64) FDB_SEL(2);
    else if (kp <= 128) FDB_SEL(4);
    else FDB_SEL(8);
#undef FDB_SEL
    FDB_LAUNCH_CHECK();
}

// ---------------------------------------------------------------------------
// exact rescoring of brute-force shortlists
// ---------------------------------------------------------------------------
constexpr int BRS_WARPS = 8;

// One warp per query: exact metric of each shortlisted row (AVX2 order), k
// best kept.  Certification: every approximate value is within E of the
// exact one (fp16 rounding of both operands, fp32 accumulation, and the
// rounding of the exact computation itself).  A row outside the shortlist
// has approximate value >= B, where B is the last shortlisted value if the
// query had at least kp candidates and tau otherwise; so if the exact k-th
// value + E < B no such row can be in the exact top-k.  Overflowing
// candidate arrays are never certified.
// DIM: 128 (the row length known at compile time, every load of a row in
// flight together) or 0 (run time).
template <int P, int DIM>
__global__ void __launch_bounds__(BRS_WARPS * 32)
    bf_rescore_kernel(const float* __restrict__ Q, int nq, const float* __restrict__ X, int dim,
                      const float* __restrict__ qnorm, const float* __restrict__ xnorm,
                      float xmax, int metric,
                      uint64_t tag_base, const uint64_t* __restrict__ approx, int kp, int k,
                      const unsigned* __restrict__ cand_cnt, int cap,
                      const float* __restrict__ tau, uint64_t* __restrict__ out,
                      uint32_t* flag_count, uint32_t* flag_list) {
    __shared__ uint64_t buf[BRS_WARPS * 64];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * BRS_WARPS + warp;
    if (q >= nq) return;
    const float* qv = Q + (size_t)q * dim;
    const uint64_t* ak = approx + (size_t)q * kp;
    WarpTopK<P> tk;
    tk.init(k, buf + warp * 64);
    const bool l2 = metric == EUCLIDEAN || metric == EUCLIDEAN_SQUARED;  // rank by L2^2
    {
        // two rows per lane, interleaved: twice the loads in flight per round
        // (cosine takes each row's squared norm from xnorm, computed in the
        // same order as the dot product it would otherwise repeat)
        const bool vec = (dim & 3) == 0;
        for (int base = 0; base < kp; base += 64) {
            const int i0 = base + lane, i1 = base + 32 + lane;
            const uint64_t k0 = i0 < kp ? ak[i0] : KEY_NONE, k1 = i1 < kp ? ak[i1] : KEY_NONE;
            const bool h0 = k0 != KEY_NONE, h1 = k1 != KEY_NONE;
            // a missing entry repeats a present row (its result is discarded)
            const uint32_t t0 = h0 ? key_tag(k0) : (h1 ? key_tag(k1) : (uint32_t)tag_base);
            const uint32_t t1 = h1 ? key_tag(k1) : t0;
            const float* rows[2] = {X + (size_t)(t0 - tag_base) * dim,
                                    X + (size_t)(t1 - tag_base) * dim};
            float d[2];
            if (l2) {
                l2sq_rows<2, DIM>(qv, rows, dim, vec, d);
            } else {
                dot_rows<2, DIM>(qv, rows, dim, d);
                if (metric == DOT_PRODUCT) {
                    d[0] = -d[0];
                    d[1] = -d[1];
                } else {
                    d[0] = cosine_from(d[0], qnorm[q], xnorm[t0 - tag_base]);
                    d[1] = cosine_from(d[1], qnorm[q], xnorm[t1 - tag_base]);
                }
            }
            const uint64_t e0 = h0 ? make_key(d[0], t0) : KEY_NONE;
            const uint64_t e1 = h1 ? make_key(d[1], t1) : KEY_NONE;
            if (__any_sync(0xffffffffu, h0)) tk.merge32(e0);
            if (__any_sync(0xffffffffu, h1)) tk.merge32(e1);
        }
    }
    const double qn = (double)qnorm[q];
    const double qlen = sqrt(qn);
    const double xm = (double)xmax;
    double E;
    if (l2) E = 2.5e-3 * qlen * xm + 1e-5 * (qn + xm * xm);
    else if (metric == DOT_PRODUCT) E = 1.25e-3 * qlen * xm;
    else E = 1.25e-3 + 1e-5;
    const unsigned c = cand_cnt[q];
    double B;
    if (c >= (unsigned)kp) B = (double)key_dist(ak[kp - 1]);
    else B = (double)tau[q];  // +inf when the sample saw fewer than 32 rows
    bool cert = c <= (unsigned)cap;
    if (cert && !isinf(B)) cert = tk.thr != KEY_NONE && ((double)key_dist(tk.thr) + E < B);
    if (cert && isinf(B) && c < (unsigned)k) cert = true;  // every row was a candidate
    if (metric == EUCLIDEAN) {
#pragma unroll
        for (int e = 0; e < P; ++e)
            if (tk.L[e] != KEY_NONE)
                tk.L[e] = make_key(__fsqrt_rn(key_dist(tk.L[e])), key_tag(tk.L[e]));
    }
    tk.store(out + (size_t)q * k);
    if (!cert && lane == 0) {
        const uint32_t idx = atomicAdd(flag_count, 1u);
        flag_list[idx] = (uint32_t)q;
    }
}

void launch_bf_rescore(cudaStream_t s, const float* Q, int nq, const float* X, int dim,
                       const float* qnorm, const float* xnorm, float xmax, int metric,
                       uint64_t tag_base, const GemmScratch& w, int kp, int k, uint64_t* out,
                       uint32_t* flag_count, uint32_t* flag_list) {
    if (nq == 0) return;
    unsigned grid = (unsigned)((nq + BRS_WARPS - 1) / BRS_WARPS);
#define FDB_BRS(PP)                                                                           \
    do {                                                                                     \
        if (dim == 128)                                                                      \
            bf_rescore_kernel<PP, 128><<<grid, BRS_WARPS * 32, 0, s>>>(                      \
                Q, nq, X, dim, qnorm, xnorm, xmax, metric, tag_base, w.approx.p, kp, k,          \
                w.cand_cnt.p,                                                                 \
                w.cap, w.tau.p, out, flag_count, flag_list);                                 \
        else                                                                                 \
            bf_rescore_kernel<PP, 0><<<grid, BRS_WARPS * 32, 0, s>>>(                        \
                Q, nq, X, dim, qnorm, xnorm, xmax, metric, tag_base, w.approx.p, kp, k,          \
                w.cand_cnt.p,                                                                 \
                w.cap, w.tau.p, out, flag_count, flag_list);                                 \
    } while (0)
    if (k <= 32) FDB_BRS(1);
    else if (k <= 64) FDB_BRS(2);
    else if (k <= 128) FDB_BRS(4);
    else FDB_BRS(8);
#undef FDB_BRS
    FDB_LAUNCH_CHECK();
}

}  // namespace fdb
