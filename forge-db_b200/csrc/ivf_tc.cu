// ivf_tc.cu -- tensor-core (tcgen05) scan of IVF-PQ inverted lists.
//
// A batch search probes `take` lists per query.  The (query, list) pairs are
// grouped by list.  For list l, the residual queries r = fl(q - c_l) (one
// fp16 row per pair, scaled by a power of two) are multiplied on the tensor
// cores with the list's decoded codes rhat = [b_{0,code_0} .. b_{m-1,code_m-1}]
// (fp16, decoded once per index), and every score becomes
//     d~ = ||r||^2 + ||rhat||^2 - 2 <r, rhat>
// with ||r||^2 the exact coarse distance and ||rhat||^2 precomputed per code:
// the reference's ADC distance (ivf_pq.rs:1005-1040, pq.rs:435-485) as a real
// number, with different rounding.  Two passes, as in the brute-force
// shortlist:
//   pass 1: each query's first probed list holding 64+ codes (else its first
//     non-empty one).  Every pair row keeps its top-64 in shared memory; the
//     64th distance is the query's admission threshold tau.
//   pass 2: the other probed lists.  A score costs one FMA and a compare;
//     scores <= tau are appended to a per-query candidate array.
// The top-64 of (pass-1 list + candidates) are rescored with the reference's
// exact LUT sums (bit for bit, in the requested order) and certified against
// a worst-case bound of the fp16/fp32 rounding (see certify_kernel); queries
// that fail are re-scanned exactly by the caller.
//
// Decoded codes live in a padded copy of the list layout in which every list
// starts on a 128-row boundary, so a B tile never mixes two lists and the
// tile's ||rhat||^2 values (512 bytes, aligned) are staged into shared memory
// by a bulk copy next to the tile itself.
//
// Work is split into items (one list x up to 128 pair rows), ordered by
// decreasing list length.  A persistent grid of one CTA per SM takes them
// from an atomic counter (longest first, so the tail is short; concurrent
// CTAs on one list's items share its codes in L2); the next item's A tile
// loads while the current item finishes.  Warp roles as in the brute-force
// kernel: warp 0 = TMA producer, warp 1 = MMA issuer and TMEM owner, warps
// 4.. = epilogue; every mbarrier wait is bounded and an abort drains the
// in-flight copies and MMAs before TMEM is freed.
#include <cub/cub.cuh>
#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>
#include <numeric>

#include "fdb_device.cuh"
#include "fdb_internal.h"
#include "fdb_kernels.h"
#include "tc_ptx.cuh"

namespace fdb {
namespace ivtc {
using namespace tc;

constexpr int THREADS = 640;
constexpr int EPI_WARP0 = 4;
constexpr int LIST_K = 64;  // pass-1 list per query = shortlist length
constexpr int EPI_DUMP = 0, EPI_FILTER = 1;
constexpr int CV_FLOATS = TILE_N;  // ||rhat||^2 values per B tile
#ifndef FDB_IVF_CHUNK_TILES
#define FDB_IVF_CHUNK_TILES 8
#endif
#ifndef FDB_IVF_SPIN_WAITS
#define FDB_IVF_SPIN_WAITS 1
#endif
constexpr int CHUNK_TILES = FDB_IVF_CHUNK_TILES;  // B tiles per item at most (long lists are split)

constexpr float INF = __builtin_huge_valf();

struct Item {
    uint32_t a0;    // first pair row of the A tile
    uint32_t na;    // pair rows in use (1..128)
    uint32_t b0;    // first row of this chunk of the list in the padded decoded layout
    uint32_t nb;    // codes in this chunk (>= 1)
    uint32_t tag0;  // row of the chunk's first code in the index (key tag)
    uint32_t col0;  // index of the chunk's first code within its list
    uint32_t pad[2];
};

struct PassParams {
    const Item* items;
    const uint32_t* range;   // device-side {first item, item count} of this pass
    unsigned* next;          // item counter of this pass, preset to 0
    int katoms;
    const uint32_t* pair_q;  // [pairs] query of each pair row
    const float* pair_rn;    // [pairs] ||q - c_l||^2 (the exact coarse distance)
    const float* pair_s2;    // [pairs] -2 * 2^-(sa + sb): undoes both fp16 scalings
    const float* colv;       // padded layout: ||rhat||^2, +inf in padding rows
    float colmax;            // largest ||rhat||^2
    float* dump;             // pass 1: every distance of each pair's list
    uint32_t* lo;            // pass 1: [nq] smallest finite distance (orderable bits), preset ~0
    uint32_t* hi;            // pass 1: [nq] ~(largest finite distance, orderable bits), preset ~0
    const unsigned* seg;     // pass 1: [pairs] offset of the pair's row in dump
    const float* tau;        // pass 2: [nq] admission threshold
    uint64_t* cand;          // pass 2: [nq][cap] candidate keys
    unsigned* cand_cnt;      // pass 2: [nq] candidates seen (may exceed cap)
    int cap;
    int* err;
    unsigned long long wait;  // limit of each bounded wait, SM clock cycles
    int stall;                // test hook: issue nothing (the waits run out)
};

#ifndef FDB_IVF_NSTAGE
#define FDB_IVF_NSTAGE 4
#endif
#ifndef FDB_IVF_ASLOTS
#define FDB_IVF_ASLOTS 2
#endif
constexpr int NSTAGE = FDB_IVF_NSTAGE;  // B tile stages
constexpr int ASLOTS = FDB_IVF_ASLOTS;  // A tile slots (2: the next item's A loads early)
constexpr int NEPI = 16;   // epilogue warps: 4 TMEM lane quadrants x 4 column chunks
constexpr int NCV = NSTAGE; // ||rhat||^2 stages (one per B stage)
constexpr int NACC = 4;    // TMEM accumulators (128 columns each: all 512 columns)


// 32 consecutive floats of a shared buffer (warp-uniform address: broadcast).
__device__ __forceinline__ void load32(const float* src, float (&cv)[32]) {
    const float4* s4 = reinterpret_cast<const float4*>(src);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 t = s4[i];
        cv[4 * i] = t.x;
        cv[4 * i + 1] = t.y;
        cv[4 * i + 2] = t.z;
        cv[4 * i + 3] = t.w;
    }
}

// Waits of the single-thread roles (TMA producer, MMA issuer): polling by
// default, since their wake-up latency is on the pipeline's critical path.
__device__ __forceinline__ bool role_wait(uint64_t* bar, uint32_t parity, int* err,
                                          unsigned long long limit) {
#if FDB_IVF_SPIN_WAITS
    return mbar_wait_spin(bar, parity, err, limit);
#else
    return mbar_wait(bar, parity, err, limit);
#endif
}

#ifndef FDB_IVF_EPI_SPIN
#define FDB_IVF_EPI_SPIN 0
#endif
// Bounded wait of one lane, verdict shared with the warp.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* err,
                                          unsigned long long limit, int lane) {
    int got = 0;
#if FDB_IVF_EPI_SPIN
    if (lane == 0) got = mbar_wait_spin(bar, parity, err, limit) ? 1 : 0;
#else
    if (lane == 0) got = mbar_wait(bar, parity, err, limit) ? 1 : 0;
#endif
    return __shfl_sync(0xffffffffu, got, 0) != 0;
}

template <int EPI>
__global__ void __launch_bounds__(THREADS, 1)
    ivf_pass_kernel(const __grid_constant__ CUtensorMap amap,
                    const __grid_constant__ CUtensorMap bmap, PassParams p) {
    constexpr int NS = NSTAGE;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    const uint32_t base = smem_u32(smem_raw);
    unsigned char* smem = smem_raw + ((1024 - (base & 1023)) & 1023);  // 1024-byte aligned
    const int KA = p.katoms;
    const uint32_t stage_bytes = (uint32_t)(KA * ATOM_BYTES);
    unsigned char* a_tile = smem;                                // ASLOTS slots of KA atoms
    unsigned char* b_tile = a_tile + ASLOTS * KA * ATOM_BYTES;   // NS stages of KA atoms
    float* cvbuf = reinterpret_cast<float*>(b_tile + NS * KA * ATOM_BYTES);
    uint64_t* bars = reinterpret_cast<uint64_t*>(cvbuf + NCV * CV_FLOATS);
    uint64_t* a_full = bars;               // [ASLOTS]
    uint64_t* a_empty = bars + ASLOTS;     // [ASLOTS]
    uint64_t* b_full = bars + 2 * ASLOTS;  // [NS]
    uint64_t* b_empty = b_full + NS;       // [NS]
    uint64_t* t_full = b_empty + NS;       // [NACC]
    uint64_t* t_empty = t_full + NACC;     // [NACC]
    uint64_t* cv_full = t_empty + NACC;    // [NCV]
    uint64_t* cv_empty = cv_full + NCV;    // [NCV]
    uint64_t* it_full = cv_empty + NCV;    // [2] item ring
    uint64_t* it_empty = it_full + 2;      // [2]
    int* ring = reinterpret_cast<int*>(it_empty + 2);        // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ring + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const Item* items = p.items + p.range[0];
    const int nitems = (int)p.range[1];

    if (threadIdx.x == 0) {
        for (int i = 0; i < ASLOTS; ++i) {
            mbar_init(a_full + i, 1);
            mbar_init(a_empty + i, 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(it_full + i, 1);
            mbar_init(it_empty + i, 1 + NEPI);
        }
        for (int i = 0; i < NS; ++i) {
            mbar_init(b_full + i, 1);
            mbar_init(b_empty + i, 1);
        }
        for (int i = 0; i < NACC; ++i) {
            mbar_init(t_full + i, 1);
            mbar_init(t_empty + i, NEPI);
        }
        for (int i = 0; i < NCV; ++i) {
            mbar_init(cv_full + i, 1);
            mbar_init(cv_empty + i, NEPI);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_slot)),
                     "r"(NACC * TILE_N));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
        tc_fence_before();
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // Last asynchronous operation each role issued, so that an aborting
    // block can wait for it (bounded) before it frees TMEM and exits.
    int last_use[NS], last_cv[NCV];
#pragma unroll
    for (int i = 0; i < NS; ++i) last_use[i] = -1;
#pragma unroll
    for (int i = 0; i < NCV; ++i) last_cv[i] = -1;
    int last_a[2] = {-1, -1};  // producer: last item whose A tile was requested, per A slot
    int last_g = -1;  // MMA issuer: last tile committed

    if (warp == 0) {
        // ---------------- TMA producer ----------------
        // (p.stall, a test hook: the ring stays empty and nothing is copied,
        // so the other roles wait on it_full until their limit runs out)
        if (lane == 0 && !p.stall) {
            // Items are taken from the pass's counter (largest first, as they
            // are ordered) and handed to the other roles through a 2-slot ring.
            int g = 0;
            bool ok = true;
            for (int r = 0; ok; ++r) {
                const int slot = r & 1;
                if (r >= 2 && !role_wait(it_empty + slot, ((r >> 1) - 1) & 1, p.err, p.wait))
                    break;
                const int idx = (int)atomicAdd(p.next, 1u);
                ring[slot] = idx;
                mbar_arrive(it_full + slot);
                if (idx >= nitems) break;
                const Item it = items[idx];
                const int as = r % ASLOTS, au = r / ASLOTS;
                if (r >= ASLOTS && !role_wait(a_empty + as, (au - 1) & 1, p.err, p.wait)) break;
                mbar_expect_tx(a_full + as, stage_bytes);
                for (int a = 0; a < KA; ++a)
                    tma_load_2d(a_tile + (as * KA + a) * ATOM_BYTES, &amap, a_full + as,
                                a * KATOM, (int)it.a0);
                last_a[as] = r;
                const int nt = (int)((it.nb + TILE_N - 1) / TILE_N);
                for (int t = 0; t < nt; ++t, ++g) {
                    const int s = g % NS, use = g / NS;
                    if (g >= NS && !role_wait(b_empty + s, (use - 1) & 1, p.err, p.wait)) {
                        ok = false;
                        break;
                    }
                    const uint32_t row = it.b0 + (uint32_t)t * TILE_N;
                    mbar_expect_tx(b_full + s, stage_bytes);
                    unsigned char* dst = b_tile + s * KA * ATOM_BYTES;
                    for (int a = 0; a < KA; ++a)
                        tma_load_2d(dst + a * ATOM_BYTES, &bmap, b_full + s, a * KATOM, (int)row);
#pragma unroll
                    for (int i = 0; i < NS; ++i)
                        if (i == s) last_use[i] = use;
                    const int c = g % NCV, cu = g / NCV;
                    if (g >= NCV && !role_wait(cv_empty + c, (cu - 1) & 1, p.err, p.wait)) {
                        ok = false;
                        break;
                    }
                    mbar_expect_tx(cv_full + c, CV_FLOATS * 4);
                    bulk_load(cvbuf + c * CV_FLOATS, p.colv + row, CV_FLOATS * 4, cv_full + c);
#pragma unroll
                    for (int i = 0; i < NCV; ++i)
                        if (i == c) last_cv[i] = cu;
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            int g = 0;
            bool ok = true;
            for (int r = 0; ok; ++r) {
                const int slot = r & 1;
                if (!role_wait(it_full + slot, (r >> 1) & 1, p.err, p.wait)) break;
                const int idx = *(volatile int*)(ring + slot);
                mbar_arrive(it_empty + slot);
                if (idx >= nitems) break;
                const Item it = items[idx];
                const int nt = (int)((it.nb + TILE_N - 1) / TILE_N);
                const int as = r % ASLOTS;
                if (!role_wait(a_full + as, (r / ASLOTS) & 1, p.err, p.wait)) break;
                tc_fence_after();
                for (int t = 0; t < nt; ++t, ++g) {
                    const int s = g % NS, use = g / NS, b = g % NACC;
                    if (g >= NACC &&
                        !role_wait(t_empty + b, ((g / NACC) - 1) & 1, p.err, p.wait)) {
                        ok = false;
                        break;
                    }
                    if (!role_wait(b_full + s, use & 1, p.err, p.wait)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t d = tmem + (uint32_t)(b * TILE_N);
                    const uint32_t abase = smem_u32(a_tile + as * KA * ATOM_BYTES);
                    const uint32_t bbase = smem_u32(b_tile + s * KA * ATOM_BYTES);
                    for (int a = 0; a < KA; ++a) {
#pragma unroll
                        for (int kk = 0; kk < 4; ++kk) {  // 4 x K16 per 64-wide atom
                            const uint32_t off = (uint32_t)(a * ATOM_BYTES + kk * 32);
                            umma_f16(d, smem_desc_sw128(abase + off),
                                     smem_desc_sw128(bbase + off), (a | kk) != 0);
                        }
                    }
                    umma_commit(b_empty + s);  // stage s may be refilled once these finish
                    umma_commit(t_full + b);   // accumulator b is ready for the epilogue
                    last_g = g;
                }
                if (ok) umma_commit(a_empty + as);  // the A slot may be refilled
            }
        }
    } else if (warp >= EPI_WARP0 && warp < EPI_WARP0 + NEPI) {
        // ---------------- epilogue ----------------
        const int w = warp - EPI_WARP0;
        const int quad = w & 3;  // TMEM lane quadrant = warp % 4
        const int part = w >> 2;  // 32-column chunk of each tile
        const int e = quad * 32 + lane;  // pair row within the tile
        const uint32_t lane_base = (uint32_t)(quad * 32) << 16;
        int g = 0;
        bool alive = true;
        for (int r = 0; alive; ++r) {
            const int slot = r & 1;
            if (!warp_wait(it_full + slot, (r >> 1) & 1, p.err, p.wait, lane)) break;
            // lane 0 performed the acquiring wait: it reads the slot for the warp
            int idx = 0;
            if (lane == 0) {
                idx = *(volatile int*)(ring + slot);
                mbar_arrive(it_empty + slot);
            }
            idx = __shfl_sync(0xffffffffu, idx, 0);
            if (idx >= nitems) break;
            const Item it = items[idx];
            const int nt = (int)((it.nb + TILE_N - 1) / TILE_N);
            if (quad * 32 >= (int)it.na) {
                // no pair row in this warp's TMEM quadrant: keep the barrier
                // phases in step (wait for each tile, release it) and skip
                // the loads and the scoring
                for (int t = 0; t < nt; ++t, ++g) {
                    const int b = g % NACC, c = g % NCV;
                    if (!warp_wait(t_full + b, (g / NACC) & 1, p.err, p.wait, lane) ||
                        !warp_wait(cv_full + c, (g / NCV) & 1, p.err, p.wait, lane)) {
                        alive = false;
                        break;
                    }
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(t_empty + b);
                        mbar_arrive(cv_empty + c);
                    }
                }
                continue;
            }
            const bool rok = e < (int)it.na;
            const uint32_t pr = it.a0 + (uint32_t)e;
            const int q = rok ? (int)p.pair_q[pr] : 0;
            const float rn = rok ? p.pair_rn[pr] : 0.0f;
            const float s2 = rok ? p.pair_s2[pr] : 0.0f;
            // Each of the item's tiles: this warp's 32-column chunk is loaded from
            // TMEM and scored against the staged ||rhat||^2 values.  Sixteen
            // epilogue warps (four per lane quadrant) hide one another's load
            // and append latencies; a warp pipelining two chunks itself with
            // half as many warps ran pass 2 of config D 1.6x slower.
            uint32_t va[32];
            auto begin_tile = [&](int gg) -> bool {
                const int b = gg % NACC, c = gg % NCV;
                if (!warp_wait(t_full + b, (gg / NACC) & 1, p.err, p.wait, lane) ||
                    !warp_wait(cv_full + c, (gg / NCV) & 1, p.err, p.wait, lane))
                    return false;
                tc_fence_after();
                tmem_ld32_nowait(tmem + lane_base + (uint32_t)(b * TILE_N + part * 32), va);
                return true;
            };
            if constexpr (EPI == EPI_FILTER) {
                const float tau = rok ? p.tau[q] : -INF;
                // Admission test fma(s2, s, ||rhat||^2) <= (tau - rn) + slack: the
                // slack covers the different rounding of the rearranged sum, so
                // every code with d~ <= tau passes; hits are re-checked with d~.
                const float tt =
                    rok ? (tau - rn) + ldexpf(2.0f * fabsf(rn) + 2.0f * p.colmax + fabsf(tau), -20)
                        : -INF;
                const uint64_t s22 = pack2(__float_as_uint(s2), __float_as_uint(s2));
                // The test of a 32-column chunk: bit g is set when some row of the
                // warp may admit a code among the chunk's columns 8g..8g+7.  Each
                // group's smallest test value comes from a short tree of minimums;
                // one vote skips the chunk when no lane can have a hit.
                auto test = [&](const uint32_t(&v)[32], const float* cvs) -> unsigned {
                    float x[32];
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        // fma.rn.f32x2: two independent fmaf_rn per instruction
                        const ulonglong2 cc = reinterpret_cast<const ulonglong2*>(cvs)[i];
                        const uint64_t x01 = fma2(s22, pack2(v[4 * i], v[4 * i + 1]), cc.x);
                        const uint64_t x23 = fma2(s22, pack2(v[4 * i + 2], v[4 * i + 3]), cc.y);
                        x[4 * i] = __uint_as_float((uint32_t)x01);
                        x[4 * i + 1] = __uint_as_float((uint32_t)(x01 >> 32));
                        x[4 * i + 2] = __uint_as_float((uint32_t)x23);
                        x[4 * i + 3] = __uint_as_float((uint32_t)(x23 >> 32));
                    }
                    float m[4];
#pragma unroll
                    for (int g8 = 0; g8 < 4; ++g8) {
                        const float* y = x + 8 * g8;
                        m[g8] = min3f(min3f(y[0], y[1], y[2]), min3f(y[3], y[4], y[5]),
                                      fminf(y[6], y[7]));
                    }
                    const float mn = fminf(fminf(m[0], m[1]), fminf(m[2], m[3]));
                    if (!__any_sync(0xffffffffu, mn <= tt)) return 0u;
                    unsigned gm = 0;
#pragma unroll
                    for (int g8 = 0; g8 < 4; ++g8)
                        gm |= __any_sync(0xffffffffu, m[g8] <= tt) ? 1u << g8 : 0u;
                    return gm;
                };
                // The groups of gm (bits 0-3: this warp's first 32 columns of the
                // tile, 4-7: the next 32) reloaded from the accumulator, which is
                // still held: every code with d~ <= tau (+inf: a tombstoned row,
                // never admitted) is appended to its query's candidates.  One copy
                // of this code serves both chunks, which keeps the loop small.
                auto admit = [&](unsigned gm, uint32_t tcol, const float* cvs, int cbase) {
                    // (bit g: columns 8g..8g+7 of this warp's chunk)
                    const uint32_t tag = it.tag0 + (uint32_t)cbase;
                    const int nvalid = (int)it.nb - cbase;
                    uint64_t* crow = p.cand + (size_t)q * p.cap;
                    while (gm) {
                        const int gi = __ffs(gm) - 1;
                        gm &= gm - 1;
                        uint32_t w[8];
                        tmem_ld8(tmem + lane_base + tcol + (uint32_t)(gi * 8), w);
                        // the row's hits in the group, reserved with one atomic
                        float d[8];
                        unsigned hm = 0;
#pragma unroll
                        for (int jj = 0; jj < 8; ++jj) {
                            const int j = gi * 8 + jj;
                            d[jj] = __fmaf_rn(s2, __uint_as_float(w[jj]), __fadd_rn(rn, cvs[j]));
                            if (rok && j < nvalid && d[jj] <= tau && d[jj] < INF) hm |= 1u << jj;
                        }
                        if (hm == 0) continue;
                        unsigned ix = atomicAdd(p.cand_cnt + q, (unsigned)__popc(hm));
#pragma unroll
                        for (int jj = 0; jj < 8; ++jj)
                            if (hm >> jj & 1u) {
                                if (ix < (unsigned)p.cap)
                                    crow[ix] = make_key(d[jj], tag + (uint32_t)(gi * 8 + jj));
                                ++ix;
                            }
                    }
                };
                for (int t = 0; t < nt; ++t, ++g) {
                    if (!begin_tile(g)) {
                        alive = false;
                        break;
                    }
                    const int b = g % NACC, c = g % NCV;
                    const float* cvs = cvbuf + c * CV_FLOATS + part * 32;
                    const uint32_t tcol = (uint32_t)(b * TILE_N + part * 32);
                    tmem_wait_regs(va);
                    const unsigned gm = test(va, cvs);
                    if (gm) admit(gm, tcol, cvs, t * TILE_N + part * 32);
                    // done with the accumulator and the staged norms
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(t_empty + b);
                        mbar_arrive(cv_empty + c);
                    }
                }
            } else {
                // pass 1: every distance of the row's list goes to its dump row;
                // padding columns carry ||rhat||^2 = +inf and store +inf
                float* drow = rok ? p.dump + p.seg[pr] + it.col0 : nullptr;
                const uint64_t s22 = pack2(__float_as_uint(s2), __float_as_uint(s2));
                const uint64_t rn2 = pack2(__float_as_uint(rn), __float_as_uint(rn));
                // The chunk's finite distances also update the query's range
                // (select1_kernel's histogram bounds), so that kernel need not
                // read the dump a third time; +inf (padding, tombstones) and
                // NaN are left out, as there.
                auto dump = [&](const uint32_t(&v)[32], const float* cvs, int col) {
                    if (!rok) return;
                    ulonglong2* dst = reinterpret_cast<ulonglong2*>(drow + col);
                    float mn = INF, mx = -INF;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        // fmaf_rn(s2, v, rn + ||rhat||^2), two per instruction
                        const ulonglong2 cc = reinterpret_cast<const ulonglong2*>(cvs)[i];
                        ulonglong2 o;
                        o.x = fma2(s22, pack2(v[4 * i], v[4 * i + 1]), add2(rn2, cc.x));
                        o.y = fma2(s22, pack2(v[4 * i + 2], v[4 * i + 3]), add2(rn2, cc.y));
                        dst[i] = o;
                        const float y[4] = {__uint_as_float((uint32_t)o.x),
                                            __uint_as_float((uint32_t)(o.x >> 32)),
                                            __uint_as_float((uint32_t)o.y),
                                            __uint_as_float((uint32_t)(o.y >> 32))};
#pragma unroll
                        for (int x = 0; x < 4; ++x)
                            if (y[x] < INF) {  // finite (NaN compares false)
                                mn = fminf(mn, y[x]);
                                mx = fmaxf(mx, y[x]);
                            }
                    }
                    if (mn < INF) {
                        atomicMin(p.lo + q, f2ord(mn));
                        atomicMin(p.hi + q, ~f2ord(mx));
                    }
                };
                for (int t = 0; t < nt; ++t, ++g) {
                    if (!begin_tile(g)) {
                        alive = false;
                        break;
                    }
                    const int b = g % NACC, c = g % NCV;
                    const float* cvs = cvbuf + c * CV_FLOATS + part * 32;
                    tmem_wait_regs(va);
                    dump(va, cvs, t * TILE_N + part * 32);
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) {
                        mbar_arrive(t_empty + b);
                        mbar_arrive(cv_empty + c);
                    }
                }
            }
        }
    }
    // One verdict for the whole block (another block may set the word while
    // this block's threads read it; the barrier inside must not diverge).
    if (__syncthreads_or(*(volatile int*)p.err != 0)) {
        // aborting: let the copies and MMAs this block issued land before exit
        // (waits on phases that already completed return at once)
        if (warp == 0 && lane == 0) {
            for (int s2 = 0; s2 < NS; ++s2)
                if (last_use[s2] >= 0) {
                    const unsigned long long t0 = clock64();
                    while (!mbar_try(b_full + s2, last_use[s2] & 1) &&
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
            for (int sl = 0; sl < ASLOTS; ++sl)
                if (last_a[sl] >= 0) {
                    const unsigned long long t0 = clock64();
                    while (!mbar_try(a_full + sl, (last_a[sl] / ASLOTS) & 1) &&
                           clock64() - t0 < WAIT_CYCLES) {
                    }
                }
        }
        if (warp == 1 && lane == 0 && last_g >= 0) {
            const unsigned long long t0 = clock64();
            while (!mbar_try(t_full + (last_g % NACC), (last_g / NACC) & 1) &&
                   clock64() - t0 < WAIT_CYCLES) {
            }
        }
        __syncthreads();
    }
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(NACC * TILE_N));
    }
}

// ---------------------------------------------------------------------------
// pair grouping
// ---------------------------------------------------------------------------
// Sort key of probe (q, p): its list for the query's pass-1 probe (the first
// holding LIST_K+ codes in the unsharded index, else the first non-empty
// one), nlist + list for the query's other probes, 2 nlist for lists that are
// empty or held by another device.  When stat is
// given, also counts the lists and codes scanned, and the codes of pass 2.
// sample_div: pass 1 samples the nearest other probes' first tiles until it
// has seen 1/sample_div of the query's probed codes (0: every probe's first
// tile).
__global__ void pair_keys_kernel(const uint32_t* __restrict__ probes, int nq, int take,
                                 const uint64_t* __restrict__ lbeg,
                                 const uint64_t* __restrict__ lend,
                                 const uint64_t* __restrict__ offs_full, int nlist,
                                 uint64_t sample_div, uint32_t* __restrict__ keys,
                                 uint32_t* __restrict__ vals, unsigned long long* stat) {
    // one warp per query, lanes over its probes (32 at a time, in order)
    const int q = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (q >= nq) return;  // whole warp
    const uint32_t* pq = probes + (size_t)q * take;
    // the pass-1 list: the first probe whose list holds >= 64 codes in the
    // unsharded index (so that on a sharded index exactly one device holds
    // it), else the first non-empty one
    int p1 = -1, pf = -1;
    uint64_t total = 0;
    for (int j0 = 0; j0 < take; j0 += 32) {
        const int j = j0 + lane;
        uint64_t full = 0, len = 0;
        if (j < take) {
            const uint32_t l = pq[j];
            full = offs_full[l + 1] - offs_full[l];
            len = lend[l] - lbeg[l];
        }
        total += len;
        const unsigned big = __ballot_sync(0xffffffffu, full >= (uint64_t)LIST_K);
        const unsigned nz = __ballot_sync(0xffffffffu, full > 0);
        if (p1 < 0 && big) p1 = j0 + __ffs(big) - 1;
        if (pf < 0 && nz) pf = j0 + __ffs(nz) - 1;
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
    if (p1 < 0) p1 = pf;
    // pass 1 scores the pass-1 list and the first tiles of the nearest other
    // probes (probes are in ascending coarse distance) until it has seen
    // 1/sample_div of the query's codes (the admission threshold is the 64th
    // of what it saw, so pass 2 admits about 64 * sample_div codes); the
    // other probes' lists are left to pass 2 whole
    uint64_t seen = p1 >= 0 ? lend[pq[p1]] - lbeg[pq[p1]] : 0;
    unsigned long long lists = 0, codes = 0;
    for (int j0 = 0; j0 < take; j0 += 32) {
        const int j = j0 + lane;
        uint32_t l = 0;
        uint64_t len = 0;
        if (j < take) {
            l = pq[j];
            len = lend[l] - lbeg[l];
        }
        const bool other = j < take && len > 0 && j != p1;
        // seen before this probe: the carry plus the earlier lanes' tiles
        uint64_t c = other ? (len < (uint64_t)TILE_N ? len : (uint64_t)TILE_N) : 0;
        uint64_t incl = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint64_t y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        const uint64_t before = seen + incl - c;
        // (sampling stops at the first probe that finds the quota met, so a
        // probe is sampled exactly when the quota was not met before it)
        const bool smp = other && (sample_div == 0 || before * sample_div < total);
        if (j < take) {
            uint32_t key;
            if (len == 0) key = 3u * (uint32_t)nlist;
            else if (j == p1) key = l;
            else if (smp) key = (uint32_t)nlist + l;
            else key = 2u * (uint32_t)nlist + l;
            const size_t i = (size_t)q * take + j;
            keys[i] = key;
            vals[i] = (uint32_t)i;
            if (len > 0) {
                ++lists;
                codes += len;
            }
        }
        // carry: only sampled probes add to `seen` (as the serial rule)
        uint64_t add = smp ? c : 0;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) add += __shfl_xor_sync(0xffffffffu, add, o);
        seen += add;
    }
    if (stat) {
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
            lists += __shfl_xor_sync(0xffffffffu, lists, o);
            codes += __shfl_xor_sync(0xffffffffu, codes, o);
        }
        if (lane == 0) {
            atomicAdd(stat, lists);
            atomicAdd(stat + 1, codes);
        }
    }
}

// off[k] = the first position of key >= k in the sorted keys (k <= nkeys):
// the segment offsets of the stable sort, without a histogram.  Position i
// (0 <= i <= n) is that first position for every k in (keys[i-1], keys[i]]
// (keys[-1] = -1, keys[n] = nkeys), so a thread per position writes each
// offset exactly once.
__global__ void seg_offsets_kernel(const uint32_t* __restrict__ keys, unsigned n, int nkeys,
                                   unsigned* __restrict__ off) {
    const unsigned i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i > n) return;
    const uint32_t lo = i == 0 ? 0u : keys[i - 1] + 1u;
    const uint32_t hi = i == n ? (uint32_t)nkeys : keys[i];
    for (uint32_t k = lo; k <= hi; ++k) off[k] = i;
}

// One warp per sorted pair: the fp16 residual row r = fl(q - c_l) * 2^sa
// (sa puts the largest |r_i| in [2^14, 2^15)), the coarse distance and the
// combined scale -2 * 2^-(sa + sb).  Pairs whose scale leaves the float range
// mark their query for the exact path.
// One warp writes the fp16 residual row of probe v (query q, list l) at
// `row`: r = fl(q - c_l) scaled by 2^sa (largest |r_i| in [2^14, 2^15));
// returns the combined scale s2 = -2^(1 - sa - sb), or 0 with *bad set when
// the row cannot be represented (the query then takes the exact path).
__device__ __forceinline__ float write_a_row(const float* __restrict__ Q,
                                             const float* __restrict__ cents, int dim, int dpad,
                                             uint32_t q, uint32_t l, int sb,
                                             __half* __restrict__ row, bool* bad_out) {
    const int lane = threadIdx.x & 31;
    const float* qv = Q + (size_t)q * dim;
    const float* cv = cents + (size_t)l * dim;
    // lane holds components 4 lane .. 4 lane + 3 (dpad <= 128)
    const bool vec = dim == dpad && ((reinterpret_cast<uintptr_t>(qv) |
                                      reinterpret_cast<uintptr_t>(cv)) & 15) == 0;
    float r[4];
    float mx = 0.0f;
    if (vec) {
        r[0] = r[1] = r[2] = r[3] = 0.0f;
        if (4 * lane < dim) {
            const float4 a = *reinterpret_cast<const float4*>(qv + 4 * lane);
            const float4 c4 = *reinterpret_cast<const float4*>(cv + 4 * lane);
            r[0] = __fsub_rn(a.x, c4.x);
            r[1] = __fsub_rn(a.y, c4.y);
            r[2] = __fsub_rn(a.z, c4.z);
            r[3] = __fsub_rn(a.w, c4.w);
        }
    } else {
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int c = 4 * lane + t;
            r[t] = (c < dim) ? __fsub_rn(qv[c], cv[c]) : 0.0f;
        }
    }
#pragma unroll
    for (int t = 0; t < 4; ++t) mx = fmaxf(mx, fabsf(r[t]));
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    // exponent of the largest magnitude (subnormals count as 2^-127)
    const int ex = mx > 0.0f ? (int)((__float_as_uint(mx) >> 23) & 0xff) - 127 : 0;
    int sa = mx > 0.0f ? 14 - ex : 0;
    sa = max(-120, min(120, sa));
    const float scale = __uint_as_float((uint32_t)(sa + 127) << 23);  // 2^sa, exact
    const int se = 1 - sa - sb;  // s2 = -2^se
    const bool bad = !(mx <= 3.0e38f) || se < -125 || se > 126;
    if (4 * lane < dpad) {
        __half2 h[2];
        h[0] = __halves2half2(__float2half_rn(bad ? 0.0f : __fmul_rn(r[0], scale)),
                              __float2half_rn(bad ? 0.0f : __fmul_rn(r[1], scale)));
        h[1] = __halves2half2(__float2half_rn(bad ? 0.0f : __fmul_rn(r[2], scale)),
                              __float2half_rn(bad ? 0.0f : __fmul_rn(r[3], scale)));
        *reinterpret_cast<uint2*>(row + 4 * lane) = *reinterpret_cast<uint2*>(h);
    }
    *bad_out = bad;
    return bad ? 0.0f : -__uint_as_float((uint32_t)(se + 127) << 23);
}

// Every sorted pair i < poff[3 nlist] gets pair_q, pair_rn and inv (a thread
// each); the pairs pass 1 scores (i < poff[2 nlist]: pass-1 lists and sampled
// first tiles) also get their A row and pair_s2 (a warp each).  A grid of a
// few blocks per SM strides over both (the counts are known on the device
// only).  Pass-2 rows are written later for the pairs pruning keeps
// (build_a2_kernel).
__global__ void __launch_bounds__(256)
    build_a_kernel(const uint32_t* __restrict__ vals, const unsigned* __restrict__ poff,
                   int nlist, int take, const uint32_t* __restrict__ probes,
                   const float* __restrict__ Q, const float* __restrict__ cents, int dim,
                   int dpad, const float* __restrict__ pdist, int sb, __half* __restrict__ a16,
                   uint32_t* __restrict__ pair_q, float* __restrict__ pair_rn,
                   float* __restrict__ pair_s2, uint32_t* __restrict__ qbad,
                   uint32_t* __restrict__ inv) {
    const unsigned npairs = poff[3 * nlist];  // pairs with a non-empty list
    const unsigned n1 = poff[2 * nlist];      // pairs pass 1 scores
    const unsigned nthreads = gridDim.x * blockDim.x;
    const unsigned gt = blockIdx.x * blockDim.x + threadIdx.x;
    for (unsigned i = gt; i < npairs; i += nthreads) {
        const uint32_t v = vals[i];
        pair_q[i] = v / (uint32_t)take;
        pair_rn[i] = pdist[v];  // the exact coarse distance of this probe
        inv[v] = i;             // where probe v = q * take + j sits among the sorted pairs
    }
    const int lane = threadIdx.x & 31;
    for (unsigned i = gt >> 5; i < n1; i += nthreads >> 5) {  // warp-uniform
        const uint32_t v = vals[i];
        const uint32_t q = v / (uint32_t)take;
        bool bad = false;
        const float s2 = write_a_row(Q, cents, dim, dpad, q, probes[v], sb, a16 + (size_t)i * dpad,
                                     &bad);
        if (lane == 0) {
            pair_s2[i] = s2;
            if (bad) qbad[q] = 1u;
        }
    }
}

// One warp per kept pass-2 pair j (sel[j] = its sorted index): its row of
// the compact pass-2 matrix and per-pair values.
// (a grid of a few blocks per SM strides over the kept pairs)
__global__ void __launch_bounds__(256)
    build_a2_kernel(const unsigned* __restrict__ sel, const unsigned* __restrict__ nsel,
                    const uint32_t* __restrict__ vals, int take,
                    const uint32_t* __restrict__ probes, const float* __restrict__ Q,
                    const float* __restrict__ cents, int dim, int dpad,
                    const float* __restrict__ pdist, int sb, __half* __restrict__ a2,
                    uint32_t* __restrict__ q2, float* __restrict__ rn2,
                    float* __restrict__ s22, uint32_t* __restrict__ qbad) {
    const int lane = threadIdx.x & 31;
    const unsigned n = *nsel;
    const unsigned nwarps = (gridDim.x * blockDim.x) >> 5;
    for (unsigned j = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; j < n; j += nwarps) {
        const uint32_t v = vals[sel[j]];
        const uint32_t q = v / (uint32_t)take;
        bool bad = false;
        const float s2 =
            write_a_row(Q, cents, dim, dpad, q, probes[v], sb, a2 + (size_t)j * dpad, &bad);
        if (lane == 0) {
            q2[j] = q;
            rn2[j] = pdist[v];
            s22[j] = s2;
            if (bad) qbad[q] = 1u;
        }
    }
}

// plen[i] = the length of pair i's dump row: its whole list (padded to whole
// tiles) for a pass-1 pair, the list's first tile for the others, 0 past the
// pairs; an exclusive sum turns it into the row's offset in the dump.
__global__ void plen_kernel(const uint32_t* __restrict__ vals, const unsigned* __restrict__ poff,
                            int nlist, const uint32_t* __restrict__ probes,
                            const uint64_t* __restrict__ lbeg, const uint64_t* __restrict__ lend,
                            int n, unsigned* __restrict__ plen) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    unsigned len = 0;
    if ((unsigned)i < poff[2 * nlist]) {
        const uint32_t l = probes[vals[i]];
        len = (unsigned)i < poff[nlist]
                  ? (unsigned)((lend[l] - lbeg[l] + TILE_N - 1) / TILE_N * TILE_N)
                  : (unsigned)TILE_N;
    }
    plen[i] = len;
}

// Items of both passes, lists in `lorder`.  An item is (list, up to 128
// pair rows, a run of at most CHUNK_TILES tiles of the list).  Pass 1 (dump)
// holds the pass-1 segments' whole lists and the pass-2 segments' first
// tiles; pass 2 (filter) holds the pass-2 segments' other tiles.  Slot
// s = kind * nlist + i describes list lorder[i] for kind 0 (pass-1 segment,
// whole list), 1 (pass-2 segment, first tile) or 2 (pass-2 segment, tiles
// 1..).  item_count_kernel counts each slot's items, an exclusive sum places
// them, item_fill_kernel writes them (one warp per slot): items[0 .. n1) are
// pass 1, items[n1 .. n1 + n2) pass 2; range = {0, n1, n1, n2}.
struct ItemSlot {
    unsigned a0, cnt, c_lo, c_hi, nchunk;
    uint32_t l;
};

// poff2 (nullable): for kind 2, the live pass-2 pairs' offsets per list
// ([nlist + 1], rows of the compacted pass-2 matrix) instead of poff's.
__device__ __forceinline__ ItemSlot item_slot(int s, const unsigned* __restrict__ poff,
                                              const unsigned* __restrict__ poff2, int nlist,
                                              const uint32_t* __restrict__ lorder,
                                              const uint64_t* __restrict__ lbeg,
                                              const uint64_t* __restrict__ lend) {
    const int kind = s / nlist, i = s - kind * nlist;
    const int seg = kind == 0 ? 0 : 1;
    ItemSlot t;
    t.l = lorder[i];
    if (kind >= 2) {
        // kept pass-2 pairs: sampled (kind 2) then unsampled (kind 3) rows
        const unsigned* o = poff2 + (kind - 2) * nlist;
        t.a0 = o[t.l];
        t.cnt = o[t.l + 1] - t.a0;
    } else {
        t.a0 = poff[seg * nlist + t.l];
        t.cnt = poff[seg * nlist + t.l + 1] - t.a0;
    }
    const unsigned len = (unsigned)(lend[t.l] - lbeg[t.l]);
    // codes [c_lo, c_hi) of the list this kind covers
    t.c_lo = kind == 2 ? (unsigned)TILE_N : 0u;  // kind 2's first tile was in pass 1
    t.c_hi = kind == 1 ? min(len, (unsigned)TILE_N) : len;
    const unsigned span = t.c_hi > t.c_lo ? t.c_hi - t.c_lo : 0u;
    t.nchunk = (span + CHUNK_TILES * TILE_N - 1) / (CHUNK_TILES * TILE_N);
    if (span == 0) t.cnt = 0;
    return t;
}

// Slots [s0, s0 + nslot): counts[s - s0] = the slot's items, counts[nslot] = 0.
__global__ void item_count_kernel(const unsigned* __restrict__ poff,
                                  const unsigned* __restrict__ poff2, int nlist, int s0, int nslot,
                                  const uint32_t* __restrict__ lorder,
                                  const uint64_t* __restrict__ lbeg,
                                  const uint64_t* __restrict__ lend, unsigned* __restrict__ counts) {
    const int u = blockIdx.x * blockDim.x + threadIdx.x;
    if (u > nslot) return;
    if (u == nslot) {  // the exclusive sum's total
        counts[u] = 0;
        return;
    }
    const ItemSlot t = item_slot(s0 + u, poff, poff2, nlist, lorder, lbeg, lend);
    counts[u] = ((t.cnt + TILE_M - 1) / TILE_M) * t.nchunk;
}

// Items of slots [s0, s0 + nslot) at items[base + ioff[u]], base = 0 for
// the pass-1 slots (kinds 0, 1: range[0..1] = {0, n1}) and range[1] for the
// pass-2 slots (kind 2: range[2..3] = {n1, n2}).
__global__ void __launch_bounds__(256)
    item_fill_kernel(const unsigned* __restrict__ poff, const unsigned* __restrict__ poff2,
                     int nlist, int s0, int nslot, const uint32_t* __restrict__ lorder,
                     const uint64_t* __restrict__ lbeg, const uint64_t* __restrict__ lend,
                     const uint32_t* __restrict__ pstart, const unsigned* __restrict__ ioff,
                     Item* __restrict__ items, unsigned cap, uint32_t* __restrict__ range) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int u = blockIdx.x * 8 + warp;
    const unsigned base = s0 == 0 ? 0u : range[1];
    if (u == 0 && lane == 0) {
        const unsigned end = min(base + ioff[nslot], cap);
        if (s0 == 0) {
            range[0] = 0;
            range[1] = end;
        } else {
            range[2] = base;
            range[3] = end - base;
        }
    }
    if (u >= nslot) return;
    const ItemSlot t = item_slot(s0 + u, poff, poff2, nlist, lorder, lbeg, lend);
    const unsigned at = base + ioff[u], nit = ioff[u + 1] - ioff[u];
    for (unsigned u = lane; u < nit; u += 32) {
        const unsigned rb = u / t.nchunk, ch = u - rb * t.nchunk;
        const unsigned c0 = t.c_lo + ch * CHUNK_TILES * TILE_N;
        Item it;
        it.a0 = t.a0 + rb * TILE_M;
        it.na = min((unsigned)TILE_M, t.cnt - rb * TILE_M);
        it.b0 = pstart[t.l] + c0;
        it.nb = min((unsigned)(CHUNK_TILES * TILE_N), t.c_hi - c0);
        it.tag0 = (uint32_t)lbeg[t.l] + c0;
        it.col0 = c0;
        it.pad[0] = it.pad[1] = 0;
        if (at + u < cap) items[at + u] = it;
    }
}

// Pass-2 pairs whose list cannot hold a code with d~ <= tadm are dropped:
// every code of list l has real distance D >= (||r|| - Rh_l)^2 and
// d~ >= D - E_l, so a pair with (||r|| - Rh_l)^2 - E_l > tadm[q] admits
// nothing (the bounds of certify_kernel).  flags[i] = 1 for the pass-2 pairs
// kept; live[l] (sampled) and live[nlist + l] (unsampled) count them per
// list, stat[2] their pass-2 scores.
__global__ void prune_kernel(const uint32_t* __restrict__ skeys, const unsigned* __restrict__ poff,
                             int nlist, unsigned np, const uint32_t* __restrict__ pair_q,
                             const float* __restrict__ pair_rn, const float* __restrict__ rh,
                             const float* __restrict__ tadm, const uint64_t* __restrict__ lbeg,
                             const uint64_t* __restrict__ lend, uint8_t* __restrict__ flags,
                             unsigned* __restrict__ live, unsigned long long* stat) {
    const unsigned i = blockIdx.x * blockDim.x + threadIdx.x;
    const unsigned n1 = poff[nlist], npairs = poff[3 * nlist];
    uint8_t keep = 0;
    unsigned long long scores = 0;
    if (i < np && i >= n1 && i < npairs) {
        // sampled pairs (keys nlist + l) cover tiles 1.., the others (keys
        // 2 nlist + l) the whole list
        const bool smp = skeys[i] < 2u * (uint32_t)nlist;
        const uint32_t l = skeys[i] - (smp ? 1u : 2u) * (uint32_t)nlist;
        const uint64_t len = lend[l] - lbeg[l];
        const uint64_t skip = smp ? (uint64_t)TILE_N : 0;
        if (len > skip) {
            const double C1 = 2.0 * (9.765625e-4 + 1.220703125e-4) * 1.05;
            const double C2 = 1.52587890625e-5;
            const double r = (double)rh[l];
            const double D = (double)pair_rn[i];
            const double R = sqrt(D) * (1.0 + 1.52587890625e-5);
            const double El = C1 * R * r + C2 * (R * R + r * r) + 1e-30;
            const double Rl = sqrt(D) * (1.0 - 1.52587890625e-5) - r;
            const double lower = Rl > 0.0 ? Rl * Rl * (1.0 - 1e-6) - El : -1.0;
            if (!(lower > (double)tadm[pair_q[i]])) {
                keep = 1;
                atomicAdd(live + (smp ? 0 : nlist) + l, 1u);
                scores = len - skip;
            }
        }
    }
    if (i < np) flags[i] = keep;
    if (stat) {
        // one atomic per warp (every lane of the warp is still here)
        for (int o = 16; o >= 1; o >>= 1) scores += __shfl_xor_sync(0xffffffffu, scores, o);
        if ((threadIdx.x & 31) == 0 && scores) atomicAdd(stat + 2, scores);
    }
}

// One warp per query: the top-64 keys over its dump rows (the whole pass-1
// list and the first tile of each other list it probes here; 128 values per
// step) into part[q]; tau[q] = their 64th distance (+inf if fewer).
__global__ void __launch_bounds__(256)
    select1_kernel(const float* __restrict__ dump, const unsigned* __restrict__ seg,
                   const uint32_t* __restrict__ inv, const unsigned* __restrict__ poff,
                   int nlist, const uint32_t* __restrict__ probes, int take,
                   const uint64_t* __restrict__ lbeg, const uint64_t* __restrict__ lend, int nq,
                   const uint32_t* __restrict__ qlo, const uint32_t* __restrict__ qhi,
                   uint64_t* __restrict__ part, float* __restrict__ tau) {
    __shared__ uint64_t buf[8 * 64];
    __shared__ unsigned hist[8 * 256];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * 8 + warp;
    if (q >= nq) return;
    const unsigned n1 = poff[nlist], npairs = poff[2 * nlist];
    // Visits the query's dump rows: probes in batches of 32 (each lane looks
    // up one probe's row: the index chain inv -> list -> bounds runs in
    // parallel across lanes), then the rows one probe at a time, 128 entries
    // per step, f(d[4], tag of entry 0, entries valid) per lane.
    auto visit = [&](auto&& f) {
        for (int jp0 = 0; jp0 < take; jp0 += 32) {
            const int jp = jp0 + lane;
            unsigned start = 0, nbl = 0, tagl = 0;
            if (jp < take) {
                const size_t v = (size_t)q * take + jp;
                const uint32_t i = inv[v];
                if (i < npairs) {  // else: list empty or held elsewhere
                    const uint32_t l = probes[v];
                    const unsigned len = (unsigned)(lend[l] - lbeg[l]);
                    nbl = i < n1 ? len : min(len, (unsigned)TILE_N);
                    start = seg[i];
                    tagl = (uint32_t)lbeg[l];
                }
            }
            unsigned live = __ballot_sync(0xffffffffu, nbl > 0);
            while (live) {
                const int p = __ffs(live) - 1;
                live &= live - 1;
                const int nb = (int)__shfl_sync(0xffffffffu, nbl, p);
                const uint32_t tag0 = __shfl_sync(0xffffffffu, tagl, p);
                // rows are padded to a multiple of 128 floats
                const float4* row4 =
                    reinterpret_cast<const float4*>(dump + __shfl_sync(0xffffffffu, start, p));
                for (int base = 0; base < nb; base += 128) {
                    const float4 x4 = row4[(base >> 2) + lane];
                    const int j = base + 4 * lane;
                    const float d[4] = {x4.x, x4.y, x4.z, x4.w};
                    f(d, tag0 + (uint32_t)j, nb - j);
                }
            }
        }
    };
    // 1. the range of the query's finite distances (+inf marks a tombstoned
    //    row), gathered by pass 1's epilogue as it wrote the dump rows
    const uint32_t lo = qlo[q], hi = ~qhi[q];
    // 2. a threshold t with at least LIST_K entries d <= t: the rounded-up
    //    upper edge of the first of 256 bins (between lo and hi) whose running
    //    count reaches LIST_K (all entries when there are fewer)
    float t = INF;
    if (lo <= hi) {
        unsigned* hs = hist + warp * 256;
#pragma unroll
        for (int j = 0; j < 8; ++j) hs[j * 32 + lane] = 0u;
        __syncwarp();
        const float scale = 256.0f / ((float)(hi - lo) + 1.0f);
        visit([&](const float(&d)[4], uint32_t, int nv) {
#pragma unroll
            for (int x = 0; x < 4; ++x)
                if (x < nv && d[x] < INF)
                    atomicAdd(&hs[min(255, (int)((float)(f2ord(d[x]) - lo) * scale))], 1u);
        });
        __syncwarp();
        unsigned c[8], sum = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            c[j] = hs[8 * lane + j];
            sum += c[j];
        }
        unsigned incl = sum;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        const unsigned reach = __ballot_sync(0xffffffffu, incl >= (unsigned)LIST_K);
        if (reach) {
            const int owner = __ffs(reach) - 1;
            int bs = 255;
            unsigned run = incl - sum;
            bool found = false;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                run += c[j];
                if (!found && run >= (unsigned)LIST_K) {
                    bs = 8 * lane + j;
                    found = true;
                }
            }
            const int bstar = __shfl_sync(0xffffffffu, bs, owner);
            if (bstar < 255) {
                // every entry in bins <= bstar has (bits - lo) * scale < bstar + 1
                // in float arithmetic; the bound is widened for both roundings
                const double w = ((double)bstar + 1.0) / (double)scale * (1.0 + 1e-6) + 2.0;
                t = ord2f((uint32_t)min((double)hi, (double)lo + ceil(w)));
            }
        }
    }
    // 3. the top-LIST_K keys among the entries d <= t
    WarpTopK<2> tk;
    tk.init(LIST_K, buf + warp * 64);
    visit([&](const float(&d)[4], uint32_t tag, int nv) {
        uint64_t key[4];
        bool any = false;
#pragma unroll
        for (int x = 0; x < 4; ++x) {
            key[x] = (x < nv && d[x] < INF && d[x] <= t) ? make_key(d[x], tag + (uint32_t)x)
                                                          : KEY_NONE;
            any |= key[x] < tk.thr;
        }
        if (!__any_sync(0xffffffffu, any)) return;
#pragma unroll
        for (int x = 0; x < 4; ++x) tk.add(key[x], key[x] != KEY_NONE);
    });
    tk.flush();
    tk.store(part + (size_t)q * LIST_K);
    if (lane == 0) tau[q] = tk.thr == KEY_NONE ? INF : key_dist(tk.thr);
}

// One warp per query: the 64 best of its pass-1 list and pass-2 candidates.
__global__ void __launch_bounds__(256)
    select_kernel(const uint64_t* __restrict__ part, const uint64_t* __restrict__ cand,
                  const unsigned* __restrict__ cnt, int cap, int nq,
                  const float* __restrict__ tau, uint64_t* __restrict__ out) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * 8 + warp;
    if (q >= nq) return;
    WarpTopK<2> tk;
    tk.init(LIST_K, nullptr);
    // the pass-1 list, ascending; on a sharded index entries above the
    // exchanged threshold cannot be in the answer and are dropped
    const float t = tau[q];
    uint64_t a0 = part[(size_t)q * LIST_K + lane], a1 = part[(size_t)q * LIST_K + 32 + lane];
    if (a0 != KEY_NONE && key_dist(a0) > t) a0 = KEY_NONE;
    if (a1 != KEY_NONE && key_dist(a1) > t) a1 = KEY_NONE;
    tk.L[0] = a0;
    tk.L[1] = a1;
    tk.thr = __shfl_sync(0xffffffffu, tk.L[1], 31);
    tk.ingest(cand + (size_t)q * cap, (int)min(cnt[q], (unsigned)cap));
    tk.store(out + (size_t)q * LIST_K);
}

// One warp per query: tadm = tau + 2 (E_adc + max_l E_l), the pass-2
// admission threshold (the bounds of certify_kernel; rounded up).  With the
// factor 2 the certificate extension always applies (dk <= tau + E); a
// smaller factor admits fewer candidates and extends when dk is below
// tau + (factor - 1) E.
#ifndef FDB_IVF_MARGIN
#define FDB_IVF_MARGIN 2.0
#endif
__global__ void __launch_bounds__(256)
    margin_kernel(const float* __restrict__ Q, int nq, int dim, int m,
                  const float* __restrict__ cmax, const float* __restrict__ bmax,
                  const uint32_t* __restrict__ probes, const float* __restrict__ pdist, int take,
                  const uint64_t* __restrict__ lbeg, const uint64_t* __restrict__ lend,
                  const float* __restrict__ rh, const float* __restrict__ tau,
                  float* __restrict__ tadm, float* __restrict__ ebound) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q = blockIdx.x * 8 + warp;
    if (q >= nq) return;
    const int sub = dim / m;
    const float* qv = Q + (size_t)q * dim;
    double part = 0.0;
    for (int s = lane; s < m; s += 32) {
        double qn = 0.0;
        for (int i = 0; i < sub; ++i) {
            const double x = qv[s * sub + i];
            qn += x * x;
        }
        const double t = sqrt(qn) + (double)cmax[s] + (double)bmax[s];
        part += t * t;
    }
    double emax = 0.0;
    const double C1 = 2.0 * (9.765625e-4 + 1.220703125e-4) * 1.05;
    const double C2 = 1.52587890625e-5;
    for (int j = lane; j < take; j += 32) {
        const uint32_t l = probes[(size_t)q * take + j];
        if (lend[l] <= lbeg[l]) continue;
        const double r = (double)rh[l];
        const double R = sqrt((double)pdist[(size_t)q * take + j]) * (1.0 + 1.52587890625e-5);
        emax = fmax(emax, C1 * R * r + C2 * (R * R + r * r) + 1e-30);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        part += __shfl_xor_sync(0xffffffffu, part, o);
        emax = fmax(emax, __shfl_xor_sync(0xffffffffu, emax, o));
    }
    if (lane == 0) {
        const double eadc = (32.0 + 4.0 * m) * 5.9604644775390625e-8 * part * 1.01;
        const float delta = __double2float_ru(FDB_IVF_MARGIN * (eadc + emax) * (1.0 + 1e-6));
        tadm[q] = __fadd_ru(tau[q], delta);
        ebound[q] = __double2float_ru((eadc + emax) * (1.0 + 1e-6));
    }
}

// ---------------------------------------------------------------------------
// exact rescoring and certification
// ---------------------------------------------------------------------------
struct CertParams {
    const float* Q;
    int nq, dim, m;
    const float* cents;
    const float* cb;
    const uint64_t* offs_full;  // [nlist+1] unsharded offsets (key tags are their rows)
    int nlist;
    const uint8_t* codes;
    const uint64_t* approx;     // [nq][64] tensor-core shortlist, ascending
    int k;
    uint64_t* out_keys;         // [nq][k]
    uint64_t* ekeys;            // [nq][64] exact keys of the shortlist (rescore -> certify)
    int* elist;                 // [nq][64] their lists (-1: none)
    float* dk;                  // [nq] exact k-th distance (+inf if fewer); min over ranks
    const float* cmax;          // [m]
    const float* bmax;          // [m]
    const unsigned* cand_cnt;
    int cap;
    const float* tau;
    const float* pdist;         // [nq][take] exact coarse distances of the probes
    const uint32_t* probes;     // [nq][take]
    int take;
    const uint64_t* lbeg;
    const uint64_t* lend;
    const float* rh;            // [nlist] upper bound of ||rhat|| over the list's codes
    const uint32_t* qbad;
    uint32_t qbase;             // global id of query 0 of this chunk
    uint32_t* flag_count;
    uint32_t* flag_list;
    uint32_t* fail_probes;      // [flag slot][take] lists to re-scan exactly
    uint32_t* fail_cnt;         // [flag slot]
    const uint64_t* part;       // [nq][64] pass-1 keys (the extension's first source)
    const uint64_t* cand;       // [nq][cap] pass-2 candidates (its second source)
    uint32_t* ext_count;        // queries certified by extension
    uint32_t* ext_list;         // their local indices
    float* ext_thr;             // their extension thresholds
    unsigned long long* stat;   // [3] counts extended queries (nullable)
    uint32_t* over_count;       // extensions that held too many entries
    uint32_t* over_list;
    const float* tadm;          // [nq] pass-2 admission threshold tau + delta
    const float* ebound;        // [nq] E_adc + max_l E_l over the query's lists (rounded up)
    const float* dump;          // pass-1 distances, their rows and pair lookups
    const unsigned* seg;
    const uint32_t* inv;
    const unsigned* poff;
};

constexpr int CERT_WARPS = 8;
#ifndef FDB_IVF_EXT_MAX
#define FDB_IVF_EXT_MAX 1024
#endif
constexpr unsigned EXT_MAX = FDB_IVF_EXT_MAX;  // entries an extension may rescore
constexpr int EXT_THREADS = 1024;
constexpr int EXT_MAX_TAKE = 256;  // probes per query an extension handles
static_assert(EXT_MAX <= (unsigned)EXT_THREADS, "one thread rescores one collected entry");

// Two warps per query, 32 shortlisted codes each: the codes rescored with
// exact_adc (the reference's arithmetic), their exact keys and lists kept for
// certify_kernel; then the query's first warp writes the k best and the exact
// k-th distance dk.  P = 1 for k <= 32, 2 for k <= 64.  For k <= 32 the
// second warp's codes (shortlist entries 32..63) are skipped when they cannot
// matter: each has d~ >= d~_32 and so an exact distance >= d~_32 - E, while the
// exact k-th is at most d~_(k-1) + E (E = E_adc + max_l E_l, the bounds of
// certify_kernel); when d~_32 - E > d~_(k-1) + E none of them can enter the
// answer or a seed, and their keys stay empty.
constexpr int RS_QUERIES = CERT_WARPS / 2;  // queries per block
// MS selects a compile-time ADC shape (1: m = 16 x 8 floats, 2: m = 48 x 2
// floats; 0: any shape, loops with run-time bounds).
template <int ORDER, int P, int MS>
__global__ void __launch_bounds__(CERT_WARPS * 32, 4) rescore_kernel(CertParams r) {
    __shared__ uint64_t keys[RS_QUERIES][LIST_K];
    __shared__ uint64_t buf[RS_QUERIES * 64];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int lq = warp >> 1, h = warp & 1;
    const int q = blockIdx.x * RS_QUERIES + lq;
    const bool qok = q < r.nq;
    if (qok) {  // warp-uniform
        const int m = r.m, sub = r.dim / m;
        const float* qv = r.Q + (size_t)q * r.dim;
        const size_t row = (size_t)q * LIST_K;
        bool skip = false;
        if (P == 1 && h == 1) {
            const uint64_t a32 = r.approx[row + 32], akm1 = r.approx[row + r.k - 1];
            const float e = r.ebound[q];
            skip = a32 == KEY_NONE ||
                   (akm1 != KEY_NONE &&
                    __fsub_rd(key_dist(a32), e) > __fadd_ru(key_dist(akm1), e));
        }
        const uint64_t key = skip ? KEY_NONE : r.approx[row + h * 32 + lane];
        uint64_t ek = KEY_NONE;
        int el = -1;
        if (key != KEY_NONE) {
            const uint32_t pos = key_tag(key);
            int lo = 0, hi = r.nlist;  // the list l with offs[l] <= pos < offs[l+1]
            while (lo < hi) {
                const int mid = (lo + hi) >> 1;
                if (r.offs_full[mid + 1] <= pos) lo = mid + 1;
                else hi = mid;
            }
            // one code per lane: 32 independent chains keep many loads in flight
            const float* cl = r.cents + (size_t)lo * r.dim;
            const uint8_t* cd = r.codes + (size_t)pos * m;
            float d;
            if constexpr (MS == 1) d = exact_adc_fixed<ORDER, 16, 8>(qv, cl, r.cb, cd);
            else if constexpr (MS == 2) d = exact_adc_fixed<ORDER, 48, 2>(qv, cl, r.cb, cd);
            else d = exact_adc<ORDER>(qv, cl, r.cb, cd, m, sub);
            ek = make_key(d, pos);
            el = lo;
        }
        r.ekeys[row + h * 32 + lane] = ek;
        r.elist[row + h * 32 + lane] = el;
        keys[lq][h * 32 + lane] = ek;
    }
    __syncthreads();
    if (!qok || h != 0) return;
    WarpTopK<P> tk;
    tk.init(r.k, buf + lq * 64);
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
        const uint64_t ek = keys[lq][hh * 32 + lane];
        if (__any_sync(0xffffffffu, ek != KEY_NONE)) tk.merge32(ek);
    }
    tk.store(r.out_keys + (size_t)q * r.k);
    if (lane == 0) r.dk[q] = tk.thr == KEY_NONE ? INF : key_dist(tk.thr);
}

// One warp per query.  Certification: for a code of list l, |d~ - D| <= E_l
// and |exact - D| <= E_adc, where D is the real ADC distance of r = fl(q - c_l):
//   E_l  = C1 R_l Rh_l + C2 (R_l^2 + Rh_l^2),  R_l >= ||r||, Rh_l >= ||rhat||
//          over the list's codes, C1 = 2 (2^-10 + 2^-13) * 1.05: fp16
//          rounding of both operands (2^-11 each, relative) and an allowance
//          of 2^-13 for the tensor core's fp32 accumulation; C2 = 2^-16
//          covers the fp32 roundings of ||r||^2, ||rhat||^2 and the final
//          fused multiply-add;
//   E_adc = (32 + 4m) 2^-24 sum_s (||q_s|| + cmax_s + bmax_s)^2 * 1.01.
// dk is an upper bound of the exact k-th distance of the answer: this
// device's exact k-th over its shortlist, or on a sharded index the minimum of
// that over all devices.  Every code outside the shortlist has d~ >= B (B =
// the 64th shortlisted value when the shortlist is full, tau otherwise), so
// it cannot enter the answer if, for its list, dk + E_adc + E_l < B, or if
// its real distance is above dk anyway: (||r|| - Rh_l)^2 - E_adc > dk.  The
// device's output (its exact top-k over the shortlist) then holds every one of
// its codes that can be in the answer.  Overflowing candidate arrays and
// queries marked bad are never certified.  A query with failing lists gets
// them listed for an exact re-scan, and its output row becomes the seed: the
// exact top-k of its shortlisted codes in the other lists.
template <int P>
__global__ void __launch_bounds__(CERT_WARPS * 32) certify_kernel(CertParams r, int forced) {
    __shared__ uint64_t buf[CERT_WARPS * 64];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // forced: the queries whose extension held too many entries, sent to
    // the re-scan path
    int q;
    if (forced) {
        const uint32_t sl = blockIdx.x * CERT_WARPS + warp;
        if (sl >= *r.over_count) return;  // whole warp
        q = (int)r.over_list[sl];
    } else {
        q = blockIdx.x * CERT_WARPS + warp;
        if (q >= r.nq) return;  // whole warp
    }
    const int m = r.m, sub = r.dim / m;
    const float* qv = r.Q + (size_t)q * r.dim;
    const uint64_t* ak = r.approx + (size_t)q * LIST_K;
    double part = 0.0;
    for (int s = lane; s < m; s += 32) {
        double qn = 0.0;
        for (int i = 0; i < sub; ++i) {
            const double x = qv[s * sub + i];
            qn += x * x;
        }
        const double t = sqrt(qn) + (double)r.cmax[s] + (double)r.bmax[s];
        part += t * t;
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    const double Eadc = (32.0 + 4.0 * m) * 5.9604644775390625e-8 * part * 1.01;
    const double C1 = 2.0 * (9.765625e-4 + 1.220703125e-4) * 1.05;
    const double C2 = 1.52587890625e-5;
    const unsigned c = r.cand_cnt[q];
    const uint64_t last = ak[LIST_K - 1];
    // (stored entries are the shortlist when it is not full; anything else
    // has d~ above the admission threshold)
    const double B = last != KEY_NONE ? (double)key_dist(last) : (double)r.tadm[q];
    const double dk = (double)r.dk[q];
    // whole-query failures: every list is re-scanned and nothing is kept
    const bool fail_all = c > (unsigned)r.cap || r.qbad[q] != 0u || (!isinf(B) && isinf(dk));
    // per-list verdict for probe j (true: no code of the list outside the
    // shortlist can enter the answer)
    auto list_ok = [&](int j) -> bool {
        const uint32_t l = r.probes[(size_t)q * r.take + j];
        if (r.lend[l] <= r.lbeg[l]) return true;
        if (isinf(B)) return true;  // every code of the list is in the shortlist
        const double rh = (double)r.rh[l];
        const double D = (double)r.pdist[(size_t)q * r.take + j];
        const double R = sqrt(D) * (1.0 + 1.52587890625e-5);
        const double El = C1 * R * rh + C2 * (R * R + rh * rh) + 1e-30;
        const double Rl = sqrt(D) * (1.0 - 1.52587890625e-5) - rh;
        const double lower = Rl > 0.0 ? Rl * Rl * (1.0 - 1e-6) - Eadc : -1.0;
        return (dk + Eadc + El < B) || (dk < lower);
    };
    bool ok = !fail_all && !forced;
    for (int j0 = 0; ok && j0 < r.take; j0 += 32) {
        const int j = j0 + lane;
        ok = __all_sync(0xffffffffu, j >= r.take || list_ok(j));
    }
    if (ok) return;  // rescore_kernel's output stands
    // Extension.  Every pass-1 distance is in the dump and pass 2 stores
    // every code with d~ <= tadm = tau + 2 (E_adc + max_l E_l), so if
    //   T = dk + E_adc + max_l E_l  <  tadm
    // (always, as dk <= tau + E_adc + max_l E_l) rescoring every stored
    // entry outside the shortlist with d~ <= T leaves only codes with
    // d~ > T >= (new dk) + E_adc + E_l unscored: the merged exact top-k is
    // certified without re-scanning any list.
    if (!fail_all && !forced && c <= (unsigned)r.cap && r.take <= EXT_MAX_TAKE) {
        double emax = 0.0;
        for (int j = lane; j < r.take; j += 32) {
            const uint32_t l = r.probes[(size_t)q * r.take + j];
            if (r.lend[l] <= r.lbeg[l]) continue;
            const double rh = (double)r.rh[l];
            const double R = sqrt((double)r.pdist[(size_t)q * r.take + j]) * (1.0 + 1.52587890625e-5);
            emax = fmax(emax, C1 * R * rh + C2 * (R * R + rh * rh) + 1e-30);
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) emax = fmax(emax, __shfl_xor_sync(0xffffffffu, emax, o));
        const double T = (dk + Eadc + emax) * (1.0 + 1e-9);
        if (T < (double)r.tadm[q]) {
            if (lane == 0) {
                // the largest float not above T: entries with d~ up to it are
                // rescored, the rest have d~ > T
                float tf = (float)T;
                if ((double)tf > T) tf = nextafterf(tf, 0.0f);
                const uint32_t slot = atomicAdd(r.ext_count, 1u);
                r.ext_list[slot] = (uint32_t)q;
                r.ext_thr[slot] = tf;
            }
            return;  // extend_kernel merges into rescore_kernel's output
        }
    }
    uint32_t slot = 0;
    if (lane == 0) {
        slot = atomicAdd(r.flag_count, 1u);
        r.flag_list[slot] = r.qbase + (uint32_t)q;
    }
    slot = __shfl_sync(0xffffffffu, slot, 0);
    uint32_t* fp = r.fail_probes + (size_t)slot * r.take;
    const uint64_t ek[2] = {r.ekeys[(size_t)q * LIST_K + lane],
                            r.ekeys[(size_t)q * LIST_K + 32 + lane]};
    const int el[2] = {r.elist[(size_t)q * LIST_K + lane], r.elist[(size_t)q * LIST_K + 32 + lane]};
    // failed lists, compacted; shortlisted codes of those lists are dropped
    // from the seed (the exact re-scan meets them again)
    unsigned nf = 0;
    bool drop0 = false, drop1 = false;
    for (int j0 = 0; j0 < r.take; j0 += 32) {
        const int j = j0 + lane;
        const bool inr = j < r.take;
        const uint32_t l = inr ? r.probes[(size_t)q * r.take + j] : 0u;
        const bool bad = inr && (fail_all || !list_ok(j));
        unsigned mask = __ballot_sync(0xffffffffu, bad);
        if (bad) fp[nf + __popc(mask & ((1u << lane) - 1u))] = l;
        nf += __popc(mask);
        while (mask) {
            const int b = __ffs(mask) - 1;
            mask &= mask - 1;
            const int lf = (int)__shfl_sync(0xffffffffu, l, b);
            drop0 |= el[0] == lf;
            drop1 |= el[1] == lf;
        }
    }
    if (lane == 0) r.fail_cnt[slot] = nf;
    WarpTopK<P> seed;
    seed.init(r.k, buf + warp * 64);
    const uint64_t s0 = drop0 ? KEY_NONE : ek[0], s1 = drop1 ? KEY_NONE : ek[1];
    if (__any_sync(0xffffffffu, s0 != KEY_NONE)) seed.merge32(s0);
    if (__any_sync(0xffffffffu, s1 != KEY_NONE)) seed.merge32(s1);
    seed.store(r.out_keys + (size_t)q * r.k);
}

// One block per extended query (see certify_kernel): every pass-1 distance
// (dump) and pass-2 candidate that lies outside the shortlist (key above its
// 64th) with d~ <= the query's threshold is collected, rescored exactly (one
// entry per thread) and merged into its exact top-k row.  A query with more
// than EXT_MAX such entries goes to the re-scan path instead.
typedef cub::BlockScan<unsigned, EXT_THREADS> ExtScan;
struct ExtShared {
    uint64_t keys[EXT_MAX];
    uint64_t buf[64];
    unsigned pstart[EXT_MAX_TAKE], plen[EXT_MAX_TAKE], ptag[EXT_MAX_TAKE];
    unsigned cnt;
    float dres[EXT_THREADS / 32][32];
    typename ExtScan::TempStorage scan_tmp;
};

// One extended query (flag slot `slot`), the whole block.  MS: a
// compile-time ADC shape as in rescore_kernel (0: any shape).
template <int ORDER, int P, int MS>
__device__ __forceinline__ void extend_slot(const CertParams& r, uint32_t slot, ExtShared& sh) {
    uint64_t* keys = sh.keys;
    unsigned* pstart = sh.pstart;
    unsigned* plen = sh.plen;
    unsigned* ptag = sh.ptag;
    unsigned& cnt = sh.cnt;
    const int t = threadIdx.x;
    const int q = (int)r.ext_list[slot];
    const float thr = r.ext_thr[slot];
    const uint64_t last = r.approx[(size_t)q * LIST_K + LIST_K - 1];
    if (t == 0) cnt = 0;
    // the query's pass-1 dump rows (as select1_kernel) and their prefix
    const unsigned n1 = r.poff[r.nlist], npairs = r.poff[2 * r.nlist];
    unsigned nb = 0;
    if (t < r.take) {
        const size_t v = (size_t)q * r.take + t;
        const uint32_t i = r.inv[v];
        if (i < npairs) {
            const uint32_t l = r.probes[v];
            const unsigned len = (unsigned)(r.lend[l] - r.lbeg[l]);
            nb = i < n1 ? len : min(len, (unsigned)TILE_N);
            pstart[t] = r.seg[i];
            ptag[t] = (uint32_t)r.lbeg[l];
        }
    }
    unsigned off, total;
    ExtScan(sh.scan_tmp).ExclusiveSum(nb, off, total);
    if (t < r.take) plen[t] = off;  // prefix
    __syncthreads();
    const int take = r.take;
    auto keep = [&](uint64_t key) {
        if (key == KEY_NONE || key <= last || key_dist(key) > thr) return;
        const unsigned ix = atomicAdd(&cnt, 1u);
        if (ix < EXT_MAX) keys[ix] = key;
    };
    for (unsigned f = t; f < total; f += EXT_THREADS) {
        int lo = 0, hi = take - 1;  // the last pair whose prefix is <= f
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (plen[mid] <= f) lo = mid;
            else hi = mid - 1;
        }
        const unsigned j = f - plen[lo];
        const float d = r.dump[pstart[lo] + j];
        if (d <= thr) keep(make_key(d, ptag[lo] + j));
    }
    const unsigned nc = min(r.cand_cnt[q], (unsigned)r.cap);
    for (unsigned e = t; e < nc; e += EXT_THREADS) keep(r.cand[(size_t)q * r.cap + e]);
    __syncthreads();
    const unsigned n = cnt;
    if (n > EXT_MAX) {
        if (t == 0) r.over_list[atomicAdd(r.over_count, 1u)] = (uint32_t)q;
        return;  // whole block
    }
    {
        // warp w rescores entries [32 w, 32 w + 32) by lane groups
        const bool valid = t < (int)n;
        uint32_t pos = 0;
        int lo = 0;
        if (valid) {
            pos = key_tag(keys[t]);
            int hi = r.nlist;  // the list l with offs[l] <= pos < offs[l+1]
            while (lo < hi) {
                const int mid = (lo + hi) >> 1;
                if (r.offs_full[mid + 1] <= pos) lo = mid + 1;
                else hi = mid;
            }
        }
        const int m = r.m, sub = r.dim / m;
        float d;
        if constexpr (MS != 0) {
            // one entry per thread, every load of its code in flight together
            d = 0.0f;
            if (valid) {
                const float* qv = r.Q + (size_t)q * r.dim;
                const float* cl = r.cents + (size_t)lo * r.dim;
                const uint8_t* cd = r.codes + (size_t)pos * m;
                if constexpr (MS == 1) d = exact_adc_fixed<ORDER, 16, 8>(qv, cl, r.cb, cd);
                else d = exact_adc_fixed<ORDER, 48, 2>(qv, cl, r.cb, cd);
            }
        } else {
            d = warp_exact_adc<ORDER>(r.Q + (size_t)q * r.dim, r.cents, r.dim, r.cb, r.codes,
                                      m, sub, pos, lo, valid, sh.dres[t >> 5]);
        }
        if (valid) keys[t] = make_key(d, pos);
    }
    __syncthreads();
    if (t >= 32) return;
    // the current exact top-k first: its k-th then skips most batches of the
    // collected entries (the result is the top-k of the union either way)
    WarpTopK<P> tk;
    tk.init(r.k, sh.buf);
    uint64_t* row = r.out_keys + (size_t)q * r.k;
    tk.ingest(row, r.k);
    tk.ingest(keys, (int)n);
    tk.store(row);
    if (t == 0 && r.stat) atomicAdd(r.stat + 3, 1ull);
}

// A grid of a few blocks per SM walks the extended queries (their count is
// only known on the device).
template <int ORDER, int P, int MS>
__global__ void __launch_bounds__(EXT_THREADS) extend_kernel(CertParams r) {
    __shared__ ExtShared sh;
    const uint32_t count = *r.ext_count;
    for (uint32_t slot = blockIdx.x; slot < count; slot += gridDim.x) {
        __syncthreads();  // the previous slot's shared state is no longer read
        extend_slot<ORDER, P, MS>(r, slot, sh);
    }
}

// ---------------------------------------------------------------------------
// exact re-scan of failed lists, one block per (query, list)
// ---------------------------------------------------------------------------
// Unit offsets: uoff[f] = the failed lists of flag slots 0 .. f-1 (flags[0]
// slots, fail_cnt[f] lists each); *nunits = their total.  One block.
__global__ void __launch_bounds__(1024)
    unit_offsets_kernel(const uint32_t* __restrict__ flags, const uint32_t* __restrict__ fail_cnt,
                        uint32_t* __restrict__ uoff, uint32_t* __restrict__ nunits) {
    typedef cub::BlockScan<unsigned, 1024> Scan;
    __shared__ typename Scan::TempStorage tmp;
    __shared__ unsigned carry;
    const unsigned nflag = flags[0];
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (unsigned b = 0; b < nflag; b += 1024) {
        const unsigned f = b + threadIdx.x;
        const unsigned v = f < nflag ? fail_cnt[f] : 0u;
        unsigned ex, tot;
        Scan(tmp).ExclusiveSum(v, ex, tot);
        const unsigned c0 = carry;
        if (f < nflag) uoff[f] = c0 + ex;
        __syncthreads();  // every thread has read carry (and tmp is free)
        if (threadIdx.x == 0) carry = c0 + tot;
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        uoff[nflag] = carry;
        *nunits = carry;
    }
}

// The units u in [r0, r0 + ucap) of flag slot f (units uoff[f] .. uoff[f+1]:
// its query and its failed lists in order), written at u - r0.
__global__ void expand_units_kernel(const uint32_t* __restrict__ flags, int take,
                                    const uint32_t* __restrict__ fail_probes,
                                    const uint32_t* __restrict__ uoff, uint32_t r0, uint32_t ucap,
                                    uint32_t* __restrict__ unit_q, uint32_t* __restrict__ unit_l) {
    const uint32_t f = blockIdx.x * blockDim.x + threadIdx.x;
    if (f >= flags[0]) return;
    const uint32_t q = flags[1 + f];
    const uint32_t u0 = uoff[f], u1 = uoff[f + 1];
    const uint32_t lo = max(u0, r0), hi = min(u1, r0 + ucap);
    for (uint32_t u = lo; u < hi; ++u) {
        unit_q[u - r0] = q;
        unit_l[u - r0] = fail_probes[(size_t)f * take + (u - u0)];
    }
}

// One warp per flag slot (grid-stride over flags[0] slots): the query's row
// (its seed, or the merge of earlier rounds) and the exact top-k of each of
// its units in [r0, r0 + ucap), merged into its out_keys row.
template <int P>
__global__ void __launch_bounds__(256)
    merge_units_kernel(int k, const uint32_t* __restrict__ flags,
                       const uint32_t* __restrict__ uoff, uint32_t r0, uint32_t ucap,
                       const uint64_t* __restrict__ unit_keys, uint64_t* __restrict__ out_keys) {
    __shared__ uint64_t buf[8 * 64];
    const int warp = threadIdx.x >> 5;
    const uint32_t nflag = flags[0];
    for (uint32_t f = blockIdx.x * 8 + warp; f < nflag; f += gridDim.x * 8) {
        const uint32_t lo = max(uoff[f], r0), hi = min(uoff[f + 1], r0 + ucap);
        if (lo >= hi) continue;  // warp-uniform
        uint64_t* row = out_keys + (size_t)flags[1 + f] * k;
        WarpTopK<P> tk;
        tk.init(k, buf + warp * 64);
        tk.ingest(row, k);
        for (uint32_t u = lo; u < hi; ++u) tk.ingest(unit_keys + (size_t)(u - r0) * k, k);
        tk.store(row);
    }
}

// ---------------------------------------------------------------------------
// per-index preparation: decoded codes in the padded list layout
// ---------------------------------------------------------------------------
// One warp per code row j: rhat scaled by 2^sb in fp16 (zero padded to dpad)
// at row pstart[l] + (j - offs[l]) of the padded layout, and ||rhat||^2 from
// the unscaled fp32 values.
__global__ void decode_kernel(const uint8_t* __restrict__ codes, size_t n, int m, int sub,
                              int dim, int dpad, const float* __restrict__ cb, float bscale,
                              const uint64_t* __restrict__ offs, int nlist,
                              const uint32_t* __restrict__ pstart, __half* __restrict__ dec,
                              float* __restrict__ norm) {
    const size_t row = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= n) return;
    int lo = 0, hi = nlist;  // the list l with offs[l] <= row < offs[l+1]
    while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (offs[mid + 1] <= row) lo = mid + 1;
        else hi = mid;
    }
    const size_t prow = (size_t)pstart[lo] + (row - offs[lo]);
    const uint8_t* code = codes + row * m;
    float acc = 0.0f;
    for (int c = lane; c < dpad; c += 32) {
        float x = 0.0f;
        if (c < dim) {
            const int s = c / sub;
            x = cb[((size_t)s * KSUB + code[s]) * sub + (c - s * sub)];
        }
        acc = __fmaf_rn(x, x, acc);
        dec[prow * dpad + c] = __float2half_rn(__fmul_rn(x, bscale));
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
    if (lane == 0) norm[prow] = acc;
}

__global__ void fill_inf_kernel(float* p, size_t n) {
    const size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t < n) p[t] = INF;
}

// rh[l] = sqrt(max ||rhat||^2 over the list's codes), rounded up (one warp per list).
__global__ void list_rh_kernel(const float* __restrict__ norm, const uint32_t* __restrict__ pstart,
                               const uint64_t* __restrict__ offs, int nlist,
                               float* __restrict__ rh) {
    const int l = (int)(((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (l >= nlist) return;
    const size_t len = offs[l + 1] - offs[l];
    float mx = 0.0f;
    for (size_t i = lane; i < len; i += 32) mx = fmaxf(mx, norm[pstart[l] + i]);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) rh[l] = sqrtf(mx) * (1.0f + 1e-5f);
}

size_t pass_smem(int katoms) {
    return 1024 + (size_t)(ASLOTS + NSTAGE) * katoms * ATOM_BYTES + (size_t)NCV * CV_FLOATS * 4 +
           (size_t)(2 * ASLOTS + 2 * NSTAGE + 2 * NACC + 2 * NCV + 4) * 8 + 2 * 4 + 16;
}

template <int EPI>
void launch_pass(cudaStream_t s, const CUtensorMap& am, const CUtensorMap& bm, int grid,
                 const PassParams& p) {
    const size_t smem = pass_smem(p.katoms);
    FDB_REQUIRE(smem <= 227 * 1024, FDB_ERR_UNSUPPORTED, "list scan needs too much shared memory");
    FDB_CUDA(cudaFuncSetAttribute(ivf_pass_kernel<EPI>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    ivf_pass_kernel<EPI><<<grid, THREADS, smem, s>>>(am, bm, p);
    FDB_LAUNCH_CHECK();
}

int bits_for(uint32_t v) {
    int b = 1;
    while ((1ull << b) <= v) ++b;
    return b;
}

}  // namespace ivtc

// ---------------------------------------------------------------------------
// host entry points
// ---------------------------------------------------------------------------
bool ivf_tc_eligible(const fdb_ivfpq* h, size_t k) {
    return h->dec16.p != nullptr && k >= 1 && k <= (size_t)ivtc::LIST_K;
}

// Decoded codes and their norms in the padded list layout, per-list bounds
// of ||rhat||, and the list order.  Needs the table mode's bound terms.
void ivf_tc_prepare(fdb_ivfpq* h, const std::vector<float>& cb_host,
                    const std::vector<float>& bmax_host) {
    (void)bmax_host;
    h->dec16.release();
    h->dnorm.release();
    h->lorder.release();
    h->tc_pstart.release();
    h->tc_rhl.release();
    const size_t n = h->n_total, dim = h->dim, m = h->m, sub = dim / m, nlist = h->nlist;
    const int dpad = (int)((dim + 63) / 64 * 64);
    if (dpad > 128 || n == 0) return;
    double amax = 0.0;
    for (float x : cb_host) amax = std::max(amax, (double)std::fabs(x));
    if (!(amax > 0.0) || !std::isfinite(amax)) return;
    const int sb = 13 - std::ilogb(amax);  // largest |b| * 2^sb in [2^13, 2^14)
    if (sb < -100 || sb > 100) return;
    // padded layout: list l starts at pstart[l], a multiple of 128 rows
    std::vector<uint32_t> pstart(nlist);
    size_t rows = 0;
    for (size_t l = 0; l < nlist; ++l) {
        pstart[l] = (uint32_t)rows;
        const size_t len = h->h_offs_full[l + 1] - h->h_offs_full[l];
        rows += (len + ivtc::TILE_N - 1) / ivtc::TILE_N * ivtc::TILE_N;
        if (rows >= (1ull << 31)) return;
    }
    Ctx& c = h->ctx->c;
    cudaStream_t st = c.stream;
    h->tc_dpad = dpad;
    h->tc_sb = sb;
    h->tc_rows = rows;
    h->tc_maxpad = 0;
    for (size_t l = 0; l < nlist; ++l)
        h->tc_maxpad = std::max<size_t>(h->tc_maxpad, (l + 1 < nlist ? pstart[l + 1] : rows) - pstart[l]);
    double rh2 = 0.0;
    for (size_t s = 0; s < m; ++s) rh2 += (double)bmax_host[s] * bmax_host[s];
    h->tc_colmax = (float)(rh2 * (1.0 + 1e-5));
    h->tc_pstart.alloc(nlist);
    FDB_CUDA(cudaMemcpyAsync(h->tc_pstart.p, pstart.data(), nlist * 4, cudaMemcpyHostToDevice, st));
    h->dec16.alloc(std::max<size_t>(rows, 1) * dpad);
    h->dnorm.alloc(std::max<size_t>(rows, 1));
    FDB_CUDA(cudaMemsetAsync(h->dec16.p, 0, h->dec16.bytes(), st));
    ivtc::fill_inf_kernel<<<(unsigned)((h->dnorm.n + 255) / 256), 256, 0, st>>>(h->dnorm.p,
                                                                                 h->dnorm.n);
    FDB_LAUNCH_CHECK();
    const unsigned blocks = (unsigned)((n * 32 + 255) / 256);
    ivtc::decode_kernel<<<blocks, 256, 0, st>>>(h->codes.p, n, (int)m, (int)sub, (int)dim, dpad,
                                                 h->cb.p, std::ldexp(1.0f, sb), h->offs.p,
                                                 (int)nlist, h->tc_pstart.p, h->dec16.p,
                                                 h->dnorm.p);
    FDB_LAUNCH_CHECK();
    h->tc_rhl.alloc(nlist);
    ivtc::list_rh_kernel<<<(unsigned)((nlist * 32 + 255) / 256), 256, 0, st>>>(
        h->dnorm.p, h->tc_pstart.p, h->offs.p, (int)nlist, h->tc_rhl.p);
    FDB_LAUNCH_CHECK();
    // lists by decreasing length (ties by list id)
    std::vector<uint32_t> order(nlist);
    std::iota(order.begin(), order.end(), 0u);
    std::stable_sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) {
        return h->h_offs_full[a + 1] - h->h_offs_full[a] > h->h_offs_full[b + 1] - h->h_offs_full[b];
    });
    h->lorder.alloc(nlist);
    FDB_CUDA(cudaMemcpyAsync(h->lorder.p, order.data(), nlist * 4, cudaMemcpyHostToDevice, st));
    FDB_CUDA(cudaStreamSynchronize(st));
}

namespace {

// One chunk of queries [q0, q0 + nq) through the whole tensor path.  probes
// and pdist point at the chunk's rows; flag entries are global query ids.
void tc_chunk(fdb_ivfpq* h, const float* dQ, size_t nq, size_t k, int order, size_t take,
              const uint32_t* probes, const float* pdist, const uint64_t* lbeg,
              const uint64_t* lend, uint64_t* out_keys, uint32_t* flags, uint32_t qbase,
              unsigned long long* stat, int* err, uint32_t* fail_probes, uint32_t* fail_cnt,
              StageTimer* pass_tm) {
    using namespace ivtc;
    Ctx& c = h->ctx->c;
    cudaStream_t s = c.stream;
    const int nlist = (int)h->nlist;
    const size_t np = nq * take;
    const int dpad = h->tc_dpad;
    const int nkeys = 3 * nlist + 1;
    // --- group the pairs by (pass, list) ---
    h->t_keys.ensure(2 * np);
    h->t_vals.ensure(2 * np);
    h->t_off.ensure((size_t)nkeys + 1);
    pair_keys_kernel<<<(unsigned)((nq * 32 + 255) / 256), 256, 0, s>>>(
        probes, (int)nq, (int)take, lbeg, lend, h->offs.p, nlist, h->tc_sample_div,
        h->t_keys.p, h->t_vals.p, stat);
    FDB_LAUNCH_CHECK();
    h->t_plen.ensure(np + 1);
    h->t_seg.ensure(np + 1);
    size_t tmp_sort = 0, tmp_seg = 0;
    const int end_bit = bits_for((uint32_t)nkeys);
    FDB_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, tmp_sort, h->t_keys.p, h->t_keys.p + np,
                                             h->t_vals.p, h->t_vals.p + np, (int)np, 0, end_bit,
                                             s));
    FDB_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, tmp_seg, h->t_plen.p, h->t_seg.p,
                                           (int)np + 1, s));
    h->t_tmp.ensure(std::max(tmp_sort, tmp_seg));
    FDB_CUDA(cub::DeviceRadixSort::SortPairs(h->t_tmp.p, tmp_sort, h->t_keys.p, h->t_keys.p + np,
                                             h->t_vals.p, h->t_vals.p + np, (int)np, 0, end_bit,
                                             s));
    seg_offsets_kernel<<<(unsigned)((np + 1 + 255) / 256), 256, 0, s>>>(
        h->t_keys.p + np, (unsigned)np, nkeys, h->t_off.p);
    FDB_LAUNCH_CHECK();
    const uint32_t* svals = h->t_vals.p + np;
    // --- residual rows, dump rows and items ---
    h->t_a16.ensure(np * dpad);
    h->t_pq.ensure(np);
    h->t_rn.ensure(np);
    h->t_s2.ensure(np);
    h->t_qbad.ensure(nq);
    h->t_inv.ensure(np);
    FDB_CUDA(cudaMemsetAsync(h->t_qbad.p, 0, nq * 4, s));
    FDB_CUDA(cudaMemsetAsync(h->t_inv.p, 0xff, np * 4, s));
    const unsigned rows_grid =
        (unsigned)std::min<size_t>((np * 32 + 255) / 256, (size_t)c.sm_count * 8);
    build_a_kernel<<<rows_grid, 256, 0, s>>>(
        svals, h->t_off.p, nlist, (int)take, probes, dQ, h->cents.p, (int)h->dim, dpad, pdist,
        h->tc_sb, h->t_a16.p, h->t_pq.p, h->t_rn.p, h->t_s2.p, h->t_qbad.p, h->t_inv.p);
    FDB_LAUNCH_CHECK();
    plen_kernel<<<(unsigned)((np + 1 + 255) / 256), 256, 0, s>>>(
        svals, h->t_off.p, nlist, probes, lbeg, lend, (int)np + 1, h->t_plen.p);
    FDB_LAUNCH_CHECK();
    FDB_CUDA(cub::DeviceScan::ExclusiveSum(h->t_tmp.p, tmp_seg, h->t_plen.p, h->t_seg.p,
                                           (int)np + 1, s));
    // a whole (padded) list per pass-1 pair, one tile per other pair
    h->t_dump.ensure(std::max<size_t>(1, nq * h->tc_maxpad + np * TILE_N));
    // items per (kind, list) = ceil(P / 128) * ceil(tiles / CHUNK_TILES) <= (a + 1)(b + 1)
    // with a = P / 128, b = tiles / CHUNK_TILES: the whole-list kinds (0 and 2)
    // plus the first-tile kind (1, one chunk per row block)
    const size_t max_tiles = h->tc_maxpad / TILE_N;
    const size_t all_tiles = h->tc_rows / TILE_N;
    const size_t max_items = np * ((max_tiles + CHUNK_TILES - 1) / CHUNK_TILES) / TILE_M +
                             np / TILE_M + 2 * (all_tiles / CHUNK_TILES + 1) +
                             2 * (size_t)nlist + (np / TILE_M + nlist) + 2 +
                             (all_tiles / CHUNK_TILES + 1) + 2 * (size_t)nlist;
    h->t_items.ensure(max_items * sizeof(Item));
    Item* items = reinterpret_cast<Item*>(h->t_items.p);
    // items of slots [s0, s0 + nslot): count, exclusive sum, fill
    h->t_icnt.ensure(2 * (3 * (size_t)nlist + 1));
    auto make_items = [&](int s0, int nslot, const unsigned* poff2) {
        unsigned* icnt = h->t_icnt.p;
        unsigned* ioff = h->t_icnt.p + nslot + 1;
        item_count_kernel<<<(unsigned)((nslot + 1 + 255) / 256), 256, 0, s>>>(
            h->t_off.p, poff2, nlist, s0, nslot, h->lorder.p, lbeg, lend, icnt);
        FDB_LAUNCH_CHECK();
        size_t tmp_items = 0;
        FDB_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, tmp_items, icnt, ioff, nslot + 1, s));
        h->t_tmp2.ensure(std::max<size_t>(tmp_items, 1));
        FDB_CUDA(cub::DeviceScan::ExclusiveSum(h->t_tmp2.p, tmp_items, icnt, ioff, nslot + 1, s));
        item_fill_kernel<<<(unsigned)((nslot + 7) / 8), 256, 0, s>>>(
            h->t_off.p, poff2, nlist, s0, nslot, h->lorder.p, lbeg, lend, h->tc_pstart.p, ioff,
            items, (unsigned)max_items, h->t_range.p);
        FDB_LAUNCH_CHECK();
    };
    make_items(0, 2 * nlist, nullptr);  // pass 1: whole pass-1 lists, first tiles
    // --- pass 1: distances of each query's first list; its top-64 and tau ---
    const CUtensorMap am = make_map(h->t_a16.p, np, dpad);
    const CUtensorMap bm = make_map(h->dec16.p, h->tc_rows, dpad);
    const int cap = 4096;  // candidates per query (uniform data can admit a few thousand)
    h->t_part.ensure(nq * LIST_K);
    h->t_tau.ensure(nq);
    h->t_cand_cnt.ensure(nq);
    h->t_cand.ensure(nq * (size_t)cap);
    FDB_CUDA(cudaMemsetAsync(h->t_cand_cnt.p, 0, nq * 4, s));
    PassParams p{};
    p.items = items;
    p.range = h->t_range.p;
    p.katoms = dpad / KATOM;
    p.pair_q = h->t_pq.p;
    p.pair_rn = h->t_rn.p;
    p.pair_s2 = h->t_s2.p;
    p.colv = h->tc_colv ? h->tc_colv : h->dnorm.p;
    p.colmax = h->tc_colmax;
    p.dump = h->t_dump.p;
    p.seg = h->t_seg.p;
    p.tau = h->t_tau.p;
    p.cand = h->t_cand.p;
    p.cand_cnt = h->t_cand_cnt.p;
    p.cap = cap;
    p.err = err;
    p.wait = wait_limit_cycles(c, h->call_wait_cycles);
    p.stall = take_test_stall(c) ? 1 : 0;
    p.next = h->t_range.p + 5;
    FDB_CUDA(cudaMemsetAsync(h->t_range.p + 5, 0, 8, s));
    h->t_qrange.ensure(2 * nq);
    FDB_CUDA(cudaMemsetAsync(h->t_qrange.p, 0xff, 2 * nq * 4, s));
    p.lo = h->t_qrange.p;
    p.hi = h->t_qrange.p + nq;
    const int grid = c.sm_count;
    launch_pass<EPI_DUMP>(s, am, bm, grid, p);
    select1_kernel<<<(unsigned)((nq + 7) / 8), 256, 0, s>>>(
        h->t_dump.p, h->t_seg.p, h->t_inv.p, h->t_off.p, nlist, probes, (int)take, lbeg, lend,
        (int)nq, h->t_qrange.p, h->t_qrange.p + nq, h->t_part.p, h->t_tau.p);
    FDB_LAUNCH_CHECK();
    if (h->sharded) {
        // the device holding a query's pass-1 list sets its threshold (+inf elsewhere)
        comm_mark(c, COMM_TAU);
        FDB_NCCL_C(ncclAllReduce(h->t_tau.p, h->t_tau.p, nq, ncclFloat, ncclMin, c.comm, s), c.comm);
        comm_mark(c, COMM_TAU);
    }
    // --- pass 2: the other lists against tau + the certification margin ---
    h->t_tadm.ensure(nq);
    h->t_eb.ensure(nq);
    margin_kernel<<<(unsigned)((nq + 7) / 8), 256, 0, s>>>(
        dQ, (int)nq, (int)h->dim, (int)h->m, h->cmax.p, h->bmax.p, probes, pdist, (int)take,
        lbeg, lend, h->tc_rhl.p, h->t_tau.p, h->t_tadm.p, h->t_eb.p);
    FDB_LAUNCH_CHECK();
    // --- drop the pass-2 pairs whose list cannot admit a code; compact the rest ---
    h->t_live.ensure(2 * (2 * (size_t)nlist + 1));
    h->t_pflag.ensure(np);
    h->t_sel.ensure(np + 1);
    unsigned* live = h->t_live.p;
    unsigned* live_off = h->t_live.p + 2 * nlist + 1;
    FDB_CUDA(cudaMemsetAsync(live, 0, (2 * (size_t)nlist + 1) * 4, s));
    prune_kernel<<<(unsigned)((np + 255) / 256), 256, 0, s>>>(
        h->t_keys.p + np, h->t_off.p, nlist, (unsigned)np, h->t_pq.p, h->t_rn.p, h->tc_rhl.p,
        h->t_tadm.p, lbeg, lend, h->t_pflag.p, live, stat);
    FDB_LAUNCH_CHECK();
    {
        size_t t1 = 0, t2 = 0;
        cub::CountingInputIterator<unsigned> ids(0u);
        FDB_CUDA(cub::DeviceSelect::Flagged(nullptr, t1, ids, h->t_pflag.p, h->t_sel.p + 1,
                                            h->t_sel.p, (int)np, s));
        FDB_CUDA(cub::DeviceScan::ExclusiveSum(nullptr, t2, live, live_off, 2 * nlist + 1, s));
        h->t_tmp3.ensure(std::max<size_t>(std::max(t1, t2), 1));
        FDB_CUDA(cub::DeviceSelect::Flagged(h->t_tmp3.p, t1, ids, h->t_pflag.p, h->t_sel.p + 1,
                                            h->t_sel.p, (int)np, s));
        FDB_CUDA(cub::DeviceScan::ExclusiveSum(h->t_tmp3.p, t2, live, live_off, 2 * nlist + 1,
                                               s));
    }
    h->t_a2.ensure(np * dpad);
    h->t_q2.ensure(np);
    h->t_rn2.ensure(np);
    h->t_s22.ensure(np);
    build_a2_kernel<<<rows_grid, 256, 0, s>>>(
        h->t_sel.p + 1, h->t_sel.p, svals, (int)take, probes, dQ, h->cents.p, (int)h->dim, dpad,
        pdist, h->tc_sb, h->t_a2.p, h->t_q2.p, h->t_rn2.p, h->t_s22.p, h->t_qbad.p);
    FDB_LAUNCH_CHECK();
    make_items(2 * nlist, 2 * nlist, live_off);  // pass 2: the kept pairs' lists
    const CUtensorMap am2 = make_map(h->t_a2.p, np, dpad);
    p.pair_q = h->t_q2.p;
    p.pair_rn = h->t_rn2.p;
    p.pair_s2 = h->t_s22.p;
    p.tau = h->t_tadm.p;
    p.range = h->t_range.p + 2;
    p.next = h->t_range.p + 6;
    p.stall = take_test_stall(c) ? 1 : 0;
    if (pass_tm) pass_tm->mark();
    launch_pass<EPI_FILTER>(s, am2, bm, grid, p);
    if (pass_tm) pass_tm->mark();
    // --- shortlist, exact rescoring, certification ---
    h->s_approx.ensure(nq * LIST_K);
    select_kernel<<<(unsigned)((nq + 7) / 8), 256, 0, s>>>(h->t_part.p, h->t_cand.p,
                                                           h->t_cand_cnt.p, cap, (int)nq,
                                                           h->t_tau.p, h->s_approx.p);
    FDB_LAUNCH_CHECK();
    CertParams r{};
    r.Q = dQ;
    r.nq = (int)nq;
    r.dim = (int)h->dim;
    r.m = (int)h->m;
    r.cents = h->cents.p;
    r.cb = h->cb.p;
    r.offs_full = h->offs.p;
    r.nlist = nlist;
    r.codes = h->codes.p;
    r.approx = h->s_approx.p;
    r.k = (int)k;
    r.out_keys = out_keys;
    r.cmax = h->cmax.p;
    r.bmax = h->bmax.p;
    r.cand_cnt = h->t_cand_cnt.p;
    r.cap = cap;
    r.tau = h->t_tau.p;
    r.pdist = pdist;
    r.probes = probes;
    r.take = (int)take;
    r.lbeg = lbeg;
    r.lend = lend;
    r.rh = h->tc_rhl.p;
    r.qbad = h->t_qbad.p;
    r.qbase = qbase;
    r.flag_count = flags;
    r.flag_list = flags + 1;
    r.fail_probes = fail_probes;
    r.fail_cnt = fail_cnt;
    h->t_ekeys.ensure(nq * LIST_K);
    h->t_elist.ensure(nq * LIST_K);
    h->t_dk.ensure(nq);
    r.ekeys = h->t_ekeys.p;
    r.elist = h->t_elist.p;
    r.dk = h->t_dk.p;
    h->t_ext.ensure(2 * nq + 2);
    h->t_ext_thr.ensure(nq);
    FDB_CUDA(cudaMemsetAsync(h->t_ext.p, 0, 4, s));
    FDB_CUDA(cudaMemsetAsync(h->t_ext.p + nq + 1, 0, 4, s));
    r.over_count = h->t_ext.p + nq + 1;
    r.over_list = h->t_ext.p + nq + 2;
    r.part = h->t_part.p;
    r.cand = h->t_cand.p;
    r.ext_count = h->t_ext.p;
    r.ext_list = h->t_ext.p + 1;
    r.ext_thr = h->t_ext_thr.p;
    r.stat = stat;
    r.tadm = h->t_tadm.p;
    r.ebound = h->t_eb.p;
    r.dump = h->t_dump.p;
    r.seg = h->t_seg.p;
    r.inv = h->t_inv.p;
    r.poff = h->t_off.p;
    const unsigned cgrid = (unsigned)((nq + CERT_WARPS - 1) / CERT_WARPS);
    const unsigned rgrid = (unsigned)((nq + RS_QUERIES - 1) / RS_QUERIES);
    const bool p2 = k > 32;
    // compile-time ADC shapes for the common layouts (rows 16-byte aligned)
    const int sub = (int)(h->dim / h->m);
    const int ms = (h->m == 16 && sub == 8) ? 1 : (h->m == 48 && sub == 2) ? 2 : 0;
#define FDB_RESCORE(O, PP, MM) rescore_kernel<O, PP, MM><<<rgrid, CERT_WARPS * 32, 0, s>>>(r)
#define FDB_RESCORE_MS(O, PP)                  \
    if (ms == 1) { FDB_RESCORE(O, PP, 1); }    \
    else if (ms == 2) { FDB_RESCORE(O, PP, 2); } \
    else { FDB_RESCORE(O, PP, 0); }
    if (order == ORDER_LANE8) {
        if (p2) { FDB_RESCORE_MS(ORDER_LANE8, 2) }
        else { FDB_RESCORE_MS(ORDER_LANE8, 1) }
    } else {
        if (p2) { FDB_RESCORE_MS(ORDER_FAST4, 2) }
        else { FDB_RESCORE_MS(ORDER_FAST4, 1) }
    }
#undef FDB_RESCORE_MS
#undef FDB_RESCORE
    FDB_LAUNCH_CHECK();
    if (h->sharded) {
        // the answer's k-th distance is at most the smallest exact k-th of any device
        comm_mark(c, COMM_DK);
        FDB_NCCL_C(ncclAllReduce(h->t_dk.p, h->t_dk.p, nq, ncclFloat, ncclMin, c.comm, s), c.comm);
        comm_mark(c, COMM_DK);
    }
    if (p2) certify_kernel<2><<<cgrid, CERT_WARPS * 32, 0, s>>>(r, 0);
    else certify_kernel<1><<<cgrid, CERT_WARPS * 32, 0, s>>>(r, 0);
    FDB_LAUNCH_CHECK();
    // extended queries (a block each, in turn); those with too many entries
    // then take the re-scan path
    const unsigned egrid = (unsigned)std::min<size_t>(nq, (size_t)c.sm_count * 8);
#define FDB_EXTEND(O, PP, MM) extend_kernel<O, PP, MM><<<egrid, EXT_THREADS, 0, s>>>(r)
#define FDB_EXTEND_MS(O, PP)                   \
    if (ms == 1) { FDB_EXTEND(O, PP, 1); }     \
    else if (ms == 2) { FDB_EXTEND(O, PP, 2); } \
    else { FDB_EXTEND(O, PP, 0); }
    if (order == ORDER_LANE8) {
        if (p2) { FDB_EXTEND_MS(ORDER_LANE8, 2) }
        else { FDB_EXTEND_MS(ORDER_LANE8, 1) }
    } else {
        if (p2) { FDB_EXTEND_MS(ORDER_FAST4, 2) }
        else { FDB_EXTEND_MS(ORDER_FAST4, 1) }
    }
#undef FDB_EXTEND_MS
#undef FDB_EXTEND
    FDB_LAUNCH_CHECK();
    if (p2) certify_kernel<2><<<cgrid, CERT_WARPS * 32, 0, s>>>(r, 1);
    else certify_kernel<1><<<cgrid, CERT_WARPS * 32, 0, s>>>(r, 1);
    FDB_LAUNCH_CHECK();
}

}  // namespace

// Tensor-core shortlist + exact rescoring of nq queries whose probes and
// their coarse distances are in h->s_probe / h->s_pdist, enqueued without a
// host synchronisation.  Writes [nq][k] exact keys and lists uncertified
// queries in flags (flags[0] = count, then indices); for each listed query,
// t_fprobes / t_fcnt name the lists to re-scan exactly (ivf_tc_rescan) and its
// out_keys row holds the seed (the exact top-k of its shortlisted codes in
// the other lists).  A bounded wait that ran out sets the word that
// ivf_tc_error_word names.  Queries run in chunks that keep the pass-1 dump
// (one row of distances per query, sized for the longest list) within 4 GiB:
// every chunk re-reads the lists it probes and fills its list-scan items with
// fewer pair rows, so one chunk per batch is best.  pass_tm (nullable) gets a
// mark before and after each pass-2 launch.
void ivf_tc_search(fdb_ivfpq* h, const float* dQ, size_t nq, size_t k, int order, size_t take,
                   const uint64_t* lbeg, const uint64_t* lend, uint64_t* out_keys,
                   uint32_t* flags, unsigned long long* stat, StageTimer* pass_tm) {
    Ctx& c = h->ctx->c;
    cudaStream_t s = c.stream;
    FDB_REQUIRE(nq * take < (1ull << 31), FDB_ERR_UNSUPPORTED, "too many (query, list) pairs");
    const size_t budget = (size_t)1 << 30;  // floats
    const size_t per_query = h->tc_maxpad + take * ivtc::TILE_N;  // dump floats per query
    const size_t chunk = std::max<size_t>(1, std::min(nq, budget / per_query));
    h->t_range.ensure(8);
    h->t_fprobes.ensure(nq * take);
    h->t_fcnt.ensure(nq);
    int* err = ivf_tc_error_word(h);  // cleared by the caller at the start of the call
    FDB_CUDA(cudaMemsetAsync(flags, 0, 4, s));
    for (size_t q0 = 0; q0 < nq; q0 += chunk) {
        const size_t nc = std::min(chunk, nq - q0);
        tc_chunk(h, dQ + q0 * h->dim, nc, k, order, take, h->s_probe.p + q0 * take,
                 h->s_pdist.p + q0 * take, lbeg, lend, out_keys + q0 * k, flags,
                 (uint32_t)q0, stat, err, h->t_fprobes.p, h->t_fcnt.p, pass_tm);
    }
}

int* ivf_tc_error_word(fdb_ivfpq* h) {
    h->t_range.ensure(8);
    return reinterpret_cast<int*>(h->t_range.p + 4);
}

}  // namespace fdb

namespace fdb {

// Exact re-scan of the lists that failed certification, driven by the
// counts on the device (no host synchronisation): one block per (flagged
// query, failed list) unit computes that list's exact top-k, and each flagged
// query's seed and lists are merged into its out_keys row.  Units run in
// rounds of at most ucap, which bounds the per-unit key buffer; one round
// covers every unit the batch can produce unless nq * take * k is large.
void ivf_tc_rescan(fdb_ivfpq* h, const ScanParams& base, size_t nq, size_t k, int order,
                   uint64_t* out_keys) {
    if (nq == 0) return;
    cudaStream_t s = h->ctx->c.stream;
    const size_t take = (size_t)base.nprobe;
    const size_t worst = nq * take;
    const size_t key_budget = (size_t)64 << 20;  // bytes of per-unit keys
    const size_t ucap = std::max<size_t>(1, std::min(worst, key_budget / (k * sizeof(uint64_t))));
    FDB_REQUIRE(worst < (1ull << 31), FDB_ERR_UNSUPPORTED, "too many (query, list) units");
    h->t_uoff.ensure(nq + 2);  // offsets per flag slot, then the unit count
    h->t_unit_q.ensure(ucap);
    h->t_unit_l.ensure(ucap);
    h->t_unit_keys.ensure(ucap * k);
    uint32_t* nunits = h->t_uoff.p + nq + 1;
    const uint32_t* flags = h->s_flags.p;
    ivtc::unit_offsets_kernel<<<1, 1024, 0, s>>>(flags, h->t_fcnt.p, h->t_uoff.p, nunits);
    FDB_LAUNCH_CHECK();
    const int sms = h->ctx->c.sm_count;
    const unsigned mgrid = (unsigned)std::min<size_t>((nq + 7) / 8, (size_t)sms * 8);
    for (size_t r0 = 0; r0 < worst; r0 += ucap) {
        ivtc::expand_units_kernel<<<(unsigned)((nq + 127) / 128), 128, 0, s>>>(
            flags, (int)take, h->t_fprobes.p, h->t_uoff.p, (uint32_t)r0, (uint32_t)ucap,
            h->t_unit_q.p, h->t_unit_l.p);
        FDB_LAUNCH_CHECK();
        ScanParams e = base;
        e.nq = (int)ucap;
        e.nq_dev = nunits;
        e.nq_dev_base = (uint32_t)r0;
        e.grid_cap = sms * 8;
        e.qidx = h->t_unit_q.p;
        e.probe_list = h->t_unit_l.p;
        e.probe_cnt = nullptr;
        e.nprobe = 1;
        e.k = (int)k;
        e.out_keys = h->t_unit_keys.p;
        e.out_by_block = true;
        e.seed = false;
        e.stat = nullptr;
        e.btab = nullptr;
        launch_scan(s, e, order);
        if (k > 32)
            ivtc::merge_units_kernel<2><<<mgrid, 256, 0, s>>>(
                (int)k, flags, h->t_uoff.p, (uint32_t)r0, (uint32_t)ucap, h->t_unit_keys.p,
                out_keys);
        else
            ivtc::merge_units_kernel<1><<<mgrid, 256, 0, s>>>(
                (int)k, flags, h->t_uoff.p, (uint32_t)r0, (uint32_t)ucap, h->t_unit_keys.p,
                out_keys);
        FDB_LAUNCH_CHECK();
    }
}

}  // namespace fdb
