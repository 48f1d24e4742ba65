// fdb_device.cuh -- device helpers shared by every kernel.
//
// 1. Distances in the reference's AVX2 summation order (bit-exact):
//    8 lane accumulators over i = j (mod 8) with fused multiply-add, a
//    left-to-right sum of the 8 lanes, then an unfused scalar tail
//    (forge-db src/distance/simd.rs:338-366, 427-456, 469-517).  All
//    arithmetic goes through __f*_rn intrinsics and the translation units are
//    built with -fmad=false, so the compiler cannot re-associate or contract.
// 2. Orderable 64-bit keys: (monotone image of the f32 distance) << 32 | tag.
//    Ascending key order is ascending distance with ties broken by the tag
//    (a row position), which makes every top-k result unique and independent
//    of how the rows are split across warps, blocks or devices.
// 3. WarpTopK: a warp-wide sorted list of the K = 32*P smallest keys held in
//    registers, fed through a per-warp shared-memory buffer and merged 32
//    candidates at a time with a bitonic network.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace fdb {

constexpr int KSUB = 256;              // codewords per PQ subspace (constants.rs:10)
constexpr uint64_t KEY_NONE = ~0ull;   // empty slot: sorts after every real key

// ---------------------------------------------------------------------------
// orderable keys
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t f2ord(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float ord2f(uint32_t o) {
    uint32_t u = (o & 0x80000000u) ? (o & 0x7fffffffu) : ~o;
    return __uint_as_float(u);
}
__device__ __forceinline__ uint64_t make_key(float d, uint32_t tag) {
    return ((uint64_t)f2ord(d) << 32) | tag;
}
__device__ __forceinline__ float key_dist(uint64_t key) { return ord2f((uint32_t)(key >> 32)); }
__device__ __forceinline__ uint32_t key_tag(uint64_t key) { return (uint32_t)key; }

// ---------------------------------------------------------------------------
// exact-order distances (generic length, any alignment)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float lane_sum(const float (&acc)[8]) {
    float t = acc[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) t = __fadd_rn(t, acc[j]);
    return t;
}

// euclidean_distance_squared_avx2 (simd.rs:338-366)
__device__ __forceinline__ float l2sq_exact(const float* a, const float* b, int len) {
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
    int i = 0;
    for (; i + 8 <= len; i += 8) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            float d = __fsub_rn(a[i + j], b[i + j]);
            acc[j] = __fmaf_rn(d, d, acc[j]);
        }
    }
    float t = lane_sum(acc);
    for (; i < len; ++i) {
        float d = __fsub_rn(a[i], b[i]);
        t = __fadd_rn(t, __fmul_rn(d, d));
    }
    return t;
}

// Exact L2^2 of one query row (shared or global memory; the same address in
// every lane of a warp is a broadcast) and NC other rows in global memory, in
// the order of l2sq_exact, the NC rows interleaved for memory-level
// parallelism; 128-bit loads when the rows are 16-byte aligned.
// DIM > 0: a compile-time length (a multiple of 8, the rows 16-byte
// aligned), every loop unrolled so that all loads of a row are in flight
// together; DIM == 0: the run-time length dim.
template <int NC, int DIM = 0>
__device__ __forceinline__ void l2sq_rows(const float* __restrict__ qs,
                                          const float* const (&c)[NC], int dim, bool vec,
                                          float (&out)[NC]) {
    float acc[NC][8];
#pragma unroll
    for (int r = 0; r < NC; ++r)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[r][j] = 0.0f;
    if constexpr (DIM > 0) {
        static_assert(DIM % 8 == 0, "whole lane groups");
        const float4* q4 = reinterpret_cast<const float4*>(qs);
#pragma unroll
        for (int i = 0; i < DIM; i += 8) {
            const float4 qa = q4[i >> 2], qb = q4[(i >> 2) + 1];
            const float qv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
            for (int r = 0; r < NC; ++r) {
                const float4* c4 = reinterpret_cast<const float4*>(c[r]);
                const float4 u = __ldg(c4 + (i >> 2)), w = __ldg(c4 + (i >> 2) + 1);
                const float cv[8] = {u.x, u.y, u.z, u.w, w.x, w.y, w.z, w.w};
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float d = __fsub_rn(qv[j], cv[j]);
                    acc[r][j] = __fmaf_rn(d, d, acc[r][j]);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < NC; ++r) out[r] = lane_sum(acc[r]);
        return;
    }
    const int full = dim & ~7;
    if (vec) {
        const float4* q4 = reinterpret_cast<const float4*>(qs);
#pragma unroll 2
        for (int i = 0; i < full; i += 8) {
            const float4 qa = q4[i >> 2], qb = q4[(i >> 2) + 1];
            const float qv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
            float cv[NC][8];
#pragma unroll
            for (int r = 0; r < NC; ++r) {
                const float4* c4 = reinterpret_cast<const float4*>(c[r]);
                const float4 u = __ldg(c4 + (i >> 2)), w = __ldg(c4 + (i >> 2) + 1);
                cv[r][0] = u.x; cv[r][1] = u.y; cv[r][2] = u.z; cv[r][3] = u.w;
                cv[r][4] = w.x; cv[r][5] = w.y; cv[r][6] = w.z; cv[r][7] = w.w;
            }
#pragma unroll
            for (int r = 0; r < NC; ++r)
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float d = __fsub_rn(qv[j], cv[r][j]);
                    acc[r][j] = __fmaf_rn(d, d, acc[r][j]);
                }
        }
    } else {
        for (int i = 0; i < full; i += 8) {
#pragma unroll
            for (int r = 0; r < NC; ++r)
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float d = __fsub_rn(qs[i + j], __ldg(c[r] + i + j));
                    acc[r][j] = __fmaf_rn(d, d, acc[r][j]);
                }
        }
    }
#pragma unroll
    for (int r = 0; r < NC; ++r) {
        float t = lane_sum(acc[r]);
        for (int i = full; i < dim; ++i) {
            const float d = __fsub_rn(qs[i], __ldg(c[r] + i));
            t = __fadd_rn(t, __fmul_rn(d, d));
        }
        out[r] = t;
    }
}

// dot_product_avx2 (simd.rs:427-456)
__device__ __forceinline__ float dot_exact(const float* a, const float* b, int len) {
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
    int i = 0;
    for (; i + 8 <= len; i += 8) {
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = __fmaf_rn(a[i + j], b[i + j], acc[j]);
    }
    float t = lane_sum(acc);
    for (; i < len; ++i) t = __fadd_rn(t, __fmul_rn(a[i], b[i]));
    return t;
}

// dot_exact of one row against NC rows, the NC rows interleaved (as
// l2sq_rows).  DIM > 0: a compile-time length (a multiple of 8, the rows
// 16-byte aligned), every load in flight together; DIM == 0: one dot_exact
// per row.
template <int NC, int DIM>
__device__ __forceinline__ void dot_rows(const float* __restrict__ qs,
                                         const float* const (&c)[NC], int dim,
                                         float (&out)[NC]) {
    if constexpr (DIM == 0) {
#pragma unroll
        for (int r = 0; r < NC; ++r) out[r] = dot_exact(qs, c[r], dim);
    } else {
        static_assert(DIM % 8 == 0, "whole lane groups");
        float acc[NC][8];
#pragma unroll
        for (int r = 0; r < NC; ++r)
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[r][j] = 0.0f;
        const float4* q4 = reinterpret_cast<const float4*>(qs);
#pragma unroll
        for (int i = 0; i < DIM; i += 8) {
            const float4 qa = q4[i >> 2], qb = q4[(i >> 2) + 1];
            const float qv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
            for (int r = 0; r < NC; ++r) {
                const float4* c4 = reinterpret_cast<const float4*>(c[r]);
                const float4 u = __ldg(c4 + (i >> 2)), w = __ldg(c4 + (i >> 2) + 1);
                const float cv[8] = {u.x, u.y, u.z, u.w, w.x, w.y, w.z, w.w};
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[r][j] = __fmaf_rn(qv[j], cv[j], acc[r][j]);
            }
        }
#pragma unroll
        for (int r = 0; r < NC; ++r) out[r] = lane_sum(acc[r]);
    }
}

// manhattan_distance_avx2 (simd.rs:378-418)
__device__ __forceinline__ float l1_exact(const float* a, const float* b, int len) {
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
    int i = 0;
    for (; i + 8 <= len; i += 8) {
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = __fadd_rn(acc[j], fabsf(__fsub_rn(a[i + j], b[i + j])));
    }
    float t = lane_sum(acc);
    for (; i < len; ++i) t = __fadd_rn(t, fabsf(__fsub_rn(a[i], b[i])));
    return t;
}

// cosine_distance_avx2 (simd.rs:469-517) from a dot product and the two
// squared norms, each already summed in the AVX2 order.
__device__ __forceinline__ float cosine_from(float dot, float na, float nb) {
    float np = __fsqrt_rn(__fmul_rn(na, nb));
    if (np == 0.0f) return 0.0f;
    return __fsub_rn(1.0f, __fdiv_rn(dot, np));
}

enum Metric : int { EUCLIDEAN = 0, EUCLIDEAN_SQUARED = 1, COSINE = 2, DOT_PRODUCT = 3, MANHATTAN = 4 };

// ---------------------------------------------------------------------------
// PQ asymmetric distance summation orders
// ---------------------------------------------------------------------------
// ORDER_LANE8: asymmetric_distance_simd_avx2 / batch_asymmetric_distance_avx2
//   (pq.rs:318-402, 435-485): lane j sums t[j], t[j+8], ... over full groups of
//   8 subspaces; lanes summed left to right; serial tail.  Used by batch_search.
// ORDER_FAST4: asymmetric_distance_fast (pq.rs:218-245): running sum of
//   ((t0+t1)+t2)+t3 per group of 4, serial tail.  Used by search.
constexpr int ORDER_LANE8 = 0;
constexpr int ORDER_FAST4 = 1;

template <int ORDER>
__device__ __forceinline__ float adc_sum(const float* t, int m) {
    if (ORDER == ORDER_LANE8) {
        int full = m & ~7;
        float total;
        if (full > 0) {
            float acc[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) acc[j] = t[j];
            for (int i = 8; i < full; i += 8) {
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[j] = __fadd_rn(acc[j], t[i + j]);
            }
            total = lane_sum(acc);
        } else {
            total = 0.0f;
        }
        for (int i = full; i < m; ++i) total = __fadd_rn(total, t[i]);
        return total;
    } else {
        float sum = 0.0f;
        int i = 0;
        for (; i + 4 <= m; i += 4) {
            float g = __fadd_rn(__fadd_rn(__fadd_rn(t[i], t[i + 1]), t[i + 2]), t[i + 3]);
            sum = __fadd_rn(sum, g);
        }
        for (; i < m; ++i) sum = __fadd_rn(sum, t[i]);
        return sum;
    }
}

// ---------------------------------------------------------------------------
// warp top-k
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint64_t kmin(uint64_t a, uint64_t b) { return a < b ? a : b; }
__device__ __forceinline__ uint64_t kmax(uint64_t a, uint64_t b) { return a < b ? b : a; }

// Sort one key per lane ascending across the warp (bitonic network).
__device__ __forceinline__ uint64_t warp_sort32(uint64_t c, int lane) {
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            uint64_t o = __shfl_xor_sync(0xffffffffu, c, stride);
            bool up = (lane & size) == 0;
            bool lower = (lane & stride) == 0;
            c = (lower == up) ? kmin(c, o) : kmax(c, o);
        }
    }
    return c;
}

// Entry i of the sorted list lives in register i / 32 of lane i % 32.
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

// One exact LUT entry: L2^2(fl(q_s - c_s) - b) in the AVX2 order, for
// subspace s of length sub and codeword b.
__device__ __forceinline__ float exact_lut_entry(const float* __restrict__ qs,
                                                 const float* __restrict__ cs,
                                                 const float* __restrict__ b, int sub) {
    {
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
        int i = 0;
        if (((reinterpret_cast<uintptr_t>(qs) | reinterpret_cast<uintptr_t>(cs) |
              reinterpret_cast<uintptr_t>(b)) & 15) == 0) {
            // same operations, operands fetched with 128-bit loads
            for (; i + 8 <= sub; i += 8) {
                const float4 q0 = __ldg(reinterpret_cast<const float4*>(qs + i));
                const float4 q1 = __ldg(reinterpret_cast<const float4*>(qs + i + 4));
                const float4 c0 = __ldg(reinterpret_cast<const float4*>(cs + i));
                const float4 c1 = __ldg(reinterpret_cast<const float4*>(cs + i + 4));
                const float4 b0 = __ldg(reinterpret_cast<const float4*>(b + i));
                const float4 b1 = __ldg(reinterpret_cast<const float4*>(b + i + 4));
                const float qa[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
                const float ca[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
                const float ba[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    float d = __fsub_rn(__fsub_rn(qa[j], ca[j]), ba[j]);
                    acc[j] = __fmaf_rn(d, d, acc[j]);
                }
            }
        }
        for (; i + 8 <= sub; i += 8) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                float d = __fsub_rn(__fsub_rn(__ldg(qs + i + j), __ldg(cs + i + j)), __ldg(b + i + j));
                acc[j] = __fmaf_rn(d, d, acc[j]);
            }
        }
        float t = lane_sum(acc);
        for (; i < sub; ++i) {
            float d = __fsub_rn(__fsub_rn(__ldg(qs + i), __ldg(cs + i)), __ldg(b + i));
            t = __fadd_rn(t, __fmul_rn(d, d));
        }
        return t;
    }
}

// Exact ADC of one code: every LUT entry recomputed as L2^2(fl(q - c) - b)
// in the AVX2 order and summed in the requested order -- the same
// operations, in the same order, as the exact-mode scan.
template <int ORDER>
__device__ __forceinline__ float exact_adc(const float* __restrict__ q,
                                           const float* __restrict__ c,
                                           const float* __restrict__ cb,
                                           const uint8_t* __restrict__ code, int m, int sub) {
    auto entry = [&](int s) -> float {
        return exact_lut_entry(q + s * sub, c + s * sub, cb + ((size_t)s * KSUB + code[s]) * sub,
                               sub);
    };
    return adc_order<ORDER>(entry, m);
}

// exact_adc for a compile-time shape (M subvectors of SUB floats, SUB a
// multiple of 4, the rows 16-byte aligned): every loop is unrolled, so the
// loads of all M entries can be in flight together instead of one entry's
// after another's.  Same operations in the same order as exact_adc.
template <int ORDER, int M, int SUB>
__device__ __forceinline__ float exact_adc_fixed(const float* __restrict__ q,
                                                 const float* __restrict__ c,
                                                 const float* __restrict__ cb,
                                                 const uint8_t* __restrict__ code) {
    static_assert(SUB % 4 == 0 || SUB == 2, "row segments of whole 128- or 64-bit loads");
    uint8_t cd[M];
#pragma unroll
    for (int s = 0; s < M; ++s) cd[s] = __ldg(code + s);
    float lut[M];
#pragma unroll
    for (int s = 0; s < M; ++s) {
        const float* qs = q + s * SUB;
        const float* cs = c + s * SUB;
        const float* b = cb + ((size_t)s * KSUB + cd[s]) * SUB;
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.0f;
        float t;
        if constexpr (SUB >= 8) {
#pragma unroll
            for (int i = 0; i + 8 <= SUB; i += 8) {
                const float4 q0 = __ldg(reinterpret_cast<const float4*>(qs + i));
                const float4 q1 = __ldg(reinterpret_cast<const float4*>(qs + i + 4));
                const float4 c0 = __ldg(reinterpret_cast<const float4*>(cs + i));
                const float4 c1 = __ldg(reinterpret_cast<const float4*>(cs + i + 4));
                const float4 b0 = __ldg(reinterpret_cast<const float4*>(b + i));
                const float4 b1 = __ldg(reinterpret_cast<const float4*>(b + i + 4));
                const float qa[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
                const float ca[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
                const float ba[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float d = __fsub_rn(__fsub_rn(qa[j], ca[j]), ba[j]);
                    acc[j] = __fmaf_rn(d, d, acc[j]);
                }
            }
            t = lane_sum(acc);
#pragma unroll
            for (int i = SUB & ~7; i < SUB; ++i) {
                const float d = __fsub_rn(__fsub_rn(__ldg(qs + i), __ldg(cs + i)), __ldg(b + i));
                t = __fadd_rn(t, __fmul_rn(d, d));
            }
        } else {
            // fewer than 8 floats: no full lane group, the unfused tail only
            t = lane_sum(acc);
#pragma unroll
            for (int i = 0; i < SUB; ++i) {
                const float d = __fsub_rn(__fsub_rn(__ldg(qs + i), __ldg(cs + i)), __ldg(b + i));
                t = __fadd_rn(t, __fmul_rn(d, d));
            }
        }
        lut[s] = t;
    }
    return adc_order<ORDER>([&](int i) { return lut[i]; }, M);
}

// The same value computed by a group of G lanes (G = 8, 16 or 32, m <= G,
// the warp split into 32 / G groups that all call this together): lane gl
// of the group computes LUT entry gl, and the entries are summed in the
// requested order through shuffles, so every operation and its order are
// those of exact_adc.  `code` is the group's code (may differ per group).
// Every lane of the group returns the total.
template <int ORDER, int G>
__device__ __forceinline__ float group_exact_adc(const float* __restrict__ q,
                                                 const float* __restrict__ c,
                                                 const float* __restrict__ cb,
                                                 const uint8_t* __restrict__ code, int m, int sub,
                                                 int gl, bool active) {
    float t = 0.0f;
    if (active && gl < m)
        t = exact_lut_entry(q + gl * sub, c + gl * sub,
                            cb + ((size_t)gl * KSUB + code[gl]) * sub, sub);
    auto at = [&](int i) { return __shfl_sync(0xffffffffu, t, i, G); };
    if (ORDER == ORDER_LANE8) {
        const int full = m & ~7;
        float total = 0.0f;
        if (full > 0) {
            // acc_j = t_j + t_{j+8} + ... (lane j < 8), then acc_0 + ... + acc_7
            float acc = t;
            for (int i = 8; i < full; i += 8) {
                const float o = __shfl_down_sync(0xffffffffu, t, i, G);
                acc = __fadd_rn(acc, o);
            }
            total = __shfl_sync(0xffffffffu, acc, 0, G);
#pragma unroll
            for (int j = 1; j < 8; ++j) total = __fadd_rn(total, __shfl_sync(0xffffffffu, acc, j, G));
        }
        for (int i = full; i < m; ++i) total = __fadd_rn(total, at(i));
        return total;
    } else {
        float sum = 0.0f;
        int i = 0;
        for (; i + 4 <= m; i += 4) {
            const float g = __fadd_rn(__fadd_rn(__fadd_rn(at(i), at(i + 1)), at(i + 2)), at(i + 3));
            sum = __fadd_rn(sum, g);
        }
        for (; i < m; ++i) sum = __fadd_rn(sum, at(i));
        return sum;
    }
}

// Exact distances of up to 32 codes, one per lane (row `pos` of `codes`, in
// list `list`; `valid` false for none), computed by lane groups of G; each
// lane gets its own code's distance.  dres: 32 floats of this warp's shared
// memory.  Whole warp.
template <int ORDER, int G>
__device__ __forceinline__ float warp_exact_adc_g(const float* __restrict__ qv,
                                                  const float* __restrict__ cents, int dim,
                                                  const float* __restrict__ cb,
                                                  const uint8_t* __restrict__ codes, int m,
                                                  int sub, uint32_t pos, int list, bool valid,
                                                  float* dres) {
    constexpr int NG = 32 / G;  // codes per round
    const int lane = threadIdx.x & 31, g = lane / G, gl = lane % G;
    const unsigned any = __ballot_sync(0xffffffffu, valid);
    for (int r0 = 0; r0 < 32; r0 += NG) {
        const int c = r0 + g;  // the code this lane's group computes this round
        const uint32_t cpos = __shfl_sync(0xffffffffu, pos, c);
        const int clist = __shfl_sync(0xffffffffu, list, c);
        const bool cval = (any >> c) & 1u;
        if (!__any_sync(0xffffffffu, cval)) continue;
        const float d = group_exact_adc<ORDER, G>(
            qv, cents + (size_t)(cval ? clist : 0) * dim, cb, codes + (size_t)cpos * m, m, sub,
            gl, cval);
        if (gl == 0) dres[c] = d;
    }
    __syncwarp();
    const float mine = dres[lane];
    __syncwarp();
    return valid ? mine : 0.0f;
}

template <int ORDER>
__device__ __forceinline__ float warp_exact_adc(const float* __restrict__ qv,
                                                const float* __restrict__ cents, int dim,
                                                const float* __restrict__ cb,
                                                const uint8_t* __restrict__ codes, int m, int sub,
                                                uint32_t pos, int list, bool valid,
                                                float* dres) {
    if (m <= 8)
        return warp_exact_adc_g<ORDER, 8>(qv, cents, dim, cb, codes, m, sub, pos, list, valid,
                                          dres);
    if (m <= 16)
        return warp_exact_adc_g<ORDER, 16>(qv, cents, dim, cb, codes, m, sub, pos, list, valid,
                                           dres);
    if (m <= 32)
        return warp_exact_adc_g<ORDER, 32>(qv, cents, dim, cb, codes, m, sub, pos, list, valid,
                                           dres);
    return valid ? exact_adc<ORDER>(qv, cents + (size_t)list * dim, cb, codes + (size_t)pos * m,
                                    m, sub)
                 : 0.0f;
}

template <int P>
struct WarpTopK {
    static constexpr int K = 32 * P;
    uint64_t L[P];
    uint64_t thr;     // key of entry k-1: only keys below it can enter
    int k;            // 1 <= k <= K
    int nbuf;         // warp-uniform count of buffered candidates
    uint64_t* buf;    // this warp's 64-entry shared buffer
    int lane;

    __device__ __forceinline__ void init(int k_, uint64_t* buf_) {
        lane = threadIdx.x & 31;
#pragma unroll
        for (int e = 0; e < P; ++e) L[e] = KEY_NONE;
        thr = KEY_NONE;
        k = k_;
        nbuf = 0;
        buf = buf_;
    }

    // Merge one candidate per lane (KEY_NONE for none) into the list.
    __device__ __forceinline__ void merge32(uint64_t c) {
        c = warp_sort32(c, lane);
        // Pair L[K-1-i] with candidate i: the result is bitonic and holds the
        // K smallest of both sequences.
        uint64_t o = __shfl_sync(0xffffffffu, c, 31 - lane);
        L[P - 1] = kmin(L[P - 1], o);
#pragma unroll
        for (int t = P / 2; t >= 1; t >>= 1) {
#pragma unroll
            for (int e = 0; e < P; ++e) {
                if ((e & t) == 0) {
                    uint64_t a = L[e], b = L[e + t];
                    L[e] = kmin(a, b);
                    L[e + t] = kmax(a, b);
                }
            }
        }
#pragma unroll
        for (int s = 16; s >= 1; s >>= 1) {
#pragma unroll
            for (int e = 0; e < P; ++e) {
                uint64_t v = __shfl_xor_sync(0xffffffffu, L[e], s);
                L[e] = ((lane & s) == 0) ? kmin(L[e], v) : kmax(L[e], v);
            }
        }
        uint64_t t = KEY_NONE;
        const int idx = k - 1;
#pragma unroll
        for (int e = 0; e < P; ++e)
            if (e == (idx >> 5)) t = L[e];
        thr = __shfl_sync(0xffffffffu, t, idx & 31);
    }

    // Offer one key per lane (all 32 lanes must call).
    __device__ __forceinline__ void add(uint64_t key, bool valid) {
        bool pass = valid && key < thr;
        unsigned mask = __ballot_sync(0xffffffffu, pass);
        if (mask == 0) return;
        if (pass) {
            int pos = nbuf + __popc(mask & ((1u << lane) - 1u));
            buf[pos] = key;
        }
        nbuf += __popc(mask);
        if (nbuf >= 32) {
            __syncwarp();
            uint64_t c = buf[lane];
            uint64_t rest = (lane + 32 < nbuf) ? buf[lane + 32] : KEY_NONE;
            __syncwarp();
            if (lane + 32 < nbuf) buf[lane] = rest;
            nbuf -= 32;
            __syncwarp();
            merge32(c);
        }
    }

    __device__ __forceinline__ void flush() {
        if (nbuf > 0) {
            __syncwarp();
            uint64_t c = (lane < nbuf) ? buf[lane] : KEY_NONE;
            __syncwarp();
            nbuf = 0;
            merge32(c);
        }
    }

    // Ingest n keys from memory (shared or global) as candidates.
    __device__ __forceinline__ void ingest(const uint64_t* keys, int n) {
        for (int base = 0; base < n; base += 32) {
            uint64_t c = (base + lane < n) ? keys[base + lane] : KEY_NONE;
            bool any = __any_sync(0xffffffffu, c < thr);
            if (any) merge32(c < thr ? c : KEY_NONE);
        }
    }

    // Write the first k entries to out[0..k).
    __device__ __forceinline__ void store(uint64_t* out) const {
#pragma unroll
        for (int e = 0; e < P; ++e) {
            int i = e * 32 + lane;
            if (i < k) out[i] = L[e];
        }
    }
};

// Threshold pre-pass for a warp's top-k over a stream of keys.  Offering
// every key to WarpTopK admits, for keys in arbitrary order, about
// k (1 + ln(n / k)) of them, each through a 64-bit bitonic merge; binning the
// keys first lets only the bins that hold the k smallest be offered.
// visit(f) must make the same warp-uniform sequence of f(key, valid) calls
// on every lane each time it runs (it runs twice here, and the caller's
// collecting pass is the third).  Bins split [min, max] of the keys' distance
// bits (the high 32 bits) into 256 ranges; the bin of a key never decreases
// as the key grows, so the keys in bins <= bstar are a prefix of the sorted
// keys holding at least k of them (all keys if there are fewer) and contain
// the k smallest.  hist: 256 words of this warp's shared memory.
struct KeyBins {
    uint32_t umin;
    float scale;
    int bstar;
    __device__ __forceinline__ bool keep(uint64_t key) const {
        const float b = (float)((uint32_t)(key >> 32) - umin) * scale;
        return min(255, (int)b) <= bstar;
    }
};

template <class Visit>
__device__ __forceinline__ KeyBins warp_key_bins(Visit&& visit, int k, unsigned* hist) {
    const int lane = threadIdx.x & 31;
    uint32_t lo = 0xffffffffu, hi = 0u;
    visit([&](uint64_t key, bool valid) {
        if (valid) {
            const uint32_t u = (uint32_t)(key >> 32);
            lo = min(lo, u);
            hi = max(hi, u);
        }
    });
    lo = __reduce_min_sync(0xffffffffu, lo);
    hi = __reduce_max_sync(0xffffffffu, hi);
    KeyBins b;
    b.umin = lo;
    b.bstar = 255;
    b.scale = 0.0f;
    if (lo > hi) return b;  // no valid key
    b.scale = 256.0f / ((float)(hi - lo) + 1.0f);
#pragma unroll
    for (int j = 0; j < 8; ++j) hist[j * 32 + lane] = 0u;
    __syncwarp();
    visit([&](uint64_t key, bool valid) {
        if (valid) {
            const float f = (float)((uint32_t)(key >> 32) - lo) * b.scale;
            atomicAdd(&hist[min(255, (int)f)], 1u);
        }
    });
    __syncwarp();
    // lane owns bins 8 lane .. 8 lane + 7; the first bin where the running
    // count reaches k is bstar
    unsigned c[8], sum = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        c[j] = hist[8 * lane + j];
        sum += c[j];
    }
    unsigned incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    const unsigned reach = __ballot_sync(0xffffffffu, incl >= (unsigned)k);
    if (reach) {
        const int owner = __ffs(reach) - 1;
        int bs = 255;
        unsigned run = incl - sum;
        bool found = false;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            run += c[j];
            if (!found && run >= (unsigned)k) {
                bs = 8 * lane + j;
                found = true;
            }
        }
        b.bstar = __shfl_sync(0xffffffffu, bs, owner);
    }
    __syncwarp();  // hist may be reused
    return b;
}

// Block-wide merge: every warp has stored its k best to smem[w*k ...]; warp 0
// folds them into its own list.  Caller syncs before and after.
template <int P>
__device__ __forceinline__ void block_merge_warp0(WarpTopK<P>& tk, const uint64_t* lists,
                                                  int nwarps) {
    for (int w = 1; w < nwarps; ++w) tk.ingest(lists + w * tk.k, tk.k);
}

}  // namespace fdb
