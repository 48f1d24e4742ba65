// fdb_oracle.cpp -- TEST INFRASTRUCTURE ONLY.
//
// A CPU restatement of forge-db's nearest-neighbour search and training path
// (the Rust crate HueCodes/forge-db), written to serve as the parity checker
// for the CUDA engine and as the timed CPU baseline.  Nothing in the product
// links, loads or calls this file; only the test suite, the smoke check and
// the benchmark's CPU-baseline leg do.
//
// Numeric contract: the reference's default x86_64 build (AVX2 + FMA, the
// `avx512` cargo feature off).  Every reduction below follows the reference's
// summation order exactly, so results are bit-identical to it given the same
// inputs:
//   * L2^2 / dot / cosine: 8 FMA lanes over i = j (mod 8), a left-to-right sum
//     of the 8 lanes, then an unfused scalar tail
//     (src/distance/simd.rs:338-366, 427-456, 469-517).
//   * k-means: first-minimum argmin, per-cluster serial sums in point order,
//     empty clusters keep their centroid, mean-squared-shift stop at 1e-3
//     (src/kmeans.rs:87-193, 257-329).
//   * PQ: per-subspace k-means(256, 25), first-minimum encode, flat/nested LUTs
//     (src/pq.rs:55-189), the two ADC summation orders (src/pq.rs:218-245 and
//     318-485).
//   * IVF-PQ: build (src/index/ivf_pq.rs:374-506), single search (:590-677),
//     batch search (:850-1047) and its Rayon chunking (:1060-1084).
//   * Brute force: exact top-k with strict '<' admission
//     (src/index/brute_force.rs:105-225).
//
// Randomness: the reference draws training samples and initial centroids from
// an unseeded `rand::thread_rng` (src/kmeans.rs:54,97,107; ivf_pq.rs:388,426),
// so it never reproduces itself.  Here every random choice is an input: sample
// index lists, initial-centroid index lists and the k-means++ uniform draws.
// No reference test pins a training outcome (there are no seeds or golden
// files upstream), so training parity is "given the same injected draws".
//
// Build: g++ -O3 -mavx2 -mfma -ffp-contract=off -fopenmp (see Makefile).

#include <immintrin.h>
#include <omp.h>

#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <queue>
#include <utility>
#include <vector>

namespace {

// ---------------------------------------------------------------------------
// Distances (src/distance/simd.rs)
// ---------------------------------------------------------------------------

inline float lane_sum8(__m256 v) {
    alignas(32) float a[8];
    _mm256_store_ps(a, v);
    // `sum_array.iter().sum()` folds left to right.
    float t = 0.0f;
    for (int j = 0; j < 8; ++j) t += a[j];
    return t;
}

// euclidean_distance_squared_avx2, src/distance/simd.rs:338-366
inline float l2sq(const float* a, const float* b, size_t len) {
    __m256 sum = _mm256_setzero_ps();
    size_t i = 0;
    while (i + 8 <= len) {
        __m256 va = _mm256_loadu_ps(a + i);
        __m256 vb = _mm256_loadu_ps(b + i);
        __m256 d = _mm256_sub_ps(va, vb);
        sum = _mm256_fmadd_ps(d, d, sum);
        i += 8;
    }
    float total = lane_sum8(sum);
    while (i < len) {
        float d = a[i] - b[i];
        float sq = d * d;  // unfused (-ffp-contract=off)
        total += sq;
        ++i;
    }
    return total;
}

// dot_product_avx2, src/distance/simd.rs:427-456
inline float dot(const float* a, const float* b, size_t len) {
    __m256 sum = _mm256_setzero_ps();
    size_t i = 0;
    while (i + 8 <= len) {
        sum = _mm256_fmadd_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i), sum);
        i += 8;
    }
    float total = lane_sum8(sum);
    while (i < len) {
        float p = a[i] * b[i];
        total += p;
        ++i;
    }
    return total;
}

// cosine_distance_avx2, src/distance/simd.rs:469-517
inline float cosine(const float* a, const float* b, size_t len) {
    __m256 ds = _mm256_setzero_ps(), as = _mm256_setzero_ps(), bs = _mm256_setzero_ps();
    size_t i = 0;
    while (i + 8 <= len) {
        __m256 va = _mm256_loadu_ps(a + i), vb = _mm256_loadu_ps(b + i);
        ds = _mm256_fmadd_ps(va, vb, ds);
        as = _mm256_fmadd_ps(va, va, as);
        bs = _mm256_fmadd_ps(vb, vb, bs);
        i += 8;
    }
    float d = lane_sum8(ds), na = lane_sum8(as), nb = lane_sum8(bs);
    while (i < len) {
        float p = a[i] * b[i];
        d += p;
        float pa = a[i] * a[i];
        na += pa;
        float pb = b[i] * b[i];
        nb += pb;
        ++i;
    }
    float np = std::sqrt(na * nb);
    if (np == 0.0f) return 0.0f;
    return 1.0f - (d / np);
}

// manhattan_distance_avx2, src/distance/simd.rs:378-418
inline float manhattan(const float* a, const float* b, size_t len) {
    const __m256 mask = _mm256_castsi256_ps(_mm256_set1_epi32(0x7FFFFFFF));
    __m256 sum = _mm256_setzero_ps();
    size_t i = 0;
    while (i + 8 <= len) {
        __m256 d = _mm256_sub_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i));
        sum = _mm256_add_ps(sum, _mm256_and_ps(d, mask));
        i += 8;
    }
    float total = lane_sum8(sum);
    while (i < len) {
        total += std::fabs(a[i] - b[i]);
        ++i;
    }
    return total;
}

enum Metric { EUCLIDEAN = 0, EUCLIDEAN_SQUARED = 1, COSINE = 2, DOT_PRODUCT = 3, MANHATTAN = 4 };

// DistanceMetric::compute, src/distance/mod.rs:40-48
inline float metric_compute(int metric, const float* a, const float* b, size_t len) {
    switch (metric) {
        case EUCLIDEAN: return std::sqrt(l2sq(a, b, len));
        case EUCLIDEAN_SQUARED: return l2sq(a, b, len);
        case COSINE: return cosine(a, b, len);
        case DOT_PRODUCT: return -dot(a, b, len);
        case MANHATTAN: return manhattan(a, b, len);
        default: return NAN;
    }
}

// First-minimum argmin: Iterator::min_by with partial_cmp().unwrap_or(Equal)
// keeps the running minimum unless it compares Greater (src/kmeans.rs:262-268).
inline uint32_t argmin_l2sq(const float* x, const float* cents, size_t k, size_t dim) {
    uint32_t best = 0;
    float bd = l2sq(x, cents, dim);
    for (size_t c = 1; c < k; ++c) {
        float d = l2sq(x, cents + c * dim, dim);
        if (bd > d) { bd = d; best = (uint32_t)c; }
    }
    return best;
}

// ---------------------------------------------------------------------------
// k-means (src/kmeans.rs)
// ---------------------------------------------------------------------------

constexpr size_t KMEANSPP_THRESHOLD = 64;        // src/constants.rs:25
constexpr float CONVERGENCE_THRESHOLD = 0.001f;  // src/constants.rs:29

// Returns 0 on success, -3 empty, -5 insufficient vectors.
int kmeans_fit(const float* data, size_t n, size_t dim, size_t k, size_t max_iters,
               const uint32_t* init_idx, const float* kpp_u, float* cent, int* iters_run,
               int nthreads) {
    if (n == 0 || dim == 0) return -3;
    if (k == 0) return -1;
    if (k > KMEANSPP_THRESHOLD) {
        // Shuffled first-k sample (src/kmeans.rs:95-105).  With fewer than k
        // points the reference would index past its centroid list in the
        // update step and panic; this is reported as an error instead.
        if (n < k) return -5;
        for (size_t c = 0; c < k; ++c) {
            if (init_idx[c] >= n) return -1;
            std::memcpy(cent + c * dim, data + (size_t)init_idx[c] * dim, dim * sizeof(float));
        }
    } else {
        // k-means++ on raw data (src/kmeans.rs:106-141).  init_idx[0] is the
        // first pick; for c >= 1, kpp_u[c] is the uniform draw in [0,1) that
        // `gen_range(0.0..total)` turns into `u * total`, and init_idx[c] is
        // the pick used when every point already sits on a centroid.
        if (init_idx[0] >= n) return -1;
        std::memcpy(cent, data + (size_t)init_idx[0] * dim, dim * sizeof(float));
        std::vector<float> mind(n, FLT_MAX);
        for (size_t c = 1; c < k; ++c) {
            const float* last = cent + (c - 1) * dim;
#pragma omp parallel for num_threads(nthreads) schedule(static)
            for (size_t i = 0; i < n; ++i) {
                float d = l2sq(data + i * dim, last, dim);
                mind[i] = std::fmin(mind[i], d);  // fold(f32::MAX, f32::min)
            }
            float total = 0.0f;
            for (size_t i = 0; i < n; ++i) total += mind[i];
            size_t sel;
            if (total == 0.0f) {
                sel = init_idx[c];
                if (sel >= n) return -1;
            } else {
                float r = kpp_u[c] * total;
                sel = n - 1;
                for (size_t i = 0; i < n; ++i) {
                    r -= mind[i];
                    if (r <= 0.0f) { sel = i; break; }
                }
            }
            std::memcpy(cent + c * dim, data + sel * dim, dim * sizeof(float));
        }
    }

    std::vector<uint32_t> assign(n);
    std::vector<float> sums(k * dim);
    std::vector<size_t> counts(k);
    std::vector<float> next(k * dim);
    int iters = 0;
    for (size_t it = 0; it < max_iters; ++it) {
        ++iters;
#pragma omp parallel for num_threads(nthreads) schedule(static)
        for (size_t i = 0; i < n; ++i) assign[i] = argmin_l2sq(data + i * dim, cent, k, dim);
        // Per-cluster serial sums in point order (src/kmeans.rs:162-185): the
        // cluster's accumulator sees its points in increasing index order.
        std::fill(sums.begin(), sums.end(), 0.0f);
        std::fill(counts.begin(), counts.end(), 0);
        for (size_t i = 0; i < n; ++i) {
            float* s = sums.data() + (size_t)assign[i] * dim;
            const float* row = data + i * dim;
            for (size_t j = 0; j < dim; ++j) s[j] += row[j];
            counts[assign[i]]++;
        }
        for (size_t c = 0; c < k; ++c) {
            if (counts[c] == 0) {
                std::memcpy(next.data() + c * dim, cent + c * dim, dim * sizeof(float));
            } else {
                float cf = (float)counts[c];
                for (size_t j = 0; j < dim; ++j) next[c * dim + j] = sums[c * dim + j] / cf;
            }
        }
        // measure_change (src/kmeans.rs:320-329): ordered sum / k.
        float total = 0.0f;
        for (size_t c = 0; c < k; ++c) total += l2sq(cent + c * dim, next.data() + c * dim, dim);
        float change = total / (float)k;
        std::memcpy(cent, next.data(), k * dim * sizeof(float));
        if (change < CONVERGENCE_THRESHOLD) break;
    }
    if (iters_run) *iters_run = iters;
    return 0;
}

// ---------------------------------------------------------------------------
// Product quantizer (src/pq.rs)
// ---------------------------------------------------------------------------

constexpr size_t KSUB = 256;  // CENTROIDS_8BIT, src/constants.rs:10

// ProductQuantizer::try_train, src/pq.rs:55-95.  codebooks: [m][256][sub].
int pq_train(const float* x, size_t n, size_t dim, size_t m, size_t iters,
             const uint32_t* init_idx, float* codebooks, int* iters_out, int nthreads) {
    if (n == 0) return -3;
    if (m == 0) return -1;
    if (dim % m != 0) return -4;
    if (n < KSUB) return -5;
    const size_t sub = dim / m;
    int rc_all = 0;
#pragma omp parallel for num_threads(nthreads) schedule(dynamic, 1)
    for (size_t s = 0; s < m; ++s) {
        std::vector<float> sd(n * sub);
        for (size_t i = 0; i < n; ++i)
            std::memcpy(sd.data() + i * sub, x + i * dim + s * sub, sub * sizeof(float));
        int it = 0;
        int rc = kmeans_fit(sd.data(), n, sub, KSUB, iters, init_idx + s * KSUB, nullptr,
                            codebooks + s * KSUB * sub, &it, 1);
        if (iters_out) iters_out[s] = it;
        if (rc != 0) {
#pragma omp critical
            rc_all = rc;
        }
    }
    return rc_all;
}

// ProductQuantizer::encode, src/pq.rs:114-139
inline void pq_encode_one(const float* cb, size_t m, size_t sub, const float* v, uint8_t* code) {
    for (size_t s = 0; s < m; ++s)
        code[s] = (uint8_t)argmin_l2sq(v + s * sub, cb + s * KSUB * sub, KSUB, sub);
}

// build_lookup_table_flat, src/pq.rs:175-189 (the nested table of :149-170
// holds the same values).
inline void lut_flat(const float* cb, size_t m, size_t sub, const float* q, float* lut) {
    for (size_t s = 0; s < m; ++s)
        for (size_t j = 0; j < KSUB; ++j)
            lut[s * KSUB + j] = l2sq(q + s * sub, cb + (s * KSUB + j) * sub, sub);
}

// asymmetric_distance_fast, src/pq.rs:218-245: groups of four summed
// ((t0+t1)+t2)+t3 and added to the running sum, then a serial tail.
inline float adc_fast(const float* lut, const uint8_t* code, size_t m) {
    float sum = 0.0f;
    size_t i = 0;
    while (i + 4 <= m) {
        float g = lut[i * KSUB + code[i]] + lut[(i + 1) * KSUB + code[i + 1]];
        g = g + lut[(i + 2) * KSUB + code[i + 2]];
        g = g + lut[(i + 3) * KSUB + code[i + 3]];
        sum += g;
        i += 4;
    }
    while (i < m) { sum += lut[i * KSUB + code[i]]; ++i; }
    return sum;
}

// asymmetric_distance_simd_avx2, src/pq.rs:435-485 (also the per-query order
// of batch_asymmetric_distance_avx2, :318-402): 8 gather lanes over full
// groups of 8 subspaces, a left-to-right lane sum, then a serial tail.
inline float adc_lane8(const float* lut, const uint8_t* code, size_t m) {
    __m256 sum = _mm256_setzero_ps();
    size_t i = 0;
    while (i + 8 <= m) {
        __m256i idx = _mm256_set_epi32(
            (int)((i + 7) * KSUB + code[i + 7]), (int)((i + 6) * KSUB + code[i + 6]),
            (int)((i + 5) * KSUB + code[i + 5]), (int)((i + 4) * KSUB + code[i + 4]),
            (int)((i + 3) * KSUB + code[i + 3]), (int)((i + 2) * KSUB + code[i + 2]),
            (int)((i + 1) * KSUB + code[i + 1]), (int)(i * KSUB + code[i]));
        sum = _mm256_add_ps(sum, _mm256_i32gather_ps(lut, idx, 4));
        i += 8;
    }
    alignas(32) float a[8];
    _mm256_store_ps(a, sum);
    float total = a[0] + a[1];
    for (int j = 2; j < 8; ++j) total = total + a[j];
    while (i < m) { total += lut[i * KSUB + code[i]]; ++i; }
    return total;
}

// asymmetric_distance_flat_scalar, src/pq.rs:410-418: serial sum.
inline float adc_scalar(const float* lut, const uint8_t* code, size_t m) {
    float s = 0.0f;
    for (size_t i = 0; i < m; ++i) s += lut[i * KSUB + code[i]];
    return s;
}

// ---------------------------------------------------------------------------
// Bounded max-heap with the reference's admission rules.
// ---------------------------------------------------------------------------

struct Item {
    float d;
    uint64_t id;
};
struct ByDist {
    bool operator()(const Item& a, const Item& b) const { return a.d < b.d; }
};
using MaxHeap = std::priority_queue<Item, std::vector<Item>, ByDist>;

// Sort ascending by distance (stable, as `sort_by` is) and write out.
inline size_t heap_out(MaxHeap& h, size_t k, uint64_t* ids, float* dists) {
    std::vector<Item> v;
    v.reserve(h.size());
    while (!h.empty()) { v.push_back(h.top()); h.pop(); }
    std::reverse(v.begin(), v.end());
    std::stable_sort(v.begin(), v.end(), [](const Item& a, const Item& b) { return a.d < b.d; });
    size_t cnt = std::min(k, v.size());
    for (size_t i = 0; i < k; ++i) {
        ids[i] = i < cnt ? v[i].id : UINT64_MAX;
        dists[i] = i < cnt ? v[i].d : INFINITY;
    }
    return cnt;
}

// Coarse probe selection: the nprobe smallest L2^2 to the centroids
// (select_nth_unstable_by, src/index/ivf_pq.rs:538-553 and :865-888).  The
// reference leaves boundary ties unordered; ties are broken by list index.
void nearest_lists(const float* q, const float* cents, size_t nlist, size_t dim, size_t take,
                   std::vector<uint32_t>& out) {
    std::vector<std::pair<float, uint32_t>> cd(nlist);
    for (size_t l = 0; l < nlist; ++l) cd[l] = {l2sq(q, cents + l * dim, dim), (uint32_t)l};
    take = std::min(take, nlist);
    std::partial_sort(cd.begin(), cd.begin() + take, cd.end());
    out.resize(take);
    for (size_t i = 0; i < take; ++i) out[i] = cd[i].second;
}

struct IvfView {
    const float* cents;
    const float* cb;
    size_t nlist, m, dim;
    const uint64_t* offsets;  // nlist + 1
    const uint64_t* ids;      // list-major
    const uint8_t* codes;     // list-major, m bytes each
    const uint8_t* skip = nullptr;  // per row, nullable: 1 = skipped (tombstone /
                                    // filter, ivf_pq.rs:655-657 and :778-792)
};

// IVFPQIndex::search, src/index/ivf_pq.rs:590-677 (no reranking: fetch_k = k).
size_t ivf_search_one(const IvfView& ix, size_t nprobe, const float* q, size_t k, uint64_t* ids,
                      float* dists) {
    const size_t sub = ix.dim / ix.m;
    // `partition_ids` takes nprobe.min(nlist) entries; nprobe == 0 probes none.
    std::vector<uint32_t> probe;
    nearest_lists(q, ix.cents, ix.nlist, ix.dim, std::min(nprobe, ix.nlist), probe);
    if (nprobe == 0) probe.clear();
    MaxHeap heap;
    std::vector<float> res(ix.dim), lut(ix.m * KSUB);
    for (uint32_t l : probe) {
        const float* c = ix.cents + (size_t)l * ix.dim;
        for (size_t j = 0; j < ix.dim; ++j) res[j] = q[j] - c[j];
        lut_flat(ix.cb, ix.m, sub, res.data(), lut.data());
        // Threshold read once per partition (:638-642).
        float thr = (heap.size() >= k && !heap.empty()) ? heap.top().d : FLT_MAX;
        for (uint64_t p = ix.offsets[l]; p < ix.offsets[l + 1]; ++p) {
            if (ix.skip && ix.skip[p]) continue;
            float d = adc_fast(lut.data(), ix.codes + p * ix.m, ix.m);
            if (d < thr || heap.size() < k) {
                heap.push({d, ix.ids[p]});
                if (heap.size() > k) heap.pop();
            }
        }
    }
    return heap_out(heap, k, ids, dists);
}

// IVFPQIndex::batch_search, src/index/ivf_pq.rs:850-1047, on one chunk.
void ivf_batch_chunk(const IvfView& ix, size_t nprobe, const float* Q, size_t nq, size_t k,
                     uint64_t* ids, float* dists, uint32_t* counts) {
    const size_t sub = ix.dim / ix.m;
    // nth = nprobe.min(nlist).saturating_sub(1); [..=nth] -> nprobe == 0 probes one.
    size_t take = std::max<size_t>(1, std::min(nprobe, ix.nlist));
    std::vector<std::vector<uint32_t>> part_q(ix.nlist);
    std::vector<uint32_t> probe;
    for (size_t qi = 0; qi < nq; ++qi) {
        nearest_lists(Q + qi * ix.dim, ix.cents, ix.nlist, ix.dim, take, probe);
        for (uint32_t l : probe) part_q[l].push_back((uint32_t)qi);
    }
    std::vector<MaxHeap> heaps(nq);
    std::vector<float> res(ix.dim);
    std::vector<float> tables;
    // The reference walks a HashMap (random order); partition order only
    // affects which of several equal distances survives.
    for (size_t l = 0; l < ix.nlist; ++l) {
        const auto& qs = part_q[l];
        if (qs.empty()) continue;
        const float* c = ix.cents + l * ix.dim;
        tables.resize(qs.size() * ix.m * KSUB);
        for (size_t t = 0; t < qs.size(); ++t) {
            const float* q = Q + (size_t)qs[t] * ix.dim;
            for (size_t j = 0; j < ix.dim; ++j) res[j] = q[j] - c[j];
            lut_flat(ix.cb, ix.m, sub, res.data(), tables.data() + t * ix.m * KSUB);
        }
        for (uint64_t p = ix.offsets[l]; p < ix.offsets[l + 1]; ++p) {
            if (ix.skip && ix.skip[p]) continue;
            const uint8_t* code = ix.codes + p * ix.m;
            for (size_t t = 0; t < qs.size(); ++t) {
                float d = adc_lane8(tables.data() + t * ix.m * KSUB, code, ix.m);
                MaxHeap& h = heaps[qs[t]];
                float thr = (h.size() >= k && !h.empty()) ? h.top().d : FLT_MAX;
                if (d < thr || h.size() < k) {
                    h.push({d, ix.ids[p]});
                    if (h.size() > k) h.pop();
                }
            }
        }
    }
    for (size_t qi = 0; qi < nq; ++qi) {
        size_t c = heap_out(heaps[qi], k, ids + qi * k, dists + qi * k);
        if (counts) counts[qi] = (uint32_t)c;
    }
}

}  // namespace

// ===========================================================================
// C entry points (ctypes)
// ===========================================================================
extern "C" {

float orc_l2sq(const float* a, const float* b, size_t d) { return l2sq(a, b, d); }
float orc_dot(const float* a, const float* b, size_t d) { return dot(a, b, d); }
float orc_cosine(const float* a, const float* b, size_t d) { return cosine(a, b, d); }
float orc_manhattan(const float* a, const float* b, size_t d) { return manhattan(a, b, d); }
float orc_metric(int metric, const float* a, const float* b, size_t d) {
    return metric_compute(metric, a, b, d);
}

// Scalar references of src/distance/scalar.rs:30-93 (serial sums), used to
// restate the reference's SIMD-vs-scalar tolerance tests.
float orc_l2sq_scalar(const float* a, const float* b, size_t d) {
    float s = 0.0f;
    for (size_t i = 0; i < d; ++i) { float t = a[i] - b[i]; float sq = t * t; s += sq; }
    return s;
}
float orc_dot_scalar(const float* a, const float* b, size_t d) {
    float s = 0.0f;
    for (size_t i = 0; i < d; ++i) { float p = a[i] * b[i]; s += p; }
    return s;
}

// out[i] = metric(a[i], b[i]) for n row pairs.
void orc_pairwise(int metric, const float* a, const float* b, size_t n, size_t d, float* out) {
    for (size_t i = 0; i < n; ++i) out[i] = metric_compute(metric, a + i * d, b + i * d, d);
}

// Nearest-centroid assignment with the first-minimum rule
// (src/kmeans.rs:257-270, src/index/ivf_pq.rs:403-414).
void orc_assign(const float* x, size_t n, const float* cents, size_t k, size_t dim,
                uint32_t* out, int nthreads) {
#pragma omp parallel for num_threads(nthreads) schedule(static)
    for (size_t i = 0; i < n; ++i) out[i] = argmin_l2sq(x + i * dim, cents, k, dim);
}

// KMeans::find_nearest_centroids, src/kmeans.rs:334-345 (stable sort).
void orc_find_nearest_centroids(const float* cents, size_t kc, size_t dim, const float* q,
                                size_t k, uint32_t* out) {
    std::vector<std::pair<float, uint32_t>> cd(kc);
    for (size_t c = 0; c < kc; ++c) cd[c] = {l2sq(q, cents + c * dim, dim), (uint32_t)c};
    std::stable_sort(cd.begin(), cd.end(),
                     [](const auto& a, const auto& b) { return a.first < b.first; });
    for (size_t i = 0; i < std::min(k, kc); ++i) out[i] = cd[i].second;
}

int orc_kmeans_fit(const float* data, size_t n, size_t dim, size_t k, size_t max_iters,
                   const uint32_t* init_idx, const float* kpp_u, float* centroids_out,
                   int* iters_run, int nthreads) {
    return kmeans_fit(data, n, dim, k, max_iters, init_idx, kpp_u, centroids_out, iters_run,
                      nthreads);
}

int orc_pq_train(const float* x, size_t n, size_t dim, size_t m, size_t iters,
                 const uint32_t* init_idx, float* codebooks, int* iters_out, int nthreads) {
    return pq_train(x, n, dim, m, iters, init_idx, codebooks, iters_out, nthreads);
}

void orc_pq_encode(const float* cb, size_t m, size_t dim, const float* x, size_t n,
                   uint8_t* codes, int nthreads) {
    const size_t sub = dim / m;
#pragma omp parallel for num_threads(nthreads) schedule(static)
    for (size_t i = 0; i < n; ++i) pq_encode_one(cb, m, sub, x + i * dim, codes + i * m);
}

void orc_lut_flat(const float* cb, size_t m, size_t dim, const float* q, float* lut) {
    lut_flat(cb, m, dim / m, q, lut);
}

float orc_adc_fast(const float* lut, const uint8_t* code, size_t m) { return adc_fast(lut, code, m); }
float orc_adc_lane8(const float* lut, const uint8_t* code, size_t m) { return adc_lane8(lut, code, m); }
float orc_adc_scalar(const float* lut, const uint8_t* code, size_t m) { return adc_scalar(lut, code, m); }

// IVFPQIndex::build, src/index/ivf_pq.rs:374-506, with injected randomness.
//   ivf_sample_idx[n_ivf]: the IVF training sample (the reference uses every
//     vector, in order, when n <= 30000, and a shuffled prefix otherwise).
//   ivf_init_idx / ivf_kpp_u: k-means initialisation draws (see kmeans_fit).
//   pq_sample_idx[n_pq]: the shuffled prefix of residuals used for PQ training.
//   pq_init_idx[m*256]: per-subspace initial codeword picks.
// Outputs: centroids[nlist*dim], codebooks[m*256*sub], assign[n],
//   offsets[nlist+1], list_ids[n], list_codes[n*m] (lists in input order).
int orc_ivfpq_build(const float* x, const uint64_t* ids, size_t n, size_t dim, size_t nlist,
                    size_t m, const uint32_t* ivf_sample_idx, size_t n_ivf,
                    const uint32_t* ivf_init_idx, const float* ivf_kpp_u,
                    const uint32_t* pq_sample_idx, size_t n_pq, const uint32_t* pq_init_idx,
                    size_t ivf_iters, size_t pq_iters, float* centroids, float* codebooks,
                    uint32_t* assign, uint64_t* offsets, uint64_t* list_ids, uint8_t* list_codes,
                    int nthreads) {
    if (n == 0) return -10;
    if (m == 0 || nlist == 0) return -1;
    if (dim % m != 0) return -4;
    std::vector<float> sample(n_ivf * dim);
    for (size_t i = 0; i < n_ivf; ++i) {
        if (ivf_sample_idx[i] >= n) return -1;
        std::memcpy(sample.data() + i * dim, x + (size_t)ivf_sample_idx[i] * dim, dim * sizeof(float));
    }
    int it = 0;
    int rc = kmeans_fit(sample.data(), n_ivf, dim, nlist, ivf_iters, ivf_init_idx, ivf_kpp_u,
                        centroids, &it, nthreads);
    if (rc) return rc;
    orc_assign(x, n, centroids, nlist, dim, assign, nthreads);
    std::vector<float> resid(n_pq * dim);
    for (size_t i = 0; i < n_pq; ++i) {
        size_t v = pq_sample_idx[i];
        if (v >= n) return -1;
        const float* c = centroids + (size_t)assign[v] * dim;
        for (size_t j = 0; j < dim; ++j) resid[i * dim + j] = x[v * dim + j] - c[j];
    }
    rc = pq_train(resid.data(), n_pq, dim, m, pq_iters, pq_init_idx, codebooks, nullptr, nthreads);
    if (rc) return rc;
    std::vector<uint64_t> cnt(nlist + 1, 0);
    for (size_t i = 0; i < n; ++i) cnt[assign[i] + 1]++;
    for (size_t l = 0; l < nlist; ++l) cnt[l + 1] += cnt[l];
    std::memcpy(offsets, cnt.data(), (nlist + 1) * sizeof(uint64_t));
    std::vector<uint64_t> pos(cnt.begin(), cnt.end() - 1);
    std::vector<uint64_t> where(n);
    for (size_t i = 0; i < n; ++i) where[i] = pos[assign[i]]++;
    const size_t sub = dim / m;
#pragma omp parallel num_threads(nthreads)
    {
        std::vector<float> r(dim);
#pragma omp for schedule(static)
        for (size_t i = 0; i < n; ++i) {
            const float* c = centroids + (size_t)assign[i] * dim;
            for (size_t j = 0; j < dim; ++j) r[j] = x[i * dim + j] - c[j];
            pq_encode_one(codebooks, m, sub, r.data(), list_codes + where[i] * m);
            list_ids[where[i]] = ids[i];
        }
    }
    return 0;
}

// IVFPQIndex::search over one query (single-query order and semantics).
size_t orc_ivfpq_search(const float* cents, const float* cb, size_t nlist, size_t m, size_t dim,
                        const uint64_t* offsets, const uint64_t* ids, const uint8_t* codes,
                        size_t nprobe, const float* q, size_t k, uint64_t* out_ids,
                        float* out_d) {
    IvfView ix{cents, cb, nlist, m, dim, offsets, ids, codes};
    return ivf_search_one(ix, nprobe, q, k, out_ids, out_d);
}

// search() / search_filtered() with rows skipped (skip[p] != 0), k = fetch_k.
size_t orc_ivfpq_search_skip(const float* cents, const float* cb, size_t nlist, size_t m,
                             size_t dim, const uint64_t* offsets, const uint64_t* ids,
                             const uint8_t* codes, const uint8_t* skip, size_t nprobe,
                             const float* q, size_t k, uint64_t* out_ids, float* out_d) {
    IvfView ix{cents, cb, nlist, m, dim, offsets, ids, codes, skip};
    return ivf_search_one(ix, nprobe, q, k, out_ids, out_d);
}

// IVFPQIndex::batch_search_parallel, src/index/ivf_pq.rs:1060-1084: chunks of
// clamp(256 KiB / (nprobe * m * 1 KiB), 4, 64) queries, each chunk through
// batch_search, chunks spread over `nthreads` threads.  chunk == 0 selects the
// reference's rule; chunk > 0 forces one chunk size (chunk >= nq reproduces a
// plain batch_search call).
// skip (per row, nullable): tombstoned rows (ivf_pq.rs:958-961).
void orc_ivfpq_batch_search_skip(const float* cents, const float* cb, size_t nlist, size_t m,
                                 size_t dim, const uint64_t* offsets, const uint64_t* ids,
                                 const uint8_t* codes, const uint8_t* skip, size_t nprobe,
                                 const float* Q, size_t nq, size_t k, size_t chunk,
                                 uint64_t* out_ids, float* out_d, uint32_t* counts,
                                 int nthreads) {
    IvfView ix{cents, cb, nlist, m, dim, offsets, ids, codes, skip};
    if (nq == 0) return;
    if (chunk == 0) {
        size_t table_bytes = m * 256 * 4;
        chunk = (256 * 1024) / (std::max<size_t>(nprobe, 1) * table_bytes);
        chunk = std::min<size_t>(std::max<size_t>(chunk, 4), 64);
    }
    size_t nchunks = (nq + chunk - 1) / chunk;
#pragma omp parallel for num_threads(nthreads) schedule(dynamic, 1)
    for (size_t c = 0; c < nchunks; ++c) {
        size_t q0 = c * chunk, q1 = std::min(nq, q0 + chunk);
        ivf_batch_chunk(ix, nprobe, Q + q0 * dim, q1 - q0, k, out_ids + q0 * k, out_d + q0 * k,
                        counts ? counts + q0 : nullptr);
    }
}

void orc_ivfpq_batch_search(const float* cents, const float* cb, size_t nlist, size_t m,
                            size_t dim, const uint64_t* offsets, const uint64_t* ids,
                            const uint8_t* codes, size_t nprobe, const float* Q, size_t nq,
                            size_t k, size_t chunk, uint64_t* out_ids, float* out_d,
                            uint32_t* counts, int nthreads) {
    orc_ivfpq_batch_search_skip(cents, cb, nlist, m, dim, offsets, ids, codes, nullptr, nprobe,
                                Q, nq, k, chunk, out_ids, out_d, counts, nthreads);
}

// rerank_results (src/index/ivf_pq.rs:556-582) for nq queries: candidate
// row q holds cnt[q] PQ results (ascending); those whose id has an original
// vector (rr_ids ascending, rr_x in that order) get sqrt(L2^2) in the
// euclidean_distance_squared order, are stable-sorted and cut to k.
void orc_rerank(const float* Q, size_t nq, size_t dim, const uint64_t* cand, const uint32_t* cnt,
                size_t fetch, const uint64_t* rr_ids, const float* rr_x, size_t nrr, size_t k,
                uint64_t* out_ids, float* out_d, uint32_t* out_cnt, int nthreads) {
#pragma omp parallel for num_threads(nthreads) schedule(static)
    for (size_t q = 0; q < nq; ++q) {
        std::vector<std::pair<float, uint64_t>> r;
        for (size_t i = 0; i < cnt[q]; ++i) {
            const uint64_t id = cand[q * fetch + i];
            const uint64_t* it = std::lower_bound(rr_ids, rr_ids + nrr, id);
            if (it == rr_ids + nrr || *it != id) continue;
            const float d = std::sqrt(l2sq(Q + q * dim, rr_x + (size_t)(it - rr_ids) * dim, dim));
            r.push_back({d, id});
        }
        std::stable_sort(r.begin(), r.end(),
                         [](const auto& a, const auto& b) { return a.first < b.first; });
        const size_t c = std::min(k, r.size());
        for (size_t i = 0; i < k; ++i) {
            out_ids[q * k + i] = i < c ? r[i].second : UINT64_MAX;
            out_d[q * k + i] = i < c ? r[i].first : INFINITY;
        }
        out_cnt[q] = (uint32_t)c;
    }
}

// BruteForceIndex::batch_search -> search_parallel -> scan_range,
// src/index/brute_force.rs:105-225.  Admission: fill to k, then replace the
// max on strict '<'.  The 1000-row chunk heaps of search_parallel merge under
// the same rule, so one heap per query yields the same set (ties aside).
void orc_bf_batch_search(const float* x, const uint64_t* ids, size_t n, size_t dim, int metric,
                         const float* Q, size_t nq, size_t k, uint64_t* out_ids, float* out_d,
                         uint32_t* counts, int nthreads) {
#pragma omp parallel for num_threads(nthreads) schedule(dynamic, 1)
    for (size_t qi = 0; qi < nq; ++qi) {
        MaxHeap h;
        const float* q = Q + qi * dim;
        for (size_t i = 0; i < n; ++i) {
            float d = metric_compute(metric, q, x + i * dim, dim);
            if (h.size() < k) h.push({d, ids[i]});
            else if (k > 0 && d < h.top().d) { h.pop(); h.push({d, ids[i]}); }
        }
        size_t c = heap_out(h, k, out_ids + qi * k, out_d + qi * k);
        if (counts) counts[qi] = (uint32_t)c;
    }
}

int orc_max_threads(void) { return omp_get_max_threads(); }

}  // extern "C"
