// mutate.cu -- the IVF-PQ index's state around the scan: tombstones (delete,
// compact), insert_batch, the re-ranking store with its device re-scoring,
// and the per-call row filter of search_filtered.
//
// Layout rules kept by every change here: lists stay contiguous and in list
// order, a list's rows keep their order (new rows go to its end, compaction
// keeps the survivors' order), and the row position stays the tie-break tag.
// Every change rebuilds the derived tables (ivfpq_prepare_tables) so all scan
// modes see the same rows.
#include <cub/cub.cuh>

#include <algorithm>
#include <cmath>
#include <numeric>

#include "fdb_device.cuh"
#include "fdb_internal.h"
#include "fdb_kernels.h"

namespace fdb {

static unsigned grid_for(size_t n, unsigned threads = 256) {
    return (unsigned)std::max<size_t>(1, (n + threads - 1) / threads);
}

// ---------------------------------------------------------------------------
// kernels
// ---------------------------------------------------------------------------
// One block per list: the tensor scan's ||rhat||^2 of every dead row becomes
// +inf, so its score is +inf and it is never admitted or selected.
__global__ void mask_dead_kernel(const uint32_t* __restrict__ dead,
                                 const uint64_t* __restrict__ offs,
                                 const uint32_t* __restrict__ pstart, float* __restrict__ dnorm) {
    const int l = blockIdx.x;
    const uint64_t b = offs[l], e = offs[l + 1];
    for (uint64_t p = b + threadIdx.x; p < e; p += blockDim.x)
        if ((dead[p >> 5] >> (p & 31)) & 1u) dnorm[pstart[l] + (p - b)] = __int_as_float(0x7f800000);
}

// One block per list: copy its rows (ids and codes, contiguous) to the list's
// start in the new layout.
__global__ void relayout_kernel(const uint64_t* __restrict__ old_offs,
                                const uint64_t* __restrict__ new_offs, int m,
                                const uint8_t* __restrict__ codes, const uint64_t* __restrict__ ids,
                                uint8_t* __restrict__ codes2, uint64_t* __restrict__ ids2) {
    const int l = blockIdx.x;
    const uint64_t b = old_offs[l], e = old_offs[l + 1], nb = new_offs[l];
    for (uint64_t p = b + threadIdx.x; p < e; p += blockDim.x) ids2[nb + (p - b)] = ids[p];
    const uint64_t nbytes = (e - b) * (uint64_t)m;
    const uint8_t* src = codes + b * (uint64_t)m;
    uint8_t* dst = codes2 + nb * (uint64_t)m;
    for (uint64_t t = threadIdx.x; t < nbytes; t += blockDim.x) dst[t] = src[t];
}

__global__ void scatter_ids_kernel(const uint64_t* __restrict__ ids, const uint32_t* __restrict__ slot,
                                   size_t n, uint64_t* __restrict__ out) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[slot[i]] = ids[i];
}

// Kept rows (ascending) gathered into a dense layout.
__global__ void gather_rows_kernel(const uint32_t* __restrict__ rows, size_t nkeep, int m,
                                   const uint8_t* __restrict__ codes,
                                   const uint64_t* __restrict__ ids, uint8_t* __restrict__ codes2,
                                   uint64_t* __restrict__ ids2) {
    const size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= nkeep * (size_t)m) return;
    const size_t i = t / m, j = t % m;
    const uint32_t r = rows[i];
    codes2[t] = codes[(size_t)r * m + j];
    if (j == 0) ids2[i] = ids[r];
}

// One thread per allowed id: every row holding it (a range of the
// (id, row) index sorted by id) gets its bit set in `allow`.
__global__ void allow_rows_kernel(const uint64_t* __restrict__ allowed, size_t na,
                                  const uint64_t* __restrict__ sorted_ids,
                                  const uint32_t* __restrict__ sorted_rows, size_t n,
                                  uint32_t* __restrict__ allow) {
    const size_t a = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (a >= na) return;
    const uint64_t id = allowed[a];
    size_t lo = 0, hi = n;
    while (lo < hi) {
        const size_t mid = (lo + hi) >> 1;
        if (sorted_ids[mid] < id) lo = mid + 1;
        else hi = mid;
    }
    for (size_t p = lo; p < n && sorted_ids[p] == id; ++p) {
        const uint32_t r = sorted_rows[p];
        atomicOr(allow + (r >> 5), 1u << (r & 31));
    }
}

// skip = not allowed, or dead; rows past n stay allowed (never scanned).
__global__ void skip_words_kernel(const uint32_t* __restrict__ allow,
                                  const uint32_t* __restrict__ dead, size_t n,
                                  uint32_t* __restrict__ skip) {
    const size_t w = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (w >= (n + 31) / 32) return;
    const size_t rem = n - w * 32;
    const uint32_t valid = rem >= 32 ? 0xffffffffu : ((1u << rem) - 1u);
    skip[w] = ((~allow[w]) & valid) | (dead ? dead[w] : 0u);
}

// rerank_results (ivf_pq.rs:556-582), one block per query.  Candidate i of
// the PQ list (ascending) that has an original vector gets sqrt(L2^2(q, v))
// (euclidean_distance_squared in the AVX2 order, correctly rounded square
// root); candidates without one are dropped.  Eight threads score one
// candidate: thread j runs the order's accumulator j (elements i = j mod 8)
// and the eight are summed left to right through shuffles, then the tail --
// the same operations in the same order as l2sq_exact.  A stable sort by
// distance is a sort by (distance, i); each candidate's rank is the number
// of smaller keys, and the first k ranks are written.
constexpr int RERANK_MAX = FDB_MAX_K;
constexpr int RERANK_THREADS = 256;  // 32 candidates scored at a time
__global__ void __launch_bounds__(RERANK_THREADS)
    rerank_kernel(const uint64_t* __restrict__ keys, const uint64_t* __restrict__ cand_ids,
                  int fetch, const float* __restrict__ Q, int dim,
                  const uint64_t* __restrict__ rr_ids, const uint32_t* __restrict__ rr_slot,
                  size_t nrr, const float* __restrict__ rr_x, int k, uint64_t* __restrict__ out_ids,
                  float* __restrict__ out_d, uint32_t* __restrict__ counts) {
    __shared__ uint64_t skey[RERANK_MAX];
    __shared__ uint64_t sid[RERANK_MAX];
    __shared__ int sslot[RERANK_MAX];
    const size_t q = blockIdx.x;
    const int t = threadIdx.x;
    const float* qv = Q + q * dim;
    // look up each candidate's original vector
    for (int c = t; c < RERANK_MAX; c += RERANK_THREADS) {
        int slot = -1;
        uint64_t id = 0;
        if (c < fetch && keys[q * fetch + c] != KEY_NONE) {
            id = cand_ids[q * fetch + c];
            size_t lo = 0, hi = nrr;
            while (lo < hi) {
                const size_t mid = (lo + hi) >> 1;
                if (rr_ids[mid] < id) lo = mid + 1;
                else hi = mid;
            }
            if (lo < nrr && rr_ids[lo] == id) slot = (int)rr_slot[lo];
        }
        sslot[c] = slot;
        sid[c] = id;
        skey[c] = KEY_NONE;
    }
    __syncthreads();
    // score: 32 candidates per pass, 8 lanes each
    const int g = t >> 3, j = t & 7;
    const int full = dim & ~7;
    for (int c0 = 0; c0 < fetch; c0 += RERANK_THREADS / 8) {
        const int c = c0 + g;
        const int slot = c < fetch ? sslot[c] : -1;
        float acc = 0.0f;
        if (slot >= 0) {
            const float* x = rr_x + (size_t)slot * dim;
            for (int i = j; i < full; i += 8) {
                const float d = __fsub_rn(qv[i], x[i]);
                acc = __fmaf_rn(d, d, acc);
            }
        }
        // acc_0 + acc_1 + ... + acc_7, then the unfused tail
        float tot = __shfl_sync(0xffffffffu, acc, 0, 8);
#pragma unroll
        for (int u = 1; u < 8; ++u) tot = __fadd_rn(tot, __shfl_sync(0xffffffffu, acc, u, 8));
        if (slot >= 0 && j == 0) {
            const float* x = rr_x + (size_t)slot * dim;
            for (int i = full; i < dim; ++i) {
                const float d = __fsub_rn(qv[i], x[i]);
                tot = __fadd_rn(tot, __fmul_rn(d, d));
            }
            const float dd = __fsqrt_rn(tot);
            skey[c] = ((uint64_t)f2ord(dd) << 32) | (uint32_t)c;
        }
    }
    __syncthreads();
    // rank among present keys
    int present = 0;
    for (int c = 0; c < fetch; ++c) present += skey[c] != KEY_NONE;
    for (int c = t; c < fetch; c += RERANK_THREADS) {
        const uint64_t key = skey[c];
        if (key == KEY_NONE) continue;
        int r = 0;
        for (int u = 0; u < fetch; ++u) r += skey[u] < key;
        if (r < k) {
            out_ids[q * k + r] = sid[c];
            out_d[q * k + r] = key_dist(key);
        }
    }
    const int cnt = min(present, k);
    for (int r = cnt + t; r < k; r += RERANK_THREADS) {
        out_ids[q * k + r] = ~0ull;
        out_d[q * k + r] = __int_as_float(0x7f800000);
    }
    if (t == 0 && counts) counts[q] = (uint32_t)cnt;
}

// ---------------------------------------------------------------------------
// host helpers
// ---------------------------------------------------------------------------
static size_t words_for(size_t n) { return (n + 31) / 32; }

// Rebuilds the host dead bitmap from the per-list tombstone sets.
static void rebuild_dead(fdb_ivfpq* h) {
    h->h_dead.clear();
    if (h->n_tomb == 0) return;
    h->h_dead.assign(words_for(h->n_total), 0u);
    for (size_t l = 0; l < h->tomb.size(); ++l) {
        if (h->tomb[l].empty()) continue;
        for (uint64_t p = h->h_offs_full[l]; p < h->h_offs_full[l + 1]; ++p)
            if (h->tomb[l].count(h->h_ids[p])) h->h_dead[p >> 5] |= 1u << (p & 31);
    }
}

void ivfpq_sync_state(fdb_ivfpq* h) {
    Ctx& c = h->ctx->c;
    cudaStream_t s = c.stream;
    if (h->dead_dirty) {
        if (h->h_dead.empty()) {
            h->dead.release();
        } else {
            h->dead.alloc(h->h_dead.size());
            FDB_CUDA(cudaMemcpyAsync(h->dead.p, h->h_dead.data(), h->dead.bytes(),
                                     cudaMemcpyHostToDevice, s));
            if (h->dnorm.p && h->tc_pstart.p && h->nlist > 0) {
                mask_dead_kernel<<<(unsigned)h->nlist, 256, 0, s>>>(h->dead.p, h->offs.p,
                                                                    h->tc_pstart.p, h->dnorm.p);
                FDB_LAUNCH_CHECK();
            }
        }
        FDB_CUDA(cudaStreamSynchronize(s));
        h->dead_dirty = false;
    }
    if (h->rerank && h->rr_dirty) {
        const size_t n = h->rr_ids.size();
        std::vector<std::pair<uint64_t, uint32_t>> order(n);
        for (size_t i = 0; i < n; ++i) order[i] = {h->rr_ids[i], (uint32_t)i};
        std::sort(order.begin(), order.end());
        std::vector<uint64_t> sid(n);
        std::vector<uint32_t> sslot(n);
        for (size_t i = 0; i < n; ++i) {
            sid[i] = order[i].first;
            sslot[i] = order[i].second;
        }
        h->rr_sorted.alloc(std::max<size_t>(n, 1));
        h->rr_sorted_slot.alloc(std::max<size_t>(n, 1));
        h->rr_dev.alloc(std::max<size_t>(n * h->dim, 1));
        if (n) {
            FDB_CUDA(cudaMemcpyAsync(h->rr_sorted.p, sid.data(), n * 8, cudaMemcpyHostToDevice, s));
            FDB_CUDA(cudaMemcpyAsync(h->rr_sorted_slot.p, sslot.data(), n * 4,
                                     cudaMemcpyHostToDevice, s));
            FDB_CUDA(cudaMemcpyAsync(h->rr_dev.p, h->rr_x.data(), n * h->dim * 4,
                                     cudaMemcpyHostToDevice, s));
        }
        FDB_CUDA(cudaStreamSynchronize(s));
        h->rr_dirty = false;
    }
}

static void rr_put(fdb_ivfpq* h, uint64_t id, const float* v) {
    auto it = h->rr_slot.find(id);
    size_t slot;
    if (it != h->rr_slot.end()) {
        slot = it->second;
    } else {
        slot = h->rr_ids.size();
        h->rr_ids.push_back(id);
        h->rr_x.resize(h->rr_x.size() + h->dim);
        h->rr_slot.emplace(id, slot);
    }
    std::copy(v, v + h->dim, h->rr_x.begin() + slot * h->dim);
    h->rr_dirty = true;
}

static void rr_remove(fdb_ivfpq* h, uint64_t id) {
    auto it = h->rr_slot.find(id);
    if (it == h->rr_slot.end()) return;
    const size_t slot = it->second, last = h->rr_ids.size() - 1;
    h->rr_slot.erase(it);
    if (slot != last) {
        h->rr_ids[slot] = h->rr_ids[last];
        std::copy(h->rr_x.begin() + last * h->dim, h->rr_x.begin() + (last + 1) * h->dim,
                  h->rr_x.begin() + slot * h->dim);
        h->rr_slot[h->rr_ids[slot]] = slot;
    }
    h->rr_ids.pop_back();
    h->rr_x.resize(last * h->dim);
    h->rr_dirty = true;
}

void ivfpq_enable_reranking(fdb_ivfpq* h, const float* x, const uint64_t* ids, size_t n,
                            size_t factor) {
    h->rr_ids.clear();
    h->rr_x.clear();
    h->rr_slot.clear();
    // HashMap collect: a repeated id keeps its last vector
    for (size_t i = 0; i < n; ++i) rr_put(h, ids[i], x + i * h->dim);
    h->rerank = true;
    h->rerank_factor = std::max<size_t>(factor, 1);
    h->rr_dirty = true;
}

void launch_rerank(fdb_ivfpq* h, const uint64_t* keys, const uint64_t* cand_ids, size_t nq,
                   size_t fetch, const float* dQ, size_t k, uint64_t* d_ids, float* d_dists,
                   uint32_t* d_counts) {
    FDB_REQUIRE(fetch <= (size_t)RERANK_MAX, FDB_ERR_UNSUPPORTED,
                "k * rerank_factor above FDB_MAX_K");
    if (nq == 0 || k == 0) return;
    rerank_kernel<<<(unsigned)nq, RERANK_THREADS, 0, h->ctx->c.stream>>>(
        keys, cand_ids, (int)fetch, dQ, (int)h->dim, h->rr_sorted.p, h->rr_sorted_slot.p,
        h->rr_ids.size(), h->rr_dev.p, (int)k, d_ids, d_dists, d_counts);
    FDB_LAUNCH_CHECK();
}

// Lazily built (id, row) index, ascending, for delete's lookups.
static void ensure_id_index(fdb_ivfpq* h) {
    if (h->id_index_ok) return;
    h->id_index.resize(h->n_total);
    for (size_t p = 0; p < h->n_total; ++p) h->id_index[p] = {h->h_ids[p], (uint32_t)p};
    std::sort(h->id_index.begin(), h->id_index.end());
    h->id_index_ok = true;
}

static size_t list_of_row(const fdb_ivfpq* h, uint64_t p) {
    return (size_t)(std::upper_bound(h->h_offs_full.begin(), h->h_offs_full.end(), p) -
                    h->h_offs_full.begin()) - 1;
}

bool ivfpq_delete(fdb_ivfpq* h, uint64_t id) {
    ensure_id_index(h);
    auto lo = std::lower_bound(h->id_index.begin(), h->id_index.end(),
                               std::make_pair(id, (uint32_t)0));
    // rows holding the id, ascending, hence in list order
    for (auto it = lo; it != h->id_index.end() && it->first == id;) {
        const size_t l = list_of_row(h, it->second);
        auto next = it;
        while (next != h->id_index.end() && next->first == id &&
               list_of_row(h, next->second) == l)
            ++next;
        const bool already = !h->tomb.empty() && h->tomb[l].count(id);
        if (!already) {
            if (h->tomb.empty()) h->tomb.resize(h->nlist);
            h->tomb[l].insert(id);
            h->n_tomb++;
            if (h->h_dead.empty()) h->h_dead.assign(words_for(h->n_total), 0u);
            for (auto r = it; r != next; ++r) h->h_dead[r->second >> 5] |= 1u << (r->second & 31);
            h->dead_dirty = true;
            if (h->rerank) rr_remove(h, id);
            return true;
        }
        it = next;
    }
    return false;
}

size_t ivfpq_live_len(const fdb_ivfpq* h) {
    // len(): ids.len() - tombstones.len() over the lists held here
    if (h->n_tomb == 0) return h->n_local;
    size_t t = 0;
    for (size_t l = 0; l < h->tomb.size(); ++l) {
        if (h->tomb[l].empty()) continue;
        if (!h->sharded || h->owned[l]) t += h->tomb[l].size();
    }
    return h->n_local - t;
}

// After any layout change: new derived tables, dead bitmap, sharding.
static void relayout_done(fdb_ivfpq* h) {
    h->id_index.clear();
    h->id_index_ok = false;
    h->d_idx_ok = false;
    rebuild_dead(h);
    h->dead_dirty = true;
    ivfpq_prepare_tables(h);
    if (h->shard_world > 1) ivfpq_shard(h, h->shard_rank, h->shard_world);
    ivfpq_sync_state(h);
}

void ivfpq_compact(fdb_ivfpq* h) {
    if (h->n_tomb == 0) return;
    Ctx& c = h->ctx->c;
    cudaStream_t s = c.stream;
    const size_t nlist = h->nlist, m = h->m;
    std::vector<uint32_t> keep;
    keep.reserve(h->n_total);
    std::vector<uint64_t> offs(nlist + 1, 0);
    for (size_t l = 0; l < nlist; ++l) {
        const bool t = !h->tomb[l].empty();
        for (uint64_t p = h->h_offs_full[l]; p < h->h_offs_full[l + 1]; ++p)
            if (!t || !h->tomb[l].count(h->h_ids[p])) keep.push_back((uint32_t)p);
        offs[l + 1] = keep.size();
    }
    const size_t nk = keep.size();
    DevBuf<uint32_t> d_keep(std::max<size_t>(nk, 1));
    DevBuf<uint8_t> codes2(std::max<size_t>(nk * m, 1));
    DevBuf<uint64_t> ids2(std::max<size_t>(nk, 1));
    if (nk) {
        FDB_CUDA(cudaMemcpyAsync(d_keep.p, keep.data(), nk * 4, cudaMemcpyHostToDevice, s));
        gather_rows_kernel<<<grid_for(nk * m), 256, 0, s>>>(d_keep.p, nk, (int)m, h->codes.p,
                                                             h->ids.p, codes2.p, ids2.p);
        FDB_LAUNCH_CHECK();
    }
    FDB_CUDA(cudaMemcpyAsync(h->offs.p, offs.data(), (nlist + 1) * 8, cudaMemcpyHostToDevice, s));
    FDB_CUDA(cudaStreamSynchronize(s));
    h->codes = std::move(codes2);
    h->ids = std::move(ids2);
    std::vector<uint64_t> hid(nk);
    for (size_t i = 0; i < nk; ++i) hid[i] = h->h_ids[keep[i]];
    h->h_ids.swap(hid);
    h->h_offs_full = offs;
    h->h_offs = offs;
    h->n_total = h->n_local = nk;
    h->tomb.clear();
    h->n_tomb = 0;
    relayout_done(h);
}

void ivfpq_insert_batch(fdb_ivfpq* h, const float* x_host, const uint64_t* ids_host, size_t n) {
    if (n == 0) return;
    Ctx& c = h->ctx->c;
    cudaStream_t s = c.stream;
    const size_t nlist = h->nlist, m = h->m, dim = h->dim, n_old = h->n_total;
    FDB_REQUIRE(n_old + n < (1ull << 32), FDB_ERR_UNSUPPORTED, "at most 2^32-1 vectors per index");
    DevBuf<float> X(n * dim);
    DevBuf<uint32_t> assign(n), slot(n);
    FDB_CUDA(cudaMemcpyAsync(X.p, x_host, X.bytes(), cudaMemcpyHostToDevice, s));
    // nearest list, first minimum (ivf_pq.rs:1737-1744)
    launch_assign(s, X.p, n, (int)dim, (int)dim, h->cents.p, (int)nlist, assign.p);
    std::vector<uint32_t> a(n);
    FDB_CUDA(cudaMemcpyAsync(a.data(), assign.p, n * 4, cudaMemcpyDeviceToHost, s));
    FDB_CUDA(cudaStreamSynchronize(s));
    std::vector<uint64_t> cnt(nlist, 0), offs(nlist + 1, 0);
    for (size_t i = 0; i < n; ++i) cnt[a[i]]++;
    for (size_t l = 0; l < nlist; ++l)
        offs[l + 1] = offs[l] + (h->h_offs_full[l + 1] - h->h_offs_full[l]) + cnt[l];
    // new rows go to the end of their list, in input order
    std::vector<uint64_t> fill(nlist);
    for (size_t l = 0; l < nlist; ++l) fill[l] = offs[l] + (h->h_offs_full[l + 1] - h->h_offs_full[l]);
    std::vector<uint32_t> sl(n);
    for (size_t i = 0; i < n; ++i) sl[i] = (uint32_t)(fill[a[i]]++);
    const size_t n_new = n_old + n;
    DevBuf<uint64_t> old_offs(nlist + 1), new_offs(nlist + 1), new_ids_in(n);
    DevBuf<uint8_t> codes2(n_new * m);
    DevBuf<uint64_t> ids2(n_new);
    FDB_CUDA(cudaMemcpyAsync(old_offs.p, h->h_offs_full.data(), (nlist + 1) * 8,
                             cudaMemcpyHostToDevice, s));
    FDB_CUDA(cudaMemcpyAsync(new_offs.p, offs.data(), (nlist + 1) * 8, cudaMemcpyHostToDevice, s));
    FDB_CUDA(cudaMemcpyAsync(slot.p, sl.data(), n * 4, cudaMemcpyHostToDevice, s));
    FDB_CUDA(cudaMemcpyAsync(new_ids_in.p, ids_host, n * 8, cudaMemcpyHostToDevice, s));
    if (n_old) {
        relayout_kernel<<<(unsigned)nlist, 256, 0, s>>>(old_offs.p, new_offs.p, (int)m,
                                                        h->codes.p, h->ids.p, codes2.p, ids2.p);
        FDB_LAUNCH_CHECK();
    }
    // residual of each new vector to its list's centroid, PQ-encoded into its slot
    launch_pq_encode(s, X.p, n, (int)dim, h->cents.p, assign.p, h->cb.p, (int)m, slot.p, codes2.p);
    scatter_ids_kernel<<<grid_for(n), 256, 0, s>>>(new_ids_in.p, slot.p, n, ids2.p);
    FDB_LAUNCH_CHECK();
    FDB_CUDA(cudaMemcpyAsync(h->offs.p, offs.data(), (nlist + 1) * 8, cudaMemcpyHostToDevice, s));
    FDB_CUDA(cudaStreamSynchronize(s));
    h->codes = std::move(codes2);
    h->ids = std::move(ids2);
    std::vector<uint64_t> hid(n_new);
    for (size_t l = 0; l < nlist; ++l)
        std::copy(h->h_ids.begin() + h->h_offs_full[l], h->h_ids.begin() + h->h_offs_full[l + 1],
                  hid.begin() + offs[l]);
    for (size_t i = 0; i < n; ++i) hid[sl[i]] = ids_host[i];
    h->h_ids.swap(hid);
    h->h_offs_full = offs;
    h->h_offs = offs;
    h->n_total = h->n_local = n_new;
    // partition.tombstones.remove(&id) in the list the vector joined
    if (h->n_tomb) {
        for (size_t i = 0; i < n; ++i) h->n_tomb -= h->tomb[a[i]].erase(ids_host[i]);
    }
    if (h->rerank)
        for (size_t i = 0; i < n; ++i) rr_put(h, ids_host[i], x_host + i * dim);
    relayout_done(h);
}

// The tensor scan's ||rhat||^2 for one filtered call: the index's values
// with +inf on every row the call skips (so the filter costs one copy of
// 4 bytes per padded row, not a change of the scan).
const float* ivfpq_call_colv(fdb_ivfpq* h, const uint32_t* skip) {
    cudaStream_t s = h->ctx->c.stream;
    h->f_colv.ensure(h->dnorm.n);
    FDB_CUDA(cudaMemcpyAsync(h->f_colv.p, h->dnorm.p, h->dnorm.bytes(), cudaMemcpyDeviceToDevice,
                             s));
    mask_dead_kernel<<<(unsigned)h->nlist, 256, 0, s>>>(skip, h->offs.p, h->tc_pstart.p,
                                                        h->f_colv.p);
    FDB_LAUNCH_CHECK();
    return h->f_colv.p;
}

// The (id, row) index sorted by id on the device, built on first use after
// a layout change.
static void ensure_dev_id_index(fdb_ivfpq* h) {
    if (h->d_idx_ok) return;
    cudaStream_t s = h->ctx->c.stream;
    const size_t n = h->n_total;
    h->d_idx_ids.alloc(std::max<size_t>(n, 1));
    h->d_idx_rows.alloc(std::max<size_t>(n, 1));
    if (n) {
        DevBuf<uint32_t> rows(n);
        std::vector<uint32_t> iota(n);
        std::iota(iota.begin(), iota.end(), 0u);
        FDB_CUDA(cudaMemcpyAsync(rows.p, iota.data(), n * 4, cudaMemcpyHostToDevice, s));
        size_t tmp = 0;
        FDB_CUDA(cub::DeviceRadixSort::SortPairs(nullptr, tmp, h->ids.p, h->d_idx_ids.p, rows.p,
                                                 h->d_idx_rows.p, (int)n, 0, 64, s));
        DevBuf<uint8_t> t(std::max<size_t>(tmp, 1));
        FDB_CUDA(cub::DeviceRadixSort::SortPairs(t.p, tmp, h->ids.p, h->d_idx_ids.p, rows.p,
                                                 h->d_idx_rows.p, (int)n, 0, 64, s));
        FDB_CUDA(cudaStreamSynchronize(s));
    }
    h->d_idx_ok = true;
}

// Per-call skip bitmap of search_filtered: dead rows and rows whose id is
// not allowed.  Returns the device bitmap (in h->f_skip).
const uint32_t* ivfpq_filter_bitmap(fdb_ivfpq* h, const uint64_t* allowed, size_t na,
                                    bool on_device) {
    Ctx& c = h->ctx->c;
    cudaStream_t s = c.stream;
    FDB_REQUIRE(na < (1ull << 31), FDB_ERR_UNSUPPORTED, "at most 2^31-1 allowed ids");
    FDB_REQUIRE(h->n_total < (1ull << 31), FDB_ERR_UNSUPPORTED, "at most 2^31-1 rows");
    ensure_dev_id_index(h);
    const uint64_t* a = allowed;
    if (!on_device) {
        h->f_sorted.ensure(na);
        FDB_CUDA(cudaMemcpyAsync(h->f_sorted.p, allowed, na * 8, cudaMemcpyHostToDevice, s));
        a = h->f_sorted.p;
    }
    const size_t nw = words_for(h->n_total);
    h->f_skip.ensure(2 * std::max<size_t>(nw, 1));
    uint32_t* allow = h->f_skip.p + std::max<size_t>(nw, 1);
    if (nw) {
        FDB_CUDA(cudaMemsetAsync(allow, 0, nw * 4, s));
        allow_rows_kernel<<<grid_for(na), 256, 0, s>>>(a, na, h->d_idx_ids.p, h->d_idx_rows.p,
                                                       h->n_total, allow);
        FDB_LAUNCH_CHECK();
        skip_words_kernel<<<grid_for(nw), 256, 0, s>>>(allow, h->n_tomb ? h->dead.p : nullptr,
                                                       h->n_total, h->f_skip.p);
        FDB_LAUNCH_CHECK();
    }
    return h->f_skip.p;
}

}  // namespace fdb
