// engine.cu -- host orchestration of the IVF-PQ and brute-force indexes.
//
// IVF-PQ build follows IVFPQIndex::build (forge-db src/index/ivf_pq.rs:374-506):
//   1. k-means(nlist, 25) on a training sample        (:383-400)
//   2. assign every vector, lists keep input order     (:403-419)
//   3. PQ trained on a sample of residuals v - c(v)    (:422-447)
//   4. every vector's residual encoded into its list   (:450-478)
// Search follows batch_search (:850-1047) / search (:590-677): coarse
// quantizer, probe selection, per-(query, list) LUT + scan + top-k, and, for
// an index whose lists are sharded over several devices, an ncclAllGather of
// the local top-k lists followed by a merge on every device.
#include <algorithm>
#include <cmath>
#include <numeric>

#include "fdb_device.cuh"
#include "fdb_internal.h"
#include "fdb_kernels.h"

namespace fdb {

void pq_train_dev(Ctx& ctx, const float* x, size_t n, int dim, int m, int iters,
                  const uint32_t* init_idx_host, float* cb, int* iters_out);

// ---------------------------------------------------------------------------
// small build kernels
// ---------------------------------------------------------------------------
__global__ void scatter_slot_kernel(const uint32_t* __restrict__ perm, size_t n,
                                    uint32_t* __restrict__ slot) {
    size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t < n) slot[perm[t]] = (uint32_t)t;
}

__global__ void permute_ids_kernel(const uint32_t* __restrict__ perm, size_t n,
                                   const uint64_t* __restrict__ ids, uint64_t* __restrict__ out) {
    size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t < n) out[t] = ids ? ids[perm[t]] : (uint64_t)perm[t];
}

// residual sample: out[i] = x[idx[i]] - cents[assign[idx[i]]]  (ivf_pq.rs:431-442)
__global__ void residual_gather_kernel(const float* __restrict__ x, size_t dim,
                                       const uint32_t* __restrict__ idx, size_t count,
                                       const uint32_t* __restrict__ assign,
                                       const float* __restrict__ cents, float* __restrict__ out) {
    size_t total = count * dim;
    for (size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (size_t)gridDim.x * blockDim.x) {
        size_t r = t / dim, c = t - r * dim;
        size_t v = idx[r];
        out[t] = __fsub_rn(x[v * dim + c], cents[(size_t)assign[v] * dim + c]);
    }
}

static unsigned blocks_for(size_t n, unsigned threads = 256) {
    return (unsigned)((n + threads - 1) / threads);
}

// ---------------------------------------------------------------------------
// k-means entry used by the C ABI and by the IVF build
// ---------------------------------------------------------------------------
// Draws for one k-means problem over n points (see fdb_train_opts).
static void kmeans_draws(size_t n, size_t k, const uint32_t* init_idx, const float* kpp_u,
                         uint64_t seed, std::vector<uint32_t>& idx, std::vector<float>& u) {
    idx.resize(k);
    u.assign(k, 0.0f);
    if (init_idx) {
        std::copy(init_idx, init_idx + k, idx.begin());
    } else if (k > 64) {
        sample_indices(seed, n, k, idx.data());
    } else {
        uint64_t st = seed ^ 0x6b6d65616e737070ull;  // independent stream for k-means++ picks
        for (size_t c = 0; c < k; ++c)
            idx[c] = (uint32_t)(((unsigned __int128)splitmix64(st) * n) >> 64);
    }
    if (k <= 64) {
        if (kpp_u) std::copy(kpp_u, kpp_u + k, u.begin());
        else uniform_draws(seed + 0x9e37ull, k, u.data());
    }
}

// Fits k centroids on device rows x[n][dim] (KMeans::fit_raw, kmeans.rs:87-193).
void kmeans_fit_dev(Ctx& ctx, const float* x, size_t n, int dim, int k, int max_iters,
                    const uint32_t* init_idx, const float* kpp_u, uint64_t seed, float* cent,
                    int* iters_run, uint32_t* init_rows, uint8_t* ever) {
    FDB_REQUIRE(n > 0 && dim > 0, FDB_ERR_EMPTY_TRAINING_SET, "k-means needs at least one point");
    FDB_REQUIRE(k > 0, FDB_ERR_INVALID_ARG, "k must be positive");
    std::vector<uint32_t> idx;
    std::vector<float> u;
    if (k > 64) {
        FDB_REQUIRE(n >= (size_t)k, FDB_ERR_INSUFFICIENT_VECTORS,
                    "random-sample init needs at least k points");
    }
    kmeans_draws(n, k, init_idx, kpp_u, seed, idx, u);
    if (k > 64) {
        for (int c = 0; c < k; ++c)
            FDB_REQUIRE(idx[c] < n, FDB_ERR_INVALID_ARG, "init index out of range");
        DevBuf<uint32_t> d_idx(k);
        FDB_CUDA(cudaMemcpyAsync(d_idx.p, idx.data(), k * sizeof(uint32_t),
                                 cudaMemcpyHostToDevice, ctx.stream));
        launch_gather_rows(ctx.stream, x, dim, d_idx.p, k, cent);
        FDB_CUDA(cudaStreamSynchronize(ctx.stream));
        if (init_rows) std::copy(idx.begin(), idx.end(), init_rows);
    } else {
        kmeans_pp_init(ctx, x, n, dim, k, idx.data(), u.data(), cent, init_rows);
    }
    KMeansProblem pb{x, n, dim, dim, 1, k, max_iters};
    int it = 0;
    kmeans_run(ctx, pb, cent, &it, ever);
    if (iters_run) *iters_run = it;
}

// ---------------------------------------------------------------------------
// IVF-PQ build
// ---------------------------------------------------------------------------
void ivfpq_build(fdb_ivfpq* h, const float* x_host, const uint64_t* ids_host, size_t n,
                 const fdb_train_opts& o) {
    Ctx& c = h->ctx->c;
    cudaStream_t s = c.stream;
    const int dim = (int)h->dim, nlist = (int)h->nlist, m = (int)h->m;
    FDB_REQUIRE(n > 0, FDB_ERR_EMPTY_VECTOR_SET, "IVF-PQ build needs at least one vector");
    FDB_REQUIRE(n < (1ull << 32), FDB_ERR_UNSUPPORTED, "at most 2^32-1 vectors per index");
    FDB_REQUIRE(h->dim % h->m == 0, FDB_ERR_DIM_NOT_DIVISIBLE,
                "dimension not divisible by the number of subvectors");
    const size_t ivf_n = o.ivf_sample ? std::min(o.ivf_sample, n) : std::min<size_t>(n, 30000);
    const size_t pq_n = o.pq_sample ? std::min(o.pq_sample, n) : std::min<size_t>(n, 100000);
    const int ivf_iters = o.ivf_iters ? (int)o.ivf_iters : 25;
    const int pq_iters = o.pq_iters ? (int)o.pq_iters : 25;
    FDB_REQUIRE(pq_n >= (size_t)KSUB, FDB_ERR_INSUFFICIENT_VECTORS,
                "PQ training needs at least 256 vectors");

    DevBuf<float> X(n * dim);
    FDB_CUDA(cudaMemcpyAsync(X.p, x_host, X.bytes(), cudaMemcpyHostToDevice, s));

    // 1. IVF training sample and k-means.
    std::vector<uint32_t> sidx(ivf_n);
    if (o.ivf_sample_idx) std::copy(o.ivf_sample_idx, o.ivf_sample_idx + ivf_n, sidx.begin());
    else if (ivf_n == n) std::iota(sidx.begin(), sidx.end(), 0u);  // all vectors, in order
    else sample_indices(o.seed, n, ivf_n, sidx.data());
    for (size_t i = 0; i < ivf_n; ++i)
        FDB_REQUIRE(sidx[i] < n, FDB_ERR_INVALID_ARG, "IVF sample index out of range");
    DevBuf<uint32_t> d_sidx(ivf_n);
    DevBuf<float> S(ivf_n * dim);
    FDB_CUDA(cudaMemcpyAsync(d_sidx.p, sidx.data(), ivf_n * 4, cudaMemcpyHostToDevice, s));
    launch_gather_rows(s, X.p, dim, d_sidx.p, ivf_n, S.p);
    h->cents.alloc((size_t)nlist * dim);
    int it = 0;
    std::vector<uint32_t> init_rows(nlist);
    std::vector<uint8_t> ever(std::max<size_t>((size_t)nlist, (size_t)m * KSUB));
    kmeans_fit_dev(c, S.p, ivf_n, dim, nlist, ivf_iters, o.ivf_init_idx, o.ivf_kpp_u,
                   o.seed + 1, h->cents.p, &it, init_rows.data(), ever.data());
    S.release();
    // Vector ids of the centroids as the reference stores them: a centroid
    // starts as a clone of a training vector (its id) and becomes
    // Vector::new(c, mean) once its cluster has members (kmeans.rs:52-61, 183).
    h->cent_ids.resize(nlist);
    for (int l = 0; l < nlist; ++l) {
        const uint32_t row = sidx[init_rows[l]];
        h->cent_ids[l] = ever[l] ? (uint64_t)l : (ids_host ? ids_host[row] : (uint64_t)row);
    }

    // 2. Assign all vectors; stable grouping keeps input order inside lists.
    DevBuf<uint32_t> assign(n), perm(n), slot(n);
    launch_assign(s, X.p, n, dim, dim, h->cents.p, nlist, assign.p);
    h->offs.alloc(nlist + 1);
    group_by_assignment(c, assign.p, n, nlist, perm.p, h->offs.p);
    scatter_slot_kernel<<<blocks_for(n), 256, 0, s>>>(perm.p, n, slot.p);
    FDB_LAUNCH_CHECK();

    // 3. PQ on a sample of residuals.
    std::vector<uint32_t> pidx(pq_n);
    if (o.pq_sample_idx) std::copy(o.pq_sample_idx, o.pq_sample_idx + pq_n, pidx.begin());
    else sample_indices(o.seed + 2, n, pq_n, pidx.data());
    for (size_t i = 0; i < pq_n; ++i)
        FDB_REQUIRE(pidx[i] < n, FDB_ERR_INVALID_ARG, "PQ sample index out of range");
    DevBuf<uint32_t> d_pidx(pq_n);
    DevBuf<float> R(pq_n * dim);
    FDB_CUDA(cudaMemcpyAsync(d_pidx.p, pidx.data(), pq_n * 4, cudaMemcpyHostToDevice, s));
    residual_gather_kernel<<<std::min<unsigned>(blocks_for(pq_n * dim), 148 * 32), 256, 0, s>>>(
        X.p, dim, d_pidx.p, pq_n, assign.p, h->cents.p, R.p);
    FDB_LAUNCH_CHECK();
    std::vector<uint32_t> pinit((size_t)m * KSUB);
    if (o.pq_init_idx) {
        std::copy(o.pq_init_idx, o.pq_init_idx + pinit.size(), pinit.begin());
    } else {
        for (int q = 0; q < m; ++q)
            sample_indices(o.seed + 3 + (uint64_t)q, pq_n, KSUB, pinit.data() + (size_t)q * KSUB);
    }
    const int sub = dim / m;
    h->cb.alloc((size_t)m * KSUB * sub);
    std::vector<int> pq_its(m);
    pq_train_dev(c, R.p, pq_n, dim, m, pq_iters, pinit.data(), h->cb.p, pq_its.data(),
                 ever.data());
    R.release();
    // codebook entries: fit_raw names a pick by its sample row (kmeans.rs:103)
    h->cb_ids.resize((size_t)m * KSUB);
    for (size_t e = 0; e < (size_t)m * KSUB; ++e)
        h->cb_ids[e] = ever[e] ? (uint64_t)(e % KSUB) : (uint64_t)pinit[e];

    // 4. Encode every residual into its list slot; ids in list order.
    h->codes.alloc(n * m);
    launch_pq_encode(s, X.p, n, dim, h->cents.p, assign.p, h->cb.p, m, slot.p, h->codes.p);
    DevBuf<uint64_t> d_ids_in;
    if (ids_host) {
        d_ids_in.alloc(n);
        FDB_CUDA(cudaMemcpyAsync(d_ids_in.p, ids_host, n * 8, cudaMemcpyHostToDevice, s));
    }
    h->ids.alloc(n);
    permute_ids_kernel<<<blocks_for(n), 256, 0, s>>>(perm.p, n, d_ids_in.p, h->ids.p);
    FDB_LAUNCH_CHECK();
    h->h_offs_full.resize(nlist + 1);
    FDB_CUDA(cudaMemcpyAsync(h->h_offs_full.data(), h->offs.p, (nlist + 1) * 8,
                             cudaMemcpyDeviceToHost, s));
    h->h_ids.resize(n);
    FDB_CUDA(cudaMemcpyAsync(h->h_ids.data(), h->ids.p, n * 8, cudaMemcpyDeviceToHost, s));
    FDB_CUDA(cudaStreamSynchronize(s));
    h->h_offs = h->h_offs_full;
    h->n_total = h->n_local = n;
    ivfpq_prepare_tables(h);
}

// Table and tensor modes need, per index: the bound terms cmax_s = max_l
// ||c_ls||, bmax_s = max_j ||b_sj|| (rounded up); the table mode also the
// per-list table btab (subvectors of 8+ floats only), the tensor mode the
// decoded codes (ivf_tc_prepare).
void ivfpq_prepare_tables(fdb_ivfpq* h) {
    const size_t nlist = h->nlist, dim = h->dim, m = h->m, sub = dim / m;
    h->btab.release();
    h->cmax.release();
    h->bmax.release();
    h->dec16.release();
    h->dnorm.release();
    h->centsT.release();
    if (dim <= (size_t)COARSE_TILED_MAX_DIM && nlist > 0) {
        h->nlist_pad = (int)((nlist + 127) / 128 * 128);
        h->centsT.alloc(dim * h->nlist_pad);
        launch_transpose_pad(h->ctx->c.stream, h->cents.p, (int)nlist, (int)dim, h->nlist_pad,
                             h->centsT.p);
    }
    coarse_tc_prepare(h);
    if (nlist == 0 || m == 0) return;
    Ctx& c = h->ctx->c;
    cudaStream_t s = c.stream;
    // the per-list table pays off for subvectors of 8+ floats (an exact LUT
    // entry then costs 8+ FMAs); the bound terms serve every certified mode
    if (sub >= 8) {
        h->btab.alloc(nlist * m * KSUB);
        launch_ivf_tables(s, h->cents.p, h->cb.p, (int)nlist, (int)m, (int)dim, h->btab.p);
    }
    std::vector<float> cents(nlist * dim), cb(m * KSUB * sub);
    FDB_CUDA(cudaMemcpyAsync(cents.data(), h->cents.p, cents.size() * 4, cudaMemcpyDeviceToHost, s));
    FDB_CUDA(cudaMemcpyAsync(cb.data(), h->cb.p, cb.size() * 4, cudaMemcpyDeviceToHost, s));
    FDB_CUDA(cudaStreamSynchronize(s));
    std::vector<float> cmax(m, 0.0f), bmax(m, 0.0f);
    for (size_t q = 0; q < m; ++q) {
        double cm = 0.0, bm = 0.0;
        for (size_t l = 0; l < nlist; ++l) {
            double t = 0.0;
            for (size_t i = 0; i < sub; ++i) {
                double x = cents[l * dim + q * sub + i];
                t += x * x;
            }
            cm = std::max(cm, std::sqrt(t));
        }
        for (size_t j = 0; j < (size_t)KSUB; ++j) {
            double t = 0.0;
            for (size_t i = 0; i < sub; ++i) {
                double x = cb[(q * KSUB + j) * sub + i];
                t += x * x;
            }
            bm = std::max(bm, std::sqrt(t));
        }
        cmax[q] = (float)(cm * (1.0 + 1e-6));
        bmax[q] = (float)(bm * (1.0 + 1e-6));
    }
    h->cmax.alloc(m);
    h->bmax.alloc(m);
    FDB_CUDA(cudaMemcpyAsync(h->cmax.p, cmax.data(), m * 4, cudaMemcpyHostToDevice, s));
    FDB_CUDA(cudaMemcpyAsync(h->bmax.p, bmax.data(), m * 4, cudaMemcpyHostToDevice, s));
    FDB_CUDA(cudaStreamSynchronize(s));
    ivf_tc_prepare(h, cb, bmax);
}

void ivfpq_load(fdb_ivfpq* h, const float* cents, const float* cb, const uint64_t* offsets,
                const uint64_t* ids, const uint8_t* codes) {
    Ctx& c = h->ctx->c;
    cudaStream_t s = c.stream;
    const size_t nlist = h->nlist, dim = h->dim, m = h->m;
    FDB_REQUIRE(offsets[0] == 0, FDB_ERR_INVALID_ARG, "offsets[0] must be 0");
    for (size_t l = 0; l < nlist; ++l)
        FDB_REQUIRE(offsets[l + 1] >= offsets[l], FDB_ERR_INVALID_ARG, "offsets must not decrease");
    const size_t n = offsets[nlist];
    FDB_REQUIRE(n < (1ull << 32), FDB_ERR_UNSUPPORTED, "at most 2^32-1 vectors per index");
    h->cents.alloc(nlist * dim);
    h->cb.alloc(m * KSUB * (dim / m));
    h->offs.alloc(nlist + 1);
    h->ids.alloc(n);
    h->codes.alloc(n * m);
    FDB_CUDA(cudaMemcpyAsync(h->cents.p, cents, h->cents.bytes(), cudaMemcpyHostToDevice, s));
    FDB_CUDA(cudaMemcpyAsync(h->cb.p, cb, h->cb.bytes(), cudaMemcpyHostToDevice, s));
    FDB_CUDA(cudaMemcpyAsync(h->offs.p, offsets, h->offs.bytes(), cudaMemcpyHostToDevice, s));
    if (n) {
        FDB_CUDA(cudaMemcpyAsync(h->ids.p, ids, n * 8, cudaMemcpyHostToDevice, s));
        FDB_CUDA(cudaMemcpyAsync(h->codes.p, codes, n * m, cudaMemcpyHostToDevice, s));
    }
    FDB_CUDA(cudaStreamSynchronize(s));
    h->h_offs_full.assign(offsets, offsets + nlist + 1);
    h->h_offs = h->h_offs_full;
    h->h_ids.assign(ids, ids + n);
    h->n_total = h->n_local = n;
    // ids the reference's trained Vectors would carry after a full fit
    if (h->cent_ids.size() != nlist) {
        h->cent_ids.resize(nlist);
        std::iota(h->cent_ids.begin(), h->cent_ids.end(), (uint64_t)0);
    }
    if (h->cb_ids.size() != m * KSUB) {
        h->cb_ids.resize(m * KSUB);
        for (size_t e = 0; e < m * KSUB; ++e) h->cb_ids[e] = e % KSUB;
    }
    ivfpq_prepare_tables(h);
}

// Greedy balance of list bytes: largest list first, onto the least-loaded
// device (ties: lower list index first, lower rank first).
void shard_plan(const uint64_t* sizes, size_t nlist, int world, int* owner) {
    std::vector<size_t> order(nlist);
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(),
                     [&](size_t a, size_t b) { return sizes[a] > sizes[b]; });
    std::vector<uint64_t> load(world, 0);
    for (size_t l : order) {
        int best = 0;
        for (int r = 1; r < world; ++r)
            if (load[r] < load[best]) best = r;
        owner[l] = best;
        load[best] += sizes[l];
    }
}

void ivfpq_shard(fdb_ivfpq* h, int rank, int world) {
    FDB_REQUIRE(world >= 1 && rank >= 0 && rank < world, FDB_ERR_INVALID_ARG, "bad rank/world");
    const size_t nlist = h->nlist;
    std::vector<uint64_t> sizes(nlist);
    for (size_t l = 0; l < nlist; ++l) sizes[l] = h->h_offs_full[l + 1] - h->h_offs_full[l];
    std::vector<int> owner(nlist);
    shard_plan(sizes.data(), nlist, world, owner.data());
    // Lists are scanned over [begin[l], end[l]).  A list held by another
    // device gets end == begin.  Row positions (the tie-break tags) stay
    // those of the unsharded index, so results do not depend on `world`.
    std::vector<uint64_t> be(2 * nlist);
    size_t held = 0;
    h->owned.assign(nlist, 0);
    for (size_t l = 0; l < nlist; ++l) {
        be[l] = h->h_offs_full[l];
        be[nlist + l] = owner[l] == rank ? h->h_offs_full[l + 1] : h->h_offs_full[l];
        if (owner[l] == rank) held += sizes[l];
        h->owned[l] = owner[l] == rank;
    }
    Ctx& c = h->ctx->c;
    h->shard_be.alloc(2 * nlist);
    FDB_CUDA(cudaMemcpyAsync(h->shard_be.p, be.data(), be.size() * 8, cudaMemcpyHostToDevice,
                             c.stream));
    FDB_CUDA(cudaStreamSynchronize(c.stream));
    h->n_local = held;
    h->sharded = world > 1;
    h->shard_world = world;
    h->shard_rank = rank;
}

void bf_shard(fdb_bf* h, int rank, int world) {
    FDB_REQUIRE(world >= 1 && rank >= 0 && rank < world, FDB_ERR_INVALID_ARG, "bad rank/world");
    const size_t total = h->h_ids.size();
    const size_t r0 = total * (size_t)rank / (size_t)world;
    const size_t r1 = total * (size_t)(rank + 1) / (size_t)world;
    h->row0 = r0;
    h->n = r1 - r0;
    h->sharded = world > 1;
    h->shard_world = world;
    h->dirty = true;
}

// ---------------------------------------------------------------------------
// IVF-PQ search on device buffers
// ---------------------------------------------------------------------------
static void exchange_and_merge(Ctx& c, size_t nq, int k, const uint64_t* local_keys,
                               const uint64_t* local_ids, DevBuf<uint64_t>& gather,
                               DevBuf<uint64_t>& merged, DevBuf<uint64_t>& merged_ids) {
    cudaStream_t s = c.stream;
    const size_t per = nq * (size_t)k;
    gather.ensure(per * 2 * (size_t)(c.world + 1));
    uint64_t* send = gather.p + per * 2 * (size_t)c.world;
    FDB_CUDA(cudaMemcpyAsync(send, local_keys, per * 8, cudaMemcpyDeviceToDevice, s));
    FDB_CUDA(cudaMemcpyAsync(send + per, local_ids, per * 8, cudaMemcpyDeviceToDevice, s));
    comm_mark(c, COMM_RESULTS);
    FDB_NCCL_C(ncclAllGather(send, gather.p, per * 2, ncclUint64, c.comm, s), c.comm);
    comm_mark(c, COMM_RESULTS);
    merged.ensure(per);
    merged_ids.ensure(per);
    launch_merge_lists(s, gather.p, c.world, per * 2, nq, k, merged.p);
    launch_lookup_gathered(s, merged.p, gather.p, gather.p + per, c.world, per * 2, nq, k,
                           merged_ids.p);
}

namespace {

using SearchRun = GraphSlot::Run;

// Every piece of device work of one search, enqueued on the context stream
// without a host synchronisation: probe selection, the scan, rescoring, the
// exchange of a sharded index, the results (and, with io, their copies to
// the host) and the end-of-call readbacks into pinned words.  The timers
// get their marks here.
SearchRun ivfpq_enqueue(fdb_ivfpq* h, const float* dQ, size_t nq, size_t k_out, size_t k,
                        int order, size_t take, uint64_t* d_ids, float* d_dists,
                        uint32_t* d_counts, fdb_stats* st, const uint32_t* call_skip,
                        const uint32_t* skip, const HostIO* io, StageTimer& tm,
                        StageTimer& pass_tm) {
    Ctx& c = h->ctx->c;
    cudaStream_t s = c.stream;
    const int nlist = (int)h->nlist;
    const size_t per = nq * k;
    bool tensor_ran = false;  // the tensor-core list scan ran
    bool waits_ran = false;   // some kernel with bounded waits ran (error word)
    tm.mark();
    h->s_keys.ensure(per);
    h->s_ids.ensure(per);
    if (take == 0) {  // marks 1..3 still taken so stage times line up
        // search() with nprobe == 0 probes nothing (ivf_pq.rs:548-552)
        FDB_CUDA(cudaMemsetAsync(h->s_keys.p, 0xff, per * 8, s));
    } else {
        // Probe selection.  Every device of a sharded index holds all
        // centroids, so each selects the probes of one slice of the queries
        // and an all-gather gives every device all probes and their coarse
        // distances (the slices are contiguous: rank-major = query-major).
        const int world = h->sharded ? c.world : 1, rank = h->sharded ? c.rank : 0;
        const size_t slice = (nq + world - 1) / world;
        const size_t q0 = std::min(nq, slice * (size_t)rank);
        const size_t nql = std::min(nq, q0 + slice) - q0;
        h->s_probe.ensure(slice * world * take);
        h->s_pdist.ensure(slice * world * take);
        // the error word of the bounded waits in the tensor-core kernels
        FDB_CUDA(cudaMemsetAsync(ivf_tc_error_word(h), 0, 4, s));
        if (nql > 0 && coarse_tc_eligible(h, nql, take)) {
            coarse_tc(h, dQ + q0 * h->dim, nql, take, h->s_probe.p + q0 * take,
                      h->s_pdist.p + q0 * take);
            waits_ran = true;
        } else if (nql > 0) {
            const float* Ql = dQ + q0 * h->dim;
            h->s_coarse.ensure(nql * (size_t)nlist);
            if (h->centsT.p) {
                const int nq_pad = (int)((nql + 31) / 32 * 32);
                h->s_qT.ensure(h->dim * (size_t)nq_pad);
                launch_transpose_pad(s, Ql, (int)nql, (int)h->dim, nq_pad, h->s_qT.p);
                launch_coarse_tiled(s, h->s_qT.p, (int)nql, nq_pad, (int)h->dim, h->centsT.p,
                                    nlist, h->nlist_pad, h->s_coarse.p);
            } else {
                launch_coarse_dist(s, Ql, (int)nql, (int)h->dim, h->cents.p, nlist,
                                   h->s_coarse.p);
            }
            launch_select(s, h->s_coarse.p, (int)nql, nlist, (int)take, h->s_probe.p + q0 * take,
                          h->s_pdist.p + q0 * take);
        }
        if (world > 1) {
            const size_t cnt = slice * take;
            comm_mark(c, COMM_PROBES);
            FDB_NCCL_C(ncclGroupStart(), c.comm);
            FDB_NCCL_C(ncclAllGather(h->s_probe.p + cnt * rank, h->s_probe.p, cnt, ncclUint32,
                                   c.comm, s), c.comm);
            FDB_NCCL_C(ncclAllGather(h->s_pdist.p + cnt * rank, h->s_pdist.p, cnt, ncclFloat,
                                   c.comm, s), c.comm);
            FDB_NCCL_C(ncclGroupEnd(), c.comm);
            comm_mark(c, COMM_PROBES);
        }
        tm.mark();
        h->s_stat.ensure(4);
        FDB_CUDA(cudaMemsetAsync(h->s_stat.p, 0, 32, s));
        const uint64_t* lbeg = h->sharded ? h->shard_be.p : h->offs.p;
        const uint64_t* lend = h->sharded ? h->shard_be.p + nlist : h->offs.p + 1;
        // Tensor mode: lists scored on the tensor cores into a shortlist,
        // exact rescoring + certification; failures are re-scanned exactly.
        // (rows a call skips -- tombstones, filters -- are +inf in the
        // tensor scan's ||rhat||^2 and never admitted)
        const bool tensor = ivf_tc_eligible(h, k) &&
                            (h->scan_mode == FDB_SCAN_TENSOR ||
                             (h->scan_mode == FDB_SCAN_AUTO && nq >= 256));
        // Table mode: approximate scan into a shortlist of kp keys, then
        // exact rescoring + certification; failures are re-scanned exactly.
        const bool tables = !tensor && h->btab.p && h->scan_mode != FDB_SCAN_EXACT && k <= 128;
        const size_t kp = tables ? std::min<size_t>(FDB_MAX_K, std::max<size_t>(32, 2 * k)) : k;
        if (tables) h->s_approx.ensure(nq * kp);
        ScanParams a{};
        a.Q = dQ;
        a.nq = (int)nq;
        a.dim = (int)h->dim;
        a.m = (int)h->m;
        a.cents = h->cents.p;
        a.cb = h->cb.p;
        a.offs = lbeg;
        a.ends = lend;
        a.codes = h->codes.p;
        a.probes = h->s_probe.p;
        a.nprobe = (int)take;
        a.k = (int)kp;
        a.out_keys = tables ? h->s_approx.p : h->s_keys.p;
        a.stat = h->s_stat.p;
        a.btab = tables ? h->btab.p : nullptr;
        a.skip = skip;
        if (tensor) {
            h->s_flags.ensure(nq + 1);
            h->tc_colv = call_skip ? ivfpq_call_colv(h, call_skip) : nullptr;
            try {
                ivf_tc_search(h, dQ, nq, k, order, take, lbeg, lend, h->s_keys.p,
                              h->s_flags.p, h->s_stat.p, st ? &pass_tm : nullptr);
            } catch (...) {
                h->tc_colv = nullptr;
                throw;
            }
            h->tc_colv = nullptr;
            tensor_ran = true;
            tm.mark();
            // exact re-scan of the lists that failed, merged with the certified
            // rest (counts stay on the device: no synchronisation here)
            ivf_tc_rescan(h, a, nq, k, order, h->s_keys.p);
        } else {
            launch_scan(s, a, order);
            tm.mark();
        }
        if (tables) {
            h->s_flags.ensure(nq + 1);
            FDB_CUDA(cudaMemsetAsync(h->s_flags.p, 0, 4, s));
            RescoreParams r{};
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
            r.kp = (int)kp;
            r.k = (int)k;
            r.out_keys = h->s_keys.p;
            r.cmax = h->cmax.p;
            r.bmax = h->bmax.p;
            r.flag_count = h->s_flags.p;
            r.flag_list = h->s_flags.p + 1;
            launch_rescore(s, r, order);
            uint32_t nflag = 0;
            FDB_CUDA(cudaMemcpyAsync(&nflag, h->s_flags.p, 4, cudaMemcpyDeviceToHost, s));
            FDB_CUDA(cudaStreamSynchronize(s));
            if (nflag > 0) {
                ScanParams e = a;
                e.nq = (int)nflag;
                e.qidx = h->s_flags.p + 1;
                e.k = (int)k;
                e.out_keys = h->s_keys.p;
                e.stat = nullptr;
                e.btab = nullptr;
                launch_scan(s, e, order);
            }
            if (st) st->exact_rescans = nflag;
        }
    }
    tm.mark();
    launch_keys_to_ids(s, h->s_keys.p, per, h->ids.p, 0, h->s_ids.p);
    const uint64_t* keys = h->s_keys.p;
    const uint64_t* ids = h->s_ids.p;
    if (h->sharded) {
        exchange_and_merge(c, nq, (int)k, h->s_keys.p, h->s_ids.p, h->s_gather, h->s_merged,
                           h->s_merged_ids);
        keys = h->s_merged.p;
        ids = h->s_merged_ids.p;
    }
    if (h->rerank) launch_rerank(h, keys, ids, nq, k, dQ, k_out, d_ids, d_dists, d_counts);
    else launch_finalize(s, keys, ids, nq, (int)k, d_ids, d_dists, d_counts);
    tm.mark();
    if (io && io->ids && k_out > 0) {  // results to the host before the one synchronisation
        FDB_CUDA(cudaMemcpyAsync(io->ids, d_ids, nq * k_out * 8, cudaMemcpyDeviceToHost, s));
        FDB_CUDA(cudaMemcpyAsync(io->dists, d_dists, nq * k_out * 4, cudaMemcpyDeviceToHost, s));
        if (io->counts)
            FDB_CUDA(cudaMemcpyAsync(io->counts, d_counts, nq * 4, cudaMemcpyDeviceToHost, s));
    }
    // The error word of the bounded waits and the statistics are read into
    // pinned words (after the caller's one synchronisation): pin[0..3]
    // statistics, pin[4] error word, pin[5] the number of re-scanned queries.
    waits_ran = waits_ran || tensor_ran;
    if (waits_ran || st || io) {
        uint64_t* pin = h->s_pin.get();
        if (waits_ran)
            FDB_CUDA(cudaMemcpyAsync(pin + 4, ivf_tc_error_word(h), 4, cudaMemcpyDeviceToHost, s));
        if (tensor_ran && st)
            FDB_CUDA(cudaMemcpyAsync(pin + 5, h->s_flags.p, 4, cudaMemcpyDeviceToHost, s));
        if (st && take > 0)
            FDB_CUDA(cudaMemcpyAsync(pin, h->s_stat.p, 32, cudaMemcpyDeviceToHost, s));
    }
    SearchRun r;
    r.tensor_ran = tensor_ran;
    r.waits_ran = waits_ran;
    return r;
}

// The pass-1 sampling quota for `take` probes on the tensor path: the one
// set or calibrated for this nprobe, else calibrated now on the first ns
// queries of this batch (up to 16384: the item structure of a small sample
// differs from a full batch's) -- each candidate quota runs the whole search
// on that sample twice (the first sizes the scratch) and the fastest second
// run (device time) wins.  The quota changes only how the work is split between
// the two list-scan passes; every quota returns the same (exact) answer.
uint64_t pass1_quota(fdb_ivfpq* h, const float* dQ, size_t nq, size_t k_out, size_t k,
                     int order, size_t take, const uint32_t* skip) {
    for (const auto& e : h->tc_quota)
        if (e.first == take) return e.second;
    constexpr uint64_t kDefault = 64;
    if (h->sharded || nq < 1024) return kDefault;  // ranks must agree; too small to time
    cudaStream_t s = h->ctx->c.stream;
    const size_t ns = std::min<size_t>(nq, 16384);
    h->s_cal_ids.ensure(ns * k_out);
    h->s_cal_d.ensure(ns * k_out);
    h->s_cal_c.ensure(ns);
    cudaEvent_t e0, e1;
    FDB_CUDA(cudaEventCreate(&e0));
    FDB_CUDA(cudaEventCreate(&e1));
    struct Ev {
        cudaEvent_t a, b;
        ~Ev() { cudaEventDestroy(a); cudaEventDestroy(b); }
    } ev{e0, e1};
    uint64_t best = kDefault;
    float best_ms = 0.0f;
    for (const uint64_t div : {128ull, 64ull, 16ull, 4ull, 0ull}) {
        h->tc_sample_div = div;
        float ms = 0.0f;
        for (int rep = 0; rep < 2; ++rep) {
            StageTimer off0(s, false), off1(s, false);
            FDB_CUDA(cudaEventRecord(e0, s));
            ivfpq_enqueue(h, dQ, ns, k_out, k, order, take, h->s_cal_ids.p, h->s_cal_d.p,
                          h->s_cal_c.p, nullptr, nullptr, skip, nullptr, off0, off1);
            FDB_CUDA(cudaEventRecord(e1, s));
            FDB_CUDA(cudaEventSynchronize(e1));
            FDB_CUDA(cudaEventElapsedTime(&ms, e0, e1));
        }
        if (best_ms == 0.0f || ms < best_ms) {
            best_ms = ms;
            best = div;
        }
    }
    h->tc_quota.emplace_back(take, best);
    return best;
}

// The search key of a captured graph: every value the enqueued work bakes
// into its launches (pointers, sizes, modes) besides the scratch buffers,
// whose addresses stay put while the allocation epoch is unchanged.
GraphKey search_key(const fdb_ivfpq* h, const float* dQ, size_t nq, size_t k_out, size_t k,
                    int order, size_t take, const uint64_t* d_ids, const float* d_dists,
                    const uint32_t* d_counts, const fdb_stats* st, const uint32_t* call_skip,
                    const uint32_t* skip, const HostIO* io) {
    GraphKey g{};
    g[0] = (uint64_t)dQ;
    g[1] = nq;
    g[2] = k_out;
    g[3] = k;
    g[4] = (uint64_t)order;
    g[5] = take;
    g[6] = (uint64_t)d_ids;
    g[7] = (uint64_t)d_dists;
    g[8] = (uint64_t)d_counts;
    g[9] = st != nullptr;
    g[10] = (uint64_t)call_skip;
    g[11] = (uint64_t)skip;
    g[12] = io ? (uint64_t)io->ids : 0;
    g[13] = io ? (uint64_t)io->dists : 0;
    g[14] = io ? (uint64_t)io->counts : 0;
    g[15] = ((uint64_t)h->scan_mode << 32) | (uint64_t)h->rerank;
    g[16] = h->rerank_factor;
    // a valid key; which marks are recorded (only a call with statistics has any)
    g[17] = 1 | ((st != nullptr && h->stage_timers) ? 2u : 0u);
    g[18] = h->tc_sample_div;
    return g;
}

}  // namespace

void ivfpq_search_dev(fdb_ivfpq* h, const float* dQ, size_t nq, size_t k_out, int order,
                      size_t take, uint64_t* d_ids, float* d_dists, uint32_t* d_counts,
                      fdb_stats* st, const uint32_t* call_skip, size_t fetch_mult,
                      const HostIO* io) {
    Ctx& c = h->ctx->c;
    cudaStream_t s = c.stream;
    if (st) std::memset(st, 0, sizeof(*st));
    if (nq == 0) return;
    ivfpq_sync_state(h);
    // fetch_k: with re-ranking, k * rerank_factor PQ candidates (ivf_pq.rs:591-596)
    const size_t k = h->rerank ? k_out * h->rerank_factor * fetch_mult : k_out;
    FDB_REQUIRE(k <= FDB_MAX_K, FDB_ERR_UNSUPPORTED,
                h->rerank ? "k * rerank_factor above FDB_MAX_K" : "k above FDB_MAX_K");
    // rows the scan skips: this call's filter, else the tombstoned rows
    const uint32_t* skip = call_skip ? call_skip : (h->n_tomb ? h->dead.p : nullptr);
    FDB_REQUIRE(!h->sharded || (c.comm && c.world == h->shard_world), FDB_ERR_INVALID_ARG,
                "sharded index needs a communicator of the same size");
    if (k == 0) return;
    // the tensor path's pass-1 quota for this nprobe (calibrated on first use)
    const bool tensor_path = ivf_tc_eligible(h, k) &&
                             (h->scan_mode == FDB_SCAN_TENSOR ||
                              (h->scan_mode == FDB_SCAN_AUTO && nq >= 256));
    if (tensor_path && take > 0)
        h->tc_sample_div = call_skip ? 64 : pass1_quota(h, dQ, nq, k_out, k, order, take, skip);
    // (the stage and collective marks are event records inside the step,
    // each a dependency point of its own; with stage_timers off a call with
    // statistics records only the two around the list scan's pass 2)
    StageTimer tm(s, st != nullptr && h->stage_timers);
    StageTimer pass_tm(s, st != nullptr);  // around each pass-2 launch (tensor mode)
    StageTimer comm_tm(s, st != nullptr && h->sharded && h->stage_timers);  // around collectives
    CommTimerScope comm_scope(c, comm_tm);
    uint64_t* pin = h->s_pin.get();
    for (int i = 0; i < 6; ++i) pin[i] = 0;
    // A search of one device whose work has no host synchronisation (it has
    // none unless the table mode's count readback) runs as a CUDA graph from
    // its second call with the same key: the first call runs eagerly (and
    // sizes every scratch buffer), the second is captured, later ones replay
    // it -- one launch instead of ~40.  The test hooks and a call's own
    // deadline keep a call eager.
    GraphCache& gc = h->graphs_cache;
    const bool graphable = h->graphs && !h->sharded && take > 0 &&
                           c.test_stalls.load() == 0 && h->call_wait_cycles == 0 &&
                           !(h->btab.p && h->scan_mode != FDB_SCAN_EXACT &&
                             !(ivf_tc_eligible(h, k) &&
                               (h->scan_mode == FDB_SCAN_TENSOR ||
                                (h->scan_mode == FDB_SCAN_AUTO && nq >= 256))) &&
                             k <= 128);
    const GraphKey key = search_key(h, dQ, nq, k_out, k, order, take, d_ids, d_dists, d_counts,
                                    st, call_skip, skip, io);
    const uint64_t epoch = devbuf_epoch().load();
    SearchRun r;
    GraphSlot* hit = graphable ? gc.find(key, epoch) : nullptr;
    if (hit) {
        FDB_CUDA(cudaGraphLaunch(hit->exec, s));
        r = hit->run;
        tm.borrow(hit->tm_ev);
        pass_tm.borrow(hit->pass_ev);
    } else if (graphable && gc.was_seen(key, epoch) && !gc.is_refused(key)) {
        GraphSlot* g = gc.take();
        g->ensure_events(32);
        tm.use_pool(&g->pool, 0);
        pass_tm.use_pool(&g->pool, 16);
        FDB_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
        bool ok = true;
        try {
            r = ivfpq_enqueue(h, dQ, nq, k_out, k, order, take, d_ids, d_dists, d_counts, st,
                              call_skip, skip, io, tm, pass_tm);
        } catch (...) {
            ok = false;
        }
        cudaGraph_t graph = nullptr;
        const cudaError_t ec = cudaStreamEndCapture(s, &graph);
        cudaGraphExec_t exec = nullptr;
        ok = ok && ec == cudaSuccess && graph && devbuf_epoch().load() == epoch &&
             cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess;
        if (graph) cudaGraphDestroy(graph);
        if (ok) {
            g->exec = exec;
            g->key = key;
            g->epoch = epoch;
            g->used = ++gc.clock;
            g->run = r;
            g->tm_ev = tm.ev;
            g->pass_ev = pass_tm.ev;
            FDB_CUDA(cudaGraphLaunch(exec, s));
        } else {
            // not capturable: this key stays eager
            if (exec) cudaGraphExecDestroy(exec);
            cudaGetLastError();
            if (gc.refused.size() == GraphCache::kSeen) gc.refused.erase(gc.refused.begin());
            gc.refused.push_back(key);
            tm.reset();
            pass_tm.reset();
            r = ivfpq_enqueue(h, dQ, nq, k_out, k, order, take, d_ids, d_dists, d_counts, st,
                              call_skip, skip, io, tm, pass_tm);
        }
    } else {
        r = ivfpq_enqueue(h, dQ, nq, k_out, k, order, take, d_ids, d_dists, d_counts, st,
                          call_skip, skip, io, tm, pass_tm);
        if (graphable) gc.note_seen(key, devbuf_epoch().load());  // after this call's allocations
    }
    const bool tensor_ran = r.tensor_ran;
    int tc_err = 0;
    if (r.waits_ran || st || io) {
        FDB_CUDA(cudaStreamSynchronize(s));
        tc_err = (int)(uint32_t)pin[4];
    }
    if (st) {
        const uint64_t* hs = h->s_pin.get();
        if (tensor_ran) {
            double pass_ms = 0.0;
            for (size_t i = 0; i + 1 < pass_tm.ev.size(); i += 2) pass_ms += pass_tm.ms(i, i + 1);
            st->kernel_ms = pass_ms;
            st->exact_rescans = (uint32_t)hs[5];
        }
        comm_scope.read(st);
        st->lists_probed = hs[0];
        st->extended = hs[3];
        st->codes_scanned = hs[1];
        st->bytes_scanned = hs[1] * h->m;
        size_t last = tm.ev.size() - 1;
        if (take > 0) {
            st->coarse_ms = tm.ms(0, 1);
            st->scan_ms = tm.ms(1, 2);
            st->rescore_ms = tm.ms(2, 3);
            st->merge_ms = tm.ms(3, 4);
            if (st->kernel_ms > 0.0) {
                st->kernel_scores = hs[2];  // tensor mode: pass 2 of the list scan
            } else {
                st->kernel_ms = st->scan_ms;  // the scan kernel
                st->kernel_scores = hs[1];
            }
        }
        st->total_ms = tm.ms(0, last);
    }
    FDB_REQUIRE(tc_err == 0, FDB_ERR_TIMEOUT, "a tensor-core kernel timed out on the device");
}

// ---------------------------------------------------------------------------
// brute force
// ---------------------------------------------------------------------------
__global__ void fill_f32_kernel(float* p, size_t n, float v) {
    size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    for (; t < n; t += (size_t)gridDim.x * blockDim.x) p[t] = v;
}

// 1/||x|| for the cosine shortlist (0 for a zero row).
__global__ void rsqrt_kernel(const float* __restrict__ norms, size_t n, float* __restrict__ out) {
    size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t < n) out[t] = norms[t] > 0.0f ? rsqrtf(norms[t]) : 0.0f;
}

__global__ void max_norm_kernel(const float* __restrict__ norms, size_t n, unsigned* out) {
    unsigned best = 0;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        best = max(best, __float_as_uint(norms[i]));  // non-negative floats order as uints
    atomicMax(out, best);
}

__global__ void scatter_rows_u64(const uint64_t* __restrict__ src, const uint32_t* __restrict__ idx,
                                 size_t count, int k, uint64_t* __restrict__ dst) {
    size_t t = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= count * (size_t)k) return;
    size_t r = t / k;
    dst[(size_t)idx[r] * k + (t - r * k)] = src[t];
}

// The tensor-core shortlist serves every metric but Manhattan, dims up to 256
// and k up to 128 (shortlists of max(32, 2k) keys).
static bool bf_tensor_ok(const fdb_bf* h, size_t k) {
    return h->scan_mode != FDB_SCAN_EXACT && h->metric != MANHATTAN && h->dim <= 256 &&
           k >= 1 && k <= 128;
}

void bf_upload(fdb_bf* h) {
    if (!h->dirty) return;
    Ctx& c = h->ctx->c;
    cudaStream_t s = c.stream;
    h->x.alloc(h->n * h->dim);
    h->ids.alloc(h->n);
    if (h->n) {
        FDB_CUDA(cudaMemcpyAsync(h->x.p, h->h_x.data() + h->row0 * h->dim, h->x.bytes(),
                                 cudaMemcpyHostToDevice, s));
        FDB_CUDA(cudaMemcpyAsync(h->ids.p, h->h_ids.data() + h->row0, h->ids.bytes(),
                                 cudaMemcpyHostToDevice, s));
    }
    // squared norms in the AVX2 order (cosine needs them exactly; the
    // tensor-core path uses them for every metric).  Padded by two tiles of
    // +inf so the epilogue's whole-chunk loads stay in bounds.
    h->norms.alloc(h->n + 256);
    fill_f32_kernel<<<1, 256, 0, s>>>(h->norms.p + h->n, 256, INFINITY);
    FDB_LAUNCH_CHECK();
    launch_row_norms(s, h->x.p, h->n, (int)h->dim, h->norms.p);
    h->rnorms.release();
    if (h->metric == COSINE) {
        h->rnorms.alloc(h->n + 256);
        FDB_CUDA(cudaMemsetAsync(h->rnorms.p, 0, (h->n + 256) * 4, s));
        rsqrt_kernel<<<(unsigned)((h->n + 255) / 256), 256, 0, s>>>(h->norms.p, h->n,
                                                                    h->rnorms.p);
        FDB_LAUNCH_CHECK();
    }
    h->x16.release();
    h->xmax = 0.0f;
    if (h->metric != MANHATTAN && h->dim <= 256 && h->n > 0) {
        h->kpad = (int)((h->dim + 63) / 64 * 64);
        h->x16.alloc(h->n * (size_t)h->kpad);
        launch_to_half(s, h->x.p, h->n, (int)h->dim, h->kpad, h->x16.p);
        DevBuf<unsigned> mx(1);
        FDB_CUDA(cudaMemsetAsync(mx.p, 0, 4, s));
        max_norm_kernel<<<148, 256, 0, s>>>(h->norms.p, h->n, mx.p);
        FDB_LAUNCH_CHECK();
        unsigned bits = 0;
        FDB_CUDA(cudaMemcpyAsync(&bits, mx.p, 4, cudaMemcpyDeviceToHost, s));
        FDB_CUDA(cudaStreamSynchronize(s));
        float m2;
        std::memcpy(&m2, &bits, 4);
        h->xmax = (float)(std::sqrt((double)m2) * (1.0 + 1e-6));
    }
    FDB_CUDA(cudaStreamSynchronize(s));
    h->dirty = false;
}

// Exact SIMT scan of nq contiguous queries into keys[nq][k].
static void bf_exact_scan(fdb_bf* h, const float* dQ, size_t nq, size_t k, const float* qn,
                          uint64_t* keys) {
    Ctx& c = h->ctx->c;
    cudaStream_t s = c.stream;
    size_t psz = bf_part_size(h->n, (int)nq, (int)k, c.sm_count);
    h->s_part.ensure(psz);
    int chunks = launch_bf_scan(s, h->metric, dQ, (int)nq, qn, h->x.p, h->n, (int)h->dim,
                                h->norms.p, h->row0, (int)k, c.sm_count, h->s_part.p, h->s_part.n);
    launch_merge_lists(s, h->s_part.p, chunks, nq * k, nq, (int)k, keys);
}

void bf_search_dev(fdb_bf* h, const float* dQ, size_t nq, size_t k, uint64_t* d_ids,
                   float* d_dists, uint32_t* d_counts, fdb_stats* st) {
    Ctx& c = h->ctx->c;
    cudaStream_t s = c.stream;
    if (st) std::memset(st, 0, sizeof(*st));
    if (nq == 0) return;
    bf_upload(h);
    FDB_REQUIRE(k <= FDB_MAX_K, FDB_ERR_UNSUPPORTED, "k above FDB_MAX_K");
    FDB_REQUIRE(!h->sharded || (c.comm && c.world == h->shard_world), FDB_ERR_INVALID_ARG,
                "sharded index needs a communicator of the same size");
    StageTimer tm(s, st != nullptr);
    StageTimer comm_tm(s, st != nullptr && h->sharded);  // around the exchange
    CommTimerScope comm_scope(c, comm_tm);
    tm.mark();
    if (k == 0) return;
    const size_t per = nq * k;
    h->s_keys.ensure(per);
    h->s_ids.ensure(per);
    uint32_t nflag = 0;
    if (h->n == 0) {
        FDB_CUDA(cudaMemsetAsync(h->s_keys.p, 0xff, per * 8, s));
        tm.mark();
    } else {
        h->s_qnorm.ensure(nq);
        launch_row_norms(s, dQ, nq, (int)h->dim, h->s_qnorm.p);
        const float* qn = h->s_qnorm.p;
        if (h->x16.p && bf_tensor_ok(h, k)) {
            // tensor-core shortlist -> exact rescore -> certified, else exact re-scan
            const size_t kp = std::min<size_t>(256, std::max<size_t>(32, 2 * k));
            h->s_q16.ensure(nq * (size_t)h->kpad);
            launch_to_half(s, dQ, nq, (int)h->dim, h->kpad, h->s_q16.p);
            h->s_flags.ensure(nq + 2);
            FDB_CUDA(cudaMemsetAsync(h->s_flags.p, 0, 8, s));
            int* err = reinterpret_cast<int*>(h->s_flags.p + nq + 1);
            FDB_CUDA(cudaMemsetAsync(err, 0, 4, s));
            h->gemm.err = err;
            h->gemm.wait_cycles = wait_limit_cycles(c);
            // device time of the filter pass, when statistics are asked for
            cudaEvent_t fev[2] = {nullptr, nullptr};
            if (st) {
                FDB_CUDA(cudaEventCreate(&fev[0]));
                FDB_CUDA(cudaEventCreate(&fev[1]));
            }
            struct EvPair {
                cudaEvent_t* e;
                ~EvPair() { for (int i = 0; i < 2; ++i) if (e[i]) cudaEventDestroy(e[i]); }
            } fev_free{fev};
            h->gemm.filter_ev0 = fev[0];
            h->gemm.filter_ev1 = fev[1];
            gemm_shortlist(s, h->s_q16.p, (int)nq, qn, h->x16.p, h->n, h->kpad,
                           h->metric == COSINE ? h->rnorms.p : h->norms.p, h->metric, h->row0,
                           (int)kp, c.sm_count, h->xmax * h->xmax, h->gemm);
            tm.mark();
            launch_bf_rescore(s, dQ, (int)nq, h->x.p, (int)h->dim, qn, h->norms.p, h->xmax,
                              h->metric,
                              h->row0, h->gemm, (int)kp, (int)k, h->s_keys.p, h->s_flags.p,
                              h->s_flags.p + 1);
            uint32_t hv[2] = {0, 0};
            FDB_CUDA(cudaMemcpyAsync(&hv[0], h->s_flags.p, 4, cudaMemcpyDeviceToHost, s));
            FDB_CUDA(cudaMemcpyAsync(&hv[1], err, 4, cudaMemcpyDeviceToHost, s));
            FDB_CUDA(cudaStreamSynchronize(s));
            FDB_REQUIRE(hv[1] == 0, FDB_ERR_TIMEOUT, "tensor-core scan timed out on the device");
            nflag = hv[0];
            if (st) {
                float ms = 0.0f;
                FDB_CUDA(cudaEventElapsedTime(&ms, fev[0], fev[1]));
                st->kernel_ms = ms;
                st->kernel_scores = (uint64_t)nq * h->n;
            }
            h->gemm.filter_ev0 = h->gemm.filter_ev1 = nullptr;
            if (nflag > 0) {
                DevBuf<float> qf(nflag * h->dim), qfn(nflag);
                DevBuf<uint64_t> kf(nflag * k);
                launch_gather_rows(s, dQ, h->dim, h->s_flags.p + 1, nflag, qf.p);
                launch_row_norms(s, qf.p, nflag, (int)h->dim, qfn.p);
                bf_exact_scan(h, qf.p, nflag, k, qfn.p, kf.p);
                scatter_rows_u64<<<(unsigned)((nflag * k + 255) / 256), 256, 0, s>>>(
                    kf.p, h->s_flags.p + 1, nflag, (int)k, h->s_keys.p);
                FDB_LAUNCH_CHECK();
                FDB_CUDA(cudaStreamSynchronize(s));
            }
        } else {
            bf_exact_scan(h, dQ, nq, k, qn, h->s_keys.p);
            tm.mark();
        }
    }
    tm.mark();
    launch_keys_to_ids(s, h->s_keys.p, per, h->ids.p, h->row0, h->s_ids.p);
    const uint64_t* keys = h->s_keys.p;
    const uint64_t* ids = h->s_ids.p;
    if (h->sharded) {
        exchange_and_merge(c, nq, (int)k, h->s_keys.p, h->s_ids.p, h->s_gather, h->s_merged,
                           h->s_merged_ids);
        keys = h->s_merged.p;
        ids = h->s_merged_ids.p;
    }
    launch_finalize(s, keys, ids, nq, (int)k, d_ids, d_dists, d_counts);
    tm.mark();
    if (st) {
        FDB_CUDA(cudaStreamSynchronize(s));
        st->lists_probed = 0;
        st->codes_scanned = (uint64_t)nq * h->n;
        if (st->kernel_ms == 0.0 && tm.ev.size() >= 4) {  // exact SIMT scan
            st->kernel_ms = tm.ms(0, 1);
            st->kernel_scores = (uint64_t)nq * h->n;
        }
        st->bytes_scanned = (uint64_t)h->n * h->dim * 4;
        st->exact_rescans = nflag;
        if (tm.ev.size() >= 4) {
            st->scan_ms = tm.ms(0, 1);
            st->rescore_ms = tm.ms(1, 2);
            st->merge_ms = tm.ms(2, 3);
            st->total_ms = tm.ms(0, 3);
        }
        comm_scope.read(st);
    }
}

}  // namespace fdb
