// capi.cu -- the extern "C" entry points of include/forgegpu.h.
//
// Each entry point validates its arguments the way the reference's Rust
// method does (panics become error codes), makes the context's device
// current, runs the engine and converts any failure into a status code plus
// a thread-local message.  The product path has no CPU fallback: if the
// device work cannot run, the call fails.
#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <memory>
#include <new>
#include <numeric>
#include <thread>

#include "fdb_device.cuh"
#include "fdb_internal.h"
#include "fdb_kernels.h"

namespace fdb {

static thread_local std::string g_last_error;

void fail(int code, const std::string& msg) { throw Error{code, msg}; }
void set_last_error(const std::string& msg) { g_last_error = msg; }

static double now_s() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch())
        .count();
}

// Polls a non-blocking communicator until its pending operation leaves
// ncclInProgress or `limit_s` passes.  Returns the final state, or
// ncclInProgress if the limit ran out.
static ncclResult_t nccl_settle(ncclComm_t comm, double limit_s) {
    const double t0 = now_s();
    ncclResult_t st = ncclInProgress;
    for (;;) {
        if (ncclCommGetAsyncError(comm, &st) != ncclSuccess) return ncclInternalError;
        if (st != ncclInProgress) return st;
        if (now_s() - t0 > limit_s) return ncclInProgress;
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

void nccl_complete(ncclResult_t r, ncclComm_t comm, const char* what) {
    if (r == ncclInProgress && comm) r = nccl_settle(comm, 300.0);
    if (r == ncclInProgress)
        fail(FDB_ERR_TIMEOUT, std::string(what) + ": did not complete within 300 s");
    if (r != ncclSuccess) fail(FDB_ERR_NCCL, std::string(what) + ": " + ncclGetErrorString(r));
}

// Releases a communicator: finalize (flushes its operations; bounded), then
// destroy, or abort when the finalize does not complete.
static void release_comm(ncclComm_t comm) {
    if (!comm) return;
    ncclResult_t r = ncclCommFinalize(comm);
    if (r == ncclInProgress) r = nccl_settle(comm, 10.0);
    if (r == ncclSuccess) ncclCommDestroy(comm);
    else ncclCommAbort(comm);
}

uint64_t splitmix64(uint64_t& state) {
    uint64_t z = (state += 0x9e3779b97f4a7c15ull);
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

// Partial Fisher-Yates over 0..n-1; the first `take` slots are a uniform
// random ordered sample without replacement.
void sample_indices(uint64_t seed, size_t n, size_t take, uint32_t* out) {
    FDB_REQUIRE(take <= n, FDB_ERR_INVALID_ARG, "cannot take more indices than exist");
    FDB_REQUIRE(n < (1ull << 32), FDB_ERR_UNSUPPORTED, "index space above 2^32");
    std::vector<uint32_t> idx(n);
    std::iota(idx.begin(), idx.end(), 0u);
    uint64_t st = seed;
    for (size_t i = 0; i < take; ++i) {
        uint64_t range = n - i;
        size_t j = i + (size_t)(((unsigned __int128)splitmix64(st) * range) >> 64);
        std::swap(idx[i], idx[j]);
    }
    std::copy(idx.begin(), idx.begin() + take, out);
}

// rand's f32 sampler keeps 23 random bits: u = bits * 2^-23 in [0, 1).
void uniform_draws(uint64_t seed, size_t count, float* out) {
    uint64_t st = seed;
    for (size_t i = 0; i < count; ++i)
        out[i] = (float)(splitmix64(st) >> 41) * (1.0f / 8388608.0f);
}

}  // namespace fdb

using namespace fdb;

namespace {

template <class F>
int guarded(F&& f) {
    try {
        f();
        return FDB_OK;
    } catch (const Error& e) {
        set_last_error(e.msg);
        return e.code;
    } catch (const std::bad_alloc&) {
        set_last_error("host allocation failed");
        return FDB_ERR_OOM;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return FDB_ERR_INVALID_ARG;
    }
}

void check_metric(int metric) {
    FDB_REQUIRE(metric >= FDB_METRIC_EUCLIDEAN && metric <= FDB_METRIC_MANHATTAN,
                FDB_ERR_INVALID_ARG, "unknown metric");
}

// Pinned-or-not host <-> device staging for the host-buffer entry points.
struct Staged {
    DevBuf<uint64_t> ids;
    DevBuf<float> dists;
    DevBuf<uint32_t> counts;
};

}  // namespace

extern "C" {

const char* fdb_last_error(void) { return g_last_error.c_str(); }

int fdb_version(void) { return 100; }

int fdb_ctx_create(int device, fdb_ctx** out) {
    return guarded([&] {
        FDB_REQUIRE(out, FDB_ERR_INVALID_ARG, "out is NULL");
        int ndev = 0;
        FDB_CUDA(cudaGetDeviceCount(&ndev));
        FDB_REQUIRE(device >= 0 && device < ndev, FDB_ERR_INVALID_ARG, "no such CUDA device");
        std::unique_ptr<fdb_ctx> c(new fdb_ctx());
        c->c.device = device;
        DeviceGuard g(device);
        cudaDeviceProp prop;
        FDB_CUDA(cudaGetDeviceProperties(&prop, device));
        FDB_REQUIRE(prop.major >= 10, FDB_ERR_UNSUPPORTED,
                    "this build targets sm_100a (B200); device is older");
        c->c.sm_count = prop.multiProcessorCount;
        int khz = 0;
        if (cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, device) == cudaSuccess && khz > 0)
            c->c.clock_khz = khz;
        c->c.wait_cycles = seconds_to_cycles(c->c, c->c.wait_s.load());
        FDB_CUDA(cudaStreamCreateWithFlags(&c->c.stream, cudaStreamNonBlocking));
        *out = c.release();
    });
}

int fdb_ctx_free(fdb_ctx* ctx) {
    return guarded([&] {
        if (!ctx) return;
        {
            DeviceGuard g(ctx->c.device);
            release_comm(ctx->c.comm);
            if (ctx->c.stream) cudaStreamDestroy(ctx->c.stream);
        }
        delete ctx;
    });
}

int fdb_ctx_stream(fdb_ctx* ctx, void** stream_out) {
    return guarded([&] {
        FDB_REQUIRE(ctx && stream_out, FDB_ERR_INVALID_ARG, "NULL argument");
        *stream_out = (void*)ctx->c.stream;
    });
}

int fdb_nccl_unique_id(void* id_out) {
    return guarded([&] {
        FDB_REQUIRE(id_out, FDB_ERR_INVALID_ARG, "NULL argument");
        static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id is 128 bytes");
        ncclUniqueId id;
        FDB_NCCL(ncclGetUniqueId(&id));
        std::memcpy(id_out, &id, sizeof(id));
    });
}

int fdb_ctx_init_comm_timeout(fdb_ctx* ctx, int rank, int world, const void* nccl_id,
                              double timeout_s) {
    return guarded([&] {
        FDB_REQUIRE(ctx && nccl_id, FDB_ERR_INVALID_ARG, "NULL argument");
        FDB_REQUIRE(world >= 1 && rank >= 0 && rank < world, FDB_ERR_INVALID_ARG,
                    "bad rank/world");
        FDB_REQUIRE(timeout_s > 0.0, FDB_ERR_INVALID_ARG, "timeout must be positive");
        DeviceGuard g(ctx->c.device);
        std::lock_guard<std::mutex> lk(ctx->c.mu);
        release_comm(ctx->c.comm);
        ctx->c.comm = nullptr;
        ctx->c.rank = 0;
        ctx->c.world = 1;
        ncclUniqueId id;
        std::memcpy(&id, nccl_id, sizeof(id));
        // non-blocking: the join of all ranks can be given up on a deadline
        ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
        cfg.blocking = 0;
        ncclComm_t comm = nullptr;
        ncclResult_t r = ncclCommInitRankConfig(&comm, world, id, rank, &cfg);
        if (r == ncclInProgress) r = nccl_settle(comm, timeout_s);
        if (r != ncclSuccess) {
            if (comm) ncclCommAbort(comm);
            if (r == ncclInProgress)
                fail(FDB_ERR_TIMEOUT, "NCCL communicator: not every rank joined within the "
                                      "timeout; initialisation aborted");
            fail(FDB_ERR_NCCL, std::string("ncclCommInitRankConfig: ") + ncclGetErrorString(r));
        }
        ctx->c.comm = comm;
        ctx->c.rank = rank;
        ctx->c.world = world;
    });
}

int fdb_ctx_init_comm(fdb_ctx* ctx, int rank, int world, const void* nccl_id) {
    return fdb_ctx_init_comm_timeout(ctx, rank, world, nccl_id, 300.0);
}

int fdb_ctx_set_wait_limit(fdb_ctx* ctx, double seconds) {
    return guarded([&] {
        FDB_REQUIRE(ctx, FDB_ERR_INVALID_ARG, "NULL context");
        FDB_REQUIRE(seconds > 0.0 && seconds <= 3600.0, FDB_ERR_INVALID_ARG,
                    "wait limit must be in (0, 3600] seconds");
        ctx->c.wait_s = seconds;
        ctx->c.wait_cycles = seconds_to_cycles(ctx->c, seconds);
    });
}

int fdb_ctx_test_stall_scans(fdb_ctx* ctx, int count) {
    return guarded([&] {
        FDB_REQUIRE(ctx && count >= 0, FDB_ERR_INVALID_ARG, "bad arguments");
        ctx->c.test_stalls = count;
    });
}

int fdb_host_alloc(size_t bytes, void** out) {
    return guarded([&] {
        FDB_REQUIRE(out, FDB_ERR_INVALID_ARG, "NULL argument");
        FDB_CUDA(cudaHostAlloc(out, bytes ? bytes : 1, cudaHostAllocPortable));
    });
}

int fdb_host_free(void* p) {
    return guarded([&] {
        if (p) FDB_CUDA(cudaFreeHost(p));
    });
}

int fdb_sample_indices(uint64_t seed, size_t n, size_t take, uint32_t* out) {
    return guarded([&] {
        FDB_REQUIRE(out || take == 0, FDB_ERR_INVALID_ARG, "NULL argument");
        sample_indices(seed, n, take, out);
    });
}

int fdb_uniform_draws(uint64_t seed, size_t count, float* out) {
    return guarded([&] {
        FDB_REQUIRE(out || count == 0, FDB_ERR_INVALID_ARG, "NULL argument");
        uniform_draws(seed, count, out);
    });
}

// ---------------------------------------------------------------------------
// distances
// ---------------------------------------------------------------------------
int fdb_pairwise_distance(fdb_ctx* ctx, int metric, const float* a, const float* b, size_t n,
                          size_t dim, float* out) {
    return guarded([&] {
        FDB_REQUIRE(ctx && (n == 0 || (a && b && out)), FDB_ERR_INVALID_ARG, "NULL argument");
        check_metric(metric);
        if (n == 0) return;
        DeviceGuard g(ctx->c.device);
        std::lock_guard<std::mutex> lk(ctx->c.mu);
        cudaStream_t s = ctx->c.stream;
        DevBuf<float> da(n * dim), db(n * dim), dout(n);
        FDB_CUDA(cudaMemcpyAsync(da.p, a, da.bytes(), cudaMemcpyHostToDevice, s));
        FDB_CUDA(cudaMemcpyAsync(db.p, b, db.bytes(), cudaMemcpyHostToDevice, s));
        launch_pairwise(s, metric, da.p, db.p, n, (int)dim, dout.p);
        FDB_CUDA(cudaMemcpyAsync(out, dout.p, n * 4, cudaMemcpyDeviceToHost, s));
        FDB_CUDA(cudaStreamSynchronize(s));
    });
}

// ---------------------------------------------------------------------------
// k-means
// ---------------------------------------------------------------------------
int fdb_kmeans_fit(fdb_ctx* ctx, const float* data, size_t n, size_t dim, size_t k,
                   size_t max_iters, const uint32_t* init_idx, const float* kpp_u, uint64_t seed,
                   float* centroids_out, uint32_t* assign_out, int* iters_run) {
    return guarded([&] {
        FDB_REQUIRE(ctx && centroids_out, FDB_ERR_INVALID_ARG, "NULL argument");
        FDB_REQUIRE(n > 0 && dim > 0 && data, FDB_ERR_EMPTY_TRAINING_SET,
                    "k-means needs at least one point");
        FDB_REQUIRE(k > 0 && k < (1u << 31), FDB_ERR_INVALID_ARG, "bad k");
        FDB_REQUIRE(n < (1ull << 32), FDB_ERR_UNSUPPORTED, "at most 2^32-1 points");
        DeviceGuard g(ctx->c.device);
        std::lock_guard<std::mutex> lk(ctx->c.mu);
        cudaStream_t s = ctx->c.stream;
        DevBuf<float> X(n * dim), C(k * dim);
        FDB_CUDA(cudaMemcpyAsync(X.p, data, X.bytes(), cudaMemcpyHostToDevice, s));
        int it = 0;
        kmeans_fit_dev(ctx->c, X.p, n, (int)dim, (int)k, (int)max_iters, init_idx, kpp_u, seed,
                       C.p, &it);
        FDB_CUDA(cudaMemcpyAsync(centroids_out, C.p, C.bytes(), cudaMemcpyDeviceToHost, s));
        if (assign_out) {
            DevBuf<uint32_t> A(n);
            launch_assign(s, X.p, n, (int)dim, (int)dim, C.p, (int)k, A.p);
            FDB_CUDA(cudaMemcpyAsync(assign_out, A.p, n * 4, cudaMemcpyDeviceToHost, s));
            FDB_CUDA(cudaStreamSynchronize(s));
        }
        FDB_CUDA(cudaStreamSynchronize(s));
        if (iters_run) *iters_run = it;
    });
}

int fdb_assign(fdb_ctx* ctx, const float* x, size_t n, const float* centroids, size_t k,
               size_t dim, uint32_t* out) {
    return guarded([&] {
        FDB_REQUIRE(ctx && (n == 0 || (x && out)) && centroids, FDB_ERR_INVALID_ARG,
                    "NULL argument");
        FDB_REQUIRE(k > 0, FDB_ERR_INVALID_ARG, "no centroids");
        if (n == 0) return;
        DeviceGuard g(ctx->c.device);
        std::lock_guard<std::mutex> lk(ctx->c.mu);
        cudaStream_t s = ctx->c.stream;
        DevBuf<float> X(n * dim), C(k * dim);
        DevBuf<uint32_t> A(n);
        FDB_CUDA(cudaMemcpyAsync(X.p, x, X.bytes(), cudaMemcpyHostToDevice, s));
        FDB_CUDA(cudaMemcpyAsync(C.p, centroids, C.bytes(), cudaMemcpyHostToDevice, s));
        launch_assign(s, X.p, n, (int)dim, (int)dim, C.p, (int)k, A.p);
        FDB_CUDA(cudaMemcpyAsync(out, A.p, n * 4, cudaMemcpyDeviceToHost, s));
        FDB_CUDA(cudaStreamSynchronize(s));
    });
}

int fdb_find_nearest_centroids(fdb_ctx* ctx, const float* centroids, size_t kc, size_t dim,
                               const float* query, size_t k, uint32_t* out) {
    return guarded([&] {
        FDB_REQUIRE(ctx && centroids && query && (k == 0 || out), FDB_ERR_INVALID_ARG,
                    "NULL argument");
        size_t take = std::min(k, kc);
        if (take == 0) return;
        DeviceGuard g(ctx->c.device);
        std::lock_guard<std::mutex> lk(ctx->c.mu);
        cudaStream_t s = ctx->c.stream;
        DevBuf<float> C(kc * dim), Q(dim), D(kc);
        DevBuf<uint32_t> P(take);
        FDB_CUDA(cudaMemcpyAsync(C.p, centroids, C.bytes(), cudaMemcpyHostToDevice, s));
        FDB_CUDA(cudaMemcpyAsync(Q.p, query, Q.bytes(), cudaMemcpyHostToDevice, s));
        launch_coarse_dist(s, Q.p, 1, (int)dim, C.p, (int)kc, D.p);
        launch_select(s, D.p, 1, (int)kc, (int)take, P.p);
        FDB_CUDA(cudaMemcpyAsync(out, P.p, take * 4, cudaMemcpyDeviceToHost, s));
        FDB_CUDA(cudaStreamSynchronize(s));
    });
}

}  // extern "C"

// Distance matrix of fdb_find_nearest_centroids_noalloc.  It is part of the
// library's device image (reserved when the module loads on a device), so
// that entry point never allocates.  The distance kernel writes every entry
// the selection reads, so nothing in it has to start at zero.
static __device__ __align__(256) float g_noalloc_dist[FDB_NOALLOC_MAX_DISTANCES];

namespace {

// Address of g_noalloc_dist on `device`, looked up once per device with that
// device current (the caller's DeviceGuard) and remembered for the life of
// the process.  A cudaDeviceReset of that device unloads the module and
// leaves the remembered address stale; like every other handle of this
// library on that device, it must not be used after a reset.
float* noalloc_scratch(int device) {
    constexpr int kMaxDevices = 64;
    static std::mutex mu;
    static float* table[kMaxDevices] = {};
    FDB_REQUIRE(device >= 0 && device < kMaxDevices, FDB_ERR_UNSUPPORTED,
                "device ordinal above 63");
    std::lock_guard<std::mutex> lk(mu);
    if (!table[device]) {
        void* p = nullptr;
        FDB_CUDA(cudaGetSymbolAddress(&p, g_noalloc_dist));
        FDB_REQUIRE(p != nullptr, FDB_ERR_CUDA, "scratch symbol has no device address");
        table[device] = static_cast<float*>(p);
    }
    return table[device];
}

}  // namespace

extern "C" {

int fdb_find_nearest_centroids_noalloc(fdb_ctx* ctx, const float* d_centroids, size_t kc,
                                       size_t dim, const float* d_queries, size_t nq, size_t k,
                                       uint32_t* d_out) {
    return guarded([&] {
        FDB_REQUIRE(ctx, FDB_ERR_INVALID_ARG, "NULL context");
        const size_t take = std::min(k, kc);
        const bool work = nq > 0 && take > 0;
        FDB_REQUIRE(nq <= FDB_NOALLOC_MAX_QUERIES, FDB_ERR_INVALID_ARG,
                    "nq above FDB_NOALLOC_MAX_QUERIES (262144); split the queries into batches");
        FDB_REQUIRE(kc <= FDB_NOALLOC_MAX_DISTANCES &&
                        (kc == 0 || nq <= FDB_NOALLOC_MAX_DISTANCES / kc),
                    FDB_ERR_INVALID_ARG,
                    "nq * kc above FDB_NOALLOC_MAX_DISTANCES (4194304 distances, the fixed "
                    "scratch); split the queries into batches");
        // more than 256 nearest ids are selected by a sort of each whole row in
        // shared memory (the row padded to a power of two), which holds at most
        // 16384 centroids
        FDB_REQUIRE(take <= 256 || kc <= FDB_NOALLOC_MAX_SORTED_CENTROIDS, FDB_ERR_INVALID_ARG,
                    "min(k, kc) above 256 needs kc <= FDB_NOALLOC_MAX_SORTED_CENTROIDS (16384)");
        FDB_REQUIRE(!work || (d_centroids && d_queries && d_out), FDB_ERR_INVALID_ARG,
                    "NULL argument");
        DeviceGuard g(ctx->c.device);
        float* D = noalloc_scratch(ctx->c.device);  // set-up, also on an empty call
        if (!work) return;
        std::lock_guard<std::mutex> lk(ctx->c.mu);
        cudaStream_t s = ctx->c.stream;
        launch_coarse_dist(s, d_queries, (int)nq, (int)dim, d_centroids, (int)kc, D);
        launch_select(s, D, (int)nq, (int)kc, (int)take, d_out);
        FDB_CUDA(cudaStreamSynchronize(s));
    });
}

// ---------------------------------------------------------------------------
// product quantizer
// ---------------------------------------------------------------------------
int fdb_pq_train(fdb_ctx* ctx, const float* x, size_t n, size_t dim, size_t m, size_t iters,
                 const uint32_t* init_idx, uint64_t seed, float* codebooks_out, int* iters_out) {
    return guarded([&] {
        FDB_REQUIRE(ctx && codebooks_out, FDB_ERR_INVALID_ARG, "NULL argument");
        FDB_REQUIRE(n > 0 && x, FDB_ERR_EMPTY_TRAINING_SET, "empty training set");
        FDB_REQUIRE(m > 0, FDB_ERR_INVALID_ARG, "m must be positive");
        FDB_REQUIRE(dim % m == 0, FDB_ERR_DIM_NOT_DIVISIBLE,
                    "dimension not divisible by the number of subvectors");
        FDB_REQUIRE(n >= (size_t)KSUB, FDB_ERR_INSUFFICIENT_VECTORS,
                    "PQ training needs at least 256 vectors");
        FDB_REQUIRE(n < (1ull << 32), FDB_ERR_UNSUPPORTED, "at most 2^32-1 vectors");
        DeviceGuard g(ctx->c.device);
        std::lock_guard<std::mutex> lk(ctx->c.mu);
        cudaStream_t s = ctx->c.stream;
        std::vector<uint32_t> idx(m * KSUB);
        if (init_idx) std::copy(init_idx, init_idx + idx.size(), idx.begin());
        else
            for (size_t q = 0; q < m; ++q) sample_indices(seed + q, n, KSUB, idx.data() + q * KSUB);
        DevBuf<float> X(n * dim), CB(m * KSUB * (dim / m));
        FDB_CUDA(cudaMemcpyAsync(X.p, x, X.bytes(), cudaMemcpyHostToDevice, s));
        std::vector<int> its(m);
        pq_train_dev(ctx->c, X.p, n, (int)dim, (int)m, iters ? (int)iters : 25, idx.data(), CB.p,
                     its.data());
        FDB_CUDA(cudaMemcpyAsync(codebooks_out, CB.p, CB.bytes(), cudaMemcpyDeviceToHost, s));
        FDB_CUDA(cudaStreamSynchronize(s));
        if (iters_out) std::copy(its.begin(), its.end(), iters_out);
    });
}

int fdb_pq_encode(fdb_ctx* ctx, const float* codebooks, size_t m, size_t dim, const float* x,
                  size_t n, uint8_t* codes_out) {
    return guarded([&] {
        FDB_REQUIRE(ctx && codebooks && (n == 0 || (x && codes_out)), FDB_ERR_INVALID_ARG,
                    "NULL argument");
        FDB_REQUIRE(m > 0 && dim % m == 0, FDB_ERR_DIM_NOT_DIVISIBLE,
                    "dimension not divisible by the number of subvectors");
        if (n == 0) return;
        DeviceGuard g(ctx->c.device);
        std::lock_guard<std::mutex> lk(ctx->c.mu);
        cudaStream_t s = ctx->c.stream;
        DevBuf<float> X(n * dim), CB(m * KSUB * (dim / m));
        DevBuf<uint8_t> codes(n * m);
        FDB_CUDA(cudaMemcpyAsync(X.p, x, X.bytes(), cudaMemcpyHostToDevice, s));
        FDB_CUDA(cudaMemcpyAsync(CB.p, codebooks, CB.bytes(), cudaMemcpyHostToDevice, s));
        launch_pq_encode(s, X.p, n, (int)dim, nullptr, nullptr, CB.p, (int)m, nullptr, codes.p);
        FDB_CUDA(cudaMemcpyAsync(codes_out, codes.p, n * m, cudaMemcpyDeviceToHost, s));
        FDB_CUDA(cudaStreamSynchronize(s));
    });
}

int fdb_pq_lookup_tables(fdb_ctx* ctx, const float* codebooks, size_t m, size_t dim,
                         const float* queries, size_t nq, float* lut_out) {
    return guarded([&] {
        FDB_REQUIRE(ctx && codebooks && (nq == 0 || (queries && lut_out)), FDB_ERR_INVALID_ARG,
                    "NULL argument");
        FDB_REQUIRE(m > 0 && dim % m == 0, FDB_ERR_DIM_MISMATCH,
                    "query dimension does not match the quantizer");
        if (nq == 0) return;
        DeviceGuard g(ctx->c.device);
        std::lock_guard<std::mutex> lk(ctx->c.mu);
        cudaStream_t s = ctx->c.stream;
        DevBuf<float> Q(nq * dim), CB(m * KSUB * (dim / m)), L(nq * m * KSUB);
        FDB_CUDA(cudaMemcpyAsync(Q.p, queries, Q.bytes(), cudaMemcpyHostToDevice, s));
        FDB_CUDA(cudaMemcpyAsync(CB.p, codebooks, CB.bytes(), cudaMemcpyHostToDevice, s));
        launch_lut(s, CB.p, (int)m, (int)dim, Q.p, nq, L.p);
        FDB_CUDA(cudaMemcpyAsync(lut_out, L.p, L.bytes(), cudaMemcpyDeviceToHost, s));
        FDB_CUDA(cudaStreamSynchronize(s));
    });
}

// ---------------------------------------------------------------------------
// IVF-PQ
// ---------------------------------------------------------------------------
int fdb_ivfpq_build(fdb_ctx* ctx, const float* x, const uint64_t* ids, size_t n, size_t dim,
                    size_t nlist, size_t m, int metric, const fdb_train_opts* opts,
                    fdb_ivfpq** out) {
    return guarded([&] {
        FDB_REQUIRE(ctx && out, FDB_ERR_INVALID_ARG, "NULL argument");
        check_metric(metric);
        FDB_REQUIRE(n > 0 && x, FDB_ERR_EMPTY_VECTOR_SET, "IVF-PQ build needs vectors");
        FDB_REQUIRE(dim > 0 && nlist > 0 && m > 0, FDB_ERR_INVALID_ARG,
                    "dim, nlist and m must be positive");
        FDB_REQUIRE(dim % m == 0, FDB_ERR_DIM_NOT_DIVISIBLE,
                    "dimension not divisible by the number of subvectors");
        DeviceGuard g(ctx->c.device);
        std::lock_guard<std::mutex> lk(ctx->c.mu);
        std::unique_ptr<fdb_ivfpq> h(new fdb_ivfpq());
        h->ctx = ctx;
        h->dim = dim;
        h->nlist = nlist;
        h->m = m;
        h->metric = metric;  // stored, unused by search, as in the reference (ivf_pq.rs:353)
        fdb_train_opts o{};
        if (opts) o = *opts;
        ivfpq_build(h.get(), x, ids, n, o);
        *out = h.release();
    });
}

int fdb_ivfpq_from_trained(fdb_ctx* ctx, const float* centroids, const float* codebooks,
                           size_t nlist, size_t m, size_t dim, const uint64_t* offsets,
                           const uint64_t* ids, const uint8_t* codes, int metric,
                           fdb_ivfpq** out) {
    return guarded([&] {
        FDB_REQUIRE(ctx && out && centroids && codebooks && offsets, FDB_ERR_INVALID_ARG,
                    "NULL argument");
        check_metric(metric);
        FDB_REQUIRE(dim > 0 && nlist > 0 && m > 0, FDB_ERR_INVALID_ARG,
                    "dim, nlist and m must be positive");
        FDB_REQUIRE(dim % m == 0, FDB_ERR_DIM_NOT_DIVISIBLE,
                    "dimension not divisible by the number of subvectors");
        FDB_REQUIRE(offsets[nlist] == 0 || (ids && codes), FDB_ERR_INVALID_ARG, "NULL lists");
        DeviceGuard g(ctx->c.device);
        std::lock_guard<std::mutex> lk(ctx->c.mu);
        std::unique_ptr<fdb_ivfpq> h(new fdb_ivfpq());
        h->ctx = ctx;
        h->dim = dim;
        h->nlist = nlist;
        h->m = m;
        h->metric = metric;
        ivfpq_load(h.get(), centroids, codebooks, offsets, ids, codes);
        *out = h.release();
    });
}

int fdb_ivfpq_export(fdb_ivfpq* h, float* centroids, float* codebooks, uint64_t* offsets,
                     uint64_t* ids, uint8_t* codes) {
    return guarded([&] {
        FDB_REQUIRE(h, FDB_ERR_INVALID_ARG, "NULL handle");
        DeviceGuard g(h->ctx->c.device);
        std::lock_guard<std::mutex> lk(h->mu);
        cudaStream_t s = h->ctx->c.stream;
        if (centroids)
            FDB_CUDA(cudaMemcpyAsync(centroids, h->cents.p, h->cents.bytes(),
                                     cudaMemcpyDeviceToHost, s));
        if (codebooks)
            FDB_CUDA(cudaMemcpyAsync(codebooks, h->cb.p, h->cb.bytes(), cudaMemcpyDeviceToHost, s));
        if (ids && h->n_total)
            FDB_CUDA(cudaMemcpyAsync(ids, h->ids.p, h->n_total * 8, cudaMemcpyDeviceToHost, s));
        if (codes && h->n_total)
            FDB_CUDA(cudaMemcpyAsync(codes, h->codes.p, h->n_total * h->m, cudaMemcpyDeviceToHost,
                                     s));
        FDB_CUDA(cudaStreamSynchronize(s));
        if (offsets) std::copy(h->h_offs_full.begin(), h->h_offs_full.end(), offsets);
    });
}

int fdb_ivfpq_shard(fdb_ivfpq* h, int rank, int world) {
    return guarded([&] {
        FDB_REQUIRE(h, FDB_ERR_INVALID_ARG, "NULL handle");
        DeviceGuard g(h->ctx->c.device);
        std::lock_guard<std::mutex> lk(h->mu);
        ivfpq_shard(h, rank, world);
    });
}

int fdb_ivfpq_set_nprobe(fdb_ivfpq* h, size_t nprobe) {
    return guarded([&] {
        FDB_REQUIRE(h, FDB_ERR_INVALID_ARG, "NULL handle");
        h->nprobe.store(std::min(nprobe, h->nlist), std::memory_order_relaxed);
    });
}

int fdb_ivfpq_set_scan_mode(fdb_ivfpq* h, int mode) {
    return guarded([&] {
        FDB_REQUIRE(h, FDB_ERR_INVALID_ARG, "NULL handle");
        FDB_REQUIRE(mode >= FDB_SCAN_AUTO && mode <= FDB_SCAN_TENSOR, FDB_ERR_INVALID_ARG,
                    "unknown scan mode");
        std::lock_guard<std::mutex> lk(h->mu);
        h->scan_mode = mode;
    });
}

int fdb_ivfpq_set_pass1_quota(fdb_ivfpq* h, size_t nprobe, uint64_t div) {
    return guarded([&] {
        FDB_REQUIRE(h, FDB_ERR_INVALID_ARG, "NULL handle");
        std::lock_guard<std::mutex> lk(h->mu);
        const size_t take = std::max<size_t>(1, std::min(nprobe, h->nlist));
        for (auto& e : h->tc_quota)
            if (e.first == take) {
                e.second = div;
                return;
            }
        h->tc_quota.emplace_back(take, div);
    });
}

int fdb_ivfpq_get_pass1_quota(fdb_ivfpq* h, size_t nprobe, int64_t* div) {
    return guarded([&] {
        FDB_REQUIRE(h && div, FDB_ERR_INVALID_ARG, "NULL argument");
        std::lock_guard<std::mutex> lk(h->mu);
        const size_t take = std::max<size_t>(1, std::min(nprobe, h->nlist));
        *div = -1;
        for (const auto& e : h->tc_quota)
            if (e.first == take) *div = (int64_t)e.second;
    });
}

int fdb_ivfpq_set_stage_timers(fdb_ivfpq* h, int enable) {
    return guarded([&] {
        FDB_REQUIRE(h, FDB_ERR_INVALID_ARG, "NULL handle");
        std::lock_guard<std::mutex> lk(h->mu);
        h->stage_timers = enable != 0;
    });
}

int fdb_ivfpq_set_graphs(fdb_ivfpq* h, int enable) {
    return guarded([&] {
        FDB_REQUIRE(h, FDB_ERR_INVALID_ARG, "NULL handle");
        std::lock_guard<std::mutex> lk(h->mu);
        h->graphs = enable != 0;
    });
}

size_t fdb_ivfpq_nprobe(const fdb_ivfpq* h) {
    return h ? h->nprobe.load(std::memory_order_relaxed) : 0;
}
size_t fdb_ivfpq_len(const fdb_ivfpq* h) { return h ? ivfpq_live_len(h) : 0; }
size_t fdb_ivfpq_n_partitions(const fdb_ivfpq* h) { return h ? h->nlist : 0; }
size_t fdb_ivfpq_dim(const fdb_ivfpq* h) { return h ? h->dim : 0; }
size_t fdb_ivfpq_n_subvectors(const fdb_ivfpq* h) { return h ? h->m : 0; }

static void ivfpq_host_search(fdb_ivfpq* h, const float* queries, size_t nq, size_t k, int order,
                              size_t take, uint64_t* ids, float* dists, uint32_t* counts,
                              fdb_stats* stats, const uint32_t* skip = nullptr,
                              size_t fetch_mult = 1) {
    cudaStream_t s = h->ctx->c.stream;
    const size_t per = nq * k;
    h->s_q.ensure(nq * h->dim);
    h->s_out_ids.ensure(per);
    h->s_dists.ensure(per);
    h->s_counts.ensure(nq);
    if (k == 0) {
        FDB_CUDA(cudaMemcpyAsync(h->s_q.p, queries, nq * h->dim * 4, cudaMemcpyHostToDevice, s));
        ivfpq_search_dev(h, h->s_q.p, nq, k, order, take, h->s_out_ids.p, h->s_dists.p,
                         h->s_counts.p, stats, skip, fetch_mult);
        if (counts) std::fill(counts, counts + nq, 0u);
        FDB_CUDA(cudaStreamSynchronize(s));
        return;
    }
    FDB_CUDA(cudaMemcpyAsync(h->s_q.p, queries, nq * h->dim * 4, cudaMemcpyHostToDevice, s));
    // the engine copies the results back before its one synchronisation
    HostIO io;
    io.ids = ids;
    io.dists = dists;
    io.counts = counts;
    try {
        ivfpq_search_dev(h, h->s_q.p, nq, k, order, take, h->s_out_ids.p, h->s_dists.p,
                         h->s_counts.p, stats, skip, fetch_mult, &io);
    } catch (...) {
        cudaStreamSynchronize(s);  // the caller's buffers may go once this returns
        throw;
    }
}

int fdb_ivfpq_search(fdb_ivfpq* h, const float* query, size_t k, uint64_t* ids, float* dists,
                     size_t* n_out) {
    return guarded([&] {
        FDB_REQUIRE(h && query && (k == 0 || (ids && dists)), FDB_ERR_INVALID_ARG,
                    "NULL argument");
        DeviceGuard g(h->ctx->c.device);
        std::lock_guard<std::mutex> lk(h->mu);
        // search(): nprobe.min(nlist) lists; nprobe == 0 probes none.
        size_t take = std::min(h->nprobe.load(std::memory_order_relaxed), h->nlist);
        uint32_t cnt = 0;
        ivfpq_host_search(h, query, 1, k, ORDER_FAST4, take, ids, dists, &cnt, nullptr);
        if (n_out) *n_out = cnt;
    });
}

int fdb_ivfpq_batch_search(fdb_ivfpq* h, const float* queries, size_t nq, size_t k,
                           uint64_t* ids, float* dists, uint32_t* counts, fdb_stats* stats) {
    return guarded([&] {
        FDB_REQUIRE(h && (nq == 0 || queries) && (nq == 0 || k == 0 || (ids && dists)),
                    FDB_ERR_INVALID_ARG, "NULL argument");
        if (nq == 0) { if (stats) std::memset(stats, 0, sizeof(*stats)); return; }
        DeviceGuard g(h->ctx->c.device);
        std::lock_guard<std::mutex> lk(h->mu);
        // batch_search(): nth = nprobe.min(nlist).saturating_sub(1), [..=nth].
        size_t take = std::max<size_t>(1, std::min(h->nprobe.load(std::memory_order_relaxed),
                                                   h->nlist));
        ivfpq_host_search(h, queries, nq, k, ORDER_LANE8, take, ids, dists, counts, stats);
    });
}

}  // extern "C"

namespace {

// Runs `search` under a deadline `timeout_s` from now (IVFPQIndex::
// search_with_timeout, ivf_pq.rs:1369-1455): the bounded waits inside the
// tensor-core kernels give up at the deadline, and a call whose results come
// back after it reports FDB_ERR_TIMEOUT, as the reference's checks between
// its stages do.  elapsed_out (nullable) gets the call's duration in seconds.
template <class F>
void with_deadline(fdb_ivfpq* h, double timeout_s, double* elapsed_out, F&& search) {
    FDB_REQUIRE(timeout_s >= 0.0, FDB_ERR_INVALID_ARG, "timeout must not be negative");
    const double t0 = now_s();
    struct Reset {
        fdb_ivfpq* h;
        ~Reset() { h->call_wait_cycles = 0; }
    } reset{h};
    h->call_wait_cycles = seconds_to_cycles(h->ctx->c, timeout_s);
    search();
    const double dt = now_s() - t0;
    if (elapsed_out) *elapsed_out = dt;
    FDB_REQUIRE(dt <= timeout_s, FDB_ERR_TIMEOUT, "search did not complete within the timeout");
}

}  // namespace

extern "C" {

int fdb_ivfpq_search_with_timeout(fdb_ivfpq* h, const float* query, size_t k, double timeout_s,
                                  uint64_t* ids, float* dists, size_t* n_out,
                                  double* elapsed_s) {
    return guarded([&] {
        FDB_REQUIRE(h && query && (k == 0 || (ids && dists)), FDB_ERR_INVALID_ARG,
                    "NULL argument");
        DeviceGuard g(h->ctx->c.device);
        std::lock_guard<std::mutex> lk(h->mu);
        size_t take = std::min(h->nprobe.load(std::memory_order_relaxed), h->nlist);
        uint32_t cnt = 0;
        with_deadline(h, timeout_s, elapsed_s, [&] {
            ivfpq_host_search(h, query, 1, k, ORDER_FAST4, take, ids, dists, &cnt, nullptr);
        });
        if (n_out) *n_out = cnt;
    });
}

int fdb_ivfpq_batch_search_with_timeout(fdb_ivfpq* h, const float* queries, size_t nq, size_t k,
                                        double timeout_s, uint64_t* ids, float* dists,
                                        uint32_t* counts, double* elapsed_s) {
    return guarded([&] {
        FDB_REQUIRE(h && (nq == 0 || queries) && (nq == 0 || k == 0 || (ids && dists)),
                    FDB_ERR_INVALID_ARG, "NULL argument");
        DeviceGuard g(h->ctx->c.device);
        std::lock_guard<std::mutex> lk(h->mu);
        size_t take = std::max<size_t>(1, std::min(h->nprobe.load(std::memory_order_relaxed),
                                                   h->nlist));
        with_deadline(h, timeout_s, elapsed_s, [&] {
            if (nq > 0)
                ivfpq_host_search(h, queries, nq, k, ORDER_LANE8, take, ids, dists, counts,
                                  nullptr);
        });
    });
}

int fdb_ivfpq_batch_search_device(fdb_ivfpq* h, const float* d_queries, size_t nq, size_t k,
                                  uint64_t* d_ids, float* d_dists, uint32_t* d_counts,
                                  fdb_stats* stats) {
    return guarded([&] {
        FDB_REQUIRE(h && (nq == 0 || d_queries) && (nq == 0 || k == 0 || (d_ids && d_dists)),
                    FDB_ERR_INVALID_ARG, "NULL argument");
        DeviceGuard g(h->ctx->c.device);
        std::lock_guard<std::mutex> lk(h->mu);
        size_t take = std::max<size_t>(1, std::min(h->nprobe.load(std::memory_order_relaxed),
                                                   h->nlist));
        ivfpq_search_dev(h, d_queries, nq, k, ORDER_LANE8, take, d_ids, d_dists, d_counts, stats);
        FDB_CUDA(cudaStreamSynchronize(h->ctx->c.stream));
    });
}

int fdb_ivfpq_free(fdb_ivfpq* h) {
    return guarded([&] {
        if (!h) return;
        DeviceGuard g(h->ctx->c.device);
        delete h;
    });
}

int fdb_ivfpq_shard_plan(const uint64_t* sizes, size_t nlist, int world, int* owner) {
    return guarded([&] {
        FDB_REQUIRE(world >= 1 && (nlist == 0 || (sizes && owner)), FDB_ERR_INVALID_ARG,
                    "bad arguments");
        shard_plan(sizes, nlist, world, owner);
    });
}

// ---------------------------------------------------------------------------
// brute force
// ---------------------------------------------------------------------------
int fdb_bf_create(fdb_ctx* ctx, int metric, const float* x, const uint64_t* ids, size_t n,
                  size_t dim, fdb_bf** out) {
    return guarded([&] {
        FDB_REQUIRE(ctx && out && (n == 0 || x), FDB_ERR_INVALID_ARG, "NULL argument");
        check_metric(metric);
        std::unique_ptr<fdb_bf> h(new fdb_bf());
        h->ctx = ctx;
        h->metric = metric;
        *out = h.release();
        if (n) {
            int rc = fdb_bf_add(*out, x, ids, n, dim);
            if (rc != FDB_OK) {
                std::string msg = g_last_error;
                delete *out;
                *out = nullptr;
                fail(rc, msg);
            }
        }
    });
}

int fdb_bf_add(fdb_bf* h, const float* x, const uint64_t* ids, size_t n, size_t dim) {
    return guarded([&] {
        FDB_REQUIRE(h && (n == 0 || x), FDB_ERR_INVALID_ARG, "NULL argument");
        if (n == 0) return;
        std::lock_guard<std::mutex> lk(h->mu);
        // add() adopts the first vector's dimension (brute_force.rs:75-80);
        // later rows must match it.
        if (h->dim == 0) h->dim = dim;
        FDB_REQUIRE(dim == h->dim, FDB_ERR_DIM_MISMATCH, "vector dimension mismatch");
        FDB_REQUIRE(h->h_ids.size() + n < (1ull << 32), FDB_ERR_UNSUPPORTED,
                    "at most 2^32-1 rows");
        size_t base = h->h_ids.size();
        h->h_x.insert(h->h_x.end(), x, x + n * dim);
        for (size_t i = 0; i < n; ++i) h->h_ids.push_back(ids ? ids[i] : (uint64_t)(base + i));
        h->row0 = 0;
        h->n = h->h_ids.size();
        h->sharded = false;
        h->shard_world = 1;
        h->dirty = true;
    });
}

int fdb_bf_shard(fdb_bf* h, int rank, int world) {
    return guarded([&] {
        FDB_REQUIRE(h, FDB_ERR_INVALID_ARG, "NULL handle");
        std::lock_guard<std::mutex> lk(h->mu);
        bf_shard(h, rank, world);
    });
}

int fdb_bf_set_scan_mode(fdb_bf* h, int mode) {
    return guarded([&] {
        FDB_REQUIRE(h, FDB_ERR_INVALID_ARG, "NULL handle");
        FDB_REQUIRE(mode >= FDB_SCAN_AUTO && mode <= FDB_SCAN_TABLES, FDB_ERR_INVALID_ARG,
                    "unknown scan mode");
        std::lock_guard<std::mutex> lk(h->mu);
        h->scan_mode = mode;
    });
}

size_t fdb_bf_len(const fdb_bf* h) { return h ? h->n : 0; }
size_t fdb_bf_dimension(const fdb_bf* h) { return (h && !h->h_ids.empty()) ? h->dim : 0; }

static void bf_host_search(fdb_bf* h, const float* queries, size_t nq, size_t k, uint64_t* ids,
                           float* dists, uint32_t* counts, fdb_stats* stats) {
    cudaStream_t s = h->ctx->c.stream;
    const size_t per = nq * k;
    h->s_q.ensure(nq * h->dim);
    h->s_out_ids.ensure(per);
    h->s_dists.ensure(per);
    h->s_counts.ensure(nq);
    FDB_CUDA(cudaMemcpyAsync(h->s_q.p, queries, nq * h->dim * 4, cudaMemcpyHostToDevice, s));
    bf_search_dev(h, h->s_q.p, nq, k, h->s_out_ids.p, h->s_dists.p, h->s_counts.p, stats);
    FDB_CUDA(cudaMemcpyAsync(ids, h->s_out_ids.p, per * 8, cudaMemcpyDeviceToHost, s));
    FDB_CUDA(cudaMemcpyAsync(dists, h->s_dists.p, per * 4, cudaMemcpyDeviceToHost, s));
    if (counts)
        FDB_CUDA(cudaMemcpyAsync(counts, h->s_counts.p, nq * 4, cudaMemcpyDeviceToHost, s));
    FDB_CUDA(cudaStreamSynchronize(s));
}

static void bf_check_k(fdb_bf* h, size_t k) {
    // With rows present, k == 0 makes the reference peek an empty heap and
    // panic (brute_force.rs:140-146).
    FDB_REQUIRE(k > 0 || h->h_ids.empty(), FDB_ERR_INVALID_ARG, "k must be positive");
}

int fdb_bf_search(fdb_bf* h, const float* query, size_t k, uint64_t* ids, float* dists,
                  size_t* n_out) {
    return guarded([&] {
        FDB_REQUIRE(h && query && (k == 0 || (ids && dists)), FDB_ERR_INVALID_ARG,
                    "NULL argument");
        bf_check_k(h, k);
        DeviceGuard g(h->ctx->c.device);
        std::lock_guard<std::mutex> lk(h->mu);
        uint32_t cnt = 0;
        if (k > 0) bf_host_search(h, query, 1, k, ids, dists, &cnt, nullptr);
        if (n_out) *n_out = cnt;
    });
}

int fdb_bf_batch_search(fdb_bf* h, const float* queries, size_t nq, size_t k, uint64_t* ids,
                        float* dists, uint32_t* counts, fdb_stats* stats) {
    return guarded([&] {
        FDB_REQUIRE(h && (nq == 0 || queries) && (nq == 0 || k == 0 || (ids && dists)),
                    FDB_ERR_INVALID_ARG, "NULL argument");
        if (stats) std::memset(stats, 0, sizeof(*stats));
        if (nq == 0) return;
        bf_check_k(h, k);
        DeviceGuard g(h->ctx->c.device);
        std::lock_guard<std::mutex> lk(h->mu);
        if (k == 0) { if (counts) std::fill(counts, counts + nq, 0u); return; }
        bf_host_search(h, queries, nq, k, ids, dists, counts, stats);
    });
}

int fdb_bf_batch_search_device(fdb_bf* h, const float* d_queries, size_t nq, size_t k,
                               uint64_t* d_ids, float* d_dists, uint32_t* d_counts,
                               fdb_stats* stats) {
    return guarded([&] {
        FDB_REQUIRE(h && (nq == 0 || d_queries) && (nq == 0 || k == 0 || (d_ids && d_dists)),
                    FDB_ERR_INVALID_ARG, "NULL argument");
        bf_check_k(h, k);
        DeviceGuard g(h->ctx->c.device);
        std::lock_guard<std::mutex> lk(h->mu);
        bf_search_dev(h, d_queries, nq, k, d_ids, d_dists, d_counts, stats);
        FDB_CUDA(cudaStreamSynchronize(h->ctx->c.stream));
    });
}

int fdb_bf_free(fdb_bf* h) {
    return guarded([&] {
        if (!h) return;
        DeviceGuard g(h->ctx->c.device);
        delete h;
    });
}

// ---------------------------------------------------------------------------
// IVF-PQ: re-ranking, filters, updates
// ---------------------------------------------------------------------------
int fdb_ivfpq_enable_reranking(fdb_ivfpq* h, const float* x, const uint64_t* ids, size_t n,
                               size_t dim, size_t rerank_factor) {
    return guarded([&] {
        FDB_REQUIRE(h && (n == 0 || (x && ids)), FDB_ERR_INVALID_ARG, "NULL argument");
        FDB_REQUIRE(n == 0 || dim == h->dim, FDB_ERR_DIM_MISMATCH, "vector dimension mismatch");
        DeviceGuard g(h->ctx->c.device);
        std::lock_guard<std::mutex> lk(h->mu);
        ivfpq_enable_reranking(h, x, ids, n, rerank_factor);
    });
}

static void filtered_search(fdb_ivfpq* h, const float* queries, size_t nq, size_t k,
                            const uint64_t* allowed, size_t na, uint64_t* ids, float* dists,
                            uint32_t* counts) {
    // search_filtered: no matching id -> no results (ivf_pq.rs:701-704)
    if (na == 0 || k == 0) {
        for (size_t i = 0; i < nq * k; ++i) {
            ids[i] = ~0ull;
            dists[i] = INFINITY;
        }
        if (counts) std::fill(counts, counts + nq, 0u);
        return;
    }
    // nprobe.min(nlist) lists (:717-723), single-query ADC order
    const size_t take = std::min(h->nprobe.load(std::memory_order_relaxed), h->nlist);
    ivfpq_sync_state(h);
    const uint32_t* skip = ivfpq_filter_bitmap(h, allowed, na);
    ivfpq_host_search(h, queries, nq, k, ORDER_FAST4, take, ids, dists, counts, nullptr, skip,
                      4);
}

int fdb_ivfpq_search_filtered(fdb_ivfpq* h, const float* query, size_t k,
                              const uint64_t* allowed_ids, size_t n_allowed, uint64_t* ids,
                              float* dists, size_t* n_out) {
    return guarded([&] {
        FDB_REQUIRE(h && query && (k == 0 || (ids && dists)) && (n_allowed == 0 || allowed_ids),
                    FDB_ERR_INVALID_ARG, "NULL argument");
        DeviceGuard g(h->ctx->c.device);
        std::lock_guard<std::mutex> lk(h->mu);
        uint32_t cnt = 0;
        filtered_search(h, query, 1, k, allowed_ids, n_allowed, ids, dists, &cnt);
        if (n_out) *n_out = cnt;
    });
}

int fdb_ivfpq_batch_search_filtered(fdb_ivfpq* h, const float* queries, size_t nq, size_t k,
                                    const uint64_t* allowed_ids, size_t n_allowed,
                                    uint64_t* ids, float* dists, uint32_t* counts) {
    return guarded([&] {
        FDB_REQUIRE(h && (nq == 0 || queries) && (nq == 0 || k == 0 || (ids && dists)) &&
                        (n_allowed == 0 || allowed_ids),
                    FDB_ERR_INVALID_ARG, "NULL argument");
        if (nq == 0) return;
        DeviceGuard g(h->ctx->c.device);
        std::lock_guard<std::mutex> lk(h->mu);
        filtered_search(h, queries, nq, k, allowed_ids, n_allowed, ids, dists, counts);
    });
}

int fdb_ivfpq_batch_search_filtered_device(fdb_ivfpq* h, const float* d_queries, size_t nq,
                                           size_t k, const uint64_t* d_allowed_ids,
                                           size_t n_allowed, uint64_t* d_ids, float* d_dists,
                                           uint32_t* d_counts, fdb_stats* stats) {
    return guarded([&] {
        if (stats) std::memset(stats, 0, sizeof(*stats));
        FDB_REQUIRE(h && (nq == 0 || d_queries) && (nq == 0 || k == 0 || (d_ids && d_dists)) &&
                        (n_allowed == 0 || d_allowed_ids),
                    FDB_ERR_INVALID_ARG, "NULL argument");
        if (nq == 0 || k == 0) return;
        DeviceGuard g(h->ctx->c.device);
        std::lock_guard<std::mutex> lk(h->mu);
        cudaStream_t s = h->ctx->c.stream;
        if (n_allowed == 0) {  // no results: padding only
            const std::vector<float> inf(nq * k, INFINITY);
            FDB_CUDA(cudaMemsetAsync(d_ids, 0xff, nq * k * 8, s));
            FDB_CUDA(cudaMemcpyAsync(d_dists, inf.data(), nq * k * 4, cudaMemcpyHostToDevice, s));
            if (d_counts) FDB_CUDA(cudaMemsetAsync(d_counts, 0, nq * 4, s));
            FDB_CUDA(cudaStreamSynchronize(s));
        } else {
            const size_t take = std::min(h->nprobe.load(std::memory_order_relaxed), h->nlist);
            ivfpq_sync_state(h);
            const uint32_t* skip = ivfpq_filter_bitmap(h, d_allowed_ids, n_allowed, true);
            ivfpq_search_dev(h, d_queries, nq, k, ORDER_FAST4, take, d_ids, d_dists, d_counts,
                             stats, skip, 4);
        }
        FDB_CUDA(cudaStreamSynchronize(s));
    });
}

int fdb_ivfpq_insert_batch(fdb_ivfpq* h, const float* x, const uint64_t* ids, size_t n,
                           size_t dim) {
    return guarded([&] {
        FDB_REQUIRE(h && (n == 0 || (x && ids)), FDB_ERR_INVALID_ARG, "NULL argument");
        if (n == 0) return;  // insert_batch of nothing is a no-op (:1732-1734)
        FDB_REQUIRE(dim == h->dim, FDB_ERR_DIM_MISMATCH, "vector dimension mismatch");
        DeviceGuard g(h->ctx->c.device);
        std::lock_guard<std::mutex> lkc(h->ctx->c.mu);
        std::lock_guard<std::mutex> lk(h->mu);
        ivfpq_insert_batch(h, x, ids, n);
    });
}

int fdb_ivfpq_delete(fdb_ivfpq* h, uint64_t id, int* deleted) {
    return guarded([&] {
        FDB_REQUIRE(h, FDB_ERR_INVALID_ARG, "NULL handle");
        std::lock_guard<std::mutex> lk(h->mu);
        const bool d = ivfpq_delete(h, id);
        if (deleted) *deleted = d ? 1 : 0;
    });
}

size_t fdb_ivfpq_num_tombstones(const fdb_ivfpq* h) { return h ? h->n_tomb : 0; }
size_t fdb_ivfpq_len_with_tombstones(const fdb_ivfpq* h) { return h ? h->n_local : 0; }
float fdb_ivfpq_fragmentation_ratio(const fdb_ivfpq* h) {
    // tombstones / len(), 0 for an empty index (ivf_pq.rs:1815-1822)
    if (!h) return 0.0f;
    const size_t total = ivfpq_live_len(h);
    return total == 0 ? 0.0f : (float)h->n_tomb / (float)total;
}

int fdb_ivfpq_compact(fdb_ivfpq* h) {
    return guarded([&] {
        FDB_REQUIRE(h, FDB_ERR_INVALID_ARG, "NULL handle");
        DeviceGuard g(h->ctx->c.device);
        std::lock_guard<std::mutex> lkc(h->ctx->c.mu);
        std::lock_guard<std::mutex> lk(h->mu);
        ivfpq_compact(h);
    });
}

int fdb_ivfpq_rebuild(fdb_ivfpq* h, const fdb_train_opts* opts) {
    return guarded([&] {
        FDB_REQUIRE(h, FDB_ERR_INVALID_ARG, "NULL handle");
        FDB_REQUIRE(h->rerank, FDB_ERR_UNSUPPORTED,
                    "operation not supported: rebuild requires original vectors (enable "
                    "re-ranking)");
        FDB_REQUIRE(!h->rr_ids.empty(), FDB_ERR_EMPTY_VECTOR_SET,
                    "empty vector set: operation requires at least one vector");
        DeviceGuard g(h->ctx->c.device);
        std::lock_guard<std::mutex> lkc(h->ctx->c.mu);
        std::lock_guard<std::mutex> lk(h->mu);
        const std::vector<float> x = h->rr_x;
        const std::vector<uint64_t> ids = h->rr_ids;
        const size_t nprobe = h->nprobe.load(std::memory_order_relaxed);
        const size_t factor = h->rerank_factor;
        // IVFPQIndex::build(vectors, n_clusters, n_subvectors, metric) replaces
        // the whole index; the result is unsharded
        h->tomb.clear();
        h->n_tomb = 0;
        h->h_dead.clear();
        h->dead.release();
        h->dead_dirty = false;
        h->id_index.clear();
        h->id_index_ok = false;
        h->d_idx_ok = false;
        h->sharded = false;
        h->shard_world = 1;
        h->shard_rank = 0;
        h->owned.clear();
        h->shard_be.release();
        fdb_train_opts o{};
        if (opts) o = *opts;
        ivfpq_build(h, x.data(), ids.data(), ids.size(), o);
        h->nprobe.store(std::min(nprobe, h->nlist), std::memory_order_relaxed);
        ivfpq_enable_reranking(h, x.data(), ids.data(), ids.size(), factor);
    });
}

int fdb_bf_remove(fdb_bf* h, uint64_t id, int* removed) {
    return guarded([&] {
        FDB_REQUIRE(h, FDB_ERR_INVALID_ARG, "NULL handle");
        std::lock_guard<std::mutex> lk(h->mu);
        // VectorStore::find_id + swap_remove (vector.rs:256-276)
        auto it = std::find(h->h_ids.begin(), h->h_ids.end(), id);
        if (removed) *removed = it != h->h_ids.end() ? 1 : 0;
        if (it == h->h_ids.end()) return;
        const size_t i = (size_t)(it - h->h_ids.begin()), last = h->h_ids.size() - 1;
        h->h_ids[i] = h->h_ids[last];
        h->h_ids.pop_back();
        if (i != last)
            std::copy(h->h_x.begin() + last * h->dim, h->h_x.begin() + (last + 1) * h->dim,
                      h->h_x.begin() + i * h->dim);
        h->h_x.resize(last * h->dim);
        h->row0 = 0;
        h->n = h->h_ids.size();
        h->sharded = false;
        h->shard_world = 1;
        h->dirty = true;
    });
}

// ---------------------------------------------------------------------------
// IVFPQIndexBuilder (src/index/ivf_pq_builder.rs)
// ---------------------------------------------------------------------------
void fdb_builder_defaults(fdb_builder_opts* o) {
    if (!o) return;
    std::memset(o, 0, sizeof(*o));
    o->metric = FDB_METRIC_EUCLIDEAN;
    o->auto_tune = 1;
    o->target_recall = -1.0f;
    o->nprobe = 1;
    o->rerank_factor = 1;
}

static void builder_plan(const fdb_builder_opts& o, size_t n, size_t dim, size_t* clusters_out,
                         size_t* m_out, size_t* nprobe_out, size_t* mb_out) {
    // auto_tune_clusters: explicit, else round(sqrt(n)), clamped to
    // [min(256, n), min(65536, n)] when auto-tuning
    size_t clusters = o.num_clusters;
    if (clusters == 0) {
        const size_t sq = (size_t)std::round(std::sqrt((double)n));
        clusters = o.auto_tune ? std::min(std::max(sq, std::min<size_t>(256, n)),
                                          std::min<size_t>(65536, n))
                               : sq;
    }
    // auto_tune_subvectors: explicit, else dim / 4 (must divide), or with
    // auto-tuning the largest divisor of dim not above dim / 4 (1 at least)
    size_t m = o.num_subvectors;
    if (m == 0) {
        const size_t target = dim / 4;
        if (!o.auto_tune) {
            FDB_REQUIRE(target > 0 && dim % target == 0, FDB_ERR_INVALID_ARG,
                        "invalid parameter: default num_subvectors " + std::to_string(target) +
                            " does not divide dimension " + std::to_string(dim));
            m = target;
        } else {
            m = 1;
            for (size_t c = target; c >= 1; --c)
                if (dim % c == 0) { m = c; break; }
        }
    }
    // auto_tune_nprobe: an explicit nprobe > 1 (at most the clusters), else a
    // fraction of the clusters by target recall (f32 arithmetic), else 1
    size_t nprobe = 1;
    if (o.nprobe > 1) {
        nprobe = std::min(o.nprobe, clusters);
    } else if (o.target_recall >= 0.0f) {
        const float r = std::min(std::max(o.target_recall, 0.0f), 1.0f);
        const float c = (float)clusters;
        size_t p = 1;
        if (r >= 0.95f) p = (size_t)std::ceil(c * 0.1f);
        else if (r >= 0.9f) p = (size_t)std::ceil(c * 0.05f);
        else if (r >= 0.8f) p = (size_t)std::ceil(c * 0.02f);
        nprobe = std::min(std::max<size_t>(p, 1), std::max<size_t>(clusters, 1));
    }
    FDB_REQUIRE(clusters <= n, FDB_ERR_INSUFFICIENT_VECTORS,
                "insufficient vectors: required " + std::to_string(clusters) + ", got " +
                    std::to_string(n));
    FDB_REQUIRE(m > 0 && dim % m == 0, FDB_ERR_INVALID_ARG,
                "invalid parameter: vector dimension " + std::to_string(dim) +
                    " must be divisible by num_subvectors " + std::to_string(m));
    // estimate_memory_mb: codes + ids + centroids + codebooks, whole MiB
    const size_t bytes = n * m + n * 8 + clusters * dim * 4 + m * 256 * (dim / m) * 4;
    *clusters_out = clusters;
    *m_out = m;
    *nprobe_out = nprobe;
    if (mb_out) *mb_out = bytes / (1024 * 1024);
}

int fdb_builder_plan(const fdb_builder_opts* o, size_t n, size_t dim, size_t* num_clusters,
                     size_t* num_subvectors, size_t* nprobe, size_t* estimated_mb) {
    return guarded([&] {
        FDB_REQUIRE(o && num_clusters && num_subvectors && nprobe, FDB_ERR_INVALID_ARG,
                    "NULL argument");
        FDB_REQUIRE(n > 0, FDB_ERR_EMPTY_VECTOR_SET,
                    "empty vector set: operation requires at least one vector");
        builder_plan(*o, n, dim, num_clusters, num_subvectors, nprobe, estimated_mb);
    });
}

int fdb_builder_build(fdb_ctx* ctx, const fdb_builder_opts* o, const float* x,
                      const uint64_t* ids, size_t n, size_t dim, const fdb_train_opts* train,
                      fdb_ivfpq** out) {
    return guarded([&] {
        FDB_REQUIRE(o && out, FDB_ERR_INVALID_ARG, "NULL argument");
        FDB_REQUIRE(x, FDB_ERR_INVALID_ARG, "invalid parameter: vectors are required");
        FDB_REQUIRE(n > 0, FDB_ERR_EMPTY_VECTOR_SET,
                    "empty vector set: operation requires at least one vector");
        FDB_REQUIRE(ctx, FDB_ERR_INVALID_ARG, "NULL context");
        size_t clusters = 0, m = 0, nprobe = 1, mb = 0;
        builder_plan(*o, n, dim, &clusters, &m, &nprobe, &mb);
        if (o->target_memory_mb && mb > o->target_memory_mb)
            std::fprintf(stderr, "Warning: estimated memory %zuMB exceeds target %zuMB\n", mb,
                         o->target_memory_mb);
        fdb_ivfpq* h = nullptr;
        int rc = fdb_ivfpq_build(ctx, x, ids, n, dim, clusters, m, o->metric, train, &h);
        if (rc != FDB_OK) fail(rc, g_last_error);
        std::unique_ptr<fdb_ivfpq> hold(h);
        hold->nprobe.store(std::min(nprobe, hold->nlist), std::memory_order_relaxed);
        if (o->enable_reranking) {
            std::vector<uint64_t> iv(n);
            for (size_t i = 0; i < n; ++i) iv[i] = ids ? ids[i] : (uint64_t)i;
            DeviceGuard g(ctx->c.device);
            ivfpq_enable_reranking(hold.get(), x, iv.data(), n, o->rerank_factor);
        }
        *out = hold.release();
    });
}

// ---------------------------------------------------------------------------
// .fdb files
// ---------------------------------------------------------------------------
int fdb_ivfpq_save(fdb_ivfpq* h, const char* path) {
    return guarded([&] {
        FDB_REQUIRE(h && path, FDB_ERR_INVALID_ARG, "NULL argument");
        DeviceGuard g(h->ctx->c.device);
        std::lock_guard<std::mutex> lk(h->mu);
        ivfpq_save(h, path);
    });
}

int fdb_ivfpq_load(fdb_ctx* ctx, const char* path, fdb_ivfpq** out) {
    return guarded([&] {
        FDB_REQUIRE(ctx && path && out, FDB_ERR_INVALID_ARG, "NULL argument");
        DeviceGuard g(ctx->c.device);
        std::lock_guard<std::mutex> lk(ctx->c.mu);
        std::unique_ptr<fdb_ivfpq> h(new fdb_ivfpq());
        h->ctx = ctx;
        ivfpq_load_file(h.get(), path);
        *out = h.release();
    });
}

int fdb_bf_save(fdb_bf* h, const char* path) {
    return guarded([&] {
        FDB_REQUIRE(h && path, FDB_ERR_INVALID_ARG, "NULL argument");
        std::lock_guard<std::mutex> lk(h->mu);
        bf_save(h, path);
    });
}

int fdb_bf_load(fdb_ctx* ctx, const char* path, fdb_bf** out) {
    return guarded([&] {
        FDB_REQUIRE(ctx && path && out, FDB_ERR_INVALID_ARG, "NULL argument");
        std::unique_ptr<fdb_bf> h(new fdb_bf());
        h->ctx = ctx;
        bf_load_file(h.get(), path);
        *out = h.release();
    });
}

int fdb_file_inspect(const char* path, fdb_file_info* info) {
    return guarded([&] {
        FDB_REQUIRE(path && info, FDB_ERR_INVALID_ARG, "NULL argument");
        file_inspect(path, info);
    });
}

uint32_t fdb_crc32(const void* data, size_t n) {
    return crc32(static_cast<const uint8_t*>(data), n);
}

}  // extern "C"
