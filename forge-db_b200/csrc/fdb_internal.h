// fdb_internal.h -- host-side internals shared by the engine's translation
// units: error propagation, device buffers, the per-device context and the
// index handles behind the opaque C types of include/forgegpu.h.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <array>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "forgegpu.h"

namespace fdb {

// ---------------------------------------------------------------------------
// errors: thrown inside the engine, turned into a status code at the C ABI
// ---------------------------------------------------------------------------
struct Error {
    int code;
    std::string msg;
};

[[noreturn]] void fail(int code, const std::string& msg);
void set_last_error(const std::string& msg);

#define FDB_CUDA(x)                                                                           \
    do {                                                                                      \
        cudaError_t e__ = (x);                                                                \
        if (e__ != cudaSuccess)                                                               \
            ::fdb::fail(e__ == cudaErrorMemoryAllocation ? FDB_ERR_OOM : FDB_ERR_CUDA,         \
                        std::string(#x) + ": " + cudaGetErrorString(e__));                    \
    } while (0)

#define FDB_LAUNCH_CHECK() FDB_CUDA(cudaGetLastError())

#define FDB_NCCL(x)                                                                           \
    do {                                                                                      \
        ncclResult_t r__ = (x);                                                               \
        if (r__ != ncclSuccess)                                                               \
            ::fdb::fail(FDB_ERR_NCCL, std::string(#x) + ": " + ncclGetErrorString(r__));      \
    } while (0)

// An NCCL call on the context's communicator, which is non-blocking (so that
// initialisation can have a deadline): a call that returns ncclInProgress is
// complete once the communicator's asynchronous state leaves that value.
void nccl_complete(ncclResult_t r, ncclComm_t comm, const char* what);
#define FDB_NCCL_C(x, comm) ::fdb::nccl_complete((x), (comm), #x)

#define FDB_REQUIRE(cond, code, msg)          \
    do {                                              \
        if (!(cond)) ::fdb::fail((code), (msg));      \
    } while (0)

// ---------------------------------------------------------------------------
// device memory
// ---------------------------------------------------------------------------
// Counts every device allocation and release made through DevBuf: a captured
// CUDA graph bakes in buffer addresses, and stays valid while this is unchanged.
inline std::atomic<uint64_t>& devbuf_epoch() {
    static std::atomic<uint64_t> e{0};
    return e;
}

template <typename T>
struct DevBuf {
    T* p = nullptr;
    size_t n = 0;
    DevBuf() = default;
    explicit DevBuf(size_t count) { alloc(count); }
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    DevBuf(DevBuf&& o) noexcept : p(o.p), n(o.n) { o.p = nullptr; o.n = 0; }
    DevBuf& operator=(DevBuf&& o) noexcept {
        if (this != &o) { release(); p = o.p; n = o.n; o.p = nullptr; o.n = 0; }
        return *this;
    }
    ~DevBuf() { release(); }
    void alloc(size_t count) {
        release();
        if (count) {
            FDB_CUDA(cudaMalloc(&p, count * sizeof(T)));
            devbuf_epoch().fetch_add(1);
        }
        n = count;
    }
    // Grow-only: keep the allocation if it is already large enough.
    void ensure(size_t count) {
        if (count > n) alloc(count);
    }
    void release() {
        if (p) {
            cudaFree(p);
            devbuf_epoch().fetch_add(1);
        }
        p = nullptr;
        n = 0;
    }
    size_t bytes() const { return n * sizeof(T); }
};

// ---------------------------------------------------------------------------
// context: one device, one stream, optional communicator
// ---------------------------------------------------------------------------
struct StageTimer;
struct Ctx {
    int device = 0;
    int sm_count = 0;
    int clock_khz = 1965000;  // SM clock (cycles per ms): converts wait limits
    cudaStream_t stream = nullptr;
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
    std::mutex mu;  // serialises use of the context's scratch buffers
    // Limit of every bounded wait inside the tensor-core kernels, in SM clock
    // cycles and in seconds (fdb_ctx_set_wait_limit); a call with its own
    // deadline lowers it for its duration.
    std::atomic<unsigned long long> wait_cycles{4000000000ull};
    std::atomic<double> wait_s{2.0};
    std::atomic<int> test_stalls{0};  // test hook: list-scan launches left to stall
    // A timed call on a sharded index: event marks before and after each
    // collective (comm_ids: which one, FDB_COMM_*), read into fdb_stats.comm_ms.
    StageTimer* comm_tm = nullptr;
    std::vector<int> comm_ids;
};
// the collectives of a sharded search, in fdb_stats.comm_ms order
constexpr int COMM_PROBES = 0, COMM_TAU = 1, COMM_DK = 2, COMM_RESULTS = 3;

// The wait limit in force for a call (call_cycles: the call's own limit, 0 =
// none), in SM clock cycles.
inline unsigned long long wait_limit_cycles(const Ctx& c, unsigned long long call_cycles = 0) {
    const unsigned long long w = c.wait_cycles.load(std::memory_order_relaxed);
    return call_cycles ? std::min(call_cycles, w) : w;
}
inline unsigned long long seconds_to_cycles(const Ctx& c, double s) {
    const double cyc = s * (double)c.clock_khz * 1000.0;
    return cyc < 1.0 ? 1ull : (cyc > 1.8e19 ? 18000000000000000000ull : (unsigned long long)cyc);
}
// Test hook: true (once per requested stall) if this list-scan launch is to
// issue no work, so that its bounded waits run out.
inline bool take_test_stall(Ctx& c) {
    int n = c.test_stalls.load();
    while (n > 0)
        if (c.test_stalls.compare_exchange_weak(n, n - 1)) return true;
    return false;
}

// Makes the context's device current for the lifetime of the guard.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) FDB_CUDA(cudaSetDevice(dev));
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

// A few words of pinned host memory for small device-to-host readbacks: an
// asynchronous copy into pageable memory waits for the stream and costs a
// round trip each, into pinned memory it is queued like a kernel.
struct PinnedWords {
    uint64_t* p = nullptr;
    PinnedWords() = default;
    PinnedWords(const PinnedWords&) = delete;
    PinnedWords& operator=(const PinnedWords&) = delete;
    ~PinnedWords() {
        if (p) cudaFreeHost(p);
    }
    uint64_t* get() {  // 8 words
        if (!p) FDB_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&p), 64, cudaHostAllocPortable));
        return p;
    }
};

// Host result buffers of one search (ivfpq_search_dev): the results are
// copied to them before the call's one synchronisation.
struct HostIO {
    uint64_t* ids = nullptr;      // host [nq][k] (nullable: no copies)
    float* dists = nullptr;
    uint32_t* counts = nullptr;   // nullable
};

// Times device stages on a stream with CUDA events.  Inside a stream
// capture it records into events of a pool that outlives the call (external
// records: graph nodes that record the event at each replay).
struct StageTimer {
    cudaStream_t s;
    bool on;
    std::vector<cudaEvent_t> ev;
    std::vector<cudaEvent_t>* pool = nullptr;  // owner of the events (capture, replay)
    size_t next = 0;                           // next pool event
    bool owned = true;
    StageTimer(cudaStream_t s_, bool on_) : s(s_), on(on_) {}
    ~StageTimer() { reset(); }
    void reset() {
        if (owned)
            for (auto e : ev) cudaEventDestroy(e);
        ev.clear();
        pool = nullptr;
        owned = true;
    }
    void use_pool(std::vector<cudaEvent_t>* p, size_t first) {
        reset();
        pool = p;
        next = first;
        owned = false;
    }
    // the events a replayed graph records (owned by the graph's pool)
    void borrow(const std::vector<cudaEvent_t>& e) {
        reset();
        ev = e;
        owned = false;
    }
    void mark() {
        if (!on) return;
        cudaEvent_t e;
        if (pool) {
            FDB_REQUIRE(next < pool->size(), FDB_ERR_UNSUPPORTED, "stage timer pool exhausted");
            e = (*pool)[next++];
            FDB_CUDA(cudaEventRecordWithFlags(e, s, cudaEventRecordExternal));
        } else {
            FDB_CUDA(cudaEventCreate(&e));
            FDB_CUDA(cudaEventRecord(e, s));
        }
        ev.push_back(e);
    }
    // Milliseconds between marks a and b (after the stream is synced).
    double ms(size_t a, size_t b) const {
        if (!on || b >= ev.size()) return 0.0;
        float t = 0.f;
        cudaEventElapsedTime(&t, ev[a], ev[b]);
        return t;
    }
};

// A mark before (and, called again, after) collective `id` of a timed call.
inline void comm_mark(Ctx& c, int id) {
    if (!c.comm_tm) return;
    c.comm_tm->mark();
    c.comm_ids.push_back(id);
}

// Times the collectives of one call on a sharded index (timer on) and
// detaches the timer from the context when the call ends.
struct CommTimerScope {
    Ctx& c;
    StageTimer& tm;
    CommTimerScope(Ctx& c_, StageTimer& tm_) : c(c_), tm(tm_) {
        c.comm_ids.clear();
        c.comm_tm = tm.on ? &tm : nullptr;
    }
    ~CommTimerScope() { c.comm_tm = nullptr; }
    // after the stream is synchronised
    void read(fdb_stats* st) const {
        if (!c.comm_tm) return;
        for (size_t i = 0; i + 1 < c.comm_ids.size(); i += 2)
            st->comm_ms[c.comm_ids[i]] += tm.ms(i, i + 1);
    }
};

// ---------------------------------------------------------------------------
// seeded draws (host): deterministic across processes and devices
// ---------------------------------------------------------------------------
uint64_t splitmix64(uint64_t& state);
void sample_indices(uint64_t seed, size_t n, size_t take, uint32_t* out);
void uniform_draws(uint64_t seed, size_t count, float* out);

// ---------------------------------------------------------------------------
// kernel launchers implemented in the .cu files
// ---------------------------------------------------------------------------
// distances.cu
void launch_pairwise(cudaStream_t s, int metric, const float* a, const float* b, size_t n,
                     int dim, float* out);
void launch_gather_rows(cudaStream_t s, const float* x, size_t dim, const uint32_t* idx,
                        size_t count, float* out);

// kmeans.cu: k-means over a strided view of `n` rows; `nsub` independent
// problems (PQ subspaces) share one launch, problem s reading columns
// [s*dim, (s+1)*dim) of rows with stride `ld`.
struct KMeansProblem {
    const float* x;  // device rows
    size_t n;
    int dim;         // columns per problem
    int ld;          // row stride in floats
    int nsub;        // independent problems (1 for plain k-means)
    int k;
    int max_iters;
};
// cent: device [nsub][k][dim] initial centroids, updated in place.
// iters_out: host [nsub].  ever_out (host [nsub][k], nullable): 1 where the
// cluster had points in some iteration, i.e. where the reference's centroid
// was rebuilt as Vector::new(k, mean) and so carries id k (kmeans.rs:183).
void kmeans_run(Ctx& ctx, const KMeansProblem& pb, float* cent, int* iters_out,
                uint8_t* ever_out = nullptr);
// k-means++ initialisation of one problem (nsub == 1, k <= 64); picks_out
// (host [k], nullable) receives the row chosen for each centroid.
void kmeans_pp_init(Ctx& ctx, const float* x, size_t n, int dim, int k,
                    const uint32_t* init_idx_host, const float* kpp_u_host, float* cent,
                    uint32_t* picks_out = nullptr);
void launch_assign(cudaStream_t s, const float* x, size_t n, int dim, int ld, const float* cent,
                   int k, uint32_t* out);
// Stable grouping of points by assignment: perm (point ids in group order)
// and offsets[k+1].  Scratch comes from the caller's buffers.
void group_by_assignment(Ctx& ctx, const uint32_t* assign, size_t n, int k, uint32_t* perm,
                         uint64_t* offsets);

// pq.cu
void launch_pq_encode(cudaStream_t s, const float* x, size_t n, int dim, const float* cents,
                      const uint32_t* assign, const float* cb, int m, const uint32_t* slot,
                      uint8_t* codes);
void launch_lut(cudaStream_t s, const float* cb, int m, int dim, const float* q, size_t nq,
                float* lut);
void pq_train_dev(Ctx& ctx, const float* x, size_t n, int dim, int m, int iters,
                  const uint32_t* init_idx_host, float* cb, int* iters_out,
                  uint8_t* ever_out = nullptr);

// engine.cu
// init_rows (host [k], nullable): the point each initial centroid was
// copied from; ever (host [k], nullable): see kmeans_run.
void kmeans_fit_dev(Ctx& ctx, const float* x, size_t n, int dim, int k, int max_iters,
                    const uint32_t* init_idx, const float* kpp_u, uint64_t seed, float* cent,
                    int* iters_run, uint32_t* init_rows = nullptr, uint8_t* ever = nullptr);
void shard_plan(const uint64_t* sizes, size_t nlist, int world, int* owner);

// gemm_topk.cu: the tensor-core shortlist of brute force (sample pass,
// threshold, filter pass, top-kp selection) and its exact rescoring.
struct GemmScratch {
    DevBuf<uint64_t> part, top32, cand, approx;
    DevBuf<unsigned> tau_bits, cand_cnt, seg_cnt;
    DevBuf<float> tau;
    int cap = 0;
    int* err = nullptr;  // device error word (timeouts)
    unsigned long long wait_cycles = 4000000000ull;  // limit of each bounded wait
    // optional: recorded around the filter pass (the dominant kernel)
    cudaEvent_t filter_ev0 = nullptr, filter_ev1 = nullptr;
};
void gemm_shortlist(cudaStream_t s, const __half* q16, int nq, const float* qnorm,
                    const __half* x16, size_t n, int kpad, const float* xnorm, int metric,
                    uint64_t tag_base, int kp, int sm_count, float colmax, GemmScratch& w);
// xnorm: [rows] squared norms of X in the AVX2 order (dot_exact(x, x)).
void launch_bf_rescore(cudaStream_t s, const float* Q, int nq, const float* X, int dim,
                       const float* qnorm, const float* xnorm, float xmax, int metric,
                       uint64_t tag_base, const GemmScratch& w, int kp, int k, uint64_t* out,
                       uint32_t* flag_count, uint32_t* flag_list);

}  // namespace fdb

// A captured search (see ivfpq_search_dev): the key of the call it replays,
// the allocation epoch its buffer addresses belong to, and its timing events.
namespace fdb {
using GraphKey = std::array<uint64_t, 19>;
struct GraphSlot {
    GraphKey key{};
    uint64_t epoch = 0;
    uint64_t used = 0;  // last use (LRU)
    cudaGraphExec_t exec = nullptr;
    struct Run {
        bool tensor_ran = false, waits_ran = false;
    } run;
    std::vector<cudaEvent_t> pool, tm_ev, pass_ev;
    void drop() {
        if (exec) cudaGraphExecDestroy(exec);
        exec = nullptr;
        key = GraphKey{};
        tm_ev.clear();
        pass_ev.clear();
    }
    void ensure_events(size_t n) {
        while (pool.size() < n) {
            cudaEvent_t e;
            FDB_CUDA(cudaEventCreate(&e));
            pool.push_back(e);
        }
    }
    ~GraphSlot() {
        drop();
        for (auto e : pool) cudaEventDestroy(e);
    }
};
// Captured searches of one index (a few keys: a caller typically alternates
// between a couple of call shapes) and the keys seen once, eagerly.
struct GraphCache {
    static constexpr size_t kSlots = 4, kSeen = 8;
    std::vector<std::unique_ptr<GraphSlot>> slots;
    std::vector<std::pair<GraphKey, uint64_t>> seen;  // (key, epoch after the call)
    std::vector<GraphKey> refused;                    // keys that could not be captured
    uint64_t clock = 0;
    GraphSlot* find(const GraphKey& k, uint64_t epoch) {
        for (auto& g : slots)
            if (g->exec && g->key == k && g->epoch == epoch) {
                g->used = ++clock;
                return g.get();
            }
        return nullptr;
    }
    bool was_seen(const GraphKey& k, uint64_t epoch) const {
        for (auto& e : seen)
            if (e.first == k && e.second == epoch) return true;
        return false;
    }
    bool is_refused(const GraphKey& k) const {
        for (auto& r : refused)
            if (r == k) return true;
        return false;
    }
    void note_seen(const GraphKey& k, uint64_t epoch) {
        for (auto& e : seen)
            if (e.first == k) {
                e.second = epoch;
                return;
            }
        if (seen.size() == kSeen) seen.erase(seen.begin());
        seen.emplace_back(k, epoch);
    }
    // a slot for a new capture: a free one, else the least recently used
    GraphSlot* take() {
        if (slots.size() < kSlots) {
            slots.emplace_back(new GraphSlot());
            return slots.back().get();
        }
        GraphSlot* lru = slots[0].get();
        for (auto& g : slots)
            if (g->used < lru->used) lru = g.get();
        lru->drop();
        return lru;
    }
};
}  // namespace fdb

struct fdb_ivfpq;
struct fdb_bf;
namespace fdb {
void ivfpq_build(fdb_ivfpq* h, const float* x_host, const uint64_t* ids_host, size_t n,
                 const fdb_train_opts& o);
void ivfpq_load(fdb_ivfpq* h, const float* cents, const float* cb, const uint64_t* offsets,
                const uint64_t* ids, const uint8_t* codes);
void ivfpq_shard(fdb_ivfpq* h, int rank, int world);
void ivfpq_prepare_tables(fdb_ivfpq* h);
// mutate.cu: tombstones, insert_batch, re-ranking, filters
void ivfpq_sync_state(fdb_ivfpq* h);  // uploads the dead bitmap / re-ranking store if changed
void ivfpq_enable_reranking(fdb_ivfpq* h, const float* x, const uint64_t* ids, size_t n,
                            size_t factor);
void launch_rerank(fdb_ivfpq* h, const uint64_t* keys, const uint64_t* cand_ids, size_t nq,
                   size_t fetch, const float* dQ, size_t k, uint64_t* d_ids, float* d_dists,
                   uint32_t* d_counts);
bool ivfpq_delete(fdb_ivfpq* h, uint64_t id);
size_t ivfpq_live_len(const fdb_ivfpq* h);
void ivfpq_compact(fdb_ivfpq* h);
void ivfpq_insert_batch(fdb_ivfpq* h, const float* x_host, const uint64_t* ids_host, size_t n);
const float* ivfpq_call_colv(fdb_ivfpq* h, const uint32_t* skip);
// allowed: host array, or a device array when on_device
const uint32_t* ivfpq_filter_bitmap(fdb_ivfpq* h, const uint64_t* allowed, size_t na,
                                    bool on_device = false);
// persist.cu: .fdb files
uint32_t crc32(const uint8_t* p, size_t n);
void ivfpq_save(fdb_ivfpq* h, const char* path);
void ivfpq_load_file(fdb_ivfpq* h, const char* path);
void bf_save(fdb_bf* h, const char* path);
void bf_load_file(fdb_bf* h, const char* path);
void file_inspect(const char* path, fdb_file_info* info);
// call_skip (nullable): rows this call skips, dead rows included (a filter);
// fetch_mult: candidates per result before re-ranking, on top of
// rerank_factor (4 for search_filtered).
// io (nullable): host result buffers; with io the call ends synchronised.
void ivfpq_search_dev(fdb_ivfpq* h, const float* dQ, size_t nq, size_t k, int order, size_t take,
                      uint64_t* d_ids, float* d_dists, uint32_t* d_counts, fdb_stats* st,
                      const uint32_t* call_skip = nullptr, size_t fetch_mult = 1,
                      const HostIO* io = nullptr);
// ivf_tc.cu: tensor-core list scan (see there)
bool ivf_tc_eligible(const fdb_ivfpq* h, size_t k);
void ivf_tc_prepare(fdb_ivfpq* h, const std::vector<float>& cb_host,
                    const std::vector<float>& bmax_host);
void ivf_tc_search(fdb_ivfpq* h, const float* dQ, size_t nq, size_t k, int order, size_t take,
                   const uint64_t* lbeg, const uint64_t* lend, uint64_t* out_keys,
                   uint32_t* flags, unsigned long long* stat, StageTimer* pass_tm);
int* ivf_tc_error_word(fdb_ivfpq* h);
// coarse_tc.cu: the coarse quantizer on the tensor cores
void coarse_tc_prepare(fdb_ivfpq* h);
bool coarse_tc_eligible(const fdb_ivfpq* h, size_t nq, size_t take);
void coarse_tc(fdb_ivfpq* h, const float* dQ, size_t nq, size_t take, uint32_t* probes,
               float* pdist);
struct ScanParams;
void ivf_tc_rescan(fdb_ivfpq* h, const ScanParams& base, size_t nq, size_t k, int order,
                   uint64_t* out_keys);
void bf_upload(fdb_bf* h);
void bf_shard(fdb_bf* h, int rank, int world);
void bf_search_dev(fdb_bf* h, const float* dQ, size_t nq, size_t k, uint64_t* d_ids,
                   float* d_dists, uint32_t* d_counts, fdb_stats* st);
}  // namespace fdb

// ---------------------------------------------------------------------------
// the opaque handles
// ---------------------------------------------------------------------------
struct fdb_ctx {
    fdb::Ctx c;
};

struct fdb_ivfpq {
    fdb_ctx* ctx = nullptr;
    size_t dim = 0, nlist = 0, m = 0;
    int metric = 0;
    std::atomic<size_t> nprobe{1};
    unsigned long long call_wait_cycles = 0;  // a call's own wait limit (0: none)
    bool graphs = true;                       // replay repeated searches as CUDA graphs
    bool stage_timers = true;                 // fill the stage times of fdb_stats
    fdb::GraphCache graphs_cache;
    size_t n_total = 0;  // vectors in the unsharded index
    size_t n_local = 0;  // vectors whose lists live on this device
    fdb::DevBuf<float> cents;     // [nlist][dim]
    fdb::DevBuf<float> cb;        // [m][256][dim/m]
    fdb::DevBuf<uint64_t> offs;   // [nlist+1], empty ranges for lists not held here
    fdb::DevBuf<uint64_t> ids;    // [n_total] list-major
    fdb::DevBuf<uint8_t> codes;   // [n_total][m] list-major
    std::vector<uint64_t> h_offs_full;  // unsharded offsets (host)
    std::vector<uint64_t> h_offs;       // offsets as held on this device
    bool sharded = false;
    int shard_world = 1, shard_rank = 0;
    fdb::DevBuf<uint64_t> shard_be;     // [2][nlist] list begin / end when sharded
    std::vector<uint8_t> owned;         // [nlist] lists held here (sharded)
    // table mode (subvectors of 8+ floats): per-list tables and error-bound terms
    int scan_mode = FDB_SCAN_AUTO;
    fdb::DevBuf<float> centsT;          // [dim][nlist_pad] for the tiled coarse kernel
    int nlist_pad = 0;
    // tensor-core coarse quantizer: centroids as fp16 rows scaled by 2^c16_sb,
    // zero-padded to [c16_npad][c16_dpad], their squared norms, max norm
    fdb::DevBuf<__half> c16;
    fdb::DevBuf<float> c16_norm;
    int c16_dpad = 0, c16_sb = 0, c16_npad = 0;
    float c16_cmax = 0.0f;
    fdb::DevBuf<float> btab;            // [nlist][m][256]
    fdb::DevBuf<float> cmax, bmax;      // [m]
    // tensor mode (dim <= 128 after padding): codes decoded to fp16 residual
    // vectors scaled by 2^tc_sb, their squared norms, and lists by length
    fdb::DevBuf<__half> dec16;          // [tc_rows][tc_dpad], lists 128-row aligned
    fdb::DevBuf<float> dnorm;           // [tc_rows] ||rhat||^2, +inf in padding rows
    fdb::DevBuf<uint32_t> lorder;       // [nlist] lists by decreasing length
    fdb::DevBuf<uint32_t> tc_pstart;    // [nlist] first row of each list, 128-row aligned
    fdb::DevBuf<float> tc_rhl;          // [nlist] upper bound of ||rhat|| per list
    int tc_dpad = 0, tc_sb = 0;
    size_t tc_rows = 0;                 // rows of the padded layout
    size_t tc_maxpad = 0;               // longest padded list
    float tc_colmax = 0.0f;             // upper bound of ||rhat||^2
    // pass-1 sampling quota: 1/div of a query's probed codes (0: every probe's
    // first tile); chosen per nprobe by timing a sample batch (calibrated)
    uint64_t tc_sample_div = 64;
    std::vector<std::pair<size_t, uint64_t>> tc_quota;  // (nprobe, div) calibrated
    // Vector ids the reference keeps on centroids and codebook entries; no
    // role in search, carried so .fdb files round-trip unchanged
    std::vector<uint64_t> cent_ids;     // [nlist]
    std::vector<uint64_t> cb_ids;       // [m*256]
    // re-ranking store (enable_reranking, ivf_pq.rs:513-517): original
    // vectors by id; host copy in slot order, device copy rebuilt when dirty
    bool rerank = false;
    size_t rerank_factor = 1;
    std::vector<uint64_t> rr_ids;       // [slots]
    std::vector<float> rr_x;            // [slots][dim]
    std::unordered_map<uint64_t, size_t> rr_slot;
    bool rr_dirty = false;
    fdb::DevBuf<uint64_t> rr_sorted;    // ids ascending
    fdb::DevBuf<uint32_t> rr_sorted_slot;
    fdb::DevBuf<float> rr_dev;          // [slots][dim]
    // tombstones (delete, ivf_pq.rs:1786-1805): per list, the deleted ids;
    // `dead` marks every row of the list-major layout they hide
    std::vector<std::unordered_set<uint64_t>> tomb;  // [nlist] (empty: none)
    size_t n_tomb = 0;                  // sum of the per-list set sizes
    std::vector<uint64_t> h_ids;        // host mirror of ids (list-major)
    std::vector<uint32_t> h_dead;       // host dead bitmap (empty: no tombstones)
    fdb::DevBuf<uint32_t> dead;         // device copy, uploaded when dead_dirty
    bool dead_dirty = false;
    std::vector<std::pair<uint64_t, uint32_t>> id_index;  // (id, row) ascending, lazy
    bool id_index_ok = false;
    fdb::DevBuf<uint32_t> f_skip;       // per-call filter bitmap (search_filtered)
    fdb::DevBuf<uint64_t> f_sorted;     // allowed ids copied from the host
    fdb::DevBuf<uint64_t> d_idx_ids;    // ids sorted, with their rows (filters)
    fdb::DevBuf<uint32_t> d_idx_rows;
    bool d_idx_ok = false;
    fdb::DevBuf<float> f_colv;          // tensor scan ||rhat||^2 with a call's filter
    const float* tc_colv = nullptr;     // set for one call: overrides dnorm
    std::mutex mu;
    // per-call scratch
    fdb::DevBuf<float> s_q, s_coarse, s_qT, s_pdist;
    fdb::DevBuf<__half> s_cq16;         // tensor coarse: fp16 query rows
    fdb::DevBuf<float> s_cqn, s_cqs2, s_cqerr, s_cdapprox;
    fdb::DevBuf<uint32_t> s_crange;     // tensor coarse: per-row min / max of d~
    fdb::DevBuf<uint32_t> s_probe;
    fdb::DevBuf<uint64_t> s_keys, s_ids, s_gather, s_merged, s_merged_ids, s_out_ids, s_approx;
    fdb::DevBuf<float> s_dists;
    fdb::DevBuf<uint32_t> s_counts, s_flags;
    fdb::DevBuf<uint64_t> s_cal_ids;    // pass-1 quota calibration outputs
    fdb::DevBuf<float> s_cal_d;
    fdb::DevBuf<uint32_t> s_cal_c;
    fdb::DevBuf<unsigned long long> s_stat;
    fdb::PinnedWords s_pin;  // end-of-call readbacks (statistics, error word, counts)
    // tensor-mode scratch: pair grouping, residual rows, items, shortlists
    fdb::DevBuf<uint32_t> t_keys, t_vals, t_off, t_pq, t_qbad, t_range, t_inv, t_plen,
        t_seg, t_fprobes, t_fcnt, t_uoff, t_unit_q, t_unit_l, t_qrange;
    fdb::DevBuf<uint64_t> t_unit_keys;
    fdb::DevBuf<float> t_dump, t_dk;
    fdb::DevBuf<uint64_t> t_ekeys;
    fdb::DevBuf<int> t_elist;
    fdb::DevBuf<uint8_t> t_tmp, t_items;
    fdb::DevBuf<__half> t_a16;
    fdb::DevBuf<float> t_rn, t_s2, t_tau;
    fdb::DevBuf<uint64_t> t_part, t_cand;
    fdb::DevBuf<unsigned> t_cand_cnt;
    fdb::DevBuf<uint32_t> t_ext;        // [0] extended queries, then their indices
    fdb::DevBuf<float> t_ext_thr, t_tadm, t_eb;
    fdb::DevBuf<unsigned> t_icnt;       // item counts per (kind, list) and their offsets
    fdb::DevBuf<uint8_t> t_tmp2;        // scan scratch for the item offsets
    // pass-2 pruning: kept pairs per list and their offsets, flags, the kept
    // pair ids (count first) and their compacted rows
    fdb::DevBuf<unsigned> t_live, t_sel;
    fdb::DevBuf<uint8_t> t_pflag, t_tmp3;
    fdb::DevBuf<__half> t_a2;
    fdb::DevBuf<uint32_t> t_q2;
    fdb::DevBuf<float> t_rn2, t_s22;
};

struct fdb_bf {
    fdb_ctx* ctx = nullptr;
    int metric = 0;
    size_t dim = 0;
    size_t n = 0;          // rows held on this device
    size_t row0 = 0;       // global index of the first held row
    std::vector<float> h_x;      // host copy kept only while rows are appended
    std::vector<uint64_t> h_ids;
    fdb::DevBuf<float> x;        // [n][dim]
    fdb::DevBuf<uint64_t> ids;   // [n]
    fdb::DevBuf<float> norms;    // [n + 256] squared norms in AVX2 order, +inf padding
    fdb::DevBuf<float> rnorms;   // cosine: [n + 256] 1/||x|| (0 for zero rows and padding)
    bool dirty = true;
    bool sharded = false;
    int shard_world = 1;
    // tensor-core shortlist: fp16 rows padded to a multiple of 64 columns
    int scan_mode = FDB_SCAN_AUTO;
    int kpad = 0;
    float xmax = 0.0f;           // largest row norm (rounded up), for the error bound
    fdb::DevBuf<__half> x16;     // [n][kpad]
    std::mutex mu;
    fdb::DevBuf<float> s_q, s_qnorm;
    fdb::DevBuf<__half> s_q16;
    fdb::GemmScratch gemm;
    fdb::DevBuf<uint64_t> s_part, s_keys, s_ids, s_gather, s_merged, s_merged_ids, s_out_ids;
    fdb::DevBuf<float> s_dists;
    fdb::DevBuf<uint32_t> s_counts, s_flags;
    fdb::DevBuf<uint64_t> s_cal_ids;    // pass-1 quota calibration outputs
    fdb::DevBuf<float> s_cal_d;
    fdb::DevBuf<uint32_t> s_cal_c;
};
