/*
 * forgegpu.h -- C ABI of the B200 (sm_100a) engine for forge-db's
 * nearest-neighbour search and training path.
 *
 * Every entry point replaces one method of the reference crate's Rust API
 * (HueCodes/forge-db; file:line cited beside each declaration).  The ABI is
 * plain C: opaque handles, caller-owned input and output buffers, sizes as
 * size_t, and an int status (0 = OK, negative = error) whose codes map one to
 * one onto ForgeDbError variants (src/error.rs:14-145).  Where the reference
 * panics on bad input, the matching call returns an error code instead and
 * fdb_last_error() holds the message.
 *
 * Distances keep the reference's meaning: IVF-PQ returns squared ADC sums
 * (src/index/ivf_pq.rs:590-677, 850-1047); brute force returns the metric of
 * src/distance/mod.rs:40-48 (Euclidean = sqrt(L2^2), DotProduct = -dot,
 * Cosine = 1 - cos).  Result rows are sorted ascending; rows with fewer than
 * k hits are padded with id UINT64_MAX and distance +inf, and the per-row
 * count says how many are real.
 *
 * Threading: search calls on one handle are safe from several threads (a
 * per-handle lock serialises GPU submission); fdb_ivfpq_set_nprobe is atomic
 * and may race with searches, as in the reference (ivf_pq.rs:524-533).
 */
#ifndef FORGEGPU_H
#define FORGEGPU_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (ForgeDbError, src/error.rs:14-145) ------------------- */
#define FDB_OK 0
#define FDB_ERR_INVALID_ARG (-1)          /* InvalidParameter / panicking input */
#define FDB_ERR_DIM_MISMATCH (-2)         /* DimensionMismatch */
#define FDB_ERR_EMPTY_TRAINING_SET (-3)   /* EmptyTrainingSet */
#define FDB_ERR_DIM_NOT_DIVISIBLE (-4)    /* DimensionNotDivisible */
#define FDB_ERR_INSUFFICIENT_VECTORS (-5) /* InsufficientVectors */
#define FDB_ERR_TIMEOUT (-6)              /* Timeout */
#define FDB_ERR_CUDA (-7)                 /* device error (no reference analogue) */
#define FDB_ERR_NCCL (-8)                 /* collective error (no reference analogue) */
#define FDB_ERR_OOM (-9)                  /* MemoryLimitExceeded */
#define FDB_ERR_EMPTY_VECTOR_SET (-10)    /* EmptyVectorSet */
#define FDB_ERR_UNSUPPORTED (-11)         /* NotSupported */
#define FDB_ERR_IO (-12)                  /* Io */
#define FDB_ERR_SERIALIZATION (-13)       /* SerializationError (bincode) */
#define FDB_ERR_CHECKSUM (-14)            /* ChecksumMismatch */
#define FDB_ERR_INVALID_FORMAT (-15)      /* InvalidFormat */
#define FDB_ERR_DISK_SPACE (-16)          /* InsufficientDiskSpace */

/* ---- DistanceMetric (src/distance/mod.rs:16-33) ------------------------- */
#define FDB_METRIC_EUCLIDEAN 0
#define FDB_METRIC_EUCLIDEAN_SQUARED 1
#define FDB_METRIC_COSINE 2
#define FDB_METRIC_DOT_PRODUCT 3
#define FDB_METRIC_MANHATTAN 4

/* Largest k (and nprobe for the warp selector) served by the search kernels. */
#define FDB_MAX_K 256

typedef struct fdb_ctx fdb_ctx;
typedef struct fdb_ivfpq fdb_ivfpq;
typedef struct fdb_bf fdb_bf;

/* Per-call statistics (the counters of search_with_stats,
 * src/index/ivf_pq.rs:1218-1349, plus device stage times). */
typedef struct fdb_stats {
    uint64_t lists_probed;   /* (query, list) pairs scanned on this device */
    uint64_t codes_scanned;  /* PQ codes (or database rows) scored */
    uint64_t bytes_scanned;  /* algorithmic bytes: codes_scanned * code bytes */
    double coarse_ms;        /* coarse quantizer + probe selection */
    double scan_ms;          /* LUT build + code scan + local top-k (scan kernel); tensor
                                mode: both list-scan passes with the shortlist, exact
                                rescoring, certification and its extension */
    double rescore_ms;       /* table mode: exact rescoring, certification, re-scans;
                                tensor mode: the exact re-scan of failed lists */
    double merge_ms;         /* cross-device exchange + final merge */
    double total_ms;         /* whole call, device clock */
    uint64_t exact_rescans;  /* table/tensor mode: queries re-scanned exactly after
                                failing certification */
    double kernel_ms;        /* device time of the dominant scan kernel: the tensor
                                list scan's second pass (IVF-PQ tensor mode), the
                                filter pass (brute force, tensor path), else the scan */
    uint64_t kernel_scores;  /* (query, code/row) scores that kernel computed */
    uint64_t extended;       /* tensor mode: queries certified by rescoring every stored
                                candidate below a widened threshold instead of a re-scan */
    double comm_ms[4];       /* sharded index: device time inside each collective, its wait
                                for the slowest device included: [0] all-gather of the
                                probes, [1] all-reduce of the pass-1 thresholds, [2]
                                all-reduce of the exact k-th distances, [3] all-gather of
                                the local top-k lists (within coarse_ms, scan_ms, scan_ms
                                and merge_ms) */
} fdb_stats;

/* IVF-PQ scan modes (fdb_ivfpq_set_scan_mode).  All return the reference's
 * exact distances.  EXACT builds every (query, list) table in the AVX2 order.
 * TABLES builds it from a per-list table precomputed at build time plus a
 * per-query table, keeps a shortlist of max(32, 2k) candidates, recomputes
 * their distances exactly, and certifies the result with a worst-case
 * rounding bound; a query that fails the bound is re-scanned in EXACT mode.
 * TENSOR (k <= 64 -- with re-ranking, k * rerank_factor -- and dim <= 128
 * after padding to 64) groups the probed (query, list) pairs by list and
 * scores them on the tcgen05 tensor cores against fp16 codes decoded at build
 * time, keeps a shortlist of 64, and rescores and certifies it the same way.  AUTO picks TENSOR for batches of
 * 256+ queries where it applies, else TABLES for subvectors of 8+ floats and
 * k <= 128, else EXACT. */
#define FDB_SCAN_AUTO 0
#define FDB_SCAN_EXACT 1
#define FDB_SCAN_TABLES 2
#define FDB_SCAN_TENSOR 3

/* Training options for fdb_ivfpq_build.  Zero-initialise and set what you
 * need.  The reference draws samples and initial centroids from an unseeded
 * thread_rng (src/index/ivf_pq.rs:383-396, 422-446; src/kmeans.rs:52-64);
 * here they are either injected (the index arrays) or drawn from `seed`. */
typedef struct fdb_train_opts {
    size_t ivf_sample;              /* 0 -> min(n, 30000)   (ivf_pq.rs:383) */
    size_t pq_sample;               /* 0 -> min(n, 100000)  (ivf_pq.rs:422) */
    size_t ivf_iters;               /* 0 -> 25              (ivf_pq.rs:398) */
    size_t pq_iters;                /* 0 -> 25              (constants.rs:18) */
    const uint32_t* ivf_sample_idx; /* [ivf_sample] or NULL */
    const uint32_t* ivf_init_idx;   /* [nlist] or NULL */
    const float* ivf_kpp_u;         /* [nlist] k-means++ draws (nlist <= 64) or NULL */
    const uint32_t* pq_sample_idx;  /* [pq_sample] or NULL */
    const uint32_t* pq_init_idx;    /* [m*256] or NULL */
    uint64_t seed;                  /* used for every NULL draw above */
} fdb_train_opts;

/* ---- errors, version ---------------------------------------------------- */
const char* fdb_last_error(void); /* thread-local message of the last failure */
int fdb_version(void);            /* major*10000 + minor*100 + patch */

/* ---- context: one device, one stream, optional NCCL communicator -------- */
int fdb_ctx_create(int device, fdb_ctx** out);
int fdb_ctx_free(fdb_ctx* ctx);
/* The CUDA stream (cudaStream_t) every call of this context runs on. */
int fdb_ctx_stream(fdb_ctx* ctx, void** stream_out);
/* Multi-GPU: rank 0 creates the 128-byte NCCL unique id, every rank passes it
 * to fdb_ctx_init_comm.  Searches on a sharded index then exchange local
 * top-k lists over NVLink (ncclAllGather) and merge on every device.  The
 * communicator is non-blocking: if not every rank joins within timeout_s
 * (300 s for fdb_ctx_init_comm) the initialisation is aborted and the call
 * returns FDB_ERR_TIMEOUT; the context stays usable without a communicator.
 * (No reference counterpart: the reference runs on one host's cores.) */
int fdb_nccl_unique_id(void* id_out /* 128 bytes */);
int fdb_ctx_init_comm(fdb_ctx* ctx, int rank, int world, const void* nccl_id);
int fdb_ctx_init_comm_timeout(fdb_ctx* ctx, int rank, int world, const void* nccl_id,
                              double timeout_s);
/* Limit of every bounded wait inside the tensor-core kernels (default 2 s).
 * A wait that runs out makes the kernel stop, drain the copies it issued and
 * return; the call then fails with FDB_ERR_TIMEOUT and the context stays
 * usable (the next call starts clean).  Counterpart of the deadline checks of
 * search_with_timeout (ivf_pq.rs:1369-1455). */
int fdb_ctx_set_wait_limit(fdb_ctx* ctx, double seconds);
/* Test hook for the timeout path: the next `count` list-scan launches of the
 * tensor path on this context issue no work, so the waits inside them find a
 * flag that nothing sets and run out after the wait limit (no fault, no hang:
 * nothing is in flight).  The call that contains them returns
 * FDB_ERR_TIMEOUT. */
int fdb_ctx_test_stall_scans(fdb_ctx* ctx, int count);
/* Host memory the device can copy from at full speed (cudaHostAlloc). */
int fdb_host_alloc(size_t bytes, void** out);
int fdb_host_free(void* p);

/* ---- seeded draws (replacing thread_rng; deterministic across devices) -- */
/* First `take` entries of a seeded Fisher-Yates shuffle of 0..n-1 (the
 * `indices.shuffle(&mut rng); take(k)` idiom of src/kmeans.rs:53-61). */
int fdb_sample_indices(uint64_t seed, size_t n, size_t take, uint32_t* out);
/* `count` uniform draws in [0,1) on the 2^-23 grid of rand's f32 sampler. */
int fdb_uniform_draws(uint64_t seed, size_t count, float* out);

/* ---- distances (src/distance/mod.rs:40-48; simd.rs:293-517) ------------- */
/* out[i] = metric(a[i], b[i]) for n row pairs of `dim` floats, computed on the
 * device in the reference's AVX2 summation order (bit-exact). */
int fdb_pairwise_distance(fdb_ctx* ctx, int metric, const float* a, const float* b, size_t n,
                          size_t dim, float* out);

/* ---- KMeans (src/kmeans.rs:18-193, 257-345) ----------------------------- */
/* KMeans::new(k, max_iters).fit_raw(data, dim, n) (kmeans.rs:87-193; fit at
 * :45-78 is the same algorithm).  init_idx[k]: the shuffled-prefix picks for
 * k > 64, or for k <= 64 the first k-means++ pick (init_idx[0]) and the
 * fallback picks; kpp_u[k]: the k-means++ uniform draws (k <= 64 only).  NULL
 * arrays are drawn from `seed`.  assign_out[n] (nullable) receives each
 * point's nearest final centroid (first minimum). */
int fdb_kmeans_fit(fdb_ctx* ctx, const float* data, size_t n, size_t dim, size_t k,
                   size_t max_iters, const uint32_t* init_idx, const float* kpp_u, uint64_t seed,
                   float* centroids_out, uint32_t* assign_out, int* iters_run);
/* Nearest-centroid assignment, first minimum wins (kmeans.rs:257-270;
 * ivf_pq.rs:403-414). */
int fdb_assign(fdb_ctx* ctx, const float* x, size_t n, const float* centroids, size_t k,
               size_t dim, uint32_t* out);
/* KMeans::find_nearest_centroids (kmeans.rs:334-345): the k nearest centroid
 * ids of one query, ascending. */
int fdb_find_nearest_centroids(fdb_ctx* ctx, const float* centroids, size_t kc, size_t dim,
                               const float* query, size_t k, uint32_t* out);

/* No reference counterpart.  An allocation-free form of
 * fdb_find_nearest_centroids for callers that cannot call cudaMalloc at
 * search time: a serving process that reserved all of its device memory in
 * a pool at start-up (another allocation would fail or evict its pool), or a
 * latency-bound loop where cudaMalloc's implicit device synchronisation is
 * not allowed.  It serves nq queries at once on device buffers
 * (d_centroids[kc][dim], d_queries[nq][dim] -> d_out[nq][min(k, kc)], each
 * row ascending, the same ids as the host-buffer call).  Its only scratch,
 * the nq x kc distance matrix, lives in a fixed array in the library's
 * device image (16 MiB on every device that loads the library, held until
 * the process exits), so the call itself never allocates.
 *   - nq * kc must not exceed FDB_NOALLOC_MAX_DISTANCES (4 Mi floats) and nq
 *     must not exceed FDB_NOALLOC_MAX_QUERIES; when min(k, kc) is above 256,
 *     kc must not exceed FDB_NOALLOC_MAX_SORTED_CENTROIDS.  Larger requests
 *     fail with FDB_ERR_INVALID_ARG before any device work.  Split them into
 *     batches.
 *   - The first call on a device does the set-up: it looks up the scratch
 *     array's device address (with that device current) and keeps it for the
 *     life of the process.  Make that first call (nq = 0 is enough) before
 *     any stream capture.  A call with min(k, kc) above 256 and kc above
 *     4096 also raises the selection kernel's shared-memory limit
 *     (cudaFuncSetAttribute, no allocation) on each such call.
 *   - After cudaDeviceReset of a device the kept address is stale, like every
 *     other handle of this library on that device: do not call it again.
 *   - There is one scratch array per device and each call reuses it: calls
 *     that overlap on a device (two contexts, or two threads with separate
 *     contexts) race on it.  Calls through one context are serialised, and
 *     the call returns after its work on the device is complete. */
#define FDB_NOALLOC_MAX_DISTANCES (1u << 22)
#define FDB_NOALLOC_MAX_QUERIES (1u << 18)
#define FDB_NOALLOC_MAX_SORTED_CENTROIDS (1u << 14)
int fdb_find_nearest_centroids_noalloc(fdb_ctx* ctx, const float* d_centroids, size_t kc,
                                       size_t dim, const float* d_queries, size_t nq, size_t k,
                                       uint32_t* d_out);

/* ---- ProductQuantizer (src/pq.rs:33-245) -------------------------------- */
/* ProductQuantizer::try_train (pq.rs:55-95): codebooks_out[m][256][dim/m].
 * init_idx[m*256] (NULL -> seed) are the per-subspace initial picks. */
int fdb_pq_train(fdb_ctx* ctx, const float* x, size_t n, size_t dim, size_t m, size_t iters,
                 const uint32_t* init_idx, uint64_t seed, float* codebooks_out, int* iters_out);
/* ProductQuantizer::encode (pq.rs:114-139) over n vectors: codes_out[n][m]. */
int fdb_pq_encode(fdb_ctx* ctx, const float* codebooks, size_t m, size_t dim, const float* x,
                  size_t n, uint8_t* codes_out);
/* build_lookup_table_flat (pq.rs:175-189) for nq queries: lut_out[nq][m*256]. */
int fdb_pq_lookup_tables(fdb_ctx* ctx, const float* codebooks, size_t m, size_t dim,
                         const float* queries, size_t nq, float* lut_out);

/* ---- IVFPQIndex (src/index/ivf_pq.rs:343-1084) -------------------------- */
/* IVFPQIndex::build (ivf_pq.rs:374-506).  `ids` may be NULL (ids 0..n-1).
 * nprobe starts at 1 as in the reference. */
int fdb_ivfpq_build(fdb_ctx* ctx, const float* x, const uint64_t* ids, size_t n, size_t dim,
                    size_t nlist, size_t m, int metric, const fdb_train_opts* opts,
                    fdb_ivfpq** out);
/* An index from trained artefacts (the parity path: the same centroids,
 * codebooks and lists as a reference-built index).  offsets[nlist+1] delimit
 * each list's rows of ids[] and codes[][m] (list-major). */
int fdb_ivfpq_from_trained(fdb_ctx* ctx, const float* centroids, const float* codebooks,
                           size_t nlist, size_t m, size_t dim, const uint64_t* offsets,
                           const uint64_t* ids, const uint8_t* codes, int metric,
                           fdb_ivfpq** out);
/* Copy the trained artefacts out (NULL pointers are skipped). */
int fdb_ivfpq_export(fdb_ivfpq* h, float* centroids, float* codebooks, uint64_t* offsets,
                     uint64_t* ids, uint8_t* codes);
/* Keep only this rank's share of the inverted lists (greedy balance of
 * list bytes over `world` devices); the other lists become empty here. */
int fdb_ivfpq_shard(fdb_ivfpq* h, int rank, int world);
/* The list -> device plan fdb_ivfpq_shard uses: owner[l] in [0, world) for
 * each of nlist lists of the given sizes (host only; needs no device). */
int fdb_ivfpq_shard_plan(const uint64_t* sizes, size_t nlist, int world, int* owner);
/* Scan mode (FDB_SCAN_*); no reference counterpart (the reference has one
 * CPU scan).  Results are identical in every mode. */
int fdb_ivfpq_set_scan_mode(fdb_ivfpq* h, int mode);
/* Repeated batch searches of one shape (the same buffers, sizes and modes)
 * replay a CUDA graph of the whole device step from their second call
 * instead of launching ~40 kernels (default: on).  No reference counterpart
 * (a launch-overhead choice of this engine); results are identical. */
int fdb_ivfpq_set_graphs(fdb_ivfpq* h, int enable);
/* Whether a search given an fdb_stats fills its stage times (coarse_ms,
 * scan_ms, rescore_ms, merge_ms, total_ms, comm_ms; default: on).  Each stage
 * mark is an event record inside the step; off, a call with statistics
 * records only the two events around the list scan's pass 2 (kernel_ms) and
 * the counters.  No reference counterpart. */
int fdb_ivfpq_set_stage_timers(fdb_ivfpq* h, int enable);
/* The tensor path's pass-1 sampling quota for batch searches with `nprobe`
 * probes: pass 1 scores each query's first list plus the first tile of its
 * nearest other probes until it has seen 1/div of the query's probed codes
 * (div 0: every probe's first tile).  Unset, it is calibrated on the first
 * batch of 1024+ queries with that nprobe (up to 16384 of its queries timed under
 * div 128, 64, 16, 4, 0; the fastest is kept).  It splits the work between
 * the two passes only: results are identical for every div.  No reference
 * counterpart. */
int fdb_ivfpq_set_pass1_quota(fdb_ivfpq* h, size_t nprobe, uint64_t div);
/* The quota in use for `nprobe` probes (set or calibrated), -1 if none yet. */
int fdb_ivfpq_get_pass1_quota(fdb_ivfpq* h, size_t nprobe, int64_t* div);
/* set_nprobe (ivf_pq.rs:524-528): stores min(nprobe, nlist). */
int fdb_ivfpq_set_nprobe(fdb_ivfpq* h, size_t nprobe);
size_t fdb_ivfpq_nprobe(const fdb_ivfpq* h);
size_t fdb_ivfpq_len(const fdb_ivfpq* h);          /* vectors held on this device */
size_t fdb_ivfpq_n_partitions(const fdb_ivfpq* h); /* nlist */
size_t fdb_ivfpq_dim(const fdb_ivfpq* h);
size_t fdb_ivfpq_n_subvectors(const fdb_ivfpq* h);  /* PQ subvectors m (pq.rs:37) */
/* IVFPQIndex::search (ivf_pq.rs:590-677): one query, the single-query ADC
 * order (pq.rs:218-245); n_out receives the number of results (<= k). */
int fdb_ivfpq_search(fdb_ivfpq* h, const float* query, size_t k, uint64_t* ids, float* dists,
                     size_t* n_out);
/* IVFPQIndex::batch_search / batch_search_parallel (ivf_pq.rs:850-1084):
 * host buffers; ids/dists are [nq][k], counts [nq] (nullable), stats
 * nullable. */
int fdb_ivfpq_batch_search(fdb_ivfpq* h, const float* queries, size_t nq, size_t k,
                           uint64_t* ids, float* dists, uint32_t* counts, fdb_stats* stats);
/* IVFPQIndex::search_with_timeout (ivf_pq.rs:1369-1455): search() under a
 * deadline timeout_s from the call.  Returns FDB_ERR_TIMEOUT (results not
 * valid) when the deadline passes -- the kernels' bounded waits give up at it
 * and results that come back after it are refused; elapsed_s (nullable)
 * receives the call's duration, the reference's Ok((results, elapsed)).
 * The batch form applies one deadline to batch_search() of nq queries. */
int fdb_ivfpq_search_with_timeout(fdb_ivfpq* h, const float* query, size_t k, double timeout_s,
                                  uint64_t* ids, float* dists, size_t* n_out,
                                  double* elapsed_s);
int fdb_ivfpq_batch_search_with_timeout(fdb_ivfpq* h, const float* queries, size_t nq, size_t k,
                                        double timeout_s, uint64_t* ids, float* dists,
                                        uint32_t* counts, double* elapsed_s);
/* The same search on DEVICE buffers of this context's device, enqueued on the
 * context stream; returns after the results are written (stream synced). */
int fdb_ivfpq_batch_search_device(fdb_ivfpq* h, const float* d_queries, size_t nq, size_t k,
                                  uint64_t* d_ids, float* d_dists, uint32_t* d_counts,
                                  fdb_stats* stats);
int fdb_ivfpq_free(fdb_ivfpq* h);

/* ---- IVFPQIndex: re-ranking, filters, updates (ivf_pq.rs:513-831, 1731-1890) */
/* enable_reranking (ivf_pq.rs:513-517): keep the n original vectors (ids[i]
 * names x[i]; a repeated id keeps its last vector) and from now on fetch
 * k * max(rerank_factor, 1) PQ candidates per query, re-score those that have
 * an original vector with sqrt(L2^2) on the device (the reference's
 * euclidean_distance_squared order, then a correctly rounded square root),
 * sort stably and keep k (rerank_results, ivf_pq.rs:556-582).  Results are
 * then Euclidean distances.  k * rerank_factor must not exceed FDB_MAX_K. */
int fdb_ivfpq_enable_reranking(fdb_ivfpq* h, const float* x, const uint64_t* ids, size_t n,
                               size_t dim, size_t rerank_factor);
/* search_filtered (ivf_pq.rs:692-831): search() restricted to the vectors
 * whose id is in allowed_ids[n_allowed] (the ids of the reference's
 * MetadataStore::filter_bitmap(filter); rows with other ids are skipped during
 * the scan).  n_allowed == 0 returns no results.  With re-ranking on, 4 *
 * k * rerank_factor candidates are re-ranked (filter_fetch_k, :720). */
int fdb_ivfpq_search_filtered(fdb_ivfpq* h, const float* query, size_t k,
                              const uint64_t* allowed_ids, size_t n_allowed, uint64_t* ids,
                              float* dists, size_t* n_out);
/* No reference counterpart: search_filtered for nq queries sharing one
 * filter, on host buffers (ids/dists [nq][k], counts [nq] nullable). */
int fdb_ivfpq_batch_search_filtered(fdb_ivfpq* h, const float* queries, size_t nq, size_t k,
                                    const uint64_t* allowed_ids, size_t n_allowed,
                                    uint64_t* ids, float* dists, uint32_t* counts);
/* The same on DEVICE buffers of this context's device (queries, allowed ids
 * and outputs), enqueued on the context stream; returns when done. */
int fdb_ivfpq_batch_search_filtered_device(fdb_ivfpq* h, const float* d_queries, size_t nq,
                                           size_t k, const uint64_t* d_allowed_ids,
                                           size_t n_allowed, uint64_t* d_ids, float* d_dists,
                                           uint32_t* d_counts, fdb_stats* stats);
/* insert_batch (ivf_pq.rs:1731-1773): each vector goes to its nearest list
 * (first minimum), its residual is PQ-encoded and appended to that list, a
 * tombstone on its id in that list is lifted, and with re-ranking on it
 * enters the original-vector store.  ids must not be NULL. */
int fdb_ivfpq_insert_batch(fdb_ivfpq* h, const float* x, const uint64_t* ids, size_t n,
                           size_t dim);
/* delete (ivf_pq.rs:1786-1805): tombstones `id` in the first list that holds
 * it and has not tombstoned it yet (every row of that list with the id is
 * then skipped); *deleted = 1 if so, else 0.  Removes it from the re-ranking
 * store. */
int fdb_ivfpq_delete(fdb_ivfpq* h, uint64_t id, int* deleted);
size_t fdb_ivfpq_num_tombstones(const fdb_ivfpq* h);      /* ivf_pq.rs:1807-1812 */
size_t fdb_ivfpq_len_with_tombstones(const fdb_ivfpq* h); /* ivf_pq.rs:1098-1103 */
float fdb_ivfpq_fragmentation_ratio(const fdb_ivfpq* h);  /* ivf_pq.rs:1815-1822 */
/* compact (ivf_pq.rs:1828-1852): drop tombstoned rows, keeping row order. */
int fdb_ivfpq_compact(fdb_ivfpq* h);
/* rebuild (ivf_pq.rs:1860-1890): retrain on the re-ranking store's vectors
 * with the same nlist, m, metric, nprobe and rerank_factor; FDB_ERR_UNSUPPORTED
 * without re-ranking, FDB_ERR_EMPTY_VECTOR_SET when the store is empty.
 * opts (nullable) gives the training draws as for fdb_ivfpq_build.  The
 * vectors are taken in insertion order (the reference takes hash-map order);
 * the rebuilt index is unsharded.  If training fails the handle is left
 * unusable and must be freed. */
int fdb_ivfpq_rebuild(fdb_ivfpq* h, const fdb_train_opts* opts);

/* ---- IVFPQIndexBuilder (src/index/ivf_pq_builder.rs:56-331) ------------ */
/* Zero-initialise, then fdb_builder_defaults() gives IVFPQIndexBuilder::new()
 * (auto_tune on, nprobe 1, rerank_factor 1, Euclidean, no targets). */
typedef struct fdb_builder_opts {
    size_t num_clusters;      /* 0: auto_tune_clusters (:269-282) */
    size_t num_subvectors;    /* 0: auto_tune_subvectors (:284-311) */
    int metric;               /* FDB_METRIC_* */
    int auto_tune;
    size_t target_memory_mb;  /* 0: none; over budget only warns (:238-248) */
    float target_recall;      /* < 0: none; else clamped to [0, 1] (:160-163) */
    size_t nprobe;            /* auto_tune_nprobe (:313-337) */
    size_t rerank_factor;     /* max(1, .) (:171-174) */
    int enable_reranking;     /* keep the build vectors as originals */
} fdb_builder_opts;
void fdb_builder_defaults(fdb_builder_opts* o);
/* Host only: the parameters build() would use for n vectors of `dim` floats
 * (the auto-tune rules and their validation: InsufficientVectors when
 * clusters > n, InvalidParameter when dim % m != 0) and the memory estimate
 * of estimate_memory_mb (:340-361) in MiB. */
int fdb_builder_plan(const fdb_builder_opts* o, size_t n, size_t dim, size_t* num_clusters,
                     size_t* num_subvectors, size_t* nprobe, size_t* estimated_mb);
/* IVFPQIndexBuilder::build (:188-259): plan, IVFPQIndex::build, set_nprobe,
 * enable_reranking(vectors, rerank_factor) when asked.  x NULL -> "vectors
 * are required" (InvalidParameter); n == 0 -> EmptyVectorSet.  train (nullable)
 * gives the training draws as for fdb_ivfpq_build. */
int fdb_builder_build(fdb_ctx* ctx, const fdb_builder_opts* o, const float* x,
                      const uint64_t* ids, size_t n, size_t dim, const fdb_train_opts* train,
                      fdb_ivfpq** out);

/* ---- BruteForceIndex (src/index/brute_force.rs:60-225) ------------------ */
/* BruteForceIndex::new(metric) followed by add() of n rows
 * (brute_force.rs:67-80).  `ids` may be NULL (ids 0..n-1). */
int fdb_bf_create(fdb_ctx* ctx, int metric, const float* x, const uint64_t* ids, size_t n,
                  size_t dim, fdb_bf** out);
/* BruteForceIndex::add for n more rows (brute_force.rs:75-80). */
int fdb_bf_add(fdb_bf* h, const float* x, const uint64_t* ids, size_t n, size_t dim);
/* Keep only this rank's contiguous share of the rows. */
int fdb_bf_shard(fdb_bf* h, int rank, int world);
/* Scan mode (FDB_SCAN_*); no reference counterpart.  TABLES/AUTO use the
 * tcgen05 tensor-core shortlist (fp16 operands, fp32 accumulation) for every
 * metric but Manhattan, dims <= 256 and k <= 128, then rescore the shortlist
 * exactly and certify it; EXACT scans every row in the AVX2 order.  Results
 * are identical in every mode. */
int fdb_bf_set_scan_mode(fdb_bf* h, int mode);
size_t fdb_bf_len(const fdb_bf* h);
size_t fdb_bf_dimension(const fdb_bf* h); /* 0 when empty (brute_force.rs:92-99) */
/* BruteForceIndex::search / search_parallel (brute_force.rs:162-214). */
int fdb_bf_search(fdb_bf* h, const float* query, size_t k, uint64_t* ids, float* dists,
                  size_t* n_out);
/* BruteForceIndex::batch_search (brute_force.rs:220-225). */
int fdb_bf_batch_search(fdb_bf* h, const float* queries, size_t nq, size_t k, uint64_t* ids,
                        float* dists, uint32_t* counts, fdb_stats* stats);
int fdb_bf_batch_search_device(fdb_bf* h, const float* d_queries, size_t nq, size_t k,
                               uint64_t* d_ids, float* d_dists, uint32_t* d_counts,
                               fdb_stats* stats);
int fdb_bf_free(fdb_bf* h);
/* MutableVectorIndex::remove (brute_force.rs:267-274): swap-remove the first
 * row with this id; *removed = 1 if one was found. */
int fdb_bf_remove(fdb_bf* h, uint64_t id, int* removed);

/* ---- .fdb files (src/persistence/mod.rs, format.rs) --------------------- */
/* A 24-byte header (magic "FORGEDB\0", version u32 = 1, index type u32,
 * flags u32, CRC-32 of the payload u32; format.rs:76-133) and the payload:
 * for IVF-PQ the bincode-1.3 encoding of SerializableIVFPQ (ivf_pq.rs:197-262,
 * 1894-1914), for brute force [metric u8][n u64][dim u64][ids][rows]
 * (brute_force.rs:277-318).  Files are interchangeable with the reference's
 * save()/load() (Persistable, ivf_pq.rs:1970-1994).  Saving an IVF-PQ index
 * writes its tombstoned rows and no tombstones, as the reference does; the
 * original-vector store is written in insertion order (the reference writes
 * hash-map order).  A sharded index cannot be saved. */
#define FDB_INDEX_IVFPQ 1
#define FDB_INDEX_HNSW 2
#define FDB_INDEX_IVF 3
#define FDB_INDEX_BRUTE_FORCE 4
int fdb_ivfpq_save(fdb_ivfpq* h, const char* path);
/* load / load_mmap: checks the header (magic, version <= 1, type) and the
 * CRC, then rebuilds the index on ctx's device. */
int fdb_ivfpq_load(fdb_ctx* ctx, const char* path, fdb_ivfpq** out);
int fdb_bf_save(fdb_bf* h, const char* path);
int fdb_bf_load(fdb_ctx* ctx, const char* path, fdb_bf** out);
/* Host only (no device): header fields and, for IVF-PQ and brute-force
 * files, the shape of the payload.  Checks what load() checks. */
typedef struct fdb_file_info {
    uint32_t version, index_type, flags, checksum;
    uint64_t n;              /* vectors (rows incl. tombstoned ones for IVF-PQ) */
    uint64_t dim;
    uint64_t nlist, m;       /* IVF-PQ */
    uint64_t nprobe;         /* IVF-PQ */
    int32_t metric;          /* FDB_METRIC_* */
    int32_t has_rerank;      /* IVF-PQ: original vectors present */
    uint64_t n_rerank, rerank_factor;
} fdb_file_info;
int fdb_file_inspect(const char* path, fdb_file_info* info);
/* crc32fast::hash: CRC-32/ISO-HDLC of n bytes (the header's checksum). */
uint32_t fdb_crc32(const void* data, size_t n);

#ifdef __cplusplus
}
#endif

#endif /* FORGEGPU_H */
