// fdb_kernels.h -- launchers of the search kernels (host-callable).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace fdb {

struct ScanParams {
    const float* Q;
    int nq;
    int dim;
    int m;
    const float* cents;
    const float* cb;
    const uint64_t* offs;  // list l spans rows [offs[l], ends[l])
    const uint64_t* ends;
    const uint8_t* codes;
    const uint32_t* probes;
    int nprobe;
    int k;
    uint64_t* out_keys;
    unsigned long long* stat;  // [0] lists scanned, [1] codes scanned (nullable)
    const uint32_t* qidx;      // nullable: block i scans query qidx[i] (and writes its row)
    const float* btab;         // non-null selects table mode: [nlist][m][256]
    // nullable, with qidx: block i scans only the lists probe_list[i][0 .. probe_cnt[i])
    // (row stride nprobe; probe_cnt nullable: every row holds nprobe lists) and,
    // with seed, starts from the k keys already in its output row (which must
    // not repeat codes of those lists)
    const uint32_t* probe_list;
    const uint32_t* probe_cnt;
    bool seed;
    // with qidx: block i writes its k keys to out_keys[i] instead of out_keys[qidx[i]]
    bool out_by_block;
    // nullable bitmap over rows: set bits are skipped (tombstones, filters)
    const uint32_t* skip;
    // nullable: the number of queries (blocks of work) is *nq_dev - nq_dev_base,
    // read on the device (clamped to [0, nq]); grid_cap > 0 caps the grid
    const uint32_t* nq_dev;
    uint32_t nq_dev_base;
    int grid_cap;
};

struct RescoreParams {
    const float* Q;
    int nq;
    int dim;
    int m;
    const float* cents;
    const float* cb;
    const uint64_t* offs_full;  // [nlist+1] offsets of the unsharded layout
    int nlist;
    const uint8_t* codes;
    const uint64_t* approx;  // [nq][kp] table-mode shortlist, ascending
    int kp;
    int k;
    uint64_t* out_keys;       // [nq][k] exact keys
    const float* cmax;        // [m] max_l ||c_ls||
    const float* bmax;        // [m] max_j ||b_sj||
    uint32_t* flag_count;     // queries that failed certification
    uint32_t* flag_list;
};

// ivfpq_kernels.cu
void launch_coarse_dist(cudaStream_t s, const float* Q, int nq, int dim, const float* cents,
                        int nlist, float* D);
// probes[q][j] = the j-th nearest list of query q (ascending (distance, list));
// pdist (nullable) receives the distances.
void launch_select(cudaStream_t s, const float* D, int nq, int nlist, int take,
                   uint32_t* probes, float* pdist = nullptr);
// Register-tiled coarse distances (bit-identical to launch_coarse_dist) for
// dim <= 256 from transposed, zero-padded operands: QT [dim][nq_pad] with
// nq_pad a multiple of 32, CT [dim][nlist_pad] with nlist_pad a multiple of 128.
constexpr int COARSE_TILED_MAX_DIM = 256;
void launch_transpose_pad(cudaStream_t s, const float* x, int n, int dim, int npad, float* out);
void launch_coarse_tiled(cudaStream_t s, const float* QT, int nq, int nq_pad, int dim,
                         const float* CT, int nlist, int nlist_pad, float* D);
void launch_scan(cudaStream_t s, const ScanParams& a, int order);
void launch_rescore(cudaStream_t s, const RescoreParams& r, int order);
void launch_ivf_tables(cudaStream_t s, const float* cents, const float* cb, int nlist, int m,
                       int dim, float* btab);
void launch_merge_lists(cudaStream_t s, const uint64_t* lists, int nlists, size_t list_stride,
                        size_t nq, int k, uint64_t* out);
void launch_lookup_gathered(cudaStream_t s, const uint64_t* keys, const uint64_t* gkeys,
                            const uint64_t* gids, int world, size_t list_stride, size_t nq, int k,
                            uint64_t* ids);
void launch_keys_to_ids(cudaStream_t s, const uint64_t* keys, size_t total,
                        const uint64_t* row_ids, uint64_t tag_base, uint64_t* ids);
void launch_finalize(cudaStream_t s, const uint64_t* keys, const uint64_t* ids_in, size_t nq,
                     int k, uint64_t* ids, float* dists, uint32_t* counts);

// bf_kernels.cu
void launch_row_norms(cudaStream_t s, const float* x, size_t n, int dim, float* norms);
// Exact brute-force scan: partial top-k per (row chunk, query) into
// part[nchunks][nq][k]; returns nchunks.
int launch_bf_scan(cudaStream_t s, int metric, const float* Q, int nq, const float* qnorm,
                   const float* X, size_t n, int dim, const float* xnorm, uint64_t tag_base,
                   int k, int sm_count, uint64_t* part, size_t part_capacity);
size_t bf_part_size(size_t n, int nq, int k, int sm_count);

// gemm_topk.cu: fp32 -> fp16 copies with zero padding to kpad columns.
void launch_to_half(cudaStream_t s, const float* x, size_t n, int dim, int kpad, __half* out);

}  // namespace fdb
