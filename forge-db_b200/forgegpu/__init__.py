"""forgegpu -- Python binding of the B200 engine's C ABI (include/forgegpu.h).

The classes mirror the reference crate's Rust API (HueCodes/forge-db) so that
code written against it reads the same:

    IVFPQIndex.build(vectors, n_clusters, n_subvectors, metric)   ivf_pq.rs:374
    index.set_nprobe(n); index.search(q, k); index.batch_search(Q, k)
    BruteForceIndex(metric).add(...); .search(q, k); .batch_search(Q, k)
    KMeans(k, max_iters).fit(data)                                   kmeans.rs:33-193
    ProductQuantizer.train(x, m) / .encode(x) / .build_lookup_table_flat(q)

Every call runs on the GPU through libforgegpu.so.  There is no CPU fallback:
if the library is missing or no B200 is visible, calls raise ForgeGpuError.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libforgegpu.so")

OK = 0
ERRORS = {
    -1: "InvalidParameter", -2: "DimensionMismatch", -3: "EmptyTrainingSet",
    -4: "DimensionNotDivisible", -5: "InsufficientVectors", -6: "Timeout", -7: "Cuda",
    -8: "Nccl", -9: "MemoryLimitExceeded", -10: "EmptyVectorSet", -11: "NotSupported",
    -12: "Io", -13: "SerializationError", -14: "ChecksumMismatch", -15: "InvalidFormat",
    -16: "InsufficientDiskSpace",
}


class IndexType:
    """src/persistence/format.rs:12-23"""
    IvfPq = 1
    Hnsw = 2
    Ivf = 3
    BruteForce = 4


class DistanceMetric:
    """src/distance/mod.rs:16-33"""
    Euclidean = 0
    EuclideanSquared = 1
    Cosine = 2
    DotProduct = 3
    Manhattan = 4


class ForgeGpuError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code
        self.kind = ERRORS.get(code, str(code))


class Stats(C.Structure):
    _fields_ = [("lists_probed", C.c_uint64), ("codes_scanned", C.c_uint64),
                ("bytes_scanned", C.c_uint64), ("coarse_ms", C.c_double),
                ("scan_ms", C.c_double), ("rescore_ms", C.c_double), ("merge_ms", C.c_double),
                ("total_ms", C.c_double), ("exact_rescans", C.c_uint64),
                ("kernel_ms", C.c_double), ("kernel_scores", C.c_uint64),
                ("extended", C.c_uint64), ("comm_ms", C.c_double * 4)]


class FileInfo(C.Structure):
    _fields_ = [("version", C.c_uint32), ("index_type", C.c_uint32), ("flags", C.c_uint32),
                ("checksum", C.c_uint32), ("n", C.c_uint64), ("dim", C.c_uint64),
                ("nlist", C.c_uint64), ("m", C.c_uint64), ("nprobe", C.c_uint64),
                ("metric", C.c_int32), ("has_rerank", C.c_int32), ("n_rerank", C.c_uint64),
                ("rerank_factor", C.c_uint64)]


class BuilderOpts(C.Structure):
    _fields_ = [("num_clusters", C.c_size_t), ("num_subvectors", C.c_size_t),
                ("metric", C.c_int), ("auto_tune", C.c_int), ("target_memory_mb", C.c_size_t),
                ("target_recall", C.c_float), ("nprobe", C.c_size_t),
                ("rerank_factor", C.c_size_t), ("enable_reranking", C.c_int)]


class TrainOpts(C.Structure):
    _fields_ = [("ivf_sample", C.c_size_t), ("pq_sample", C.c_size_t),
                ("ivf_iters", C.c_size_t), ("pq_iters", C.c_size_t),
                ("ivf_sample_idx", C.c_void_p), ("ivf_init_idx", C.c_void_p),
                ("ivf_kpp_u", C.c_void_p), ("pq_sample_idx", C.c_void_p),
                ("pq_init_idx", C.c_void_p), ("seed", C.c_uint64)]


_vp = C.c_void_p
_sz = C.c_size_t
_SIGS = {
    "fdb_last_error": (C.c_char_p, []),
    "fdb_version": (C.c_int, []),
    "fdb_ctx_create": (C.c_int, [C.c_int, C.POINTER(_vp)]),
    "fdb_ctx_free": (C.c_int, [_vp]),
    "fdb_ctx_stream": (C.c_int, [_vp, C.POINTER(_vp)]),
    "fdb_nccl_unique_id": (C.c_int, [_vp]),
    "fdb_ctx_init_comm": (C.c_int, [_vp, C.c_int, C.c_int, _vp]),
    "fdb_ctx_init_comm_timeout": (C.c_int, [_vp, C.c_int, C.c_int, _vp, C.c_double]),
    "fdb_ctx_set_wait_limit": (C.c_int, [_vp, C.c_double]),
    "fdb_ctx_test_stall_scans": (C.c_int, [_vp, C.c_int]),
    "fdb_host_alloc": (C.c_int, [_sz, C.POINTER(_vp)]),
    "fdb_host_free": (C.c_int, [_vp]),
    "fdb_sample_indices": (C.c_int, [C.c_uint64, _sz, _sz, _vp]),
    "fdb_uniform_draws": (C.c_int, [C.c_uint64, _sz, _vp]),
    "fdb_pairwise_distance": (C.c_int, [_vp, C.c_int, _vp, _vp, _sz, _sz, _vp]),
    "fdb_kmeans_fit": (C.c_int, [_vp, _vp, _sz, _sz, _sz, _sz, _vp, _vp, C.c_uint64, _vp, _vp,
                                 C.POINTER(C.c_int)]),
    "fdb_assign": (C.c_int, [_vp, _vp, _sz, _vp, _sz, _sz, _vp]),
    "fdb_find_nearest_centroids": (C.c_int, [_vp, _vp, _sz, _sz, _vp, _sz, _vp]),
    "fdb_find_nearest_centroids_noalloc": (C.c_int, [_vp, _vp, _sz, _sz, _vp, _sz, _sz, _vp]),
    "fdb_pq_train": (C.c_int, [_vp, _vp, _sz, _sz, _sz, _sz, _vp, C.c_uint64, _vp, _vp]),
    "fdb_pq_encode": (C.c_int, [_vp, _vp, _sz, _sz, _vp, _sz, _vp]),
    "fdb_pq_lookup_tables": (C.c_int, [_vp, _vp, _sz, _sz, _vp, _sz, _vp]),
    "fdb_ivfpq_build": (C.c_int, [_vp, _vp, _vp, _sz, _sz, _sz, _sz, C.c_int,
                                  C.POINTER(TrainOpts), C.POINTER(_vp)]),
    "fdb_ivfpq_from_trained": (C.c_int, [_vp, _vp, _vp, _sz, _sz, _sz, _vp, _vp, _vp, C.c_int,
                                         C.POINTER(_vp)]),
    "fdb_ivfpq_export": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp]),
    "fdb_ivfpq_shard": (C.c_int, [_vp, C.c_int, C.c_int]),
    "fdb_ivfpq_shard_plan": (C.c_int, [_vp, _sz, C.c_int, _vp]),
    "fdb_ivfpq_set_nprobe": (C.c_int, [_vp, _sz]),
    "fdb_ivfpq_set_scan_mode": (C.c_int, [_vp, C.c_int]),
    "fdb_ivfpq_set_graphs": (C.c_int, [_vp, C.c_int]),
    "fdb_ivfpq_set_pass1_quota": (C.c_int, [_vp, _sz, C.c_uint64]),
    "fdb_ivfpq_set_stage_timers": (C.c_int, [_vp, C.c_int]),
    "fdb_ivfpq_get_pass1_quota": (C.c_int, [_vp, _sz, C.POINTER(C.c_int64)]),
    "fdb_ivfpq_nprobe": (_sz, [_vp]),
    "fdb_ivfpq_len": (_sz, [_vp]),
    "fdb_ivfpq_n_partitions": (_sz, [_vp]),
    "fdb_ivfpq_dim": (_sz, [_vp]),
    "fdb_ivfpq_n_subvectors": (_sz, [_vp]),
    "fdb_ivfpq_search": (C.c_int, [_vp, _vp, _sz, _vp, _vp, C.POINTER(_sz)]),
    "fdb_ivfpq_batch_search": (C.c_int, [_vp, _vp, _sz, _sz, _vp, _vp, _vp, C.POINTER(Stats)]),
    "fdb_ivfpq_batch_search_device": (C.c_int, [_vp, _vp, _sz, _sz, _vp, _vp, _vp,
                                                C.POINTER(Stats)]),
    "fdb_ivfpq_search_with_timeout": (C.c_int, [_vp, _vp, _sz, C.c_double, _vp, _vp,
                                                C.POINTER(_sz), C.POINTER(C.c_double)]),
    "fdb_ivfpq_batch_search_with_timeout": (C.c_int, [_vp, _vp, _sz, _sz, C.c_double, _vp, _vp,
                                                      _vp, C.POINTER(C.c_double)]),
    "fdb_ivfpq_free": (C.c_int, [_vp]),
    "fdb_bf_create": (C.c_int, [_vp, C.c_int, _vp, _vp, _sz, _sz, C.POINTER(_vp)]),
    "fdb_bf_add": (C.c_int, [_vp, _vp, _vp, _sz, _sz]),
    "fdb_bf_shard": (C.c_int, [_vp, C.c_int, C.c_int]),
    "fdb_bf_set_scan_mode": (C.c_int, [_vp, C.c_int]),
    "fdb_bf_len": (_sz, [_vp]),
    "fdb_bf_dimension": (_sz, [_vp]),
    "fdb_bf_search": (C.c_int, [_vp, _vp, _sz, _vp, _vp, C.POINTER(_sz)]),
    "fdb_bf_batch_search": (C.c_int, [_vp, _vp, _sz, _sz, _vp, _vp, _vp, C.POINTER(Stats)]),
    "fdb_bf_batch_search_device": (C.c_int, [_vp, _vp, _sz, _sz, _vp, _vp, _vp,
                                             C.POINTER(Stats)]),
    "fdb_bf_free": (C.c_int, [_vp]),
    "fdb_bf_remove": (C.c_int, [_vp, C.c_uint64, C.POINTER(C.c_int)]),
    "fdb_ivfpq_enable_reranking": (C.c_int, [_vp, _vp, _vp, _sz, _sz, _sz]),
    "fdb_ivfpq_search_filtered": (C.c_int, [_vp, _vp, _sz, _vp, _sz, _vp, _vp, C.POINTER(_sz)]),
    "fdb_ivfpq_batch_search_filtered": (C.c_int, [_vp, _vp, _sz, _sz, _vp, _sz, _vp, _vp, _vp]),
    "fdb_ivfpq_batch_search_filtered_device": (C.c_int, [_vp, _vp, _sz, _sz, _vp, _sz, _vp, _vp,
                                                         _vp, C.POINTER(Stats)]),
    "fdb_ivfpq_insert_batch": (C.c_int, [_vp, _vp, _vp, _sz, _sz]),
    "fdb_ivfpq_delete": (C.c_int, [_vp, C.c_uint64, C.POINTER(C.c_int)]),
    "fdb_ivfpq_num_tombstones": (_sz, [_vp]),
    "fdb_ivfpq_len_with_tombstones": (_sz, [_vp]),
    "fdb_ivfpq_fragmentation_ratio": (C.c_float, [_vp]),
    "fdb_ivfpq_compact": (C.c_int, [_vp]),
    "fdb_ivfpq_rebuild": (C.c_int, [_vp, C.POINTER(TrainOpts)]),
    "fdb_ivfpq_save": (C.c_int, [_vp, C.c_char_p]),
    "fdb_ivfpq_load": (C.c_int, [_vp, C.c_char_p, C.POINTER(_vp)]),
    "fdb_bf_save": (C.c_int, [_vp, C.c_char_p]),
    "fdb_bf_load": (C.c_int, [_vp, C.c_char_p, C.POINTER(_vp)]),
    "fdb_file_inspect": (C.c_int, [C.c_char_p, C.POINTER(FileInfo)]),
    "fdb_crc32": (C.c_uint32, [_vp, _sz]),
    "fdb_builder_defaults": (None, [C.POINTER(BuilderOpts)]),
    "fdb_builder_plan": (C.c_int, [C.POINTER(BuilderOpts), _sz, _sz, C.POINTER(_sz),
                                   C.POINTER(_sz), C.POINTER(_sz), C.POINTER(_sz)]),
    "fdb_builder_build": (C.c_int, [_vp, C.POINTER(BuilderOpts), _vp, _vp, _sz, _sz,
                                    C.POINTER(TrainOpts), C.POINTER(_vp)]),
}

_lib = None
_lock = threading.Lock()


def lib():
    """Load libforgegpu.so (raises if it was not built)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ForgeGpuError(-11, f"{LIB_PATH} is missing: build it with "
                                         "`python forge-db_b200/build.py`")
            L = C.CDLL(LIB_PATH)
            for name, (res, args) in _SIGS.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def exported_symbols():
    return list(_SIGS)


def _check(rc: int):
    if rc != OK:
        raise ForgeGpuError(rc, lib().fdb_last_error().decode(errors="replace"))


def _p(a):
    return None if a is None else C.c_void_p(a.ctypes.data)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


# ---------------------------------------------------------------------------
# context
# ---------------------------------------------------------------------------
class Context:
    """One device, one stream (and, for sharded indexes, one communicator)."""

    def __init__(self, device: int = 0):
        h = C.c_void_p()
        _check(lib().fdb_ctx_create(device, C.byref(h)))
        self.h = h
        self.device = device

    def stream(self) -> int:
        s = C.c_void_p()
        _check(lib().fdb_ctx_stream(self.h, C.byref(s)))
        return s.value or 0

    def init_comm(self, rank: int, world: int, nccl_id: bytes, timeout_s: float = 300.0):
        """The NCCL communicator of a sharded index; FDB_ERR_TIMEOUT (and no
        communicator) if not every rank joins within timeout_s."""
        buf = C.create_string_buffer(bytes(nccl_id), 128)
        _check(lib().fdb_ctx_init_comm_timeout(self.h, rank, world, buf, float(timeout_s)))

    def set_wait_limit(self, seconds: float):
        """Limit of each bounded wait inside the tensor-core kernels."""
        _check(lib().fdb_ctx_set_wait_limit(self.h, float(seconds)))

    def test_stall_scans(self, count: int):
        """Test hook: the next `count` list-scan launches issue no work, so
        their bounded waits run out (the call returns FDB_ERR_TIMEOUT)."""
        _check(lib().fdb_ctx_test_stall_scans(self.h, int(count)))

    def close(self):
        if self.h:
            _check(lib().fdb_ctx_free(self.h))
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def nccl_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    _check(lib().fdb_nccl_unique_id(buf))
    return buf.raw


_default_ctx = None


def default_context() -> Context:
    global _default_ctx
    if _default_ctx is None:
        _default_ctx = Context(0)
    return _default_ctx


def sample_indices(seed: int, n: int, take: int) -> np.ndarray:
    out = np.empty(take, np.uint32)
    _check(lib().fdb_sample_indices(seed, n, take, _p(out)))
    return out


def uniform_draws(seed: int, count: int) -> np.ndarray:
    out = np.empty(count, np.float32)
    _check(lib().fdb_uniform_draws(seed, count, _p(out)))
    return out


def crc32(data: bytes) -> int:
    """crc32fast::hash, the .fdb header's checksum (host only)."""
    buf = C.create_string_buffer(bytes(data), max(len(data), 1))
    return lib().fdb_crc32(buf, len(data))


def inspect_file(path) -> FileInfo:
    """Header and payload shape of a .fdb file (host only; checks what load does)."""
    info = FileInfo()
    _check(lib().fdb_file_inspect(os.fsencode(path), C.byref(info)))
    return info


def shard_plan(sizes, world: int) -> np.ndarray:
    sizes = np.ascontiguousarray(sizes, np.uint64)
    owner = np.empty(sizes.size, np.int32)
    _check(lib().fdb_ivfpq_shard_plan(_p(sizes), sizes.size, world, _p(owner)))
    return owner


def pairwise_distance(metric: int, a, b, ctx: Context | None = None) -> np.ndarray:
    ctx = ctx or default_context()
    a, b = _f32(a), _f32(b)
    out = np.empty(a.shape[0], np.float32)
    _check(lib().fdb_pairwise_distance(ctx.h, metric, _p(a), _p(b), a.shape[0], a.shape[1],
                                       _p(out)))
    return out


def assign(x, centroids, ctx: Context | None = None) -> np.ndarray:
    ctx = ctx or default_context()
    x, c = _f32(x), _f32(centroids)
    out = np.empty(x.shape[0], np.uint32)
    _check(lib().fdb_assign(ctx.h, _p(x), x.shape[0], _p(c), c.shape[0], x.shape[1], _p(out)))
    return out


# ---------------------------------------------------------------------------
# KMeans / ProductQuantizer
# ---------------------------------------------------------------------------
class KMeans:
    """KMeans::new(k, max_iters) (src/kmeans.rs:33-39)."""

    def __init__(self, k: int, max_iters: int, ctx: Context | None = None):
        self.k, self.max_iters = k, max_iters
        self.ctx = ctx or default_context()
        self.centroids = None
        self.iters = 0
        self.assignments = None

    def fit(self, data, init_idx=None, kpp_u=None, seed: int = 0):
        """fit / fit_raw (kmeans.rs:45-193); draws injected or from `seed`."""
        x = _f32(data)
        n, dim = x.shape
        cents = np.empty((self.k, dim), np.float32)
        assign_out = np.empty(n, np.uint32)
        it = C.c_int(0)
        ii = None if init_idx is None else np.ascontiguousarray(init_idx, np.uint32)
        uu = None if kpp_u is None else _f32(kpp_u)
        _check(lib().fdb_kmeans_fit(self.ctx.h, _p(x), n, dim, self.k, self.max_iters, _p(ii),
                                    _p(uu), seed, _p(cents), _p(assign_out), C.byref(it)))
        self.centroids, self.iters, self.assignments = cents, it.value, assign_out
        return self

    fit_raw = fit

    def find_nearest_centroids(self, query, k: int) -> np.ndarray:
        q = _f32(query)
        out = np.empty(min(k, self.k), np.uint32)
        _check(lib().fdb_find_nearest_centroids(self.ctx.h, _p(self.centroids), self.k,
                                                q.size, _p(q), k, _p(out)))
        return out


class ProductQuantizer:
    """ProductQuantizer (src/pq.rs:33-245)."""

    def __init__(self, codebooks, ctx: Context | None = None):
        self.codebooks = _f32(codebooks)
        self.n_subvectors, _, self.subvector_dim = self.codebooks.shape
        self.dim = self.n_subvectors * self.subvector_dim
        self.ctx = ctx or default_context()
        self.iters = None

    @classmethod
    def try_train(cls, vectors, n_subvectors: int, init_idx=None, seed: int = 0, iters: int = 25,
                  ctx: Context | None = None):
        ctx = ctx or default_context()
        x = _f32(vectors)
        n, dim = (x.shape if x.ndim == 2 else (0, 0))
        cb = np.empty((n_subvectors, 256, dim // max(n_subvectors, 1) if n_subvectors else 0),
                      np.float32)
        its = np.empty(max(n_subvectors, 1), np.int32)
        ii = None if init_idx is None else np.ascontiguousarray(init_idx, np.uint32)
        _check(lib().fdb_pq_train(ctx.h, _p(x) if n else None, n, dim, n_subvectors, iters,
                                  _p(ii), seed, _p(cb), _p(its)))
        pq = cls(cb, ctx)
        pq.iters = its
        return pq

    train = try_train

    def encode(self, vectors) -> np.ndarray:
        x = _f32(vectors)
        if x.ndim == 1:
            x = x[None]
        out = np.empty((x.shape[0], self.n_subvectors), np.uint8)
        _check(lib().fdb_pq_encode(self.ctx.h, _p(self.codebooks), self.n_subvectors, x.shape[1],
                                   _p(x), x.shape[0], _p(out)))
        return out

    def build_lookup_table_flat(self, queries) -> np.ndarray:
        q = _f32(queries)
        single = q.ndim == 1
        if single:
            q = q[None]
        out = np.empty((q.shape[0], self.n_subvectors * 256), np.float32)
        _check(lib().fdb_pq_lookup_tables(self.ctx.h, _p(self.codebooks), self.n_subvectors,
                                          q.shape[1], _p(q), q.shape[0], _p(out)))
        return out[0] if single else out


# ---------------------------------------------------------------------------
# indexes
# ---------------------------------------------------------------------------
def _train_opts(seed=0, ivf_sample=0, pq_sample=0, ivf_iters=0, pq_iters=0, ivf_sample_idx=None,
                ivf_init_idx=None, ivf_kpp_u=None, pq_sample_idx=None, pq_init_idx=None):
    keep = []

    def arr(a, dt):
        if a is None:
            return None
        a = np.ascontiguousarray(a, dt)
        keep.append(a)
        return a.ctypes.data

    o = TrainOpts(ivf_sample, pq_sample, ivf_iters, pq_iters,
                  arr(ivf_sample_idx, np.uint32), arr(ivf_init_idx, np.uint32),
                  arr(ivf_kpp_u, np.float32), arr(pq_sample_idx, np.uint32),
                  arr(pq_init_idx, np.uint32), seed)
    if ivf_sample_idx is not None:
        o.ivf_sample = len(ivf_sample_idx)
    if pq_sample_idx is not None:
        o.pq_sample = len(pq_sample_idx)
    return o, keep


def _results(ids, dists, counts):
    return [list(zip(ids[i, :counts[i]].tolist(), dists[i, :counts[i]].tolist()))
            for i in range(ids.shape[0])]


class IVFPQIndex:
    """IVFPQIndex (src/index/ivf_pq.rs:343-1084) on one B200."""

    def __init__(self, handle, ctx: Context):
        self.h = handle
        self.ctx = ctx

    @classmethod
    def build(cls, vectors, n_clusters: int, n_subvectors: int,
              metric: int = DistanceMetric.Euclidean, ids=None, ctx: Context | None = None,
              seed: int = 0, ivf_sample=0, pq_sample=0, ivf_iters=0, pq_iters=0,
              ivf_sample_idx=None, ivf_init_idx=None, ivf_kpp_u=None, pq_sample_idx=None,
              pq_init_idx=None):
        ctx = ctx or default_context()
        x = _f32(vectors)
        n, dim = x.shape
        o, keep = _train_opts(seed, ivf_sample, pq_sample, ivf_iters, pq_iters, ivf_sample_idx,
                              ivf_init_idx, ivf_kpp_u, pq_sample_idx, pq_init_idx)
        idv = None if ids is None else np.ascontiguousarray(ids, np.uint64)
        h = C.c_void_p()
        _check(lib().fdb_ivfpq_build(ctx.h, _p(x), _p(idv), n, dim, n_clusters, n_subvectors,
                                     metric, C.byref(o), C.byref(h)))
        return cls(h, ctx)

    @classmethod
    def from_trained(cls, centroids, codebooks, offsets, ids, codes,
                     metric: int = DistanceMetric.Euclidean, ctx: Context | None = None):
        ctx = ctx or default_context()
        cents = _f32(centroids)
        cb = _f32(codebooks)
        offs = np.ascontiguousarray(offsets, np.uint64)
        idv = np.ascontiguousarray(ids, np.uint64)
        codes = np.ascontiguousarray(codes, np.uint8)
        nlist, dim = cents.shape
        m = cb.shape[0]
        h = C.c_void_p()
        _check(lib().fdb_ivfpq_from_trained(ctx.h, _p(cents), _p(cb), nlist, m, dim, _p(offs),
                                            _p(idv), _p(codes), metric, C.byref(h)))
        return cls(h, ctx)

    def export(self):
        nlist, dim = self.n_partitions(), self.dim()
        offs = np.empty(nlist + 1, np.uint64)
        _check(lib().fdb_ivfpq_export(self.h, None, None, _p(offs), None, None))
        n = int(offs[-1])
        cents = np.empty((nlist, dim), np.float32)
        m = self.n_subvectors()
        cb = np.empty((m, 256, dim // m), np.float32)
        ids = np.empty(n, np.uint64)
        codes = np.empty((n, m), np.uint8)
        _check(lib().fdb_ivfpq_export(self.h, _p(cents), _p(cb), None, _p(ids), _p(codes)))
        return cents, cb, offs, ids, codes

    def shard(self, rank: int, world: int):
        _check(lib().fdb_ivfpq_shard(self.h, rank, world))

    SCAN_AUTO, SCAN_EXACT, SCAN_TABLES, SCAN_TENSOR = 0, 1, 2, 3

    def set_nprobe(self, nprobe: int):
        _check(lib().fdb_ivfpq_set_nprobe(self.h, nprobe))

    def set_scan_mode(self, mode: int):
        _check(lib().fdb_ivfpq_set_scan_mode(self.h, mode))

    def set_pass1_quota(self, nprobe: int, div: int):
        """The tensor path's pass-1 sampling quota (1/div of the probed codes,
        0: every probe's first tile) for batches with `nprobe` probes."""
        _check(lib().fdb_ivfpq_set_pass1_quota(self.h, int(nprobe), int(div)))

    def pass1_quota(self, nprobe: int):
        """The pass-1 quota in use for `nprobe` probes, None before the first
        large tensor-path batch calibrates it."""
        v = C.c_int64()
        _check(lib().fdb_ivfpq_get_pass1_quota(self.h, int(nprobe), C.byref(v)))
        return None if v.value < 0 else v.value

    def set_stage_timers(self, enable: bool):
        """Fill fdb_stats' stage times (on by default); off, statistics keep
        the counters and the list scan's pass-2 time only."""
        _check(lib().fdb_ivfpq_set_stage_timers(self.h, 1 if enable else 0))

    def set_graphs(self, enable: bool):
        """Replay repeated same-shape batch searches as CUDA graphs."""
        _check(lib().fdb_ivfpq_set_graphs(self.h, int(bool(enable))))

    def nprobe(self) -> int:
        return lib().fdb_ivfpq_nprobe(self.h)

    def len(self) -> int:
        return lib().fdb_ivfpq_len(self.h)

    __len__ = len

    def n_partitions(self) -> int:
        return lib().fdb_ivfpq_n_partitions(self.h)

    def dim(self) -> int:
        return lib().fdb_ivfpq_dim(self.h)

    def n_subvectors(self) -> int:
        return lib().fdb_ivfpq_n_subvectors(self.h)

    def search(self, query, k: int):
        q = _f32(query)
        ids = np.empty(max(k, 1), np.uint64)
        d = np.empty(max(k, 1), np.float32)
        n = C.c_size_t(0)
        _check(lib().fdb_ivfpq_search(self.h, _p(q), k, _p(ids), _p(d), C.byref(n)))
        return list(zip(ids[:n.value].tolist(), d[:n.value].tolist()))

    def batch_search_arrays(self, queries, k: int, stats: bool = False):
        Q = _f32(queries)
        nq = Q.shape[0] if Q.ndim == 2 else 0
        ids = np.empty((nq, k), np.uint64)
        d = np.empty((nq, k), np.float32)
        cnt = np.empty(nq, np.uint32)
        st = Stats()
        _check(lib().fdb_ivfpq_batch_search(self.h, _p(Q) if nq else None, nq, k, _p(ids), _p(d),
                                            _p(cnt), C.byref(st) if stats else None))
        return (ids, d, cnt, st) if stats else (ids, d, cnt)

    def batch_search(self, queries, k: int):
        ids, d, cnt = self.batch_search_arrays(queries, k)
        return _results(ids, d, cnt)

    batch_search_parallel = batch_search

    def search_with_timeout(self, query, k: int, timeout_s: float):
        """search_with_timeout (ivf_pq.rs:1369-1455): (results, elapsed
        seconds), or ForgeGpuError kind "Timeout" past the deadline."""
        q = _f32(query)
        ids = np.empty(max(k, 1), np.uint64)
        d = np.empty(max(k, 1), np.float32)
        n = C.c_size_t(0)
        el = C.c_double(0.0)
        _check(lib().fdb_ivfpq_search_with_timeout(self.h, _p(q), k, float(timeout_s), _p(ids),
                                                   _p(d), C.byref(n), C.byref(el)))
        return list(zip(ids[:n.value].tolist(), d[:n.value].tolist())), el.value

    def batch_search_with_timeout_arrays(self, queries, k: int, timeout_s: float):
        """batch_search under one deadline: (ids, dists, counts, elapsed)."""
        Q = _f32(queries)
        nq = Q.shape[0]
        ids = np.empty((nq, k), np.uint64)
        d = np.empty((nq, k), np.float32)
        cnt = np.empty(nq, np.uint32)
        el = C.c_double(0.0)
        _check(lib().fdb_ivfpq_batch_search_with_timeout(self.h, _p(Q), nq, k, float(timeout_s),
                                                         _p(ids), _p(d), _p(cnt),
                                                         C.byref(el)))
        return ids, d, cnt, el.value

    # --- re-ranking, filters, updates (ivf_pq.rs:513-831, 1731-1890) ---
    def enable_reranking(self, vectors, ids, rerank_factor: int):
        x = _f32(vectors)
        idv = np.ascontiguousarray(ids, np.uint64)
        n = x.shape[0] if x.ndim == 2 else 0
        _check(lib().fdb_ivfpq_enable_reranking(self.h, _p(x) if n else None,
                                                _p(idv) if n else None, n,
                                                x.shape[1] if n else self.dim(), rerank_factor))

    def search_filtered(self, query, k: int, allowed_ids):
        """search_filtered with the matching ids of the metadata filter."""
        q = _f32(query)
        al = np.ascontiguousarray(allowed_ids, np.uint64)
        ids = np.empty(max(k, 1), np.uint64)
        d = np.empty(max(k, 1), np.float32)
        n = C.c_size_t(0)
        _check(lib().fdb_ivfpq_search_filtered(self.h, _p(q), k, _p(al) if al.size else None,
                                               al.size, _p(ids), _p(d), C.byref(n)))
        return list(zip(ids[:n.value].tolist(), d[:n.value].tolist()))

    def batch_search_filtered_arrays(self, queries, k: int, allowed_ids):
        Q = _f32(queries)
        nq = Q.shape[0]
        al = np.ascontiguousarray(allowed_ids, np.uint64)
        ids = np.empty((nq, k), np.uint64)
        d = np.empty((nq, k), np.float32)
        cnt = np.empty(nq, np.uint32)
        _check(lib().fdb_ivfpq_batch_search_filtered(self.h, _p(Q), nq, k,
                                                     _p(al) if al.size else None, al.size,
                                                     _p(ids), _p(d), _p(cnt)))
        return ids, d, cnt

    def insert_batch(self, vectors, ids):
        x = _f32(vectors)
        if x.ndim == 1:
            x = x[None]
        idv = np.ascontiguousarray(np.atleast_1d(ids), np.uint64)
        _check(lib().fdb_ivfpq_insert_batch(self.h, _p(x), _p(idv), x.shape[0], x.shape[1]))

    def delete(self, id_: int) -> bool:
        out = C.c_int(0)
        _check(lib().fdb_ivfpq_delete(self.h, int(id_), C.byref(out)))
        return bool(out.value)

    def num_tombstones(self) -> int:
        return lib().fdb_ivfpq_num_tombstones(self.h)

    def len_with_tombstones(self) -> int:
        return lib().fdb_ivfpq_len_with_tombstones(self.h)

    def fragmentation_ratio(self) -> float:
        return lib().fdb_ivfpq_fragmentation_ratio(self.h)

    def is_empty(self) -> bool:
        return self.len() == 0

    def compact(self):
        _check(lib().fdb_ivfpq_compact(self.h))

    def rebuild(self, seed: int = 0, **draws):
        o, keep = _train_opts(seed, **draws)
        _check(lib().fdb_ivfpq_rebuild(self.h, C.byref(o)))

    # --- Persistable (src/persistence/mod.rs:34-73) ---
    def save(self, path):
        _check(lib().fdb_ivfpq_save(self.h, os.fsencode(path)))

    @classmethod
    def load(cls, path, ctx: Context | None = None):
        ctx = ctx or default_context()
        h = C.c_void_p()
        _check(lib().fdb_ivfpq_load(ctx.h, os.fsencode(path), C.byref(h)))
        return cls(h, ctx)

    load_mmap = load

    def close(self):
        if self.h:
            _check(lib().fdb_ivfpq_free(self.h))
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class IVFPQIndexBuilder:
    """IVFPQIndexBuilder (src/index/ivf_pq_builder.rs:56-331): fluent setters,
    auto-tuned parameters, build() on the GPU."""

    def __init__(self):
        self.o = BuilderOpts()
        lib().fdb_builder_defaults(C.byref(self.o))
        self._vectors = None
        self._ids = None

    def vectors(self, vectors, ids=None):
        self._vectors = _f32(vectors)
        self._ids = None if ids is None else np.ascontiguousarray(ids, np.uint64)
        return self

    def num_clusters(self, n):
        self.o.num_clusters = n
        return self

    def num_subvectors(self, m):
        self.o.num_subvectors = m
        return self

    def metric(self, metric):
        self.o.metric = metric
        return self

    def auto_tune(self, enable: bool):
        self.o.auto_tune = int(bool(enable))
        return self

    def target_memory_mb(self, mb):
        self.o.target_memory_mb = mb
        return self

    def target_recall(self, recall):
        self.o.target_recall = min(max(float(recall), 0.0), 1.0)
        return self

    def nprobe(self, nprobe):
        self.o.nprobe = nprobe
        return self

    def rerank_factor(self, factor):
        self.o.rerank_factor = max(int(factor), 1)
        return self

    def enable_reranking(self, enable: bool):
        self.o.enable_reranking = int(bool(enable))
        return self

    def plan(self, n: int, dim: int):
        """(num_clusters, num_subvectors, nprobe, estimated MiB) for n x dim."""
        c, m, p, mb = C.c_size_t(), C.c_size_t(), C.c_size_t(), C.c_size_t()
        _check(lib().fdb_builder_plan(C.byref(self.o), n, dim, C.byref(c), C.byref(m),
                                      C.byref(p), C.byref(mb)))
        return c.value, m.value, p.value, mb.value

    def build(self, ctx: Context | None = None, seed: int = 0, **draws) -> IVFPQIndex:
        x = self._vectors
        n = 0 if x is None else (x.shape[0] if x.ndim == 2 else 0)
        dim = 0 if n == 0 else x.shape[1]
        # the argument checks come before any device work (no context needed)
        ctx = ctx or (default_context() if n else None)
        t, keep = _train_opts(seed, **draws)
        h = C.c_void_p()
        _check(lib().fdb_builder_build(ctx.h if ctx else None, C.byref(self.o),
                                       None if x is None else (_p(x) if n else C.c_void_p(1)),
                                       _p(self._ids), n, dim, C.byref(t), C.byref(h)))
        return IVFPQIndex(h, ctx)


class BruteForceIndex:
    """BruteForceIndex (src/index/brute_force.rs:60-225) on one B200."""

    def __init__(self, metric: int = DistanceMetric.Euclidean, ctx: Context | None = None):
        self.ctx = ctx or default_context()
        h = C.c_void_p()
        _check(lib().fdb_bf_create(self.ctx.h, metric, None, None, 0, 0, C.byref(h)))
        self.h = h
        self.metric = metric

    def add(self, vectors, ids=None):
        x = _f32(vectors)
        if x.ndim == 1:
            x = x[None]
        idv = None if ids is None else np.ascontiguousarray(np.atleast_1d(ids), np.uint64)
        _check(lib().fdb_bf_add(self.h, _p(x), _p(idv), x.shape[0], x.shape[1]))
        return self

    def shard(self, rank: int, world: int):
        _check(lib().fdb_bf_shard(self.h, rank, world))

    def set_scan_mode(self, mode: int):
        _check(lib().fdb_bf_set_scan_mode(self.h, mode))

    def len(self) -> int:
        return lib().fdb_bf_len(self.h)

    __len__ = len

    def dimension(self) -> int:
        return lib().fdb_bf_dimension(self.h)

    def search(self, query, k: int):
        q = _f32(query)
        ids = np.empty(max(k, 1), np.uint64)
        d = np.empty(max(k, 1), np.float32)
        n = C.c_size_t(0)
        _check(lib().fdb_bf_search(self.h, _p(q), k, _p(ids), _p(d), C.byref(n)))
        return list(zip(ids[:n.value].tolist(), d[:n.value].tolist()))

    search_parallel = search

    def batch_search_arrays(self, queries, k: int, stats: bool = False):
        Q = _f32(queries)
        nq = Q.shape[0]
        ids = np.empty((nq, k), np.uint64)
        d = np.empty((nq, k), np.float32)
        cnt = np.empty(nq, np.uint32)
        st = Stats()
        _check(lib().fdb_bf_batch_search(self.h, _p(Q), nq, k, _p(ids), _p(d), _p(cnt),
                                         C.byref(st) if stats else None))
        return (ids, d, cnt, st) if stats else (ids, d, cnt)

    def batch_search(self, queries, k: int):
        ids, d, cnt = self.batch_search_arrays(queries, k)
        return _results(ids, d, cnt)

    def remove(self, id_: int) -> bool:
        out = C.c_int(0)
        _check(lib().fdb_bf_remove(self.h, int(id_), C.byref(out)))
        return bool(out.value)

    def is_empty(self) -> bool:
        return self.len() == 0

    def save(self, path):
        _check(lib().fdb_bf_save(self.h, os.fsencode(path)))

    @classmethod
    def load(cls, path, ctx: Context | None = None):
        ctx = ctx or default_context()
        self = cls.__new__(cls)
        self.ctx = ctx
        h = C.c_void_p()
        _check(lib().fdb_bf_load(ctx.h, os.fsencode(path), C.byref(h)))
        self.h = h
        self.metric = inspect_file(path).metric
        return self

    def close(self):
        if self.h:
            _check(lib().fdb_bf_free(self.h))
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
