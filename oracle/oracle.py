"""ctypes binding of the CPU oracle (fdb_oracle.cpp) -- TEST INFRASTRUCTURE ONLY.

The oracle restates forge-db's search/training arithmetic on the CPU in the
reference's exact summation order.  Only the tests, ``__graft_entry__.smoke``
and the CPU-baseline leg of ``bench.py`` import this module; the CUDA engine
never does.  See fdb_oracle.cpp for the reference file:line of each routine.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "build", "liboracle.so")
_lib = None

EUCLIDEAN, EUCLIDEAN_SQUARED, COSINE, DOT_PRODUCT, MANHATTAN = range(5)

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_u64p = np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_sz = C.c_size_t


def build() -> str:
    """Compile the oracle with its Makefile (g++, AVX2+FMA, no contraction)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        sig = {
            "orc_l2sq": (C.c_float, [_f32p, _f32p, _sz]),
            "orc_dot": (C.c_float, [_f32p, _f32p, _sz]),
            "orc_cosine": (C.c_float, [_f32p, _f32p, _sz]),
            "orc_manhattan": (C.c_float, [_f32p, _f32p, _sz]),
            "orc_metric": (C.c_float, [C.c_int, _f32p, _f32p, _sz]),
            "orc_l2sq_scalar": (C.c_float, [_f32p, _f32p, _sz]),
            "orc_dot_scalar": (C.c_float, [_f32p, _f32p, _sz]),
            "orc_pairwise": (None, [C.c_int, _f32p, _f32p, _sz, _sz, _f32p]),
            "orc_assign": (None, [_f32p, _sz, _f32p, _sz, _sz, _u32p, C.c_int]),
            "orc_find_nearest_centroids": (None, [_f32p, _sz, _sz, _f32p, _sz, _u32p]),
            "orc_kmeans_fit": (C.c_int, [_f32p, _sz, _sz, _sz, _sz, _u32p, _f32p, _f32p,
                                         C.POINTER(C.c_int), C.c_int]),
            "orc_pq_train": (C.c_int, [_f32p, _sz, _sz, _sz, _sz, _u32p, _f32p, _i32p, C.c_int]),
            "orc_pq_encode": (None, [_f32p, _sz, _sz, _f32p, _sz, _u8p, C.c_int]),
            "orc_lut_flat": (None, [_f32p, _sz, _sz, _f32p, _f32p]),
            "orc_adc_fast": (C.c_float, [_f32p, _u8p, _sz]),
            "orc_adc_lane8": (C.c_float, [_f32p, _u8p, _sz]),
            "orc_adc_scalar": (C.c_float, [_f32p, _u8p, _sz]),
            "orc_ivfpq_build": (C.c_int, [_f32p, _u64p, _sz, _sz, _sz, _sz, _u32p, _sz, _u32p,
                                          _f32p, _u32p, _sz, _u32p, _sz, _sz, _f32p, _f32p,
                                          _u32p, _u64p, _u64p, _u8p, C.c_int]),
            "orc_ivfpq_search": (_sz, [_f32p, _f32p, _sz, _sz, _sz, _u64p, _u64p, _u8p, _sz,
                                       _f32p, _sz, _u64p, _f32p]),
            "orc_ivfpq_batch_search": (None, [_f32p, _f32p, _sz, _sz, _sz, _u64p, _u64p, _u8p,
                                              _sz, _f32p, _sz, _sz, _sz, _u64p, _f32p, _u32p,
                                              C.c_int]),
            "orc_ivfpq_search_skip": (_sz, [_f32p, _f32p, _sz, _sz, _sz, _u64p, _u64p, _u8p,
                                            _u8p, _sz, _f32p, _sz, _u64p, _f32p]),
            "orc_ivfpq_batch_search_skip": (None, [_f32p, _f32p, _sz, _sz, _sz, _u64p, _u64p,
                                                   _u8p, _u8p, _sz, _f32p, _sz, _sz, _sz,
                                                   _u64p, _f32p, _u32p, C.c_int]),
            "orc_rerank": (None, [_f32p, _sz, _sz, _u64p, _u32p, _sz, _u64p, _f32p, _sz, _sz,
                                  _u64p, _f32p, _u32p, C.c_int]),
            "orc_bf_batch_search": (None, [_f32p, _u64p, _sz, _sz, C.c_int, _f32p, _sz, _sz,
                                           _u64p, _f32p, _u32p, C.c_int]),
            "orc_max_threads": (C.c_int, []),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _threads(n):
    return int(n) if n else lib().orc_max_threads()


# --- distances --------------------------------------------------------------

def l2sq(a, b):
    a, b = _f32(a), _f32(b)
    return lib().orc_l2sq(a, b, a.size)


def dot(a, b):
    a, b = _f32(a), _f32(b)
    return lib().orc_dot(a, b, a.size)


def cosine(a, b):
    a, b = _f32(a), _f32(b)
    return lib().orc_cosine(a, b, a.size)


def metric(m, a, b):
    a, b = _f32(a), _f32(b)
    return lib().orc_metric(int(m), a, b, a.size)


def pairwise(m, A, B):
    A, B = _f32(A), _f32(B)
    out = np.empty(A.shape[0], np.float32)
    lib().orc_pairwise(int(m), A, B, A.shape[0], A.shape[1], out)
    return out


# --- k-means / PQ -------------------------------------------------------------

def assign(X, cents, threads=0):
    X, cents = _f32(X), _f32(cents)
    out = np.empty(X.shape[0], np.uint32)
    lib().orc_assign(X, X.shape[0], cents, cents.shape[0], X.shape[1], out, _threads(threads))
    return out


def find_nearest_centroids(cents, q, k):
    cents, q = _f32(cents), _f32(q)
    out = np.empty(min(k, cents.shape[0]), np.uint32)
    lib().orc_find_nearest_centroids(cents, cents.shape[0], cents.shape[1], q, k, out)
    return out


def kmeans_fit(X, k, max_iters, init_idx, kpp_u=None, threads=0):
    X = _f32(X)
    n, dim = X.shape
    init_idx = np.ascontiguousarray(init_idx, np.uint32)
    kpp_u = np.zeros(k, np.float32) if kpp_u is None else _f32(kpp_u)
    cents = np.zeros((k, dim), np.float32)
    it = C.c_int(0)
    rc = lib().orc_kmeans_fit(X, n, dim, k, max_iters, init_idx, kpp_u, cents, C.byref(it),
                              _threads(threads))
    if rc != 0:
        raise ValueError(f"oracle kmeans_fit failed: {rc}")
    return cents, it.value


def pq_train(X, m, init_idx, iters=25, threads=0):
    X = _f32(X)
    n, dim = X.shape
    init_idx = np.ascontiguousarray(init_idx, np.uint32)
    cb = np.zeros((m, 256, dim // m), np.float32)
    its = np.zeros(m, np.int32)
    rc = lib().orc_pq_train(X, n, dim, m, iters, init_idx, cb, its, _threads(threads))
    if rc != 0:
        raise ValueError(f"oracle pq_train failed: {rc}")
    return cb, its


def pq_encode(cb, X, threads=0):
    cb, X = _f32(cb), _f32(X)
    m = cb.shape[0]
    out = np.empty((X.shape[0], m), np.uint8)
    lib().orc_pq_encode(cb, m, X.shape[1], X, X.shape[0], out, _threads(threads))
    return out


def lut_flat(cb, q):
    cb, q = _f32(cb), _f32(q)
    m = cb.shape[0]
    out = np.empty(m * 256, np.float32)
    lib().orc_lut_flat(cb, m, q.size, q, out)
    return out


def adc(order, lut, code):
    lut = _f32(lut)
    code = np.ascontiguousarray(code, np.uint8)
    fn = {"fast": lib().orc_adc_fast, "lane8": lib().orc_adc_lane8,
          "scalar": lib().orc_adc_scalar}[order]
    return fn(lut, code, code.size)


# --- indexes ------------------------------------------------------------------

class OracleIVFPQ:
    """Trained IVF-PQ artefacts in list-major layout plus the oracle searches."""

    def __init__(self, centroids, codebooks, offsets, ids, codes):
        self.centroids = _f32(centroids)
        self.codebooks = _f32(codebooks)
        self.offsets = np.ascontiguousarray(offsets, np.uint64)
        self.ids = np.ascontiguousarray(ids, np.uint64)
        self.codes = np.ascontiguousarray(codes, np.uint8)
        self.nlist, self.dim = self.centroids.shape
        self.m = self.codebooks.shape[0]
        self.nprobe = 1

    @classmethod
    def build(cls, X, ids, nlist, m, ivf_sample_idx, ivf_init_idx, ivf_kpp_u, pq_sample_idx,
              pq_init_idx, ivf_iters=25, pq_iters=25, threads=0):
        X = _f32(X)
        n, dim = X.shape
        ids = np.ascontiguousarray(ids, np.uint64)
        ivf_sample_idx = np.ascontiguousarray(ivf_sample_idx, np.uint32)
        ivf_init_idx = np.ascontiguousarray(ivf_init_idx, np.uint32)
        ivf_kpp_u = _f32(ivf_kpp_u if ivf_kpp_u is not None else np.zeros(nlist))
        pq_sample_idx = np.ascontiguousarray(pq_sample_idx, np.uint32)
        pq_init_idx = np.ascontiguousarray(pq_init_idx, np.uint32)
        cents = np.zeros((nlist, dim), np.float32)
        cb = np.zeros((m, 256, dim // m), np.float32)
        assign = np.zeros(n, np.uint32)
        offsets = np.zeros(nlist + 1, np.uint64)
        lids = np.zeros(n, np.uint64)
        codes = np.zeros((n, m), np.uint8)
        rc = lib().orc_ivfpq_build(X, ids, n, dim, nlist, m, ivf_sample_idx, ivf_sample_idx.size,
                                   ivf_init_idx, ivf_kpp_u, pq_sample_idx, pq_sample_idx.size,
                                   pq_init_idx, ivf_iters, pq_iters, cents, cb, assign, offsets,
                                   lids, codes, _threads(threads))
        if rc != 0:
            raise ValueError(f"oracle ivfpq_build failed: {rc}")
        ix = cls(cents, cb, offsets, lids, codes)
        ix.assign = assign
        return ix

    def set_nprobe(self, nprobe):
        self.nprobe = min(int(nprobe), self.nlist)

    def search(self, q, k):
        q = _f32(q)
        ids = np.empty(k, np.uint64)
        d = np.empty(k, np.float32)
        cnt = lib().orc_ivfpq_search(self.centroids, self.codebooks, self.nlist, self.m, self.dim,
                                     self.offsets, self.ids, self.codes, self.nprobe, q, k, ids, d)
        return ids[:cnt], d[:cnt]

    def batch_search(self, Q, k, chunk=0, threads=0):
        Q = _f32(Q)
        nq = Q.shape[0]
        ids = np.empty((nq, k), np.uint64)
        d = np.empty((nq, k), np.float32)
        counts = np.empty(nq, np.uint32)
        lib().orc_ivfpq_batch_search(self.centroids, self.codebooks, self.nlist, self.m, self.dim,
                                     self.offsets, self.ids, self.codes, self.nprobe, Q, nq, k,
                                     chunk, ids, d, counts, _threads(threads))
        return ids, d, counts


def bf_batch_search(X, ids, metric_id, Q, k, threads=0):
    X, Q = _f32(X), _f32(Q)
    ids = np.ascontiguousarray(ids, np.uint64)
    nq = Q.shape[0]
    out_ids = np.empty((nq, k), np.uint64)
    out_d = np.empty((nq, k), np.float32)
    counts = np.empty(nq, np.uint32)
    lib().orc_bf_batch_search(X, ids, X.shape[0], X.shape[1], int(metric_id), Q, nq, k, out_ids,
                              out_d, counts, _threads(threads))
    return out_ids, out_d, counts


def max_threads():
    return lib().orc_max_threads()


def host_threads():
    """Every core this process may run on (OMP_NUM_THREADS, which torchrun
    sets to 1, does not limit the count passed explicitly to the oracle)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# --- the engine's default draws, restated ---------------------------------------
# The reference draws its training samples and initial centroids from
# rand::thread_rng (src/index/ivf_pq.rs:388, 426; src/kmeans.rs:54, 97, 107),
# which no run can reproduce.  The engine replaces it with a documented
# splitmix64 stream; restating that stream here lets the oracle build the very
# index a GPU run builds from the same seed (the draws are inputs to both).

_M64 = (1 << 64) - 1


def _splitmix64(state):
    state = (state + 0x9E3779B97F4A7C15) & _M64
    z = state
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & _M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & _M64
    return state, z ^ (z >> 31)


def splitmix_sample_indices(seed, n, take):
    """Partial Fisher-Yates over 0..n-1 driven by splitmix64: slot i swaps with
    i + floor(r * (n - i) / 2^64).  The first `take` slots are the sample."""
    idx = np.arange(n, dtype=np.uint32)
    st = int(seed) & _M64
    for i in range(int(take)):
        st, r = _splitmix64(st)
        j = i + ((r * (n - i)) >> 64)
        idx[i], idx[j] = idx[j], idx[i]
    return idx[:take].copy()


def splitmix_uniform(seed, count):
    """23 random bits per draw: u = (r >> 41) * 2^-23 in [0, 1)."""
    st = int(seed) & _M64
    out = np.empty(int(count), np.float32)
    for i in range(int(count)):
        st, r = _splitmix64(st)
        out[i] = np.float32(r >> 41) * np.float32(1.0 / 8388608.0)
    return out


def engine_build_draws(seed, n, nlist, m, ivf_sample=30000, pq_sample=100000):
    """The draws an engine build with `seed` and default options takes:
    (ivf_sample_idx, ivf_init_idx, ivf_kpp_u, pq_sample_idx, pq_init_idx).
    Random-sample init for nlist > 64, k-means++ picks and draws otherwise."""
    seed = int(seed)
    ivf_n = min(ivf_sample, n)
    pq_n = min(pq_sample, n)
    sidx = (np.arange(n, dtype=np.uint32) if ivf_n == n
            else splitmix_sample_indices(seed, n, ivf_n))
    kseed = (seed + 1) & _M64
    if nlist > 64:
        init = splitmix_sample_indices(kseed, ivf_n, nlist)
        kpp_u = None
    else:
        st = kseed ^ 0x6B6D65616E737070
        init = np.empty(nlist, np.uint32)
        for c in range(nlist):
            st, r = _splitmix64(st)
            init[c] = (r * ivf_n) >> 64
        kpp_u = splitmix_uniform((kseed + 0x9E37) & _M64, nlist)
    pidx = splitmix_sample_indices((seed + 2) & _M64, n, pq_n)
    pinit = np.concatenate([splitmix_sample_indices((seed + 3 + q) & _M64, pq_n, 256)
                            for q in range(m)]).astype(np.uint32)
    return sidx, init, kpp_u, pidx, pinit


# --- the reference's mutable IVF-PQ state (re-ranking, tombstones, filters) ----

class OracleMutableIVFPQ(OracleIVFPQ):
    """OracleIVFPQ plus the reference's state around the scan, restated in Python:

    - enable_reranking / rerank_results      src/index/ivf_pq.rs:513-517, 556-582
    - delete / len / num_tombstones / compact                     :1786-1852, 1087-1103
    - insert_batch                                                :1731-1773
    - search / batch_search with fetch_k and tombstones          :590-677, 850-1047
    - search_filtered (filter_fetch_k = 4 * fetch_k)             :692-831
    The scan arithmetic is the C restatement (orc_ivfpq_*_skip)."""

    def __init__(self, centroids, codebooks, offsets, ids, codes):
        super().__init__(centroids, codebooks, offsets, ids, codes)
        self.tomb = [set() for _ in range(self.nlist)]
        self.rr = None          # dict id -> vector (HashMap<u64, Vector>)
        self.rerank_factor = 1

    # ids of list l
    def _list_ids(self, l):
        return self.ids[int(self.offsets[l]):int(self.offsets[l + 1])]

    def skip_mask(self):
        skip = np.zeros(self.ids.size, np.uint8)
        for l in range(self.nlist):
            if self.tomb[l]:
                b = int(self.offsets[l])
                for j, i in enumerate(self._list_ids(l).tolist()):
                    if i in self.tomb[l]:
                        skip[b + j] = 1
        return skip

    def enable_reranking(self, X, ids, factor):
        X = _f32(X)
        self.rr = {}
        for i, v in zip(np.asarray(ids, np.uint64).tolist(), X):
            self.rr[i] = v.copy()           # collect(): a later duplicate wins
        self.rerank_factor = max(int(factor), 1)

    def delete(self, id_):
        for l in range(self.nlist):
            if id_ in set(self._list_ids(l).tolist()) and id_ not in self.tomb[l]:
                self.tomb[l].add(id_)
                if self.rr is not None:
                    self.rr.pop(id_, None)
                return True
        return False

    def len(self):
        return int(self.ids.size) - sum(len(t) for t in self.tomb)

    def num_tombstones(self):
        return sum(len(t) for t in self.tomb)

    def compact(self):
        keep = self.skip_mask() == 0
        sizes = [int(keep[int(self.offsets[l]):int(self.offsets[l + 1])].sum())
                 for l in range(self.nlist)]
        self.ids = np.ascontiguousarray(self.ids[keep])
        self.codes = np.ascontiguousarray(self.codes[keep])
        self.offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.uint64)
        self.tomb = [set() for _ in range(self.nlist)]

    def insert_batch(self, X, ids, threads=0):
        X = _f32(X)
        ids = np.asarray(ids, np.uint64)
        a = assign(X, self.centroids, threads)
        resid = _f32(X - self.centroids[a])
        codes = pq_encode(self.codebooks, resid, threads)
        lists_ids = [list(self._list_ids(l)) for l in range(self.nlist)]
        lists_codes = [list(self.codes[int(self.offsets[l]):int(self.offsets[l + 1])])
                       for l in range(self.nlist)]
        for i in range(X.shape[0]):
            l = int(a[i])
            lists_ids[l].append(ids[i])
            lists_codes[l].append(codes[i])
            self.tomb[l].discard(int(ids[i]))
            if self.rr is not None:
                self.rr[int(ids[i])] = X[i].copy()
        sizes = [len(x) for x in lists_ids]
        self.offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.uint64)
        self.ids = np.array([i for x in lists_ids for i in x], np.uint64)
        self.codes = np.ascontiguousarray(
            np.array([c for x in lists_codes for c in x], np.uint8).reshape(-1, self.m))

    def _rerank(self, q, ids, d, cnt, k):
        """rerank_results: exact sqrt(L2^2) of the candidates with an original
        vector, stable-sorted, first k."""
        if self.rr is None:
            return ids[:k][:min(cnt, k)].tolist(), d[:min(cnt, k)].tolist()
        out = []
        for i in ids[:cnt].tolist():
            v = self.rr.get(i)
            if v is not None:
                out.append((i, np.float32(np.sqrt(np.float32(l2sq(q, v))))))
        out.sort(key=lambda t: t[1])
        out = out[:k]
        return [i for i, _ in out], [float(x) for _, x in out]

    def _fetch(self, k):
        return k * self.rerank_factor if self.rr is not None else k

    def search(self, q, k):
        q = _f32(q)
        f = self._fetch(k)
        ids = np.empty(max(f, 1), np.uint64)
        d = np.empty(max(f, 1), np.float32)
        cnt = lib().orc_ivfpq_search_skip(self.centroids, self.codebooks, self.nlist, self.m,
                                          self.dim, self.offsets, self.ids, self.codes,
                                          self.skip_mask(), self.nprobe, q, f, ids, d)
        return self._rerank(q, ids, d, cnt, k)

    def batch_search_arrays(self, Q, k, threads=0):
        """batch_search as (ids, dists, counts) arrays; re-ranking in C++."""
        Q = _f32(Q)
        nq = Q.shape[0]
        f = self._fetch(k)
        ids = np.empty((nq, f), np.uint64)
        d = np.empty((nq, f), np.float32)
        counts = np.empty(nq, np.uint32)
        lib().orc_ivfpq_batch_search_skip(self.centroids, self.codebooks, self.nlist, self.m,
                                          self.dim, self.offsets, self.ids, self.codes,
                                          self.skip_mask(), self.nprobe, Q, nq, f, 0, ids, d,
                                          counts, _threads(threads))
        if self.rr is None:
            return ids, d, counts
        rid = np.array(sorted(self.rr), np.uint64)
        rx = _f32(np.stack([self.rr[i] for i in rid.tolist()])) if rid.size else \
            np.zeros((0, self.dim), np.float32)
        oi = np.empty((nq, k), np.uint64)
        od = np.empty((nq, k), np.float32)
        oc = np.empty(nq, np.uint32)
        lib().orc_rerank(Q, nq, self.dim, ids, counts, f, rid, rx, rid.size, k, oi, od, oc,
                         _threads(threads))
        return oi, od, oc

    def batch_search(self, Q, k, threads=0):
        Q = _f32(Q)
        nq = Q.shape[0]
        f = self._fetch(k)
        ids = np.empty((nq, f), np.uint64)
        d = np.empty((nq, f), np.float32)
        counts = np.empty(nq, np.uint32)
        lib().orc_ivfpq_batch_search_skip(self.centroids, self.codebooks, self.nlist, self.m,
                                          self.dim, self.offsets, self.ids, self.codes,
                                          self.skip_mask(), self.nprobe, Q, nq, f, nq, ids, d,
                                          counts, _threads(threads))
        return [self._rerank(Q[i], ids[i], d[i], int(counts[i]), k) for i in range(nq)]

    def search_filtered(self, q, k, allowed):
        q = _f32(q)
        allowed = set(np.asarray(allowed, np.uint64).tolist())
        if not allowed:
            return [], []
        f = self._fetch(k) * 4
        skip = self.skip_mask()
        for p, i in enumerate(self.ids.tolist()):
            if i not in allowed:
                skip[p] = 1
        ids = np.empty(f, np.uint64)
        d = np.empty(f, np.float32)
        cnt = lib().orc_ivfpq_search_skip(self.centroids, self.codebooks, self.nlist, self.m,
                                          self.dim, self.offsets, self.ids, self.codes, skip,
                                          self.nprobe, q, f, ids, d)
        return self._rerank(q, ids, d, cnt, k)
