"""The allocation-free nearest-centroid search, called through the C ABI.

fdb_find_nearest_centroids_noalloc serves callers that cannot allocate
device memory at search time (a process whose device memory is all reserved
in a pool at start-up, or a loop that must not take cudaMalloc's implicit
synchronisation): it keeps its distance matrix in a fixed device array
instead of allocating one per call.  These tests compare it, on device
buffers the test owns, with the host-buffer entry point
fdb_find_nearest_centroids (one query per call) and with the oracle's
restatement of KMeans::find_nearest_centroids (src/kmeans.rs:334-345), twice
in a row so that a second call over the reused scratch is checked too.  The
file name sorts last so the tests also run after everything else in the
suite.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _dev_ptr(t):
    return C.c_void_p(t.data_ptr())


def _host_nearest(lib, ctx, cents, q, k):
    out = np.empty(min(k, cents.shape[0]), np.uint32)
    rc = lib.fdb_find_nearest_centroids(ctx.h, C.c_void_p(cents.ctypes.data), cents.shape[0],
                                        cents.shape[1], C.c_void_p(q.ctypes.data), k,
                                        C.c_void_p(out.ctypes.data))
    assert rc == 0, lib.fdb_last_error()
    return out


def _noalloc(lib, ctx, d_cents, kc, dim, d_q, nq, k, d_out):
    return lib.fdb_find_nearest_centroids_noalloc(ctx.h, _dev_ptr(d_cents), kc, dim,
                                                  _dev_ptr(d_q), nq, k, _dev_ptr(d_out))


@pytest.mark.parametrize("k", [1, 16, 40, 300])
def test_noalloc_matches_host_entry_point_twice(ctx, orc, k):
    import torch
    import forgegpu as fg
    lib = fg.lib()
    rng = np.random.default_rng(11 + k)
    kc, dim, nq = 1000, 64, 96
    cents = rng.standard_normal((kc, dim)).astype(np.float32)
    take = min(k, kc)
    # set-up call: nothing to do, only the scratch lookup
    assert lib.fdb_find_nearest_centroids_noalloc(ctx.h, None, kc, dim, None, 0, k, None) == 0
    dev = torch.device("cuda", 0)
    d_cents = torch.from_numpy(cents).to(dev)
    for call in range(2):
        q = rng.standard_normal((nq, dim)).astype(np.float32)
        d_q = torch.from_numpy(q).to(dev)
        d_out = torch.full((nq, take), -1, dtype=torch.int32, device=dev)
        torch.cuda.synchronize()
        rc = _noalloc(lib, ctx, d_cents, kc, dim, d_q, nq, k, d_out)
        assert rc == 0, lib.fdb_last_error()
        got = d_out.cpu().numpy().view(np.uint32)
        for i in range(nq):
            want = _host_nearest(lib, ctx, cents, np.ascontiguousarray(q[i]), k)
            assert np.array_equal(got[i], want), (call, i)
            assert np.array_equal(got[i], orc.find_nearest_centroids(cents, q[i], k)), (call, i)


def test_noalloc_rejects_sizes_above_the_scratch(ctx):
    import forgegpu as fg
    lib = fg.lib()
    # the size checks come before any device work; NULL buffers make sure of it
    rc = lib.fdb_find_nearest_centroids_noalloc(ctx.h, None, 1 << 20, 8, None, 5, 4, None)
    assert rc == -1
    assert b"FDB_NOALLOC_MAX_DISTANCES" in lib.fdb_last_error()
    rc = lib.fdb_find_nearest_centroids_noalloc(ctx.h, None, 4, 8, None, (1 << 18) + 1, 4, None)
    assert rc == -1
    assert b"FDB_NOALLOC_MAX_QUERIES" in lib.fdb_last_error()
    # more than 256 ids per query are sorted in shared memory: at most 16384
    # centroids then
    rc = lib.fdb_find_nearest_centroids_noalloc(ctx.h, None, (1 << 14) + 1, 8, None, 5, 300,
                                                None)
    assert rc == -1
    assert b"FDB_NOALLOC_MAX_SORTED_CENTROIDS" in lib.fdb_last_error()
    rc = lib.fdb_find_nearest_centroids_noalloc(ctx.h, None, 1 << 14, 8, None, 5, 300, None)
    assert rc == -1 and b"NULL" in lib.fdb_last_error()
    # exactly at the limit passes the size checks and then needs buffers
    rc = lib.fdb_find_nearest_centroids_noalloc(ctx.h, None, 1 << 12, 8, None, 1 << 10, 4, None)
    assert rc == -1 and b"NULL" in lib.fdb_last_error()
