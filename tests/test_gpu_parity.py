"""Parity of the CUDA engine (through the C ABI) with the oracle.

Integer and byte outputs (assignments, list layout, PQ codes) must be
bit-exact; so must every distance the engine computes in the reference's
summation order.  Top-k results use the port's contract (see parity.py).
"""
import os

import numpy as np
import pytest

from parity import assert_topk_match

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
U64MAX = np.iinfo(np.uint64).max


@pytest.fixture(scope="module")
def fg():
    import forgegpu
    return forgegpu


@pytest.fixture(scope="module")
def small():
    return np.load(os.path.join(HERE, "golden", "ivfpq_small.npz"))


# ---------------------------------------------------------------------------
# distances
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("dim", [1, 2, 7, 8, 9, 15, 16, 64, 96, 128, 256, 768])
def test_pairwise_bit_exact(fg, ctx, orc, dim):
    rng = np.random.default_rng(dim)
    a = rng.standard_normal((257, dim)).astype(np.float32)
    b = rng.standard_normal((257, dim)).astype(np.float32)
    for metric in range(5):
        got = fg.pairwise_distance(metric, a, b, ctx)
        want = orc.pairwise(metric, a, b)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (metric, dim)


def test_golden_known_values_on_gpu(fg, ctx):
    a = np.zeros((1, 8), np.float32)
    b = np.array([[3, 4, 0, 0, 0, 0, 0, 0]], np.float32)
    assert fg.pairwise_distance(0, a, b, ctx)[0] == 5.0
    assert fg.pairwise_distance(1, a, b, ctx)[0] == 25.0
    assert fg.pairwise_distance(3, [[1, 0]], [[1, 0]], ctx)[0] == -1.0
    assert fg.pairwise_distance(2, [[1, 0]], [[0, 1]], ctx)[0] == 1.0
    assert fg.pairwise_distance(4, [[0, 0]], [[3, 4]], ctx)[0] == 7.0


# ---------------------------------------------------------------------------
# k-means, PQ
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("n,dim,k", [(5000, 128, 1024), (3000, 37, 100), (777, 8, 256)])
def test_assign_bit_exact(fg, ctx, orc, n, dim, k):
    rng = np.random.default_rng(n + dim)
    X = rng.standard_normal((n, dim)).astype(np.float32)
    C = rng.standard_normal((k, dim)).astype(np.float32)
    C[5] = C[3]  # duplicate centroid: the first minimum must win
    assert np.array_equal(fg.assign(X, C, ctx), orc.assign(X, C))


def _unit_rows(rng, n, dim):
    X = rng.standard_normal((n, dim)).astype(np.float32)
    return (X / np.linalg.norm(X, axis=1, keepdims=True)).astype(np.float32)


def test_config_e_shape_training_bit_exact(fg, ctx, orc):
    """Config E's shapes (unit-normalised 768-d rows, random-sample init for
    k > 64, PQ with M = 96) at a size the oracle finishes in seconds:
    centroids, assignments, codebooks and codes bit-exact."""
    rng = np.random.default_rng(11)
    X = _unit_rows(rng, 6000, 768)
    k = 300
    init = rng.permutation(len(X))[:k].astype(np.uint32)
    km = fg.KMeans(k, 4, ctx).fit(X, init_idx=init)
    cents, it = orc.kmeans_fit(X, k, 4, init)
    assert km.iters == it
    assert np.array_equal(km.centroids.view(np.uint32), cents.view(np.uint32))
    assert np.array_equal(km.assignments, orc.assign(X, cents))
    pinit = np.concatenate([rng.permutation(len(X))[:256] for _ in range(96)]).astype(np.uint32)
    pq = fg.ProductQuantizer.train(X, 96, init_idx=pinit, iters=3, ctx=ctx)
    cb, its = orc.pq_train(X, 96, pinit, 3)
    assert np.array_equal(pq.iters, its)
    assert np.array_equal(pq.codebooks.view(np.uint32), cb.view(np.uint32))
    assert np.array_equal(pq.encode(X), orc.pq_encode(cb, X))


@pytest.mark.parametrize("mode", [1, 3])
def test_config_d_shape_search(fg, ctx, orc, mode):
    """Config D's shapes (unit-normalised 96-d rows, M = 48: subvectors of two
    floats, cosine metric stored and ignored) at a size the oracle finishes in
    seconds, in the exact and the tensor scan modes."""
    rng = np.random.default_rng(9)
    X = _unit_rows(rng, 40000, 96)
    Q = _unit_rows(np.random.default_rng(10), 300, 96)
    ix = fg.IVFPQIndex.build(X, 256, 48, fg.DistanceMetric.Cosine, ctx=ctx, seed=4)
    ox = _oracle_index(orc, ix)
    ix.set_scan_mode(mode)
    for nprobe in (4, 16):
        ix.set_nprobe(nprobe)
        ox.set_nprobe(nprobe)
        ids, d, cnt, st = ix.batch_search_arrays(Q, 10, stats=True)
        oi, od, oc = ox.batch_search(Q, 10)
        assert_topk_match(ids, d, cnt, oi, od, oc, f"config D shape mode={mode} nprobe={nprobe}")
        if mode == 3:
            assert st.exact_rescans <= len(Q) // 10


@pytest.mark.parametrize("n,dim,k,iters", [(4000, 16, 100, 25), (2000, 32, 32, 25),
                                           (3000, 8, 256, 10), (600, 5, 64, 30)])
def test_kmeans_bit_exact(fg, ctx, orc, n, dim, k, iters):
    rng = np.random.default_rng(k)
    X = rng.random((n, dim), dtype=np.float32)
    init = rng.permutation(n)[:k].astype(np.uint32)
    u = (rng.integers(0, 1 << 23, k) / float(1 << 23)).astype(np.float32)
    km = fg.KMeans(k, iters, ctx).fit(X, init_idx=init, kpp_u=u)
    cents, it = orc.kmeans_fit(X, k, iters, init, u)
    assert km.iters == it
    assert np.array_equal(km.centroids.view(np.uint32), cents.view(np.uint32))
    assert np.array_equal(km.assignments, orc.assign(X, cents))


def test_kmeans_errors(fg, ctx):
    with pytest.raises(fg.ForgeGpuError) as e:
        fg.KMeans(100, 5, ctx).fit(np.zeros((50, 4), np.float32))
    assert e.value.kind == "InsufficientVectors"


@pytest.mark.parametrize("n,dim,m", [(3000, 128, 16), (2000, 96, 48), (1500, 50, 10)])
def test_pq_train_encode_lut_bit_exact(fg, ctx, orc, n, dim, m):
    rng = np.random.default_rng(dim)
    X = rng.standard_normal((n, dim)).astype(np.float32)
    init = np.concatenate([rng.permutation(n)[:256] for _ in range(m)]).astype(np.uint32)
    pq = fg.ProductQuantizer.train(X, m, init_idx=init, iters=25, ctx=ctx)
    cb, its = orc.pq_train(X, m, init, 25)
    assert np.array_equal(pq.iters, its)
    assert np.array_equal(pq.codebooks.view(np.uint32), cb.view(np.uint32))
    assert np.array_equal(pq.encode(X), orc.pq_encode(cb, X))
    q = rng.standard_normal((3, dim)).astype(np.float32)
    lut = pq.build_lookup_table_flat(q)
    for i in range(3):
        assert np.array_equal(lut[i], orc.lut_flat(cb, q[i]))


def test_pq_errors(fg, ctx):
    with pytest.raises(fg.ForgeGpuError) as e:
        fg.ProductQuantizer.train(np.zeros((300, 10), np.float32), 3, ctx=ctx)
    assert e.value.kind == "DimensionNotDivisible"
    with pytest.raises(fg.ForgeGpuError) as e:
        fg.ProductQuantizer.train(np.zeros((100, 16), np.float32), 4, ctx=ctx)
    assert e.value.kind == "InsufficientVectors"


# ---------------------------------------------------------------------------
# IVF-PQ
# ---------------------------------------------------------------------------
def test_ivfpq_build_bit_exact(fg, ctx, small):
    g = small
    ix = fg.IVFPQIndex.build(g["X"], int(g["nlist"]), int(g["m"]), ids=g["ids"], ctx=ctx,
                             ivf_sample_idx=g["ivf_sample_idx"], ivf_init_idx=g["ivf_init_idx"],
                             ivf_kpp_u=g["ivf_kpp_u"], pq_sample_idx=g["pq_sample_idx"],
                             pq_init_idx=g["pq_init_idx"])
    cents, cb, offs, ids, codes = ix.export()
    assert np.array_equal(cents.view(np.uint32), g["centroids"].view(np.uint32))
    assert np.array_equal(cb.view(np.uint32), g["codebooks"].view(np.uint32))
    assert np.array_equal(offs, g["offsets"])
    assert np.array_equal(ids, g["list_ids"])
    assert np.array_equal(codes, g["codes"])
    assert len(ix) == g["X"].shape[0] and ix.n_partitions() == int(g["nlist"])


def test_ivfpq_search_vs_golden(fg, ctx, small):
    g = small
    ix = fg.IVFPQIndex.from_trained(g["centroids"], g["codebooks"], g["offsets"], g["list_ids"],
                                    g["codes"], ctx=ctx)
    assert ix.nprobe() == 1
    ix.set_nprobe(int(g["nprobe"]))
    k = int(g["k"])
    ids, d, cnt = ix.batch_search_arrays(g["Q"], k)
    rate = assert_topk_match(ids, d, cnt, g["batch_ids"], g["batch_d"], g["batch_cnt"], "batch")
    assert rate > 0.9
    for q in range(len(g["Q"])):
        res = ix.search(g["Q"][q], k)
        c = int(g["single_cnt"][q])
        si = np.array([r[0] for r in res], np.uint64)
        sd = np.array([r[1] for r in res], np.float32)
        assert_topk_match(si[None], sd[None], [len(res)], g["single_ids"][q:q + 1, :c],
                          g["single_d"][q:q + 1, :c], [c], f"single {q}")


def _oracle_index(orc, fgix):
    cents, cb, offs, ids, codes = fgix.export()
    return orc.OracleIVFPQ(cents, cb, offs, ids, codes)


@pytest.mark.parametrize("nprobe,k", [(1, 10), (8, 10), (32, 1), (32, 100), (64, 256),
                                      (300, 20), (0, 10)])
def test_ivfpq_config_a_parity(fg, ctx, orc, nprobe, k):
    """Config A shapes (10k x 128 U[0,1), nlist 32, M 8) at many nprobe / k."""
    rng = np.random.default_rng(1)
    X = rng.random((10000, 128), dtype=np.float32)
    Q = np.random.default_rng(2).random((300, 128), dtype=np.float32)
    ix = fg.IVFPQIndex.build(X, 32, 8, ctx=ctx, seed=123)
    ox = _oracle_index(orc, ix)
    ix.set_nprobe(nprobe)
    ox.set_nprobe(nprobe)
    assert ix.nprobe() == min(nprobe, 32)
    ids, d, cnt = ix.batch_search_arrays(Q, k)
    oi, od, oc = ox.batch_search(Q, k)
    assert_topk_match(ids, d, cnt, oi, od, oc, f"batch nprobe={nprobe} k={k}")
    for q in range(0, 300, 37):
        res = ix.search(Q[q], k)
        si, sd = ox.search(Q[q], k)
        assert len(res) == len(si)
        assert_topk_match(np.array([[r[0] for r in res]], np.uint64),
                          np.array([[r[1] for r in res]], np.float32), [len(res)],
                          si[None], sd[None], [len(si)], f"single q={q}")


def test_ivfpq_ragged_lists_and_short_results(fg, ctx, orc):
    """Lists shorter than k, empty lists and M not a multiple of 8."""
    rng = np.random.default_rng(9)
    X = rng.random((600, 40), dtype=np.float32)
    ix = fg.IVFPQIndex.build(X, 64, 10, ctx=ctx, seed=5)  # M=10 -> generic code path
    ox = _oracle_index(orc, ix)
    ix.set_nprobe(2)
    ox.set_nprobe(2)
    Q = rng.random((50, 40), dtype=np.float32)
    ids, d, cnt = ix.batch_search_arrays(Q, 50)
    oi, od, oc = ox.batch_search(Q, 50)
    assert_topk_match(ids, d, cnt, oi, od, oc, "ragged")
    assert (cnt < 50).any()  # some queries see fewer than k codes


def test_ivfpq_edge_cases(fg, ctx, small):
    g = small
    ix = fg.IVFPQIndex.from_trained(g["centroids"], g["codebooks"], g["offsets"], g["list_ids"],
                                    g["codes"], ctx=ctx)
    assert ix.batch_search(np.zeros((0, g["X"].shape[1]), np.float32), 10) == []
    ids, d, cnt = ix.batch_search_arrays(g["Q"][:3], 0)
    assert ids.shape == (3, 0)
    ix.set_nprobe(100)
    assert ix.nprobe() == int(g["nlist"])
    with pytest.raises(fg.ForgeGpuError):
        ix.batch_search(g["Q"][:2], 257)  # above FDB_MAX_K
    with pytest.raises(fg.ForgeGpuError) as e:
        fg.IVFPQIndex.build(np.zeros((300, 30), np.float32), 4, 7, ctx=ctx)
    assert e.value.kind == "DimensionNotDivisible"
    with pytest.raises(fg.ForgeGpuError) as e:
        fg.IVFPQIndex.build(np.zeros((100, 32), np.float32), 4, 8, ctx=ctx)
    assert e.value.kind == "InsufficientVectors"


# ---------------------------------------------------------------------------
# brute force
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("metric", [0, 1, 2, 3, 4])
@pytest.mark.parametrize("n,dim,k", [(20000, 128, 100), (5000, 13, 10), (300, 64, 256)])
def test_bf_parity(fg, ctx, orc, metric, n, dim, k):
    rng = np.random.default_rng(n + metric)
    X = rng.standard_normal((n, dim)).astype(np.float32)
    Q = rng.standard_normal((64, dim)).astype(np.float32)
    ids = rng.permutation(n * 3)[:n].astype(np.uint64)
    bf = fg.BruteForceIndex(metric, ctx).add(X, ids)
    gi, gd, gc = bf.batch_search_arrays(Q, k)
    oi, od, oc = orc.bf_batch_search(X, ids, metric, Q, k)
    assert_topk_match(gi, gd, gc, oi, od, oc, f"bf metric={metric}")
    res = bf.search(Q[0], k)
    assert [r[0] for r in res][:5] == gi[0, :5].tolist()


def test_bf_self_query_and_edges(fg, ctx):
    rng = np.random.default_rng(4)
    X = rng.standard_normal((1000, 32)).astype(np.float32)
    bf = fg.BruteForceIndex(1, ctx)
    assert bf.dimension() == 0 and bf.search(X[0], 5) == []
    bf.add(X[:500]).add(X[500:])
    assert len(bf) == 1000 and bf.dimension() == 32
    ids, d, cnt = bf.batch_search_arrays(X[:50], 1)
    assert np.array_equal(ids[:, 0], np.arange(50, dtype=np.uint64))
    assert np.all(d[:, 0] == 0)
    with pytest.raises(fg.ForgeGpuError):
        bf.search(X[0], 0)  # the reference panics on k == 0 with rows present
    with pytest.raises(fg.ForgeGpuError) as e:
        bf.add(np.zeros((1, 31), np.float32))
    assert e.value.kind == "DimensionMismatch"


# ---------------------------------------------------------------------------
# scan modes: exact LUT vs precomputed tables + exact rescoring
# ---------------------------------------------------------------------------
@pytest.fixture(scope="module")
def gmm_index(fg, ctx):
    from forgegpu.datasets import gmm_descriptors
    X = gmm_descriptors(20000, components=64, seed=11)
    Q = gmm_descriptors(400, components=64, seed=12)
    ix = fg.IVFPQIndex.build(X, 64, 16, ctx=ctx, seed=3)
    return ix, X, Q


@pytest.mark.parametrize("mode", [1, 2, 3])
@pytest.mark.parametrize("k", [1, 10, 100])
def test_scan_modes_match_oracle(fg, ctx, orc, gmm_index, mode, k):
    ix, X, Q = gmm_index
    ox = _oracle_index(orc, ix)
    ix.set_scan_mode(mode)
    ix.set_nprobe(8)
    ox.set_nprobe(8)
    ids, d, cnt, st = ix.batch_search_arrays(Q, k, stats=True)
    oi, od, oc = ox.batch_search(Q, k)
    rate = assert_topk_match(ids, d, cnt, oi, od, oc, f"mode={mode} k={k}")
    assert rate > 0.95
    if mode >= 2:
        assert st.exact_rescans <= len(Q) // 20  # nearly every query certifies
    for q in range(0, len(Q), 97):
        res = ix.search(Q[q], k)
        si, sd = ox.search(Q[q], k)
        assert np.array_equal(np.array([r[1] for r in res], np.float32), sd)
    ix.set_scan_mode(0)


def test_table_mode_ties_fall_back_to_exact(fg, ctx, orc):
    """Fifty copies of each of 40 vectors: distances tie exactly, the
    shortlist cannot be certified, and the exact re-scan must take over."""
    rng = np.random.default_rng(21)
    base = (rng.random((40, 64), dtype=np.float32) * 10).astype(np.float32)
    X = np.repeat(base, 50, axis=0)
    ix = fg.IVFPQIndex.build(X, 8, 8, ctx=ctx, seed=2)
    ix.set_scan_mode(2)
    ix.set_nprobe(8)
    ox = _oracle_index(orc, ix)
    ox.set_nprobe(8)
    Q = base[:20] + np.float32(0.01)
    ids, d, cnt, st = ix.batch_search_arrays(Q, 10, stats=True)
    assert st.exact_rescans > 0
    oi, od, oc = ox.batch_search(Q, 10)
    assert_topk_match(ids, d, cnt, oi, od, oc, "ties")


# ---------------------------------------------------------------------------
# IVF-PQ tensor mode: lists scored on tcgen05 + exact rescoring
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("nprobe,k,nq", [(1, 10, 300), (8, 1, 50), (8, 16, 300), (32, 10, 7),
                                         (32, 16, 1000)])
def test_ivfpq_tensor_mode_config_a(fg, ctx, orc, nprobe, k, nq):
    rng = np.random.default_rng(1)
    X = rng.random((10000, 128), dtype=np.float32)
    Q = np.random.default_rng(4).random((nq, 128), dtype=np.float32)
    ix = fg.IVFPQIndex.build(X, 32, 8, ctx=ctx, seed=123)
    ox = _oracle_index(orc, ix)
    ix.set_scan_mode(ix.SCAN_TENSOR)
    ix.set_nprobe(nprobe)
    ox.set_nprobe(nprobe)
    ids, d, cnt, st = ix.batch_search_arrays(Q, k, stats=True)
    oi, od, oc = ox.batch_search(Q, k)
    assert_topk_match(ids, d, cnt, oi, od, oc, f"tensor nprobe={nprobe} k={k}")
    assert st.lists_probed == nq * nprobe
    for q in range(0, nq, 61):
        res = ix.search(Q[q], k)
        si, sd = ox.search(Q[q], k)
        assert np.array_equal(np.array([r[1] for r in res], np.float32), sd)


def test_ivfpq_tensor_mode_ties_and_short_lists(fg, ctx, orc):
    """Exact ties longer than the 64-entry shortlist cannot be certified from
    the shortlist alone; lists shorter than 64 codes leave the admission
    threshold at +inf.  Both must end on the exact re-scan or the extended
    certificate with the oracle's answer."""
    rng = np.random.default_rng(21)
    base = (rng.random((40, 64), dtype=np.float32) * 10).astype(np.float32)
    X = np.repeat(base, 100, axis=0)
    ix = fg.IVFPQIndex.build(X, 8, 8, ctx=ctx, seed=2)
    ix.set_scan_mode(ix.SCAN_TENSOR)
    ix.set_nprobe(8)
    ox = _oracle_index(orc, ix)
    ox.set_nprobe(8)
    Q = base[:20] + np.float32(0.01)
    ids, d, cnt, st = ix.batch_search_arrays(Q, 10, stats=True)
    oi, od, oc = ox.batch_search(Q, 10)
    assert_topk_match(ids, d, cnt, oi, od, oc, "tensor ties")
    # many tiny lists: 600 vectors in 64 lists, dim 64 -> subvectors of 8
    X2 = rng.random((600, 64), dtype=np.float32)
    ix2 = fg.IVFPQIndex.build(X2, 64, 8, ctx=ctx, seed=5)
    ix2.set_scan_mode(ix2.SCAN_TENSOR)
    ox2 = _oracle_index(orc, ix2)
    Q2 = rng.random((300, 64), dtype=np.float32)
    for nprobe in (1, 2, 5):
        ix2.set_nprobe(nprobe)
        ox2.set_nprobe(nprobe)
        ids, d, cnt = ix2.batch_search_arrays(Q2, 16)
        oi, od, oc = ox2.batch_search(Q2, 16)
        assert_topk_match(ids, d, cnt, oi, od, oc, f"tensor tiny lists nprobe={nprobe}")


def test_ivfpq_tensor_mode_rescan_rounds(fg, ctx, orc):
    """The exact re-scan runs from counts kept on the device, in rounds of at
    most 64 MiB of per-unit keys (131072 units at k = 64).  8200 queries x 16
    probes can produce more units than one round holds; runs of 1200 identical
    codes exceed both the shortlist and the extension (1024 entries), so
    queries re-scan."""
    rng = np.random.default_rng(33)
    base = (rng.random((25, 64), dtype=np.float32) * 10).astype(np.float32)
    X = np.repeat(base, 1200, axis=0)
    ix = fg.IVFPQIndex.build(X, 16, 8, ctx=ctx, seed=3)
    ix.set_scan_mode(ix.SCAN_TENSOR)
    ix.set_nprobe(16)
    ox = _oracle_index(orc, ix)
    ox.set_nprobe(16)
    Q = base[rng.integers(0, 25, 8200)] + rng.random((8200, 64), dtype=np.float32) * 0.05
    ids, d, cnt, st = ix.batch_search_arrays(Q, 64, stats=True)
    oi, od, oc = ox.batch_search(Q, 64)
    assert_topk_match(ids, d, cnt, oi, od, oc, "tensor re-scan rounds")
    assert st.exact_rescans > 0


def test_ivfpq_pinned_host_batch_matches_device_entry(fg, ctx, orc, gmm_index):
    """The host-buffer batch search (pinned buffers, results copied back
    before the call's one synchronisation) returns what the device-buffer
    entry point and the oracle return, on repeated calls."""
    import ctypes as C
    import torch
    ix, X, _ = gmm_index
    from forgegpu.datasets import gmm_descriptors
    Q = gmm_descriptors(3001, components=64, seed=13)
    ix.set_nprobe(8)
    L = fg.lib()
    nq, k = Q.shape[0], 10
    hQ = torch.from_numpy(Q).pin_memory()
    h_ids = torch.empty((nq, k), dtype=torch.int64).pin_memory()
    h_d = torch.empty((nq, k), dtype=torch.float32).pin_memory()
    h_c = torch.empty((nq,), dtype=torch.int32).pin_memory()
    for _ in range(2):
        fg._check(L.fdb_ivfpq_batch_search(ix.h, C.c_void_p(hQ.data_ptr()), nq, k,
                                           C.c_void_p(h_ids.data_ptr()),
                                           C.c_void_p(h_d.data_ptr()),
                                           C.c_void_p(h_c.data_ptr()), None))
        dQ = torch.from_numpy(Q).cuda()
        d_ids = torch.empty((nq, k), dtype=torch.int64, device="cuda")
        d_d = torch.empty((nq, k), dtype=torch.float32, device="cuda")
        d_c = torch.empty((nq,), dtype=torch.int32, device="cuda")
        fg._check(L.fdb_ivfpq_batch_search_device(ix.h, C.c_void_p(dQ.data_ptr()), nq, k,
                                                  C.c_void_p(d_ids.data_ptr()),
                                                  C.c_void_p(d_d.data_ptr()),
                                                  C.c_void_p(d_c.data_ptr()), None))
        assert torch.equal(h_ids, d_ids.cpu()) and torch.equal(h_d, d_d.cpu())
        assert torch.equal(h_c, d_c.cpu())
    ox = _oracle_index(orc, ix)
    ox.set_nprobe(8)
    oi, od, oc = ox.batch_search(Q, k)
    assert_topk_match(h_ids.numpy().view(np.uint64), h_d.numpy(), h_c.numpy().view(np.uint32),
                      oi, od, oc, "pinned host batch")
    ix.set_nprobe(1)


def test_ivfpq_tensor_mode_gmm_certifies(fg, ctx, orc, gmm_index):
    """Descriptor-like data: the fp16 bound certifies nearly every query."""
    ix, X, Q = gmm_index
    ox = _oracle_index(orc, ix)
    ix.set_scan_mode(ix.SCAN_TENSOR)
    for nprobe in (1, 4, 16):
        ix.set_nprobe(nprobe)
        ox.set_nprobe(nprobe)
        ids, d, cnt, st = ix.batch_search_arrays(Q, 10, stats=True)
        oi, od, oc = ox.batch_search(Q, 10)
        assert_topk_match(ids, d, cnt, oi, od, oc, f"tensor gmm nprobe={nprobe}")
        assert st.exact_rescans <= len(Q) // 20
    ix.set_scan_mode(0)


# ---------------------------------------------------------------------------
# brute force: tcgen05 tensor-core shortlist + exact rescoring
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("metric", [0, 1, 2, 3])
def test_bf_tensor_path_certifies_and_matches(fg, ctx, orc, metric):
    rng = np.random.default_rng(100 + metric)
    X = rng.standard_normal((60000, 128)).astype(np.float32)
    Q = rng.standard_normal((300, 128)).astype(np.float32)
    bf = fg.BruteForceIndex(metric, ctx).add(X)
    for k in (10, 100):
        ids, d, cnt, st = bf.batch_search_arrays(Q, k, stats=True)
        assert st.exact_rescans <= len(Q) // 20, f"tensor path fell back {st.exact_rescans}x"
        oi, od, oc = orc.bf_batch_search(X, np.arange(60000), metric, Q, k)
        assert_topk_match(ids, d, cnt, oi, od, oc, f"bf tensor metric={metric} k={k}")
    bf.set_scan_mode(1)
    ids2, d2, c2 = bf.batch_search_arrays(Q, 10)
    bf.set_scan_mode(0)
    ids1, d1, c1 = bf.batch_search_arrays(Q, 10)
    assert np.array_equal(d1, d2)


@pytest.mark.parametrize("n,dim,nq", [(129, 64, 1), (1000, 96, 130), (3000, 160, 200),
                                      (5000, 200, 257)])
def test_bf_tensor_ragged_shapes(fg, ctx, orc, n, dim, nq):
    """Row counts and query counts off the 128 tile, dims padded to 64/256."""
    rng = np.random.default_rng(n)
    X = rng.standard_normal((n, dim)).astype(np.float32)
    Q = rng.standard_normal((nq, dim)).astype(np.float32)
    bf = fg.BruteForceIndex(1, ctx).add(X)
    ids, d, cnt = bf.batch_search_arrays(Q, 32)
    oi, od, oc = orc.bf_batch_search(X, np.arange(n), 1, Q, 32)
    assert_topk_match(ids, d, cnt, oi, od, oc, f"bf ragged n={n}")
