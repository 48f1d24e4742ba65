"""The oracle against the reference's known answers and the golden fixtures
(CPU only).  An oracle that fails here cannot be trusted as the checker of the
GPU engine."""
import json
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = os.path.join(HERE, "golden")


@pytest.fixture(scope="module")
def kv():
    with open(os.path.join(GOLD, "known_values.json")) as f:
        return json.load(f)


def test_distance_known_values(orc, kv):
    ids = {"euclidean": orc.EUCLIDEAN, "euclidean_squared": orc.EUCLIDEAN_SQUARED,
           "cosine": orc.COSINE, "dot_product": orc.DOT_PRODUCT, "manhattan": orc.MANHATTAN}
    for metric, a, b, want, tol, cite in kv["distance"]:
        if metric == "dot_raw":
            got = orc.dot(a, b)
        else:
            got = orc.metric(ids[metric], a, b)
        assert abs(got - want) < tol, (metric, cite, got, want)


def test_kmeans_nearest_known(orc, kv):
    t = kv["kmeans_nearest"]
    got = orc.find_nearest_centroids(np.array(t["centroids"]), np.array(t["query"]), t["k"])
    assert len(got) == t["k"] and got[0] == t["first"]


def test_recall_known(kv):
    from forgegpu.datasets import recall_at_k
    for pred, truth, k, want, cite in kv["recall"]:
        assert abs(recall_at_k(np.array([pred]), np.array([truth]), k) - want) < 1e-7, cite


def test_avx2_order_bit_exact(orc):
    g = np.load(os.path.join(GOLD, "avx2_order.npz"))
    for d in [1, 2, 7, 8, 9, 15, 16, 64, 128, 256]:
        a, b = g[f"a_{d}"], g[f"b_{d}"]
        for i in range(a.shape[0]):
            assert np.float32(orc.l2sq(a[i], b[i])) == g[f"l2sq_{d}"][i], ("l2sq", d, i)
            assert np.float32(orc.dot(a[i], b[i])) == g[f"dot_{d}"][i], ("dot", d, i)
            assert np.float32(orc.cosine(a[i], b[i])) == g[f"cos_{d}"][i], ("cos", d, i)


def test_adc_orders_bit_exact(orc):
    g = np.load(os.path.join(GOLD, "avx2_order.npz"))
    for m in [4, 8, 10, 16, 48]:
        lut, codes = g[f"lut_{m}"], g[f"codes_{m}"]
        for i in range(codes.shape[0]):
            assert np.float32(orc.adc("fast", lut, codes[i])) == g[f"adc_fast_{m}"][i]
            assert np.float32(orc.adc("lane8", lut, codes[i])) == g[f"adc_lane8_{m}"][i]


@pytest.mark.parametrize("dim", [1, 7, 8, 15, 16, 64, 128, 256])
def test_simd_matches_scalar(orc, dim):
    """tests/correctness.rs:8-78: SIMD vs scalar within 1e-5 (relative for L2^2)."""
    rng = np.random.default_rng(dim)
    a = rng.uniform(-1, 1, dim).astype(np.float32)
    b = rng.uniform(-1, 1, dim).astype(np.float32)
    s = orc.lib().orc_l2sq_scalar(a, b, dim)
    assert abs(orc.l2sq(a, b) - s) < abs(s) * 1e-5 + 1e-5
    sd = orc.lib().orc_dot_scalar(a, b, dim)
    assert abs(orc.dot(a, b) - sd) < max(abs(sd) * 1e-4, 1e-4)


@pytest.mark.parametrize("m", [8, 10, 16, 32])
def test_adc_simd_vs_scalar(orc, m):
    """pq.rs:1150-1310: SIMD vs scalar ADC within 1e-4 absolute."""
    rng = np.random.default_rng(m)
    lut = rng.random(m * 256, dtype=np.float32)
    code = rng.integers(0, 256, m).astype(np.uint8)
    s = orc.adc("scalar", lut, code)
    assert abs(orc.adc("lane8", lut, code) - s) < 1e-4
    assert abs(orc.adc("fast", lut, code) - s) < 1e-4


def test_ivfpq_small_regression(orc):
    """The committed small IVF-PQ fixture reproduces exactly."""
    g = np.load(os.path.join(GOLD, "ivfpq_small.npz"))
    ix = orc.OracleIVFPQ.build(g["X"], g["ids"], int(g["nlist"]), int(g["m"]),
                               g["ivf_sample_idx"], g["ivf_init_idx"], g["ivf_kpp_u"],
                               g["pq_sample_idx"], g["pq_init_idx"])
    assert np.array_equal(ix.centroids, g["centroids"])
    assert np.array_equal(ix.codebooks, g["codebooks"])
    assert np.array_equal(ix.offsets, g["offsets"])
    assert np.array_equal(ix.ids, g["list_ids"])
    assert np.array_equal(ix.codes, g["codes"])
    ix.set_nprobe(int(g["nprobe"]))
    bi, bd, bc = ix.batch_search(g["Q"], int(g["k"]), chunk=len(g["Q"]))
    assert np.array_equal(bd, g["batch_d"]) and np.array_equal(bc, g["batch_cnt"])


def test_batch_vs_single_same_ids_at_full_probe(orc):
    """ivf_pq.rs:2089-2121: batch_search and search find the same id sets
    when every list is probed."""
    rng = np.random.default_rng(3)
    n, dim, nlist, m = 500, 32, 8, 4
    X = rng.uniform(-1, 1, (n, dim)).astype(np.float32)
    ix = orc.OracleIVFPQ.build(X, np.arange(n), nlist, m, np.arange(n), rng.permutation(n)[:nlist],
                               rng.random(nlist), rng.permutation(n),
                               np.concatenate([rng.permutation(n)[:256] for _ in range(m)]))
    ix.set_nprobe(8)
    Q = X[[0, 10, 20]]
    bi, bd, bc = ix.batch_search(Q, 5)
    for q in range(3):
        si, sd = ix.search(Q[q], 5)
        assert set(bi[q].tolist()) == set(si.tolist())
        assert np.all(np.diff(bd[q]) >= 0)


def test_nprobe_zero_semantics(orc):
    """search() probes nothing at nprobe 0; batch_search probes one list
    (ivf_pq.rs:548-552 vs :878-886)."""
    g = np.load(os.path.join(GOLD, "ivfpq_small.npz"))
    ix = orc.OracleIVFPQ(g["centroids"], g["codebooks"], g["offsets"], g["list_ids"], g["codes"])
    ix.nprobe = 0
    i, d = ix.search(g["Q"][0], 10)
    assert len(i) == 0
    bi, bd, bc = ix.batch_search(g["Q"][:2], 10)
    assert bc[0] > 0


def test_bf_top1_is_scalar_argmin(orc):
    """tests/property.rs:175-201."""
    rng = np.random.default_rng(11)
    for n, dim in [(10, 2), (57, 13), (199, 63)]:
        X = rng.uniform(-1, 1, (n, dim)).astype(np.float32)
        q = rng.uniform(-1, 1, (1, dim)).astype(np.float32)
        ids, d, c = orc.bf_batch_search(X, np.arange(n), orc.EUCLIDEAN_SQUARED, q, 1)
        scal = [orc.lib().orc_l2sq_scalar(q[0], X[i], dim) for i in range(n)]
        assert ids[0, 0] == int(np.argmin(scal))


def test_kmeans_basic_finite_inertia(orc):
    """kmeans.rs:348-379."""
    rng = np.random.default_rng(5)
    X = rng.uniform(-1, 1, (300, 8)).astype(np.float32)
    cents, it = orc.kmeans_fit(X, 5, 50, rng.permutation(300)[:5], rng.random(5))
    a = orc.assign(X, cents)
    inertia = sum(orc.l2sq(X[i], cents[a[i]]) for i in range(300))
    assert np.isfinite(inertia) and inertia > 0 and 1 <= it <= 50
