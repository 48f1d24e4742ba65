"""Parity at the shapes the benchmark runs, where the tensor path takes
branches the small indexes never reach.

Config C (1M x 128, nlist 1024, nprobe 32) has lists of ~1000 codes and
probes ~31k codes per query.  The indexes below have longer lists (1,500+
codes, so list-scan items split into chunks of at most 8 tiles), probe every
list (so pass 1 samples the first tiles of several probes to reach its
quota of the probed codes), and hold crowds of identical PQ codes (integer
descriptors, as in config C), which drive queries through the certificate
extension and the exact re-scan.  Semantics matched: IVFPQIndex::batch_search
(src/index/ivf_pq.rs:850-1047) with the AVX2 lane order of
asymmetric_distance_simd_avx2 (src/pq.rs:435-485); find_nearest_centroids
(src/kmeans.rs:334-345); the index build (ivf_pq.rs:374-506) from the
engine's seeded draws.
"""
import numpy as np
import pytest

from parity import assert_topk_match

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def fg():
    import forgegpu
    return forgegpu


@pytest.fixture(scope="module")
def long_lists(fg, ctx, orc):
    from forgegpu.datasets import gmm_descriptors
    X = gmm_descriptors(200_000, components=128, seed=21)
    # crowds: 1200 copies each of 10 rows (more identical codes than the
    # 64-entry shortlist and the 1024 entries an extension rescores), placed
    # among the others
    crowd = gmm_descriptors(10, components=128, seed=23)
    X = np.concatenate([X[:100_000], np.repeat(crowd, 1200, axis=0), X[100_000:]])
    Q = gmm_descriptors(2000, components=128, seed=22)
    ix = fg.IVFPQIndex.build(X, 128, 16, ctx=ctx, seed=7)
    cents, cb, offs, ids, codes = ix.export()
    ox = orc.OracleIVFPQ(cents, cb, offs, ids, codes)
    return ix, ox, X, Q, np.diff(offs.astype(np.int64)), crowd


@pytest.mark.parametrize("nprobe,k", [(32, 10), (128, 10), (32, 40), (8, 64)])
def test_tensor_path_long_lists(fg, orc, long_lists, nprobe, k):
    ix, ox, X, Q, sizes, _ = long_lists
    assert sizes.mean() > 1024 and sizes.max() > 1024  # items span several 8-tile chunks
    ix.set_scan_mode(ix.SCAN_TENSOR)
    ix.set_nprobe(nprobe)
    ox.set_nprobe(nprobe)
    ids, d, cnt, st = ix.batch_search_arrays(Q, k, stats=True)
    oi, od, oc = ox.batch_search(Q, k)
    # the contract holds row by row; rows equal outright (ids and distances)
    # are most of them (near-ties at the k-th distance may order differently)
    rate = assert_topk_match(ids, d, cnt, oi, od, oc, f"long lists nprobe={nprobe} k={k}")
    assert rate > 0.8
    assert 0 < st.lists_probed <= len(Q) * nprobe  # empty lists are not counted
    # the tensor path ran and pruned part of the probed codes
    assert 0 < st.kernel_scores < st.codes_scanned
    ix.set_scan_mode(0)


def test_tensor_path_long_lists_take_every_fallback(fg, orc, long_lists):
    """Over the whole batch the certificate extension and the exact re-scan
    both run: queries next to a crowd of 1200 identical codes cannot be
    certified from 64 shortlisted entries nor by extending over 1024."""
    ix, ox, X, Q, _, crowd = long_lists
    ix.set_scan_mode(ix.SCAN_TENSOR)
    ix.set_nprobe(32)
    ox.set_nprobe(32)
    rng = np.random.default_rng(5)
    near = crowd[rng.integers(0, len(crowd), 300)] + rng.random((300, 128), dtype=np.float32)
    Qd = np.concatenate([Q, near.astype(np.float32)])
    ids, d, cnt, st = ix.batch_search_arrays(Qd, 10, stats=True)
    oi, od, oc = ox.batch_search(Qd, 10)
    assert_topk_match(ids, d, cnt, oi, od, oc, "long lists, duplicates")
    assert st.extended > 0, "no query took the certificate extension"
    assert st.exact_rescans > 0, "no query took the exact re-scan"
    ix.set_scan_mode(0)


def test_tensor_path_matches_exact_mode_on_long_lists(fg, long_lists):
    """The tensor path and the exact LUT scan return the same keys."""
    ix, ox, X, Q, _, _ = long_lists
    ix.set_nprobe(32)
    ix.set_scan_mode(ix.SCAN_TENSOR)
    a = ix.batch_search_arrays(Q[:600], 10)
    ix.set_scan_mode(1)
    b = ix.batch_search_arrays(Q[:600], 10)
    ix.set_scan_mode(0)
    assert np.array_equal(a[0], b[0])
    assert np.array_equal(a[1].view(np.uint32), b[1].view(np.uint32))


@pytest.mark.parametrize("kc,dim,k", [(1000, 64, 10), (3, 2, 5), (4096, 128, 300),
                                      (500, 17, 500), (1024, 128, 32)])
def test_find_nearest_centroids_matches_oracle(fg, ctx, orc, kc, dim, k):
    rng = np.random.default_rng(kc + dim + k)
    cents = rng.standard_normal((kc, dim)).astype(np.float32)
    cents[kc // 2] = cents[0]  # a duplicate centroid: the lower id comes first
    km = fg.KMeans(kc, 1, ctx)
    km.centroids = cents
    for i in range(6):
        q = rng.standard_normal(dim).astype(np.float32)
        if i == 0:
            q = cents[0] + np.float32(1e-3)
        got = km.find_nearest_centroids(q, k)
        want = orc.find_nearest_centroids(cents, q, k)
        assert np.array_equal(got, want), (kc, dim, k, i)


@pytest.mark.parametrize("n,nlist,m", [(20000, 32, 8), (30000, 128, 16)])
def test_oracle_build_from_engine_draws_is_the_gpu_index(fg, ctx, orc, n, nlist, m):
    """The oracle, given the engine's seeded draws (k-means++ for nlist <= 64,
    random-sample init above), trains the very index the engine builds:
    centroids, codebooks, list layout and codes bit-exact."""
    from forgegpu.datasets import gmm_descriptors
    X = gmm_descriptors(n, components=nlist, seed=nlist)
    ix = fg.IVFPQIndex.build(X, nlist, m, ctx=ctx, seed=99, ivf_sample=8000, pq_sample=6000)
    cents, cb, offs, ids, codes = ix.export()
    draws = orc.engine_build_draws(99, n, nlist, m, ivf_sample=8000, pq_sample=6000)
    ox = orc.OracleIVFPQ.build(X, np.arange(n), nlist, m, *draws)
    assert np.array_equal(cents.view(np.uint32), ox.centroids.view(np.uint32))
    assert np.array_equal(cb.view(np.uint32), ox.codebooks.view(np.uint32))
    assert np.array_equal(offs, ox.offsets)
    assert np.array_equal(ids, ox.ids)
    assert np.array_equal(codes, ox.codes)


@pytest.mark.parametrize("dim,nlist", [(8, 50), (37, 300), (64, 1024), (100, 130), (256, 257),
                                       (128, 2048), (96, 3000), (33, 5000), (128, 16384)])
@pytest.mark.parametrize("nprobe", [1, 7, 64, 200])
def test_tensor_coarse_quantizer_probes_match_oracle(fg, ctx, orc, dim, nlist, nprobe):
    """Batches of 64+ queries pick their probes with the tcgen05 coarse
    quantizer (fp16 GEMM, certified band, exact rescoring; above 2048 lists
    the band is taken by a block per query from memory).  In the exact
    scan mode that is the only approximate step, so any probe that differs
    from find_nearest_partitions (ivf_pq.rs:865-888) shows in the results."""
    if nprobe > nlist:
        pytest.skip("nprobe above nlist")
    rng = np.random.default_rng(dim * 1000 + nlist)
    n = max(4 * nlist, 3000)
    X = (rng.standard_normal((n, dim)) * rng.uniform(0.1, 50)).astype(np.float32)
    Q = X[rng.integers(0, n, 300)] + rng.standard_normal((300, dim)).astype(np.float32)
    m = 1 if dim % 2 else 2
    ix = fg.IVFPQIndex.build(X, nlist, m, ctx=ctx, seed=dim, ivf_sample=min(n, max(6000, 2 * nlist)),
                             pq_sample=min(n, 4000), ivf_iters=4, pq_iters=2)
    ox = _oracle(orc, ix)
    ix.set_scan_mode(1)
    ix.set_nprobe(nprobe)
    ox.set_nprobe(nprobe)
    ids, d, cnt = ix.batch_search_arrays(Q, 10)
    oi, od, oc = ox.batch_search(Q, 10)
    assert_topk_match(ids, d, cnt, oi, od, oc, f"coarse dim={dim} nlist={nlist} p={nprobe}")
    ix.set_scan_mode(0)


def _oracle(orc, ix):
    cents, cb, offs, ids, codes = ix.export()
    return orc.OracleIVFPQ(cents, cb, offs, ids, codes)


@pytest.mark.parametrize("div", [0, 4, 64, 128])
def test_pass1_quota_does_not_change_the_answer(fg, orc, long_lists, div):
    """Every pass-1 sampling quota (every probe's first tile, 1/4 .. 1/128 of
    the probed codes) returns the oracle's answer; it only moves work between
    the two list-scan passes."""
    ix, ox, X, Q, _, _ = long_lists
    ix.set_scan_mode(ix.SCAN_TENSOR)
    ix.set_nprobe(32)
    ox.set_nprobe(32)
    ix.set_pass1_quota(32, div)
    ids, d, cnt = ix.batch_search_arrays(Q, 10)
    oi, od, oc = ox.batch_search(Q, 10)
    assert_topk_match(ids, d, cnt, oi, od, oc, f"pass-1 quota 1/{div}")
    ix.set_scan_mode(0)


def test_pass1_quota_calibrates_on_a_large_batch(fg, ctx, orc):
    """A first batch of 1024+ queries calibrates the quota (timing a sample
    under several quotas) and still returns the oracle's answer."""
    from forgegpu.datasets import gmm_descriptors
    X = gmm_descriptors(60000, components=64, seed=61)
    Q = gmm_descriptors(1500, components=64, seed=62)
    ix = fg.IVFPQIndex.build(X, 64, 16, ctx=ctx, seed=11)
    ix.set_nprobe(16)
    ox = _oracle(orc, ix)
    ox.set_nprobe(16)
    assert ix.pass1_quota(16) is None
    for _ in range(2):
        ids, d, cnt = ix.batch_search_arrays(Q, 10)
        oi, od, oc = ox.batch_search(Q, 10)
        assert_topk_match(ids, d, cnt, oi, od, oc, "calibrated quota")
    assert ix.pass1_quota(16) in (0, 4, 16, 64, 128)
