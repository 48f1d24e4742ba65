"""Parity of the index's state around the scan, on the GPU through the C ABI:
.fdb files, re-ranking, tombstones, compaction, insert_batch, filtered
search, brute-force removal and rebuild (src/index/ivf_pq.rs:513-831,
1731-1890, 1970-1994; src/index/brute_force.rs:254-385), against the
oracle's restatement (OracleMutableIVFPQ, fdb_format)."""
import os

import numpy as np
import pytest

import fdb_format as F
from parity import assert_topk_match

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))
U64MAX = np.iinfo(np.uint64).max
MODES = [1, 2, 3]  # EXACT, TABLES, TENSOR


@pytest.fixture(scope="module")
def fg():
    import forgegpu
    return forgegpu


@pytest.fixture(scope="module")
def small():
    return np.load(os.path.join(HERE, "golden", "ivfpq_small.npz"))


def _pair(fg, ctx, orc, g, nprobe=4):
    args = (g["centroids"], g["codebooks"], g["offsets"], g["list_ids"], g["codes"])
    ix = fg.IVFPQIndex.from_trained(*args, ctx=ctx)
    ox = orc.OracleMutableIVFPQ(*args)
    ix.set_nprobe(nprobe)
    ox.set_nprobe(nprobe)
    return ix, ox


def _arrays(results, k):
    nq = len(results)
    ids = np.full((nq, k), U64MAX, np.uint64)
    d = np.full((nq, k), np.inf, np.float32)
    cnt = np.zeros(nq, np.uint32)
    for q, (i, dd) in enumerate(results):
        ids[q, :len(i)] = i
        d[q, :len(dd)] = dd
        cnt[q] = len(i)
    return ids, d, cnt


def _single(fg_results):
    return ([r[0] for r in fg_results], [r[1] for r in fg_results])


def _check_batch(ix, ox, Q, k, label):
    ids, d, cnt = ix.batch_search_arrays(Q, k)
    oi, od, oc = _arrays(ox.batch_search(Q, k), k)
    return assert_topk_match(ids, d, cnt, oi, od, oc, label)


def _check_single(ix, ox, Q, k, label, step=7):
    for q in range(0, len(Q), step):
        g = _arrays([_single(ix.search(Q[q], k))], k)
        o = _arrays([ox.search(Q[q], k)], k)
        assert_topk_match(*g, *o, f"{label} q={q}")


# ---------------------------------------------------------------------------
# .fdb files
# ---------------------------------------------------------------------------
def test_golden_files_load_and_write_back_unchanged(fg, ctx, orc, tmp_path):
    for name, cls in (("ivfpq_tiny.fdb", fg.IVFPQIndex), ("bf_tiny.fdb", fg.BruteForceIndex)):
        src = os.path.join(HERE, "golden", name)
        ix = cls.load(src, ctx=ctx)
        out = str(tmp_path / name)
        ix.save(out)
        assert open(out, "rb").read() == open(src, "rb").read(), name


def test_golden_ivfpq_file_searches_like_the_oracle(fg, ctx, orc):
    src = os.path.join(HERE, "golden", "ivfpq_tiny.fdb")
    d = F.decode_ivfpq(F.split_file(open(src, "rb").read(), F.IVFPQ)[4])
    ix = fg.IVFPQIndex.load(src, ctx=ctx)
    assert ix.nprobe() == d["nprobe"] == 3 and ix.dim() == 8 and len(ix) == 40
    ox = orc.OracleMutableIVFPQ(d["centroids"], d["codebooks"], d["offsets"], d["ids"],
                                d["codes"])
    ox.nprobe = d["nprobe"]
    ox.enable_reranking(d["rerank"][1], d["rerank"][0], d["rerank_factor"])
    Q = np.random.default_rng(3).normal(size=(60, 8)).astype(np.float32)
    for k in (1, 4, 10):
        _check_batch(ix, ox, Q, k, f"tiny batch k={k}")
        _check_single(ix, ox, Q, k, f"tiny single k={k}", step=5)


def test_golden_bf_file(fg, ctx, orc, tmp_path):
    src = os.path.join(HERE, "golden", "bf_tiny.fdb")
    metric, ids, X = F.decode_bf(F.split_file(open(src, "rb").read(), F.BRUTE_FORCE)[4])
    bf = fg.BruteForceIndex.load(src, ctx=ctx)
    assert len(bf) == ids.size and bf.dimension() == X.shape[1]
    Q = np.random.default_rng(4).normal(size=(20, X.shape[1])).astype(np.float32)
    g = bf.batch_search_arrays(Q, 5)
    o = orc.bf_batch_search(X, ids, metric, Q, 5)
    assert_topk_match(*g, *o, "bf file")


def test_build_save_load_roundtrip(fg, ctx, orc, small, tmp_path):
    """test_persistence_roundtrip (ivf_pq.rs:2137-2175), plus the payload
    checked against the exported arrays and a byte-identical second save."""
    g = small
    ix = fg.IVFPQIndex.build(g["X"], int(g["nlist"]), int(g["m"]), ids=g["ids"], ctx=ctx,
                             seed=17)
    ix.set_nprobe(4)
    a = str(tmp_path / "a.fdb")
    ix.save(a)
    d = F.decode_ivfpq(F.split_file(open(a, "rb").read(), F.IVFPQ)[4])
    cents, cb, offs, ids, codes = ix.export()
    assert np.array_equal(d["centroids"], cents) and np.array_equal(d["codebooks"], cb)
    assert np.array_equal(d["offsets"], offs) and np.array_equal(d["ids"], ids)
    assert np.array_equal(d["codes"], codes)
    assert d["nprobe"] == 4 and d["metric"] == 0 and d["rerank"] is None
    assert d["rerank_factor"] == 1 and d["consumed"] == len(F.split_file(open(a, "rb").read())[4])
    # a centroid whose cluster ever had members carries its list index as id
    assert (d["cent_ids"] == np.arange(int(g["nlist"]))).mean() > 0.5
    assert (d["cb_ids"] == np.arange(d["cb_ids"].size) % 256).mean() > 0.5
    lx = fg.IVFPQIndex.load(a, ctx=ctx)
    assert lx.nprobe() == 4 and len(lx) == len(ix) and lx.n_partitions() == ix.n_partitions()
    r1 = ix.batch_search_arrays(g["Q"], 10)
    r2 = lx.batch_search_arrays(g["Q"], 10)
    for x, y in zip(r1, r2):
        assert np.array_equal(x, y)
    b = str(tmp_path / "b.fdb")
    lx.save(b)
    assert open(a, "rb").read() == open(b, "rb").read()


def test_load_rejects_corrupt_and_wrong_type(fg, ctx, tmp_path):
    raw = bytearray(open(os.path.join(HERE, "golden", "ivfpq_tiny.fdb"), "rb").read())
    raw[-3] ^= 0x40
    p = tmp_path / "bad.fdb"
    p.write_bytes(bytes(raw))
    with pytest.raises(fg.ForgeGpuError) as e:
        fg.IVFPQIndex.load(str(p), ctx=ctx)
    assert e.value.kind == "ChecksumMismatch"
    with pytest.raises(fg.ForgeGpuError) as e:
        fg.IVFPQIndex.load(os.path.join(HERE, "golden", "bf_tiny.fdb"), ctx=ctx)
    assert e.value.kind == "InvalidFormat"
    with pytest.raises(fg.ForgeGpuError) as e:
        fg.BruteForceIndex.load(os.path.join(HERE, "golden", "ivfpq_tiny.fdb"), ctx=ctx)
    assert e.value.kind == "InvalidFormat"


# ---------------------------------------------------------------------------
# re-ranking
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("factor,k", [(1, 10), (4, 10), (10, 10), (3, 1), (2, 100)])
def test_rerank_parity(fg, ctx, orc, small, factor, k, tmp_path):
    g = small
    ix, ox = _pair(fg, ctx, orc, g)
    # originals for 90% of the rows: candidates without one are dropped
    keep = np.random.default_rng(8).random(g["X"].shape[0]) < 0.9
    ix.enable_reranking(g["X"][keep], g["ids"][keep], factor)
    ox.enable_reranking(g["X"][keep], g["ids"][keep], factor)
    Q = g["Q"]
    rate = _check_batch(ix, ox, Q, k, f"rerank f={factor} k={k}")
    assert rate > 0.9
    _check_single(ix, ox, Q, k, f"rerank single f={factor} k={k}")
    # test_persistence_with_reranking (ivf_pq.rs:2178-2210)
    p = str(tmp_path / "r.fdb")
    ix.save(p)
    lx = fg.IVFPQIndex.load(p, ctx=ctx)
    for x, y in zip(ix.batch_search_arrays(Q, k), lx.batch_search_arrays(Q, k)):
        assert np.array_equal(x, y)


def test_rerank_fetch_limit(fg, ctx, orc, small):
    ix, _ = _pair(fg, ctx, orc, small)
    ix.enable_reranking(small["X"], small["ids"], 30)
    with pytest.raises(fg.ForgeGpuError) as e:
        ix.batch_search_arrays(small["Q"][:4], 10)  # fetch_k 300 > FDB_MAX_K
    assert e.value.kind == "NotSupported"


# ---------------------------------------------------------------------------
# tombstones, compaction, insert_batch
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("mode", MODES)
def test_delete_skips_rows_in_every_scan_mode(fg, ctx, orc, small, mode):
    g = small
    ix, ox = _pair(fg, ctx, orc, g, nprobe=6)
    ix.set_scan_mode(mode)
    rng = np.random.default_rng(31)
    victims = rng.choice(g["ids"], 400, replace=False).tolist()
    for v in victims:
        assert ix.delete(v) == ox.delete(v) == True
    assert ix.delete(victims[0]) is False and ox.delete(victims[0]) is False
    assert ix.delete(10 ** 9) is False
    assert ix.num_tombstones() == ox.num_tombstones() == 400
    assert len(ix) == ox.len() == g["X"].shape[0] - 400
    assert ix.len_with_tombstones() == g["X"].shape[0]
    assert abs(ix.fragmentation_ratio() - 400 / (g["X"].shape[0] - 400)) < 1e-6
    Q = np.concatenate([g["Q"]] * 8)  # 320 queries: the tensor path's batch size
    for k in (1, 10, 32):
        _check_batch(ix, ox, Q, k, f"tombstones mode={mode} k={k}")
    _check_single(ix, ox, g["Q"], 10, f"tombstones single mode={mode}")
    # deleted vectors never come back (queries at the deleted points)
    dead = set(victims)
    ids, _, cnt = ix.batch_search_arrays(g["X"][np.isin(g["ids"], victims)], 10)
    assert not any(int(i) in dead for q in range(ids.shape[0]) for i in ids[q, :cnt[q]])


def test_delete_with_duplicate_ids_and_tensor_short_lists(fg, ctx, orc):
    """An id held in two lists is tombstoned list by list (ivf_pq.rs:1786-1805);
    lists left with fewer than 64 live codes still search exactly."""
    rng = np.random.default_rng(12)
    X = rng.random((3000, 32), dtype=np.float32)
    ids = np.arange(3000, dtype=np.uint64) % 2900  # ids 0..99 appear twice
    ix = fg.IVFPQIndex.build(X, 16, 8, ids=ids, ctx=ctx, seed=4)
    cents, cb, offs, lids, codes = ix.export()
    ox = orc.OracleMutableIVFPQ(cents, cb, offs, lids, codes)
    ix.set_nprobe(5)
    ox.set_nprobe(5)
    for v in list(range(0, 100, 3)) + list(range(0, 100, 3)) + list(range(0, 100, 3)):
        assert ix.delete(v) == ox.delete(v)
    # empty most of one list
    l0 = lids[int(offs[3]):int(offs[4])].tolist()
    for v in l0[:-10]:
        assert ix.delete(v) == ox.delete(v)
    assert ix.num_tombstones() == ox.num_tombstones()
    assert len(ix) == ox.len()
    Q = rng.random((300, 32), dtype=np.float32)
    for mode in MODES:
        ix.set_scan_mode(mode)
        _check_batch(ix, ox, Q, 10, f"dup ids mode={mode}")


def test_compact_matches_oracle(fg, ctx, orc, small):
    g = small
    ix, ox = _pair(fg, ctx, orc, g)
    for v in np.random.default_rng(2).choice(g["ids"], 700, replace=False).tolist():
        ix.delete(v)
        ox.delete(v)
    ix.compact()
    ox.compact()
    cents, cb, offs, ids, codes = ix.export()
    assert np.array_equal(offs, ox.offsets) and np.array_equal(ids, ox.ids)
    assert np.array_equal(codes, ox.codes)
    assert ix.num_tombstones() == 0 and len(ix) == ix.len_with_tombstones() == ox.len()
    for mode in MODES:
        ix.set_scan_mode(mode)
        _check_batch(ix, ox, np.concatenate([g["Q"]] * 8), 10, f"compact mode={mode}")


def test_insert_batch_matches_oracle(fg, ctx, orc, small):
    g = small
    ix, ox = _pair(fg, ctx, orc, g)
    rng = np.random.default_rng(5)
    victims = rng.choice(g["ids"], 200, replace=False)
    for v in victims.tolist():
        ix.delete(v)
        ox.delete(v)
    # new vectors: fresh ids, and 50 tombstoned ids coming back
    Xn = rng.random((900, g["X"].shape[1]), dtype=np.float32)
    idn = np.concatenate([np.arange(10 ** 7, 10 ** 7 + 850, dtype=np.uint64), victims[:50]])
    ix.insert_batch(Xn, idn)
    ox.insert_batch(Xn, idn)
    cents, cb, offs, ids, codes = ix.export()
    assert np.array_equal(offs, ox.offsets) and np.array_equal(ids, ox.ids)
    assert np.array_equal(codes, ox.codes)
    assert ix.num_tombstones() == ox.num_tombstones() and len(ix) == ox.len()
    Q = np.concatenate([g["Q"], Xn[:280]])
    for mode in MODES:
        ix.set_scan_mode(mode)
        _check_batch(ix, ox, Q, 10, f"insert mode={mode}")
    _check_single(ix, ox, Q, 10, "insert single", step=13)


def test_insert_into_reranked_index(fg, ctx, orc, small):
    g = small
    ix, ox = _pair(fg, ctx, orc, g)
    ix.enable_reranking(g["X"], g["ids"], 4)
    ox.enable_reranking(g["X"], g["ids"], 4)
    rng = np.random.default_rng(6)
    Xn = rng.random((300, g["X"].shape[1]), dtype=np.float32)
    idn = np.arange(5 * 10 ** 6, 5 * 10 ** 6 + 300, dtype=np.uint64)
    ix.insert_batch(Xn, idn)
    ox.insert_batch(Xn, idn)
    for v in g["ids"][:50].tolist():
        ix.delete(v)
        ox.delete(v)
    _check_batch(ix, ox, np.concatenate([g["Q"], Xn[:40]]), 10, "insert+rerank")


# ---------------------------------------------------------------------------
# filtered search
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("rerank", [False, True])
@pytest.mark.parametrize("mode", [0, 3])  # AUTO (tables / exact here), TENSOR forced
def test_search_filtered_matches_oracle(fg, ctx, orc, small, rerank, mode):
    g = small
    ix, ox = _pair(fg, ctx, orc, g, nprobe=8)
    ix.set_scan_mode(mode)
    if rerank:
        ix.enable_reranking(g["X"], g["ids"], 3)
        ox.enable_reranking(g["X"], g["ids"], 3)
    for v in g["ids"][::11].tolist():  # tombstones and a filter together
        ix.delete(v)
        ox.delete(v)
    # "category == electronics" for one id in three (test_search_filtered,
    # ivf_pq.rs:2229-2262), plus ids that are not in the index at all
    allowed = np.concatenate([g["ids"][g["ids"] % 3 == 0], np.arange(5, 50, dtype=np.uint64)])
    Q = g["Q"]
    for k in (1, 10):
        rows = [_single(ix.search_filtered(Q[q], k, allowed)) for q in range(len(Q))]
        orows = [ox.search_filtered(Q[q], k, allowed) for q in range(len(Q))]
        assert_topk_match(*_arrays(rows, k), *_arrays(orows, k), f"filtered k={k}")
        allowed_set = set(allowed.tolist())
        assert all(i in allowed_set for r in rows for i in r[0])
        bi, bd, bc = ix.batch_search_filtered_arrays(Q, k, allowed)
        assert_topk_match(bi, bd, bc, *_arrays(rows, k), f"batch filtered k={k}")
    assert ix.search_filtered(Q[0], 10, []) == []
    assert ix.search_filtered(Q[0], 10, [10 ** 12]) == []


# ---------------------------------------------------------------------------
# brute force removal, rebuild
# ---------------------------------------------------------------------------
def test_bf_remove_swap_semantics_and_file(fg, ctx, orc, tmp_path):
    rng = np.random.default_rng(7)
    X = rng.normal(size=(500, 24)).astype(np.float32)
    ids = np.arange(500, dtype=np.uint64) + 1000
    bf = fg.BruteForceIndex(fg.DistanceMetric.Cosine, ctx=ctx).add(X, ids)
    hx, hid = X.copy(), list(ids.tolist())
    for v in [1000, 1499, 1250, 1250, 77]:
        got = bf.remove(v)
        if v in hid:  # VectorStore::swap_remove (vector.rs:256-270)
            i = hid.index(v)
            hid[i] = hid[-1]
            hx[i] = hx[len(hid) - 1]
            hid.pop()
            hx = hx[:len(hid)]
            assert got
        else:
            assert not got
    assert len(bf) == len(hid) == 497
    Q = rng.normal(size=(40, 24)).astype(np.float32)
    g = bf.batch_search_arrays(Q, 7)
    o = orc.bf_batch_search(hx, np.array(hid, np.uint64), 2, Q, 7)
    assert_topk_match(*g, *o, "bf after remove")
    p = str(tmp_path / "bf.fdb")
    bf.save(p)
    assert open(p, "rb").read() == F.file_bytes(F.BRUTE_FORCE,
                                                F.encode_bf(2, np.array(hid, np.uint64), hx))


def test_rebuild_equals_a_fresh_build(fg, ctx, small):
    g = small
    ix = fg.IVFPQIndex.from_trained(g["centroids"], g["codebooks"], g["offsets"],
                                    g["list_ids"], g["codes"], ctx=ctx)
    with pytest.raises(fg.ForgeGpuError) as e:
        ix.rebuild(seed=9)
    assert e.value.kind == "NotSupported"
    ix.set_nprobe(5)
    ix.enable_reranking(g["X"], g["ids"], 2)
    ix.rebuild(seed=9)
    fresh = fg.IVFPQIndex.build(g["X"], int(g["nlist"]), int(g["m"]), ids=g["ids"], ctx=ctx,
                                seed=9)
    for a, b in zip(ix.export(), fresh.export()):
        assert np.array_equal(a, b)
    assert ix.nprobe() == 5
    fresh.set_nprobe(5)
    fresh.enable_reranking(g["X"], g["ids"], 2)
    for a, b in zip(ix.batch_search_arrays(g["Q"], 10), fresh.batch_search_arrays(g["Q"], 10)):
        assert np.array_equal(a, b)


# ---------------------------------------------------------------------------
# IVFPQIndexBuilder
# ---------------------------------------------------------------------------
def test_builder_builds_like_the_reference(fg, ctx, orc):
    """test_builder_basic / test_builder_with_reranking (ivf_pq_builder.rs:
    367-420) on the device, against IVFPQIndex::build and the oracle."""
    rng = np.random.default_rng(14)
    X = rng.random((500, 32), dtype=np.float32)
    ix = (fg.IVFPQIndexBuilder().vectors(X).num_clusters(8).num_subvectors(4).nprobe(4)
          .build(ctx=ctx, seed=3))
    assert ix.n_partitions() == 8 and ix.nprobe() == 4 and len(ix) == 500
    same = fg.IVFPQIndex.build(X, 8, 4, ctx=ctx, seed=3)
    for a, b in zip(ix.export(), same.export()):
        assert np.array_equal(a, b)
    rx = (fg.IVFPQIndexBuilder().vectors(X).num_clusters(8).num_subvectors(4)
          .enable_reranking(True).rerank_factor(10).build(ctx=ctx, seed=3))
    ox = orc.OracleMutableIVFPQ(*rx.export())
    ox.enable_reranking(X, np.arange(500, dtype=np.uint64), 10)
    Q = rng.random((30, 32), dtype=np.float32)
    for q in Q:
        res = rx.search(q, 10)
        assert len(res) == 10
        assert_topk_match(*_arrays([_single(res)], 10), *_arrays([ox.search(q, 10)], 10),
                          "builder rerank")


def test_batch_search_filtered_device_entry(fg, ctx, orc, small):
    """The device-buffer filtered entry returns what the host entry does."""
    import ctypes as C
    import torch
    g = small
    ix, _ = _pair(fg, ctx, orc, g, nprobe=8)
    ix.enable_reranking(g["X"], g["ids"], 2)
    allowed = g["ids"][g["ids"] % 4 == 1]
    Q = np.concatenate([g["Q"]] * 8)  # 320 queries: the tensor path in AUTO mode
    hi, hd, hc = ix.batch_search_filtered_arrays(Q, 10, allowed)
    dev = torch.device("cuda", ctx.device)
    dQ = torch.from_numpy(np.ascontiguousarray(Q)).to(dev)
    da = torch.from_numpy(allowed.view(np.int64)).to(dev)
    di = torch.empty((len(Q), 10), dtype=torch.int64, device=dev)
    dd = torch.empty((len(Q), 10), dtype=torch.float32, device=dev)
    dc = torch.empty(len(Q), dtype=torch.int32, device=dev)
    st = fg.Stats()
    fg._check(fg.lib().fdb_ivfpq_batch_search_filtered_device(
        ix.h, C.c_void_p(dQ.data_ptr()), len(Q), 10, C.c_void_p(da.data_ptr()), allowed.size,
        C.c_void_p(di.data_ptr()), C.c_void_p(dd.data_ptr()), C.c_void_p(dc.data_ptr()),
        C.byref(st)))
    assert np.array_equal(di.cpu().numpy().view(np.uint64), hi)
    assert np.array_equal(dd.cpu().numpy(), hd) and np.array_equal(dc.cpu().numpy(), hc)
    assert st.lists_probed > 0
    # no allowed id: padding only
    fg._check(fg.lib().fdb_ivfpq_batch_search_filtered_device(
        ix.h, C.c_void_p(dQ.data_ptr()), len(Q), 10, None, 0, C.c_void_p(di.data_ptr()),
        C.c_void_p(dd.data_ptr()), C.c_void_p(dc.data_ptr()), None))
    assert (dc.cpu().numpy() == 0).all() and torch.isinf(dd).all()


@pytest.mark.parametrize("k", [33, 40, 64])
def test_tensor_mode_k_above_32(fg, ctx, orc, small, k):
    """k in 33..64 (re-ranked fetch sizes) on the tensor path: the shortlist
    of 64 is certified or re-scanned, results equal the oracle's."""
    g = small
    ix, ox = _pair(fg, ctx, orc, g, nprobe=6)
    ix.set_scan_mode(3)
    Q = np.concatenate([g["Q"]] * 8)
    _check_batch(ix, ox, Q, k, f"tensor k={k}")
