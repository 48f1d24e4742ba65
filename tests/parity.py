"""Parity helpers shared by the tests.

The engine and the oracle compute the same f32 operations in the same order,
so distances are expected to be bit-identical; the assertions below are the
looser contract of the port (distances within 1e-4 relative; top-k ids
identical except at near-ties, |d - d_k| <= 1e-5 relative to the k-th
distance), and the exact-match rate is reported beside them.
"""
import numpy as np

DIST_RTOL = 1e-4
TIE_RTOL = 1e-5


def assert_topk_match(g_ids, g_d, g_cnt, o_ids, o_d, o_cnt, label=""):
    g_ids = np.atleast_2d(g_ids); o_ids = np.atleast_2d(o_ids)
    g_d = np.atleast_2d(g_d); o_d = np.atleast_2d(o_d)
    g_cnt = np.atleast_1d(g_cnt); o_cnt = np.atleast_1d(o_cnt)
    assert np.array_equal(g_cnt, o_cnt), f"{label}: result counts differ"
    exact = 0
    for q in range(g_ids.shape[0]):
        c = int(o_cnt[q])
        gd, od = g_d[q, :c], o_d[q, :c]
        assert np.all(np.diff(gd) >= 0), f"{label}: query {q} not sorted ascending"
        scale = np.maximum(np.abs(od), 1e-30)
        assert np.all(np.abs(gd - od) <= DIST_RTOL * scale + 1e-30), \
            f"{label}: query {q} distances differ:\n{gd}\n{od}"
        gs, os_ = set(g_ids[q, :c].tolist()), set(o_ids[q, :c].tolist())
        if gs != os_ and c > 0:
            dk = float(od[c - 1])
            tol = TIE_RTOL * max(abs(dk), 1e-30)
            gmap = dict(zip(g_ids[q, :c].tolist(), gd.tolist()))
            omap = dict(zip(o_ids[q, :c].tolist(), od.tolist()))
            for i in gs ^ os_:
                d = gmap.get(i, omap.get(i))
                assert abs(d - dk) <= tol, f"{label}: query {q} id {i} (d={d}) differs away from the k-th distance {dk}"
        if np.array_equal(gd, od) and np.array_equal(g_ids[q, :c], o_ids[q, :c]):
            exact += 1
        # padding
        assert np.all(g_ids[q, c:] == np.iinfo(np.uint64).max)
        assert np.all(np.isinf(g_d[q, c:]))
    return exact / max(1, g_ids.shape[0])
