"""Repeated batch searches of one shape replay a CUDA graph of the device step.

The first call of a shape runs eagerly, the second is captured, later ones
replay the graph.  Replays must return what an eager call returns (and the
oracle's batch_search, src/index/ivf_pq.rs:850-1047), also after the index
changes between calls: a delete (tombstones, ivf_pq.rs:1786-1805) changes
what the replayed kernels read, an insert_batch (:1731-1773) reallocates the
index and forces a new capture.
"""
import ctypes as C

import numpy as np
import pytest

from parity import assert_topk_match

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def fg():
    import forgegpu
    return forgegpu


def _dev(t):
    return C.c_void_p(t.data_ptr())


def test_replayed_searches_match_eager_and_oracle(fg, ctx, orc):
    import torch
    from forgegpu.datasets import gmm_descriptors
    X = gmm_descriptors(30000, components=64, seed=51)
    Q = gmm_descriptors(500, components=64, seed=52)
    ix = fg.IVFPQIndex.build(X, 64, 16, ctx=ctx, seed=9)
    ix.set_nprobe(8)
    cents, cb, offs, ids, codes = ix.export()
    mx = orc.OracleMutableIVFPQ(cents, cb, offs, ids, codes)
    mx.set_nprobe(8)
    L = fg.lib()
    dev = torch.device("cuda", 0)
    k = 10
    dQ = torch.from_numpy(Q).to(dev)
    d_ids = torch.empty((len(Q), k), dtype=torch.int64, device=dev)
    d_d = torch.empty((len(Q), k), dtype=torch.float32, device=dev)
    d_c = torch.empty((len(Q),), dtype=torch.int32, device=dev)
    st = fg.Stats()

    def device_call():
        rc = L.fdb_ivfpq_batch_search_device(ix.h, _dev(dQ), len(Q), k, _dev(d_ids), _dev(d_d),
                                             _dev(d_c), C.byref(st))
        assert rc == 0, L.fdb_last_error()
        return (d_ids.cpu().numpy().astype(np.uint64), d_d.cpu().numpy().copy(),
                d_c.cpu().numpy().astype(np.uint32))

    def check(res, label):
        oi, od, oc = mx.batch_search_arrays(Q, k)
        assert_topk_match(res[0], res[1], res[2], oi, od, oc, label)

    runs = [device_call() for _ in range(4)]  # eager, capture, replay, replay
    for r in runs[1:]:
        assert np.array_equal(r[0], runs[0][0])
        assert np.array_equal(r[1].view(np.uint32), runs[0][1].view(np.uint32))
        assert np.array_equal(r[2], runs[0][2])
    check(runs[0], "eager")
    assert st.kernel_ms > 0.0 and 0 < st.kernel_scores < st.codes_scanned  # timed on replay

    # host buffers, pinned (a capture copies results into them)
    hQ = torch.from_numpy(Q).pin_memory()
    h_ids = torch.empty((len(Q), k), dtype=torch.int64).pin_memory()
    h_d = torch.empty((len(Q), k), dtype=torch.float32).pin_memory()
    h_c = torch.empty((len(Q),), dtype=torch.int32).pin_memory()
    for _ in range(3):
        rc = L.fdb_ivfpq_batch_search(ix.h, _dev(hQ), len(Q), k, _dev(h_ids), _dev(h_d),
                                      _dev(h_c), None)
        assert rc == 0, L.fdb_last_error()
        assert np.array_equal(h_ids.numpy().astype(np.uint64), runs[0][0])
        assert np.array_equal(h_d.numpy().view(np.uint32), runs[0][1].view(np.uint32))

    # tombstones between replays: the replayed kernels read the new rows
    for victim in (int(runs[0][0][0, 0]), int(runs[0][0][1, 0]), int(runs[0][0][2, 0])):
        assert ix.delete(victim) and mx.delete(victim)
        for _ in range(3):
            check(device_call(), f"after deleting {victim}")

    # insert_batch reallocates the index: a new capture, the oracle's answer
    Xn = gmm_descriptors(3000, components=64, seed=53)
    idn = np.arange(10**6, 10**6 + len(Xn), dtype=np.uint64)
    ix.insert_batch(Xn, idn)
    mx.insert_batch(Xn, idn)
    for _ in range(3):
        check(device_call(), "after insert_batch")

    # graphs off: the same answer eagerly
    ix.set_graphs(False)
    eager = device_call()
    ix.set_graphs(True)
    again = device_call()
    assert np.array_equal(eager[0], again[0])
    assert np.array_equal(eager[1].view(np.uint32), again[1].view(np.uint32))


def test_stage_timers_off_keeps_pass2_time_and_answer(fg, ctx, orc):
    """With the stage timers off a call with statistics still reports the
    counters and the list scan's pass-2 time, not the stage times, and the
    answer (replayed or eager) does not change."""
    from forgegpu.datasets import gmm_descriptors
    X = gmm_descriptors(30000, components=64, seed=54)
    Q = gmm_descriptors(600, components=64, seed=55)
    ix = fg.IVFPQIndex.build(X, 64, 16, ctx=ctx, seed=12)
    ix.set_nprobe(8)
    ix.set_scan_mode(ix.SCAN_TENSOR)
    on = ix.batch_search_arrays(Q, 10, stats=True)
    assert on[3].coarse_ms > 0.0 and on[3].kernel_ms > 0.0
    ix.set_stage_timers(False)
    for _ in range(3):  # eager, capture, replay
        off = ix.batch_search_arrays(Q, 10, stats=True)
        assert np.array_equal(off[0], on[0])
        assert np.array_equal(off[1].view(np.uint32), on[1].view(np.uint32))
        assert off[3].coarse_ms == 0.0 and off[3].total_ms == 0.0
        assert off[3].kernel_ms > 0.0 and off[3].kernel_scores == on[3].kernel_scores
    ix.set_stage_timers(True)
    again = ix.batch_search_arrays(Q, 10, stats=True)
    assert again[3].coarse_ms > 0.0
