"""Failure detection, tested without faulting, trapping or hanging a GPU.

- A bounded device wait runs out: a test hook makes the list-scan kernel
  issue nothing, so its consumers wait on a ring flag that nothing sets.
  They give up after the context's wait limit, drain (nothing is in flight),
  free their tensor memory and return; the call reports FDB_ERR_TIMEOUT and
  the next call on the same context matches the oracle.
- search_with_timeout (src/index/ivf_pq.rs:1369-1455): results equal to
  search() within the deadline, Timeout past it.
- A rank that never joins: NCCL initialisation with a deadline gives up and
  reports FDB_ERR_TIMEOUT (host-side bootstrap only; no collective and no
  kernel runs).  It runs in a child process bounded by a timeout.
"""
import os
import subprocess
import sys
import time

import numpy as np
import pytest

from parity import assert_topk_match

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def fg():
    import forgegpu
    return forgegpu


@pytest.fixture(scope="module")
def own(fg, orc):
    """A context of its own (wait limits and the stall hook are per context)
    and a GMM index on it, with the oracle over the same artefacts."""
    from forgegpu.datasets import gmm_descriptors
    ctx = fg.Context(0)
    X = gmm_descriptors(30000, components=64, seed=41)
    Q = gmm_descriptors(400, components=64, seed=42)
    ix = fg.IVFPQIndex.build(X, 64, 16, ctx=ctx, seed=5)
    ix.set_scan_mode(ix.SCAN_TENSOR)
    ix.set_nprobe(8)
    cents, cb, offs, ids, codes = ix.export()
    ox = orc.OracleIVFPQ(cents, cb, offs, ids, codes)
    ox.set_nprobe(8)
    return ctx, ix, ox, Q


@pytest.mark.parametrize("stalls", [1, 2])
def test_bounded_wait_runs_out_and_the_context_recovers(fg, own, stalls):
    ctx, ix, ox, Q = own
    ctx.set_wait_limit(0.05)
    ctx.test_stall_scans(stalls)  # pass 1 (and, with 2, pass 2) issues nothing
    t0 = time.time()
    with pytest.raises(fg.ForgeGpuError) as e:
        ix.batch_search_arrays(Q, 10)
    assert e.value.kind == "Timeout", e.value
    assert time.time() - t0 < 30
    ctx.set_wait_limit(2.0)
    ids, d, cnt = ix.batch_search_arrays(Q, 10)
    oi, od, oc = ox.batch_search(Q, 10)
    assert_topk_match(ids, d, cnt, oi, od, oc, "after a timeout")


def test_search_with_timeout(fg, own):
    ctx, ix, ox, Q = own
    want = ix.search(Q[0], 10)
    got, elapsed = ix.search_with_timeout(Q[0], 10, 30.0)
    assert got == want and 0.0 < elapsed < 30.0
    with pytest.raises(fg.ForgeGpuError) as e:
        ix.search_with_timeout(Q[0], 10, 0.0)
    assert e.value.kind == "Timeout"
    ids, d, cnt, el = ix.batch_search_with_timeout_arrays(Q, 10, 60.0)
    wi, wd, wc = ix.batch_search_arrays(Q, 10)
    assert np.array_equal(ids, wi) and np.array_equal(d.view(np.uint32), wd.view(np.uint32))
    assert np.array_equal(cnt, wc) and el > 0.0
    # past the deadline (the exact scan mode: the deadline is checked on the
    # host when the results come back; the tensor path's device waits are
    # made to run out by the stall hook above, with nothing in flight)
    ix.set_scan_mode(1)
    with pytest.raises(fg.ForgeGpuError) as e:
        ix.batch_search_with_timeout_arrays(Q, 10, 1e-7)
    assert e.value.kind == "Timeout"
    ix.set_scan_mode(ix.SCAN_TENSOR)
    # the deadline of one call does not outlive it
    ids2, d2, cnt2 = ix.batch_search_arrays(Q, 10)
    assert np.array_equal(ids2, wi)


_ABSENT_RANK = r"""
import sys, time
sys.path.insert(0, %r)
import forgegpu as fg
ctx = fg.Context(0)
uid = fg.nccl_unique_id()
t0 = time.time()
try:
    ctx.init_comm(0, 2, uid, timeout_s=3.0)   # rank 1 never comes
    print("JOINED")
except fg.ForgeGpuError as e:
    print("KIND", e.kind, round(time.time() - t0, 1))
# the context works without a communicator
import numpy as np
X = np.random.default_rng(0).random((2000, 32), dtype=np.float32)
bf = fg.BruteForceIndex(fg.DistanceMetric.EuclideanSquared, ctx).add(X)
ids, d, cnt = bf.batch_search_arrays(X[:4], 1)
print("SEARCH", ids[:, 0].tolist())
"""


def test_comm_init_gives_up_when_a_rank_is_absent():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    code = _ABSENT_RANK % os.path.join(ROOT, "forge-db_b200")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=180,
                       env=env)
    assert r.returncode == 0, r.stderr[-3000:]
    lines = dict(l.split(" ", 1) for l in r.stdout.strip().splitlines() if " " in l)
    assert "KIND" in lines, r.stdout
    kind, secs = lines["KIND"].split()
    assert kind == "Timeout" and float(secs) < 60
    assert lines["SEARCH"] == "[0, 1, 2, 3]"
