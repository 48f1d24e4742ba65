"""Sharded search on two GPUs: each process owns one device and a share of
the inverted lists (or brute-force rows); local top-k lists are exchanged
with ncclAllGather inside the engine and merged on every device.  The merged
result must be identical to the single-GPU result (row positions break
ties, so the split cannot change the answer).  Skipped with fewer than two
GPUs."""
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


def _rank_main(rank, world, q_in, q_out):
    try:
        sys.path.insert(0, os.path.join(HERE, "..", "forge-db_b200"))
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        import forgegpu as fg
        ctx = fg.Context(rank)
        if rank == 0:
            uid = fg.nccl_unique_id()
            for _ in range(world - 1):
                q_in.put(uid)
        else:
            uid = q_in.get(timeout=60)
        ctx.init_comm(rank, world, uid)
        rng = np.random.default_rng(1)
        X = rng.random((20000, 64), dtype=np.float32)
        Q = np.random.default_rng(2).random((257, 64), dtype=np.float32)
        ix = fg.IVFPQIndex.build(X, 64, 8, ctx=ctx, seed=7)
        ix.set_nprobe(16)
        modes = (ix.SCAN_AUTO, ix.SCAN_TABLES, ix.SCAN_TENSOR)
        single, sharded = [], []
        for mode in modes:  # before sharding: the whole index
            ix.set_scan_mode(mode)
            single += list(ix.batch_search_arrays(Q, 20))
        ix.shard(rank, world)
        part_len = len(ix)
        for mode in modes:
            ix.set_scan_mode(mode)
            sharded += list(ix.batch_search_arrays(Q, 20))
        bf = fg.BruteForceIndex(fg.DistanceMetric.DotProduct, ctx).add(X)
        bf_single = bf.batch_search_arrays(Q, 100)
        bf.shard(rank, world)
        bf_sharded = bf.batch_search_arrays(Q, 100)
        q_out.put((rank, part_len, single, sharded, bf_single, bf_sharded))
    except Exception as e:  # report instead of hanging the parent
        q_out.put((rank, "error", repr(e), None, None, None))


def test_two_gpu_sharded_search_equals_single():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q_in, q_out = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, q_in, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r = q_out.get(timeout=300)
        res[r[0]] = r
    for p in procs:
        p.join(timeout=120)
    for r in range(2):
        assert res[r][1] != "error", res[r][2]
    assert res[0][1] + res[1][1] == 20000  # every vector held exactly once
    for r in range(2):
        _, _, single, sharded, bfs, bfsh = res[r]
        for a, b in zip(single, sharded):
            assert np.array_equal(a, b)
        for a, b in zip(bfs, bfsh):
            assert np.array_equal(a, b)
