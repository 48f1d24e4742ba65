"""The sharded (N > 1) search path on CPU ranks: two gloo processes each
own the inverted lists the engine's shard plan gives them, search only those
lists (the oracle stands in for the device scan), exchange their local top-k
lists with all_gather -- the step the engine does with ncclAllGather -- and
merge by (distance, row position).  The merged result must equal the
unsharded search."""
import os
import sys

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

HERE = os.path.dirname(os.path.abspath(__file__))


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    for p in (os.path.join(HERE, "..", "forge-db_b200"), os.path.join(HERE, "..", "oracle")):
        sys.path.insert(0, p)
    import torch
    import forgegpu as fg
    import oracle as O
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = np.load(os.path.join(HERE, "golden", "ivfpq_small.npz"))
        offs = g["offsets"].astype(np.uint64)
        sizes = np.diff(offs)
        owner = fg.shard_plan(sizes, world)
        # this rank's view: lists held elsewhere are empty
        keep = owner == rank
        new_codes, new_ids, new_offs, pos = [], [], [0], []
        for l in range(len(sizes)):
            if keep[l]:
                s, e = int(offs[l]), int(offs[l + 1])
                new_codes.append(g["codes"][s:e]); new_ids.append(g["list_ids"][s:e])
                pos.append(np.arange(s, e, dtype=np.uint64))
            new_offs.append(new_offs[-1] + (int(sizes[l]) if keep[l] else 0))
        codes = np.concatenate(new_codes) if new_codes else np.zeros((0, int(g["m"])), np.uint8)
        ids = np.concatenate(new_ids) if new_ids else np.zeros(0, np.uint64)
        ix = O.OracleIVFPQ(g["centroids"], g["codebooks"], np.array(new_offs, np.uint64),
                           ids, codes)
        ix.set_nprobe(int(g["nprobe"]))
        k = int(g["k"])
        li, ld, lc = ix.batch_search(g["Q"], k, chunk=len(g["Q"]))
        # exchange (distance, id) lists
        t = torch.from_numpy(np.stack([ld.astype(np.float64), li.astype(np.float64)]))
        parts = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(parts, t)
        if rank == 0:
            allp = np.concatenate([p.numpy() for p in parts], axis=2)  # [2, nq, world*k]
            d, i = allp[0], allp[1]
            merged_d = np.full((d.shape[0], k), np.inf)
            merged_i = np.zeros((d.shape[0], k))
            for qq in range(d.shape[0]):
                o = np.lexsort((i[qq], d[qq]))[:k]
                merged_d[qq], merged_i[qq] = d[qq][o], i[qq][o]
            q.put((merged_d, merged_i))
    finally:
        dist.destroy_process_group()


def test_two_rank_shard_merge_equals_unsharded():
    g = np.load(os.path.join(HERE, "golden", "ivfpq_small.npz"))
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + (os.getpid() % 1000)
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    merged_d, merged_i = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want_d = g["batch_d"].astype(np.float64)
    assert np.array_equal(merged_d, want_d)
    for qq in range(want_d.shape[0]):
        assert set(merged_i[qq].astype(np.uint64).tolist()) == set(g["batch_ids"][qq].tolist())
