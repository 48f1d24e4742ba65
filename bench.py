"""Benchmark of the IVF-PQ batch-search hot path (config C: 1M x 128
descriptor-like vectors, nlist 1024, M 16, nprobe 32, 10k queries, k 10).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--nprobe P] [--mode lists|replicas]

One step = one batch_search of the 10k-query batch.  `value` is whole-job
QPS with queries already in HBM (device clock, max over ranks); `e2e` is the
same through the C ABI entry point with pinned host buffers, the query
upload and the result download inside the timed region.  L2 (126 MB) is
flushed between steps by writing a 256 MB buffer outside the timed window,
because the index (16 MB of codes) would otherwise stay L2-resident.  Every
run checks the answer for the whole batch against the oracle (`parity`).

Multi-GPU (torchrun, one rank per GPU): `--mode replicas` (default) holds the
whole index on every rank and gives each rank its own 10k-query batch (weak
scaling; queries are independent, so there is no collective on the data
path).  `--mode lists` gives each rank a share of the inverted lists; every
rank runs the full 10k batch on its lists, the local top-k lists are
exchanged with ncclAllGather inside the engine and merged on every device
(strong scaling: the index and batch are fixed; `shard_parity` checks the
sharded answer against the unsharded one).

`--impl reference` times the reference's CPU path (the oracle's restatement
of IVFPQIndex::batch_search_parallel, all host threads) on a bounded sample.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "forge-db_b200"))

METRIC = "IVF-PQ QPS @ matched recall@10, 1M×128 nprobe=32, 1/2/4/8 B200"
N_BASE, N_QUERY, DIM, NLIST, M, K = 1_000_000, 10_000, 128, 1024, 16, 10
SEED = 2024
WORKLOAD = "ivfpq_config_c"
DATA_NOTE = "seeded GMM descriptor-like (1024 centres U[0,255], sigma 20, clipped, rounded)"
DEFAULT_NPROBE = 32

# IVF-PQ workloads: the headline (config C) and the embedding-scale config D
IVF_CONFIGS = {
    "ivfpq": dict(METRIC=METRIC, N_BASE=1_000_000, N_QUERY=10_000, DIM=128, NLIST=1024, M=16,
                  K=10, WORKLOAD="ivfpq_config_c", DEFAULT_NPROBE=32,
                  DATA_NOTE="seeded GMM descriptor-like (1024 centres U[0,255], sigma 20, "
                            "clipped, rounded)"),
    "ivfpq_d": dict(METRIC="IVF-PQ QPS, 20M×96 unit-norm (cosine), nlist 16384, M 48, nprobe=64",
                    N_BASE=20_000_000, N_QUERY=10_000, DIM=96, NLIST=16384, M=48, K=10,
                    WORKLOAD="ivfpq_config_d", DEFAULT_NPROBE=64,
                    DATA_NOTE="seeded unit-norm N(0,1), 96 dims"),
}


def use_ivf_config(name):
    globals().update(IVF_CONFIGS[name])


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def tensor_peak():
    """Dense bf16/fp16 tensor peak (burst: the kernel runs in short launches)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["bf16_tflops"]), "measured bf16_tflops (dense fp16 has the same rate)"
    except Exception:
        return 1590.0, "fallback"


class ClockSampler:
    """Samples SM clocks and clock-event reasons through NVML while running."""
    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, index: int):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            pass

    def _run(self):
        while not self._stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit and bit != 0x1:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.05)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self.ok:
            self.t.join()

    def summary(self):
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                "samples": len(self.samples)}


def nvml_index(local_rank: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        try:
            return int(vis.split(",")[local_rank])
        except ValueError:
            return local_rank
    return local_rank


def make_data():
    from forgegpu import datasets
    if WORKLOAD == "ivfpq_config_d":
        return datasets.config_d(N_BASE, N_QUERY)
    return datasets.config_c(N_BASE, N_QUERY)


def rank_queries(rank):
    """The query batch of one replica rank: rank 0 takes the N=1 batch, the
    others draw their own from the same distribution (other seeds)."""
    from forgegpu import datasets
    if WORKLOAD == "ivfpq_config_d":
        return datasets.normal(N_QUERY, DIM, seed=10 + 1000 * rank, unit=True)
    return datasets.gmm_descriptors(N_QUERY, seed=7 + 1000 * rank)


SCAN_MODES = {"auto": 0, "exact": 1, "tables": 2, "tensor": 3}
RECALL_QUERIES = 2000  # queries whose recall@10 both arms report
SCALING = "strong"     # the batch and the index are fixed as N grows

# DRAM bytes (read + write) per launch of the dominant kernel, per workload,
# from one ncu capture (dram__bytes_read.sum + dram__bytes_write.sum) of that
# workload at its bench size; None where only a smaller case was captured
# (config D: its traffic does not scale by a known factor).
NCU_TRAFFIC = {"ivfpq_config_c": 87.5e6, "ivfpq_config_d": None, "bf_config_b": None}
# brute force, tensor path: row norms, query to fp16, sample pass, merge, tau,
# filter pass, segment compaction, candidate selection, exact rescore,
# keys->ids, finalize
BF_LAUNCHES = 11


DIST_RTOL, TIE_RTOL = 1e-4, 1e-5  # north_star: distances 1e-4 rel, near-ties 1e-5 rel


def parity_summary(g_ids, g_d, g_cnt, o_ids, o_d, o_cnt):
    """The port's parity contract over a batch, vectorised: result counts
    equal, rows ascending, distances within 1e-4 relative, and every id in
    one answer but not the other within 1e-5 relative of the k-th distance
    (a near-tie).  Reports the share of rows that are identical outright."""
    g_ids = np.asarray(g_ids).astype(np.uint64)
    o_ids = np.asarray(o_ids).astype(np.uint64)
    g_d = np.asarray(g_d, np.float32)
    o_d = np.asarray(o_d, np.float32)
    g_cnt = np.asarray(g_cnt).astype(np.int64)
    o_cnt = np.asarray(o_cnt).astype(np.int64)
    nq, k = o_ids.shape
    count_bad = int((g_cnt != o_cnt).sum())
    valid = np.arange(k)[None, :] < o_cnt[:, None]
    od = np.where(valid, o_d, 0).astype(np.float64)
    gd = np.where(valid, g_d, 0).astype(np.float64)
    rel = np.abs(gd - od) / np.maximum(np.abs(od), 1e-30)
    max_rel = float(rel[valid].max()) if valid.any() else 0.0
    dist_bad = int(((rel > DIST_RTOL) & valid).any(axis=1).sum())
    unsorted = int((np.diff(np.where(valid, g_d, np.inf), axis=1) < 0).any(axis=1).sum())
    exact = (np.where(valid, g_ids == o_ids, True).all(axis=1) &
             np.where(valid, g_d.view(np.uint32) == o_d.view(np.uint32), True).all(axis=1))
    beyond = 0
    near_tie_rows = 0
    for q in np.nonzero(~exact)[0]:
        c = int(o_cnt[q])
        gs, os_ = set(g_ids[q, :c].tolist()), set(o_ids[q, :c].tolist())
        if gs == os_:
            continue
        near_tie_rows += 1
        dk = float(o_d[q, c - 1])
        tol = TIE_RTOL * max(abs(dk), 1e-30)
        dmap = dict(zip(o_ids[q, :c].tolist(), o_d[q, :c].tolist()))
        dmap.update(zip(g_ids[q, :c].tolist(), g_d[q, :c].tolist()))
        beyond += sum(1 for i in gs ^ os_ if abs(dmap[i] - dk) > tol)
    ok = count_bad == 0 and dist_bad == 0 and unsorted == 0 and beyond == 0
    return {"queries": int(nq), "exact_rate": float(exact.mean()) if nq else 1.0,
            "max_rel_dist": max_rel, "rows_dist_beyond_1e-4": dist_bad,
            "rows_count_mismatch": count_bad, "rows_unsorted": unsorted,
            "rows_with_near_tie_swaps": near_tie_rows, "id_mismatch_beyond_ties": beyond,
            "ok": bool(ok)}


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def config_dict(args, world, extra=None):
    d = {"workload": WORKLOAD, "n_base": N_BASE, "dim": DIM, "nlist": NLIST, "m": M,
         "nprobe": args.nprobe,
         "global_batch": N_QUERY * (world if args.mode == "replicas" else 1),
         "queries_per_gpu": N_QUERY, "k": K,
         "data": DATA_NOTE,
         "parallelism": (f"lists{world}" if args.mode == "lists" else f"replicas{world}"),
         "scan_mode": args.scan_mode,
         "l2": "flushed between steps (256 MB write outside the timed window)"}
    if getattr(args, "ivf_sample", 0):
        d["ivf_sample"] = args.ivf_sample
    if getattr(args, "rerank", 0):
        d["rerank_factor"] = args.rerank
    if getattr(args, "filter_every", 0):
        d["filter"] = f"search_filtered, ids divisible by {args.filter_every} allowed"
    if extra:
        d.update(extra)
    return d


# ---------------------------------------------------------------------------
# reference arm: the CPU path of the reference (oracle restatement)
# ---------------------------------------------------------------------------
def run_reference(args, rank, world):
    """The reference's CPU path: the oracle's restatement of
    IVFPQIndex::batch_search_parallel (ivf_pq.rs:1060-1084) on every host
    core, over the index the GPU arm builds (the oracle trains it from the
    same seeded draws, so both arms search identical centroids, codebooks and
    lists; the printed index checksum shows it)."""
    if rank != 0:
        return
    if args.workload not in IVF_CONFIGS or args.rerank or args.filter_every:
        print(json.dumps({"impl": "reference", "workload": args.workload,
                          "unavailable": "the reference arm is defined for the IVF-PQ "
                                         "workloads (configs C and D) without re-ranking "
                                         "or filters"}), flush=True)
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    X, Q = make_data()
    n = X.shape[0]
    threads = O.host_threads()
    t0 = time.time()
    sidx, init, kpp_u, pidx, pinit = O.engine_build_draws(SEED, n, NLIST, M,
                                                          ivf_sample=args.ivf_sample or 30000)
    ix = O.OracleIVFPQ.build(X, np.arange(n), NLIST, M, sidx, init, kpp_u, pidx, pinit,
                             threads=threads)
    build_s = time.time() - t0
    ix.set_nprobe(args.nprobe)
    # size the per-step sample to about 8 s of work
    probe = Q[:256]
    t0 = time.time()
    ix.batch_search(probe, K, threads=threads)
    per_q = (time.time() - t0) / len(probe)
    sample = int(min(N_QUERY, max(256, 8.0 / max(per_q, 1e-9))))
    for w in range(args.warmup):
        ix.batch_search(Q[:min(sample, 256)], K, threads=threads)
    times = []
    for s in range(args.steps):
        off = (s * sample) % max(1, N_QUERY - sample + 1)
        t0 = time.perf_counter()
        ix.batch_search(Q[off:off + sample], K, threads=threads)
        times.append(time.perf_counter() - t0)
    qps = sample * len(times) / sum(times)
    # recall@10 of the same queries the GPU arm scores, against exact L2
    # ground truth (compute_ground_truth, dataset.rs:39-59: brute force)
    from forgegpu.datasets import recall_at_k
    nr = min(N_QUERY, RECALL_QUERIES)
    oi, _, _ = ix.batch_search(Q[:nr], K, threads=threads)
    gt, _, _ = O.bf_batch_search(X, np.arange(n), O.EUCLIDEAN_SQUARED, Q[:nr], K,
                                 threads=threads)
    recall = recall_at_k(oi, gt, K)
    line = {
        "impl": "reference", "metric": METRIC, "value": qps, "unit": "queries/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000 * statistics.mean(times), "higher_is_better": True,
        "scaling": SCALING, "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_dict(args, world),
        "details": {"recall_at_10": recall, "recall_queries": nr,
                    "sample_queries_per_step": sample, "cpu_build_s": round(build_s, 1),
                    "index_crc32": index_checksum(ix.centroids, ix.codebooks, ix.offsets,
                                                  ix.ids, ix.codes)},
        "cpu_baseline": {"value": qps, "unit": "queries/s", "cores": threads, "kind": "port",
                         "cpu_model": cpu_model(),
                         "sample": f"{sample} of the {N_QUERY} queries per step, oracle "
                                   "restatement of batch_search_parallel "
                                   "(ivf_pq.rs:1060-1084), "
                                   f"{threads} OpenMP threads ({cpu_model()}); index trained "
                                   "by the oracle from the GPU arm's seeded draws"},
        "e2e": {"value": qps, "unit": "queries/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def index_checksum(cents, cb, offs, ids, codes):
    """CRC-32 over the trained artefacts (equal checksums: the same index)."""
    import zlib
    c = 0
    for a in (cents, cb, offs, ids, codes):
        c = zlib.crc32(np.ascontiguousarray(a).tobytes(), c)
    return c


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def cpu_baseline_rows(ix, X, Q, args):
    """CPU baselines of the re-ranked and filtered variants: the oracle's
    batch_search_parallel + rerank_results (all threads), or its
    single-query search_filtered loop (one thread, as the reference)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    cents, cb, offs, ids, codes = ix.export()
    ox = O.OracleMutableIVFPQ(cents, cb, offs, ids, codes)
    ox.set_nprobe(args.nprobe)
    if args.rerank:
        ox.enable_reranking(X, np.arange(X.shape[0], dtype=np.uint64), args.rerank)
    threads = O.max_threads()
    if args.filter_every:
        allowed = np.arange(0, X.shape[0], args.filter_every, dtype=np.uint64)
        skip = (ids % args.filter_every != 0).astype(np.uint8)
        f = (K * args.rerank if args.rerank else K) * 4
        oid = np.empty(f, np.uint64)
        od = np.empty(f, np.float32)
        t0 = time.perf_counter()
        nsample = 0
        while time.perf_counter() - t0 < 10.0 and nsample < len(Q):
            q = Q[nsample]
            O.lib().orc_ivfpq_search_skip(ox.centroids, ox.codebooks, ox.nlist, ox.m, ox.dim,
                                          ox.offsets, ox.ids, ox.codes, skip, ox.nprobe, q, f,
                                          oid, od)
            nsample += 1
        dt = time.perf_counter() - t0
        del allowed
        return {"value": nsample / dt, "unit": "queries/s", "cores": 1, "kind": "port",
                "sample": f"first {nsample} queries through the oracle's single-query "
                          "search_filtered (ivf_pq.rs:692-831), one thread"}
    t0 = time.time()
    ox.batch_search_arrays(Q[:256], K, threads=threads)
    per_q = (time.time() - t0) / 256
    sample = int(min(len(Q), max(256, 12.0 / max(per_q, 1e-9))))
    t0 = time.perf_counter()
    ox.batch_search_arrays(Q[:sample], K, threads=threads)
    dt = time.perf_counter() - t0
    return {"value": sample / dt, "unit": "queries/s", "cores": threads, "kind": "port",
            "sample": f"first {sample} of the 10k queries, batch_search_parallel + "
                      f"rerank_results x{args.rerank} (oracle restatement), {threads} threads"}


def oracle_answer(exported, Q, nprobe, timed):
    """The oracle's batch_search over the GPU-built index (its exported
    artefacts) for every query of Q: the parity checker, and, when `timed`,
    the CPU baseline -- a pass over a bounded sample (about 12 s of CPU work)
    timed on every host core; the remaining queries run untimed."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    cents, cb, offs, ids, codes = exported
    ox = O.OracleIVFPQ(cents, cb, offs, ids, codes)
    ox.set_nprobe(nprobe)
    threads = O.host_threads()
    nq = len(Q)
    cb_line = None
    if timed:
        t0 = time.time()
        ox.batch_search(Q[:256], K, threads=threads)
        per_q = (time.time() - t0) / 256
        sample = int(min(nq, max(256, 12.0 / max(per_q, 1e-9))))
        t0 = time.perf_counter()
        oi, od, oc = ox.batch_search(Q[:sample], K, threads=threads)
        dt = time.perf_counter() - t0
        cb_line = {"value": sample / dt, "unit": "queries/s", "cores": threads, "kind": "port",
                   "cpu_model": cpu_model(),
                   "sample": f"first {sample} of the {nq} queries, one batch_search_parallel "
                             "pass (oracle restatement, ivf_pq.rs:1060-1084) over the "
                             f"GPU-built index, {threads} threads ({cpu_model()})"}
    else:
        sample = 0
        oi = np.empty((0, K), np.uint64)
        od = np.empty((0, K), np.float32)
        oc = np.empty(0, np.uint32)
    if sample < nq:
        ri, rd, rc = ox.batch_search(Q[sample:], K, threads=threads)
        oi, od, oc = np.concatenate([oi, ri]), np.concatenate([od, rd]), np.concatenate([oc, rc])
    return cb_line, (oi, od, oc)


def run_ours(args, rank, world, local_rank, dist):
    import ctypes as C
    import torch
    import forgegpu as fg

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    ctx = fg.Context(local_rank)
    if world > 1 and args.mode == "lists":
        uid = [fg.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        ctx.init_comm(rank, world, uid[0])

    X, Q = make_data()
    t0 = time.time()
    ix = fg.IVFPQIndex.build(X, NLIST, M, ctx=ctx, seed=SEED, ivf_sample=args.ivf_sample)
    torch.cuda.synchronize()
    build_s = time.time() - t0
    ix.set_nprobe(args.nprobe)
    ix.set_scan_mode(SCAN_MODES[args.scan_mode])
    if args.rerank:
        ix.enable_reranking(X, np.arange(N_BASE, dtype=np.uint64), args.rerank)
    # the trained artefacts, for the oracle's parity check on rank 0
    exported = ix.export() if rank == 0 else None
    unsharded = None
    if world > 1 and args.mode == "lists":
        # the single-device answer of this rank's index before sharding: the
        # sharded answer must equal it bit for bit (shard_parity)
        if rank == 0 and not (args.rerank or args.filter_every):
            unsharded = ix.batch_search_arrays(Q, K)
        ix.shard(rank, world)
        Qr = Q
    elif world > 1:
        # replicas: the whole index on every rank, a batch of queries per rank
        Qr = Q if rank == 0 else rank_queries(rank)
    else:
        Qr = Q
    nq = Qr.shape[0]

    stream = torch.cuda.ExternalStream(ctx.stream(), device=dev)
    dQ = torch.from_numpy(np.ascontiguousarray(Qr)).to(dev)
    d_ids = torch.empty((nq, K), dtype=torch.int64, device=dev)
    d_d = torch.empty((nq, K), dtype=torch.float32, device=dev)
    d_c = torch.empty((nq,), dtype=torch.int32, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    L = fg.lib()
    st = fg.Stats()

    allowed = None
    if args.filter_every:
        allowed = np.arange(0, N_BASE, args.filter_every, dtype=np.uint64)
        d_allowed = torch.from_numpy(allowed.view(np.int64)).to(dev)
        h_allowed = torch.from_numpy(allowed.view(np.int64)).pin_memory()

    def step_device(stats=True):
        if allowed is not None:
            rc = L.fdb_ivfpq_batch_search_filtered_device(
                ix.h, C.c_void_p(dQ.data_ptr()), nq, K, C.c_void_p(d_allowed.data_ptr()),
                allowed.size, C.c_void_p(d_ids.data_ptr()), C.c_void_p(d_d.data_ptr()),
                C.c_void_p(d_c.data_ptr()), C.byref(st) if stats else None)
        else:
            rc = L.fdb_ivfpq_batch_search_device(ix.h, C.c_void_p(dQ.data_ptr()), nq, K,
                                                 C.c_void_p(d_ids.data_ptr()),
                                                 C.c_void_p(d_d.data_ptr()),
                                                 C.c_void_p(d_c.data_ptr()),
                                                 C.byref(st) if stats else None)
        fg._check(rc)

    # pinned host buffers for the end-to-end path
    hQ = torch.from_numpy(np.ascontiguousarray(Qr)).pin_memory()
    h_ids = torch.empty((nq, K), dtype=torch.int64).pin_memory()
    h_d = torch.empty((nq, K), dtype=torch.float32).pin_memory()
    h_c = torch.empty((nq,), dtype=torch.int32).pin_memory()

    def step_e2e():
        if allowed is not None:
            rc = L.fdb_ivfpq_batch_search_filtered(
                ix.h, C.c_void_p(hQ.data_ptr()), nq, K, C.c_void_p(h_allowed.data_ptr()),
                allowed.size, C.c_void_p(h_ids.data_ptr()), C.c_void_p(h_d.data_ptr()),
                C.c_void_p(h_c.data_ptr()))
        else:
            rc = L.fdb_ivfpq_batch_search(ix.h, C.c_void_p(hQ.data_ptr()), nq, K,
                                          C.c_void_p(h_ids.data_ptr()),
                                          C.c_void_p(h_d.data_ptr()),
                                          C.c_void_p(h_c.data_ptr()), None)
        fg._check(rc)

    for _ in range(max(3, args.warmup)):
        step_device()
        step_e2e()
    torch.cuda.synchronize()
    # In tensor mode the timed steps record only the two events around pass 2
    # (kernel_ms, the roofline's kernel time) besides the counters: every
    # stage mark is an event record inside the replayed step and together
    # they added ~50 us to it.  The stage breakdown comes from one untimed
    # step with all marks after the timed region (details.stage_ms).
    tensor_steps = st.kernel_scores < st.bytes_scanned / M
    if tensor_steps:
        ix.set_stage_timers(False)
        step_device()  # sizes and captures the timed steps' shape
        step_device()
        torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()

    times, scan_ms, bytes_scanned, launches, rescans, extended = [], [], [], 0, [], []
    kern_ms, kern_scores = [], []
    stage = {"coarse_ms": [], "rescore_ms": [], "merge_ms": []}
    # sharded lists: device time inside each collective (waits for the
    # slowest rank included)
    comm_names = ("allgather_probes", "allreduce_tau", "allreduce_dk", "allgather_results")
    comm = {n: [] for n in comm_names}
    # rounds of the exact re-scan: units (query, failed list) at most nq * nprobe,
    # per-unit keys of the fetched k (k x rerank factor, x4 when filtered with
    # re-ranking) within 64 MiB a round
    k_fetch = K * max(1, args.rerank) * (4 if (args.filter_every and args.rerank) else 1)
    units = N_QUERY * args.nprobe
    ucap = max(1, min(units, (64 << 20) // (k_fetch * 8)))
    rescan_rounds = (units + ucap - 1) // ucap
    with ClockSampler(nvml_index(local_rank)) as clk:
        for s in range(args.steps):
            flush.zero_()
            torch.cuda.synchronize()
            if args.profile_range and s == 0:
                torch.cuda.profiler.start()  # for ncu --profile-from-start off
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            step_device()
            e1.record(stream)
            e1.synchronize()
            if args.profile_range and s == 0:
                torch.cuda.profiler.stop()
            times.append(e0.elapsed_time(e1))
            scan_ms.append(st.scan_ms)
            stage["coarse_ms"].append(st.coarse_ms)
            stage["rescore_ms"].append(st.rescore_ms)
            stage["merge_ms"].append(st.merge_ms)
            for i, n in enumerate(comm_names):
                comm[n].append(st.comm_ms[i])
            rescans.append(st.exact_rescans)
            extended.append(st.extended)
            bytes_scanned.append(st.bytes_scanned)
            kern_ms.append(st.kernel_ms)
            kern_scores.append(st.kernel_scores)
            codes = st.bytes_scanned / M
            if st.kernel_scores < codes:
                # tensor mode (own kernels; the CUB sort, scans and selection are
                # library kernels): transpose, coarse, probe selection, pair keys,
                # segment offsets, residual rows, dump-row lengths, item counts and
                # fills (2 + 2), pass 1, pass-1 selection, margin, pruning, pass-2
                # rows, pass 2, shortlist, rescore, certify (2), extend, keys->ids,
                # finalize = 24; the device-driven re-scan: unit offsets, then
                # expand + scan + merge per round of units (launched whether or
                # not any query failed certification)
                launches += 24 + 1 + 3 * rescan_rounds
            else:
                # coarse, select, scan, [rescore (+ exact re-scan)], keys->ids, finalize
                launches += 5 + (1 if st.rescore_ms > 0 else 0) + (1 if st.exact_rescans else 0)
            launches += 2 if (world > 1 and args.mode == "lists") else 0
        e2e_times = []
        for s in range(args.steps):
            flush.zero_()
            torch.cuda.synchronize()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            step_e2e()
            e1.record(stream)
            e1.synchronize()
            e2e_times.append(e0.elapsed_time(e1))
    torch.cuda.synchronize()
    if tensor_steps:
        # the stage breakdown: one untimed step with every stage mark
        ix.set_stage_timers(True)
        step_device()
        torch.cuda.synchronize()
        for k in stage:
            stage[k] = [getattr(st, k)]
        scan_ms = [st.scan_ms]
        for i, n in enumerate(comm_names):
            comm[n] = [st.comm_ms[i]]
    tot = torch.tensor([sum(times), sum(e2e_times)], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.barrier()
        dist.all_reduce(tot, op=dist.ReduceOp.MAX)
    total_ms, total_e2e_ms = float(tot[0]), float(tot[1])
    # queries answered by the whole job per step (replicas: one batch per rank)
    job_queries = N_QUERY * (world if args.mode == "replicas" else 1)
    value = job_queries * args.steps / (total_ms / 1000.0)
    e2e_value = job_queries * args.steps / (total_e2e_ms / 1000.0)

    if rank != 0:
        return
    g_ids = d_ids.cpu().numpy().astype(np.uint64)
    g_d = d_d.cpu().numpy()
    g_c = d_c.cpu().numpy()
    # recall@10 against exact L2 ground truth (BF on the GPU) for the batch
    recall = None
    nr = min(nq, RECALL_QUERIES)
    if True:
        bf = fg.BruteForceIndex(fg.DistanceMetric.EuclideanSquared, ctx).add(X)
        gt, _, _ = bf.batch_search_arrays(Qr[:nr], K)
        from forgegpu.datasets import recall_at_k
        recall = recall_at_k(g_ids[:nr], gt, K)
        bf.close()
    hbm, peak_kind = peaks()
    scan_avg_ms = statistics.mean(scan_ms)
    algo_bytes = statistics.mean(bytes_scanned)
    k_ms = statistics.mean(kern_ms)
    k_scores = statistics.mean(kern_scores)
    # in tensor mode the dominant kernel scores only the pass-2 pairs' codes
    tensor_mode = st.lists_probed > 0 and k_scores < algo_bytes / M
    dpad = (DIM + 63) // 64 * 64
    if tensor_mode:
        # tcgen05 list scan (pass 2): 2 * dpad flops per (query, code) score
        tpk, tkind = tensor_peak()
        flops = 2.0 * dpad * k_scores
        achieved = flops / (k_ms / 1000.0) / 1e12
        roofline = {"bound": "tensor", "achieved": achieved, "peak": tpk, "unit": "TFLOP/s",
                    "frac": achieved / tpk,
                    "traffic": (NCU_TRAFFIC.get(WORKLOAD)
                                if (N_BASE, NLIST) == (IVF_CONFIGS[args.workload]["N_BASE"],
                                                       IVF_CONFIGS[args.workload]["NLIST"])
                                else None),
                    "kernel": "ivf_pass_kernel<FILTER> (tcgen05 fp16 scores of probed lists "
                              "1..nprobe-1 against decoded codes, fused admission test)",
                    "peak_source": tkind, "algorithmic_flops_per_launch": flops,
                    "scores_per_launch": k_scores, "kernel_ms": k_ms,
                    "code_bytes_per_step": algo_bytes,
                    "code_bytes_per_step_over_step_time_gbs":
                        algo_bytes / (total_ms / args.steps / 1000.0) / 1e9}
    else:
        achieved = k_scores * M / (k_ms / 1000.0) / 1e9
        roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                    "frac": achieved / hbm, "traffic": None,
                    "kernel": "scan_kernel (LUT build + code scan + warp top-k)",
                    "peak_source": f"{peak_kind} hbm_gbs",
                    "algorithmic_bytes_per_launch": k_scores * M, "kernel_ms": k_ms}
    line = {
        "metric": METRIC, "value": value, "unit": "queries/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": total_ms / args.steps,
        "higher_is_better": True, "scaling": SCALING, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": config_dict(args, world),
        "details": {
            "recall_at_10": recall, "recall_queries": nr, "build_s": round(build_s, 2),
            "stage_ms": {k: round(statistics.mean(v), 4) for k, v in stage.items()},
            "stage_ms_from": ("one untimed step with every stage mark (the timed steps "
                              "record only the pass-2 events)") if tensor_steps
                             else "the timed steps",
            "pass2_kernel_ms": round(statistics.mean(kern_ms), 4),
            "collective_ms": ({k: round(statistics.mean(v), 4) for k, v in comm.items()}
                              if args.mode == "lists" and world > 1 else None),
            "scan_kernel_ms": round(statistics.mean(scan_ms), 4),
            "exact_rescans_per_step": statistics.mean(rescans),
            "extended_certificates_per_step": statistics.mean(extended),
            "pass1_quota": ix.pass1_quota(args.nprobe) if tensor_mode else None,
            "index_crc32": index_checksum(*exported)},
        "e2e": {"value": e2e_value, "unit": "queries/s",
                "h2d_bytes_per_step": nq * DIM * 4,
                "d2h_bytes_per_step": nq * K * (8 + 4) + nq * 4},
        "gpu_launches": launches,
        "roofline": roofline,
        "clocks": clk.summary(),
    }
    if allowed is not None:
        # the filter's own launches per step: radix sort of the allowed ids
        # (10 passes over 64-bit keys) and the row bitmap
        line["gpu_launches"] += args.steps * 11
        line["e2e"]["h2d_bytes_per_step"] += int(allowed.nbytes)
    # the end-to-end entry point returned the device entry point's answer
    e2e_same = bool(np.array_equal(h_ids.numpy().astype(np.uint64), g_ids) and
                    np.array_equal(h_d.numpy().view(np.uint32), g_d.view(np.uint32)) and
                    np.array_equal(h_c.numpy(), g_c))
    ok = e2e_same
    if args.rerank or args.filter_every:
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_rows(ix, X, Q, args)
    else:
        # parity of every query of the batch with the oracle over the same index
        t0 = time.time()
        cb_line, (oi, od, oc) = oracle_answer(exported, Qr, args.nprobe,
                                              timed=(world == 1 and not args.no_cpu_baseline))
        par = parity_summary(g_ids, g_d, g_c, oi, od, oc)
        par["e2e_answer_identical"] = e2e_same
        par["oracle_s"] = round(time.time() - t0, 1)
        line["parity"] = par
        ok = ok and par["ok"]
        if cb_line is not None:
            line["cpu_baseline"] = cb_line
    if unsharded is not None:
        ui, ud, uc = unsharded
        same = bool(np.array_equal(ui, g_ids) and np.array_equal(ud.view(np.uint32),
                                                                  g_d.view(np.uint32)) and
                    np.array_equal(uc.astype(np.int64), g_c.astype(np.int64)))
        line["shard_parity"] = {"queries": int(nq), "identical_to_unsharded": same}
        ok = ok and same
    print(json.dumps(line), flush=True)
    if not ok:
        print("PARITY FAILURE: the GPU answer differs from the oracle's (see 'parity')",
              file=sys.stderr, flush=True)
        raise SystemExit(3)


def run_ours_bf(args, rank, world, local_rank, dist):
    """Config B: brute force, 1M x 128 N(0,1), 10k queries, k 100 (rows
    sharded across ranks, local top-k exchanged with ncclAllGather)."""
    import ctypes as C
    import torch
    import forgegpu as fg
    from forgegpu import datasets

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    ctx = fg.Context(local_rank)
    if world > 1:
        uid = [fg.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        ctx.init_comm(rank, world, uid[0])
    n, nq, k = args.bf_n, args.bf_nq, 100
    X = datasets.normal(n, DIM, seed=3)
    Q = datasets.normal(nq, DIM, seed=4)
    metric = {"l2sq": 1, "dot": 3, "cosine": 2, "l2": 0}[args.bf_metric]
    bf = fg.BruteForceIndex(metric, ctx).add(X)
    if world > 1:
        bf.shard(rank, world)
    stream = torch.cuda.ExternalStream(ctx.stream(), device=dev)
    dQ = torch.from_numpy(Q).to(dev)
    d_ids = torch.empty((nq, k), dtype=torch.int64, device=dev)
    d_d = torch.empty((nq, k), dtype=torch.float32, device=dev)
    d_c = torch.empty((nq,), dtype=torch.int32, device=dev)
    L = fg.lib()
    st = fg.Stats()

    def step():
        fg._check(L.fdb_bf_batch_search_device(bf.h, C.c_void_p(dQ.data_ptr()), nq, k,
                                               C.c_void_p(d_ids.data_ptr()),
                                               C.c_void_p(d_d.data_ptr()),
                                               C.c_void_p(d_c.data_ptr()), C.byref(st)))

    hQ = torch.from_numpy(Q).pin_memory()
    h_ids = torch.empty((nq, k), dtype=torch.int64).pin_memory()
    h_d = torch.empty((nq, k), dtype=torch.float32).pin_memory()
    h_c = torch.empty((nq,), dtype=torch.int32).pin_memory()

    def step_e2e():
        fg._check(L.fdb_bf_batch_search(bf.h, C.c_void_p(hQ.data_ptr()), nq, k,
                                        C.c_void_p(h_ids.data_ptr()), C.c_void_p(h_d.data_ptr()),
                                        C.c_void_p(h_c.data_ptr()), None))

    for _ in range(max(3, args.warmup)):
        step()
    step_e2e()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    times, scan_ms, rescans, e2e_times = [], [], [], []
    with ClockSampler(nvml_index(local_rank)) as clk:
        for i in range(args.steps):
            if args.profile_range and i == 0:
                torch.cuda.profiler.start()  # for ncu --profile-from-start off
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            step()
            e1.record(stream)
            e1.synchronize()
            if args.profile_range and i == 0:
                torch.cuda.profiler.stop()
            times.append(e0.elapsed_time(e1))
            scan_ms.append(st.kernel_ms)
            rescans.append(st.exact_rescans)
        for _ in range(args.steps):
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            step_e2e()
            e1.record(stream)
            e1.synchronize()
            e2e_times.append(e0.elapsed_time(e1))
    tot = torch.tensor([sum(times), sum(e2e_times)], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.barrier()
        dist.all_reduce(tot, op=dist.ReduceOp.MAX)
    if rank != 0:
        return
    flops = 2.0 * nq * (n // world) * DIM
    scan_avg = statistics.mean(scan_ms)
    achieved = flops / (scan_avg / 1000.0) / 1e12
    peak = 1670.2
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak = float(json.load(f)["bf16_tflops"])
    except Exception:
        pass
    line = {
        "metric": "BruteForce batch QPS, 1M x 128, k=100", "value": nq * args.steps / (float(tot[0]) / 1000),
        "unit": "queries/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": float(tot[0]) / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f16 shortlist / f32 exact rescore", "data": "synthetic",
        "config": {"workload": "bf_config_b", "n_base": n, "dim": DIM, "global_batch": nq, "k": k,
                   "metric": args.bf_metric, "parallelism": f"rows{world}",
                   "exact_rescans_per_step": statistics.mean(rescans),
                   "filter_kernel_ms": round(scan_avg, 4),
                   "l2": "not flushed: the fp16 rows (256 MB) exceed L2 every step"},
        "gpu_launches": BF_LAUNCHES * args.steps,
        "e2e": {"value": nq * args.steps / (float(tot[1]) / 1000), "unit": "queries/s",
                "h2d_bytes_per_step": nq * DIM * 4, "d2h_bytes_per_step": nq * k * 12 + nq * 4},
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak,
                     "traffic": (NCU_TRAFFIC.get("bf_config_b")
                                 if (n, nq, args.bf_metric) == (1_000_000, 10_000, "l2sq") else None),
                     "kernel": "gemm_topk_kernel<FILTER> (tcgen05 fp16 GEMM + fused admission test)",
                     "peak_source": "measured bf16_tflops (dense fp16 has the same rate)",
                     "kernel_ms": scan_avg},
        "clocks": clk.summary(),
    }
    # parity with the oracle's brute force (brute_force.rs:180-225) on a
    # bounded sample of the batch (about 15 s of CPU work on every host core)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    threads = O.host_threads()
    g_ids = d_ids.cpu().numpy().astype(np.uint64)
    g_d = d_d.cpu().numpy()
    g_c = d_c.cpu().numpy()
    ids_all = np.arange(n, dtype=np.uint64)
    t0 = time.time()
    O.bf_batch_search(X, ids_all, metric, Q[:32], k, threads=threads)
    per_q = (time.time() - t0) / 32
    ns = int(min(nq, max(200, 15.0 / max(per_q, 1e-9))))
    t0 = time.perf_counter()
    oi, od, oc = O.bf_batch_search(X, ids_all, metric, Q[:ns], k, threads=threads)
    cpu_s = time.perf_counter() - t0
    par = parity_summary(g_ids[:ns], g_d[:ns], g_c[:ns], oi, od, oc)
    par["sample"] = f"first {ns} of the {nq} queries"
    line["parity"] = par
    line["cpu_baseline"] = {"value": ns / cpu_s,
                            "unit": "queries/s", "cores": threads, "kind": "port",
                            "cpu_model": cpu_model(),
                            "sample": f"first {ns} queries through the oracle's batch_search "
                                      f"(brute_force.rs:180-225), {threads} threads"}
    print(json.dumps(line), flush=True)
    if not par["ok"]:
        print("PARITY FAILURE: brute-force answer differs from the oracle's", file=sys.stderr,
              flush=True)
        raise SystemExit(3)


def run_ours_train(args, rank, world, local_rank, dist):
    """Config E: k-means of 1M x 768 unit-norm rows into 4096 centroids (20 Lloyd
    iterations from a seeded random-sample init), PQ training with M = 96 on a
    100k-row sample, and encoding of all 1M rows, through the public API (host
    buffers in and out).  One run per step; every rank runs the whole job
    (training is replicated, 'replicas').  Bit-exactness at this size is
    checked by properties on a sample (oracle assignment and encoding)."""
    import torch
    import forgegpu as fg
    from forgegpu import datasets

    torch.cuda.set_device(local_rank)
    ctx = fg.Context(local_rank)
    n, dim, k, iters, m = 1_000_000, 768, 4096, 20, 96
    X = datasets.config_e(n)
    init = fg.sample_indices(12, n, k)
    pq_rows = fg.sample_indices(13, n, 100_000)
    Xs = np.ascontiguousarray(X[pq_rows])
    pq_init = np.concatenate([fg.sample_indices(14 + s, len(Xs), 256) for s in range(m)])

    def job():
        t = {}
        t0 = time.perf_counter()
        km = fg.KMeans(k, iters, ctx).fit(X, init_idx=init)
        t["kmeans_s"] = time.perf_counter() - t0
        t1 = time.perf_counter()
        pq = fg.ProductQuantizer.train(Xs, m, init_idx=pq_init, iters=25, ctx=ctx)
        t["pq_train_s"] = time.perf_counter() - t1
        t2 = time.perf_counter()
        codes = pq.encode(X)
        t["encode_s"] = time.perf_counter() - t2
        t["total_s"] = time.perf_counter() - t0
        return km, pq, codes, t

    for _ in range(min(args.warmup, 1)):  # one untimed run (module load, allocations)
        job()
    if dist is not None:
        dist.barrier()
    runs = []
    with ClockSampler(nvml_index(local_rank)) as clk:
        for _ in range(max(1, min(args.steps, 3))):
            torch.cuda.synchronize()
            km, pq, codes, t = job()
            runs.append(t)
    tot = torch.tensor([max(r["total_s"] for r in runs)], dtype=torch.float64,
                       device=torch.device("cuda", local_rank))
    if dist is not None:
        dist.all_reduce(tot, op=dist.ReduceOp.MAX)
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    rng = np.random.default_rng(15)
    sample = np.sort(rng.choice(n, 2000, replace=False))
    assign_ok = bool(np.array_equal(O.assign(X[sample], km.centroids), km.assignments[sample]))
    codes_ok = bool(np.array_equal(O.pq_encode(pq.codebooks, X[sample]), codes[sample]))
    # CPU baseline: the oracle's assignment step on a bounded sample, scaled to
    # the full job's assignment work (20 iterations over 1M rows)
    threads = O.max_threads()
    cs = 4000
    t0 = time.perf_counter()
    O.assign(X[:cs], km.centroids, threads=threads)
    dt = time.perf_counter() - t0
    cpu_est = dt * (n / cs) * iters
    mean = {key: statistics.mean(r[key] for r in runs) for key in runs[0]}
    line = {
        "metric": "Training wall time: k-means 1M×768 -> 4096 (20 iters) + PQ M 96 + encode 1M",
        "value": float(tot[0]), "unit": "s", "n_gpus": world, "steps": len(runs),
        "warmup": 1, "ms_per_step": 1000 * float(tot[0]), "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "train_config_e", "n": n, "dim": dim, "k": k, "iters": iters,
                   "pq_m": m, "pq_sample": len(Xs), "kmeans_iters_run": km.iters,
                   "data": "seeded unit-norm N(0,1), 768 dims",
                   "parallelism": f"replicas{world}", "phase_s": mean,
                   "sample_checks": {"assignments_match_oracle": assign_ok,
                                     "codes_match_oracle": codes_ok, "rows": len(sample)}},
        "e2e": {"value": float(tot[0]), "unit": "s", "h2d_bytes_per_step": int(X.nbytes * 2 + Xs.nbytes),
                "d2h_bytes_per_step": int(k * dim * 4 + n * 4 + n * m)},
        "gpu_launches": None,
        "cpu_baseline": {"value": cpu_est, "unit": "s", "cores": threads, "kind": "port",
                         "sample": f"oracle assignment of {cs} rows to the 4096 centroids, "
                                   f"scaled to {iters} iterations over {n} rows (assignment only)"},
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def run_ours_insert(args, rank, world, local_rank, dist):
    """insert_batch (ivf_pq.rs:1731-1773): a config C index built on the
    first N - n vectors takes the last n in one call (assignment, residual
    PQ encoding, list re-layout and the derived tables on the device).  One
    step = one insert_batch of n vectors into a fresh copy of the index."""
    import torch
    import forgegpu as fg
    if world > 1:
        raise SystemExit("the insert workload runs on one GPU")
    torch.cuda.set_device(local_rank)
    ctx = fg.Context(local_rank)
    X, Q = make_data()
    n_new = args.insert_n
    base, new = X[:-n_new], X[-n_new:]
    new_ids = np.arange(N_BASE - n_new, N_BASE, dtype=np.uint64)
    path = os.path.join("/tmp", f"fdb_insert_base_{os.getpid()}.fdb")
    ix = fg.IVFPQIndex.build(base, NLIST, M, ctx=ctx, seed=SEED)
    ix.save(path)  # each step inserts into a fresh copy of the same index
    t0 = time.perf_counter()
    fg.IVFPQIndex.load(path, ctx=ctx).close()
    load_s = time.perf_counter() - t0
    times = []
    with ClockSampler(nvml_index(local_rank)) as clk:
        for s_ in range(args.warmup + args.steps):
            cp = fg.IVFPQIndex.load(path, ctx=ctx)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            cp.insert_batch(new, new_ids)
            torch.cuda.synchronize()
            dt = time.perf_counter() - t0
            if s_ >= args.warmup:
                times.append(dt)
            if s_ == args.warmup + args.steps - 1:
                last = cp
            else:
                cp.close()
    os.remove(path)
    # parity sample: the inserted rows' codes against the oracle's encoding
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    cents, cb, offs, ids, codes = last.export()
    pos = np.searchsorted(np.sort(ids), new_ids[:2000])
    order = np.argsort(ids)
    rows = order[pos]
    a = O.assign(new[:2000], cents)
    resid = (new[:2000] - cents[a]).astype(np.float32)
    ok = bool(np.array_equal(O.pq_encode(cb, resid), codes[rows]))
    # CPU baseline: the reference's insert_batch is one vector at a time on
    # one thread: nearest centroid, residual, encode
    cs = 3000
    t0 = time.perf_counter()
    a = O.assign(new[:cs], cents, threads=1)
    O.pq_encode(cb, (new[:cs] - cents[a]).astype(np.float32), threads=1)
    cpu = cs / (time.perf_counter() - t0)
    mean_s = statistics.mean(times)
    line = {
        "metric": "insert_batch throughput into the config C index (vectors/s)",
        "value": n_new / mean_s, "unit": "vectors/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000 * mean_s, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "ivfpq_insert", "n_base": N_BASE - n_new, "n_insert": n_new,
                   "dim": DIM, "nlist": NLIST, "m": M, "data": DATA_NOTE,
                   "timing": "wall clock around the call, device synchronised on both sides "
                             "(the call includes host steps: list offsets, id mirror)",
                   "load_fdb_s": round(load_s, 3),
                   "sample_checks": {"inserted_codes_match_oracle": ok, "rows": 2000}},
        "e2e": {"value": n_new / mean_s, "unit": "vectors/s",
                "h2d_bytes_per_step": int(new.nbytes + new_ids.nbytes),
                "d2h_bytes_per_step": int(n_new * 4)},
        "gpu_launches": None,
        "cpu_baseline": {"value": cpu, "unit": "vectors/s", "cores": 1, "kind": "port",
                         "sample": f"oracle nearest-centroid + residual encode of {cs} "
                                   "vectors on one thread (insert_batch's per-vector loop, "
                                   "without the list appends)"},
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--nprobe", type=int, default=None,
                    help="default: 32 (config C), 64 (config D)")
    ap.add_argument("--mode", default="replicas", choices=["lists", "replicas"],
                    help="multi-GPU: replicas (default; the index on every rank, a batch "
                         "of queries per rank, weak scaling, no collective) or lists (the "
                         "inverted lists sharded, the batch broadcast, local top-k lists "
                         "exchanged by ncclAllGather and merged; strong scaling)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-range", action="store_true",
                    help="bracket the first timed step with cudaProfilerStart/Stop "
                         "(for ncu --profile-from-start off)")
    ap.add_argument("--scan-mode", default="auto", choices=list(SCAN_MODES),
                    help="IVF-PQ scan mode (auto picks the tensor-core list scan here)")
    ap.add_argument("--workload", default="ivfpq",
                    choices=["ivfpq", "ivfpq_d", "bf", "train", "insert"],
                    help="ivfpq: config C (the headline); ivfpq_d: config D; bf: config B; "
                         "train: config E (k-means 1M x 768 -> 4096, PQ M 96, encode); "
                         "insert: insert_batch into a config C index")
    ap.add_argument("--rerank", type=int, default=0,
                    help="IVF-PQ: enable_reranking with this rerank_factor (fetch k*F, "
                         "exact sqrt(L2^2) re-ranking on the device)")
    ap.add_argument("--filter-every", type=int, default=0,
                    help="IVF-PQ: batch search_filtered with the ids divisible by this "
                         "number allowed")
    ap.add_argument("--insert-n", type=int, default=100_000,
                    help="insert workload: vectors inserted into the config C index")
    ap.add_argument("--bf-metric", default="l2sq", choices=["l2sq", "dot", "cosine", "l2"])
    ap.add_argument("--bf-n", type=int, default=1_000_000, help="rows (smaller for profiling)")
    ap.add_argument("--bf-nq", type=int, default=10_000, help="queries (smaller for profiling)")
    ap.add_argument("--n-base", type=int, default=None,
                    help="IVF-PQ: database rows (a smaller case of the workload, for profiling)")
    ap.add_argument("--nlist", type=int, default=None, help="IVF-PQ: lists (with --n-base)")
    ap.add_argument("--ivf-sample", type=int, default=0,
                    help="IVF-PQ: k-means training sample (default: the reference's)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.workload in IVF_CONFIGS:
        use_ivf_config(args.workload)
        if args.n_base:
            globals()["N_BASE"] = args.n_base
        if args.nlist:
            globals()["NLIST"] = args.nlist
    if args.nprobe is None:
        args.nprobe = DEFAULT_NPROBE
    global SCALING
    SCALING = "weak" if args.mode == "replicas" else "strong"

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    import torch
    if world > 1:
        import datetime
        import torch.distributed as tdist
        torch.cuda.set_device(local_rank)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                 device_id=torch.device("cuda", local_rank))
        dist = tdist
    try:
        if args.workload == "bf":
            run_ours_bf(args, rank, world, local_rank, dist)
        elif args.workload == "train":
            run_ours_train(args, rank, world, local_rank, dist)
        elif args.workload == "insert":
            run_ours_insert(args, rank, world, local_rank, dist)
        else:
            run_ours(args, rank, world, local_rank, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
