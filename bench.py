"""Benchmark of the IVF-PQ batch-search hot path (config C: 1M x 128
descriptor-like vectors, nlist 1024, M 16, nprobe 32, 10k queries, k 10).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--nprobe P] [--mode lists|replicas]

One step = one batch_search of the 10k-query batch.  `value` is whole-job
QPS with queries already in HBM (device clock, max over ranks); `e2e` is the
same through the C ABI entry point with pinned host buffers, the query
upload and the result download inside the timed region.  L2 (126 MB) is
flushed between steps by writing a 256 MB buffer outside the timed window,
because the index (16 MB of codes) would otherwise stay L2-resident.

Multi-GPU (torchrun, one rank per GPU): `--mode lists` (default) gives each
rank a share of the inverted lists; every rank runs the full query batch on
its lists, the local top-k lists are exchanged with ncclAllGather inside the
engine and merged on every device (strong scaling: the index and batch are
fixed).  `--mode replicas` holds the whole index on every rank and splits
the queries (no collective).

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
    X, Q = datasets.config_c(N_BASE, N_QUERY)
    return X, Q


SCAN_MODES = {"auto": 0, "exact": 1, "tables": 2, "tensor": 3}

# DRAM bytes (read + write) per launch of the dominant kernel on the default
# workload, from one ncu capture (dram__bytes_read.sum + dram__bytes_write.sum).
NCU_TRAFFIC = {"ivf_pass_filter": 322.4e6, "bf_gemm_filter": None}
# brute force, tensor path: row norms, query to fp16, sample pass, merge, tau,
# filter pass, candidate selection, exact rescore, keys->ids, finalize
BF_LAUNCHES = 10


def config_dict(args, world, extra=None):
    d = {"workload": "ivfpq_config_c", "n_base": N_BASE, "dim": DIM, "nlist": NLIST, "m": M,
         "nprobe": args.nprobe, "global_batch": N_QUERY, "k": K,
         "data": "seeded GMM descriptor-like (1024 centres U[0,255], sigma 20, clipped, rounded)",
         "parallelism": (f"lists{world}" if args.mode == "lists" else f"replicas{world}"),
         "scan_mode": args.scan_mode,
         "l2": "flushed between steps (256 MB write outside the timed window)"}
    if extra:
        d.update(extra)
    return d


# ---------------------------------------------------------------------------
# reference arm: the CPU path of the reference (oracle restatement)
# ---------------------------------------------------------------------------
def run_reference(args, rank, world):
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    X, Q = make_data()
    rng = np.random.default_rng(SEED)
    n = X.shape[0]
    t0 = time.time()
    threads = O.max_threads()
    ix = O.OracleIVFPQ.build(
        X, np.arange(n), NLIST, M, rng.permutation(n)[:30000].astype(np.uint32),
        rng.permutation(30000)[:NLIST].astype(np.uint32), None,
        rng.permutation(n)[:100000].astype(np.uint32),
        np.concatenate([rng.permutation(100000)[:256] for _ in range(M)]).astype(np.uint32),
        threads=threads)
    build_s = time.time() - t0
    ix.set_nprobe(args.nprobe)
    # size the per-step sample to ~8 s of work
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
    line = {
        "impl": "reference", "metric": METRIC, "value": qps, "unit": "queries/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000 * statistics.mean(times), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_dict(args, world, {"sample_queries_per_step": sample,
                                            "cpu_build_s": round(build_s, 1)}),
        "cpu_baseline": {"value": qps, "unit": "queries/s", "cores": threads, "kind": "port",
                         "sample": f"{sample} of the 10k queries per step, oracle restatement "
                                   "of batch_search_parallel (ivf_pq.rs:1060-1084), "
                                   f"{threads} OpenMP threads; index trained by the oracle"},
        "e2e": {"value": qps, "unit": "queries/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def cpu_baseline(ix, Q, nprobe):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    cents, cb, offs, ids, codes = ix.export()
    ox = O.OracleIVFPQ(cents, cb, offs, ids, codes)
    ox.set_nprobe(nprobe)
    threads = O.max_threads()
    t0 = time.time()
    ox.batch_search(Q[:256], K, threads=threads)
    per_q = (time.time() - t0) / 256
    sample = int(min(len(Q), max(256, 12.0 / max(per_q, 1e-9))))
    t0 = time.perf_counter()
    oi, od, oc = ox.batch_search(Q[:sample], K, threads=threads)
    dt = time.perf_counter() - t0
    return {"value": sample / dt, "unit": "queries/s", "cores": threads, "kind": "port",
            "sample": f"first {sample} of the 10k queries, one batch_search_parallel pass "
                      "(oracle restatement, ivf_pq.rs:1060-1084) over the GPU-built index"}, \
        (oi, od, oc, sample)


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
    ix = fg.IVFPQIndex.build(X, NLIST, M, ctx=ctx, seed=SEED)
    torch.cuda.synchronize()
    build_s = time.time() - t0
    ix.set_nprobe(args.nprobe)
    ix.set_scan_mode(SCAN_MODES[args.scan_mode])
    if world > 1 and args.mode == "lists":
        ix.shard(rank, world)
        Qr = Q
    elif world > 1:
        lo, hi = N_QUERY * rank // world, N_QUERY * (rank + 1) // world
        Qr = Q[lo:hi]
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

    def step_device(stats=True):
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
        rc = L.fdb_ivfpq_batch_search(ix.h, C.c_void_p(hQ.data_ptr()), nq, K,
                                      C.c_void_p(h_ids.data_ptr()), C.c_void_p(h_d.data_ptr()),
                                      C.c_void_p(h_c.data_ptr()), None)
        fg._check(rc)

    for _ in range(max(3, args.warmup)):
        step_device()
        step_e2e()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()

    times, scan_ms, bytes_scanned, launches, rescans = [], [], [], 0, []
    kern_ms, kern_scores = [], []
    stage = {"coarse_ms": [], "rescore_ms": [], "merge_ms": []}
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
            rescans.append(st.exact_rescans)
            bytes_scanned.append(st.bytes_scanned)
            kern_ms.append(st.kernel_ms)
            kern_scores.append(st.kernel_scores)
            codes = st.bytes_scanned / M
            if st.kernel_scores < codes:
                # tensor mode: transpose + coarse, select, pair keys, radix sort (4),
                # segment offsets, residual rows, dump rows, scan (2), items, pass 1,
                # pass-1 selection, pass 2, shortlist, certify, [exact re-scan],
                # keys->ids, finalize
                launches += 21 + (1 if st.exact_rescans else 0)
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
    tot = torch.tensor([sum(times), sum(e2e_times)], dtype=torch.float64, device=dev)
    if dist is not None:
        dist.barrier()
        dist.all_reduce(tot, op=dist.ReduceOp.MAX)
    total_ms, total_e2e_ms = float(tot[0]), float(tot[1])
    value = N_QUERY * args.steps / (total_ms / 1000.0)
    e2e_value = N_QUERY * args.steps / (total_e2e_ms / 1000.0)

    if rank != 0:
        return
    # recall@10 against exact L2 ground truth (BF on the GPU) for the batch
    ids_h = d_ids.cpu().numpy().astype(np.uint64)
    recall = None
    if world == 1 or args.mode == "lists":
        bf = fg.BruteForceIndex(fg.DistanceMetric.EuclideanSquared, ctx).add(X)
        gt, _, _ = bf.batch_search_arrays(Q[:2000], K)
        from forgegpu.datasets import recall_at_k
        recall = recall_at_k(ids_h[:2000], gt, K)
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
                    "frac": achieved / tpk, "traffic": NCU_TRAFFIC.get("ivf_pass_filter"),
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
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": config_dict(args, world, {
            "recall_at_10": recall, "build_s": round(build_s, 2),
            "stage_ms": {k: round(statistics.mean(v), 4) for k, v in stage.items()},
            "scan_kernel_ms": round(statistics.mean(scan_ms), 4),
            "exact_rescans_per_step": statistics.mean(rescans)}),
        "e2e": {"value": e2e_value, "unit": "queries/s",
                "h2d_bytes_per_step": nq * DIM * 4,
                "d2h_bytes_per_step": nq * K * (8 + 4) + nq * 4},
        "gpu_launches": launches,
        "roofline": roofline,
        "clocks": clk.summary(),
    }
    if world == 1 and not args.no_cpu_baseline:
        cb, _ = cpu_baseline(ix, Q, args.nprobe)
        line["cpu_baseline"] = cb
    print(json.dumps(line), flush=True)


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
                     "frac": achieved / peak, "traffic": None,
                     "kernel": "gemm_topk_kernel<FILTER> (tcgen05 fp16 GEMM + fused admission test)",
                     "peak_source": "measured bf16_tflops (dense fp16 has the same rate)",
                     "kernel_ms": scan_avg},
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--nprobe", type=int, default=32)
    ap.add_argument("--mode", default="lists", choices=["lists", "replicas"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile-range", action="store_true",
                    help="bracket the first timed step with cudaProfilerStart/Stop "
                         "(for ncu --profile-from-start off)")
    ap.add_argument("--scan-mode", default="auto", choices=list(SCAN_MODES),
                    help="IVF-PQ scan mode (auto picks the tensor-core list scan here)")
    ap.add_argument("--workload", default="ivfpq", choices=["ivfpq", "bf"])
    ap.add_argument("--bf-metric", default="l2sq", choices=["l2sq", "dot", "cosine", "l2"])
    ap.add_argument("--bf-n", type=int, default=1_000_000, help="rows (smaller for profiling)")
    ap.add_argument("--bf-nq", type=int, default=10_000, help="queries (smaller for profiling)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

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
        else:
            run_ours(args, rank, world, local_rank, dist)
    finally:
        if dist is not None:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
