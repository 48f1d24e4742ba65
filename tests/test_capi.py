"""The C ABI library loads and exports every symbol include/forgegpu.h
declares; host-only entry points work without a GPU; device entry points
fail cleanly (an error code, not a crash) where no GPU is visible."""
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    src = open(os.path.join(ROOT, "include", "forgegpu.h")).read()
    return sorted(set(re.findall(r"\b(fdb_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    import forgegpu as fg
    L = fg.lib()
    declared = header_symbols()
    assert len(declared) >= 40
    for name in declared:
        assert hasattr(L, name), name
    assert set(declared) == set(fg.exported_symbols())


def test_torch_imports_after_the_library():
    # the library and torch must resolve to one libnccl.so.2; loading the
    # library first used to break torch's import with missing NCCL symbols
    import subprocess
    import sys
    code = ("import sys; sys.path.insert(0, %r); import forgegpu as fg; fg.lib(); "
            "import torch; print('ok')" % os.path.join(ROOT, "forge-db_b200"))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0 and r.stdout.strip().endswith("ok"), r.stderr[-2000:]


def test_version_and_error_string():
    import forgegpu as fg
    assert fg.lib().fdb_version() >= 100
    assert isinstance(fg.lib().fdb_last_error(), bytes)


def test_seeded_draws_deterministic():
    import forgegpu as fg
    a = fg.sample_indices(42, 1000, 100)
    b = fg.sample_indices(42, 1000, 100)
    assert np.array_equal(a, b)
    assert len(set(a.tolist())) == 100 and a.max() < 1000
    full = fg.sample_indices(7, 50, 50)
    assert sorted(full.tolist()) == list(range(50))
    u = fg.uniform_draws(1, 1000)
    assert np.all((u >= 0) & (u < 1))
    assert np.all(u * (1 << 23) == np.floor(u * (1 << 23)))  # on the 2^-23 grid
    with pytest.raises(fg.ForgeGpuError):
        fg.sample_indices(1, 10, 11)


def test_oracle_restates_the_engine_draws(orc):
    """The oracle's splitmix64 restatement gives the engine's default build
    draws, so the reference arm can train the index the GPU arm trains."""
    import forgegpu as fg
    for seed, n, take in [(2024, 1_000_000, 3000), (0, 50, 50), ((1 << 64) - 2, 977, 13)]:
        assert np.array_equal(orc.splitmix_sample_indices(seed, n, take),
                              fg.sample_indices(seed, n, take))
    assert np.array_equal(orc.splitmix_uniform(99, 257).view(np.uint32),
                          fg.uniform_draws(99, 257).view(np.uint32))
    sidx, init, kpp, pidx, pinit = orc.engine_build_draws(5, 40000, 32, 4, ivf_sample=3000,
                                                          pq_sample=2000)
    assert np.array_equal(sidx, fg.sample_indices(5, 40000, 3000))
    assert kpp is not None and kpp.size == 32 and init.max() < 3000
    assert np.array_equal(pidx, fg.sample_indices(7, 40000, 2000))
    assert np.array_equal(pinit[256:512], fg.sample_indices(9, 2000, 256))


def test_shard_plan_covers_every_list_once():
    import forgegpu as fg
    rng = np.random.default_rng(0)
    sizes = rng.integers(0, 5000, 1024).astype(np.uint64)
    for world in (1, 2, 4, 8):
        owner = fg.shard_plan(sizes, world)
        assert owner.min() >= 0 and owner.max() < world
        loads = np.bincount(owner, weights=sizes.astype(np.float64), minlength=world)
        # greedy largest-first keeps every device within one list of the mean
        assert loads.max() - loads.min() <= sizes.max()


def test_no_gpu_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    import forgegpu as fg
    with pytest.raises(fg.ForgeGpuError) as e:
        fg.Context(0)
    assert e.value.code in (-1, -7)


def test_tuning_switches_reject_null_handles():
    """The switches and deadlines of the C ABI fail with FDB_ERR_INVALID_ARG
    on a NULL handle (no device needed)."""
    import ctypes as C
    import forgegpu as fg
    L = fg.lib()
    div = C.c_int64()
    calls = [
        lambda: L.fdb_ivfpq_set_stage_timers(None, 0),
        lambda: L.fdb_ivfpq_set_graphs(None, 1),
        lambda: L.fdb_ivfpq_set_pass1_quota(None, 32, 64),
        lambda: L.fdb_ivfpq_get_pass1_quota(None, 32, C.byref(div)),
        lambda: L.fdb_ctx_set_wait_limit(None, 1.0),
        lambda: L.fdb_ctx_test_stall_scans(None, 1),
    ]
    for call in calls:
        assert call() == -1
