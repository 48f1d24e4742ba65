"""IVFPQIndexBuilder's parameter rules (src/index/ivf_pq_builder.rs:188-361),
host only: the reference's builder tests (:363-454) restated on the plan,
plus the auto-tune branches they leave out."""
import numpy as np
import pytest

import forgegpu as fg


def _plan(n, dim, **kw):
    b = fg.IVFPQIndexBuilder()
    for k, v in kw.items():
        getattr(b, k)(v)
    return b.plan(n, dim)


def _kind(fn):
    with pytest.raises(fg.ForgeGpuError) as e:
        fn()
    return e.value.kind


def test_reference_builder_cases():
    # test_builder_basic
    assert _plan(500, 32, num_clusters=8, num_subvectors=4, nprobe=4)[:3] == (8, 4, 4)
    # test_builder_auto_tune: sqrt(1000) ~ 31.6 -> 32, clamped up to 256
    c, m, p, _ = _plan(1000, 128, auto_tune=True)
    assert c >= 31 and (c, m, p) == (256, 32, 1)
    # test_builder_target_recall: 100 clusters * 0.1 = 10 probes
    assert _plan(500, 32, num_clusters=100, num_subvectors=4, target_recall=0.95)[2] == 10
    # test_builder_invalid_subvectors: 30 is not divisible by 8
    assert _kind(lambda: _plan(500, 30, num_subvectors=8)) == "InvalidParameter"
    # test_builder_no_vectors / test_builder_empty_vectors
    assert _kind(lambda: fg.IVFPQIndexBuilder().build()) == "InvalidParameter"
    assert _kind(lambda: fg.IVFPQIndexBuilder().vectors(np.zeros((0, 8), np.float32))
                 .build()) == "EmptyVectorSet"


def test_auto_tune_branches():
    # without auto-tuning: round(sqrt(n)) clusters, dim / 4 subvectors
    assert _plan(500, 32, auto_tune=False)[:2] == (22, 8)
    assert _plan(500, 6, auto_tune=False)[1] == 1
    assert _kind(lambda: _plan(500, 3, auto_tune=False)) == "InvalidParameter"
    # with it: clusters clamped to [min(256, n), min(65536, n)]
    assert _plan(100, 16)[0] == 100
    assert _plan(10 ** 6, 16)[0] == 1000 and _plan(10 ** 10, 16)[0] == 65536
    # largest divisor of dim not above dim / 4
    assert _plan(5000, 30)[1] == 6 and _plan(5000, 7)[1] == 1 and _plan(5000, 3)[1] == 1
    # recall tiers (f32 ceil of a fraction of the clusters)
    for r, want in ((0.99, 26), (0.9, 13), (0.85, 6), (0.5, 1)):
        assert _plan(5000, 32, num_clusters=256, target_recall=r)[2] == want
    # an explicit nprobe > 1 wins, capped at the clusters
    assert _plan(5000, 32, num_clusters=64, nprobe=100)[2] == 64
    # more clusters than vectors
    assert _kind(lambda: _plan(500, 32, num_clusters=600)) == "InsufficientVectors"


def test_memory_estimate():
    # codes + ids + centroids + codebooks, whole MiB (estimate_memory_mb)
    mb = _plan(10 ** 6, 128, num_clusters=1000, num_subvectors=32)[3]
    assert mb == (10 ** 6 * 32 + 10 ** 6 * 8 + 1000 * 128 * 4 + 32 * 256 * 4 * 4) // 2 ** 20
