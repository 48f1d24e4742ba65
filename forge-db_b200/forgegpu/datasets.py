"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (the reference measures on SIFT1M, which is not
available here; configuration C stands in for it).

    A  IVF-PQ CPU-runnable: 10k x 128 U[0,1), 1k queries, nlist 32, M 8, nprobe 8, k 10
    B  brute force: 1M x 128 N(0,1), 10k queries, k 100, L2^2 and dot
    C  IVF-PQ descriptor-like: 1M x 128 from a 1024-component Gaussian mixture
       (centres U[0,255], sigma 20, clipped to [0,255], rounded), 10k queries,
       nlist 1024, M 16, nprobe 8/32/128, k 10
    D  IVF-PQ embedding-scale: 20M x 96 unit-norm N(0,1), nlist 16384, M 48,
       nprobe 64, k 10
    E  training: k-means of 1M x 768 unit-norm N(0,1) into 4096, then PQ M 96
"""
from __future__ import annotations

import numpy as np


def uniform(n: int, dim: int, seed: int) -> np.ndarray:
    return np.random.default_rng(seed).random((n, dim), dtype=np.float32)


def normal(n: int, dim: int, seed: int, unit: bool = False, chunk: int = 1 << 20) -> np.ndarray:
    rng = np.random.default_rng(seed)
    out = np.empty((n, dim), np.float32)
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        out[s:e] = rng.standard_normal((e - s, dim), dtype=np.float32)
        if unit:
            nr = np.linalg.norm(out[s:e], axis=1, keepdims=True)
            nr[nr == 0] = 1.0
            out[s:e] /= nr
    return out


def gmm_descriptors(n: int, dim: int = 128, components: int = 1024, sigma: float = 20.0,
                    centre_seed: int = 5, seed: int = 6, chunk: int = 1 << 19) -> np.ndarray:
    """Integer-valued descriptor-like vectors in [0, 255] (config C)."""
    centres = np.random.default_rng(centre_seed).uniform(0, 255, (components, dim)).astype(np.float32)
    rng = np.random.default_rng(seed)
    out = np.empty((n, dim), np.float32)
    for s in range(0, n, chunk):
        e = min(n, s + chunk)
        comp = rng.integers(0, components, e - s)
        x = centres[comp] + rng.standard_normal((e - s, dim), dtype=np.float32) * np.float32(sigma)
        np.clip(x, 0, 255, out=x)
        out[s:e] = np.rint(x)
    return out


def config_c(n: int = 1_000_000, nq: int = 10_000):
    return gmm_descriptors(n, seed=6), gmm_descriptors(nq, seed=7)


def config_d(n: int = 20_000_000, nq: int = 10_000):
    """Unit-norm N(0,1) embeddings, 96 dimensions (seeds 9 and 10)."""
    return normal(n, 96, seed=9, unit=True), normal(nq, 96, seed=10, unit=True)


def config_e(n: int = 1_000_000):
    """Unit-norm N(0,1) rows, 768 dimensions (seed 11)."""
    return normal(n, 768, seed=11, unit=True)


def recall_at_k(pred: np.ndarray, truth: np.ndarray, k: int) -> float:
    """dataset.rs:160-166: |pred_k n truth_k| / k, averaged over queries."""
    pred = np.atleast_2d(pred)
    truth = np.atleast_2d(truth)
    hits = 0
    for p, t in zip(pred, truth):
        hits += len(set(p[:k].tolist()) & set(t[:k].tolist()))
    return hits / (k * pred.shape[0])
