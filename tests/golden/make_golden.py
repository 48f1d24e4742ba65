"""Generates the golden fixtures in this folder.

    python tests/golden/make_golden.py

known_values.json
    The reference's own known-answer tests for this path, as values:
    distance known values (src/distance/mod.rs:56-105, tests/correctness.rs:
    132-178), the k-means nearest-centroid toy (src/kmeans.rs:381-395), and
    recall@k (src/dataset.rs:180-199).  The reference has no other golden
    vectors: its tests draw unseeded random data.

avx2_order.npz
    Distances of seeded random vectors at the dimensions the reference's
    SIMD-vs-scalar tests use (tests/correctness.rs:8-78: 1, 7, 8, 15, 16, 64,
    128, 256), computed here by a pure-Python restatement of the AVX2
    summation order (simd.rs:338-366, 427-456, 469-517) with exact rational
    arithmetic and IEEE round-to-nearest-even to f32 after every operation.
    Also the two ADC summation orders (pq.rs:218-245 and 435-485) on seeded
    LUTs.  This is independent of the C++ oracle and pins it bit for bit.

ivfpq_small.npz
    A small seeded IVF-PQ build (injected draws) and its batch / single
    search results from the oracle: a regression pin for the oracle and a
    fixture the GPU tests compare the engine against.

ivfpq_tiny.fdb, bf_tiny.fdb
    Index files in the reference's .fdb format (see fdb_files below);
    `python tests/golden/make_golden.py fdb` rewrites only these two.
"""
from __future__ import annotations

import json
import os
import sys
from fractions import Fraction

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


# ---------------------------------------------------------------------------
# exact f32 arithmetic
# ---------------------------------------------------------------------------
def round_f32(x: Fraction) -> float:
    """Round a rational to the nearest binary32 (ties to even)."""
    if x == 0:
        return 0.0
    sign = -1 if x < 0 else 1
    a = abs(x)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    # normalise so that 2^23 <= a / 2^(e-23) < 2^24
    while Fraction(2) ** e > a:
        e -= 1
    while Fraction(2) ** (e + 1) <= a:
        e += 1
    e = max(e, -126)  # subnormals share the minimum exponent
    scale = Fraction(2) ** (e - 23)
    m = a / scale
    q, r = divmod(m.numerator, m.denominator)
    rem = Fraction(r, m.denominator)
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and q % 2 == 1):
        q += 1
    val = Fraction(q) * scale
    return sign * float(val)


def F(v) -> Fraction:
    return Fraction(float(np.float32(v)))


def add(a, b):
    return round_f32(F(a) + F(b))


def sub(a, b):
    return round_f32(F(a) - F(b))


def mul(a, b):
    return round_f32(F(a) * F(b))


def fma(a, b, c):
    return round_f32(F(a) * F(b) + F(c))


def lanes_then_tail(a, b, lane_op, tail_op):
    n = len(a)
    acc = [0.0] * 8
    i = 0
    while i + 8 <= n:
        for j in range(8):
            acc[j] = lane_op(a[i + j], b[i + j], acc[j])
        i += 8
    t = 0.0
    for j in range(8):
        t = add(t, acc[j])
    while i < n:
        t = tail_op(t, a[i], b[i])
        i += 1
    return t


def l2sq(a, b):
    return lanes_then_tail(a, b, lambda x, y, s: fma(sub(x, y), sub(x, y), s),
                           lambda t, x, y: add(t, mul(sub(x, y), sub(x, y))))


def dot(a, b):
    return lanes_then_tail(a, b, lambda x, y, s: fma(x, y, s), lambda t, x, y: add(t, mul(x, y)))


def cosine(a, b):
    d, na, nb = dot(a, b), dot(a, a), dot(b, b)
    np_ = float(np.float32(np.sqrt(np.float64(mul(na, nb)))))  # sqrt is correctly rounded
    # check the sqrt rounding exactly: np_ must be the f32 nearest to sqrt(na*nb)
    if np_ == 0.0:
        return 0.0
    return sub(1.0, round_f32(F(d) / F(np_)))


def adc_fast(lut, code):
    m = len(code)
    s = 0.0
    i = 0
    while i + 4 <= m:
        t = [lut[(i + j) * 256 + int(code[i + j])] for j in range(4)]
        g = add(add(add(t[0], t[1]), t[2]), t[3])
        s = add(s, g)
        i += 4
    while i < m:
        s = add(s, lut[i * 256 + int(code[i])])
        i += 1
    return s


def adc_lane8(lut, code):
    m = len(code)
    acc = [0.0] * 8
    i = 0
    while i + 8 <= m:
        for j in range(8):
            acc[j] = add(acc[j], lut[(i + j) * 256 + int(code[i + j])])
        i += 8
    t = add(acc[0], acc[1])
    for j in range(2, 8):
        t = add(t, acc[j])
    while i < m:
        t = add(t, lut[i * 256 + int(code[i])])
        i += 1
    return t


# ---------------------------------------------------------------------------
def known_values():
    return {
        "source": "forge-db known-answer tests (values restated)",
        "distance": [
            # (metric, a, b, expected, abs_tol, citation)
            ["euclidean", [0, 0], [3, 4], 5.0, 1e-5, "src/distance/mod.rs:56-61"],
            ["dot_product", [1, 0], [1, 0], -1.0, 1e-5, "src/distance/mod.rs:63-70"],
            ["cosine", [1, 0], [0, 1], 1.0, 1e-5, "src/distance/mod.rs:72-82"],
            ["cosine", [1, 0], [1, 0], 0.0, 1e-5, "src/distance/mod.rs:72-82"],
            ["manhattan", [0, 0], [3, 4], 7.0, 1e-5, "src/distance/mod.rs:98-105"],
            ["euclidean", [0] * 8, [3, 4, 0, 0, 0, 0, 0, 0], 5.0, 1e-5, "tests/correctness.rs:132-153"],
            ["euclidean_squared", [0] * 8, [3, 4, 0, 0, 0, 0, 0, 0], 25.0, 1e-5, "tests/correctness.rs:132-153"],
            ["dot_raw", [1, 0, 0, 0, 0, 0, 0, 0], [0, 1, 0, 0, 0, 0, 0, 0], 0.0, 1e-6, "tests/correctness.rs:155-178"],
            ["euclidean", [1, 0, 0, 0, 0, 0, 0, 0], [0, 1, 0, 0, 0, 0, 0, 0], 1.4142135623730951, 1e-5, "tests/correctness.rs:155-178"],
        ],
        "kmeans_nearest": {
            "centroids": [[0.0, 0.0], [10.0, 0.0], [5.0, 10.0]],
            "query": [0.1, 0.1], "k": 2, "first": 0, "citation": "src/kmeans.rs:381-395",
        },
        "recall": [
            [[1, 2, 3, 4, 5], [1, 2, 3, 4, 5], 5, 1.0, "src/dataset.rs:180-185"],
            [[1, 2, 6, 7, 8], [1, 2, 3, 4, 5], 5, 0.4, "src/dataset.rs:187-192"],
            [[6, 7, 8, 9, 10], [1, 2, 3, 4, 5], 5, 0.0, "src/dataset.rs:194-199"],
        ],
    }


def avx2_order():
    rng = np.random.default_rng(20240611)
    out = {}
    dims = [1, 2, 7, 8, 9, 15, 16, 64, 128, 256]
    for d in dims:
        a = rng.uniform(-1, 1, (4, d)).astype(np.float32)
        b = rng.uniform(-1, 1, (4, d)).astype(np.float32)
        out[f"a_{d}"] = a
        out[f"b_{d}"] = b
        out[f"l2sq_{d}"] = np.array([l2sq(a[i], b[i]) for i in range(4)], np.float32)
        out[f"dot_{d}"] = np.array([dot(a[i], b[i]) for i in range(4)], np.float32)
        out[f"cos_{d}"] = np.array([cosine(a[i], b[i]) for i in range(4)], np.float32)
    for m in [4, 8, 10, 16, 48]:
        lut = (rng.random(m * 256, dtype=np.float32) * 100).astype(np.float32)
        codes = rng.integers(0, 256, (6, m)).astype(np.uint8)
        out[f"lut_{m}"] = lut
        out[f"codes_{m}"] = codes
        out[f"adc_fast_{m}"] = np.array([adc_fast(lut, c) for c in codes], np.float32)
        out[f"adc_lane8_{m}"] = np.array([adc_lane8(lut, c) for c in codes], np.float32)
    return out


def ivfpq_small():
    sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
    import oracle as O
    rng = np.random.default_rng(77)
    n, dim, nlist, m = 3000, 32, 16, 8
    X = rng.random((n, dim), dtype=np.float32)
    Q = rng.random((40, dim), dtype=np.float32)
    ids = (np.arange(n, dtype=np.uint64) * 7 + 100)
    ivf_sample_idx = np.arange(n, dtype=np.uint32)
    ivf_init_idx = rng.choice(n, nlist, replace=False).astype(np.uint32)
    ivf_kpp_u = (rng.integers(0, 1 << 23, nlist) / float(1 << 23)).astype(np.float32)
    pq_sample_idx = rng.permutation(n)[:2500].astype(np.uint32)
    pq_init_idx = np.concatenate([rng.choice(2500, 256, replace=False) for _ in range(m)]).astype(np.uint32)
    ix = O.OracleIVFPQ.build(X, ids, nlist, m, ivf_sample_idx, ivf_init_idx, ivf_kpp_u,
                             pq_sample_idx, pq_init_idx)
    ix.set_nprobe(4)
    bi, bd, bc = ix.batch_search(Q, 10, chunk=len(Q))
    si = np.full((len(Q), 10), np.iinfo(np.uint64).max, np.uint64)
    sd = np.full((len(Q), 10), np.inf, np.float32)
    sc = np.zeros(len(Q), np.uint32)
    for q in range(len(Q)):
        i, d = ix.search(Q[q], 10)
        si[q, :len(i)] = i
        sd[q, :len(d)] = d
        sc[q] = len(i)
    return dict(X=X, Q=Q, ids=ids, nlist=nlist, m=m, ivf_sample_idx=ivf_sample_idx,
                ivf_init_idx=ivf_init_idx, ivf_kpp_u=ivf_kpp_u, pq_sample_idx=pq_sample_idx,
                pq_init_idx=pq_init_idx, centroids=ix.centroids, codebooks=ix.codebooks,
                offsets=ix.offsets, list_ids=ix.ids, codes=ix.codes, assign=ix.assign,
                nprobe=4, k=10, batch_ids=bi, batch_d=bd, batch_cnt=bc, single_ids=si,
                single_d=sd, single_cnt=sc)


def fdb_files():
    """ivfpq_tiny.fdb / bf_tiny.fdb: files in the reference's format, written
    by the Python restatement of it (oracle/fdb_format.py) from seeded arrays:
    an IVF-PQ index (4 lists of 8-d vectors, 4 subvectors, random codes and
    ids, non-trivial centroid / codeword ids, nprobe 3, Cosine as the stored
    metric, 12 original vectors with rerank_factor 3) and a brute-force index
    (DotProduct, 30 rows of 6-d).  The engine must load them and write them
    back byte for byte."""
    sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
    import fdb_format as F
    rng = np.random.default_rng(4242)
    nlist, dim, m, n = 4, 8, 4, 40
    cents = rng.normal(size=(nlist, dim)).astype(np.float32)
    cb = rng.normal(size=(m, 256, dim // m)).astype(np.float32)
    sizes = np.array([13, 0, 19, 8])
    offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.uint64)
    ids = rng.choice(10 ** 6, n, replace=False).astype(np.uint64)
    codes = rng.integers(0, 256, (n, m)).astype(np.uint8)
    cent_ids = np.array([0, 1, 517, 3], np.uint64)  # list 2 kept its initial pick's id
    cb_ids = np.arange(m * 256, dtype=np.uint64) % 256
    cb_ids[5] = 901
    rr_ids = ids[:12].copy()
    rr_x = rng.normal(size=(12, dim)).astype(np.float32)
    payload = F.encode_ivfpq(cents, cent_ids, cb, cb_ids, offsets, ids, codes, nprobe=3,
                             metric=2, rerank=(rr_ids, rr_x), rerank_factor=3)
    with open(os.path.join(HERE, "ivfpq_tiny.fdb"), "wb") as f:
        f.write(F.file_bytes(F.IVFPQ, payload))
    Xb = rng.normal(size=(30, 6)).astype(np.float32)
    idb = rng.choice(10 ** 6, 30, replace=False).astype(np.uint64)
    with open(os.path.join(HERE, "bf_tiny.fdb"), "wb") as f:
        f.write(F.file_bytes(F.BRUTE_FORCE, F.encode_bf(3, idb, Xb)))


def main():
    if sys.argv[1:] == ["fdb"]:
        fdb_files()
        return
    with open(os.path.join(HERE, "known_values.json"), "w") as f:
        json.dump(known_values(), f, indent=1)
    np.savez_compressed(os.path.join(HERE, "avx2_order.npz"), **avx2_order())
    np.savez_compressed(os.path.join(HERE, "ivfpq_small.npz"), **ivfpq_small())
    fdb_files()
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
