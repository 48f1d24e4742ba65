"""The .fdb file format restated in Python -- TEST INFRASTRUCTURE ONLY.

Writes and parses the reference's index files independently of the engine's
C++ code, for the persistence parity tests:

- header, 24 bytes (src/persistence/format.rs:76-133): b"FORGEDB\\0", then
  version, index type, flags and the CRC-32 of the payload as u32 LE;
  verify_header (src/persistence/mod.rs:76-94) checks size, magic, type,
  version and checksum;
- IVF-PQ payload: bincode 1.3.3 (default options: fixed-width little-endian
  integers, usize as u64, Vec = u64 length + items, Option = u8 tag + value,
  unit enum = u32 variant index) of SerializableIVFPQ
  (src/index/ivf_pq.rs:207-262: centroids, pq {codebooks, n_subvectors,
  subvector_dim, dim}, partitions {ids, codes}, nprobe, metric,
  original_vectors, rerank_factor);
- brute-force payload (src/index/brute_force.rs:277-318): metric u8, n u64,
  dim u64, ids, rows.
The CRC is zlib's CRC-32 (the same CRC-32/ISO-HDLC crc32fast computes).
"""
from __future__ import annotations

import struct
import zlib

import numpy as np

MAGIC = b"FORGEDB\0"
VERSION = 1
IVFPQ, HNSW, IVF, BRUTE_FORCE = 1, 2, 3, 4


def crc32(b: bytes) -> int:
    return zlib.crc32(b) & 0xFFFFFFFF


def header(index_type: int, checksum: int, version: int = VERSION, flags: int = 0) -> bytes:
    return MAGIC + struct.pack("<IIII", version, index_type, flags, checksum)


def file_bytes(index_type: int, payload: bytes) -> bytes:
    return header(index_type, crc32(payload)) + payload


def split_file(data: bytes, expected_type: int | None = None):
    """verify_header: returns (version, type, flags, checksum, payload)."""
    if len(data) < 24:
        raise ValueError("file too small for header")
    if data[:8] != MAGIC:
        raise ValueError("invalid magic bytes")
    version, itype, flags, cs = struct.unpack("<IIII", data[8:24])
    if itype not in (1, 2, 3, 4):
        raise ValueError("unknown index type")
    if version > VERSION:
        raise ValueError("unsupported version")
    if expected_type is not None and itype != expected_type:
        raise ValueError("index type mismatch")
    payload = data[24:]
    if crc32(payload) != cs:
        raise ValueError("checksum mismatch")
    return version, itype, flags, cs, payload


# --- bincode pieces -----------------------------------------------------------------

def _u64(v):
    return struct.pack("<Q", int(v))


def _vector(id_, data) -> bytes:
    """SerializableVector {id: u64, data: Vec<f32>}"""
    data = np.ascontiguousarray(data, np.float32)
    return _u64(id_) + _u64(data.size) + data.tobytes()


def encode_ivfpq(centroids, cent_ids, codebooks, cb_ids, offsets, ids, codes, nprobe, metric,
                 rerank=None, rerank_factor=1) -> bytes:
    centroids = np.ascontiguousarray(centroids, np.float32)
    codebooks = np.ascontiguousarray(codebooks, np.float32)
    m, ksub, sub = codebooks.shape
    dim = centroids.shape[1]
    offsets = np.asarray(offsets, np.uint64)
    ids = np.ascontiguousarray(ids, np.uint64)
    codes = np.ascontiguousarray(codes, np.uint8)
    out = [_u64(len(centroids))]
    out += [_vector(cent_ids[l], centroids[l]) for l in range(len(centroids))]
    out.append(_u64(m))
    for s in range(m):
        out.append(_u64(ksub))
        out += [_vector(cb_ids[s * ksub + j], codebooks[s, j]) for j in range(ksub)]
    out += [_u64(m), _u64(sub), _u64(dim)]
    out.append(_u64(len(offsets) - 1))
    for l in range(len(offsets) - 1):
        b, e = int(offsets[l]), int(offsets[l + 1])
        out += [_u64(e - b), ids[b:e].tobytes(), _u64(e - b)]
        out += [_u64(m) + codes[r].tobytes() for r in range(b, e)]
    out += [_u64(nprobe), struct.pack("<I", metric)]
    if rerank is None:
        out.append(b"\0")
    else:
        rids, rx = rerank
        out += [b"\1", _u64(len(rids))]
        out += [_vector(i, v) for i, v in zip(np.asarray(rids, np.uint64).tolist(), rx)]
    out.append(_u64(rerank_factor))
    return b"".join(out)


class _R:
    def __init__(self, b):
        self.b, self.o = b, 0

    def take(self, n):
        if self.o + n > len(self.b):
            raise ValueError("unexpected end of payload")
        v = self.b[self.o:self.o + n]
        self.o += n
        return v

    def u64(self):
        return struct.unpack("<Q", self.take(8))[0]

    def vector(self):
        id_ = self.u64()
        n = self.u64()
        return id_, np.frombuffer(self.take(4 * n), np.float32)


def decode_ivfpq(payload: bytes) -> dict:
    r = _R(payload)
    nc = r.u64()
    cents = [r.vector() for _ in range(nc)]
    ncb = r.u64()
    cbs = []
    for _ in range(ncb):
        ne = r.u64()
        cbs.append([r.vector() for _ in range(ne)])
    n_sub, sub, dim = r.u64(), r.u64(), r.u64()
    npart = r.u64()
    offsets, ids, codes = [0], [], []
    for _ in range(npart):
        ni = r.u64()
        ids.append(np.frombuffer(r.take(8 * ni), np.uint64))
        nco = r.u64()
        for _ in range(nco):
            cl = r.u64()
            codes.append(np.frombuffer(r.take(cl), np.uint8))
        offsets.append(offsets[-1] + ni)
    nprobe = r.u64()
    metric = struct.unpack("<I", r.take(4))[0]
    tag = r.take(1)[0]
    rerank = None
    if tag == 1:
        nv = r.u64()
        rerank = [r.vector() for _ in range(nv)]
    rf = r.u64()
    return {
        "centroids": np.array([v for _, v in cents], np.float32).reshape(nc, -1),
        "cent_ids": np.array([i for i, _ in cents], np.uint64),
        "codebooks": np.array([[v for _, v in cb] for cb in cbs], np.float32),
        "cb_ids": np.array([i for cb in cbs for i, _ in cb], np.uint64),
        "n_subvectors": n_sub, "subvector_dim": sub, "dim": dim,
        "offsets": np.array(offsets, np.uint64),
        "ids": np.concatenate(ids) if ids else np.zeros(0, np.uint64),
        "codes": np.array(codes, np.uint8).reshape(-1, n_sub),
        "nprobe": nprobe, "metric": metric,
        "rerank": None if rerank is None else (np.array([i for i, _ in rerank], np.uint64),
                                               np.array([v for _, v in rerank], np.float32)),
        "rerank_factor": rf, "consumed": r.o,
    }


def encode_bf(metric: int, ids, X) -> bytes:
    ids = np.ascontiguousarray(ids, np.uint64)
    X = np.ascontiguousarray(X, np.float32)
    n = ids.size
    dim = X.shape[1] if n else 0
    return bytes([metric]) + _u64(n) + _u64(dim) + ids.tobytes() + X.tobytes()


def decode_bf(payload: bytes):
    if len(payload) < 17:
        raise ValueError("brute-force payload too small")
    metric = payload[0]
    n, dim = struct.unpack("<QQ", payload[1:17])
    if len(payload) < 17 + n * 8 + n * dim * 4:
        raise ValueError("brute-force payload truncated")
    ids = np.frombuffer(payload[17:17 + 8 * n], np.uint64)
    X = np.frombuffer(payload[17 + 8 * n:17 + 8 * n + 4 * n * dim], np.float32).reshape(n, dim)
    return metric, ids, X
