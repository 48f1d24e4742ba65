"""The .fdb format on the CPU: the Python restatement (oracle/fdb_format.py)
pinned by hand against the reference's layout, and the engine's host-side
parser (fdb_file_inspect) and CRC against it.  No device is used."""
import os
import struct
import zlib

import numpy as np
import pytest

import fdb_format as F
import forgegpu as fg

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_crc32_known_answers():
    # CRC-32/ISO-HDLC check value (the catalogue's "123456789" test vector)
    assert fg.crc32(b"123456789") == 0xCBF43926
    assert F.crc32(b"123456789") == 0xCBF43926
    assert fg.crc32(b"") == 0
    rng = np.random.default_rng(5)
    for n in (1, 7, 8, 9, 63, 64, 65, 1000, 65537):
        b = rng.integers(0, 256, n).astype(np.uint8).tobytes()
        assert fg.crc32(b) == zlib.crc32(b) & 0xFFFFFFFF


def test_header_roundtrip_layout():
    # format.rs:191-201: FileHeader::new(IvfPq, 0x12345678) -> to_bytes
    h = F.header(F.IVFPQ, 0x12345678)
    assert len(h) == 24
    assert h[:8] == b"FORGEDB\0"
    assert struct.unpack("<IIII", h[8:]) == (1, 1, 0, 0x12345678)


def _tiny_arrays():
    rng = np.random.default_rng(1)
    cents = rng.normal(size=(2, 4)).astype(np.float32)
    cb = rng.normal(size=(2, 256, 2)).astype(np.float32)
    offsets = np.array([0, 2, 3], np.uint64)
    ids = np.array([11, 12, 13], np.uint64)
    codes = np.array([[1, 2], [3, 4], [255, 0]], np.uint8)
    cb_ids = np.arange(512, dtype=np.uint64) % 256
    return cents, cb, offsets, ids, codes, cb_ids


def test_ivfpq_payload_layout_by_hand():
    """bincode 1.3 of SerializableIVFPQ (ivf_pq.rs:253-262), field by field."""
    cents, cb, offsets, ids, codes, cb_ids = _tiny_arrays()
    p = F.encode_ivfpq(cents, [7, 8], cb, cb_ids, offsets, ids, codes, nprobe=2, metric=1,
                       rerank=None, rerank_factor=5)
    u64 = lambda o: struct.unpack_from("<Q", p, o)[0]
    # centroids: Vec<SerializableVector{id, data: Vec<f32>}>
    assert u64(0) == 2 and u64(8) == 7 and u64(16) == 4
    assert np.frombuffer(p[24:40], np.float32).tolist() == cents[0].tolist()
    assert u64(40) == 8 and u64(48) == 4
    o = 72
    # pq.codebooks: Vec<Vec<SerializableVector>> (2 x 256 entries of 2 floats)
    assert u64(o) == 2 and u64(o + 8) == 256 and u64(o + 16) == 0 and u64(o + 24) == 2
    assert np.frombuffer(p[o + 32:o + 40], np.float32).tolist() == cb[0, 0].tolist()
    o += 8 + 2 * (8 + 256 * 24)
    # n_subvectors, subvector_dim, dim
    assert (u64(o), u64(o + 8), u64(o + 16)) == (2, 2, 4)
    o += 24
    # partitions: Vec<{ids: Vec<u64>, codes: Vec<Vec<u8>>}>
    assert u64(o) == 2
    assert u64(o + 8) == 2 and u64(o + 16) == 11 and u64(o + 24) == 12
    assert u64(o + 32) == 2 and u64(o + 40) == 2 and p[o + 48:o + 50] == bytes([1, 2])
    o += 8 + (8 + 16 + 8 + 2 * 10) + (8 + 8 + 8 + 10)
    # nprobe u64, metric u32 variant (EuclideanSquared = 1), None, rerank_factor
    assert u64(o) == 2 and struct.unpack_from("<I", p, o + 8)[0] == 1
    assert p[o + 12] == 0 and u64(o + 13) == 5 and len(p) == o + 21
    d = F.decode_ivfpq(p)
    assert d["consumed"] == len(p)
    assert np.array_equal(d["codes"], codes) and np.array_equal(d["ids"], ids)


def _write(tmp_path, name, data):
    path = tmp_path / name
    path.write_bytes(data)
    return str(path)


def test_inspect_reads_restated_files(tmp_path):
    cents, cb, offsets, ids, codes, cb_ids = _tiny_arrays()
    rr = (np.array([12, 13], np.uint64), np.ones((2, 4), np.float32))
    p = F.encode_ivfpq(cents, [0, 1], cb, cb_ids, offsets, ids, codes, nprobe=9, metric=4,
                       rerank=rr, rerank_factor=2)
    info = fg.inspect_file(_write(tmp_path, "a.fdb", F.file_bytes(F.IVFPQ, p)))
    assert (info.version, info.index_type, info.flags) == (1, 1, 0)
    assert info.checksum == F.crc32(p)
    assert (info.n, info.dim, info.nlist, info.m, info.nprobe, info.metric) == (3, 4, 2, 2, 9, 4)
    assert (info.has_rerank, info.n_rerank, info.rerank_factor) == (1, 2, 2)
    for name in ("ivfpq_tiny.fdb", "bf_tiny.fdb"):
        raw = open(os.path.join(GOLDEN, name), "rb").read()
        _, t, _, cs, payload = F.split_file(raw)
        info = fg.inspect_file(os.path.join(GOLDEN, name))
        assert info.index_type == t and info.checksum == cs
        if t == F.BRUTE_FORCE:
            metric, bid, X = F.decode_bf(payload)
            assert (info.n, info.dim, info.metric) == (bid.size, X.shape[1], metric)


def _code(fn):
    with pytest.raises(fg.ForgeGpuError) as e:
        fn()
    return e.value.kind


def test_inspect_rejects_bad_files(tmp_path):
    good = open(os.path.join(GOLDEN, "ivfpq_tiny.fdb"), "rb").read()
    bad = bytearray(good)
    bad[100] ^= 1  # payload byte: CRC fails
    assert _code(lambda: fg.inspect_file(_write(tmp_path, "c.fdb", bytes(bad)))) == "ChecksumMismatch"
    # test_persistence_corrupted_file (ivf_pq.rs:2213-2227)
    assert _code(lambda: fg.inspect_file(_write(tmp_path, "t.fdb", b"not a valid forge-db file"))) == "InvalidFormat"
    assert _code(lambda: fg.inspect_file(_write(tmp_path, "s.fdb", good[:20]))) == "InvalidFormat"
    v2 = bytearray(good)
    v2[8] = 2
    assert _code(lambda: fg.inspect_file(_write(tmp_path, "v.fdb", bytes(v2)))) == "InvalidFormat"
    t9 = bytearray(good)
    t9[12] = 9
    assert _code(lambda: fg.inspect_file(_write(tmp_path, "x.fdb", bytes(t9)))) == "InvalidFormat"
    # a payload cut short under a matching CRC: bincode's unexpected end of file
    cut = good[24:-30]
    assert _code(lambda: fg.inspect_file(_write(tmp_path, "u.fdb", F.file_bytes(F.IVFPQ, cut)))) == "SerializationError"
    assert _code(lambda: fg.inspect_file(str(tmp_path / "missing.fdb"))) == "Io"
    # codebooks with fewer than 256 entries (PQ trained on < 256 vectors)
    cents, cb, offsets, ids, codes, cb_ids = _tiny_arrays()
    p = F.encode_ivfpq(cents, [0, 1], cb[:, :200], cb_ids, offsets, ids, codes, 1, 0)
    assert _code(lambda: fg.inspect_file(_write(tmp_path, "k.fdb", F.file_bytes(F.IVFPQ, p)))) == "NotSupported"
    # brute force: truncated rows
    pb = F.encode_bf(0, np.arange(3, dtype=np.uint64), np.ones((3, 4), np.float32))[:-4]
    assert _code(lambda: fg.inspect_file(_write(tmp_path, "b.fdb", F.file_bytes(F.BRUTE_FORCE, pb)))) == "InvalidFormat"
    pm = bytearray(F.encode_bf(0, np.arange(3, dtype=np.uint64), np.ones((3, 4), np.float32)))
    pm[0] = 7
    assert _code(lambda: fg.inspect_file(_write(tmp_path, "m.fdb", F.file_bytes(F.BRUTE_FORCE, bytes(pm))))) == "InvalidFormat"
