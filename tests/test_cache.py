"""The ZKIEBCH2 weight-cache file: header bytes against an independent
restatement of bincode 1.3.3 (little-endian, fixed-width integers, u64
lengths) of (magic, BatchCacheMetadata, MerkleCap), with the metadata of the
reference's committed_batch_tree_survives_serialization_roundtrip
(pcs/whir.rs:864-889); the decoder round trip; rejection of a foreign magic
or schema version."""
import struct

import pytest


def bincode_header(model, group, ids, arity, ntab, sec, pow_bits, digest, root):
    s = lambda x: struct.pack("<Q", len(x.encode())) + x.encode()  # noqa: E731
    out = b"ZKIEBCH2" + struct.pack("<I", 2) + s(model) + s(group) + struct.pack("<Q", len(ids))
    out += b"".join(s(i) for i in ids)
    out += struct.pack("<IIII", arity, ntab, sec, pow_bits) + bytes(digest)
    return out + struct.pack("<Q", 1) + struct.pack("<8Q", *root)


def test_header_matches_bincode_restatement(zk):
    ids = [f"layer-{i}-weight" for i in range(3)]
    root = [0xFFFFFFFF00000000 - i * 977 for i in range(8)]
    meta = zk.BatchCacheMetadata("test-model", "group-0", ids, 5, 3, 32, 10, bytes([7] * 32))
    got = zk.header_bytes(meta, root)
    assert got == bincode_header("test-model", "group-0", ids, 5, 3, 32, 10, [7] * 32, root)
    assert len(got) == 8 + 4 + (8 + 10) + (8 + 7) + 8 + 3 * (8 + 14) + 16 + 32 + 8 + 64
    back, rt, n = zk.read_header(got + b"payload")
    assert back == meta and [int(v) for v in rt] == root and n == len(got)


def test_header_rejects_foreign_files(zk):
    meta = zk.BatchCacheMetadata("m", "g", [], 0, 0, 0, 0, bytes(32))
    good = zk.header_bytes(meta, [1] * 8)
    with pytest.raises(ValueError):
        zk.read_header(b"ZKIEBCH1" + good[8:])
    with pytest.raises(ValueError):
        zk.read_header(good[:8] + struct.pack("<I", 3) + good[12:])
    with pytest.raises(ValueError):
        zk.read_header(good[:20])
    with pytest.raises(ValueError):
        zk.header_bytes(zk.BatchCacheMetadata("m", "g", ["a"], 0, 2, 0, 0, bytes(32)), [1] * 8)
