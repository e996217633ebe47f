"""The ZKIEBCH2 weight-cache file of a committed batch (crates/zkie-core/src/pcs/cache.rs:7-70,
pcs/whir.rs:542-620, vendor/p3-merkle-tree write_digest_layers / read_digest_layers),
written from and read back into device buffers by libzkie_b200.so.

- ``BatchCacheMetadata``                 <- cache.rs:10-48
- ``header_bytes`` / ``read_header``     <- write_header / read_header (cache.rs:50-70)
- ``write_cache`` / ``read_cache``       <- write_header + serialize_batch_prover_data_into,
                                            read_header + restore_batch_prover_data_from
"""
import ctypes as C
import struct
from dataclasses import dataclass, field

import numpy as np
import torch

from ._lib import check, lib
from .device import empty, ptr, stream_handle, to_dev

MAGIC = b"ZKIEBCH2"
SCHEMA_VERSION = 2


@dataclass
class BatchCacheMetadata:
    model_id: str
    group_id: str
    table_ids: list
    table_arity: int
    num_tables: int
    security_level: int
    pow_bits: int
    source_digest: bytes
    schema_version: int = field(default=SCHEMA_VERSION)


def header_bytes(meta: BatchCacheMetadata, root) -> bytes:
    """bincode 1.3.3 of (MAGIC, metadata, MerkleCap([root]))."""
    if meta.schema_version != SCHEMA_VERSION or len(meta.table_ids) != meta.num_tables:
        raise ValueError("cache metadata: schema version 2 and one id per table")
    if len(meta.source_digest) != 32:
        raise ValueError("cache metadata: 32-byte source digest")
    ids = (C.c_char_p * max(len(meta.table_ids), 1))(*[t.encode() for t in meta.table_ids])
    rt = np.ascontiguousarray(np.asarray(root, dtype=np.uint64).reshape(8))
    args = (meta.model_id.encode(), meta.group_id.encode(), ids, meta.num_tables, meta.table_arity,
            meta.security_level, meta.pow_bits, bytes(meta.source_digest), rt.ctypes.data_as(C.POINTER(C.c_uint64)))
    n = lib.zkie2_cache_header(*args, None, 0)
    if n == 0:
        raise ValueError("cache header: bad argument")
    out = C.create_string_buffer(n)
    lib.zkie2_cache_header(*args, out, n)
    return out.raw


def read_header(data: bytes):
    """(metadata, root, header length) of a cache file's bytes (bincode 1.3.3 decode)."""
    pos = 0

    def take(n):
        nonlocal pos
        if pos + n > len(data):
            raise ValueError("cache header: truncated")
        b = data[pos:pos + n]
        pos += n
        return b

    def u32():
        return struct.unpack("<I", take(4))[0]

    def u64():
        return struct.unpack("<Q", take(8))[0]

    def string():
        return take(u64()).decode()

    if take(8) != MAGIC:
        raise ValueError("unsupported batch cache format")
    version = u32()
    model_id, group_id = string(), string()
    table_ids = [string() for _ in range(u64())]
    arity, num_tables, security, pow_bits = u32(), u32(), u32(), u32()
    digest = take(32)
    if version != SCHEMA_VERSION:
        raise ValueError("unsupported batch cache format")
    cap = [[u64() for _ in range(8)] for _ in range(u64())]
    meta = BatchCacheMetadata(model_id, group_id, table_ids, arity, num_tables, security, pow_bits, digest, version)
    return meta, np.array(cap[0] if cap else [], dtype=np.uint64), pos


def write_cache(path: str, meta: BatchCacheMetadata, root, lde, width: int, layers):
    """Header, then the committed matrix (rows x width, on the device) and its
    digest layers (the flat layer buffer of zkie2_merkle_tree, on the device)."""
    d_lde, d_layers = to_dev(lde).reshape(-1), to_dev(layers).reshape(-1)
    rows = d_lde.numel() // width
    if rows * width != d_lde.numel() or d_layers.numel() != 8 * lib.zkie2_merkle_total_digests(rows):
        raise ValueError("write_cache: matrix / digest-layer sizes do not match")
    hdr = header_bytes(meta, root)
    check(lib.zkie2_cache_write(path.encode(), hdr, len(hdr), ptr(d_lde), rows, width, ptr(d_layers),
                                stream_handle()), "zkie2_cache_write")


def read_cache(path: str, rows: int, width: int):
    """(metadata, root, matrix on the device, digest layers on the device)."""
    with open(path, "rb") as f:
        head = f.read(1 << 20)
    meta, root, hlen = read_header(head)
    d_lde = empty(rows * width)
    d_layers = empty(8 * lib.zkie2_merkle_total_digests(rows))
    check(lib.zkie2_cache_read(path.encode(), hlen, rows, width, ptr(d_lde), ptr(d_layers), stream_handle()),
          "zkie2_cache_read")
    return meta, root, d_lde, d_layers
