"""The ZKIEBCH2 weight-cache file written from device buffers and read back:
the whole file byte for byte against the reference layout built on the host
from the downloaded matrix and digest layers (pcs/whir.rs:542-559 and the
vendored write_digest_layers), and the read-back equal to the device buffers."""
import struct

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def expected_payload(lde, width, layers, lens):
    out = struct.pack("<QQQ", 1, width, lde.size) + lde.astype("<u8").tobytes()
    out += struct.pack("<Q", len(lens)) + struct.pack(f"<{len(lens)}Q", *lens)
    out += struct.pack(f"<{len(lens) - 1}Q", *([2] * (len(lens) - 1))) if len(lens) > 1 else b""
    return out + layers.astype("<u8").tobytes()


@pytest.mark.parametrize("n", [5, 9, 14, 20])
def test_cache_file_layout_and_read_back(zk, tmp_path, n):
    g = np.random.default_rng(n)
    evals = g.integers(0, zk.P, size=1 << n, dtype=np.uint64)
    com = zk.Whir(n).commit(evals)
    rows, width = com.lde.numel() // 32, 32
    meta = zk.BatchCacheMetadata("gpt2", f"group-{n}", ["w.0", "w.1"], n - 1, 2, 90, 17, bytes(range(32)))
    path = str(tmp_path / "batch.zkc")
    zk.write_cache(path, meta, com.root, com.lde, width, com.layers)
    data = open(path, "rb").read()
    hdr = zk.header_bytes(meta, com.root)
    lens = [int(x) for x in zk.merkle_layer_lengths(rows)]
    assert data == hdr + expected_payload(com.lde.cpu().numpy(), width, com.layers.cpu().numpy().reshape(-1), lens)
    meta2, root2, lde2, layers2 = zk.read_cache(path, rows, width)
    assert meta2 == meta and np.array_equal(root2, com.root)
    assert np.array_equal(lde2.cpu().numpy(), com.lde.cpu().numpy().reshape(-1))
    assert np.array_equal(layers2.cpu().numpy(), com.layers.cpu().numpy().reshape(-1))
    with pytest.raises(zk.ZkieError):
        zk.read_cache(path, rows // 2, width)
