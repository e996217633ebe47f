"""CPU checks of the C-ABI boundary: libzkie_b200.so loads, exports every
function declared in include/*.h, and its host-only functions (transcript,
SHA-256, constants, geometry, twiddle tables) agree with the oracle.  No
device compute is called here."""
import ctypes as C
import hashlib
import os
import re
import subprocess

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
P = 0xFFFFFFFF00000001


def _declared_functions():
    names = []
    for h in sorted(os.listdir(os.path.join(ROOT, "include"))):
        if not h.endswith(".h"):
            continue
        text = open(os.path.join(ROOT, "include", h)).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names += re.findall(r"\b(zkie2?_[a-z0-9_]+)\s*\(", text)
    return sorted(set(names))


def test_library_exports_every_declared_symbol(zk):
    names = _declared_functions()
    assert len(names) >= 40
    out = subprocess.run(["nm", "-D", "--defined-only", zk.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT\s+(\S+)$", out, flags=re.M))
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    for n in names:
        assert hasattr(zk.lib, n)


def test_reference_symbols_present(zk):
    # crates/zkie-core/src/pcs/cuda_ffi.rs:2-46
    for n in ["zkie_cuda_device_count", "zkie_ntt_forward_goldilocks", "zkie_p2_upload_constants",
              "zkie_p2_leaf_batch", "zkie_p2_leaf_scalar", "zkie_p2_compress_batch", "zkie_p2_compress_scalar"]:
        assert n in _declared_functions()


def test_binding_covers_header(zk):
    from zkie_b200 import _lib
    assert set(_declared_functions()) == set(_lib.SIGNATURES)


def test_sha256_and_transcript(zk, orc):
    for n in (0, 3, 55, 56, 64, 200):
        d = bytes(range(n % 256)) * (1 + n // 256)
        d = d[:n]
        assert zk.sha256(d) == hashlib.sha256(d).digest()
    t, o = zk.Transcript(b"zkie-test"), orc.OracleTranscript(b"zkie-test")
    for x in (b"", b"\x01\x02", bytes(100)):
        t.absorb(x)
        o.absorb(x)
    t.absorb_u64(99)
    o.absorb_u64(99)
    assert [t.field() for _ in range(20)] == [o.field() for _ in range(20)]
    assert [t.next_u64() for _ in range(5)] == [o.next_u64() for _ in range(5)]


def test_xorshift_challenger(zk, orc):
    a, b = zk.XorShift64(0x1818), orc.XorShift64(0x1818)
    assert [a.field() for _ in range(50)] == [b.field() for _ in range(50)]


def test_shard_child(zk, orc):
    ids = [[0, 1, 2], [2, 3, 4]]
    a = zk.shard_dag_child(ids, 2, 1)
    b = orc.shard_dag_child(ids, 2, 1)
    assert [a.field() for _ in range(10)] == [b.field() for _ in range(10)]


def test_default_constants_match_oracle(zk, orc):
    ri, rf, rp, d15 = zk.p2_default_constants(1)
    ei, ef, it, od15 = orc.p2_constants(1).as_arrays()
    assert np.array_equal(ri, ei) and np.array_equal(rf, ef) and np.array_equal(rp, it) and d15 == od15


def test_merkle_geometry(zk, orc):
    for h in (1, 2, 3, 5, 8, 9, 1000, 1 << 20):
        assert zk.lib.zkie2_merkle_total_digests(h) == orc.lib().orc_merkle_total_digests(h)
        assert zk.lib.zkie2_merkle_num_layers(h) == orc.lib().orc_merkle_num_layers(h)
        assert sum(zk.merkle_layer_lengths(h)) == zk.lib.zkie2_merkle_total_digests(h)


def test_reference_twiddle_table(zk, orc):
    # pcs/dft_cuda.rs:44-59: stage s at offset 2^(s-1) - 1, TWO_ADIC_GENERATORS[s]^j
    lg = 9
    tw = zk.make_twiddles(lg)
    assert tw.size == (1 << lg) - 1
    off = 0
    for s in range(1, lg + 1):
        g = orc.two_adic_generator(s)
        assert [int(x) for x in tw[off:off + (1 << (s - 1))]] == [pow(g, j, P) for j in range(1 << (s - 1))]
        off += 1 << (s - 1)


def test_scratch_queries(zk):
    L = zk.lib
    assert L.zkie2_lde_scratch_elems(5, 1, 8) == 0          # single pass, no scratch
    assert L.zkie2_lde_scratch_elems(20, 1, 32) == 32 << 21
    assert L.zkie2_whir_scratch_elems(20) == 32 << 16
    assert L.zkie2_matmul_scratch_elems(16, 1024, 1024) > 0
    assert L.zkie2_matmul_scratch_elems(3, 4, 4) == 0        # not a power of two
    # shapes the tensor path cannot take need no tensor-path scratch (field kernel)
    assert L.zkie2_matmul_fixed_scratch_elems(16, 40, 16) == 1       # k % 16 != 0
    assert L.zkie2_matmul_fixed_scratch_elems(16, 1 << 21, 16) == 1  # k / 32 = 65536 > grid.y limit
    assert L.zkie2_matmul_fixed_scratch_elems(16, 65535 * 32, 16) > 1


def test_moe_index_entries_reject_sizes_past_u32(zk):
    """zkie2_op_gather keeps per-token offsets and position lists in u32, and
    the scatter entries u32 token / expert ids and counts, so they refuse
    sizes of 2^32 and more before touching the device (the pointers here are
    never dereferenced)."""
    invalid = 1  # cudaErrorInvalidValue
    fake = 0x1000
    L = zk.lib
    assert L.zkie2_op_gather(fake, fake, fake, 1 << 32, 4, 8, fake, fake, fake, None) == invalid
    assert L.zkie2_op_gather(fake, fake, fake, 4, (1 << 32) - 1, 8, fake, fake, fake, None) == invalid
    # the scatter entries' token / expert ids and counts are u32 as well
    assert L.zkie2_op_sel_counts(fake, 1 << 32, 4, 1, fake, None) == invalid
    assert L.zkie2_op_scatter(fake, 4, 1 << 32, fake, fake, fake, fake, None) == invalid
    assert L.zkie2_op_scatter_encodings(fake, 1 << 32, 4, fake, fake, fake, 4, fake, fake, fake, fake,
                                        None) == invalid


def test_device_count_without_gpu(zk):
    import torch
    n = zk.lib.zkie_cuda_device_count()
    assert n == (torch.cuda.device_count() if torch.cuda.is_available() else 0)
