"""bincode bytes of the produced proofs against an independent struct.pack
restatement of the serde-derive layouts (sumcheck.rs:10-29, 236-240, 373-377;
matmul.rs:11-15; logup_gkr.rs:7-18), and decode round trips."""
import struct

import numpy as np
import pytest

P = 0xFFFFFFFF00000001


def q(*vals):
    return struct.pack(f"<{len(vals)}Q", *vals)


def test_sumcheck_matmul_batch_layouts(zk):
    rounds = np.array([[1, 2, 3], [4, 5, P - 1]], dtype=np.uint64)
    sp = zk.SumcheckProof(rounds, 7, 8)
    assert zk.to_bincode(sp) == q(2, 1, 2, 3, 4, 5, P - 1, 7, 8)
    mp = zk.MatmulProof(99, sp)
    assert zk.to_bincode(mp) == q(99) + q(2, 1, 2, 3, 4, 5, P - 1, 7, 8)
    bp = zk.SumcheckProofBatch(rounds[:1], 11)
    assert zk.to_bincode(bp) == q(1, 1, 2, 3, 11)
    for kind, obj in ((zk.SumcheckProof, sp), (zk.MatmulProof, mp), (zk.SumcheckProofBatch, bp)):
        back = zk.from_bincode(kind, zk.to_bincode(obj))
        assert zk.to_bincode(back) == zk.to_bincode(obj)


def test_virtual_and_fractional_layouts(zk, orc):
    vp = zk.VirtualProof(np.array([[1, 2, 3, 4], [5, 6, 7, 8]], dtype=np.uint64), np.array([9, 10, 11], np.uint64))
    assert zk.to_bincode(vp) == q(2, 4, 1, 2, 3, 4, 4, 5, 6, 7, 8, 3, 9, 10, 11)
    # a fraction tree from the oracle (fractional_roundtrip's seed, logup_gkr.rs:533-556)
    rng = orc.XorShift64(0xDEC0)
    num = [rng.field() for _ in range(64)]
    den = [i % 7 + 1 for i in range(64)]
    full_r, cs = [rng.field() for _ in range(6)], [rng.field() for _ in range(6)]
    rounds, finals, fn, fd = orc.fractional_prove(num, den, full_r, cs)
    layers = [zk.FractionalLayer(np.array(full_r[:6 - l - 1], dtype=np.uint64), cs[l],
                                 zk.VirtualProof(rounds[l], finals[l])) for l in range(6)]
    fp = zk.FractionalProof(layers, fn, fd, np.array(full_r, dtype=np.uint64))
    want = q(6)
    for l in range(6):
        t = 6 - l - 1
        want += q(t, *full_r[:t]) + q(cs[l]) + q(t) + b"".join(q(4, *map(int, row)) for row in rounds[l])
        want += q(7, *map(int, finals[l]))
    want += q(fn, fd) + q(6, *full_r)
    got = zk.to_bincode(fp)
    assert got == want
    back = zk.from_bincode(zk.FractionalProof, got)
    assert zk.to_bincode(back) == got and (back.final_num, back.final_den) == (fn, fd)


def test_decode_rejects_bad_bytes(zk):
    good = zk.to_bincode(zk.SumcheckProof(np.array([[1, 2, 3]], dtype=np.uint64), 4, 5))
    with pytest.raises(ValueError):
        zk.from_bincode(zk.SumcheckProof, good + b"\0")
    with pytest.raises(ValueError):
        zk.from_bincode(zk.SumcheckProof, good[:-1])
    with pytest.raises(TypeError):
        zk.to_bincode(object())
