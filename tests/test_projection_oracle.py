"""CPU checks of the projection-block oracle (crates/zkie-ops/src/projection.rs):
the reference's own tests replayed with their seeds and shapes, including the
tampered proof that must fail, and the witness columns against their
definition."""
import numpy as np

P = 0xFFFFFFFF00000001


def ref_case(orc, seed, m, k, n):
    """x, w, bias as projection_block_roundtrip builds them (:133-147)."""
    rng = orc.XorShift64(seed)
    x = [orc.from_i64(rng.next_u64() % 100) for _ in range(m * k)]
    w = [orc.from_i64(rng.next_u64() % 100) for _ in range(k * n)]
    bias = [orc.from_i64(rng.next_u64() % 20 - 10) for _ in range(m * n)]
    return rng, np.array(x, dtype=np.uint64), np.array(w, dtype=np.uint64), np.array(bias, dtype=np.uint64)


def test_witness_matches_definition(orc):
    shift = 4
    h = np.array([orc.from_i64(v) for v in (-33, -17, -16, -9, -8, -7, -1, 0, 1, 7, 8, 9, 15, 16, 17, 1000)],
                 dtype=np.uint64)
    bias = np.array([orc.from_i64(v) for v in (-10, 3, 0, 9, -1, 2, 0, 5, -5, 1, 1, -2, 4, 0, 7, -3)],
                    dtype=np.uint64)
    out, rem = orc.projection_witness(h, bias, shift)
    for hv, bv, o, r in zip(h, bias, out, rem):
        a, b, o, r = orc.to_i64(hv), orc.to_i64(bv), orc.to_i64(o), orc.to_i64(r)
        assert 0 <= r < 16
        assert a + 8 - (o - b) * 16 == r          # the affine constraint
        assert o - b == (a + 8) // 16                # div_round(a, 16): ties round up


def test_to_i32_index_matches_fixed_point(orc):
    for v, exp in ((0, 0), (5, 5), (0x7FFFFFFF, 0x7FFFFFFF), (P - 1, 0xFFFFFFFF), (P - 3, 0xFFFFFFFD),
                   (orc.from_i64(-(1 << 31)), 0x80000000), (1 << 40, (-((P - (1 << 40)) & 0xFFFFFFFF)) & 0xFFFFFFFF)):
        assert orc.to_i32_index(v) == exp


def test_projection_block_roundtrip(orc):
    # projection_block_roundtrip (:130-180), seed 0xABCD, 2 x 2 x 2, shift 4:
    # the proof verifies, and bumping the first fraction layer's final
    # evaluation 3 makes it fail
    m = k = n = 2
    rng, x, w, bias = ref_case(orc, 0xABCD, m, k, n)
    h = orc.matmul_field(x.reshape(m, k), w.reshape(k, n)).reshape(-1)
    out, rem = orc.projection_witness(h, bias, 4)
    proof = orc.projection_prove(x, w, bias, out, rem, m, k, n, 4, rng)
    assert orc.projection_verify(proof, 4)
    proof["frac_finals"][0, 3] = (int(proof["frac_finals"][0, 3]) + 1) % P
    assert not orc.projection_verify(proof, 4)


def test_committed_projection_shape_roundtrip(orc):
    # committed_projection_roundtrip's witness (:181-224), seed 0xDD22, 8 x 8 x 8
    m = k = n = 8
    rng, x, w, bias = ref_case(orc, 0xDD22, m, k, n)
    h = orc.matmul_field(x.reshape(m, k), w.reshape(k, n)).reshape(-1)
    out, rem = orc.projection_witness(h, bias, 4)
    assert all(0 <= orc.to_i64(r) < 16 for r in rem)
    proof = orc.projection_prove(x, w, bias, out, rem, m, k, n, 4, rng)
    assert orc.projection_verify(proof, 4)
    # a wrong output breaks the affine constraint's sum (0)
    bad_out = out.copy()
    bad_out[3] = np.uint64((int(bad_out[3]) + 1) % P)
    rng2, *_ = ref_case(orc, 0xDD22, m, k, n)
    bad = orc.projection_prove(x, w, bias, bad_out, rem, m, k, n, 4, rng2)
    assert not orc.projection_verify(bad, 4)
