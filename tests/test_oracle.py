"""CPU checks of the oracle: against independent definitions, against a
pure-Python restatement, and against the reference's own property tests
replayed with the reference's seeds (the reference holds no golden bytes)."""
import hashlib
import random

import numpy as np
import pytest

from tests import pyref

P = pyref.P


# ---- field ---------------------------------------------------------------------------
def test_field_ops_match_bigint(orc):
    rnd = random.Random(7)
    for _ in range(2000):
        a, b = rnd.randrange(P), rnd.randrange(P)
        assert orc.add(a, b) == (a + b) % P
        assert orc.sub(a, b) == (a - b) % P
        assert orc.mul(a, b) == (a * b) % P
    for a in (0, 1, P - 1, P - 2, 2 ** 32, 2 ** 63):
        for b in (0, 1, P - 1, 2 ** 32 - 1, 2 ** 64 - 2 ** 32):
            assert orc.mul(a, b) == (a * b) % P
    assert orc.mul(2, orc.inv(2)) == 1  # field.rs:42-48 inverse_of_two


def test_two_adic_generators(orc):
    # TWO_ADIC_GENERATORS[i+1]^2 == TWO_ADIC_GENERATORS[i], [0] = 1, [1] = -1.
    assert orc.two_adic_generator(0) == 1
    assert orc.two_adic_generator(1) == P - 1
    for b in range(1, 33):
        g = orc.two_adic_generator(b)
        assert pow(g, 1 << b, P) == 1 and pow(g, 1 << (b - 1), P) == P - 1
        assert orc.mul(g, g) == orc.two_adic_generator(b - 1)
    # small-order elements are powers of two in Goldilocks (2^96 = -1)
    assert orc.two_adic_generator(2) == 1 << 48
    assert orc.two_adic_generator(3) == P - (1 << 24)
    assert orc.two_adic_generator(6) == 1 << 39
    assert orc.two_adic_generator(32) == pow(7, (P - 1) >> 32, P)


def test_from_i64(orc):
    for x in (0, 1, -1, 2 ** 40, -(2 ** 40), -(2 ** 63), 2 ** 63 - 1):
        assert orc.from_i64(x) == x % P


# ---- PRNG / SHA-256 / transcript -------------------------------------------------------
def test_xorshift_matches_definition(orc):
    # field.rs:17-36
    s = (12345 + 0x9E3779B97F4A7C15) % 2 ** 64
    rng = orc.XorShift64(12345)
    for _ in range(100):
        s ^= (s << 13) % 2 ** 64
        s ^= s >> 7
        s ^= (s << 17) % 2 ** 64
        assert rng.next_u64() == s


def test_xorshift_field_canonical(orc):
    # field.rs:50-56 xorshift_produces_canonical_elements
    rng = orc.XorShift64(1)
    for _ in range(1000):
        assert rng.field() < P


def test_sha256_matches_fips(orc):
    for n in list(range(0, 130)) + [1000, 4096]:
        data = bytes((i * 7 + 3) & 0xFF for i in range(n))
        assert orc.sha256(data) == hashlib.sha256(data).digest()


def _py_transcript_draws(domain, absorbs, n):
    state = hashlib.sha256(domain).digest()
    for a in absorbs:
        state = hashlib.sha256(state + a).digest()
    ctr, out = 0, []
    while len(out) < n:
        d = hashlib.sha256(state + ctr.to_bytes(8, "little")).digest()
        ctr += 1
        c = int.from_bytes(d[:8], "little")
        if c < P:
            out.append(c)
    return out


def test_transcript_matches_definition(orc):
    t = orc.OracleTranscript(b"zkie-test")
    t.absorb(bytes([1, 2, 3]))
    t.absorb_u64(0xDEADBEEF)
    got = [t.field() for _ in range(40)]
    assert got == _py_transcript_draws(b"zkie-test", [bytes([1, 2, 3]), (0xDEADBEEF).to_bytes(8, "little")], 40)


def test_transcript_reference_properties(orc):
    # transcript.rs:88-121: deterministic_replay, absorb_changes_challenges, field_is_canonical
    a, b = orc.OracleTranscript(b"zkie-test"), orc.OracleTranscript(b"zkie-test")
    a.absorb(bytes([1, 2, 3]))
    b.absorb(bytes([1, 2, 3]))
    assert [a.field() for _ in range(16)] == [b.field() for _ in range(16)]
    a, b = orc.OracleTranscript(b"zkie-test"), orc.OracleTranscript(b"zkie-test")
    b.absorb(bytes([7]))
    assert a.field() != b.field()
    t = orc.OracleTranscript(b"zkie-test")
    assert all(t.field() < P for _ in range(1000))


# ---- DFT ---------------------------------------------------------------------------------
@pytest.mark.parametrize("lg,w", [(1, 1), (2, 3), (4, 1), (5, 4), (6, 2), (7, 3)])
def test_dft_batch_matches_naive(orc, lg, w):
    rng = orc.XorShift64(100 + lg)
    m = np.array([[rng.field() for _ in range(w)] for _ in range(1 << lg)], dtype=np.uint64)
    assert np.array_equal(orc.dft_batch(m), orc.dft_naive(m))
    if lg <= 5:
        col = [int(x) for x in m[:, 0]]
        assert [int(x) for x in orc.dft_batch(m)[:, 0]] == pyref.dft(col)


@pytest.mark.parametrize("lg,w", [(1, 4), (3, 8), (5, 9), (6, 13), (8, 16), (9, 37), (10, 256)])
def test_dft_batch_matches_naive_with_packed_columns(orc, lg, w):
    """Widths that fill the packed column blocks (one SIMD lane per column)
    and leave ragged columns for the scalar blocks."""
    rng = orc.XorShift64(300 + lg)
    m = np.array([[rng.field() for _ in range(w)] for _ in range(1 << lg)], dtype=np.uint64)
    if lg <= 6:
        assert np.array_equal(orc.dft_batch(m), orc.dft_naive(m))
    m[0, 0] = np.uint64(P)                      # non-canonical inputs
    m[-1, -1] = np.uint64(2 ** 64 - 1)
    best = orc.set_lanes(-1)
    try:
        orc.set_lanes(0)
        ref = orc.dft_batch(m)
        for lanes in sorted({4, best} - {0}):
            if lanes > best:
                continue
            assert orc.set_lanes(lanes) == lanes
            assert np.array_equal(orc.dft_batch(m), ref)
    finally:
        orc.set_lanes(best)


def test_lde_is_padded_dft(orc):
    rng = orc.XorShift64(9)
    m = np.array([[rng.field() for _ in range(3)] for _ in range(16)], dtype=np.uint64)
    for lb in (1, 2):
        padded = np.zeros((16 << lb, 3), dtype=np.uint64)
        padded[:16] = m
        assert np.array_equal(orc.lde(m, lb), orc.dft_batch(padded))
        # even rows of the blowup-2 LDE are the plain DFT (the size-L subgroup)
    assert np.array_equal(orc.lde(m, 1)[::2], orc.dft_batch(m))


def test_dft_noncanonical_inputs(orc):
    m = np.array([[2 ** 64 - 1], [P], [P + 5], [3]], dtype=np.uint64)
    mc = np.array([[(2 ** 64 - 1) % P], [0], [5], [3]], dtype=np.uint64)
    assert np.array_equal(orc.dft_batch(m), orc.dft_batch(mc))


# ---- Poseidon2 / Merkle -------------------------------------------------------------
def _consts_py(c):
    ei, ef, it, d15 = c.as_arrays()
    return ([[int(x) for x in r] for r in ei], [[int(x) for x in r] for r in ef], [int(x) for x in it], d15)


def test_constants_shape_and_canonical(consts):
    ei, ef, it, d15 = consts.as_arrays()
    assert ei.shape == (4, 16) and ef.shape == (4, 16) and it.shape == (22,)
    assert (ei < P).all() and (ef < P).all() and (it < P).all()
    assert d15 * (2 ** 32) % P == 1
    assert len(set(ei.ravel().tolist()) | set(ef.ravel().tolist()) | set(it.tolist())) == 150


def test_permutation_matches_python(orc, consts):
    cp = _consts_py(consts)
    rnd = random.Random(3)
    for trial in range(6):
        st = [rnd.randrange(P) for _ in range(16)] if trial else list(range(16))
        assert [int(x) for x in orc.p2_permute(consts, st)] == pyref.permute(st, *cp)


@pytest.mark.parametrize("w", [0, 1, 5, 8, 9, 16, 17, 32])
def test_sponge_matches_python(orc, consts, w):
    cp = _consts_py(consts)
    rnd = random.Random(w)
    row = [rnd.randrange(P) for _ in range(w)]
    assert [int(x) for x in orc.p2_hash_row(consts, row)] == pyref.hash_row(row, cp)


def test_sponge_overwrite_semantics(orc, consts):
    # partial tail overwrites only the first rem lanes: a 9-element row differs
    # from the same row padded with a zero
    row = list(range(1, 10))
    assert not np.array_equal(orc.p2_hash_row(consts, row), orc.p2_hash_row(consts, row + [0]))
    assert np.array_equal(orc.p2_hash_row(consts, []), np.zeros(8, dtype=np.uint64))


@pytest.mark.parametrize("h", [1, 2, 3, 4, 5, 7, 8, 9])
def test_merkle_root_matches_python(orc, consts, h):
    cp = _consts_py(consts)
    rnd = random.Random(h)
    rows = [[rnd.randrange(P) for _ in range(3)] for _ in range(h)]
    layers, root = orc.merkle_tree(consts, np.array(rows, dtype=np.uint64))
    assert [int(x) for x in root] == pyref.merkle_root(rows, cp)
    assert [len(l) for l in layers][0] == pyref.padded_len(h)
    assert np.array_equal(orc.merkle_root_from_leaves(consts, orc.merkle_leaves(consts, np.array(rows, dtype=np.uint64))), root)


@pytest.mark.parametrize("h,w", [(1, 8), (7, 3), (8, 0), (8, 8), (9, 9), (17, 16), (33, 1), (64, 256),
                                 (69, 33), (300, 7)])
def test_packed_merkle_matches_scalar(orc, consts, h, w):
    """The SIMD leaf and tree loops (one state per lane, several rows at once)
    give the scalar permutation's digests on every layer, including a partial
    sponge tail, non-canonical inputs and rows past the last full group."""
    rnd = np.random.default_rng(1000 * h + w)
    mat = rnd.integers(0, 2 ** 63, size=(h, w), dtype=np.uint64) * np.uint64(2) + np.uint64(1)
    if mat.size:
        mat.flat[0] = np.uint64(P)             # non-canonical: >= p
        mat.flat[-1] = np.uint64(2 ** 64 - 1)
    best = orc.set_lanes(-1)
    try:
        orc.set_lanes(0)
        ref_layers, ref_root = orc.merkle_tree(consts, mat)
        ref_leaves = orc.merkle_leaves(consts, mat, threads=1)
        for lanes in sorted({4, best} - {0}):
            if lanes > best:
                continue
            assert orc.set_lanes(lanes) == lanes
            layers, root = orc.merkle_tree(consts, mat)
            assert np.array_equal(root, ref_root)
            assert all(np.array_equal(a, b) for a, b in zip(layers, ref_layers))
            assert np.array_equal(orc.merkle_leaves(consts, mat, threads=1), ref_leaves)
    finally:
        orc.set_lanes(best)


def test_padded_len(orc):
    # merkle_tree.rs:577-585
    for raw, n, exp in [(0, 2, 0), (1, 2, 1), (2, 2, 2), (3, 2, 4), (5, 2, 6), (1, 4, 1), (3, 4, 4), (6, 4, 8)]:
        assert orc.padded_len(raw, n) == exp


def test_whir_commit_geometry(orc, consts):
    rng = orc.XorShift64(5)
    evals = np.array([rng.field() for _ in range(1 << 7)], dtype=np.uint64)
    lde, root = orc.whir_commit(consts, evals)
    assert lde.shape == (8, 32)
    assert np.array_equal(lde, orc.lde(evals.reshape(4, 32), 1))
    _, root2 = orc.merkle_tree(consts, lde)
    assert np.array_equal(root, root2)


# ---- MLE / sumchecks: the reference's own tests, same seeds ------------------------------
def test_partial_then_full_matches_full(orc):
    # mle.rs:72-82
    rng = orc.XorShift64(2)
    values = rng.fields(16)
    point = rng.fields(4)
    rest = orc.mle_partial_eval(values, point[:2])
    assert rest.size == 4
    assert orc.mle_eval(rest, point[2:]) == orc.mle_eval(values, point)
    assert orc.mle_eval(values, point) == pyref.mle_eval([int(x) for x in values], [int(x) for x in point])


def test_eq_evals_definition(orc):
    rng = orc.XorShift64(11)
    r = rng.fields(5)
    eq = orc.eq_evals(r)
    vals = rng.fields(32)
    acc = sum(int(v) * int(e) for v, e in zip(vals, eq)) % P
    assert acc == orc.mle_eval(vals, r)


def test_sumcheck_completeness_and_soundness(orc):
    # sumcheck.rs:316-335
    rng = orc.XorShift64(3)
    t = 8
    f = rng.fields(1 << t)
    h = rng.fields(1 << t)
    true_sum = sum(int(a) * int(b) for a, b in zip(f, h)) % P
    ch = rng.fields(t)
    rounds, finals = orc.sumcheck_prove(f, h, ch)
    fe, he = orc.mle_eval(f, ch), orc.mle_eval(h, ch)
    assert (int(finals[0]), int(finals[1])) == (fe, he)
    assert orc.sumcheck_verify(rounds, true_sum, ch, fe, he)
    assert not orc.sumcheck_verify(rounds, (true_sum + 1) % P, ch, fe, he)
    pr, pf, ph = pyref.sumcheck_prove([int(x) for x in f], [int(x) for x in h], [int(x) for x in ch])
    assert [tuple(int(x) for x in r) for r in rounds] == pr and (pf, ph) == (fe, he)


def test_sumcheck3_completeness_and_soundness(orc):
    # sumcheck.rs:337-366
    rng = orc.XorShift64(4)
    t = 8
    f, g, h = rng.fields(1 << t), rng.fields(1 << t), rng.fields(1 << t)
    true_sum = sum(int(a) * int(b) * int(c) for a, b, c in zip(f, g, h)) % P
    ch = rng.fields(t)
    rounds, finals = orc.sumcheck3_prove(f, g, h, ch)
    fe, ge, he = (orc.mle_eval(x, ch) for x in (f, g, h))
    assert tuple(int(x) for x in finals) == (fe, ge, he)
    assert orc.sumcheck3_verify(rounds, true_sum, ch, fe, ge, he)
    assert not orc.sumcheck3_verify(rounds, (true_sum + 1) % P, ch, fe, ge, he)


def test_virtual_sumcheck_roundtrip(orc):
    # sumcheck.rs:490-527
    rng = orc.XorShift64(0xBEEF)
    n = 1 << 6
    f, g, h = rng.fields(n), rng.fields(n), rng.fields(n)
    t = 6
    ch = rng.fields(t)
    terms = [(3, [0, 1]), (orc.from_i64(-2), [1, 2]), (1, [0, 1, 2])]
    claimed = sum(3 * int(f[i]) * int(g[i]) + orc.from_i64(-2) * int(g[i]) * int(h[i]) +
                  int(f[i]) * int(g[i]) * int(h[i]) for i in range(n)) % P
    mles = np.stack([f, g, h])
    rounds, finals = orc.virtual_prove(mles, terms, ch)
    for m, ev in zip((f, g, h), finals):
        assert orc.mle_eval(m, ch) == int(ev)
    assert orc.virtual_verify(rounds, terms, claimed, ch, finals)
    bad = finals.copy()
    bad[0] = (int(bad[0]) + 1) % P
    assert not orc.virtual_verify(rounds, terms, claimed, ch, bad)


def test_eq_weighted_sumcheck(orc):
    # sumcheck.rs:528-548
    rng = orc.XorShift64(0xC0DE)
    n = 1 << 5
    f = rng.fields(n)
    r = rng.fields(5)
    eq = orc.eq_evals(r)
    claimed = orc.mle_eval(f, r)
    rounds, finals = orc.virtual_prove(np.stack([eq, f]), [(1, [0, 1])], r)
    assert orc.virtual_verify(rounds, [(1, [0, 1])], claimed, r, finals)


def test_sum_of_products(orc):
    rng = orc.XorShift64(77)
    w = np.stack([rng.fields(16) for _ in range(3)])
    v = np.stack([rng.fields(16) for _ in range(3)])
    ch = rng.fields(4)
    claimed = sum(int(a) * int(b) for a, b in zip(w.ravel(), v.ravel())) % P
    rounds, b_eval = orc.sum_of_products_prove(w, v, ch)
    expected = sum(orc.mle_eval(w[i], ch) * orc.mle_eval(v[i], ch) for i in range(3)) % P
    assert b_eval == expected
    assert orc.sumcheck_verify(rounds, claimed, ch, 1, b_eval)  # same round algebra, final check b_eval


def _mm(a, b):
    m, k = a.shape
    n = b.shape[1]
    return np.array([[sum(int(a[i, q]) * int(b[q, j]) for q in range(k)) % P for j in range(n)] for i in range(m)],
                    dtype=np.uint64)


def test_nested_chain_roundtrip_step(orc):
    # matmul.rs:145-182 (the single-contraction proofs it chains)
    rng = orc.XorShift64(0xC0FFEE)
    m = k = n = 4
    a = np.array([rng.field() for _ in range(m * k)], dtype=np.uint64).reshape(m, k)
    b = np.array([rng.field() for _ in range(k * n)], dtype=np.uint64).reshape(k, n)
    c = _mm(a, b)
    assert np.array_equal(orc.matmul_field(a, b), c)
    u, v, ch = rng.fields(2), rng.fields(2), rng.fields(2)
    claimed, rounds, finals = orc.matmul_prove(a.T.copy(), b, c, m, k, n, u, v, ch)
    assert orc.sumcheck_verify(rounds, claimed, ch, int(finals[0]), int(finals[1]))
    assert not orc.sumcheck_verify(rounds, (claimed + 1) % P, ch, int(finals[0]), int(finals[1]))
    # final evaluations are the claims on A and B at (ch||u) and (v||ch)
    assert int(finals[0]) == orc.mle_eval(a.ravel(), np.concatenate([ch, u]))
    assert int(finals[1]) == orc.mle_eval(b.ravel(), np.concatenate([v, ch]))


def test_op_shard_matmul_roundtrip(orc):
    # compose.rs:5199-5224 shape and seed: XorShift64(0x1818), values next_u64() % 50
    rng = orc.XorShift64(0x1818)
    m, k, n = 4, 8, 8
    a = np.array([rng.next_u64() % 50 for _ in range(m * k)], dtype=np.uint64).reshape(m, k)
    b = np.array([rng.next_u64() % 50 for _ in range(k * n)], dtype=np.uint64).reshape(k, n)
    c = orc.matmul_field(a, b)
    res = orc.op_matmul_prove(a, b, c, m, k, n, rng)
    assert res["u"].size == 2 and res["v"].size == 3 and res["ch"].size == 3
    assert orc.sumcheck_verify(res["rounds"], res["claimed"], res["ch"], *map(int, res["finals"]))
    assert int(res["claims"][0]) == int(res["finals"][0])
    assert int(res["claims"][1]) == int(res["finals"][1])
    assert int(res["claims"][2]) == res["claimed"]


def test_shard_dag_child_matches_definition(orc):
    t = orc.shard_dag_child([[0, 1, 2]], 1, 0)
    state = hashlib.sha256(b"zkie-shard-dag-v1").digest()
    for x in (1, 1, 0, 1, 2, 0):
        state = hashlib.sha256(state + x.to_bytes(8, "little")).digest()
    assert t.state()[0] == state
