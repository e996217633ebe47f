"""GPU parity of the logUp GKR fraction tree (prove_fractional_with_challenges,
logup_gkr.rs:29-69) and the lookup column builders (:210-301, 340-370) against
the CPU oracle, bit-exact, through the C ABI; plus size-independent properties
at full size (a valid lookup's fractions sum to zero, the layer chain verifies,
the leaf equals the MLE of the input columns)."""
import numpy as np
import pytest

P = 0xFFFFFFFF00000001
pytestmark = pytest.mark.gpu


def fields(seed, n, noncanon=False):
    g = np.random.default_rng(seed)
    v = g.integers(0, 2 ** 64, size=n, dtype=np.uint64)
    if not noncanon:
        v[v >= np.uint64(P)] -= np.uint64(P)
    return v


def assert_same(got, ref):
    rounds, finals, fn, fd = ref
    assert len(got.layers) == len(rounds)
    for layer, r_ref, f_ref in zip(got.layers, rounds, finals):
        assert np.array_equal(layer.proof.rounds, r_ref)
        assert np.array_equal(layer.proof.final_evals, f_ref)
    assert (got.final_num, got.final_den) == (fn, fd)


@pytest.mark.parametrize("lg", [0, 1, 2, 3, 6, 9, 10, 11, 13, 16, 18, 20])
def test_fractional_matches_oracle(zk, orc, lg):
    n = 1 << lg
    num, den = fields(10 + lg, n, noncanon=True), fields(20 + lg, n, noncanon=True)
    full_r, cs = fields(30 + lg, lg), fields(40 + lg, lg)
    got = zk.prove_fractional_with_challenges(num, den, full_r, cs)
    assert_same(got, orc.fractional_prove(num, den, full_r, cs))
    for i, layer in enumerate(got.layers):
        assert np.array_equal(layer.r, full_r[:lg - i - 1]) and layer.c == int(cs[i])


def test_fractional_reference_seed(zk, orc):
    """fractional_roundtrip (logup_gkr.rs:533-556, seed 0xDEC0) through the
    product API: the device proof equals the oracle's and verifies."""
    rng, orng = zk.XorShift64(0xDEC0), orc.XorShift64(0xDEC0)
    num = np.array([rng.field() for _ in range(64)], dtype=np.uint64)
    assert [orng.field() for _ in range(64)] == [int(v) for v in num]
    den = np.array([i % 7 + 1 for i in range(64)], dtype=np.uint64)
    claimed = sum(int(a) * pow(int(b), P - 2, P) for a, b in zip(num, den)) % P
    got = zk.prove_fractional(num, den, rng)
    full_r, cs = [orng.field() for _ in range(6)], [orng.field() for _ in range(6)]
    assert list(got.full_r) == full_r and [layer.c for layer in got.layers] == cs
    ref = orc.fractional_prove(num, den, full_r, cs)
    assert_same(got, ref)
    rounds = [layer.proof.rounds for layer in got.layers]
    assert orc.fractional_verify(num, den, full_r, cs, rounds, got.final_num, got.final_den, claimed)
    assert not orc.fractional_verify(num, den, full_r, cs, rounds, (got.final_num + 1) % P, got.final_den, claimed)


def lookup_inputs(seed, n, t):
    g = np.random.default_rng(seed)
    table = fields(seed + 1, t)
    x = g.integers(0, max(t, 1), size=n).astype(np.uint32)
    y = table[x] if t else fields(seed + 2, n)
    alpha, beta = int(fields(seed + 3, 1)[0]), int(fields(seed + 4, 1)[0])
    return table, x, y, alpha, beta


@pytest.mark.parametrize("n,t", [(0, 1), (1, 1), (21, 9), (64, 16), (1000, 24), (3, 1 << 12), (1 << 15, 1 << 14),
                                 (1 << 17, 100)])
def test_lookup_columns_match_oracle(zk, orc, n, t):
    table, x, y, alpha, beta = lookup_inputs(n * 7 + t, n, t)
    m = np.bincount(x.astype(np.int64), minlength=t).astype(np.uint64)[:t]
    builders = [
        (0, lambda: zk.build_lookup_num_den(x, y, table, alpha, beta), (x, y, table, None)),
        (1, lambda: zk.build_lookup_witness_num_den(x, y, alpha, beta), (x, y, None, None)),
        (3, lambda: zk.build_lookup_table_num_den(m, table, alpha, beta), (None, None, table, m)),
    ]
    for mode, build, args in builders:
        num, den = build()
        rn, rd = orc.lookup_num_den(*args, mode, alpha, beta)
        assert np.array_equal(num.cpu().numpy(), rn), mode
        assert np.array_equal(den.cpu().numpy(), rd), mode
    assert np.array_equal(zk.lookup_multiplicity(x, t), m)


def test_lookup_index_outside_table_is_an_error(zk):
    table, x, y, alpha, beta = lookup_inputs(5, 40, 8)
    x[17] = 8
    with pytest.raises(zk.ZkieError):
        zk.build_lookup_num_den(x, y, table, alpha, beta)


def test_prove_lookup_matches_oracle(zk, orc):
    """prove_lookup_fractional / _columns / _batch, prove_lookup_witness(_batch,
    _batch_columns) and prove_lookup_table on the device against the oracle's
    columns and proofs, with the same challenge stream."""
    table, x, y, alpha, beta = lookup_inputs(99, 300, 50)
    rng, orng = zk.XorShift64(0xAB), orc.XorShift64(0xAB)

    def oracle_proof(num, den):
        lg = num.size.bit_length() - 1
        fr, cs = [orng.field() for _ in range(lg)], [orng.field() for _ in range(lg)]
        return orc.fractional_prove(num, den, fr, cs)

    got = zk.prove_lookup_fractional(x, y, table, alpha, beta, rng)
    assert got.final_num == 0
    assert_same(got, oracle_proof(*orc.lookup_num_den(x, y, table, None, 0, alpha, beta)))

    got, num, den = zk.prove_lookup_fractional_columns(x, y, table, alpha, beta, rng)
    rn, rd = orc.lookup_num_den(x, y, table, None, 0, alpha, beta)
    assert np.array_equal(num.cpu().numpy(), rn) and np.array_equal(den.cpu().numpy(), rd)
    assert_same(got, oracle_proof(rn, rd))

    xs, ys = [x[:100], x[100:130], x[130:]], [y[:100], y[100:130], y[130:]]
    got = zk.prove_lookup_fractional_batch(xs, ys, table, alpha, beta, rng)
    assert_same(got, oracle_proof(rn, rd))  # the merged batch of the same samples

    got = zk.prove_lookup_witness(x, y, alpha, beta, rng)
    assert_same(got, oracle_proof(*orc.lookup_num_den(x, y, None, None, 1, alpha, beta)))
    got = zk.prove_lookup_witness_batch(xs, ys, alpha, beta, rng)
    assert_same(got, oracle_proof(*orc.lookup_num_den(x, y, None, None, 1, alpha, beta)))

    got, xf, yf, num, den = zk.prove_lookup_witness_batch_columns([x[:5], x[5:9]], [y[:5], y[5:9]], alpha, beta, rng)
    cn, cd = orc.lookup_num_den(x[:9], y[:9], None, None, 2, alpha, beta)
    assert np.array_equal(num.cpu().numpy(), cn) and np.array_equal(den.cpu().numpy(), cd)
    assert list(xf.cpu().numpy()[:9]) == list(x[:9]) and not xf.cpu().numpy()[9:].any()
    assert list(yf.cpu().numpy()[:9]) == list(y[:9]) and not yf.cpu().numpy()[9:].any()
    assert_same(got, oracle_proof(cn, cd))

    m = zk.merge_multiplicity(xs, 50)
    got = zk.prove_lookup_table(m, table, alpha, beta, rng)
    assert_same(got, oracle_proof(*orc.lookup_num_den(None, None, table, m, 3, alpha, beta)))


@pytest.mark.parametrize("lg_n,lg_t", [(21, 20), (23, 16)])
def test_lookup_full_size_properties(zk, orc, lg_n, lg_t):
    """Full size: the valid lookup's fraction sum is zero (final_num = 0), the
    layer chain verifies from the proof alone, and the leaf (fractional_leaf)
    equals the MLEs of the device columns at full_r; a corrupted sample
    gives a nonzero sum."""
    import torch
    n, t = (1 << lg_n) - 5, 1 << lg_t
    table, x, y, alpha, beta = lookup_inputs(lg_n, n, t)
    rng = zk.XorShift64(0x5EED + lg_n)
    proof, num, den = zk.prove_lookup_fractional_columns(x, y, table, alpha, beta, rng)
    assert proof.final_num == 0 and proof.final_den != 0
    lg = num.numel().bit_length() - 1
    rounds = [layer.proof.rounds for layer in proof.layers]
    finals = np.stack([layer.proof.final_evals for layer in proof.layers])
    cs = [layer.c for layer in proof.layers]
    assert orc.fractional_chain_core(proof.full_r, cs, rounds, finals)
    full_r, num_leaf, den_leaf = zk.fractional_leaf(proof)
    assert num_leaf == zk.mle_eval(num, full_r) and den_leaf == zk.mle_eval(den, full_r)
    assert len(proof.layers) == lg
    y_bad = y.copy()
    y_bad[12345] = (int(y_bad[12345]) + 1) % P
    bad = zk.prove_lookup_fractional(x, y_bad, table, alpha, beta, zk.XorShift64(1))
    assert bad.final_num != 0
    torch.cuda.synchronize()
