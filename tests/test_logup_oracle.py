"""CPU checks of the logUp GKR oracle (crates/zkie-core/src/common/logup_gkr.rs):
the reference's own tests replayed with the reference's seeds and shapes
(:533-730), plus an independent pure-Python restatement of the first layer."""
import numpy as np

from tests import pyref

P = pyref.P


def frac_sum(num, den):
    return sum(int(a) * pow(int(b), P - 2, P) for a, b in zip(num, den)) % P


def draw(rng, lg):
    return [rng.field() for _ in range(lg)], [rng.field() for _ in range(lg)]


def seeded_fraction(orc, seed):
    rng = orc.XorShift64(seed)
    n = 1 << 6
    num = [rng.field() for _ in range(n)]
    den = [orc.from_i64(i % 7 + 1) for i in range(n)]
    return rng, num, den


def test_fractional_roundtrip(orc):
    # fractional_roundtrip (:533-556), seed 0xDEC0
    rng, num, den = seeded_fraction(orc, 0xDEC0)
    claimed = frac_sum(num, den)
    full_r, cs = draw(rng, 6)
    rounds, finals, fn, fd = orc.fractional_prove(num, den, full_r, cs)
    assert orc.fractional_verify(num, den, full_r, cs, rounds, fn, fd, claimed)
    assert not orc.fractional_verify(num, den, full_r, cs, rounds, (fn + 1) % P, fd, claimed)
    assert fn == claimed * fd % P


def test_fractional_roundtrip_storefree_and_chain(orc):
    # fractional_roundtrip_storefree (:557-571, 0xDEC1) and _chain (:572-586, 0xDEC2):
    # the stored final evaluations pass; bumping eq's (index 0) or num_lo's
    # (index 3) final evaluation in layer 0 fails.
    for seed, bump in ((0xDEC1, 0), (0xDEC2, 3)):
        rng, num, den = seeded_fraction(orc, seed)
        claimed = frac_sum(num, den)
        full_r, cs = draw(rng, 6)
        rounds, finals, fn, fd = orc.fractional_prove(num, den, full_r, cs)
        assert orc.fractional_chain_core(full_r, cs, rounds, finals) and fn == claimed * fd % P
        bad = finals.copy()
        bad[0, bump] = (int(bad[0, bump]) + 1) % P
        assert not orc.fractional_chain_core(full_r, cs, rounds, bad)


def lookup_case(orc, seed, n=64, t=16):
    rng = orc.XorShift64(seed)
    table = [rng.field() for _ in range(t)]
    x = [rng.next_u64() % t for _ in range(n)]
    y = [table[i] for i in x]
    alpha, beta = rng.field(), rng.field()
    return rng, table, x, y, alpha, beta


def test_lookup_fractional_roundtrip(orc):
    # lookup_fractional_roundtrip (:587-607), seed 0x10AD
    rng, table, x, y, alpha, beta = lookup_case(orc, 0x10AD)
    num, den = orc.lookup_num_den(x, y, table, None, 0, alpha, beta)
    assert num.size == 128
    full_r, cs = draw(rng, 7)
    rounds, finals, fn, fd = orc.fractional_prove(num, den, full_r, cs)
    assert orc.fractional_verify(num, den, full_r, cs, rounds, fn, fd, 0)
    bad_y = list(y)
    bad_y[0] = (bad_y[0] + 1) % P
    num2, den2 = orc.lookup_num_den(x, bad_y, table, None, 0, alpha, beta)
    full_r, cs = draw(rng, 7)
    rounds, finals, fn, fd = orc.fractional_prove(num2, den2, full_r, cs)
    assert not orc.fractional_verify(num2, den2, full_r, cs, rounds, fn, fd, 0)


def test_fractional_leaf_matches_direct_eval(orc):
    # fractional_leaf_matches_direct_eval (:608-637), seed 0x1EAF
    rng, table, x, y, alpha, beta = lookup_case(orc, 0x1EAF)
    num, den = orc.lookup_num_den(x, y, table, None, 0, alpha, beta)
    full_r, cs = draw(rng, 7)
    rounds, finals, fn, fd = orc.fractional_prove(num, den, full_r, cs)
    top = full_r[-1]
    num_leaf = ((1 - top) * int(finals[0, 3]) + top * int(finals[0, 4])) % P
    den_leaf = ((1 - top) * int(finals[0, 5]) + top * int(finals[0, 6])) % P
    assert num_leaf == orc.mle_eval(num, full_r)
    assert den_leaf == orc.mle_eval(den, full_r)


def test_lookup_fractional_chain_roundtrip(orc):
    # lookup_fractional_chain_roundtrip (:663-678), seed 0x11AD
    rng, table, x, y, alpha, beta = lookup_case(orc, 0x11AD)
    num, den = orc.lookup_num_den(x, y, table, None, 0, alpha, beta)
    full_r, cs = draw(rng, 7)
    rounds, finals, fn, fd = orc.fractional_prove(num, den, full_r, cs)
    assert orc.fractional_verify(num, den, full_r, cs, rounds, fn, fd, 0)
    assert orc.fractional_chain_core(full_r, cs, rounds, finals) and fn == 0
    finals[0, 3] = (int(finals[0, 3]) + 1) % P
    assert not orc.fractional_chain_core(full_r, cs, rounds, finals)


def test_lookup_split_matches_merged(orc):
    # lookup_split_matches_merged (:679-695), seed 0x5E17: the witness side
    # and the table side (own multiplicities) agree on the fractional sum.
    rng, table, x, y, alpha, beta = lookup_case(orc, 0x5E17)
    num, den = orc.lookup_num_den(x, y, table, None, 0, alpha, beta)
    full_r, cs = draw(rng, 7)
    rounds, finals, fn, fd = orc.fractional_prove(num, den, full_r, cs)
    assert orc.fractional_verify(num, den, full_r, cs, rounds, fn, fd, 0)
    m = np.bincount(np.array(x), minlength=16).astype(np.uint64)
    wn, wd = orc.lookup_num_den(x, y, None, None, 1, alpha, beta)
    wr, wc = draw(rng, 6)
    w_rounds, w_finals, w_fn, w_fd = orc.fractional_prove(wn, wd, wr, wc)
    tn, td = orc.lookup_num_den(None, None, table, m, 3, alpha, beta)
    tr, tc = draw(rng, 4)
    t_rounds, t_finals, t_fn, t_fd = orc.fractional_prove(tn, td, tr, tc)
    assert orc.fractional_chain_core(wr, wc, w_rounds, w_finals)
    assert orc.fractional_chain_core(tr, tc, t_rounds, t_finals)
    assert w_fn * t_fd % P == t_fn * w_fd % P


def test_lookup_columns_match_definition(orc):
    """The four column builders against a direct restatement, including the
    padding rows and the out-of-table rejection."""
    rng, table, x, y, alpha, beta = lookup_case(orc, 0xC01, n=21, t=9)
    den_of = lambda j, v: (alpha + j + beta * v) % P  # noqa: E731
    num, den = orc.lookup_num_den(x, y, table, None, 0, alpha, beta)
    m = np.bincount(np.array(x), minlength=9)
    assert num.size == 32
    assert list(num[:21]) == [1] * 21 and [int(d) for d in den[:21]] == [den_of(a, b) for a, b in zip(x, y)]
    assert [int(v) for v in num[21:30]] == [(-int(c)) % P for c in m]
    assert [int(d) for d in den[21:30]] == [den_of(j, table[j]) for j in range(9)]
    assert list(num[30:]) == [0, 0] and list(den[30:]) == [1, 1]
    wn, wd = orc.lookup_num_den(x, y, None, None, 1, alpha, beta)
    assert wn.size == 32 and list(wd[21:]) == [1] * 11
    cn, cd = orc.lookup_num_den(x[:3], y[:3], None, None, 2, alpha, beta)
    assert cn.size == 32 and list(cn[3:]) == [0] * 29 and [int(d) for d in cd[3:]] == [alpha] * 29
    tn, td = orc.lookup_num_den(None, None, table, m.astype(np.uint64), 3, alpha, beta)
    assert tn.size == 16 and [int(v) for v in tn[:9]] == [int(c) for c in m] and list(tn[9:]) == [0] * 7
    assert [int(d) for d in td] == [den_of(j, table[j] if j < 9 else 0) for j in range(16)]
    assert orc.lookup_num_den([9], [0], table, None, 0, alpha, beta) is None


def test_first_layer_matches_python(orc):
    """Layer 0's tables and round 0 of its virtual sumcheck, restated in plain
    Python from logup_gkr.rs:43-58 and sumcheck.rs:394-415."""
    rng = orc.XorShift64(0xF00D)
    lg = 4
    num = [rng.field() for _ in range(16)]
    den = [rng.field() for _ in range(16)]
    full_r, cs = draw(rng, lg)
    rounds, finals, fn, fd = orc.fractional_prove(num, den, full_r, cs)
    half = 8
    nn = [(num[s] * den[half + s] + num[half + s] * den[s]) % P for s in range(half)]
    nd = [den[s] * den[half + s] % P for s in range(half)]
    r = full_r[:3]
    eq = [1] * 8
    for x in range(8):
        for j in range(3):
            eq[x] = eq[x] * (r[j] if (x >> j) & 1 else (1 - r[j])) % P
    mles = [eq, nn, nd, num[:half], num[half:], den[:half], den[half:]]
    c = cs[0]
    terms = [(1, [0, 1]), (P - 1, [0, 3, 6]), (P - 1, [0, 4, 5]), (c, [0, 2]), ((P - 1) * c % P, [0, 5, 6])]
    for k in range(4):
        acc = 0
        for s in range(4):
            for coeff, ids in terms:
                prod = coeff
                for j in ids:
                    f0, f1 = mles[j][2 * s], mles[j][2 * s + 1]
                    prod = prod * ((k * f1 - (k - 1) * f0) % P) % P
                acc = (acc + prod) % P
        assert int(rounds[0][0, k]) == acc
    # the zero-layer case: a single fraction
    r0, f0, fn0, fd0 = orc.fractional_prove([5], [7], [], [])
    assert r0 == [] and (fn0, fd0) == (5, 7)
