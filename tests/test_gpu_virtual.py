"""GPU parity of the batch-opening sumcheck (prove_sum_of_products,
sumcheck.rs:243-286) and the virtual-polynomial sumcheck (prove_virtual,
sumcheck.rs:378-438) against the CPU oracle, bit-exact, through the C ABI."""
import numpy as np
import pytest

P = 0xFFFFFFFF00000001
pytestmark = pytest.mark.gpu


def fields(seed, n):
    g = np.random.default_rng(seed)
    v = g.integers(0, 2 ** 64, size=n, dtype=np.uint64)
    bad = v >= np.uint64(P)
    while bad.any():
        v[bad] = g.integers(0, 2 ** 64, size=int(bad.sum()), dtype=np.uint64)
        bad = v >= np.uint64(P)
    return v


def neg(x):
    return (P - x) % P


@pytest.mark.parametrize("n,t", [(1, 0), (1, 1), (3, 4), (5, 9), (2, 10), (7, 13), (4, 18), (1, 20)])
def test_sum_of_products_matches_oracle(zk, orc, n, t):
    w = np.stack([fields(100 * t + i, 1 << t) for i in range(n)])
    v = np.stack([fields(200 * t + i, 1 << t) for i in range(n)])
    ch = fields(300 + t, t)
    got = zk.prove_sum_of_products(w, v, 0, ch)
    rounds, b_eval = orc.sum_of_products_prove(w, v, ch)
    assert np.array_equal(got.rounds, rounds)
    assert got.b_eval == b_eval


def test_sum_of_products_verifies(zk, orc):
    """Completeness: the reference verifier relation (sumcheck_verify with the
    final check b_eval) holds, and fails for a wrong claim."""
    rng = orc.XorShift64(77)
    w = np.stack([rng.fields(1 << 10) for _ in range(3)])
    v = np.stack([rng.fields(1 << 10) for _ in range(3)])
    ch = rng.fields(10)
    claimed = sum(int(a) * int(b) for a, b in zip(w.ravel(), v.ravel())) % P
    got = zk.prove_sum_of_products(w, v, claimed, ch)
    assert orc.sumcheck_verify(got.rounds, claimed, ch, 1, got.b_eval)
    assert not orc.sumcheck_verify(got.rounds, (claimed + 1) % P, ch, 1, got.b_eval)


# Term shapes of the reference's callers: Projection affine (projection.rs:
# 74-83), the Add arm (compose.rs:380-392), a degree-3 product, a constant
# term, a term repeating one MLE.
AFFINE = [(1, [0, 1]), (neg(1), [0, 2]), (1 << 16, [0, 3]), (neg(1 << 16), [0, 4]), (neg(1 << 15), [0, 5])]
ADD = [(1, [2]), (neg(1), [0]), (neg(1), [1])]
CUBIC = [(3, [0, 1]), (neg(2), [1, 2]), (1, [0, 1, 2])]
MIXED = [(5, []), (7, [0, 0, 1]), (neg(9), [3, 2, 1, 0]), (11, [2])]


@pytest.mark.parametrize("terms,n_mles", [(AFFINE, 6), (ADD, 3), (CUBIC, 3), (MIXED, 4)])
@pytest.mark.parametrize("t", [0, 1, 5, 9, 10, 12, 17])
def test_prove_virtual_matches_oracle(zk, orc, terms, n_mles, t):
    mles = np.stack([fields(1000 * t + 17 * n_mles + j, 1 << t) for j in range(n_mles)])
    ch = fields(7 * t + n_mles, t)
    got = zk.prove_virtual(list(mles), terms, 0, ch)
    rounds, finals = orc.virtual_prove(mles, terms, ch)
    assert np.array_equal(got.rounds, rounds)
    assert np.array_equal(got.final_evals, finals)


@pytest.mark.parametrize("n_mles,t", [(16, 12), (1, 16), (8, 21)])
def test_prove_virtual_table_counts(zk, orc, n_mles, t):
    """Many tables (fewer rounds per launch), one table, and a large case."""
    mles = np.stack([fields(5000 + j, 1 << t) for j in range(n_mles)])
    terms = [(j + 1, [j, (j + 1) % n_mles]) for j in range(n_mles)] + [(2, [0])]
    ch = fields(6000 + t, t)
    got = zk.prove_virtual(list(mles), terms, 0, ch)
    rounds, finals = orc.virtual_prove(mles, terms, ch)
    assert np.array_equal(got.rounds, rounds)
    assert np.array_equal(got.final_evals, finals)


def test_prove_virtual_verifies(zk, orc):
    # sumcheck.rs:490-527 shape: f, g, h with terms 3fg - 2gh + fgh
    rng = orc.XorShift64(0xBEEF)
    t = 11
    f, g, h = rng.fields(1 << t), rng.fields(1 << t), rng.fields(1 << t)
    ch = rng.fields(t)
    terms = [(3, [0, 1]), (orc.from_i64(-2), [1, 2]), (1, [0, 1, 2])]
    ff, gg, hh = (x.astype(object) for x in (f, g, h))
    claimed = int((3 * ff * gg + orc.from_i64(-2) * gg * hh % P + ff * gg % P * hh).sum() % P)
    got = zk.prove_virtual([f, g, h], terms, claimed, ch)
    assert orc.virtual_verify(got.rounds, terms, claimed, ch, got.final_evals)
    bad = got.final_evals.copy()
    bad[1] = (int(bad[1]) + 1) % P
    assert not orc.virtual_verify(got.rounds, terms, claimed, ch, bad)


def test_prove_virtual_rejects_bad_terms(zk):
    from zkie_b200 import ZkieError
    m = fields(1, 8)
    with pytest.raises(ZkieError):
        zk.prove_virtual([m, m], [(1, [0, 2])], 0, fields(2, 3))  # index out of range
    with pytest.raises(ZkieError):
        zk.prove_virtual([m], [(1, [0] * 9)], 0, fields(2, 3))  # degree 9 > 8
