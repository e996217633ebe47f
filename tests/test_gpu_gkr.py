"""GPU parity of the matmul GKR path (MLE contractions, the degree-2
sumcheck, matmul::prove, the Op::MatMul arm) against the CPU oracle,
bit-exact, through the C ABI."""
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


def signed16(seed, n):
    g = np.random.default_rng(seed)
    x = g.integers(-(2 ** 15), 2 ** 15, size=n, dtype=np.int64)
    return np.where(x >= 0, x, np.int64(0)).astype(np.uint64) + np.where(x < 0, (np.uint64(P) - (-x).astype(np.uint64)), np.uint64(0))


@pytest.mark.parametrize("t", [0, 1, 4, 10, 15, 20])
def test_eq_and_eval(zk, orc, t):
    vals = fields(t, 1 << t)
    pt = fields(100 + t, t)
    assert zk.mle_eval(vals, pt) == orc.mle_eval(vals, pt)
    if t <= 12:
        assert np.array_equal(zk.eq_evals(pt).cpu().numpy(), orc.eq_evals(pt))


@pytest.mark.parametrize("t,f", [(4, 0), (4, 2), (10, 4), (10, 10), (20, 10), (20, 4), (22, 21)])
def test_partial_eval(zk, orc, t, f):
    vals = fields(t * 3 + f, 1 << t)
    fix = fields(7 + f, f)
    assert np.array_equal(zk.mle_partial_eval(vals, fix).cpu().numpy(), orc.mle_partial_eval(vals, fix))


@pytest.mark.parametrize("t", [0, 1, 2, 8, 10, 11, 12, 16, 22, 23])
def test_sumcheck_matches_oracle(zk, orc, t):
    f, h, ch = fields(t, 1 << t), fields(t + 50, 1 << t), fields(t + 99, t)
    got = zk.sumcheck_prove(f, h, 0, ch)
    rounds, finals = orc.sumcheck_prove(f, h, ch)
    assert np.array_equal(got.rounds, rounds)
    assert (got.f_eval, got.h_eval) == (int(finals[0]), int(finals[1]))
    if t <= 16:
        claimed = int(sum(int(a) * int(b) for a, b in zip(f, h)) % P)
        assert orc.sumcheck_verify(got.rounds, claimed, ch, got.f_eval, got.h_eval)


def noncanonical(v):
    """The same field elements, with every value below 2^32 - 1 replaced by v + p."""
    return np.where(v < np.uint64(0xFFFFFFFF), v + np.uint64(P), v)


def offset_tensor(v):
    """A device tensor holding v whose data pointer is 8 bytes past a 16-byte boundary."""
    import torch
    t = torch.zeros(v.size + 1, dtype=torch.uint64, device="cuda")
    t[1:] = torch.from_numpy(v).cuda()
    out = t[1:]
    assert out.data_ptr() % 16 == 8
    return out


@pytest.mark.parametrize("t", [3, 5, 9, 13, 17, 18, 19, 24])
def test_sumcheck_level_boundaries(zk, orc, t):
    """Sizes around the nine-round chunk levels (9 | 9+4 | 9+9 | 9+9+1 | 9+9+6),
    inputs given as non-canonical representatives."""
    f, h, ch = fields(3 * t, 1 << t), fields(3 * t + 1, 1 << t), fields(3 * t + 2, t)
    got = zk.sumcheck_prove(noncanonical(f), noncanonical(h), 0, ch)
    rounds, finals = orc.sumcheck_prove(f, h, ch)
    assert np.array_equal(got.rounds, rounds)
    assert (got.f_eval, got.h_eval) == (int(finals[0]), int(finals[1]))


@pytest.mark.parametrize("t", [4, 12, 19])
def test_sumcheck_unaligned_inputs(zk, orc, t):
    """Inputs 8 bytes off a 16-byte boundary take the scalar-load path."""
    f, h, ch = fields(5 * t, 1 << t), fields(5 * t + 1, 1 << t), fields(5 * t + 2, t)
    got = zk.sumcheck_prove(offset_tensor(f), offset_tensor(h), 0, ch)
    rounds, finals = orc.sumcheck_prove(f, h, ch)
    assert np.array_equal(got.rounds, rounds)
    assert (got.f_eval, got.h_eval) == (int(finals[0]), int(finals[1]))


@pytest.mark.parametrize("t,f", [(6, 1), (6, 3), (6, 5), (12, 6), (16, 12)])
def test_partial_eval_unaligned_noncanonical(zk, orc, t, f):
    vals = fields(t * 5 + f, 1 << t)
    fix = fields(11 + f, f)
    want = orc.mle_partial_eval(vals, fix)
    assert np.array_equal(zk.mle_partial_eval(offset_tensor(vals), fix).cpu().numpy(), want)
    assert np.array_equal(zk.mle_partial_eval(noncanonical(vals), fix).cpu().numpy(), want)


@pytest.mark.parametrize("m,k,n", [(64, 256, 128), (256, 512, 256), (1024, 32, 64)])
def test_op_matmul_row_blocks(zk, orc, m, k, n):
    """Row contraction of A split over several row blocks; A, B, C arbitrary
    field matrices (the proof is computed whether or not C = A B)."""
    a = fields(m, m * k).reshape(m, k)
    b = fields(k, k * n).reshape(k, n)
    c = fields(n, m * n).reshape(m, n)
    got = zk.op_matmul_prove(a, b, c, m, k, n, zk.XorShift64(m + k + n))
    exp = orc.op_matmul_prove(a, b, c, m, k, n, orc.XorShift64(m + k + n))
    assert got.proof.claimed == exp["claimed"]
    assert np.array_equal(got.proof.sumcheck.rounds, exp["rounds"])
    assert np.array_equal(got.claims, exp["claims"])


def test_sumcheck_reference_seed(zk, orc):
    # sumcheck.rs:316-335 with the reference's seed
    rng = orc.XorShift64(3)
    f, h = rng.fields(256), rng.fields(256)
    true_sum = sum(int(a) * int(b) for a, b in zip(f, h)) % P
    ch = rng.fields(8)
    p = zk.sumcheck_prove(f, h, true_sum, ch)
    assert orc.sumcheck_verify(p.rounds, true_sum, ch, p.f_eval, p.h_eval)
    assert not orc.sumcheck_verify(p.rounds, (true_sum + 1) % P, ch, p.f_eval, p.h_eval)


@pytest.mark.parametrize("m,k,n", [(1, 1, 1), (2, 4, 8), (4, 4, 4), (16, 64, 32), (16, 1024, 1024)])
def test_matmul_prove_matches_oracle(zk, orc, m, k, n):
    a = signed16(m + k, m * k).reshape(m, k)
    b = signed16(n + 3, k * n).reshape(k, n)
    c = orc.matmul_field(a, b)
    assert np.array_equal(zk.matmul_field(a, b, m, k, n).cpu().numpy().reshape(m, n), c)
    lm, lk, ln = (m.bit_length() - 1, k.bit_length() - 1, n.bit_length() - 1)
    u, v, ch = fields(1, lm), fields(2, ln), fields(3, lk)
    at = a.T.copy()
    got = zk.matmul_prove(at, b, c, m, k, n, u, v, ch)
    claimed, rounds, finals = orc.matmul_prove(at, b, c, m, k, n, u, v, ch)
    assert got.claimed == claimed
    assert np.array_equal(got.sumcheck.rounds, rounds)
    assert (got.sumcheck.f_eval, got.sumcheck.h_eval) == tuple(int(x) for x in finals)


def test_op_matmul_xorshift_reference_test(zk, orc):
    # compose.rs:5199-5224: XorShift64(0x1818), m,k,n = 4,8,8, entries next_u64() % 50
    zr, orr = zk.XorShift64(0x1818), orc.XorShift64(0x1818)
    m, k, n = 4, 8, 8
    a = np.array([orr.next_u64() % 50 for _ in range(m * k)], dtype=np.uint64).reshape(m, k)
    b = np.array([orr.next_u64() % 50 for _ in range(k * n)], dtype=np.uint64).reshape(k, n)
    for _ in range(m * k + k * n):
        zr.next_u64()
    c = orc.matmul_field(a, b)
    got = zk.op_matmul_prove(a, b, c, m, k, n, zr)
    exp = orc.op_matmul_prove(a, b, c, m, k, n, orr)
    assert np.array_equal(got.u, exp["u"]) and np.array_equal(got.v, exp["v"]) and np.array_equal(got.ch, exp["ch"])
    assert got.proof.claimed == exp["claimed"]
    assert np.array_equal(got.proof.sumcheck.rounds, exp["rounds"])
    assert np.array_equal(got.claims, exp["claims"])
    assert zr.field() == orr.field()  # both sources advanced identically


def test_op_matmul_cfg1_transcript(zk, orc):
    """BASELINE config 1 shape (16x768 @ 768x768 padded to 16x1024 @ 1024x1024),
    challenges from the shard-DAG child transcript."""
    m, k, n = 16, 1024, 1024
    a = np.zeros((m, k), dtype=np.uint64)
    b = np.zeros((k, n), dtype=np.uint64)
    a[:, :768] = signed16(11, m * 768).reshape(m, 768)
    b[:768, :768] = signed16(12, 768 * 768).reshape(768, 768)
    c = orc.matmul_field(a, b)
    ids = [[0, 1, 2]]
    got = zk.op_matmul_prove(a, b, c, m, k, n, zk.shard_dag_child(ids, 1, 0))
    exp = orc.op_matmul_prove(a, b, c, m, k, n, orc.shard_dag_child(ids, 1, 0))
    assert got.proof.claimed == exp["claimed"]
    assert np.array_equal(got.proof.sumcheck.rounds, exp["rounds"])
    assert np.array_equal(got.claims, exp["claims"])
    assert np.array_equal(got.u, exp["u"]) and np.array_equal(got.ch, exp["ch"])


@pytest.mark.parametrize("m,k,n", [(16, 1024, 1024), (4, 64, 32), (32, 256, 512)])
def test_shard_prove_matmul_matches_composition(zk, orc, m, k, n):
    """The fused four-stream shard call equals its parts run one by one:
    forward C, the three WHIR commits and the Op::MatMul proof with the
    shard's child transcript (and the oracle for C and the proof)."""
    zk.check(zk.lib.zkie2_p2_init_default(), "constants")
    a = signed16(m * 3 + k, m * k).reshape(m, k)
    w = signed16(n * 5 + k, k * n).reshape(k, n)
    res = zk.ShardProver(m, k, n).prove(a, w, op_ids=(4, 5, 6), ops_per_shard=1, shard_index=2)
    c = orc.matmul_field(a, w)
    assert np.array_equal(res.c.cpu().numpy(), c)
    for i, t in enumerate((w, a, c)):
        assert np.array_equal(res.roots[i], np.asarray(zk.Whir.with_params(int(t.size).bit_length() - 1, 90, 17)
                                                          .commit(t.reshape(-1)).root, dtype=np.uint64)), i
    exp = orc.op_matmul_prove(a, w, c, m, k, n, orc.shard_dag_child([[4, 5, 6]], 1, 2))
    assert res.proof.proof.claimed == exp["claimed"]
    assert np.array_equal(res.proof.proof.sumcheck.rounds, exp["rounds"])
    assert np.array_equal(res.proof.claims, exp["claims"])
    assert np.array_equal(res.proof.u, exp["u"]) and np.array_equal(res.proof.ch, exp["ch"])
