"""GPU parity of the projection block (crates/zkie-ops/src/projection.rs) with
the oracle: the witness columns, the lookup indices, and whole proofs
(prove_projection: the MatMul GKR, the affine virtual sumcheck, alpha / beta
and the logUp range check) bit for bit on the reference's test seeds and on
16-bit fixed-point shapes up to a GPT-2 layer's projection widths, with both
challenge sources; the device proof verifies with the oracle's verifier and a
tampered one does not."""
import numpy as np
import pytest
import torch

P = 0xFFFFFFFF00000001
pytestmark = pytest.mark.gpu


def fixed(seed, size, lo=-(1 << 15), hi=1 << 15):
    x = np.random.default_rng(seed).integers(lo, hi, size=size, dtype=np.int64)
    return x.astype(np.uint64) + np.where(x < 0, np.uint64(P), np.uint64(0))


def assert_same(got, exp):
    assert got.matmul.claimed == exp["claimed"]
    assert np.array_equal(got.matmul.sumcheck.rounds, exp["mm_rounds"])
    assert (got.matmul.sumcheck.f_eval, got.matmul.sumcheck.h_eval) == tuple(int(v) for v in exp["mm_finals"])
    for a, b in (("u", "u"), ("v", "v"), ("ch", "ch"), ("pt", "pt")):
        assert np.array_equal(getattr(got, a), exp[b]), a
    assert np.array_equal(got.affine.rounds, exp["affine_rounds"])
    assert np.array_equal(got.affine.final_evals, exp["affine_finals"])
    assert (got.alpha, got.beta) == (exp["alpha"], exp["beta"])
    assert np.array_equal(got.frac.full_r, exp["full_r"])
    assert len(got.frac.layers) == len(exp["frac_rounds"])
    for lay, r, f in zip(got.frac.layers, exp["frac_rounds"], exp["frac_finals"]):
        assert np.array_equal(lay.proof.rounds, r)
        assert np.array_equal(lay.proof.final_evals, f)
    assert (got.frac.final_num, got.frac.final_den) == (exp["final_num"], exp["final_den"])


def to_oracle_dict(p, exp):
    """The device proof in the oracle's dictionary form (for its verifier)."""
    return dict(claimed=p.matmul.claimed, mm_rounds=p.matmul.sumcheck.rounds,
                mm_finals=np.array([p.matmul.sumcheck.f_eval, p.matmul.sumcheck.h_eval], dtype=np.uint64),
                ch=p.ch, pt=p.pt, affine_rounds=p.affine.rounds, affine_finals=p.affine.final_evals.copy(),
                full_r=p.frac.full_r, cs=exp["cs"], frac_rounds=[lay.proof.rounds for lay in p.frac.layers],
                frac_finals=np.stack([lay.proof.final_evals for lay in p.frac.layers]).copy(),
                final_num=p.frac.final_num)


def test_witness_and_index_match_oracle(zk, orc):
    from zkie_b200.projection import lookup_index, projection_witness
    n = 4096
    for shift in (1, 4, 16, 30):
        h = fixed(shift, n, -(1 << 40), 1 << 40)
        h[:8] = [orc.from_i64(v) for v in (0, -1, 1, (1 << (shift - 1)), -(1 << (shift - 1)), 7, -7, 1 << 41)]
        bias = fixed(shift + 100, n, -(1 << 20), 1 << 20)
        out, rem, idx = projection_witness(h, bias, shift)
        eo, er = orc.projection_witness(h, bias, shift)
        assert np.array_equal(out.cpu().numpy(), eo) and np.array_equal(rem.cpu().numpy(), er)
        assert np.array_equal(idx.cpu().numpy().astype(np.uint64), er)  # in range: the index is the value
    v = np.array([0, 5, 0x7FFFFFFF, 0x80000000, P - 1, P - 3, 1 << 40, (1 << 63) + 12345, P + 2], dtype=np.uint64)
    got = lookup_index(v).cpu().numpy()
    assert [int(g) for g in got] == [orc.to_i32_index(int(x) % P) for x in v]


@pytest.mark.parametrize("seed,m,k,n", [(0xABCD, 2, 2, 2), (0xDD22, 8, 8, 8)])
def test_reference_test_seeds(zk, orc, seed, m, k, n):
    """projection_block_roundtrip / committed_projection_roundtrip's inputs
    (values from the seeded XorShift64, shift 4), the same generator then
    drawing the proof's challenges."""
    from zkie_b200.projection import projection_witness, prove_projection
    orng, zrng = orc.XorShift64(seed), zk.XorShift64(seed)
    x = np.array([orc.from_i64(orng.next_u64() % 100) for _ in range(m * k)], dtype=np.uint64)
    w = np.array([orc.from_i64(orng.next_u64() % 100) for _ in range(k * n)], dtype=np.uint64)
    b = np.array([orc.from_i64(orng.next_u64() % 20 - 10) for _ in range(m * n)], dtype=np.uint64)
    for _ in range(m * k + k * n + m * n):
        zrng.next_u64()
    h = orc.matmul_field(x.reshape(m, k), w.reshape(k, n)).reshape(-1)
    out, rem = orc.projection_witness(h, b, 4)
    dout, drem, _ = projection_witness(torch.from_numpy(h).cuda(), b, 4)
    assert np.array_equal(dout.cpu().numpy(), out) and np.array_equal(drem.cpu().numpy(), rem)
    exp = orc.projection_prove(x, w, b, out, rem, m, k, n, 4, orng)
    got = prove_projection(x, w, b, out, rem, m, k, n, 4, zrng)
    assert_same(got, exp)
    d = to_oracle_dict(got, exp)
    assert orc.projection_verify(d, 4)
    d["frac_finals"][0, 3] = (int(d["frac_finals"][0, 3]) + 1) % P
    assert not orc.projection_verify(d, 4)


@pytest.mark.parametrize("m,k,n,shift", [(4, 16, 8, 8), (16, 64, 32, 12), (64, 256, 128, 16), (32, 1024, 64, 16)])
def test_fixed_point_shapes_match_oracle(zk, orc, m, k, n, shift):
    """16-bit fixed-point inputs (the tensor-core forward where the shape
    allows), bias within 2^20, the witness from the device kernel, challenges
    from a shard's child transcript."""
    from zkie_b200.projection import projection_witness, prove_projection
    x, w = fixed(m + k, m * k), fixed(k + n, k * n)
    b = fixed(m + n, m * n, -(1 << 20), 1 << 20)
    h, _ = zk.matmul_fixed(x, w, m, k, n, force_tensor=True)
    out, rem, idx = projection_witness(h, b, shift)
    ids = [[7, 8, 9]]
    got = prove_projection(x, w, b, out, rem, m, k, n, shift, zk.shard_dag_child(ids, 1, 0), h=h)
    exp = orc.projection_prove(x, w, b, out.cpu().numpy(), rem.cpu().numpy(), m, k, n, shift,
                               orc.shard_dag_child(ids, 1, 0))
    assert np.array_equal(h.cpu().numpy(), exp["h"])
    assert_same(got, exp)
    assert orc.projection_verify(to_oracle_dict(got, exp), shift)


@pytest.mark.slow
def test_gpt2_projection_shape(zk, orc):
    """A GPT-2 layer's FFN up-projection shape (512 x 1024 @ 1024 x 4096,
    scale 2^16): the device proof verifies with the oracle's verifier (the
    oracle's own prover at this size would take minutes), the matmul claim
    equals the oracle's evaluation of h at (v || u), and the challenges are
    the generator's draws in the reference's order."""
    from zkie_b200.projection import projection_witness, prove_projection
    m, k, n, shift = 512, 1024, 4096, 16
    x, w = fixed(1, m * k), fixed(2, k * n)
    b = fixed(3, m * n, -(1 << 20), 1 << 20)
    h, path = zk.matmul_fixed(x, w, m, k, n)
    assert path == 0
    out, rem, idx = projection_witness(h, b, shift)
    got = prove_projection(x, w, b, out, rem, m, k, n, shift, zk.XorShift64(5), h=h)
    assert got.matmul.claimed == orc.mle_eval(h.cpu().numpy(), got.pt)
    orng = orc.XorShift64(5)
    lg = (m * n + (1 << shift) - 1).bit_length()
    draws = [orng.field() for _ in range(9 + 12 + 10 + 2 + 2 * lg)]  # u, v, ch, alpha, beta, full_r, cs
    assert np.array_equal(got.u, np.array(draws[:9], dtype=np.uint64))
    assert np.array_equal(got.ch, np.array(draws[21:31], dtype=np.uint64))
    assert (got.alpha, got.beta) == (draws[31], draws[32])
    exp_cs = np.array(draws[-lg:], dtype=np.uint64)
    assert np.array_equal(got.frac.full_r, np.array(draws[-2 * lg:-lg], dtype=np.uint64))
    assert orc.projection_verify(to_oracle_dict(got, {"cs": exp_cs}), shift)
