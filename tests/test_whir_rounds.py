"""WHIR round commits (commit_extension, vendor/p3-whir/src/pcs/committer/
writer.rs:21-86): the folding schedule against the reference's own test
vectors, the per-round geometry of Whir::with_params, the EF encoding against
extension-field arithmetic (CPU), and the device commit against the oracle
(GPU)."""
import numpy as np
import pytest

P = 0xFFFFFFFF00000001


def fields(seed, shape):
    g = np.random.default_rng(seed)
    v = g.integers(0, 2 ** 64, size=shape, dtype=np.uint64)
    return np.where(v >= np.uint64(P), v - np.uint64(P), v)


# folding.rs:252-276: FoldingFactor::Constant(3).compute_number_of_rounds(n)
@pytest.mark.parametrize("n,rounds,final", [(5, 0, 2), (6, 0, 3), (7, 0, 4), (9, 0, 6), (10, 1, 4), (13, 2, 4)])
def test_folding_schedule_reference_vectors(zk, n, rounds, final):
    sched = zk.Whir.folding_schedule(n, 3)
    assert (len(sched) - 1, n - sum(sched)) == (rounds, final)


def test_round_commit_geometry(zk):
    # Whir::with_params: folding 5, starting rate 1, rate += 4 per round
    assert zk.Whir(20, 90, 17).round_commits() == [(15, 5), (10, 9)]
    assert zk.Whir(14, 90, 17).round_commits() == [(9, 5)]
    assert zk.Whir(24, 90, 17).round_commits() == [(19, 5), (14, 9), (9, 13)]
    assert zk.Whir(11, 90, 17).round_commits() == []


@pytest.mark.parametrize("n,rate", [(6, 2), (5, 3)])
def test_extension_encoding_is_coefficientwise_dft(orc, consts, n, rate):
    ef = fields(n * 10 + rate, (1 << n, 2))
    enc, _ = orc.commit_extension(consts, ef, rate)
    rows = 1 << (n - 5)
    H = rows << rate
    mat = ef.reshape(rows, 32, 2)
    for c in (0, 7, 31):
        col = orc.ef_dft_naive(mat[:, c, :], H)
        assert np.array_equal(enc[:, 2 * c:2 * c + 2], col), c


@pytest.mark.gpu
@pytest.mark.parametrize("n,rate", [(5, 1), (10, 5), (12, 1), (10, 9), (15, 5)])
def test_commit_extension_matches_oracle(zk, orc, consts, n, rate):
    zk.check(zk.lib.zkie2_p2_init_default(), "constants")
    ef = fields(n + 100 * rate, (1 << n, 2))
    got = zk.Whir.commit_extension(ef, rate)
    enc, root = orc.commit_extension(consts, ef, rate)
    assert np.array_equal(np.asarray(got.root, dtype=np.uint64), root)
    assert np.array_equal(got.lde.cpu().numpy(), enc)
