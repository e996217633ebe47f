"""GPU parity of the shard-commit path (NTT + Poseidon2 Merkle) against the
CPU oracle, bit-exact, through the C ABI.  Small cases compare whole outputs;
BASELINE-sized cases use size-independent checks (sampled rows against Horner
evaluation, sampled leaf digests, the tree rebuilt by the oracle from the GPU
leaves)."""
import numpy as np
import pytest
import torch

P = 0xFFFFFFFF00000001
pytestmark = pytest.mark.gpu


def rand_mat(orc, seed, h, w):
    rng = orc.XorShift64(seed)
    return np.array([rng.field() for _ in range(h * w)], dtype=np.uint64).reshape(h, w)


def rand_mat_fast(seed, h, w):
    """Uniform [0, p) values from numpy (large cases; rejection of >= p)."""
    g = np.random.default_rng(seed)
    m = g.integers(0, 2 ** 64, size=(h, w), dtype=np.uint64)
    bad = m >= np.uint64(P)
    while bad.any():
        m[bad] = g.integers(0, 2 ** 64, size=int(bad.sum()), dtype=np.uint64)
        bad = m >= np.uint64(P)
    return m


# ---- reference entry point: zkie_ntt_forward_goldilocks ------------------------------
@pytest.mark.parametrize("lg,w", [(1, 1), (2, 3), (3, 32), (5, 1), (8, 7), (10, 32), (11, 1), (12, 5),
                                  (14, 32), (16, 3), (17, 64), (20, 2), (21, 1), (22, 1)])
def test_reference_ntt_matches_oracle(zk, orc, lg, w):
    m = rand_mat(orc, 1000 + lg * 7 + w, 1 << lg, w) if (w << lg) <= (1 << 16) else rand_mat_fast(lg * 31 + w, 1 << lg, w)
    got = zk.CudaDft().dft_batch(m)
    assert np.array_equal(got, orc.dft_batch(m))


def test_reference_ntt_noop_and_noncanonical(zk, orc):
    lib = zk.lib
    m = torch.tensor([5, 7], dtype=torch.uint64, device="cuda")
    tw = torch.tensor([1], dtype=torch.uint64, device="cuda")
    assert lib.zkie_ntt_forward_goldilocks(m.data_ptr(), m.data_ptr(), 0, 2, tw.data_ptr()) == 0
    assert lib.zkie_ntt_forward_goldilocks(m.data_ptr(), m.data_ptr(), 3, 0, tw.data_ptr()) == 0
    torch.cuda.synchronize()
    assert m.cpu().tolist() == [5, 7]
    raw = np.array([[2 ** 64 - 1, P], [P + 3, 2 ** 63], [1, 2], [P - 1, 0]], dtype=np.uint64)
    got = zk.CudaDft().dft_batch(raw)
    assert np.array_equal(got, orc.dft_batch(raw))
    assert (got < np.uint64(P)).all()
    assert lib.zkie_ntt_forward_goldilocks(0, 0, 4, 1, 0) != 0  # null pointers are rejected


# ---- zkie2_lde ---------------------------------------------------------------------------
@pytest.mark.parametrize("lg_l,lb,w", [(0, 1, 4), (1, 1, 1), (4, 1, 3), (5, 2, 8), (9, 1, 32), (10, 1, 1),
                                       (10, 2, 16), (11, 3, 2), (14, 1, 32), (15, 4, 1), (19, 2, 3)])
def test_lde_matches_oracle(zk, orc, lg_l, lb, w):
    m = rand_mat_fast(lg_l * 13 + lb * 5 + w, 1 << lg_l, w)
    com = zk.commit(m, lb)
    assert np.array_equal(com.lde.cpu().numpy(), orc.lde(m, lb))


# ---- Poseidon2 ---------------------------------------------------------------------------------
def test_permutation_matches_oracle(zk, orc, consts):
    zk.init_default_constants()
    rng = np.random.default_rng(5)
    st = rng.integers(0, 2 ** 64, size=(300, 16), dtype=np.uint64)
    st[0] = np.arange(16, dtype=np.uint64)
    st[1] = np.uint64(2 ** 64 - 1)  # non-canonical lanes
    d = torch.from_numpy(st.copy()).cuda()
    zk.check(zk.lib.zkie2_p2_permute(d.data_ptr(), 300, 2, 0), "permute")
    got = d.cpu().numpy()
    for i in range(300):
        exp = orc.p2_permute(consts, orc.p2_permute(consts, st[i]))
        assert np.array_equal(got[i], exp), i


@pytest.mark.parametrize("w", [0, 1, 3, 7, 8, 9, 15, 16, 32, 33, 64, 256])
def test_leaf_digests_match_oracle(zk, orc, consts, w):
    zk.init_default_constants()
    h = 77
    m = rand_mat_fast(w + 1, h, w) if w else np.zeros((h, 0), dtype=np.uint64)
    d_m = torch.from_numpy(m.copy()).cuda() if w else torch.zeros(1, dtype=torch.uint64, device="cuda")
    d_dig = torch.zeros(h * 8, dtype=torch.uint64, device="cuda")
    zk.check(zk.lib.zkie2_merkle_leaves(d_m.data_ptr(), h, w, d_dig.data_ptr(), 0), "leaves")
    got = d_dig.cpu().numpy().reshape(h, 8)
    exp = np.stack([orc.p2_hash_row(consts, m[r]) for r in range(h)])
    assert np.array_equal(got, exp)


@pytest.mark.parametrize("h,w", [(1, 4), (2, 8), (3, 5), (5, 32), (8, 1), (9, 9), (16, 32), (17, 8),
                                 (100, 3), (1000, 2), (1024, 32)])
def test_merkle_tree_matches_oracle(zk, orc, consts, h, w):
    m = rand_mat_fast(h * 3 + w, h, w)
    exp_layers, exp_root = orc.merkle_tree(consts, m)
    mmcs = zk.CudaMerkleTreeMmcs()
    ref_seq = mmcs.commit_reference_sequence(m)   # the reference entry points, commit_gpu order
    fused = mmcs.commit(m)                        # zkie2_merkle_tree
    for tree in (ref_seq, fused):
        assert np.array_equal(tree.root, exp_root)
        assert len(tree.layers) == len(exp_layers)
        for a, b in zip(tree.layers, exp_layers):
            assert np.array_equal(a, b)


def test_custom_constants_roundtrip(zk, orc):
    # upload seed-2 constants through the reference entry point, hash, restore seed 1
    c2 = orc.p2_constants(2)
    ei, ef, it, d15 = c2.as_arrays()
    zk.upload_constants(ei, ef, it, d15)
    m = rand_mat_fast(4, 9, 10)
    try:
        assert np.array_equal(zk.CudaMerkleTreeMmcs.__new__(zk.CudaMerkleTreeMmcs).commit(m).root,
                              orc.merkle_tree(c2, m)[1])
    finally:
        zk.upload_constants(*zk.p2_default_constants(1))


# ---- commit (LDE + Merkle), WHIR geometry, host path -------------------------------------
@pytest.mark.parametrize("lg_l,lb,w", [(4, 1, 1), (6, 2, 16), (8, 1, 256), (10, 1, 32), (12, 2, 16),
                                       (13, 1, 1)])
def test_commit_matches_oracle(zk, orc, consts, lg_l, lb, w):
    m = rand_mat_fast(lg_l * 100 + lb * 10 + w, 1 << lg_l, w)
    com = zk.commit(m, lb)
    exp_lde = orc.lde(m, lb)
    exp_layers, exp_root = orc.merkle_tree(consts, exp_lde)
    assert np.array_equal(com.lde.cpu().numpy(), exp_lde)
    assert np.array_equal(com.root, exp_root)
    got_layers = com.layer_list()
    assert all(np.array_equal(a, b) for a, b in zip(got_layers, exp_layers))


def test_commit_host_matches_device(zk, orc, consts):
    m = rand_mat_fast(17, 1 << 9, 16)
    root, lde, layers = zk.commit_host(m, 1)
    exp_lde = orc.lde(m, 1)
    _, exp_root = orc.merkle_tree(consts, exp_lde)
    assert np.array_equal(lde, exp_lde) and np.array_equal(root, exp_root)
    assert np.array_equal(layers[-1], exp_root)
    root2, lde2, layers2 = zk.commit_host(m, 1, want_lde=False, want_layers=False)
    assert np.array_equal(root2, exp_root) and lde2 is None and layers2 is None


@pytest.mark.parametrize("n", [5, 6, 10, 14, 16])
def test_whir_commit_matches_oracle(zk, orc, consts, n):
    rng = orc.XorShift64(n)
    evals = np.array([rng.field() for _ in range(1 << n)], dtype=np.uint64) if n <= 10 else \
        rand_mat_fast(n, 1 << n, 1).reshape(-1)
    com = zk.Whir.with_params(n, 90, 17).commit(evals)
    lde, root = orc.whir_commit(consts, evals)
    assert np.array_equal(com.lde.cpu().numpy(), lde)
    assert np.array_equal(com.root, root)


def test_whir_commit_batch_stacks_tables(zk, orc, consts):
    rng = orc.XorShift64(3)
    tabs = [np.array([rng.field() for _ in range(1 << 7)], dtype=np.uint64) for _ in range(3)]
    com, bw = zk.Whir.with_params(7, 90, 17).commit_batch(tabs)
    assert bw.num_variables == 9  # ceil(log2(3 * 2^7))
    stacked = np.zeros(1 << 9, dtype=np.uint64)
    stacked[:3 << 7] = np.concatenate(tabs)
    assert np.array_equal(com.root, orc.whir_commit(consts, stacked)[1])


# ---- BASELINE-sized cases: size-independent checks ------------------------------------------------
@pytest.mark.slow
@pytest.mark.parametrize("lg_l,lb,w", [(16, 1, 256), (20, 1, 16), (16, 2, 16), (20, 2, 1), (24, 1, 1),
                                        (20, 1, 256), (20, 2, 256), (24, 2, 16)])
def test_commit_sweep_sampled(zk, orc, consts, lg_l, lb, w):
    """Raw commit sweep shapes (the benched 256 x 2^20 at
    blowup 2 and the blowup-4 cases included): sampled LDE rows against
    Horner evaluation, sampled leaves against the oracle sponge, and the
    whole tree above the leaves rebuilt by the oracle from the GPU leaves."""
    m = rand_mat_fast(lg_l * 7 + lb + w, 1 << lg_l, w)
    com = zk.commit(m, lb)
    H = 1 << (lg_l + lb)
    rows = [0, 1, 2, H // 2 + 1, H - 1] + [int(x) for x in np.random.default_rng(1).integers(0, H, 3)]
    lde_rows = com.lde.view(torch.int64)[torch.tensor(rows, device="cuda")].cpu().numpy().view(np.uint64)
    cols = list(range(w)) if w <= 16 else [0, 1, w // 2, w - 1]
    exp = orc.lde_rows(m[:, cols].copy(), rows, H)
    assert np.array_equal(lde_rows[:, cols], exp)
    layers = com.layer_list()
    for a, r in enumerate(rows):
        assert np.array_equal(layers[0][r], orc.p2_hash_row(consts, lde_rows[a]))
    # every layer: sampled nodes are the compression of their two children
    g = np.random.default_rng(2)
    for lvl in range(1, len(layers)):
        raw = len(layers[lvl - 1]) // 2
        for i in set([0, raw - 1] + [int(x) for x in g.integers(0, raw, 6)]):
            exp_node = orc.p2_compress(consts, layers[lvl - 1][2 * i], layers[lvl - 1][2 * i + 1])
            assert np.array_equal(layers[lvl][i], exp_node), (lvl, i)
    assert np.array_equal(layers[-1][0], com.root)
    # determinism: a second run is bit-identical (integer math, any race would show)
    com2 = zk.commit(m, lb)
    assert np.array_equal(com2.root, com.root)


@pytest.mark.parametrize("lg_l,lb,w,lg_c", [(3, 1, 5, 0), (3, 1, 5, 1), (6, 1, 16, 2), (6, 2, 16, 3), (9, 1, 32, 3),
                                             (10, 2, 9, 1), (12, 1, 256, 2), (13, 1, 3, 4), (15, 3, 2, 5)])
def test_commit_cosets_matches_commit(zk, orc, consts, lg_l, lb, w, lg_c):
    """zkie2_commit_cosets (the LDE one coset of rows at a time, 2^lg_c cosets
    below, at and above the blowup, i.e. with and without folded inputs):
    every digest layer equal to zkie2_commit's, the root to the oracle's."""
    m = rand_mat_fast(lg_l * 41 + lb * 3 + w + lg_c, 1 << lg_l, w)
    root, layers = zk.commit_cosets(m, lb, lg_c)
    com = zk.commit(m, lb)
    assert np.array_equal(layers.cpu().numpy(), com.layers.cpu().numpy())
    assert np.array_equal(root, com.root)
    if (w << (lg_l + lb)) <= (1 << 16):
        assert np.array_equal(root, orc.merkle_tree(consts, orc.lde(m, lb))[1])


@pytest.mark.parametrize("lg", [4, 5, 6, 7, 8, 9, 10, 13])
@pytest.mark.parametrize("w", [1, 5, 64, 600])
def test_dft_every_radix_schedule(zk, orc, lg, w):
    """zkie2_dft at every single-pass size (radix-16 register steps with a
    2..16 remainder step) and a two-pass size, partially reduced inputs,
    widths below, at and above a tile's column count."""
    if (w << lg) > (1 << 21):
        pytest.skip("covered by smaller widths")
    m = rand_mat_fast(lg * 100 + w, 1 << lg, w)
    raw = m.copy()
    raw[::3] = np.where(raw[::3] < np.uint64(0xFFFFFFFF), raw[::3] + np.uint64(P), raw[::3])
    d_in = torch.from_numpy(raw.reshape(-1)).cuda()
    d_out = torch.empty_like(d_in)
    scr = torch.empty(max(zk.lib.zkie2_lde_scratch_elems(lg, 0, w), 1), dtype=torch.uint64, device="cuda")
    zk.check(zk.lib.zkie2_dft(d_in.data_ptr(), d_out.data_ptr(), scr.data_ptr(), lg, w,
                              torch.cuda.current_stream().cuda_stream), "dft")
    assert np.array_equal(d_out.cpu().numpy().reshape(1 << lg, w), orc.dft_batch(m))


@pytest.mark.parametrize("lg_l,lb,w", [(1, 1, 100), (3, 1, 72), (9, 1, 64), (12, 1, 100), (14, 2, 256), (11, 1, 65)])
def test_commit_host_column_pipeline(zk, orc, consts, lg_l, lb, w):
    """zkie2_commit_host uploads, transforms and downloads the matrix in
    column blocks (pitched copies, the LDE on a column block of the full-width
    matrix): every block boundary and a ragged last block against the oracle."""
    m = rand_mat_fast(lg_l * 7 + w, 1 << lg_l, w)
    root, lde, layers = zk.commit_host(m, lb)
    exp_lde = orc.lde(m, lb)
    assert np.array_equal(lde, exp_lde)
    _, exp_root = orc.merkle_tree(consts, exp_lde)
    assert np.array_equal(root, exp_root)
