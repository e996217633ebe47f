"""This library against the reference's OWN CUDA kernels, on the GPU.

oracle/build_ref.py compiles the reference's crates/zkie-core/cuda/
goldilocks_ntt.cu and poseidon2_merkle.cu, unmodified, into
oracle/_ref/libzkie_ref.so (the three sppark names they include come from a
stand-in under oracle/ref_shim/).  Both libraries export the seven C symbols
of crates/zkie-core/src/pcs/cuda_ffi.rs:2-46.  Every test feeds both the same
inputs, the same round constants and the same twiddle tables and compares
every output bit for bit:

- the DFT of zkie_ntt_forward_goldilocks (and, on zero-padded inputs, the LDE
  of zkie2_commit / zkie2_whir_commit);
- leaf digests (full 8-row batches and the scalar tail, widths that are and
  are not multiples of the sponge rate, non-canonical inputs);
- compression at step 1 and step 2, batch and scalar;
- whole trees driven by the reference call sequence of commit_gpu
  (pcs/merkle_cuda.rs:227-285) on the reference kernels, against this
  library's fused tree and commit.

What this pins: the DFT, permutation, sponge, compression and tree semantics
of the reference's own device code.  What stays an assumption on both sides:
the round-constant values (SmallRng restatement), diag15 = 2^-32, and the
Rust caller logic restated in commit_reference_sequence.
"""
import ctypes as C
import os

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref", "libzkie_ref.so")
P = 0xFFFFFFFF00000001
pytestmark = pytest.mark.gpu

_vp, _u32, _u64 = C.c_void_p, C.c_uint32, C.c_uint64
_pu64 = C.POINTER(C.c_uint64)
_SIGS = {
    "zkie_cuda_device_count": [],
    "zkie_ntt_forward_goldilocks": [_vp, _vp, _u32, _u64, _vp],
    "zkie_p2_upload_constants": [_pu64, _pu64, _pu64, _u64],
    "zkie_p2_leaf_batch": [_vp, _vp, _u32, _u32],
    "zkie_p2_leaf_scalar": [_vp, _vp, _u32, _u32, _u32],
    "zkie_p2_compress_batch": [_vp, _vp, _u32, _u32],
    "zkie_p2_compress_scalar": [_vp, _vp, _u32, _u32, _u32],
}


def _np_ptr(a):
    return a.ctypes.data_as(_pu64)


def _upload(lib, consts):
    ri, rf, rp, d15 = consts
    arrs = [np.ascontiguousarray(np.asarray(x, dtype=np.uint64).reshape(-1)) for x in (ri, rf, rp)]
    assert lib.zkie_p2_upload_constants(*[_np_ptr(a) for a in arrs], int(d15)) == 0


@pytest.fixture(scope="module")
def ref(zk):
    if not os.path.exists(REF):
        pytest.skip("oracle/_ref/libzkie_ref.so was not built (no reference checkout when the tree was built)")
    lib = C.CDLL(REF)
    for name, args in _SIGS.items():
        f = getattr(lib, name)
        f.restype = C.c_int
        f.argtypes = args
    _upload(lib, zk.p2_default_constants(1))
    zk.init_default_constants()
    return lib


def rand_mat(seed, h, w, noncanonical=False):
    g = np.random.default_rng(seed)
    m = g.integers(0, 2 ** 64, size=(h, w), dtype=np.uint64)
    if not noncanonical:
        m = np.where(m >= np.uint64(P), m - np.uint64(P), m)
    return m


def ref_dft(ref, zk, m):
    """zkie_ntt_forward_goldilocks of the reference on an h x w matrix."""
    h, w = m.shape
    lg = h.bit_length() - 1
    d = torch.from_numpy(np.ascontiguousarray(m).reshape(-1)).cuda()
    tmp = torch.empty_like(d)
    tw = torch.from_numpy(zk.make_twiddles(lg)).cuda()
    torch.cuda.synchronize()
    assert ref.zkie_ntt_forward_goldilocks(d.data_ptr(), tmp.data_ptr(), lg, w, tw.data_ptr()) == 0
    torch.cuda.synchronize()
    return d.cpu().numpy().reshape(h, w)


def test_ref_library_loads_and_counts_devices(zk, ref):
    assert ref.zkie_cuda_device_count() == torch.cuda.device_count() == zk.lib.zkie_cuda_device_count()


@pytest.mark.parametrize("lg,w", [(1, 1), (2, 3), (4, 8), (5, 1), (8, 7), (10, 32), (11, 5), (13, 2),
                                  (14, 32), (16, 3), (18, 8), (20, 1)])
def test_dft_matches_reference_kernel(zk, ref, lg, w):
    m = rand_mat(lg * 17 + w, 1 << lg, w, noncanonical=(lg % 2 == 0))
    got = zk.CudaDft().dft_batch(m)
    exp = ref_dft(ref, zk, m)
    assert np.array_equal(got, exp)
    assert (got < np.uint64(P)).all()


@pytest.mark.parametrize("lg_l,lb,w", [(0, 1, 4), (3, 1, 9), (6, 2, 16), (9, 1, 32), (10, 3, 5), (12, 1, 64),
                                       (14, 1, 32), (15, 2, 8), (17, 1, 3)])
def test_lde_and_commit_match_reference_kernels(zk, ref, lg_l, lb, w):
    """zkie2_commit (LDE + fused tree) against the reference: its DFT of the
    zero-padded coefficients, then its leaf and compression kernels in the
    commit_gpu call sequence."""
    m = rand_mat(lg_l * 31 + lb * 7 + w, 1 << lg_l, w)
    padded = np.zeros((m.shape[0] << lb, w), dtype=np.uint64)
    padded[:m.shape[0]] = m
    exp_lde = ref_dft(ref, zk, padded)
    com = zk.commit(m, lb)
    assert np.array_equal(com.lde.cpu().numpy(), exp_lde)
    tree = zk.CudaMerkleTreeMmcs().commit_reference_sequence(exp_lde, ffi=ref)
    got_layers = com.layer_list()
    assert len(got_layers) == len(tree.layers)
    for a, b in zip(got_layers, tree.layers):
        assert np.array_equal(a, b)
    assert np.array_equal(com.root, tree.root)


@pytest.mark.parametrize("n", [5, 9, 14, 20])
def test_whir_commit_matches_reference_kernels(zk, ref, n):
    """WHIR base commit geometry (2^(n-5) x 32, blowup 2) with configuration
    1's shapes: A and C at n = 14, W at n = 20."""
    evals = rand_mat(n, 1 << n, 1).reshape(-1)
    com = zk.Whir.with_params(n, 90, 17).commit(evals)
    padded = np.zeros((1 << (n - 4), 32), dtype=np.uint64)
    padded[:1 << (n - 5)] = evals.reshape(-1, 32)
    exp_lde = ref_dft(ref, zk, padded)
    assert np.array_equal(com.lde.cpu().numpy(), exp_lde)
    tree = zk.CudaMerkleTreeMmcs().commit_reference_sequence(exp_lde, ffi=ref)
    assert np.array_equal(com.root, tree.root)


@pytest.mark.parametrize("h", [1, 7, 8, 77, 1024])
@pytest.mark.parametrize("w", [1, 3, 7, 8, 9, 16, 33, 64, 256])
def test_leaf_digests_match_reference_kernel(zk, ref, h, w):
    m = rand_mat(h * 1000 + w, h, w, noncanonical=(w % 2 == 1))
    d_m = torch.from_numpy(m.reshape(-1).copy()).cuda()
    outs = []
    for lib in (ref, zk.lib):
        d = torch.zeros(h * 8, dtype=torch.uint64, device="cuda")
        torch.cuda.synchronize()
        assert lib.zkie_p2_leaf_batch(d_m.data_ptr(), d.data_ptr(), h, w) == 0
        assert lib.zkie_p2_leaf_scalar(d_m.data_ptr(), d.data_ptr(), h // 8 * 8, h, w) == 0
        torch.cuda.synchronize()
        outs.append(d.cpu().numpy())
    assert np.array_equal(outs[0], outs[1])
    assert (outs[1] < np.uint64(P)).all()


@pytest.mark.parametrize("step", [1, 2])
@pytest.mark.parametrize("next_len", [1, 5, 8, 13, 64, 1000])
def test_compression_matches_reference_kernel(zk, ref, step, next_len):
    prev = rand_mat(next_len * 3 + step, step * next_len, 8).reshape(-1)
    d_prev = torch.from_numpy(prev).cuda()
    outs = []
    for lib in (ref, zk.lib):
        d = torch.zeros(next_len * 8, dtype=torch.uint64, device="cuda")
        torch.cuda.synchronize()
        assert lib.zkie_p2_compress_batch(d_prev.data_ptr(), d.data_ptr(), next_len, step) == 0
        assert lib.zkie_p2_compress_scalar(d_prev.data_ptr(), d.data_ptr(), next_len // 8 * 8, next_len, step) == 0
        torch.cuda.synchronize()
        outs.append(d.cpu().numpy())
    assert np.array_equal(outs[0], outs[1])


@pytest.mark.parametrize("h,w", [(1, 4), (2, 8), (3, 5), (9, 9), (17, 8), (100, 3), (1000, 2), (1024, 32),
                                 (4097, 16)])
def test_tree_matches_reference_kernels(zk, ref, h, w):
    m = rand_mat(h * 7 + w, h, w)
    mmcs = zk.CudaMerkleTreeMmcs()
    exp = mmcs.commit_reference_sequence(m, ffi=ref)
    for tree in (mmcs.commit_reference_sequence(m), mmcs.commit(m)):
        assert len(tree.layers) == len(exp.layers)
        for a, b in zip(tree.layers, exp.layers):
            assert np.array_equal(a, b)
        assert np.array_equal(tree.root, exp.root)


def test_custom_constants_match_reference_kernel(zk, ref):
    """Another constant set uploaded through zkie_p2_upload_constants on both
    sides (the upload path itself, and no constant baked into either kernel)."""
    c2 = zk.p2_default_constants(2)
    _upload(ref, c2)
    zk.upload_constants(*c2)
    try:
        m = rand_mat(5, 40, 12)
        exp = zk.CudaMerkleTreeMmcs.__new__(zk.CudaMerkleTreeMmcs).commit_reference_sequence(m, ffi=ref)
        got = zk.CudaMerkleTreeMmcs.__new__(zk.CudaMerkleTreeMmcs).commit(m)
        assert np.array_equal(got.root, exp.root)
    finally:
        _upload(ref, zk.p2_default_constants(1))
        zk.upload_constants(*zk.p2_default_constants(1))
