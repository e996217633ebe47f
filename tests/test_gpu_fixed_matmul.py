"""GPU parity of the fixed-point forward matmul on the tensor cores
(zkie2_matmul_fixed, par::mm_par_fixed of zkie-ops/src/par.rs:41-89) with the
exact field matmul (zkie2_matmul_field) and, on small shapes, the CPU oracle:
bit-exact, across tile edges, K split into chunks, the extreme 16- and
24-bit values (two or three byte planes per operand), and the field
fallback for values outside 24 bits."""
import numpy as np
import pytest

P = 0xFFFFFFFF00000001
pytestmark = pytest.mark.gpu


def fixed(seed, shape, lo=-(1 << 15), hi=1 << 15):
    """Signed fixed-point values embedded in the field (x < 0 -> p - |x|, fixed_point.rs:53-59)."""
    x = np.random.default_rng(seed).integers(lo, hi, size=shape, dtype=np.int64)
    return x.astype(np.uint64) + np.where(x < 0, np.uint64(P), np.uint64(0))


@pytest.mark.parametrize("m,k,n", [(16, 1024, 1024), (128, 256, 512), (512, 1024, 4096), (1, 32, 4),
                                   (100, 48, 20), (130, 160, 260), (8, 16384, 64), (3, 8208, 12)])
def test_tensor_path_matches_field(zk, m, k, n):
    a, b = fixed(m * 7 + k, (m, k)), fixed(n * 11 + k, (k, n))
    got, path = zk.matmul_fixed(a, b, m, k, n, force_tensor=True)
    assert path == 0
    ref = zk.matmul_field(a, b, m, k, n)
    assert np.array_equal(got.cpu().numpy(), ref.cpu().numpy())


def test_matches_oracle_and_extremes(zk, orc):
    m, k, n = 5, 64, 8
    a, b = fixed(1, (m, k)), fixed(2, (k, n))
    got, path = zk.matmul_fixed(a, b, m, k, n, force_tensor=True)
    assert path == 0 and np.array_equal(got.cpu().numpy().reshape(m, n), orc.matmul_field(a, b))
    # every product at the largest magnitudes: sums of +-2^30 over k = 4096
    for va, vb in ((-(1 << 15), -(1 << 15)), ((1 << 15) - 1, -(1 << 15)), ((1 << 15) - 1, (1 << 15) - 1)):
        m, k, n = 64, 4096, 64
        a = fixed(0, (m, k), va, va + 1)
        b = fixed(0, (k, n), vb, vb + 1)
        got, path = zk.matmul_fixed(a, b, m, k, n, force_tensor=True)
        assert path == 0
        assert np.array_equal(got.cpu().numpy(), zk.matmul_field(a, b, m, k, n).cpu().numpy())


@pytest.mark.parametrize("bits_a,bits_b", [(24, 16), (16, 24), (24, 24), (17, 17)])
@pytest.mark.parametrize("m,k,n", [(48, 2048, 2048), (130, 160, 260), (3, 8208, 12), (8, 16384, 64)])
def test_three_plane_operands_match_field(zk, bits_a, bits_b, m, k, n):
    """Operands beyond 16 bits take three byte planes (five plane-sum GEMMs
    for 3 x 3): the exact field product."""
    a = fixed(m + k + bits_a, (m, k), -(1 << (bits_a - 1)), 1 << (bits_a - 1))
    b = fixed(n + k + bits_b, (k, n), -(1 << (bits_b - 1)), 1 << (bits_b - 1))
    got, path = zk.matmul_fixed(a, b, m, k, n, force_tensor=True)
    assert path == 0
    assert np.array_equal(got.cpu().numpy(), zk.matmul_field(a, b, m, k, n).cpu().numpy())


def test_three_plane_extremes(zk):
    """Every product at the 24-bit extremes: sums of +-2^46 over k = 4096."""
    m, k, n = 64, 4096, 64
    for va, vb in ((-(1 << 23), -(1 << 23)), ((1 << 23) - 1, -(1 << 23)), ((1 << 23) - 1, (1 << 23) - 1),
                   (-(1 << 23), (1 << 15) - 1)):
        a = fixed(0, (m, k), va, va + 1)
        b = fixed(0, (k, n), vb, vb + 1)
        got, path = zk.matmul_fixed(a, b, m, k, n, force_tensor=True)
        assert path == 0
        assert np.array_equal(got.cpu().numpy(), zk.matmul_field(a, b, m, k, n).cpu().numpy())


@pytest.mark.parametrize("odd", [1 << 15, P - (1 << 15) - 1, (1 << 23) - 1, P - (1 << 23)])
def test_values_past_16_bits_stay_on_the_tensor_path(zk, odd):
    m, k, n = 32, 256, 64
    a, b = fixed(3, (m, k)), fixed(4, (k, n))
    a[7, 9] = np.uint64(odd)
    got, path = zk.matmul_fixed(a, b, m, k, n, force_tensor=True)
    assert path == 0
    assert np.array_equal(got.cpu().numpy(), zk.matmul_field(a, b, m, k, n).cpu().numpy())


@pytest.mark.parametrize("bad", [1 << 23, P - (1 << 23) - 1, 12345678901234])
def test_out_of_range_falls_back_to_field(zk, bad):
    m, k, n = 32, 256, 64
    a, b = fixed(3, (m, k)), fixed(4, (k, n))
    a[7, 9] = np.uint64(bad)
    got, path = zk.matmul_fixed(a, b, m, k, n, force_tensor=True)
    assert path == 1
    assert np.array_equal(got.cpu().numpy(), zk.matmul_field(a, b, m, k, n).cpu().numpy())


def test_unaligned_shapes_use_field(zk):
    m, k, n = 9, 40, 6  # k % 16, n % 4
    a, b = fixed(5, (m, k)), fixed(6, (k, n))
    got, path = zk.matmul_fixed(a, b, m, k, n, force_tensor=True)
    assert path == 1
    assert np.array_equal(got.cpu().numpy(), zk.matmul_field(a, b, m, k, n).cpu().numpy())


def test_auto_policy_keeps_small_products_on_the_field_kernel(zk):
    a, b = fixed(8, (16, 1024)), fixed(9, (1024, 1024))
    got, path = zk.matmul_fixed(a, b, 16, 1024, 1024)
    assert path == 1  # 2^24 multiply-adds: the field kernel is faster
    assert np.array_equal(got.cpu().numpy(), zk.matmul_field(a, b, 16, 1024, 1024).cpu().numpy())
    a, b = fixed(10, (512, 1024)), fixed(11, (1024, 256))
    got, path = zk.matmul_fixed(a, b, 512, 1024, 256)
    assert path == 0  # 2^27
    assert np.array_equal(got.cpu().numpy(), zk.matmul_field(a, b, 512, 1024, 256).cpu().numpy())


def test_unaligned_a_pointer_uses_field(zk):
    """A that is not 16-byte aligned (the tensor path loads A 16 bytes at a time)."""
    import ctypes as C

    import torch
    m, k, n = 128, 256, 1024
    a, b = fixed(12, (m, k)), fixed(13, (k, n))
    buf = torch.empty(m * k + 1, dtype=torch.uint64, device="cuda")
    buf[1:] = torch.from_numpy(a.reshape(-1)).cuda()
    da = buf[1:]  # 8-byte offset
    db = torch.from_numpy(b.reshape(-1)).cuda()
    dc = torch.empty(m * n, dtype=torch.uint64, device="cuda")
    scr = torch.empty(zk.lib.zkie2_matmul_fixed_scratch_elems(m, k, n), dtype=torch.uint64, device="cuda")
    path = C.c_uint32(9)
    zk.check(zk.lib.zkie2_matmul_fixed(da.data_ptr(), db.data_ptr(), m, k, n, dc.data_ptr(), 1, C.byref(path),
                                       scr.data_ptr(), torch.cuda.current_stream().cuda_stream), "matmul_fixed")
    assert path.value == 1
    assert np.array_equal(dc.cpu().numpy(), zk.matmul_field(a, b, m, k, n).cpu().numpy())


def test_tall_field_matmul_runs_in_row_blocks(zk, orc):
    """More rows than one launch's grid.y (65535): the field kernel runs row
    blocks, as the reference's field matmul computes any shape."""
    m, k, n = 2 * 65535 + 3, 8, 4
    a, b = fixed(14, (m, k)), fixed(15, (k, n))
    got = zk.matmul_field(a, b, m, k, n).cpu().numpy().reshape(m, n)
    assert np.array_equal(got, orc.matmul_field(a, b))
    got, path = zk.matmul_fixed(a, b, m, k, n, force_tensor=True)
    assert path == 1  # k % 16 != 0: the field kernel
    assert np.array_equal(got.cpu().numpy().reshape(m, n), orc.matmul_field(a, b))


@pytest.mark.parametrize("bits", [16, 24, 30])
def test_runs_entry_matches_field(zk, bits):
    """zkie2_matmul_fixed_runs (the GatherMatMul forward): consecutive runs of
    rows, each times one block of a stack of expert matrices, short runs on
    the field kernel and long ones on the tensor path (or all on the field
    kernel for 30-bit operands): every row equal to its field product."""
    import torch

    from zkie_b200._lib import check, lib, pu64
    from zkie_b200.device import ptr, stream_handle, to_dev
    ne, k, n = 5, 2048, 512
    sizes = [300, 7, 1, 160, 40, 0, 200]
    experts = [3, 0, 4, 3, 1, 2, 0]
    runs, r0 = [], 0
    for e, nr in zip(experts, sizes):
        if nr:
            runs += [e, r0, nr]
            r0 += nr
    rows = r0
    a = fixed(bits, (rows, k), -(1 << (bits - 1)), 1 << (bits - 1))
    w = fixed(bits + 1, (ne, k, n), -(1 << 15), 1 << 15)
    da, dw = to_dev(a).reshape(-1), to_dev(w).reshape(-1)
    dc = torch.empty(rows * n, dtype=torch.uint64, device="cuda")
    h_runs = np.array(runs, dtype=np.uint64)
    scr = torch.empty(max(lib.zkie2_matmul_fixed_runs_scratch_elems(int(h_runs[2::3].max()), k, n), 1),
                      dtype=torch.uint64, device="cuda")
    check(lib.zkie2_matmul_fixed_runs(ptr(da), ptr(dw), ne, k, n, h_runs.ctypes.data_as(pu64), len(runs) // 3,
                                      ptr(dc), ptr(scr), stream_handle()), "zkie2_matmul_fixed_runs")
    got = dc.cpu().numpy().reshape(rows, n)
    for q in range(len(runs) // 3):
        e, r, nr = runs[3 * q:3 * q + 3]
        want = zk.matmul_field(a[r:r + nr], w[e], nr, k, n).cpu().numpy().reshape(nr, n)
        assert np.array_equal(got[r:r + nr], want), (e, r, nr)
