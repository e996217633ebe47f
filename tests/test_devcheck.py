"""Device arithmetic self-check: the Goldilocks primitives and Poseidon2
stages of zkie_b200/csrc/*.cuh, compiled for the host (checked against the
oracle and Python big integers, CPU) and for sm_100a (checked against the
host build on identical inputs, GPU)."""
import ctypes as C
import random

import numpy as np
import pytest

from tests import build_devcheck

P = 0xFFFFFFFF00000001
M64 = 2 ** 64
SCALAR_OPS = {0: "add", 1: "add_c", 2: "sub", 3: "mul", 4: "sqr", 5: "div2", 6: "div8", 7: "div16",
              8: "div32", 9: "div2^32", 10: "canon", 11: "sbox", 12: "mul_hi", 13: "reduce128",
              14: "acc160_dot4", 15: "acc160_repeat", 16: "pow2_1", 17: "pow2_33", 18: "pow2_63", 19: "pow2_64",
              20: "pow2_95", 21: "pow2_96", 22: "pow2_120", 23: "pow2_156", 24: "pow2_191", 25: "pow2_39"}
POW2_K = {16: 1, 17: 33, 18: 63, 19: 64, 20: 95, 21: 96, 22: 120, 23: 156, 24: 191, 25: 39}
STATE_OPS = {105: "mat4", 100: "mds_light", 101: "ext_round0", 102: "internal_linear", 103: "int_round0",
             104: "permute", 110: "dft16", 111: "dft16_lazy", 112: "dft16_half", 113: "dft16_half_lazy",
             114: "dft8", 115: "dft8_lazy", 116: "dft4", 117: "dft4_lazy", 118: "dft2", 119: "dft2_lazy",
             120: "dft16_quarter_lazy", 121: "dft16_eighth_lazy", 122: "dft16_first_only_lazy"}
# state op -> (log2 radix, log2 of the zero fraction: inputs e >= 2^lg >> z of each group are zero)
DFT_OPS = {110: (4, 0), 111: (4, 0), 112: (4, 1), 113: (4, 1), 114: (3, 0), 115: (3, 0),
           116: (2, 0), 117: (2, 0), 118: (1, 0), 119: (1, 0), 120: (4, 2), 121: (4, 3), 122: (4, 4)}


@pytest.fixture(scope="module")
def dc():
    lib = C.CDLL(build_devcheck.build())
    p = C.POINTER(C.c_uint64)
    lib.hostcheck_scalar.argtypes = [C.c_int, p, p, p, C.c_uint64]
    lib.hostcheck_state.argtypes = [C.c_int, p, C.c_uint64, p]
    lib.devcheck_scalar.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_uint64]
    lib.devcheck_state.argtypes = [C.c_int, C.c_void_p, C.c_uint64, p]
    lib.devcheck_permute_x4.argtypes = [C.c_void_p, C.c_uint64, p]
    return lib


def _canon(a):
    return np.where(a >= np.uint64(P), a - np.uint64(P), a)


def _p(a):
    return a.ctypes.data_as(C.POINTER(C.c_uint64))


def inputs(n=4096, seed=1):
    rnd = random.Random(seed)
    edge = [0, 1, 2, P - 1, P, P + 1, M64 - 1, M64 - 2, 2 ** 32 - 1, 2 ** 32, 2 ** 63, M64 - 2 ** 32,
            M64 - 2 ** 32 + 1, 3]
    a = edge + [rnd.getrandbits(64) for _ in range(n - len(edge))]
    b = [rnd.getrandbits(64) for _ in range(n - len(edge))] + edge[::-1]
    return np.array(a, dtype=np.uint64), np.array(b, dtype=np.uint64)


def consts151(orc):
    ei, ef, it, d15 = orc.p2_constants(1).as_arrays()
    return np.concatenate([ei.ravel(), ef.ravel(), it, np.array([d15], dtype=np.uint64)]).astype(np.uint64)


def expected_scalar(op, a, b):
    inv2 = pow(2, P - 2, P)
    if op == 0: return (a + b) % P
    if op == 1: return (a + b % P) % P
    if op == 2: return (a - b) % P
    if op == 3: return a * b % P
    if op == 4: return a * a % P
    if op in (5, 6, 7, 8, 9): return a * pow(inv2, {5: 1, 6: 3, 7: 4, 8: 5, 9: 32}[op], P) % P
    if op == 10: return a % P
    if op == 11: return pow(a, 7, P)
    if op == 12: return (a * b) >> 64
    if op == 13: return (b * M64 + a) % P
    if op == 14: return (a * b + a * a + b * b + (a ^ b) * (M64 - 1 - a)) % P
    if op == 15: return ((b & 1023) + 1) * a * a % P
    if op in POW2_K: return a * pow(2, POW2_K[op], P) % P


def test_host_scalar_ops_match_bigint(dc):
    a, b = inputs(2048)
    for op in SCALAR_OPS:
        out = np.zeros_like(a)
        dc.hostcheck_scalar(op, _p(a), _p(b), _p(out), a.size)
        for x, y, z in zip(a.tolist(), b.tolist(), out.tolist()):
            if op in (10,):
                assert z == x % P
            elif op == 12:
                assert z == expected_scalar(op, x, y)
            else:
                assert z % P == expected_scalar(op, x, y), (SCALAR_OPS[op], hex(x), hex(y), hex(z))
                assert z < M64


def test_host_permutation_matches_oracle(dc, orc):
    c = consts151(orc)
    st = np.random.default_rng(3).integers(0, 2 ** 64, size=(64, 16), dtype=np.uint64)
    st[0] = np.arange(16, dtype=np.uint64)
    out = st.copy()
    dc.hostcheck_state(104, _p(out), 64, _p(c))
    cs = orc.p2_constants(1)
    for i in range(64):
        assert np.array_equal(np.array([x % P for x in out[i].tolist()], dtype=np.uint64), orc.p2_permute(cs, st[i]))


def _dft_expected(x, lg, z):
    """Natural-order DFT of each 2^lg group, W_(2^lg) = 2^(39 * 2^(6 - lg) mod 192),
    with the inputs e >= 2^lg >> z of each group taken as zero."""
    r = 1 << lg
    w = pow(2, (39 << (6 - lg)) % 192, P)
    out = []
    for g in range(0, 16, r):
        grp = [int(v) % P for v in x[g:g + r]]
        if z:
            grp = grp[:r >> z] + [0] * (r - (r >> z))
        out += [sum(grp[d] * pow(w, d * e, P) for d in range(r)) % P for e in range(r)]
    return out


def test_host_register_dfts_match_definition(dc, orc):
    """The NTT's in-register DFTs (plain and lazy-accumulator forms) against
    the DFT's definition, on inputs anywhere in [0, 2^64), with runs of values
    near 2^64 that stress the accumulator bounds."""
    c = consts151(orc)
    rng = np.random.default_rng(11)
    st = rng.integers(0, 2 ** 64, size=(64, 16), dtype=np.uint64)
    st[1] = np.uint64(M64 - 1)
    st[2] = np.uint64(P - 1)
    st[3, ::2] = np.uint64(M64 - 1)
    st[4] = np.uint64(P)
    for op, (lg, z) in DFT_OPS.items():
        out = st.copy()
        dc.hostcheck_state(op, _p(out), 64, _p(c))
        for i in range(64):
            got = [int(v) % P for v in out[i].tolist()]
            assert got == _dft_expected(st[i].tolist(), lg, z), (STATE_OPS[op], i)


@pytest.mark.gpu
def test_device_scalar_ops_match_host(dc):
    import torch
    a, b = inputs(1 << 14, seed=5)
    da, db = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    bad = []
    for op, name in SCALAR_OPS.items():
        dout = torch.zeros_like(da)
        assert dc.devcheck_scalar(op, da.data_ptr(), db.data_ptr(), dout.data_ptr(), a.size) == 0
        hout = np.zeros_like(a)
        dc.hostcheck_scalar(op, _p(a), _p(b), _p(hout), a.size)
        got = dout.cpu().numpy()
        if op not in (10, 12):
            # partially reduced results: the device and host builds may pick
            # different representatives of the same residue
            got, hout = _canon(got), _canon(hout)
        if not np.array_equal(got, hout):
            i = int(np.nonzero(got != hout)[0][0])
            bad.append(f"{name}: a={hex(int(a[i]))} b={hex(int(b[i]))} dev={hex(int(got[i]))} host={hex(int(hout[i]))}")
    assert not bad, "\n".join(bad)


@pytest.mark.gpu
def test_device_state_ops_match_host(dc, orc):
    import torch
    c = consts151(orc)
    st = np.random.default_rng(9).integers(0, 2 ** 64, size=(512, 16), dtype=np.uint64)
    st[0] = np.arange(16, dtype=np.uint64)
    bad = []
    for op, name in STATE_OPS.items():
        d = torch.from_numpy(st.copy()).cuda()
        assert dc.devcheck_state(op, d.data_ptr(), 512, _p(c)) == 0
        h = st.copy()
        dc.hostcheck_state(op, _p(h), 512, _p(c))
        got = _canon(d.cpu().numpy())
        h = _canon(h)
        if not np.array_equal(got, h):
            rows = np.nonzero((got != h).any(axis=1))[0]
            bad.append(f"{name}: {rows.size} states differ, first {int(rows[0])}")
    assert not bad, "\n".join(bad)


@pytest.mark.gpu
@pytest.mark.parametrize("n", [1, 7, 513])
def test_device_permute_x4_matches_host(dc, orc, n):
    """The four-threads-per-state permutation (latency-bound Merkle kernels)
    against the one-thread host permutation, partially reduced inputs."""
    import torch
    c = consts151(orc)
    st = np.random.default_rng(11 + n).integers(0, 2 ** 64, size=(n, 16), dtype=np.uint64)
    st[0] = np.arange(16, dtype=np.uint64)
    d = torch.from_numpy(st.copy()).cuda()
    assert dc.devcheck_permute_x4(d.data_ptr(), n, _p(c)) == 0
    h = st.copy()
    dc.hostcheck_state(104, _p(h), n, _p(c))
    assert np.array_equal(_canon(d.cpu().numpy()), _canon(h))
