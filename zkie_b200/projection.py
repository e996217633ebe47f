"""The projection block of zkie-ops (crates/zkie-ops/src/projection.rs) on the
device: out = round((x @ W) / 2^shift) + bias, proved as

1. the forward product h = x @ W (``par::mm_par_fixed``, the tensor-core
   path for 16-bit inputs), never committed;
2. the MatMul GKR of h (u, v, ch drawn in that order from the challenge
   source, as ``matmul::prove`` on x^T) -- the Op::MatMul kernels;
3. the affine rounding constraint as ``prove_virtual`` over
   [eq(v||u), rem_off, h, out, bias, ones] with the five terms of
   prove_projection (:71-81);
4. the range check 0 <= rem_off < 2^shift as a logUp lookup into the table
   0 .. 2^shift - 1 (alpha, beta, then the fraction tree's own draws).

Every step runs in libzkie_b200.so; this module only orders the calls and
draws the challenges, exactly as prove_projection (:44-101) does.
``projection_witness`` builds out / rem_off from h and bias on the device
(the witness of the reference's tests, :136-176).
"""
from dataclasses import dataclass

import numpy as np
import torch

from ._lib import check, lib
from .device import P, empty, ptr, stream_handle, to_dev
from .gkr import MatmulProof, VirtualProof, eq_evals, matmul_fixed, op_matmul_prove, prove_virtual
from .logup import FractionalProof, build_lookup_num_den, prove_fractional


@dataclass
class ProjectionProof:
    """ProjectionProof of projection.rs:15-25."""
    matmul: MatmulProof
    affine: VirtualProof
    frac: FractionalProof
    alpha: int
    beta: int
    pt: np.ndarray
    u: np.ndarray
    v: np.ndarray
    ch: np.ndarray


def projection_terms(shift: int):
    """The five (coefficient, MLE indices) terms of prove_projection over
    [eq, rem_off, h, out, bias, ones]: eq rem - eq h + 2^s eq out - 2^s eq bias
    - 2^(s-1) eq ones."""
    two = 1 << shift
    half = 1 << (shift - 1)
    neg = P - 1
    return [(1, [0, 1]), (neg, [0, 2]), (two, [0, 3]), (neg * two % P, [0, 4]), (neg * half % P, [0, 5])]


_CONST_CACHE = {}


def _constant_column(kind: str, n: int) -> torch.Tensor:
    """ones (n) or the range table 0 .. n - 1, kept on the device across calls."""
    key = (kind, n, torch.cuda.current_device())
    if key not in _CONST_CACHE:
        if kind == "ones":
            t = torch.ones(n, dtype=torch.int64, device="cuda")
        else:
            t = torch.arange(n, dtype=torch.int64, device="cuda")
        _CONST_CACHE[key] = t.view(torch.uint64)
    return _CONST_CACHE[key]


def projection_witness(h, bias, shift: int):
    """(out, rem_off, idx) on the device from h = x @ W and bias (m n field
    elements each): out = div_round(h, 2^shift) + bias, rem_off = h - (out -
    bias) 2^shift + 2^(shift - 1), idx = to_i32(rem_off) as u32."""
    dh, db = to_dev(h).reshape(-1), to_dev(bias).reshape(-1)
    if dh.numel() != db.numel():
        raise ValueError("projection_witness: h and bias lengths differ")
    n = dh.numel()
    out, rem = empty(n), empty(n)
    idx = torch.empty(n, dtype=torch.uint32, device=dh.device)
    check(lib.zkie2_projection_witness(ptr(dh), ptr(db), n, shift, ptr(out), ptr(rem), idx.data_ptr(),
                                       stream_handle()), "zkie2_projection_witness")
    return out, rem, idx


def lookup_index(v) -> torch.Tensor:
    """to_i32(v) as u32 of every element (the range check's lookup indices)."""
    dv = to_dev(v).reshape(-1)
    idx = torch.empty(dv.numel(), dtype=torch.uint32, device=dv.device)
    check(lib.zkie2_lookup_index_i32(ptr(dv), dv.numel(), idx.data_ptr(), stream_handle()),
          "zkie2_lookup_index_i32")
    return idx


def prove_projection(x, w, bias, out, rem_off, m: int, k: int, n: int, shift: int, rng,
                     idx=None, h=None) -> ProjectionProof:
    """prove_projection (projection.rs:44-101).  x (m x k), w (k x n), bias,
    out and rem_off (m x n) are field elements (device tensors or host
    arrays); rng is a XorShift64, Transcript or shard child (advanced in
    place).  ``idx`` (the lookup indices) and ``h`` (= x @ w) may be passed
    when the caller already has them on the device."""
    if shift < 1 or shift > 30:
        raise ValueError("prove_projection: 1 <= shift <= 30")
    dx, dw = to_dev(x).reshape(-1), to_dev(w).reshape(-1)
    db, do, dr = (to_dev(t).reshape(-1) for t in (bias, out, rem_off))
    if dx.numel() != m * k or dw.numel() != k * n or not (db.numel() == do.numel() == dr.numel() == m * n):
        raise ValueError("prove_projection: shape mismatch")
    dh = to_dev(h).reshape(-1) if h is not None else matmul_fixed(dx, dw, m, k, n)[0]
    op = op_matmul_prove(dx, dw, dh, m, k, n, rng)          # draws u, v, ch; matmul::prove(x^T, w, h)
    pt = np.concatenate([op.v, op.u]).astype(np.uint64)
    eq = eq_evals(pt)
    ones = _constant_column("ones", m * n)
    affine = prove_virtual([eq, dr, dh, do, db, ones], projection_terms(shift), 0, pt)
    alpha, beta = rng.field(), rng.field()
    table = _constant_column("range", 1 << shift)
    ix = idx if idx is not None else lookup_index(dr)
    num, den = build_lookup_num_den(ix, dr, table, alpha, beta)
    frac = prove_fractional(num, den, rng)
    return ProjectionProof(op.proof, affine, frac, int(alpha), int(beta), pt, op.u, op.v, op.ch)
