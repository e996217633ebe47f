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

The whole sequence is one C-ABI call (zkie2_projection_prove), which orders
the device steps and draws the challenges exactly as prove_projection
(:44-101) does; this module rebuilds the proof object from its outputs.
``projection_witness`` builds out / rem_off from h and bias on the device
(the witness of the reference's tests, :136-176).
"""
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import check, lib
from .device import P, empty, ptr, stream_handle, to_dev
from .gkr import MatmulProof, SumcheckProof, VirtualProof
from .logup import FractionalLayer, FractionalProof


def _p(a: np.ndarray):
    return a.ctypes.data_as(_lib.pu64)


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


def prove_projection(x, w, bias, out, rem_off, m: int, k: int, n: int, shift: int, rng, h=None) -> ProjectionProof:
    """prove_projection (projection.rs:44-101) through the single C-ABI call
    zkie2_projection_prove.  x (m x k), w (k x n), bias, out and rem_off
    (m x n) are field elements (device tensors or host arrays); rng is a
    XorShift64, Transcript or shard child (advanced in place).  ``h`` (= x @ w
    on the device) may be passed when the caller already has it."""
    if shift < 1 or shift > 30:
        raise ValueError("prove_projection: 1 <= shift <= 30")
    dx, dw = to_dev(x).reshape(-1), to_dev(w).reshape(-1)
    db, do, dr = (to_dev(t).reshape(-1) for t in (bias, out, rem_off))
    if dx.numel() != m * k or dw.numel() != k * n or not (db.numel() == do.numel() == dr.numel() == m * n):
        raise ValueError("prove_projection: shape mismatch")
    ns = lib.zkie2_projection_scratch_elems(m, k, n, shift)
    if ns == 0:
        raise ValueError("prove_projection: m, k, n must be powers of two")
    dh = to_dev(h).reshape(-1) if h is not None else None
    lm, lk, ln = (v.bit_length() - 1 for v in (m, k, n))
    t = lm + ln
    lg = lib.zkie2_projection_lookup_vars(m, n, shift)
    u64 = lambda c: np.zeros(max(c, 1), dtype=np.uint64)  # noqa: E731
    claimed, mm_rounds, mm_finals = u64(1), u64(3 * lk), u64(2)
    u, v, ch = u64(lm), u64(ln), u64(lk)
    aff_rounds, aff_finals, ab = u64(3 * t), u64(6), u64(2)
    full_r, cs = u64(lg), u64(lg)
    fr_rounds, fr_finals, fr_nd = u64(2 * lg * (lg - 1)), u64(7 * lg), u64(2)
    scr = empty(ns)
    src = rng.challenger()
    check(lib.zkie2_projection_prove(ptr(dx), ptr(dw), ptr(db), ptr(do), ptr(dr), ptr(dh) if dh is not None else None,
                                     m, k, n, shift, _lib.C.byref(src), *(_p(a) for a in (
                                         claimed, mm_rounds, mm_finals, u, v, ch, aff_rounds, aff_finals, ab, full_r,
                                         cs, fr_rounds, fr_finals, fr_nd)), ptr(scr), stream_handle()),
          "zkie2_projection_prove")
    rng.sync_from(src)
    layers, off = [], 0
    for layer in range(lg):
        tl = lg - layer - 1
        layers.append(FractionalLayer(full_r[:tl].copy(), int(cs[layer]) % P,
                                      VirtualProof(fr_rounds[off:off + 4 * tl].reshape(tl, 4).copy(),
                                                   fr_finals[7 * layer:7 * layer + 7].copy())))
        off += 4 * tl
    frac = FractionalProof(layers, int(fr_nd[0]), int(fr_nd[1]), full_r[:lg].copy())
    mm = MatmulProof(int(claimed[0]), SumcheckProof(mm_rounds[:3 * lk].reshape(lk, 3), int(mm_finals[0]),
                                                    int(mm_finals[1])))
    pt = np.concatenate([v[:ln], u[:lm]]).astype(np.uint64)
    return ProjectionProof(mm, VirtualProof(aff_rounds[:3 * t].reshape(t, 3), aff_finals.copy()), frac, int(ab[0]),
                           int(ab[1]), pt, u[:lm].copy(), v[:ln].copy(), ch[:lk].copy())
