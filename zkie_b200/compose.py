"""The op layer of zkie-ops (crates/zkie-ops/src/compose.rs) on the device.

Host-side mirror of the reference's op graph and shard prover for the arms a
GPT-2 model uses, over libzkie_b200.so:

- the ``Op`` variants (compose.rs:560-800) with ``reads`` / ``writes``
  (:955-1060), and ``Store`` (:525-560) holding device tensors;
- ``forward_ops`` (:1174-1583): every arm's forward witness as device
  kernels (the matmuls on the tensor cores where the inputs allow, as
  par::mm_par_fixed);
- ``prove_shard_precomputed`` (:1602-2091), ``prove_shard`` (:1589-1597) and
  ``prove_shard_dag`` (:2289-2346), with the arms' provers:
  prove_layer_norm_centered (layer_norm_centered.rs:122-245),
  prove_layernorm_chain (layernorm_chain.rs:24-93), prove_softmax_rounded
  (softmax_scaled.rs:42-108), prove_same_poly (common/same_poly.rs:13-45),
  prove_projection (projection.rs:44-101), prove_topk / prove_argmax /
  prove_range_decomp (topk.rs:82-176, 299-318, 391-448), the Op::MatMul and
  Add arms, and
  the per-table logUp of prove_lookup_witness_batch_columns and
  prove_lookup_table (common/logup_gkr.rs:340-383).

No prover in zkie-ops absorbs proof data into its challenge source: every
challenge of a shard is a function of the statement alone.  The prover
therefore draws each challenge on the host in the reference's order and
enqueues the device work behind it without waiting; the proof, the claims'
evaluations and the error word come back in one copy at the end.  The two
reduction sumchecks of prove_layer_norm_centered whose proofs the reference
discards (:153-159, :193-201) only advance the challenge source here.
"""
import contextlib
import ctypes as C
from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np
import torch

from . import _lib
from ._lib import check, lib
from .device import P, device, empty, ptr, stream_handle, to_dev
from .gkr import MatmulProof, OpMatMulProof, SumcheckProof, Transcript, VirtualProof
from .logup import FractionalLayer, FractionalProof
from .projection import ProjectionProof

NEG = P - 1


# ---- ops (compose.rs:560-800, reads/writes :955-1060) -------------------------------------
class _Op:
    kind = ""

    def reads(self):
        return [getattr(self, f) for f in self._reads]

    def writes(self):
        return [getattr(self, f) for f in self._writes]


@dataclass
class Transpose(_Op):
    x: int
    out: int
    m: int
    k: int
    kind = "Transpose"
    _reads, _writes = ("x",), ("out",)


@dataclass
class Scale(_Op):
    x: int
    out: int
    factor: int
    shift: int
    kind = "Scale"
    _reads, _writes = ("x",), ("out",)


@dataclass
class MatMul(_Op):
    a: int
    b: int
    c: int
    m: int
    k: int
    n: int
    kind = "MatMul"
    _reads, _writes = ("a", "b"), ("c",)


@dataclass
class Projection(_Op):
    x: int
    w: int
    bias: int
    out: int
    rem: int
    m: int
    k: int
    n: int
    shift: int
    kind = "Projection"
    _reads, _writes = ("x", "w", "bias"), ("out", "rem")


@dataclass
class Add(_Op):
    a: int
    b: int
    c: int
    kind = "Add"
    _reads, _writes = ("a", "b"), ("c",)


@dataclass
class Lookup(_Op):
    idx: int
    out: int
    table: int
    kind = "Lookup"
    _reads, _writes = ("idx", "table"), ("out",)


@dataclass
class Softmax(_Op):
    idx: int
    e: int
    out: int
    table: int
    m: int
    n: int
    kind = "Softmax"
    _reads, _writes = ("idx", "table"), ("e", "out")


@dataclass
class SoftmaxIndex(_Op):
    x: int
    out: int
    table_len: int
    kind = "SoftmaxIndex"
    _reads, _writes = ("x",), ("out",)


@dataclass
class GeluIndex(_Op):
    x: int
    out: int
    offset: int
    table_len: int
    kind = "GeluIndex"
    _reads, _writes = ("x",), ("out",)


@dataclass
class StableSoftmaxIndex(_Op):
    x: int
    mask: int
    out: int
    offset: int
    table_len: int
    m: int
    n: int
    kind = "StableSoftmaxIndex"
    _reads, _writes = ("x", "mask"), ("out",)


@dataclass
class Layernorm(_Op):
    x: int
    w: int
    b: int
    out: int
    rsqrt_table: int
    m: int
    d: int
    kind = "Layernorm"
    _reads, _writes = ("x", "w", "b", "rsqrt_table"), ("out",)


@dataclass
class LayerNormCentered(_Op):
    x: int
    w: int
    b: int
    out: int
    rsqrt_table: int
    m: int
    d: int
    n_real: int
    kind = "LayerNormCentered"
    _reads, _writes = ("x", "w", "b", "rsqrt_table"), ("out",)


@dataclass
class TopKSelect(_Op):
    x: int
    sel: int
    thr: int
    gate: int
    d1: int
    d2: int
    m: int
    n: int
    k: int
    kind = "TopKSelect"
    _reads, _writes = ("x",), ("sel", "thr", "gate", "d1", "d2")


@dataclass
class Argmax(_Op):
    x: int
    sel: int
    thr: int
    gate: int
    d1: int
    d2: int
    out: int  # an index tensor
    m: int
    n: int
    kind = "Argmax"
    _reads, _writes = ("x",), ("sel", "thr", "gate", "d1", "d2")


@dataclass
class ScaleVec(_Op):
    x: int
    scale: int
    out: int
    shift: int
    kind = "ScaleVec"
    _reads, _writes = ("x", "scale"), ("out",)


@dataclass
class BroadcastScale(_Op):
    x: int
    scale: int
    out: int
    h: int
    kind = "BroadcastScale"
    _reads, _writes = ("x", "scale"), ("out",)


@dataclass
class IdxBroadcast(_Op):
    base: int  # index tensors in and out
    out: int
    b: int
    kind = "IdxBroadcast"
    _reads, _writes = ("base",), ("out",)


@dataclass
class CombineIdx(_Op):
    a: int  # index tensors in and out
    b: int
    out: int
    scale: int
    kind = "CombineIdx"
    _reads, _writes = ("a", "b"), ("out",)


@dataclass
class PadIdx(_Op):
    base: int  # index tensors in and out
    out: int
    len: int
    kind = "PadIdx"
    _reads, _writes = ("base",), ("out",)


@dataclass
class ScaleGate(_Op):
    x: int
    gate: int
    col: int
    out: int
    m: int
    n: int
    h: int
    shift: int
    kind = "ScaleGate"
    _reads, _writes = ("x", "gate"), ("out",)


@dataclass
class Relu(_Op):
    x: int
    out: int
    kind = "Relu"
    _reads, _writes = ("x",), ("out",)


@dataclass
class BatchedMatMul(_Op):
    a: int
    w: int
    c: int
    s: int
    k: int
    n: int
    kind = "BatchedMatMul"
    _reads, _writes = ("a", "w"), ("c",)


@dataclass
class RmsNorm(_Op):
    x: int
    w: int
    out: int
    rsqrt_table: int
    limb_table: int
    m: int
    d: int
    n_real: int
    kind = "RmsNorm"
    _reads, _writes = ("x", "w", "rsqrt_table", "limb_table"), ("out",)


@dataclass
class RoPE(_Op):
    x: int
    cos: int
    sin: int
    out: int
    range_table: int
    m: int
    d: int
    shift: int
    kind = "RoPE"
    _reads, _writes = ("x", "cos", "sin", "range_table"), ("out",)


@dataclass
class Scatter(_Op):
    sel: int
    token_id: int  # index tensors out
    expert_of: int
    m: int
    n: int
    kind = "Scatter"
    _reads, _writes = ("sel",), ("token_id", "expert_of")


@dataclass
class Gather(_Op):
    weighted: int
    token_id: int  # an index tensor
    gate: int
    out: int
    m: int
    h: int
    kind = "Gather"
    _reads, _writes = ("weighted", "token_id", "gate"), ("out",)


@dataclass
class GatherMatMul(_Op):
    a: int
    expert_of: int  # an index tensor
    w: int
    c: int
    s: int
    k: int
    n: int
    n_experts: int
    kind = "GatherMatMul"
    _reads, _writes = ("a", "expert_of", "w"), ("c",)


# ---- the store (compose.rs:525-560) -------------------------------------------------------
class Store:
    """Field tensors ``v`` and u32 index tensors ``idx`` on the device, two id
    spaces as in the reference.  ``proj_h`` keeps each Projection's forward
    product x W (by output id) so the prover need not recompute it."""

    def __init__(self):
        self.v: List[Optional[torch.Tensor]] = []
        self.idx: List[Optional[torch.Tensor]] = []
        self.proj_h = {}

    def push(self, t=None) -> int:
        self.v.append(None if t is None else to_dev(t).reshape(-1))
        return len(self.v) - 1

    def push_idx(self, t=None) -> int:
        if t is not None:
            t = torch.as_tensor(np.asarray(t, dtype=np.uint32) if not isinstance(t, torch.Tensor) else t)
            t = t.to(device(), torch.uint32).reshape(-1).contiguous()
        self.idx.append(t)
        return len(self.idx) - 1

    def get(self, t: int) -> torch.Tensor:
        v = self.v[t]
        if v is None:
            raise ValueError(f"tensor {t} has no value (forward not run?)")
        return v

    def get_idx(self, t: int) -> torch.Tensor:
        v = self.idx[t]
        if v is None:
            raise ValueError(f"index tensor {t} has no value (forward not run?)")
        return v


def _u32(n: int) -> torch.Tensor:
    return torch.empty(max(n, 1), dtype=torch.uint32, device=device())


def _err_word() -> torch.Tensor:
    return torch.zeros(1, dtype=torch.int32, device=device())


_ERRORS = {1: "a lookup index outside its table", 2: "a softmax row sum of zero (round_div by zero)"}


def _check_err(err: torch.Tensor, what: str):
    code = int(err.item())
    if code:
        raise ValueError(f"{what}: " + ", ".join(v for k, v in _ERRORS.items() if code & k))


def layer_norm_centered_columns(x, w, b, table, m, d, n_real, err):
    """layer_norm_forward (layer_norm_centered.rs:42-120) on the device: a dict
    of its outputs (mean, centered, var, rstd, raw, out, rem_out, sum_mean,
    rem_mean, sum_var, rem_var, s_index)."""
    names = ("mean", "centered", "var", "rstd", "raw", "out", "rem_out", "sum_mean", "rem_mean", "sum_var",
             "rem_var")
    sizes = (m, m * d, m, m, m * d, m * d, m * d, m, m, m, m)
    outs = {k: empty(s) for k, s in zip(names, sizes)}
    s_index = _u32(m)
    arr = (_lib.vp * 11)(*[ptr(outs[k]) for k in names])
    check(lib.zkie2_op_layer_norm_centered(ptr(x), ptr(w), ptr(b), ptr(table), table.numel(), m, d, n_real, arr,
                                           s_index.data_ptr(), err.data_ptr(), stream_handle()),
          "zkie2_op_layer_norm_centered")
    outs["s_index"] = s_index[:m]
    return outs


def rms_norm_columns(x, w, table, m, d, n_real, err):
    """rms_norm_forward (rms_norm.rs:37-95) on the device: a dict of ms, rstd,
    raw, out, rem_out, rem_lo, rem_hi, sum_sq, rem_s and s_index."""
    names = ("ms", "rstd", "raw", "out", "rem_out", "rem_lo", "rem_hi", "sum_sq", "rem_s")
    sizes = (m, m, m * d, m * d, m * d, m * d, m * d, m, m)
    outs = {k: empty(sz) for k, sz in zip(names, sizes)}
    s_index = _u32(m)
    arr = (_lib.vp * 9)(*[ptr(outs[k]) for k in names])
    check(lib.zkie2_op_rms_norm(ptr(x), ptr(w), ptr(table), table.numel(), m, d, n_real, arr, s_index.data_ptr(),
                                err.data_ptr(), stream_handle()), "zkie2_op_rms_norm")
    outs["s_index"] = s_index[:m]
    return outs


def _index_i32(v: torch.Tensor) -> torch.Tensor:
    """to_i32(v) as u32 of every value."""
    idx = _u32(v.numel())
    check(lib.zkie2_lookup_index_i32(ptr(v), v.numel(), idx.data_ptr(), stream_handle()), "zkie2_lookup_index_i32")
    return idx[:v.numel()]


def _gather_matmul_forward(store: Store, op, err):
    """gather_matmul_forward (batched_matmul.rs:331-357): the positions of
    each run of equal experts times that expert's K x N block (the exact
    field product, on the tensor cores where the inputs are 16-bit)."""
    a, eof, w = store.get(op.a), store.get_idx(op.expert_of), store.get(op.w)
    s, k, n, ne = op.s, op.k, op.n, op.n_experts
    if a.numel() != s * k or eof.numel() != s or w.numel() != ne * k * n:
        raise ValueError("GatherMatMul: tensor sizes do not match s, k, n, n_experts")
    c = _slot(store, op.c, s * n)
    e = eof.cpu().numpy().astype(np.int64)
    if e.size and int(e.max()) >= ne:
        raise ValueError("GatherMatMul: an expert index outside the weights")
    runs, p0 = [], 0
    while p0 < s:
        p1 = p0 + 1
        while p1 < s and e[p1] == e[p0]:
            p1 += 1
        runs += [int(e[p0]), p0, p1 - p0]
        p0 = p1
    if not runs:
        return
    h_runs = np.array(runs, dtype=np.uint64)
    longest = int(h_runs[2::3].max())
    scr = empty(max(lib.zkie2_matmul_fixed_runs_scratch_elems(longest, k, n), 1))
    check(lib.zkie2_matmul_fixed_runs(ptr(a), ptr(w), ne, k, n, _pp(h_runs), len(runs) // 3, ptr(c), ptr(scr),
                                      stream_handle()), "zkie2_matmul_fixed_runs")


def layernorm_columns(x, w, b, table, m, d):
    """The Layernorm arm's forward (compose.rs:1467-1496): mean_sq, idx, rsqrt, scale, out."""
    mean_sq, rsqrt, scale, out = empty(m), empty(m), empty(m * d), empty(m * d)
    idx = _u32(m)
    check(lib.zkie2_op_layernorm(ptr(x), ptr(w), ptr(b), ptr(table), table.numel(), m, d, ptr(mean_sq),
                                 idx.data_ptr(), ptr(rsqrt), ptr(scale), ptr(out), stream_handle()),
          "zkie2_op_layernorm")
    return dict(mean_sq=mean_sq, idx=idx[:m], rsqrt=rsqrt, scale=scale, out=out)


class _MatmulPlan:
    """The tensor path's choice for every product of one forward pass, in
    order: recorded by an eager pass (``record``), then issued without
    read-backs for a CUDA-graph capture (``replay``; a product whose
    operands outgrow its recorded planes sets bit 3 of the error word)."""

    def __init__(self):
        self.mode, self.steps, self.pos = "record", [], 0


def _matmul_fixed(a, b, m, k, n, plan: Optional[_MatmulPlan] = None, err: Optional[torch.Tensor] = None):
    from .gkr import matmul_fixed
    if plan is None:
        return matmul_fixed(a, b, m, k, n)[0]
    da, db = a.reshape(-1), b.reshape(-1)
    dc = empty(m * n)
    scr = empty(max(lib.zkie2_matmul_fixed_scratch_elems(m, k, n), 1))
    if plan.mode == "record":
        h = np.zeros(3, dtype=np.uint32)
        check(lib.zkie2_matmul_fixed_ex(ptr(da), ptr(db), m, k, n, ptr(dc), 0, h.ctypes.data_as(_lib.pu32), ptr(scr),
                                        stream_handle()), "zkie2_matmul_fixed_ex")
        plan.steps.append(((m, k, n), h))
    else:
        shape, h = plan.steps[plan.pos]
        plan.pos += 1
        if shape != (m, k, n):
            raise ValueError("recorded matmul plan does not match the ops")
        check(lib.zkie2_matmul_fixed_planned(ptr(da), ptr(db), m, k, n, ptr(dc), h.ctypes.data_as(_lib.pu32),
                                             ptr(scr), err.data_ptr(), stream_handle()), "zkie2_matmul_fixed_planned")
    return dc


def _slot(store: Store, t: int, n: int) -> torch.Tensor:
    """The output buffer of tensor t: its current buffer when it has the
    right size (so a recorded proof graph keeps reading the same memory),
    else a new one."""
    v = store.v[t]
    if v is None or v.numel() != n:
        v = empty(n)
        store.v[t] = v
    return v


def _islot(store: Store, t: int, n: int) -> torch.Tensor:
    v = store.idx[t]
    if v is None or v.numel() != n:
        v = _u32(n)[:n]
        store.idx[t] = v
    return v


# arms whose forward reads data back to the host (routing): not recordable
_HOST_READ_KINDS = ("Scatter", "GatherMatMul")
# error-word bit of a planned product whose operands outgrew its plan
ERR_PLAN = 4
# arms whose outputs are index tensors (a separate id space)
_INDEX_WRITERS = ("SoftmaxIndex", "GeluIndex", "StableSoftmaxIndex", "Scatter", "PadIdx", "IdxBroadcast", "CombineIdx")


def _projection_groups(ops):
    """Projections that read the same x (same m, k) and whose weights and
    biases no op writes at or after the first of them: {first index: [the
    group's indices]} (groups of two or more).  Their products x W_j are one
    matmul against the weights side by side, done at the first one."""
    written = {}
    for i, op in enumerate(ops):
        if op.kind not in _INDEX_WRITERS:
            for t in op.writes():
                written.setdefault(t, i)
    by_input = {}
    for i, op in enumerate(ops):
        if op.kind == "Projection":
            by_input.setdefault((op.x, op.m, op.k), []).append(i)
    groups = {}
    for members in by_input.values():
        i = members[0]
        grp = [i] + [j for j in members[1:] if all(written.get(t, -1) < i for t in (ops[j].w, ops[j].bias))]
        if len(grp) > 1:
            groups[i] = grp
    return groups


def _projection_witness(store: Store, op, h: torch.Tensor, sh):
    """out / rem of one Projection from its product h (kept for the prover)."""
    if op.out in store.proj_h and store.proj_h[op.out].numel() == h.numel():
        store.proj_h[op.out].copy_(h)
        h = store.proj_h[op.out]
    store.proj_h[op.out] = h
    out, rem = _slot(store, op.out, op.m * op.n), _slot(store, op.rem, op.m * op.n)
    check(lib.zkie2_projection_witness(ptr(h), ptr(store.get(op.bias)), op.m * op.n, op.shift, ptr(out), ptr(rem),
                                       None, sh), "zkie2_projection_witness")


def forward_ops(store: Store, ops, plan: Optional[_MatmulPlan] = None, err: Optional[torch.Tensor] = None):
    """forward_ops (compose.rs:1174-1583) on the device, writing every output
    into its existing buffer where it has one; raises where the reference
    panics on the data (after the whole pass, one read-back; with ``err``
    given the caller reads that error word instead).  Projections sharing
    their input x are multiplied as one wide matmul.  ``plan`` records or
    replays the products' tensor-path choices (GraphForward)."""
    own_err = err is None
    err = _err_word() if own_err else err
    sh = stream_handle()
    if plan is not None and plan.mode == "replay" and any(op.kind in _HOST_READ_KINDS for op in ops):
        raise ValueError("forward_ops: Scatter and GatherMatMul read routing data back and cannot be recorded")
    groups = _projection_groups(ops)
    grouped = {j for grp in groups.values() for j in grp}
    for i, op in enumerate(ops):
        k = op.kind
        g = store.get
        if i in groups:
            grp = [ops[j] for j in groups[i]]
            w_cat = torch.cat([g(o.w).view(torch.int64).reshape(op.k, o.n) for o in grp], dim=1).contiguous()
            total = sum(o.n for o in grp)
            h_all = _matmul_fixed(g(op.x), w_cat.view(torch.uint64).reshape(-1), op.m, op.k, total, plan, err)
            h2 = h_all.view(torch.int64).reshape(op.m, total)
            c0 = 0
            for o in grp:
                _projection_witness(store, o, h2[:, c0:c0 + o.n].contiguous().view(torch.uint64).reshape(-1), sh)
                c0 += o.n
            continue
        if i in grouped:
            continue  # computed with its group
        if k == "Transpose":
            out = _slot(store, op.out, op.m * op.k)
            check(lib.zkie2_op_transpose(ptr(g(op.x)), op.m, op.k, ptr(out), sh), "zkie2_op_transpose")
        elif k == "Scale":
            x = g(op.x)
            out = _slot(store, op.out, x.numel())
            check(lib.zkie2_op_scale(ptr(x), x.numel(), op.factor, op.shift, ptr(out), sh), "zkie2_op_scale")
        elif k == "MatMul":
            _slot(store, op.c, op.m * op.n).copy_(_matmul_fixed(g(op.a), g(op.b), op.m, op.k, op.n, plan, err))
        elif k == "Projection":
            _projection_witness(store, op, _matmul_fixed(g(op.x), g(op.w), op.m, op.k, op.n, plan, err), sh)
        elif k == "Add":
            a, b = g(op.a), g(op.b)
            out = _slot(store, op.c, a.numel())
            check(lib.zkie2_op_add(ptr(a), ptr(b), a.numel(), ptr(out), sh), "zkie2_op_add")
        elif k == "Lookup":
            idx, table = store.get_idx(op.idx), g(op.table)
            out = _slot(store, op.out, idx.numel())
            check(lib.zkie2_op_lookup(idx.data_ptr(), idx.numel(), ptr(table), table.numel(), ptr(out),
                                      err.data_ptr(), sh), "zkie2_op_lookup")
        elif k == "Softmax":
            idx, table = store.get_idx(op.idx), g(op.table)
            e, out = _slot(store, op.e, op.m * op.n), _slot(store, op.out, op.m * op.n)
            check(lib.zkie2_op_softmax(idx.data_ptr(), ptr(table), table.numel(), op.m, op.n, ptr(e), ptr(out),
                                       None, err.data_ptr(), sh), "zkie2_op_softmax")
        elif k == "SoftmaxIndex":
            x = g(op.x)
            idx = _islot(store, op.out, x.numel())
            check(lib.zkie2_op_softmax_index(ptr(x), x.numel(), op.table_len, idx.data_ptr(), sh),
                  "zkie2_op_softmax_index")
        elif k == "GeluIndex":
            x = g(op.x)
            idx = _islot(store, op.out, x.numel())
            check(lib.zkie2_op_gelu_index(ptr(x), x.numel(), op.offset, op.table_len, idx.data_ptr(), sh),
                  "zkie2_op_gelu_index")
        elif k == "StableSoftmaxIndex":
            idx = _islot(store, op.out, op.m * op.n)
            check(lib.zkie2_op_stable_softmax_index(ptr(g(op.x)), ptr(g(op.mask)), op.m, op.n, op.offset,
                                                    op.table_len, idx.data_ptr(), sh),
                  "zkie2_op_stable_softmax_index")
        elif k == "Layernorm":
            out = layernorm_columns(g(op.x), g(op.w), g(op.b), g(op.rsqrt_table), op.m, op.d)["out"]
            _slot(store, op.out, out.numel()).copy_(out)
        elif k == "LayerNormCentered":
            out = layer_norm_centered_columns(g(op.x), g(op.w), g(op.b), g(op.rsqrt_table), op.m, op.d, op.n_real,
                                              err)["out"]
            _slot(store, op.out, out.numel()).copy_(out)
        elif k == "RmsNorm":
            out = rms_norm_columns(g(op.x), g(op.w), g(op.rsqrt_table), op.m, op.d, op.n_real, err)["out"]
            _slot(store, op.out, out.numel()).copy_(out)
        elif k == "RoPE":
            x = g(op.x)
            out = _slot(store, op.out, x.numel())
            check(lib.zkie2_op_rope(ptr(x), x.numel(), ptr(g(op.cos)), ptr(g(op.sin)), op.m, op.d, op.shift, ptr(out),
                                    sh), "zkie2_op_rope")
        elif k == "ScaleVec":
            x, sv = g(op.x), g(op.scale)
            out = _slot(store, op.out, x.numel())
            check(lib.zkie2_op_scale_vec(ptr(x), x.numel(), ptr(sv), sv.numel(), op.shift, ptr(out), sh),
                  "zkie2_op_scale_vec")
        elif k == "BroadcastScale":
            x, sv = g(op.x), g(op.scale)
            out = _slot(store, op.out, x.numel())
            check(lib.zkie2_op_broadcast_scale(ptr(x), x.numel(), ptr(sv), sv.numel(), op.h, ptr(out), sh),
                  "zkie2_op_broadcast_scale")
        elif k == "IdxBroadcast":
            base = store.get_idx(op.base)
            out = _islot(store, op.out, base.numel() * op.b)
            check(lib.zkie2_op_idx_broadcast(base.data_ptr(), base.numel(), op.b, out.data_ptr(), sh),
                  "zkie2_op_idx_broadcast")
        elif k == "CombineIdx":
            a, b = store.get_idx(op.a), store.get_idx(op.b)
            if a.numel() != b.numel():
                raise ValueError("CombineIdx: index tensors differ in length")
            out = _islot(store, op.out, a.numel())
            check(lib.zkie2_op_combine_idx(a.data_ptr(), b.data_ptr(), a.numel(), op.scale, out.data_ptr(), sh),
                  "zkie2_op_combine_idx")
        elif k == "PadIdx":
            base = store.get_idx(op.base)
            out = _islot(store, op.out, op.len)
            check(lib.zkie2_op_pad_idx(base.data_ptr(), base.numel(), op.len, out.data_ptr(), sh), "zkie2_op_pad_idx")
        elif k == "Scatter":
            sel = g(op.sel)
            cnt = _u32(op.n)
            check(lib.zkie2_op_sel_counts(ptr(sel), op.m, op.n, 0, cnt.data_ptr(), sh), "zkie2_op_sel_counts")
            total = int(cnt[:op.n].to(torch.int64).sum().item())
            tid, eof = _islot(store, op.token_id, total), _islot(store, op.expert_of, total)
            first = empty(op.n)
            check(lib.zkie2_op_scatter(ptr(sel), op.m, op.n, cnt.data_ptr(), tid.data_ptr(), eof.data_ptr(),
                                       ptr(first), sh), "zkie2_op_scatter")
        elif k == "Gather":
            wt, tid, gate = g(op.weighted), store.get_idx(op.token_id), g(op.gate)
            s_ = tid.numel()
            if gate.numel() != s_ or wt.numel() != s_ * op.h:
                raise ValueError("Gather: weighted, token_id and gate lengths do not match")
            out = _slot(store, op.out, op.m * op.h)
            scr = _u32(lib.zkie2_op_gather_scratch_u32(s_, op.m))
            check(lib.zkie2_op_gather(ptr(wt), tid.data_ptr(), ptr(gate), s_, op.m, op.h, ptr(out), scr.data_ptr(),
                                      err.data_ptr(), sh), "zkie2_op_gather")
        elif k == "GatherMatMul":
            _gather_matmul_forward(store, op, err)
        elif k == "ScaleGate":
            x, gate = g(op.x), g(op.gate)
            out = _slot(store, op.out, x.numel())
            check(lib.zkie2_op_scale_gate(ptr(x), x.numel(), ptr(gate), gate.numel(), op.col, op.n, op.h, op.shift,
                                          ptr(out), sh), "zkie2_op_scale_gate")
        elif k == "Relu":
            x = g(op.x)
            out = _slot(store, op.out, x.numel())
            check(lib.zkie2_op_relu(ptr(x), x.numel(), ptr(out), sh), "zkie2_op_relu")
        elif k == "BatchedMatMul":
            a, w = g(op.a), g(op.w)
            if a.numel() != op.s * op.k or w.numel() != op.s * op.k * op.n:
                raise ValueError("BatchedMatMul: tensor sizes do not match s, k, n")
            out = _slot(store, op.c, op.s * op.n)
            check(lib.zkie2_op_batched_matmul(ptr(a), ptr(w), op.s, op.k, op.n, ptr(out), sh),
                  "zkie2_op_batched_matmul")
        elif k in ("TopKSelect", "Argmax"):
            mn = op.m * op.n
            thr = _slot(store, op.thr, op.m)
            sel, gate, d1, d2 = (_slot(store, t, mn) for t in (op.sel, op.gate, op.d1, op.d2))
            out = _islot(store, op.out, op.m) if k == "Argmax" else None
            check(lib.zkie2_op_topk(ptr(g(op.x)), op.m, op.n, op.k if k == "TopKSelect" else 1, ptr(thr), ptr(sel),
                                    ptr(gate), ptr(d1), ptr(d2), out.data_ptr() if out is not None else None, sh),
                  "zkie2_op_topk")
        else:
            raise ValueError(f"op {k} is not supported")
    if own_err:
        _check_err(err, "forward_ops")


# ---- proofs (compose.rs OpProof / OpShardProof, the arms' proof structs) -------------------
def _vcanon(p: VirtualProof):
    return (np.asarray(p.rounds, dtype=np.uint64), np.asarray(p.final_evals, dtype=np.uint64))


def _frac_canon(p: FractionalProof):
    layers = tuple((np.asarray(l.r, dtype=np.uint64), int(l.c), np.asarray(l.proof.rounds, dtype=np.uint64),
                    np.asarray(l.proof.final_evals, dtype=np.uint64)) for l in p.layers)
    return (layers, int(p.final_num), int(p.final_den), np.asarray(p.full_r, dtype=np.uint64))


@dataclass
class LayerNormCenteredProof:
    """layer_norm_centered.rs:25-36."""
    mean: VirtualProof
    centered: VirtualProof
    var: VirtualProof
    out: VirtualProof
    r_mean: np.ndarray
    mean_ch: np.ndarray
    centered_r: np.ndarray
    r_var: np.ndarray
    var_ch: np.ndarray
    r_out: np.ndarray

    def canonical(self):
        return ("LayerNormCentered", _vcanon(self.mean), _vcanon(self.centered), _vcanon(self.var),
                _vcanon(self.out), self.r_mean, self.mean_ch, self.centered_r, self.r_var, self.var_ch, self.r_out)


@dataclass
class LayernormChainProof:
    """layernorm_chain.rs:14-22."""
    mean_sq: VirtualProof
    out: VirtualProof
    r_mean: np.ndarray
    mean_ch: np.ndarray
    r_out: np.ndarray
    mean_claim: int

    def canonical(self):
        return ("Layernorm", _vcanon(self.mean_sq), _vcanon(self.out), self.r_mean, self.mean_ch, self.r_out,
                int(self.mean_claim))


@dataclass
class SoftmaxRoundedProof:
    """softmax_scaled.rs:31-40."""
    row_sum: VirtualProof
    rescale: VirtualProof
    r_sum: np.ndarray
    sum_ch: np.ndarray
    r_scale: np.ndarray
    claimed: int

    def canonical(self):
        return ("Softmax", _vcanon(self.row_sum), _vcanon(self.rescale), self.r_sum, self.sum_ch, self.r_scale,
                int(self.claimed))


@dataclass
class AddProof:
    """OpProof::Add(proof, r)."""
    proof: VirtualProof
    r: np.ndarray

    def canonical(self):
        return ("Add", _vcanon(self.proof), self.r)


@dataclass
class MarkerProof:
    """The arms with no proof of their own (Transpose, Scale, Lookup, the index ops)."""
    kind: str

    def canonical(self):
        return (self.kind,)


@dataclass
class SamePolyProof:
    """same_poly.rs:7-12."""
    coeffs: np.ndarray
    proof: VirtualProof
    merged_point: np.ndarray
    merged_eval: int

    def canonical(self):
        return (self.coeffs, _vcanon(self.proof), self.merged_point, int(self.merged_eval))


@dataclass
class WitnessColumn:
    """compose.rs WitnessColumn: the witness side of one table's logUp."""
    proof: FractionalProof
    x: torch.Tensor
    y: torch.Tensor
    num: torch.Tensor
    point: np.ndarray
    num_leaf: int
    den_leaf: int
    alpha: int
    beta: int
    table: int

    def canonical(self):
        return (_frac_canon(self.proof), self.x.cpu().numpy(), self.y.cpu().numpy(), self.num.cpu().numpy(),
                self.point, self.num_leaf, self.den_leaf, self.alpha, self.beta, self.table)


@dataclass
class TableColumn:
    """compose.rs TableColumn: the table side with its merged multiplicities."""
    proof: FractionalProof
    table: int
    m: torch.Tensor
    alpha: int
    beta: int
    point: np.ndarray
    num_leaf: int
    den_leaf: int

    def canonical(self):
        return (_frac_canon(self.proof), self.table, self.m.cpu().numpy(), self.alpha, self.beta, self.point,
                self.num_leaf, self.den_leaf)


@dataclass
class RangeDecompProof:
    """topk.rs:377-389."""
    c0_range: FractionalProof
    c1_range: FractionalProof
    c2_range: FractionalProof
    recompose: VirtualProof
    a0: int
    b0: int
    a1: int
    b1: int
    a2: int
    b2: int
    r: np.ndarray

    def canonical(self):
        return (_frac_canon(self.c0_range), _frac_canon(self.c1_range), _frac_canon(self.c2_range),
                _vcanon(self.recompose), self.a0, self.b0, self.a1, self.b1, self.a2, self.b2, self.r)


@dataclass
class TopKSelectProof:
    """topk.rs:22-39; ``sel`` is the one-hot witness the reference's proof
    carries (a device tensor here, read back by canonical())."""
    gate_rel: VirtualProof
    d1_rel: VirtualProof
    d2_rel: VirtualProof
    row_sum: VirtualProof
    sel_range: FractionalProof
    d1_range: FractionalProof
    d2_decomp: RangeDecompProof
    r: np.ndarray
    r_row: np.ndarray
    a_sel: int
    b_sel: int
    a_d1: int
    b_d1: int
    range_bits: int
    sel: torch.Tensor

    def canonical(self):
        return ("TopKSelect", _vcanon(self.gate_rel), _vcanon(self.d1_rel), _vcanon(self.d2_rel),
                _vcanon(self.row_sum), _frac_canon(self.sel_range), _frac_canon(self.d1_range),
                self.d2_decomp.canonical(), self.r, self.r_row, self.a_sel, self.b_sel, self.a_d1, self.b_d1,
                self.range_bits, self.sel.cpu().numpy())


@dataclass
class ArgmaxProof:
    """topk.rs:265-270: the top-1 proof, the public output positions and the
    (uncommitted path: empty) opened sel values."""
    topk: TopKSelectProof
    out: torch.Tensor

    def canonical(self):
        return ("Argmax", self.topk.canonical(), self.out.cpu().numpy(), ())


@dataclass
class RmsNormProof:
    """rms_norm.rs:25-33."""
    trunc: VirtualProof
    out: VirtualProof
    rem_split: VirtualProof
    trunc_ch: np.ndarray
    r_out: np.ndarray
    rem_split_ch: np.ndarray

    def canonical(self):
        return ("RmsNorm", _vcanon(self.trunc), _vcanon(self.out), _vcanon(self.rem_split), self.trunc_ch,
                self.r_out, self.rem_split_ch)


@dataclass
class RoPEProof:
    """rope.rs:33-40."""
    first: VirtualProof
    second: VirtualProof
    r_first: np.ndarray
    r_second: np.ndarray
    r_out: np.ndarray

    def canonical(self):
        return ("RoPE", _vcanon(self.first), _vcanon(self.second), self.r_first, self.r_second, self.r_out)


@dataclass
class PermutationProof:
    """common/logup_gkr.rs:799-805; the multisets as device tensors."""
    a_side: FractionalProof
    b_side: FractionalProof
    alpha: int
    a: torch.Tensor
    b: torch.Tensor

    def canonical(self):
        return (_frac_canon(self.a_side), _frac_canon(self.b_side), self.alpha, self.a.cpu().numpy(),
                self.b.cpu().numpy())


@dataclass
class ScatterProof:
    """scatter.rs:7-10."""
    perm: PermutationProof

    def canonical(self):
        return ("Scatter", self.perm.canonical())


@dataclass
class ScatterAddProof:
    """gather.rs:12-30 (OpProof::Gather); the columns as device tensors."""
    source_side: FractionalProof
    target_side: FractionalProof
    alpha: int
    gamma: np.ndarray
    num_source: torch.Tensor
    den_source: torch.Tensor
    num_target: torch.Tensor
    den_target: torch.Tensor
    prod_source: VirtualProof
    prod_target: VirtualProof
    r_prod_source: np.ndarray
    r_prod_target: np.ndarray
    weighted: torch.Tensor
    gate: torch.Tensor
    out: torch.Tensor
    token_id: torch.Tensor

    def canonical(self):
        h = lambda t: t.cpu().numpy()  # noqa: E731
        return ("Gather", _frac_canon(self.source_side), _frac_canon(self.target_side), self.alpha, self.gamma,
                h(self.num_source), h(self.den_source), h(self.num_target), h(self.den_target),
                _vcanon(self.prod_source), _vcanon(self.prod_target), self.r_prod_source, self.r_prod_target,
                h(self.weighted), h(self.gate), h(self.out), h(self.token_id))


@dataclass
class BatchedMatMulOpProof:
    """OpProof::BatchedMatMul(BatchedMatmulProof, u, v, ch) (batched_matmul.rs:24-28)."""
    claimed: int
    sumcheck: VirtualProof
    u: np.ndarray
    v: np.ndarray
    ch: np.ndarray

    def canonical(self):
        return ("BatchedMatMul", (int(self.claimed), _vcanon(self.sumcheck)), self.u, self.v, self.ch)


@dataclass
class GatherMatMulOpProof:
    """OpProof::GatherMatMul(GatherMatMulProof, u, v, ch) (batched_matmul.rs:462-467)."""
    claimed: int
    sumcheck: VirtualProof
    counts: np.ndarray
    table: np.ndarray
    u: np.ndarray
    v: np.ndarray
    ch: np.ndarray

    def canonical(self):
        return ("GatherMatMul", (int(self.claimed), _vcanon(self.sumcheck), self.counts, self.table), self.u, self.v,
                self.ch)


def _op_canon(p):
    if isinstance(p, OpMatMulProof):
        mm = p.proof
        return ("MatMul", mm.claimed, np.asarray(mm.sumcheck.rounds, dtype=np.uint64), mm.sumcheck.f_eval,
                mm.sumcheck.h_eval, p.u, p.v, p.ch)
    if isinstance(p, ProjectionProof):
        mm = p.matmul
        return ("Projection", (mm.claimed, np.asarray(mm.sumcheck.rounds, dtype=np.uint64), mm.sumcheck.f_eval,
                               mm.sumcheck.h_eval), _vcanon(p.affine), _frac_canon(p.frac), p.alpha, p.beta, p.pt,
                p.u, p.v, p.ch)
    return p.canonical()


@dataclass
class OpShardProof:
    """compose.rs OpShardProof: per-op proofs, the same_poly bindings, every
    raw claim (tensor, point, value) and the per-table logUp columns."""
    ops: list
    bound: List[int]
    binds: List[SamePolyProof]
    claims: list
    witness_columns: List[WitnessColumn]
    table_columns: List[TableColumn]

    def canonical(self):
        return dict(ops=[_op_canon(p) for p in self.ops], bound=list(self.bound),
                    binds=[b.canonical() for b in self.binds],
                    claims=[(t, np.asarray(pt, dtype=np.uint64), int(ev)) for t, pt, ev in self.claims],
                    witness_columns=[c.canonical() for c in self.witness_columns],
                    table_columns=[c.canonical() for c in self.table_columns])


@dataclass
class ShardDagProof:
    """compose.rs ShardDagProof."""
    shards: List[OpShardProof]
    cross_tensors: List[int]
    cross_binds: List[SamePolyProof]

    def canonical(self):
        return dict(shards=[s.canonical() for s in self.shards], cross_tensors=list(self.cross_tensors),
                    cross_binds=[b.canonical() for b in self.cross_binds])


# ---- the shard prover ---------------------------------------------------------------------
def _terms_arrays(terms):
    coeffs = np.array([int(c) % P for c, _ in terms] or [0], dtype=np.uint64)
    off, idx = [0], []
    for _, ids in terms:
        idx.extend(int(i) for i in ids)
        off.append(len(idx))
    return (coeffs, np.array(off, dtype=np.uint32), np.array(idx or [0], dtype=np.uint32),
            max((len(ids) for _, ids in terms), default=0))


def _pp(a: np.ndarray):
    return a.ctypes.data_as(_lib.pu64) if a.size else None


def _lg(n: int) -> int:
    n = int(n)
    if n <= 0 or n & (n - 1):
        raise ValueError(f"{n} is not a power of two")
    return n.bit_length() - 1


def _eq_at(r, x) -> int:
    """eq(r, x) = prod_j (r_j x_j + (1 - r_j)(1 - x_j))."""
    v = 1
    for a, b in zip(r, x):
        a, b = int(a), int(b)
        v = v * ((a * b + (1 - a) * (1 - b)) % P) % P
    return v


ADD_TERMS = [(1, [2]), (NEG, [0]), (NEG, [1])]
TRUNC_TERMS = lambda df, half: [(df % P, [0]), (1, [1]), (NEG, [2]), (NEG * half % P, [3])]  # noqa: E731
CENTERED_TERMS = [(1, [2]), (NEG, [0]), (1, [1])]
LNC_OUT_TERMS = [(1, [0, 1, 2]), (NEG, [4]), (1, [4]), (NEG * (1 << 32) % P, [5]), (1 << 32, [3]), (NEG, [6]),
                 (1 << 31, [7])]
LN_MEAN_TERMS = [(1, [0, 1, 1])]
LN_OUT_TERMS = [(1, [0, 1]), (1, [2]), (NEG, [3])]
SOFTMAX_SUM_TERMS = [(1, [0, 1])]
SOFTMAX_RESCALE_TERMS = [(1, [0, 2]), (NEG * (1 << 16) % P, [1]), (1, [3])]
PRODUCT_TERMS = [(1, [0, 1])]
GATE_TERMS = [(1, [0, 1]), (NEG, [2])]                                        # topk.rs:101
D1_TERMS = [(1, [0, 1]), (NEG, [0, 2]), (NEG, [3])]                           # :111-115
D2_TERMS = [(1, [2]), (NEG, [1]), (NEG, [0, 2]), (1, [0, 1]), (NEG, [3])]     # :119-125
ROW_SUM_TERMS = [(1, [0, 1])]                                                 # :137
RMS_OUT_TERMS = [(1, [0, 1, 2]), (NEG, [3]), (1, [3]), (NEG * (1 << 32) % P, [4]), (NEG, [5]), (1 << 31, [6])]  # rms_norm.rs:132-142
REM_SPLIT_TERMS = [(1, [0]), (NEG, [1]), (NEG * (1 << 16) % P, [2])]                  # :150-154
ROPE_TERMS = lambda shift, second: [(1, [0, 1]), ((1 if second else NEG), [2, 3]), (NEG * (1 << shift) % P, [4]),  # noqa: E731,E501
                                    (NEG, [5]), (1 << (shift - 1), [6])]          # rope.rs:152-177
SCATTER_ADD_SOURCE_TERMS = [(1, [0, 1]), (NEG, [0, 2, 3, 4])]                      # gather.rs:103-110
SCATTER_ADD_TARGET_TERMS = [(1, [0, 1]), (NEG, [0, 2, 3])]                         # :128-135
BMM_TERMS = [(1, [0, 1, 2])]                                                       # batched_matmul.rs:40-42
# the arms with no proof of their own (compose.rs:1623-1723)
MARKER_KINDS = ("Transpose", "Scale", "SoftmaxIndex", "GeluIndex", "StableSoftmaxIndex", "ScaleVec", "IdxBroadcast",
                "CombineIdx", "PadIdx", "BroadcastScale", "ScaleGate", "Relu")
RECOMPOSE_TERMS = [(1, [0]), (NEG, [1]), (NEG * (1 << 16) % P, [2]), (NEG * (1 << 32) % P, [3])]  # :428-433


def _cat_u64(parts) -> torch.Tensor:
    parts = [p.reshape(-1) for p in parts]
    if len(parts) == 1:
        return parts[0]
    return torch.cat([p.view(torch.int64) for p in parts]).view(torch.uint64)


def frac_tree_bytes(lg: int) -> int:
    """Bytes the fraction tree of 2^lg fractions touches once: each level
    reads num / den of level l and writes level l + 1; layer l's sumcheck
    reads its seven tables of 2^(lg - l - 1)."""
    total = 0
    for l in range(lg):
        half = 1 << (lg - l - 1)
        total += 8 * (4 * half + 2 * half) + 8 * 7 * half
    return total


class _Pending:
    """Device outputs of one proof in flight: every buffer a prover writes is
    registered here and fetched in one concatenated copy; ``host(h)`` then
    returns buffer h as a numpy array."""

    def __init__(self):
        self.parts = []
        self.arrays = None

    def out(self, n: int):
        t = empty(max(int(n), 1))
        self.parts.append(t)
        return len(self.parts) - 1, t

    def gather(self) -> torch.Tensor:
        """Every registered buffer in one device array (on the current stream)."""
        return _cat_u64(self.parts) if self.parts else empty(1)

    def download(self, flat: torch.Tensor, host: Optional[np.ndarray] = None):
        """Split the gathered results into the registered buffers: copied from
        ``flat`` now, or taken from ``host`` (a copy already made)."""
        if self.parts:
            host = flat.cpu().numpy() if host is None else host
            sizes = np.cumsum([p.numel() for p in self.parts])[:-1]
            self.arrays = np.split(host, sizes)
        else:
            self.arrays = []

    def fetch(self):
        self.download(self.gather())

    def host(self, h):
        return self.arrays[h]

    def value(self, ref):
        """An int, or (buffer, index) into a fetched buffer."""
        if isinstance(ref, (tuple, list)):
            return int(self.arrays[ref[0]][ref[1]])
        return int(ref)


class OpShardProver:
    """prove_shard_precomputed over a device Store (the witness already
    materialised), with ``rng`` the shard's challenge source."""

    def __init__(self, store: Store, rng, streams: int = 8):
        self.store, self.rng = store, rng
        self.pend = _Pending()
        self.err = _err_word()
        self.main = torch.cuda.current_stream()
        self.streams = stream_pool(streams) if streams > 1 else [self.main]
        self.turn = 0
        self.sh = stream_handle()
        self.claims = []      # (tensor, point, value ref)
        self.builders = []    # one per op: () -> proof object
        self.lookups = {}     # table -> [(idx tensor, value tensor, event or None)]
        self.evals = []       # evaluations waiting for flush_evals
        self.traffic = 0      # algorithmic bytes: every table a sub-proof reads, once
        self.keep = []        # columns read on streams other than the one that allocated them

    @contextlib.contextmanager
    def on(self, s):
        """Enqueue on stream s (allocations included)."""
        prev = self.sh
        with torch.cuda.stream(s):
            self.sh = s.cuda_stream
            try:
                yield
                self.flush_evals()
            finally:
                self.sh = prev

    def next_stream(self):
        s = self.streams[self.turn % len(self.streams)]
        self.turn += 1
        return s

    # -- primitives ------------------------------------------------------------------------
    def draw(self, n: int) -> np.ndarray:
        if hasattr(self.rng, "fields"):
            return self.rng.fields(n)
        return np.array([self.rng.field() for _ in range(n)], dtype=np.uint64)

    def eval(self, values: torch.Tensor, point: np.ndarray):
        """values(point), enqueued with the other evaluations of the current
        arm in one call (flush_evals); returns a reference to the result."""
        ref = [None, 0]
        self.evals.append((values, np.ascontiguousarray(point, dtype=np.uint64), ref))
        self.traffic += 8 * values.numel()
        return ref

    def flush_evals(self):
        if not self.evals:
            return
        n = len(self.evals)
        h, d = self.pend.out(n)
        ts = np.array([pt.size for _, pt, _ in self.evals], dtype=np.uint32)
        pts = np.ascontiguousarray(np.concatenate([pt for _, pt, _ in self.evals]))
        vals = (_lib.vp * n)(*[ptr(v) for v, _, _ in self.evals])
        scr = empty(max(lib.zkie2_mle_eval_many_scratch_elems(int(ts.max())), 1))
        check(lib.zkie2_mle_eval_many(vals, ts.ctypes.data_as(_lib.pu32), _pp(pts), n, ptr(d), ptr(scr), self.sh),
              "zkie2_mle_eval_many")
        for i, (_, _, ref) in enumerate(self.evals):
            ref[0], ref[1] = h, i
        self.evals = []

    def claim(self, t: int, point: np.ndarray, value=None):
        point = np.ascontiguousarray(point, dtype=np.uint64)
        self.claims.append((t, point, value if value is not None else self.eval(self.store.get(t), point)))

    def virtual(self, mles, terms, ch: np.ndarray):
        """prove_virtual enqueued -> a builder of the VirtualProof."""
        n, t = len(mles), ch.size
        self.traffic += 8 * n << t
        coeffs, off, idx, deg = _terms_arrays(terms)
        hr, dr = self.pend.out(t * (deg + 1))
        hf, df = self.pend.out(n)
        scr = empty(max(lib.zkie2_virtual_scratch_elems(n, t), 1))
        arr = (_lib.vp * n)(*[ptr(m) for m in mles])
        check(lib.zkie2_virtual_prove_async(arr, n, t, _pp(coeffs), off.ctypes.data_as(_lib.pu32),
                                            idx.ctypes.data_as(_lib.pu32), len(terms), _pp(ch), ptr(dr), ptr(df),
                                            ptr(scr), self.sh), "zkie2_virtual_prove_async")
        pend = self.pend

        def build():
            return VirtualProof(pend.host(hr)[:t * (deg + 1)].reshape(t, deg + 1).copy(), pend.host(hf)[:n].copy())
        build.final = lambda i: (hf, i)  # the folded value of table i: that table at the challenges
        return build

    def fractional(self, num: torch.Tensor, den: torch.Tensor):
        """prove_fractional (logup_gkr.rs:71-81): full_r then cs drawn."""
        lg = _lg(num.numel())
        self.traffic += frac_tree_bytes(lg)
        full_r, cs = self.draw(lg), self.draw(lg)
        h, d = self.pend.out(lib.zkie2_fractional_proof_elems(lg))
        scr = empty(max(lib.zkie2_fractional_scratch_elems(lg), 2))
        check(lib.zkie2_fractional_prove_async(ptr(num), ptr(den), lg, _pp(full_r), _pp(cs), ptr(d), ptr(scr),
                                               self.sh), "zkie2_fractional_prove_async")
        pend = self.pend

        def build():
            a = pend.host(h)
            nr = 2 * lg * (lg - 1)
            layers, off = [], 0
            for l in range(lg):
                t = lg - l - 1
                layers.append(FractionalLayer(full_r[:t].copy(), int(cs[l]) % P,
                                              VirtualProof(a[off:off + 4 * t].reshape(t, 4).copy(),
                                                           a[nr + 7 * l:nr + 7 * l + 7].copy())))
                off += 4 * t
            return FractionalProof(layers, int(a[nr + 7 * lg]), int(a[nr + 7 * lg + 1]), full_r.copy())
        return build

    def ones(self, n: int) -> torch.Tensor:
        o = empty(n)
        check(lib.zkie2_op_fill(ptr(o), n, 1, self.sh), "zkie2_op_fill")
        return o

    def broadcast(self, v: torch.Tensor, m: int, n: int) -> torch.Tensor:
        out = empty(m * n)
        check(lib.zkie2_op_row_broadcast(ptr(v), m, n, ptr(out), self.sh), "zkie2_op_row_broadcast")
        return out

    def eq_table(self, r: np.ndarray) -> torch.Tensor:
        out = empty(1 << r.size)
        check(lib.zkie2_eq_evals(_pp(r), r.size, ptr(out), self.sh), "zkie2_eq_evals")
        return out

    def lookup_fractional(self, idx: torch.Tensor, vals: torch.Tensor, table: torch.Tensor, alpha: int, beta: int):
        """prove_lookup_fractional (logup_gkr.rs:390-401): the merged witness /
        table columns (an index outside the table sets the error word), then
        the fraction tree."""
        n, t = idx.numel(), table.numel()
        total = lib.zkie2_lookup_len(n, t, 0)
        num, den = empty(total), empty(total)
        scr = empty(max(lib.zkie2_lookup_scratch_elems(t), 1))
        self.traffic += 12 * n + 8 * t + 16 * total
        check(lib.zkie2_lookup_num_den_async(idx.data_ptr(), ptr(vals), n, ptr(table), None, t, 0, alpha, beta,
                                             ptr(num), ptr(den), ptr(scr), self.err.data_ptr(), self.sh),
              "zkie2_lookup_num_den_async")
        return self.fractional(num, den)

    def range_table(self, bits: int) -> torch.Tensor:
        """0, 1, .., 2^bits - 1 on the current stream."""
        out = empty(1 << bits)
        check(lib.zkie2_op_iota(ptr(out), 1 << bits, self.sh), "zkie2_op_iota")
        return out

    def upload(self, host: np.ndarray) -> torch.Tensor:
        """A host array (challenges) on the device, copied on the current
        stream from pinned memory both of which live as long as the prover
        (so a recorded graph copies it again on every replay)."""
        pinned = torch.from_numpy(np.ascontiguousarray(host, dtype=np.uint64).view(np.int64)).pin_memory()
        dev = torch.empty(pinned.numel(), dtype=torch.int64, device=device())
        dev.copy_(pinned, non_blocking=True)
        self.keep += [pinned, dev]
        return dev.view(torch.uint64)

    def permutation(self, a: torch.Tensor, b: torch.Tensor, n: int):
        """prove_permutation (logup_gkr.rs:822-840) over the first n values of
        a and b."""
        alpha = self.rng.field()
        total = max(1 << max(n - 1, 0).bit_length(), 32)
        cols = []
        for v in (a, b):
            num, den = empty(total), empty(total)
            check(lib.zkie2_perm_num_den(ptr(v), n, total, alpha, ptr(num), ptr(den), self.sh), "zkie2_perm_num_den")
            cols.append((num, den))
        a_side = self.fractional(*cols[0])
        b_side = self.fractional(*cols[1])
        return lambda: PermutationProof(a_side(), b_side(), int(alpha) % P, a[:n], b[:n])

    # -- the arms --------------------------------------------------------------------------------
    def op_rms_norm(self, op: RmsNorm):
        """prove_rms_norm (rms_norm.rs:97-174) and its lookups (compose.rs:1898-1934)."""
        g = self.store.get
        m, d, nr = op.m, op.d, op.n_real
        x, w = g(op.x), g(op.w)
        f = rms_norm_columns(x, w, g(op.rsqrt_table), m, d, nr, self.err)
        trunc_ch = self.draw(_lg(m))
        trunc = self.virtual([f["ms"], f["rem_s"], f["sum_sq"], self.ones(m)], TRUNC_TERMS(nr, nr // 2), trunc_ch)
        r_out = self.draw(_lg(m * d))
        out = self.virtual([x, self.broadcast(f["rstd"], m, d), w, f["raw"], f["out"], f["rem_out"], self.ones(m * d)],
                           RMS_OUT_TERMS, r_out)
        rsc = self.draw(_lg(m * d))
        rem_split = self.virtual([f["rem_out"], f["rem_lo"], f["rem_hi"]], REM_SPLIT_TERMS, rsc)
        self._lookup(op.rsqrt_table, f["s_index"], f["rstd"], produced_here=True)
        for part in ("rem_lo", "rem_hi"):
            self._lookup(op.limb_table, _index_i32(f[part]), f[part], produced_here=True)
        self.claim(op.out, r_out, out.final(4))
        self.claim(op.w, r_out, out.final(2))
        return lambda: RmsNormProof(trunc(), out(), rem_split(), trunc_ch, r_out, rsc)

    def op_rope(self, op: RoPE):
        """prove_rope (rope.rs:126-196) and its lookups (compose.rs:1935-1967)."""
        g = self.store.get
        x, out = g(op.x), g(op.out)
        n = x.numel()
        cols = [empty(n // 2) for _ in range(8)]  # x_f x_s o_f o_s cos_b sin_b rem_f rem_s
        check(lib.zkie2_op_rope_columns(ptr(x), ptr(out), n, ptr(g(op.cos)), ptr(g(op.sin)), op.m, op.d, op.shift,
                                        (_lib.vp * 8)(*[ptr(c) for c in cols]), self.sh), "zkie2_op_rope_columns")
        x_f, x_s, o_f, o_s, cos_b, sin_b, rem_f, rem_s = cols
        ones = self.ones(n // 2)
        r_f = self.draw(_lg(n // 2))
        first = self.virtual([x_f, cos_b, x_s, sin_b, o_f, rem_f, ones], ROPE_TERMS(op.shift, False), r_f)
        r_s = self.draw(_lg(n // 2))
        second = self.virtual([x_s, cos_b, x_f, sin_b, o_s, rem_s, ones], ROPE_TERMS(op.shift, True), r_s)
        r_out = self.draw(_lg(n))
        for rem in (rem_f, rem_s):
            self._lookup(op.range_table, _index_i32(rem), rem, produced_here=True)
        self.claim(op.out, r_out)
        return lambda: RoPEProof(first(), second(), r_f, r_s, r_out)

    def op_scatter(self, op: Scatter):
        """prove_scatter (scatter.rs:39-55)."""
        sel = self.store.get(op.sel)
        tid, eof = self.store.get_idx(op.token_id), self.store.get_idx(op.expert_of)
        m, n, s_ = op.m, op.n, tid.numel()
        tcnt = _u32(m)
        check(lib.zkie2_op_sel_counts(ptr(sel), m, n, 1, tcnt.data_ptr(), self.sh), "zkie2_op_sel_counts")
        a, b, first = empty(m * n), empty(max(s_, 1)), empty(m)
        check(lib.zkie2_op_scatter_encodings(ptr(sel), m, n, tcnt.data_ptr(), tid.data_ptr(), eof.data_ptr(), s_,
                                             ptr(a), ptr(b), ptr(first), self.err.data_ptr(), self.sh),
              "zkie2_op_scatter_encodings")
        perm = self.permutation(a, b, s_)
        return lambda: ScatterProof(perm())

    def op_gather(self, op: Gather):
        """prove_scatter_add (gather.rs:54-157)."""
        g = self.store.get
        wt, tid, gate, out = g(op.weighted), self.store.get_idx(op.token_id), g(op.gate), g(op.out)
        m, h, s_ = op.m, op.h, tid.numel()
        alpha = int(self.rng.field()) % P
        gamma = self.draw(h)
        gd = self.upload(gamma)
        st, tt = 1 << max(s_ * h - 1, 0).bit_length(), 1 << max(m * h - 1, 0).bit_length()
        src = [empty(st) for _ in range(5)]  # num den gamma_b gate_b w_pad
        check(lib.zkie2_scatter_add_columns(ptr(wt), ptr(gate), tid.data_ptr(), ptr(gd), s_, h, st, alpha,
                                            (_lib.vp * 5)(*[ptr(c) for c in src]), self.sh),
              "zkie2_scatter_add_columns")
        tgt = [empty(tt) for _ in range(4)]  # num den gamma_b o_pad
        check(lib.zkie2_scatter_add_columns(ptr(out), None, None, ptr(gd), m, h, tt, alpha,
                                            (_lib.vp * 5)(ptr(tgt[0]), ptr(tgt[1]), ptr(tgt[2]), None, ptr(tgt[3])),
                                            self.sh), "zkie2_scatter_add_columns")
        source_side = self.fractional(src[0], src[1])
        target_side = self.fractional(tgt[0], tgt[1])
        r_ps = self.draw(_lg(st))
        prod_source = self.virtual([self.eq_table(r_ps), src[0], src[2], src[4], src[3]], SCATTER_ADD_SOURCE_TERMS,
                                   r_ps)
        r_pt = self.draw(_lg(tt))
        prod_target = self.virtual([self.eq_table(r_pt), tgt[0], tgt[2], tgt[3]], SCATTER_ADD_TARGET_TERMS, r_pt)
        return lambda: ScatterAddProof(source_side(), target_side(), alpha, gamma, src[0], src[1], tgt[0], tgt[1],
                                       prod_source(), prod_target(), r_ps, r_pt, wt, gate, out, tid)

    def op_batched_matmul(self, op: BatchedMatMul):
        """The Op::BatchedMatMul arm (compose.rs:1668-1681, batched_matmul.rs:51-83):
        w contracted with eq(v) (one partial evaluation), the eq-selector
        sumcheck; a, w and c claimed at ch, v || ch and v || u."""
        g = self.store.get
        a, w, c = g(op.a), g(op.w), g(op.c)
        s_, k, n = op.s, op.k, op.n
        ls, lk, ln = _lg(s_), _lg(k), _lg(n)
        u, v, ch = self.draw(ls), self.draw(ln), self.draw(ls + lk)
        self.traffic += 8 * (s_ * k * n + 3 * s_ * k + s_ * n)
        w_v = empty(s_ * k)
        scr = empty(max(lib.zkie2_mle_scratch_elems(ls + lk + ln), 1))
        check(lib.zkie2_mle_partial_eval(ptr(w), ls + lk + ln, _pp(v), ln, ptr(w_v), ptr(scr), self.sh),
              "zkie2_mle_partial_eval")
        claimed = self.eval(c, np.concatenate([v, u]))
        sc = self.virtual([a, w_v, self.broadcast(self.eq_table(u), s_, k)], BMM_TERMS, ch)
        self.claim(op.a, ch, sc.final(0))
        self.claim(op.w, np.concatenate([v, ch]), sc.final(1))
        self.claim(op.c, np.concatenate([v, u]), claimed)
        pend = self.pend
        return lambda: BatchedMatMulOpProof(pend.value(claimed), sc(), u, v, ch)

    def op_gather_matmul(self, op: GatherMatMul):
        """prove_gather_matmul (batched_matmul.rs:469-494, prove_streaming
        :359-390; compose.rs:1682-1705): the experts' weights contracted with
        eq(v) once (a partial evaluation over every expert), gathered per
        position, the eq-selector sumcheck, and the per-expert counts and
        table openings."""
        g = self.store.get
        a, eof, w, c = g(op.a), self.store.get_idx(op.expert_of), g(op.w), g(op.c)
        s_, k, n, ne = op.s, op.k, op.n, op.n_experts
        ls, lk, ln = _lg(s_), _lg(k), _lg(n)
        u, v, ch = self.draw(ls), self.draw(ln), self.draw(ls + lk)
        self.traffic += 8 * (ne * k * n + 3 * s_ * k + s_ * n)
        wv = empty(ne * k)
        scr = empty(max(lib.zkie2_mle_scratch_elems(lk + ln), 1))
        for e in range(ne):  # expert blocks are powers of two; the expert count need not be
            check(lib.zkie2_mle_partial_eval(ptr(w[e * k * n:(e + 1) * k * n]), lk + ln, _pp(v), ln,
                                             ptr(wv[e * k:(e + 1) * k]), ptr(scr), self.sh), "zkie2_mle_partial_eval")
        w_v = empty(s_ * k)
        check(lib.zkie2_expert_rows(ptr(wv), eof.data_ptr(), s_, k, ne, ptr(w_v), self.err.data_ptr(), self.sh),
              "zkie2_expert_rows")
        claimed = self.eval(c, np.concatenate([v, u]))
        sc = self.virtual([a, w_v, self.broadcast(self.eq_table(u), s_, k)], BMM_TERMS, ch)
        hc, dc = self.pend.out(ne)
        ht, dt = self.pend.out(ne)
        eq_pos, eq_d = self.eq_table(ch[lk:]), self.eq_table(ch[:lk])  # both alive across the call
        check(lib.zkie2_expert_open(eof.data_ptr(), s_, ptr(eq_pos), ptr(wv), k, ptr(eq_d), ne, ptr(dc), ptr(dt),
                                    self.sh), "zkie2_expert_open")
        self.claim(op.a, ch, sc.final(0))
        self.claim(op.c, np.concatenate([v, u]), claimed)
        pend = self.pend
        return lambda: GatherMatMulOpProof(pend.value(claimed), sc(), pend.host(hc)[:ne].copy(),
                                           pend.host(ht)[:ne].copy(), u, v, ch)

    def op_topk(self, op):
        """prove_topk (topk.rs:82-176) for Op::TopKSelect (range_bits 22,
        compose.rs:1968-1996) and, with k = 1, prove_argmax (topk.rs:299-318)
        for Op::Argmax (range_bits 16, compose.rs:1997-2025); x, sel and gate
        claimed at r from the gate relation's folded tables."""
        g = self.store.get
        argmax = op.kind == "Argmax"
        m, n = op.m, op.n
        k, rb, mn = (1, 16, m * n) if argmax else (op.k, 22, m * n)
        x, sel, thr, gate, d1, d2 = (g(t) for t in (op.x, op.sel, op.thr, op.gate, op.d1, op.d2))
        r = self.draw(_lg(mn))
        gate_rel = self.virtual([x, sel, gate], GATE_TERMS, r)
        thr_b = self.broadcast(thr, m, n)
        d1_rel = self.virtual([sel, x, thr_b, d1], D1_TERMS, r)
        d2_rel = self.virtual([sel, x, thr_b, d2], D2_TERMS, r)
        r_row = self.draw(_lg(m))
        row_sum = self.virtual([sel, self.broadcast(self.eq_table(r_row), m, n)], ROW_SUM_TERMS, r)
        sel_idx, d1_idx, limb_idx = _u32(mn), _u32(mn), _u32(3 * mn)
        limbs = empty(3 * mn)
        check(lib.zkie2_op_topk_limbs(ptr(sel), ptr(d1), ptr(d2), mn, sel_idx.data_ptr(), d1_idx.data_ptr(),
                                      ptr(limbs), limb_idx.data_ptr(), self.sh), "zkie2_op_topk_limbs")
        # the five range lookups are independent: each on a stream of its own
        # behind the columns (which live as long as the prover)
        ready = torch.cuda.Event()
        ready.record(torch.cuda.current_stream())
        self.keep += [sel_idx, d1_idx, limb_idx, limbs]

        def lookup(idx, vals, bits, alpha, beta):
            with self.on(self.next_stream()):
                torch.cuda.current_stream().wait_event(ready)
                return self.lookup_fractional(idx, vals, self.range_table(bits), alpha, beta)
        a_sel, b_sel = self.rng.field(), self.rng.field()
        sel_range = lookup(sel_idx, sel, 1, a_sel, b_sel)
        a_d1, b_d1 = self.rng.field(), self.rng.field()
        d1_range = lookup(d1_idx, d1, rb, a_d1, b_d1)
        ab = [int(v) for v in self.draw(6)]
        parts = [(limb_idx[c * mn:(c + 1) * mn], limbs[c * mn:(c + 1) * mn]) for c in range(3)]
        ranges = [lookup(i, v, 16, ab[2 * c], ab[2 * c + 1]) for c, (i, v) in enumerate(parts)]
        r2 = self.draw(_lg(mn))
        recompose = self.virtual([d2] + [v for _, v in parts], RECOMPOSE_TERMS, r2)
        for i, t in enumerate((op.x, op.sel, op.gate)):
            self.claim(t, r, gate_rel.final(i))
        out = self.store.get_idx(op.out) if argmax else None

        def build():
            dec = RangeDecompProof(ranges[0](), ranges[1](), ranges[2](), recompose(), *ab, r2)
            tk = TopKSelectProof(gate_rel(), d1_rel(), d2_rel(), row_sum(), sel_range(), d1_range(), dec, r, r_row,
                                 int(a_sel), int(b_sel), int(a_d1), int(b_d1), rb, sel)
            return ArgmaxProof(tk, out) if argmax else tk
        return build

    def op_matmul(self, op: MatMul):
        g = self.store.get
        lm, lk, ln = _lg(op.m), _lg(op.k), _lg(op.n)
        u, v, ch = self.draw(lm), self.draw(ln), self.draw(lk)
        h, d = self.pend.out(3 + 3 * lk)
        self.traffic += 8 * (op.m * op.k + op.k * op.n + op.m * op.n)
        scr = empty(max(lib.zkie2_op_matmul_scratch_elems(op.m, op.k, op.n), 1))
        check(lib.zkie2_op_matmul_prove_async(ptr(g(op.a)), ptr(g(op.b)), ptr(g(op.c)), op.m, op.k, op.n, _pp(u),
                                              _pp(v), _pp(ch), ptr(d), ptr(scr), self.sh),
              "zkie2_op_matmul_prove_async")
        # the claims are the proof's own values: f_eval = eval(A, ch||u), h_eval =
        # eval(B, v||ch) (the sumcheck's folded tables), claimed = eval(C, v||u)
        refs = [(h, 1 + 3 * lk), (h, 2 + 3 * lk), (h, 0)]
        for t, pt, ref in zip((op.a, op.b, op.c), (np.concatenate([ch, u]), np.concatenate([v, ch]),
                                                   np.concatenate([v, u])), refs):
            self.claim(t, pt, ref)
        pend = self.pend

        def build():
            a = pend.host(h)
            mm = MatmulProof(int(a[0]), SumcheckProof(a[1:1 + 3 * lk].reshape(lk, 3).copy(), int(a[1 + 3 * lk]),
                                                      int(a[2 + 3 * lk])))
            return OpMatMulProof(mm, u, v, ch, np.array([pend.value(r) for r in refs], dtype=np.uint64))
        return build

    def op_projection(self, op: Projection):
        g = self.store.get
        m, k, n, shift = op.m, op.k, op.n, op.shift
        lm, lk, ln = _lg(m), _lg(k), _lg(n)
        lg = lib.zkie2_projection_lookup_vars(m, n, shift)
        u, v, ch = self.draw(lm), self.draw(ln), self.draw(lk)
        alpha, beta = self.rng.field(), self.rng.field()
        full_r, cs = self.draw(lg), self.draw(lg)
        hbuf = self.store.proj_h.get(op.out)
        # GKR: x, W, h; affine: six tables of m n; lookup columns 2 x 2^lg
        # written, then the fraction tree
        self.traffic += 8 * (m * k + k * n + m * n) + 8 * 6 * m * n + 16 * (1 << lg) + frac_tree_bytes(lg)
        h, d = self.pend.out(lib.zkie2_projection_proof_elems(m, k, n, shift))
        scr = empty(max(lib.zkie2_projection_scratch_elems(m, k, n, shift), 1))
        check(lib.zkie2_projection_prove_async(ptr(g(op.x)), ptr(g(op.w)), ptr(g(op.bias)), ptr(g(op.out)),
                                               ptr(g(op.rem)), ptr(hbuf) if hbuf is not None else None, m, k, n,
                                               shift, _pp(u), _pp(v), _pp(ch), alpha, beta, _pp(full_r), _pp(cs),
                                               ptr(d), self.err.data_ptr(), ptr(scr), self.sh),
              "zkie2_projection_prove_async")
        tv = lm + ln
        o_mm, o_aff = 1, 1 + 3 * lk + 2
        o_fr = o_aff + 3 * tv + 6
        nr = 2 * lg * (lg - 1)
        pt = np.concatenate([v, u])
        # x and W at the GKR sumcheck's folded values, out and bias at the
        # affine sumcheck's finals (tables 3 and 4 at pt)
        self.claim(op.x, np.concatenate([ch, u]), (h, o_mm + 3 * lk))
        self.claim(op.w, np.concatenate([v, ch]), (h, o_mm + 3 * lk + 1))
        self.claim(op.out, pt, (h, o_aff + 3 * tv + 3))
        self.claim(op.bias, pt, (h, o_aff + 3 * tv + 4))
        pend = self.pend

        def build():
            a = pend.host(h)
            mm = MatmulProof(int(a[0]), SumcheckProof(a[o_mm:o_mm + 3 * lk].reshape(lk, 3).copy(),
                                                      int(a[o_mm + 3 * lk]), int(a[o_mm + 3 * lk + 1])))
            aff = VirtualProof(a[o_aff:o_aff + 3 * tv].reshape(tv, 3).copy(), a[o_aff + 3 * tv:o_aff + 3 * tv + 6].copy())
            layers, off = [], 0
            for l in range(lg):
                t = lg - l - 1
                layers.append(FractionalLayer(full_r[:t].copy(), int(cs[l]) % P,
                                              VirtualProof(a[o_fr + off:o_fr + off + 4 * t].reshape(t, 4).copy(),
                                                           a[o_fr + nr + 7 * l:o_fr + nr + 7 * l + 7].copy())))
                off += 4 * t
            base = o_fr + nr + 7 * lg
            frac = FractionalProof(layers, int(a[base]), int(a[base + 1]), full_r.copy())
            return ProjectionProof(mm, aff, frac, int(alpha), int(beta), pt, u, v, ch)
        return build

    def op_add(self, op: Add):
        g = self.store.get
        c = g(op.c)
        r = self.draw(_lg(c.numel()))
        vb = self.virtual([g(op.a), g(op.b), c], ADD_TERMS, r)
        for i, t in enumerate((op.a, op.b, op.c)):
            self.claim(t, r, vb.final(i))
        return lambda: AddProof(vb(), r)

    def _lookup(self, table: int, idx: torch.Tensor, vals: torch.Tensor, produced_here: bool = False):
        """Register a lookup; columns computed by this prover carry an event
        of the stream that wrote them."""
        ev = None
        if produced_here:
            ev = torch.cuda.Event()
            ev.record(torch.cuda.current_stream())
        self.lookups.setdefault(table, []).append((idx, vals, ev))

    def op_softmax(self, op: Softmax):
        g = self.store.get
        m, n = op.m, op.n
        e, out = g(op.e), g(op.out)
        s = empty(m)
        check(lib.zkie2_op_row_sums(ptr(e), m, n, n, ptr(s), self.sh), "zkie2_op_row_sums")
        r_sum = self.draw(_lg(m))
        eq_b = self.broadcast(self.eq_table(r_sum), m, n)
        sum_ch = self.draw(_lg(m * n))
        claimed = self.eval(s, r_sum)
        row_sum = self.virtual([eq_b, e], SOFTMAX_SUM_TERMS, sum_ch)
        sum_b, rem = empty(m * n), empty(m * n)
        check(lib.zkie2_op_softmax_rem(ptr(e), ptr(out), ptr(s), m, n, ptr(sum_b), ptr(rem), self.sh),
              "zkie2_op_softmax_rem")
        r_scale = self.draw(_lg(m * n))
        rescale = self.virtual([out, e, sum_b, rem], SOFTMAX_RESCALE_TERMS, r_scale)
        self.claim(op.out, r_scale, rescale.final(0))
        self._lookup(op.table, self.store.get_idx(op.idx), e)
        pend = self.pend
        return lambda: SoftmaxRoundedProof(row_sum(), rescale(), r_sum, sum_ch, r_scale, pend.value(claimed))

    def op_layernorm(self, op: Layernorm):
        g = self.store.get
        m, d = op.m, op.d
        x, w, b = g(op.x), g(op.w), g(op.b)
        cols = layernorm_columns(x, w, b, g(op.rsqrt_table), m, d)
        r_mean = self.draw(_lg(m))
        eq_b = self.broadcast(self.eq_table(r_mean), m, d)
        mean_claim = self.eval(cols["mean_sq"], r_mean)
        mean_ch = self.draw(_lg(m * d))
        mean_sq = self.virtual([eq_b, x], LN_MEAN_TERMS, mean_ch)
        r_out = self.draw(_lg(m * d))
        out = self.virtual([x, cols["scale"], b, cols["out"]], LN_OUT_TERMS, r_out)
        self._lookup(op.rsqrt_table, cols["idx"], cols["rsqrt"], produced_here=True)
        self.claim(op.out, r_out, out.final(3))
        self.claim(op.w, r_out)
        self.claim(op.b, r_out, out.final(2))
        pend = self.pend
        return lambda: LayernormChainProof(mean_sq(), out(), r_mean, mean_ch, r_out, pend.value(mean_claim))

    def op_layer_norm_centered(self, op: LayerNormCentered):
        g = self.store.get
        m, d, nr = op.m, op.d, op.n_real
        x, w, b = g(op.x), g(op.w), g(op.b)
        f = layer_norm_centered_columns(x, w, b, g(op.rsqrt_table), m, d, nr, self.err)
        lm, lmd = _lg(m), _lg(m * d)
        ones_m = self.ones(m)
        trunc = TRUNC_TERMS(nr, nr // 2)
        r_mean = self.draw(lm)
        self.draw(lmd)  # mean_ch of the discarded mean reduction (:153-159)
        m_ch = self.draw(lm)
        mean = self.virtual([f["mean"], f["rem_mean"], f["sum_mean"], ones_m], trunc, m_ch)
        centered_r = self.draw(lmd)
        centered = self.virtual([x, self.broadcast(f["mean"], m, d), f["centered"]], CENTERED_TERMS, centered_r)
        r_var = self.draw(lm)
        self.draw(lmd)  # var_ch of the discarded variance reduction (:193-201)
        v_ch = self.draw(lm)
        var = self.virtual([f["var"], f["rem_var"], f["sum_var"], ones_m], trunc, v_ch)
        r_out = self.draw(lmd)
        out = self.virtual([f["centered"], self.broadcast(f["rstd"], m, d), w, b, f["raw"], f["out"], f["rem_out"],
                            self.ones(m * d)], LNC_OUT_TERMS, r_out)
        self._lookup(op.rsqrt_table, f["s_index"], f["rstd"], produced_here=True)
        # x at the centering sumcheck's folded x; out, w, b at the output sumcheck's
        self.claim(op.x, centered_r, centered.final(0))
        self.claim(op.out, r_out, out.final(5))
        self.claim(op.w, r_out, out.final(2))
        self.claim(op.b, r_out, out.final(3))
        return lambda: LayerNormCenteredProof(mean(), centered(), var(), out(), r_mean, m_ch, centered_r, r_var,
                                              v_ch, r_out)

    def same_poly(self, f: torch.Tensor, claims):
        """prove_same_poly: coefficients then the merged point drawn; the
        reference's virtual polynomial over [f, eq_1 .. eq_c] proved as f E."""
        t = _lg(f.numel())
        coeffs = self.draw(len(claims))
        merged = self.draw(t)
        pts = np.ascontiguousarray(np.concatenate([np.asarray(pt, dtype=np.uint64) for pt, _ in claims]))
        E = empty(1 << t)
        scr = empty(max(lib.zkie2_eq_combine_scratch_elems(len(claims), t), 1))
        check(lib.zkie2_eq_combine(_pp(pts), _pp(coeffs), len(claims), t, ptr(E), ptr(scr), self.sh),
              "zkie2_eq_combine")
        vb = self.virtual([f, E], PRODUCT_TERMS, merged)
        eq_finals = [_eq_at(pt, merged) for pt, _ in claims]

        def build():
            vp = vb()
            finals = np.array([int(vp.final_evals[0])] + eq_finals, dtype=np.uint64)
            return SamePolyProof(coeffs, VirtualProof(vp.rounds, finals), merged, int(vp.final_evals[0]))
        return build

    def lookup_table(self, table: int):
        """The per-table logUp of prove_shard_precomputed (:2050-2080)."""
        g = self.store.get
        alpha, beta = self.rng.field(), self.rng.field()
        pairs = self.lookups[table]
        for _, _, ev in pairs:
            if ev is not None:
                torch.cuda.current_stream().wait_event(ev)
        x = torch.cat([i.reshape(-1).view(torch.int32) for i, _, _ in pairs]).view(torch.uint32)
        y = _cat_u64([v.reshape(-1) for _, v, _ in pairs])
        n = x.numel()
        total = lib.zkie2_lookup_len(n, 0, 2)
        num, den = empty(total), empty(total)
        check(lib.zkie2_lookup_num_den_async(x.data_ptr(), ptr(y), n, None, None, 0, 2, alpha, beta, ptr(num),
                                             ptr(den), None, self.err.data_ptr(), self.sh),
              "zkie2_lookup_num_den_async")
        x_flat = torch.zeros(total, dtype=torch.uint64, device=num.device)
        y_flat = torch.zeros(total, dtype=torch.uint64, device=num.device)
        x_flat[:n] = (x.view(torch.int32).to(torch.int64) & 0xFFFFFFFF).view(torch.uint64)
        y_flat[:n] = y
        wproof = self.fractional(num, den)
        tab = g(table)
        t = tab.numel()
        mult = empty(max(t, 1))
        for j, (i, _, _) in enumerate(pairs):
            check(lib.zkie2_lookup_multiplicity(i.data_ptr(), i.numel(), t, ptr(mult), 1 if j else 0,
                                                self.err.data_ptr(), self.sh), "zkie2_lookup_multiplicity")
        ttotal = lib.zkie2_lookup_len(0, t, 3)
        tnum, tden = empty(ttotal), empty(ttotal)
        check(lib.zkie2_lookup_num_den_async(None, None, 0, ptr(tab), ptr(mult), t, 3, alpha, beta, ptr(tnum),
                                             ptr(tden), None, self.err.data_ptr(), self.sh),
              "zkie2_lookup_num_den_async")
        tproof = self.fractional(tnum, tden)

        def leaf(p: FractionalProof):
            top = int(p.full_r[-1]) % P
            fe = [int(v) for v in p.layers[0].proof.final_evals]
            return p.full_r.copy(), ((1 - top) * fe[3] + top * fe[4]) % P, ((1 - top) * fe[5] + top * fe[6]) % P

        def build():
            wp, tp = wproof(), tproof()
            pt, nl, dl = leaf(wp)
            tpt, tnl, tdl = leaf(tp)
            return (WitnessColumn(wp, x_flat, y_flat, num, pt, nl, dl, int(alpha), int(beta), table),
                    TableColumn(tp, table, mult[:t], int(alpha), int(beta), tpt, tnl, tdl))
        return build

    # -- the shard ----------------------------------------------------------------------------
    def enqueue(self, ops, boundary=()):
        """Every arm, then the bindings, then the per-table lookups, each
        enqueued on the next of the prover's streams (they are independent
        once the witness exists; the challenges are drawn in the reference's
        order regardless), joined back into the caller's stream and gathered
        into one device array.  Nothing here waits for the device, so the
        whole call can be recorded as a CUDA graph."""
        arms = {"MatMul": self.op_matmul, "Projection": self.op_projection, "Add": self.op_add,
                "Softmax": self.op_softmax, "Layernorm": self.op_layernorm,
                "LayerNormCentered": self.op_layer_norm_centered, "TopKSelect": self.op_topk,
                "Argmax": self.op_topk, "RmsNorm": self.op_rms_norm, "RoPE": self.op_rope, "Scatter": self.op_scatter,
                "Gather": self.op_gather, "GatherMatMul": self.op_gather_matmul,
                "BatchedMatMul": self.op_batched_matmul}
        self.err.zero_()
        start = torch.cuda.Event()
        start.record(self.main)
        for st in self.streams:
            if st is not self.main:
                st.wait_event(start)
        for op in ops:
            k = op.kind
            if k in arms:
                with self.on(self.next_stream()):
                    self.builders.append(arms[k](op))
            elif k == "Lookup":
                self._lookup(op.table, self.store.get_idx(op.idx), self.store.get(op.out))
                self.builders.append(lambda k=k: MarkerProof(k))
            elif k in MARKER_KINDS:
                self.builders.append(lambda k=k: MarkerProof(k))
            else:
                raise ValueError(f"op {k} is not supported")
        by_tensor = {}
        for t, pt, ref in self.claims:
            by_tensor.setdefault(t, []).append((pt, ref))
        bset = set(boundary)
        self.bound, self.bind_builders = [], []
        for t in sorted(by_tensor):
            cs = by_tensor[t]
            if t in bset or len(cs) < 2:
                continue
            with self.on(self.next_stream()):
                self.bind_builders.append(self.same_poly(self.store.get(t), cs))
            self.bound.append(t)
        self.table_builders = []
        for t in sorted(self.lookups):
            with self.on(self.next_stream()):
                self.table_builders.append(self.lookup_table(t))
        self.join()
        self.pend.parts.append(self.err.to(torch.int64).view(torch.uint64))
        self.flat = self.pend.gather()

    def collect(self, host: Optional[np.ndarray] = None) -> OpShardProof:
        """One copy of the results to the host (or the copy ``host`` already
        made of them); the proof objects."""
        self.pend.download(self.flat, host)
        code = int(self.pend.arrays[-1][0])
        if code:
            raise ValueError("prove_shard: " + ", ".join(v for k, v in _ERRORS.items() if code & k))
        op_proofs = [b() for b in self.builders]
        binds = [b() for b in self.bind_builders]
        claims = [(t, pt, self.pend.value(ref)) for t, pt, ref in self.claims]
        cols = [b() for b in self.table_builders]
        return OpShardProof(op_proofs, list(self.bound), binds, claims, [w for w, _ in cols],
                            [tc for _, tc in cols])

    def prove(self, ops, boundary=()) -> OpShardProof:
        self.enqueue(ops, boundary)
        return self.collect()

    def join(self):
        for st in self.streams:
            if st is not self.main:
                ev = torch.cuda.Event()
                ev.record(st)
                self.main.wait_event(ev)


class GraphForward:
    """forward_ops of one statement recorded once as a CUDA graph and
    replayed (the forward's launch sequence depends on the op shapes only,
    once each product's tensor-path choice is fixed).  An eager pass records
    those choices and allocates every output; ``run`` replays the graph and
    reads the error word once: a witness whose products need more byte planes
    than recorded is recomputed by the eager forward.  Graphs with Scatter or
    GatherMatMul (routing read back to the host) stay eager."""

    def __init__(self, store: Store, ops):
        self.store, self.ops = store, list(ops)
        self.plan = _MatmulPlan()
        forward_ops(store, self.ops, plan=self.plan)
        torch.cuda.synchronize()
        self.plan.mode = "replay"
        self.err = _err_word()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.plan.pos = 0
            self.err.zero_()
            forward_ops(store, self.ops, plan=self.plan, err=self.err)
        torch.cuda.synchronize()
        self.fallbacks = 0

    def run(self):
        """The forward for the witness now in the store's inputs."""
        self.graph.replay()
        code = int(self.err.item())
        if code & ERR_PLAN:
            self.fallbacks += 1
            forward_ops(self.store, self.ops)
        elif code:
            raise ValueError("forward_ops: " + ", ".join(v for k, v in _ERRORS.items() if code & k))


class GraphShardProver:
    """prove_shard_precomputed of one statement recorded once as a CUDA graph
    and replayed.  Every challenge of a shard is fixed by the statement (the
    op list and its tensor ids), and every launch's shape by the op shapes, so
    the whole prove -- several thousand launches over the prover's streams
    and the library's fan-out streams -- is the same graph for every witness:
    write new witness values into the store's tensors (same buffers) and call
    ``prove`` again.  ``make_rng`` returns the shard's challenge source at its
    start (e.g. the child transcript); one eager proof warms the library's
    streams and the allocator before the capture.  The device columns of a
    returned proof (x, y, num, multiplicities) live in the graph's memory and
    are overwritten by the next replay."""

    def __init__(self, store: Store, ops, boundary, make_rng, streams: int = 8):
        self.store, self.ops, self.boundary = store, list(ops), list(boundary)
        OpShardProver(store, make_rng(), streams).prove(self.ops, self.boundary)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        self.prover = OpShardProver(store, make_rng(), streams)
        with torch.cuda.graph(self.graph):
            self.prover.main = torch.cuda.current_stream()
            self.prover.sh = stream_handle()
            self.prover.enqueue(self.ops, self.boundary)
        torch.cuda.synchronize()

    def replay(self):
        """Enqueue the recorded prove on the current stream (no host work)."""
        self.graph.replay()

    def prove(self) -> OpShardProof:
        self.replay()
        return self.prover.collect()

    def start(self):
        """Enqueue the recorded prove and, on a side stream behind it, the copy
        of its results into pinned host memory; nothing waits, so the host can
        collect an earlier shard while this one runs."""
        self.graph.replay()
        done = torch.cuda.Event()
        done.record(torch.cuda.current_stream())
        flat = self.prover.flat
        if getattr(self, "_host", None) is None:
            self._host = torch.empty(flat.numel(), dtype=torch.int64).pin_memory()
            self._copy_stream = torch.cuda.Stream()
        self._copy_stream.wait_event(done)
        with torch.cuda.stream(self._copy_stream):
            self._host.copy_(flat.view(torch.int64), non_blocking=True)
        self._copied = torch.cuda.Event()
        self._copied.record(self._copy_stream)

    def finish(self) -> OpShardProof:
        """The proof of the last ``start`` (waits for its copy only)."""
        self._copied.synchronize()
        return self.prover.collect(self._host.numpy().view(np.uint64).copy())


_STREAM_POOLS = {}


def stream_pool(k: int):
    """k side streams of the current device, created once and reused (the
    library keeps its own fan-out streams per caller stream)."""
    pool = _STREAM_POOLS.setdefault(torch.cuda.current_device(), [])
    while len(pool) < k:
        pool.append(torch.cuda.Stream())
    return pool[:k]


def prove_shard_precomputed(store: Store, ops, boundary, rng) -> OpShardProof:
    """compose.rs:1602-2091 (the witness already in ``store``)."""
    return OpShardProver(store, rng).prove(ops, boundary)


def prove_shard(store: Store, ops, boundary, rng) -> OpShardProof:
    """compose.rs:1589-1597: forward, then prove."""
    forward_ops(store, ops)
    return prove_shard_precomputed(store, ops, boundary, rng)


def shard_ranges(op_count: int, ops_per_shard: int):
    """compose.rs:2264-2274."""
    ops_per_shard = max(ops_per_shard, 1)
    return [(s, min(s + ops_per_shard, op_count)) for s in range(0, op_count, ops_per_shard)]


def master_transcript(ops, ops_per_shard: int) -> Transcript:
    """Transcript::new("zkie-shard-dag-v1") + absorb_statement (compose.rs:2276-2287)."""
    t = Transcript(b"zkie-shard-dag-v1")
    t.absorb_u64(ops_per_shard)
    t.absorb_u64(len(ops))
    for op in ops:
        for i in op.reads():
            t.absorb_u64(i)
        for i in op.writes():
            t.absorb_u64(i)
    return t


def prove_shard_dag(store: Store, ops, ops_per_shard: int) -> ShardDagProof:
    """compose.rs:2289-2346: forward once, each shard proven with its child
    transcript (master + the shard index), then the tensors claimed by more
    than one shard bound with the master transcript."""
    forward_ops(store, ops)
    master = master_transcript(ops, ops_per_shard)
    shards = []
    for si, (s, e) in enumerate(shard_ranges(len(ops), ops_per_shard)):
        child = master.clone()
        child.absorb_u64(si)
        shards.append(prove_shard_precomputed(store, ops[s:e], [], child))
    by_tensor, owners = {}, {}
    for si, sh in enumerate(shards):
        for t, pt, ev in sh.claims:
            by_tensor.setdefault(t, []).append((pt, ev))
            owners.setdefault(t, set()).add(si)
    cross = [t for t in sorted(by_tensor) if len(owners[t]) > 1]
    prover = OpShardProver(store, master, streams=1)
    builders = [prover.same_poly(store.get(t), by_tensor[t]) for t in cross]
    prover.pend.fetch()
    return ShardDagProof(shards, cross, [b() for b in builders])
