"""Host-side mirror of zkIE's matmul GKR primitives, backed by libzkie_b200.so.

- ``Transcript``, ``XorShift64``      <- common/transcript.rs:21-80, common/field.rs:17-36
- ``mle_eval / mle_partial_eval / eq_evals`` <- common/mle.rs:8-64
- ``sumcheck_prove`` -> ``SumcheckProof``    <- common/sumcheck.rs:10-89
- ``matmul_prove``   -> ``MatmulProof``      <- common/matmul.rs:17-46
- ``op_matmul_prove``                        <- zkie-ops/src/compose.rs:1724-1747
- ``prove_sum_of_products``                  <- common/sumcheck.rs:243-286
- ``prove_virtual`` -> ``VirtualProof``      <- common/sumcheck.rs:378-438
- ``matmul_fixed`` (forward witness)        <- zkie-ops/src/par.rs:41-89
- ``shard_dag_child``                        <- zkie-ops/src/compose.rs:2276-2311
"""
import ctypes as C
from dataclasses import dataclass, field

import numpy as np
import torch

from . import _lib
from ._lib import check, lib
from .device import empty, ptr, stream_handle, to_dev, to_host


def _arr(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.uint64))


def _p(a: np.ndarray):
    return a.ctypes.data_as(_lib.pu64) if a.size else None


def _lg(n: int) -> int:
    lg = n.bit_length() - 1
    if n != 1 << lg:
        raise ValueError("length must be a power of two")
    return lg


class Transcript:
    """SHA-256 chained Fiat-Shamir transcript."""

    def __init__(self, domain: bytes):
        self.t = _lib.Transcript()
        lib.zkie2_transcript_new(C.byref(self.t), domain, len(domain))

    def clone(self) -> "Transcript":
        c = Transcript.__new__(Transcript)
        c.t = _lib.Transcript()
        C.memmove(C.byref(c.t), C.byref(self.t), C.sizeof(_lib.Transcript))
        return c

    def absorb(self, data: bytes):
        lib.zkie2_transcript_absorb(C.byref(self.t), data, len(data))

    def absorb_u64(self, x: int):
        lib.zkie2_transcript_absorb_u64(C.byref(self.t), x)

    def absorb_field(self, x: int):
        self.absorb_u64(int(x) % 0xFFFFFFFF00000001)

    def field(self) -> int:
        return lib.zkie2_transcript_field(C.byref(self.t))

    def fields(self, n: int) -> np.ndarray:
        out = np.zeros(max(n, 1), dtype=np.uint64)
        lib.zkie2_transcript_fields(C.byref(self.t), n, out.ctypes.data_as(_lib.pu64))
        return out[:n]

    def next_u64(self) -> int:
        return lib.zkie2_transcript_next_u64(C.byref(self.t))

    def field_vec(self, n):
        return np.array([self.field() for _ in range(n)], dtype=np.uint64)

    def challenger(self) -> _lib.Challenger:
        c = _lib.Challenger()
        c.kind = 1
        C.memmove(C.byref(c.transcript), C.byref(self.t), C.sizeof(_lib.Transcript))
        return c

    def sync_from(self, c: _lib.Challenger):
        C.memmove(C.byref(self.t), C.byref(c.transcript), C.sizeof(_lib.Transcript))


class XorShift64:
    """Deterministic test PRNG producing Goldilocks elements."""

    def __init__(self, seed: int):
        self.c = _lib.Challenger()
        lib.zkie2_challenger_xorshift(C.byref(self.c), seed)

    def field(self) -> int:
        return lib.zkie2_challenger_field(C.byref(self.c))

    def fields(self, n: int) -> np.ndarray:
        out = np.zeros(max(n, 1), dtype=np.uint64)
        lib.zkie2_challenger_fields(C.byref(self.c), n, out.ctypes.data_as(_lib.pu64))
        return out[:n]

    def next_u64(self) -> int:
        x = self.c.xorshift_state
        x ^= (x << 13) & 0xFFFFFFFFFFFFFFFF
        x ^= x >> 7
        x ^= (x << 17) & 0xFFFFFFFFFFFFFFFF
        self.c.xorshift_state = x
        return x

    def field_vec(self, n):
        return np.array([self.field() for _ in range(n)], dtype=np.uint64)

    def challenger(self):
        return self.c

    def sync_from(self, c):
        pass


class ShardChild:
    """Child transcript of one shard of prove_shard_dag."""

    def __init__(self, op_ids, ops_per_shard, shard_index):
        ids = _arr(op_ids).reshape(-1)
        self.c = _lib.Challenger()
        lib.zkie2_shard_dag_child(_p(ids), ids.size // 3, ops_per_shard, shard_index, C.byref(self.c))

    def field(self) -> int:
        return lib.zkie2_challenger_field(C.byref(self.c))

    def challenger(self):
        return self.c

    def sync_from(self, c):
        pass


def shard_dag_child(op_ids, ops_per_shard, shard_index) -> ShardChild:
    return ShardChild(op_ids, ops_per_shard, shard_index)


def sha256(data: bytes) -> bytes:
    out = C.create_string_buffer(32)
    lib.zkie2_sha256(data, len(data), out)
    return out.raw


# ---- MLE -------------------------------------------------------------------------------
def eq_evals(r) -> torch.Tensor:
    r = _arr(r)
    out = empty(1 << r.size)
    check(lib.zkie2_eq_evals(_p(r), r.size, ptr(out), stream_handle()), "zkie2_eq_evals")
    return out


def mle_partial_eval(values, fix) -> torch.Tensor:
    d = to_dev(values).reshape(-1)
    fx = _arr(fix)
    t = _lg(d.numel())
    out = empty(d.numel() >> fx.size)
    scr = empty(max(lib.zkie2_mle_scratch_elems(t), 1))
    check(lib.zkie2_mle_partial_eval(ptr(d), t, _p(fx), fx.size, ptr(out), ptr(scr), stream_handle()),
          "zkie2_mle_partial_eval")
    return out


def mle_eval(values, point) -> int:
    d = to_dev(values).reshape(-1)
    pt = _arr(point)
    t = _lg(d.numel())
    if pt.size != t:
        raise ValueError("mle eval: length mismatch")
    scr = empty(max(lib.zkie2_mle_scratch_elems(t), 1))
    out = _lib.u64(0)
    check(lib.zkie2_mle_eval(ptr(d), t, _p(pt), C.byref(out), ptr(scr), stream_handle()), "zkie2_mle_eval")
    return int(out.value)


# ---- sumcheck / matmul -----------------------------------------------------------------
@dataclass
class SumcheckProof:
    rounds: np.ndarray  # (t, 3): c0, c1, c2 per round
    f_eval: int
    h_eval: int


def sumcheck_prove(f, h, claimed_sum, challenges) -> SumcheckProof:
    """sumcheck::prove: the claimed sum is not used by the prover (as in the reference)."""
    df, dh = to_dev(f).reshape(-1), to_dev(h).reshape(-1)
    ch = _arr(challenges)
    t = _lg(df.numel())
    if dh.numel() != df.numel() or ch.size != t:
        raise ValueError("sumcheck: shape mismatch")
    rounds = np.zeros((max(t, 1), 3), dtype=np.uint64)
    finals = np.zeros(2, dtype=np.uint64)
    scr = empty(lib.zkie2_sumcheck_scratch_elems(t))
    check(lib.zkie2_sumcheck_prove(ptr(df), ptr(dh), t, _p(ch), _p(rounds), _p(finals), ptr(scr),
                                   stream_handle()), "zkie2_sumcheck_prove")
    return SumcheckProof(rounds[:t], int(finals[0]), int(finals[1]))


@dataclass
class MatmulProof:
    claimed: int
    sumcheck: SumcheckProof


def matmul_prove(at, b, c, m, k, n, u, v, challenges) -> MatmulProof:
    dat, db, dc = to_dev(at).reshape(-1), to_dev(b).reshape(-1), to_dev(c).reshape(-1)
    u, v, ch = _arr(u), _arr(v), _arr(challenges)
    if dat.numel() != k * m or db.numel() != k * n or dc.numel() != m * n:
        raise ValueError("matmul: shape mismatch")
    lk = _lg(k)
    scr = empty(max(lib.zkie2_matmul_scratch_elems(m, k, n), 1))
    claimed = _lib.u64(0)
    rounds = np.zeros((max(lk, 1), 3), dtype=np.uint64)
    finals = np.zeros(2, dtype=np.uint64)
    check(lib.zkie2_matmul_prove(ptr(dat), ptr(db), ptr(dc), m, k, n, _p(u), _p(v), _p(ch),
                                 C.byref(claimed), _p(rounds), _p(finals), ptr(scr), stream_handle()),
          "zkie2_matmul_prove")
    return MatmulProof(int(claimed.value), SumcheckProof(rounds[:lk], int(finals[0]), int(finals[1])))


@dataclass
class OpMatMulProof:
    """OpProof::MatMul(p, u, v, ch) plus the op's three raw claims."""
    proof: MatmulProof
    u: np.ndarray
    v: np.ndarray
    ch: np.ndarray
    claims: np.ndarray  # eval(A, ch||u), eval(B, v||ch), eval(C, v||u)


def op_matmul_prove(a, b, c, m, k, n, rng) -> OpMatMulProof:
    """Op::MatMul arm; rng is a Transcript, XorShift64 or ShardChild (advanced in place)."""
    da, db, dc = to_dev(a).reshape(-1), to_dev(b).reshape(-1), to_dev(c).reshape(-1)
    lm, lk, ln = _lg(m), _lg(k), _lg(n)
    scr = empty(max(lib.zkie2_op_matmul_scratch_elems(m, k, n), 1))
    ch_obj = rng.challenger()
    u = np.zeros(max(lm, 1), dtype=np.uint64)
    v = np.zeros(max(ln, 1), dtype=np.uint64)
    chv = np.zeros(max(lk, 1), dtype=np.uint64)
    claimed = _lib.u64(0)
    rounds = np.zeros((max(lk, 1), 3), dtype=np.uint64)
    finals = np.zeros(2, dtype=np.uint64)
    claims = np.zeros(3, dtype=np.uint64)
    check(lib.zkie2_op_matmul_prove(ptr(da), ptr(db), ptr(dc), m, k, n, C.byref(ch_obj), _p(u), _p(v), _p(chv),
                                    C.byref(claimed), _p(rounds), _p(finals), _p(claims), ptr(scr),
                                    stream_handle()), "zkie2_op_matmul_prove")
    rng.sync_from(ch_obj)
    proof = MatmulProof(int(claimed.value), SumcheckProof(rounds[:lk], int(finals[0]), int(finals[1])))
    return OpMatMulProof(proof, u[:lm], v[:ln], chv[:lk], claims)


def matmul_field(a, b, m, k, n) -> torch.Tensor:
    da, db = to_dev(a).reshape(-1), to_dev(b).reshape(-1)
    dc = empty(m * n)
    check(lib.zkie2_matmul_field(ptr(da), ptr(db), m, k, n, ptr(dc), stream_handle()), "zkie2_matmul_field")
    return dc


def matmul_fixed(a, b, m, k, n, force_tensor=False):
    """par::mm_par_fixed: the same product as matmul_field, on the tensor cores when
    every input is fixed point of at most 24 bits (and, unless force_tensor, the product has at
    least 2^27 multiply-adds); returns (C on the device, path) with path 0 = tensor
    cores, 1 = the field kernel."""
    da, db = to_dev(a).reshape(-1), to_dev(b).reshape(-1)
    if da.numel() != m * k or db.numel() != k * n:
        raise ValueError("matmul_fixed: shape mismatch")
    dc = empty(m * n)
    scr = empty(max(lib.zkie2_matmul_fixed_scratch_elems(m, k, n), 1))
    path = C.c_uint32(0)
    check(lib.zkie2_matmul_fixed(ptr(da), ptr(db), m, k, n, ptr(dc), 1 if force_tensor else 0, C.byref(path),
                                 ptr(scr), stream_handle()),
          "zkie2_matmul_fixed")
    return dc, int(path.value)


# ---- batch-opening and virtual-polynomial sumchecks -------------------------------------
def _stack(tables) -> torch.Tensor:
    if isinstance(tables, torch.Tensor):
        d = to_dev(tables)
        return d.reshape(1, -1) if d.dim() == 1 else d.reshape(d.shape[0], -1)
    return to_dev(np.stack([np.asarray(x, dtype=np.uint64) for x in tables]))


@dataclass
class SumcheckProofBatch:
    rounds: np.ndarray  # (t, 3): c0, c1, c2 per round
    b_eval: int


def prove_sum_of_products(weights, values, claimed_sum, challenges) -> SumcheckProofBatch:
    """sumcheck::prove_sum_of_products over n tables of 2^t (the claimed sum is
    not used by the prover, as in the reference)."""
    dw, dv = _stack(weights), _stack(values)
    if dw.shape != dv.shape:
        raise ValueError("sum of products: shape mismatch")
    n, t = dw.shape[0], _lg(dw.shape[1])
    ch = _arr(challenges)
    if ch.size != t:
        raise ValueError("challenge count mismatch")
    rounds = np.zeros((max(t, 1), 3), dtype=np.uint64)
    b_eval = _lib.u64(0)
    scr = empty(lib.zkie2_sum_of_products_scratch_elems(n, t))
    check(lib.zkie2_sum_of_products_prove(ptr(dw), ptr(dv), n, t, _p(ch), _p(rounds), C.byref(b_eval), ptr(scr),
                                          stream_handle()), "zkie2_sum_of_products_prove")
    return SumcheckProofBatch(rounds[:t], int(b_eval.value))


@dataclass
class VirtualProof:
    rounds: np.ndarray       # (t, d + 1): the round polynomial's values at 0..d
    final_evals: np.ndarray  # one per MLE


def prove_virtual(mles, terms, claimed, challenges) -> VirtualProof:
    """sumcheck::prove_virtual: mles is a list of 2^t tables, terms a list of
    (coeff, [mle indices]); the claimed sum is not used by the prover."""
    ds = [to_dev(m).reshape(-1) for m in mles]
    if not ds:
        raise ValueError("prove_virtual: no MLEs")
    t = _lg(ds[0].numel())
    if any(d.numel() != ds[0].numel() for d in ds):
        raise ValueError("prove_virtual: MLE length mismatch")
    ch = _arr(challenges)
    if ch.size != t:
        raise ValueError("challenge count mismatch")
    coeffs = np.array([int(c) % 0xFFFFFFFF00000001 for c, _ in terms] or [0], dtype=np.uint64)
    off, idx = [0], []
    for _, ids in terms:
        idx.extend(int(i) for i in ids)
        off.append(len(idx))
    off = np.array(off, dtype=np.uint32)
    idx = np.array(idx or [0], dtype=np.uint32)
    deg = max((len(ids) for _, ids in terms), default=0)
    ptrs = (C.c_void_p * len(ds))(*[ptr(d) for d in ds])
    rounds = np.zeros((max(t, 1), deg + 1), dtype=np.uint64)
    finals = np.zeros(len(ds), dtype=np.uint64)
    scr = empty(max(lib.zkie2_virtual_scratch_elems(len(ds), t), 1))
    check(lib.zkie2_virtual_prove(ptrs, len(ds), t, _p(coeffs), off.ctypes.data_as(_lib.pu32),
                                  idx.ctypes.data_as(_lib.pu32), len(terms), _p(ch), _p(rounds), _p(finals),
                                  ptr(scr), stream_handle()), "zkie2_virtual_prove")
    return VirtualProof(rounds[:t], finals)


# ---- one MatMul shard in one call -------------------------------------------------------
@dataclass
class ShardMatMulProof:
    c: torch.Tensor           # C = A W (device, m x n)
    roots: np.ndarray         # (3, 8): WHIR roots of W, A, C
    proof: OpMatMulProof


class ShardProver:
    """zkie2_shard_prove_matmul with its device scratch kept across calls."""

    def __init__(self, m, k, n):
        self.m, self.k, self.n = m, k, n
        ne = lib.zkie2_shard_prove_matmul_scratch_elems(m, k, n)
        if ne == 0:
            raise ValueError("shard shape: powers of two with >= 32 elements per tensor")
        self.scr = empty(ne)
        self.c = empty(m * n)

    def prove(self, a, w, op_ids=(0, 1, 2), ops_per_shard=1, shard_index=0) -> ShardMatMulProof:
        m, k, n = self.m, self.k, self.n
        da, dw = to_dev(a).reshape(-1), to_dev(w).reshape(-1)
        if da.numel() != m * k or dw.numel() != k * n:
            raise ValueError("shard: shape mismatch")
        lm, lk, ln = _lg(m), _lg(k), _lg(n)
        ids = np.ascontiguousarray(np.asarray(op_ids, dtype=np.uint64))
        roots = np.zeros((3, 8), dtype=np.uint64)
        claimed = _lib.u64(0)
        rounds = np.zeros((max(lk, 1), 3), dtype=np.uint64)
        finals = np.zeros(2, dtype=np.uint64)
        claims = np.zeros(3, dtype=np.uint64)
        check(lib.zkie2_shard_prove_matmul(ptr(da), ptr(dw), m, k, n, _p(ids), ops_per_shard, shard_index,
                                           ptr(self.c), _p(roots), C.byref(claimed), _p(rounds), _p(finals),
                                           _p(claims), ptr(self.scr), stream_handle()), "zkie2_shard_prove_matmul")
        # the challenge draws, replayed on the host for the proof object
        child = shard_dag_child([list(op_ids)], ops_per_shard, shard_index)
        u = np.array([child.field() for _ in range(lm)], dtype=np.uint64)
        v = np.array([child.field() for _ in range(ln)], dtype=np.uint64)
        ch = np.array([child.field() for _ in range(lk)], dtype=np.uint64)
        proof = MatmulProof(int(claimed.value), SumcheckProof(rounds[:lk], int(finals[0]), int(finals[1])))
        return ShardMatMulProof(self.c.view(m, n), roots, OpMatMulProof(proof, u, v, ch, claims))
