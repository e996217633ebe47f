"""Host-side mirror of zkIE's logUp GKR (crates/zkie-core/src/common/logup_gkr.rs),
backed by libzkie_b200.so.  The fraction tree is built and proven on the device,
one layer after another, without leaving HBM; only the round messages and the
final evaluations come back.

- ``prove_fractional_with_challenges``, ``prove_fractional``  <- :29-81
- ``build_lookup_num_den``, ``build_lookup_witness_num_den``,
  ``build_lookup_table_num_den``                               <- :210-240, :261-277, :285-301
- ``lookup_multiplicity``, ``merge_multiplicity``, ``pad_table`` <- :241-260, :278-284
- ``prove_lookup_fractional`` (+ ``_columns``, ``_batch``)     <- :390-417, :458-493
- ``prove_lookup_witness`` (+ ``_batch``, ``_batch_columns``), ``prove_lookup_table`` <- :303-383
- ``fractional_leaf``                                          <- :193-201
"""
import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch

from ._lib import check, lib
from .device import P, device, empty, ptr, stream_handle, to_dev
from .gkr import VirtualProof, _arr, _lg, _p

# column modes of zkie2_lookup_num_den
MERGED, WITNESS, WITNESS_COLUMNS, TABLE = 0, 1, 2, 3


@dataclass
class FractionalLayer:
    r: np.ndarray        # full_r[: lg n - layer - 1]: the eq point and the sumcheck challenges
    c: int               # the layer's batching challenge
    proof: VirtualProof  # rounds (t, 4), final_evals (7)


@dataclass
class FractionalProof:
    layers: list
    final_num: int
    final_den: int
    full_r: np.ndarray


def prove_fractional_with_challenges(num, den, full_r, cs) -> FractionalProof:
    """Prove sum_i num[i] / den[i] with the fraction tree; num and den are 2^k
    field elements (device tensors or host arrays), full_r and cs k challenges."""
    dn, dd = to_dev(num).reshape(-1), to_dev(den).reshape(-1)
    if dn.numel() != dd.numel():
        raise ValueError("prove_fractional: num and den lengths differ")
    lg = _lg(dn.numel())
    full_r, cs = _arr(full_r).reshape(-1), _arr(cs).reshape(-1)
    if full_r.size != lg or cs.size != lg:
        raise ValueError("prove_fractional: need one full_r and one c per variable")
    rounds = np.zeros(max(2 * lg * (lg - 1), 1), dtype=np.uint64)
    finals = np.zeros(max(7 * lg, 1), dtype=np.uint64)
    fnd = np.zeros(2, dtype=np.uint64)
    scr = empty(max(lib.zkie2_fractional_scratch_elems(lg), 2))
    check(lib.zkie2_fractional_prove(ptr(dn), ptr(dd), lg, _p(full_r), _p(cs), _p(rounds), _p(finals), _p(fnd),
                                     ptr(scr), stream_handle()), "zkie2_fractional_prove")
    layers, off = [], 0
    for layer in range(lg):
        t = lg - layer - 1
        rd = rounds[off:off + 4 * t].reshape(t, 4).copy()
        layers.append(FractionalLayer(full_r[:t].copy(), int(cs[layer]) % P,
                                      VirtualProof(rd, finals[7 * layer:7 * layer + 7].copy())))
        off += 4 * t
    return FractionalProof(layers, int(fnd[0]), int(fnd[1]), full_r.copy())


def prove_fractional(num, den, rng) -> FractionalProof:
    """Draws full_r then cs (one per variable each) from the challenge source."""
    n = num.numel() if isinstance(num, torch.Tensor) else len(num)
    lg = _lg(n)
    full_r = [rng.field() for _ in range(lg)]
    cs = [rng.field() for _ in range(lg)]
    return prove_fractional_with_challenges(num, den, full_r, cs)


def fractional_leaf(proof: FractionalProof):
    """(full_r, num_0(full_r), den_0(full_r)) from the first layer's final
    evaluations, folding the peeled top variable."""
    top = int(proof.full_r[-1]) % P
    fe = [int(v) for v in proof.layers[0].proof.final_evals]
    one_m = (1 - top) % P
    return proof.full_r.copy(), (one_m * fe[3] + top * fe[4]) % P, (one_m * fe[5] + top * fe[6]) % P


# ---- lookup columns ---------------------------------------------------------------------
def _u32_dev(x) -> torch.Tensor:
    if isinstance(x, torch.Tensor):
        return x.to(device(), torch.uint32).contiguous().reshape(-1)
    arr = np.ascontiguousarray(np.asarray(x, dtype=np.uint32)).reshape(-1)
    return torch.from_numpy(arr).to(device())


def _concat(parts, to):
    parts = [to(p) for p in parts]
    if not parts:
        return to(np.zeros(0))
    return torch.cat(parts) if len(parts) > 1 else parts[0]


def _columns(x, y, table, m, mode, alpha, beta):
    dx = _u32_dev(x if x is not None else np.zeros(0))
    dy = to_dev(y if y is not None else np.zeros(0)).reshape(-1)
    dt = to_dev(table if table is not None else np.zeros(0)).reshape(-1)
    dm = to_dev(m if m is not None else np.zeros(0)).reshape(-1)
    n = dx.numel() if mode != TABLE else 0
    if mode != TABLE and dy.numel() != n:
        raise ValueError("lookup: x and y lengths differ")
    t = dt.numel()
    if mode == TABLE and dm.numel() != t:
        raise ValueError("lookup: multiplicity and table lengths differ")
    total = lib.zkie2_lookup_len(n, t, mode)
    num, den = empty(total), empty(total)
    scr = empty(lib.zkie2_lookup_scratch_elems(t))
    check(lib.zkie2_lookup_num_den(dx.data_ptr() if n else None, ptr(dy) if n else None, n,
                                   ptr(dt) if t else None, ptr(dm) if (mode == TABLE and t) else None, t, mode,
                                   int(alpha) % P, int(beta) % P, ptr(num), ptr(den), ptr(scr), stream_handle()),
          "zkie2_lookup_num_den")
    return num, den


def build_lookup_num_den(x, y, table, alpha, beta):
    """Merged columns: n witness fractions 1 / (alpha + x_i + beta y_i), then t
    table fractions -m_j / (alpha + j + beta table_j), then 0 / 1 up to a power of two."""
    return _columns(x, y, table, None, MERGED, alpha, beta)


def build_lookup_witness_num_den(x, y, alpha, beta):
    return _columns(x, y, None, None, WITNESS, alpha, beta)


def build_lookup_table_num_den(m, table, alpha, beta):
    return _columns(None, None, table, m, TABLE, alpha, beta)


def lookup_multiplicity(x, t) -> np.ndarray:
    x = np.asarray(x.cpu() if isinstance(x, torch.Tensor) else x, dtype=np.int64).reshape(-1)
    if x.size and (x.min() < 0 or x.max() >= t):
        raise ValueError("lookup_multiplicity: index outside the table")
    return np.bincount(x, minlength=t).astype(np.uint64) if x.size else np.zeros(t, dtype=np.uint64)


def merge_multiplicity(xs, t) -> np.ndarray:
    m = np.zeros(t, dtype=np.uint64)
    for x in xs:
        m += lookup_multiplicity(x, t)
    return m


def pad_table(table) -> np.ndarray:
    tb = _arr(table).reshape(-1)
    n = 1 << max(tb.size - 1, 0).bit_length() if tb.size else 1
    out = np.zeros(n, dtype=np.uint64)
    out[:tb.size] = tb
    return out


def prove_lookup_fractional(x, y, table, alpha, beta, rng) -> FractionalProof:
    num, den = build_lookup_num_den(x, y, table, alpha, beta)
    return prove_fractional(num, den, rng)


def prove_lookup_fractional_columns(x, y, table, alpha, beta, rng):
    num, den = build_lookup_num_den(x, y, table, alpha, beta)
    return prove_fractional(num, den, rng), num, den


def prove_lookup_fractional_batch(xs, ys, table, alpha, beta, rng) -> FractionalProof:
    """Several lookups into the same table as one fraction tree: the witness
    fractions of every list in order, then the table with merged multiplicities."""
    if len(xs) != len(ys):
        raise ValueError("lookup batch: xs and ys differ in length")
    num, den = build_lookup_num_den(_concat(xs, _u32_dev), _concat(ys, lambda v: to_dev(v).reshape(-1)), table,
                                    alpha, beta)
    return prove_fractional(num, den, rng)


def prove_lookup_witness(x, y, alpha, beta, rng) -> FractionalProof:
    num, den = build_lookup_witness_num_den(x, y, alpha, beta)
    return prove_fractional(num, den, rng)


def prove_lookup_witness_batch(xs, ys, alpha, beta, rng) -> FractionalProof:
    if len(xs) != len(ys):
        raise ValueError("lookup batch: xs and ys differ in length")
    num, den = build_lookup_witness_num_den(_concat(xs, _u32_dev), _concat(ys, lambda v: to_dev(v).reshape(-1)),
                                            alpha, beta)
    return prove_fractional(num, den, rng)


def prove_lookup_witness_batch_columns(xs, ys, alpha, beta, rng):
    """(proof, x_flat, y_flat, num, den): the witness side as committed
    columns, at least 32 rows, padding rows x = y = 0, num = 0, den = alpha."""
    if len(xs) != len(ys):
        raise ValueError("lookup batch: xs and ys differ in length")
    dx = _concat(xs, _u32_dev)
    dy = _concat(ys, lambda v: to_dev(v).reshape(-1))
    num, den = _columns(dx, dy, None, None, WITNESS_COLUMNS, alpha, beta)
    total, n = num.numel(), dx.numel()
    x_flat = torch.zeros(total, dtype=torch.uint64, device=num.device)
    y_flat = torch.zeros(total, dtype=torch.uint64, device=num.device)
    if n:
        x_flat[:n] = dx.to(torch.int64).to(torch.uint64)
        y_flat[:n] = dy
    return prove_fractional(num, den, rng), x_flat, y_flat, num, den


def prove_lookup_table(m, table, alpha, beta, rng) -> FractionalProof:
    num, den = build_lookup_table_num_den(m, table, alpha, beta)
    return prove_fractional(num, den, rng)
