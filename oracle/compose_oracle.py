"""CPU restatement of zkie-ops' shard prover for the op arms of a GPT-2 layer.

Test infrastructure, never part of the product: only tests/, smoke() and
bench.py's CPU legs import it.  It restates, over the oracle's field,
sumcheck and fraction-tree primitives (oracle.py over zkie_oracle.c) and
numpy's wrapping int64 arithmetic (the reference's i64 arithmetic in a
release build):

- fixed_point.rs to_i64 / from_i64 (:53-70) and compose.rs round_div (:103-111)
- forward_ops (compose.rs:1174-1583) for the arms a GPT-2 layer uses:
  Transpose, Scale, MatMul, Projection, Add, Lookup, Softmax, SoftmaxIndex,
  GeluIndex, StableSoftmaxIndex, Layernorm, LayerNormCentered, TopKSelect, Argmax
- rsqrt_index (compose.rs:884-896), layer_norm_forward and
  prove_layer_norm_centered (layer_norm_centered.rs:42-245)
- prove_layernorm_chain (layernorm_chain.rs:24-93)
- prove_softmax_rounded (softmax_scaled.rs:42-108)
- prove_same_poly (common/same_poly.rs:13-45)
- prove_lookup_witness_batch_columns, merge_multiplicity, prove_lookup_table,
  prove_fractional, fractional_leaf (common/logup_gkr.rs:71-81, 193-201,
  251-260, 340-383)
- prove_shard_precomputed (compose.rs:1602-2091), prove_shard (:1589-1597),
  absorb_statement and prove_shard_dag (:2276-2346)

Ops are read by duck typing (``op.kind`` and the field names of the
reference's Op enum); the store is a HostStore of numpy arrays.  Proofs come
back as nested tuples of ints and numpy arrays, the layout the product's
``canonical()`` methods produce, so a test compares the two directly.
"""
import numpy as np

from . import oracle as o

P = 0xFFFFFFFF00000001
NEG = P - 1
I64_MAX = 0x7FFFFFFFFFFFFFFF


class HostStore:
    """compose.rs Store: field tensors ``v`` and index tensors ``idx``."""

    def __init__(self):
        self.v = []
        self.idx = []

    def push(self, t):
        self.v.append(None if t is None else o.u64(t).reshape(-1))
        return len(self.v) - 1

    def push_idx(self, t):
        self.idx.append(None if t is None else np.asarray(t, dtype=np.uint32).reshape(-1))
        return len(self.idx) - 1

    def get(self, t):
        return self.v[t]


# ---- fixed point (fixed_point.rs:53-70, compose.rs:103-111) -----------------------------
def to_i64(v):
    v = np.asarray(v, dtype=np.uint64) % np.uint64(P)
    neg = v > np.uint64(I64_MAX)
    out = v.astype(np.int64)
    out[neg] = -((np.uint64(P) - v[neg]).astype(np.int64))
    return out


def from_i64(x):
    x = np.asarray(x, dtype=np.int64)
    u = x.astype(np.uint64)
    neg = x < 0
    out = u.copy()
    # P - |x| with |x| = 0 - u (mod 2^64), also for i64::MIN
    out[neg] = np.uint64(P) - (np.uint64(0) - u[neg])
    return out


def round_div(a, b):
    """q = a.div_euclid(b), r = a.rem_euclid(b), q + 1 when 2 r >= b (wrapping)."""
    a = np.asarray(a, dtype=np.int64)
    b = np.broadcast_to(np.asarray(b, dtype=np.int64), a.shape)
    if (b == 0).any():
        raise ZeroDivisionError("round_div by zero")
    with np.errstate(over="ignore"):
        ab = np.abs(b)
        q = a // ab
        r = a - q * ab
        q = np.where(b < 0, -q, q)
        return np.where(r * 2 >= b, q + 1, q)


def rsqrt_index(var):
    """compose.rs:884-896 on an int64 array."""
    fine, coarse = 1 << 20, 1 << 22
    coarse_end = fine + coarse * (1 << 8)
    raw = round_div(var, 1 << 18)
    with np.errstate(over="ignore"):
        out = np.where(raw < fine, np.maximum(raw, 0),
                       np.where(raw < coarse_end, fine + ((raw - fine) >> 8),
                                fine + coarse + ((raw - coarse_end) >> 16)))
    return (out.astype(np.int64).astype(np.uint64) & np.uint64(0xFFFFFFFF)).astype(np.uint32)


def _lg(n):
    n = int(n)
    if n <= 0 or n & (n - 1):
        raise ValueError(f"{n} is not a power of two")
    return n.bit_length() - 1


def _draw(rng, n):
    return np.array([rng.field() for _ in range(n)], dtype=np.uint64)


def _rows(v, m, d):
    """v[r] broadcast over the d columns of row r."""
    return np.repeat(o.u64(v).reshape(-1), d)


def _gather(table, idx):
    idx = np.asarray(idx, dtype=np.int64)
    if idx.size and idx.max() >= table.size:
        raise IndexError("lookup index outside the table")
    return table[idx]


# ---- forward (compose.rs:1174-1583) --------------------------------------------------------
def layer_norm_forward(x, w, b, table, m, d, n_real):
    """layer_norm_centered.rs:42-120 -> dict of its eleven outputs."""
    x = o.u64(x).reshape(-1)
    xi = to_i64(x).reshape(m, d)
    with np.errstate(over="ignore"):
        s = xi[:, :n_real].sum(axis=1)
    mean = from_i64(round_div(s, n_real))
    centered = o.vec_sub(x, _rows(mean, m, d))
    c = to_i64(centered).reshape(m, d)[:, :n_real]
    with np.errstate(over="ignore"):
        sq = (c * c).sum(axis=1)
    var = from_i64(round_div(sq, n_real))
    s_index = rsqrt_index(to_i64(var))
    if s_index.size and int(s_index.max()) >= table.size:
        raise IndexError("rsqrt table too short for the forward pass")
    rstd = table[s_index.astype(np.int64)]
    raw = o.vec_mul(o.vec_mul(centered, _rows(rstd, m, d)), w)
    bi = to_i64(b)
    out = from_i64(round_div(to_i64(raw), 1 << 32) + bi)
    with np.errstate(over="ignore"):
        rem_out = from_i64(to_i64(raw) - (to_i64(out) - bi) * (1 << 32) + (1 << 31))
        sum_mean = o.row_sums(x, m, d, n_real)
        rem_mean = from_i64(to_i64(sum_mean) - to_i64(mean) * n_real + n_real // 2)
        sum_var = o.row_sums(o.vec_mul(centered, centered), m, d, n_real)
        rem_var = from_i64(to_i64(sum_var) - to_i64(var) * n_real + n_real // 2)
    return dict(mean=mean, centered=centered, var=var, s_index=s_index, rstd=rstd, raw=raw, out=out,
                rem_out=rem_out, sum_mean=sum_mean, rem_mean=rem_mean, sum_var=sum_var, rem_var=rem_var)


def layernorm_forward(x, w, b, table, m, d):
    """The Layernorm arm's forward (compose.rs:1467-1496, layernorm_chain.rs:34-44)."""
    x = o.u64(x).reshape(-1)
    mean_sq = o.row_sums(o.vec_mul(x, x), m, d, d)
    idx = (np.maximum(to_i64(mean_sq), 0).astype(np.uint64) % np.uint64(table.size)).astype(np.uint32)
    rsqrt = table[idx.astype(np.int64)]
    scale = o.vec_mul(_rows(rsqrt, m, d), w)
    out = o.vec_add(o.vec_mul(x, scale), b)
    return dict(mean_sq=mean_sq, idx=idx, rsqrt=rsqrt, scale=scale, out=out)


def softmax_forward(idx, table, m, n):
    e = _gather(table, idx)
    s = o.row_sums(e, m, n, n)
    out = from_i64(round_div(to_i64(e) * (1 << 16), np.repeat(to_i64(s), n)))
    return e, out, s


def forward_ops(store, ops):
    for op in ops:
        k = op.kind
        g = store.get
        if k == "Transpose":
            store.v[op.out] = np.ascontiguousarray(g(op.x).reshape(op.m, op.k).T).reshape(-1)
        elif k == "Scale":
            with np.errstate(over="ignore"):
                store.v[op.out] = from_i64(round_div(to_i64(g(op.x)) * np.int64(op.factor), 1 << op.shift))
        elif k == "MatMul":
            store.v[op.c] = o.matmul_fixed(g(op.a).reshape(op.m, op.k), g(op.b).reshape(op.k, op.n)).reshape(-1)
        elif k == "Projection":
            h = to_i64(o.matmul_fixed(g(op.x).reshape(op.m, op.k), g(op.w).reshape(op.k, op.n)).reshape(-1))
            bi = to_i64(g(op.bias))
            out = from_i64(round_div(h, 1 << op.shift) + bi)
            with np.errstate(over="ignore"):
                rem = from_i64(h - (to_i64(out) - bi) * (1 << op.shift) + (1 << (op.shift - 1)))
            store.v[op.out], store.v[op.rem] = out, rem
        elif k == "Add":
            store.v[op.c] = o.vec_add(g(op.a), g(op.b))
        elif k == "Lookup":
            store.v[op.out] = _gather(g(op.table), store.idx[op.idx])
        elif k == "Softmax":
            e, out, _ = softmax_forward(store.idx[op.idx], g(op.table), op.m, op.n)
            store.v[op.e], store.v[op.out] = e, out
        elif k == "SoftmaxIndex":
            v = np.maximum(to_i64(g(op.x)), 0).astype(np.uint64)
            store.idx[op.out] = (v % np.uint64(op.table_len)).astype(np.uint32)
        elif k == "GeluIndex":
            with np.errstate(over="ignore"):
                v = to_i64(g(op.x)) + np.int64(op.offset)
            store.idx[op.out] = np.clip(v, 0, op.table_len - 1).astype(np.uint32)
        elif k == "StableSoftmaxIndex":
            masked = to_i64(o.vec_add(g(op.x), g(op.mask))).reshape(op.m, op.n)
            row_max = masked.max(axis=1, keepdims=True)
            with np.errstate(over="ignore"):
                v = (masked - row_max + np.int64(op.offset)).reshape(-1)
            store.idx[op.out] = np.clip(v, 0, op.table_len - 1).astype(np.uint32)
        elif k == "Layernorm":
            store.v[op.out] = layernorm_forward(g(op.x), g(op.w), g(op.b), g(op.rsqrt_table), op.m, op.d)["out"]
        elif k == "LayerNormCentered":
            store.v[op.out] = layer_norm_forward(g(op.x), g(op.w), g(op.b), g(op.rsqrt_table), op.m, op.d,
                                                 op.n_real)["out"]
        elif k == "ScaleVec":  # compose.rs:1193-1212
            x, sv = g(op.x), g(op.scale)
            sc = np.resize(to_i64(sv), x.size)
            with np.errstate(over="ignore"):
                store.v[op.out] = from_i64(round_div(to_i64(x) * sc, 1 << op.shift))
        elif k == "BroadcastScale":  # :1284-1293
            store.v[op.out] = o.vec_mul(g(op.x), np.repeat(g(op.scale), op.h)[:g(op.x).size])
        elif k == "IdxBroadcast":  # :1258-1267
            base = store.idx[op.base].astype(np.uint64)
            v = base[:, None] * np.uint64(op.b) + np.arange(op.b, dtype=np.uint64)[None, :]
            store.idx[op.out] = (v & np.uint64(0xFFFFFFFF)).astype(np.uint32).reshape(-1)
        elif k == "CombineIdx":  # :1268-1278
            a, b = store.idx[op.a].astype(np.uint64), store.idx[op.b].astype(np.uint64)
            if a.size != b.size:
                raise ValueError("CombineIdx: lengths differ")
            store.idx[op.out] = ((a * np.uint64(op.scale) + b) & np.uint64(0xFFFFFFFF)).astype(np.uint32)
        elif k == "PadIdx":  # :1279-1283
            out = np.zeros(op.len, dtype=np.uint32)
            base = store.idx[op.base][:op.len]
            out[:base.size] = base
            store.idx[op.out] = out
        elif k == "ScaleGate":  # :1294-1318
            x, gv = g(op.x), to_i64(g(op.gate))
            sc = gv[(np.arange(x.size) // op.h) * op.n + op.col]
            with np.errstate(over="ignore"):
                store.v[op.out] = from_i64(round_div(to_i64(x) * sc, 1 << op.shift))
        elif k == "Relu":  # :1319-1326
            x = g(op.x)
            store.v[op.out] = np.where(to_i64(x) > 0, x % np.uint64(P), np.uint64(0)).astype(np.uint64)
        elif k == "BatchedMatMul":  # :1241-1244
            store.v[op.c] = batched_matmul_forward(g(op.a), g(op.w), op.s, op.k, op.n)
        elif k == "Scatter":  # :1213-1223
            store.idx[op.token_id], store.idx[op.expert_of] = scatter_forward(g(op.sel), op.m, op.n)
        elif k == "Gather":  # :1224-1240
            store.v[op.out] = gather_forward(g(op.weighted), store.idx[op.token_id], g(op.gate), op.m, op.h)
        elif k == "GatherMatMul":  # :1245-1257
            store.v[op.c] = gather_matmul_forward(g(op.a), store.idx[op.expert_of], g(op.w), op.s, op.k, op.n,
                                                  op.n_experts)
        elif k == "RmsNorm":  # :1509-1528
            store.v[op.out] = rms_norm_forward(g(op.x), g(op.w), g(op.rsqrt_table), op.m, op.d, op.n_real)["out"]
        elif k == "RoPE":  # :1529-1542
            store.v[op.out] = rope_forward(g(op.x), g(op.cos), g(op.sin), op.m, op.d, op.shift)[0]
        elif k == "TopKSelect":
            (store.v[op.thr], store.v[op.sel], store.v[op.gate], store.v[op.d1],
             store.v[op.d2]) = topk_forward(g(op.x), op.m, op.n, op.k)
        elif k == "Argmax":
            (store.v[op.thr], store.v[op.sel], store.v[op.gate], store.v[op.d1], store.v[op.d2],
             store.idx[op.out]) = argmax_forward(g(op.x), op.m, op.n)
        else:
            raise ValueError(f"op {k} is not restated")


# ---- top-k selection and argmax (topk.rs) ------------------------------------------------
GATE_TERMS = [(1, [0, 1]), (NEG, [2])]
D1_TERMS = [(1, [0, 1]), (NEG, [0, 2]), (NEG, [3])]
D2_TERMS = [(1, [2]), (NEG, [1]), (NEG, [0, 2]), (1, [0, 1]), (NEG, [3])]
ROW_SUM_TERMS = [(1, [0, 1])]
RECOMPOSE_TERMS = [(1, [0]), (NEG, [1]), (NEG * (1 << 16) % P, [2]), (NEG * (1 << 32) % P, [3])]


def topk_forward(x, m, n, k):
    """topk.rs:41-80 -> (thr, sel, gate, d1, d2): per row the entries ordered
    by value (to_i64) descending, ties by position ascending; the first k
    selected, thr the k-th; gate = x sel, d1 = sel (x - thr), d2 = (1 - sel)
    (thr - x) in wrapping i64."""
    xv = o.u64(x).reshape(m, n) % np.uint64(P)
    xi = to_i64(xv.reshape(-1)).reshape(m, n)
    order = np.argsort(~xi, axis=1, kind="stable")  # ~v = -v - 1: descending, stable on ties
    rows = np.arange(m)
    thr_i = xi[rows, order[:, k - 1]]
    sel = np.zeros((m, n), dtype=np.uint64)
    sel[rows[:, None], order[:, :k]] = 1
    s = sel.astype(bool)
    with np.errstate(over="ignore"):
        d1 = np.where(s, from_i64((xi - thr_i[:, None]).reshape(-1)).reshape(m, n), np.uint64(0))
        d2 = np.where(s, np.uint64(0), from_i64((thr_i[:, None] - xi).reshape(-1)).reshape(m, n))
    gate = np.where(s, xv, np.uint64(0))
    return (xv[rows, order[:, k - 1]].copy(), sel.reshape(-1), gate.reshape(-1), d1.reshape(-1).astype(np.uint64),
            d2.reshape(-1).astype(np.uint64))


def argmax_forward(x, m, n):
    """topk.rs:272-297 -> (thr, sel, gate, d1, d2, out): top-1 plus the first
    position of each row's maximum."""
    thr, sel, gate, d1, d2 = topk_forward(x, m, n, 1)
    out = np.argmax(to_i64(x).reshape(m, n), axis=1).astype(np.uint32)
    return thr, sel, gate, d1, d2, out


def prove_lookup_fractional(idx, vals, table, alpha, beta, rng):
    """logup_gkr.rs:390-401: the merged witness / table fraction columns, then
    prove_fractional."""
    cols = o.lookup_num_den(idx, vals, table, None, 0, alpha, beta)
    if cols is None:
        raise IndexError("lookup index outside the table")
    return prove_fractional(cols[0], cols[1], rng)


def prove_range_decomp(values, rng):
    """topk.rs:391-448: to_i64(v) as u64 in three 16-bit limbs, each looked up
    in the 2^16 table, then the recomposition sumcheck."""
    v = to_i64(values).astype(np.uint64)
    limbs = [(v >> np.uint64(s)) & np.uint64(0xFFFF) for s in (0, 16, 32)]
    table = np.arange(1 << 16, dtype=np.uint64)
    ab = _draw(rng, 6)
    ranges = [prove_lookup_fractional(c.astype(np.uint32), c, table, int(ab[2 * i]), int(ab[2 * i + 1]), rng)
              for i, c in enumerate(limbs)]
    r = _draw(rng, _lg(len(v)))
    recompose = _vp([values] + limbs, RECOMPOSE_TERMS, r)
    return (ranges[0], ranges[1], ranges[2], recompose) + tuple(int(a) for a in ab) + (r,)


def prove_topk(x, sel, thr, gate, d1, d2, m, n, k, range_bits, rng):
    """topk.rs:82-176 -> ("TopKSelect", gate_rel, d1_rel, d2_rel, row_sum,
    sel_range, d1_range, d2_decomp, r, r_row, a_sel, b_sel, a_d1, b_d1,
    range_bits, sel)."""
    r = _draw(rng, _lg(m * n))
    gate_rel = _vp([x, sel, gate], GATE_TERMS, r)
    thr_b = _rows(thr, m, n)
    d1_rel = _vp([sel, x, thr_b, d1], D1_TERMS, r)
    d2_rel = _vp([sel, x, thr_b, d2], D2_TERMS, r)
    r_row = _draw(rng, _lg(m))
    row_sum = _vp([sel, _rows(o.eq_evals(r_row), m, n)], ROW_SUM_TERMS, r)
    a_sel, b_sel = rng.field(), rng.field()
    sel_range = prove_lookup_fractional(o.to_i32_indices(sel), sel, np.array([0, 1], dtype=np.uint64), a_sel, b_sel,
                                        rng)
    a_d1, b_d1 = rng.field(), rng.field()
    d1_range = prove_lookup_fractional(o.to_i32_indices(d1), d1, np.arange(1 << range_bits, dtype=np.uint64), a_d1,
                                       b_d1, rng)
    d2_decomp = prove_range_decomp(d2, rng)
    return ("TopKSelect", gate_rel, d1_rel, d2_rel, row_sum, sel_range, d1_range, d2_decomp, r, r_row, int(a_sel),
            int(b_sel), int(a_d1), int(b_d1), range_bits, o.u64(sel).reshape(-1).copy())


def prove_argmax(x, sel, thr, gate, d1, d2, out, m, n, range_bits, rng):
    """topk.rs:299-318 -> ("Argmax", topk proof, out, sel_evals = ())."""
    return ("Argmax", prove_topk(x, sel, thr, gate, d1, d2, m, n, 1, range_bits, rng),
            np.asarray(out, dtype=np.uint32).copy(), ())


# ---- the arms of an MLA / MoE layer (rms_norm.rs, rope.rs, scatter.rs, gather.rs,
# common/batched_matmul.rs, compose.rs:1193-1293) ------------------------------------------
def rms_norm_forward(x, w, table, m, d, n_real):
    """rms_norm.rs:37-95 -> dict(ms, s_index, rstd, raw, out, rem_out, rem_lo,
    rem_hi, sum_sq, rem_s): ms = round(sum x^2 / n_real) in wrapping i64, the
    rsqrt lookup, out = round(x rstd w / 2^32) and its remainder split in
    16-bit halves (arithmetic shift for the high one)."""
    x = o.u64(x).reshape(-1)
    xi = to_i64(x).reshape(m, d)[:, :n_real]
    with np.errstate(over="ignore"):
        sq = (xi * xi).sum(axis=1)
    ms = from_i64(round_div(sq, n_real))
    s_index = rsqrt_index(to_i64(ms))
    if s_index.size and int(s_index.max()) >= table.size:
        raise IndexError("rsqrt table too short for the forward pass")
    rstd = table[s_index.astype(np.int64)]
    raw = o.vec_mul(o.vec_mul(x, _rows(rstd, m, d)), w)
    ri = to_i64(raw)
    out = from_i64(round_div(ri, 1 << 32))
    with np.errstate(over="ignore"):
        rem_i = ri - to_i64(out) * (1 << 32) + (1 << 31)
        sum_sq = o.row_sums(o.vec_mul(x, x), m, d, n_real)
        rem_s = from_i64(to_i64(sum_sq) - to_i64(ms) * n_real + n_real // 2)
    rem_out = from_i64(rem_i)
    ro = to_i64(rem_out)
    return dict(ms=ms, s_index=s_index, rstd=rstd, raw=raw, out=out, rem_out=rem_out,
                rem_lo=from_i64(ro & 0xFFFF), rem_hi=from_i64(ro >> 16), sum_sq=sum_sq, rem_s=rem_s)


RMS_OUT_TERMS = [(1, [0, 1, 2]), (NEG, [3]), (1, [3]), (NEG * (1 << 32) % P, [4]), (NEG, [5]), (1 << 31, [6])]
REM_SPLIT_TERMS = [(1, [0]), (NEG, [1]), (NEG * (1 << 16) % P, [2])]


def rms_trunc_terms(n_real):
    return [(n_real % P, [0]), (1, [1]), (NEG, [2]), (NEG * (n_real // 2) % P, [3])]


def prove_rms_norm(x, w, table, m, d, n_real, rng):
    """rms_norm.rs:97-174 -> (("RmsNorm", trunc, out, rem_split, trunc_ch,
    r_out, rem_split_ch), forward dict)."""
    f = rms_norm_forward(x, w, table, m, d, n_real)
    trunc_ch = _draw(rng, _lg(m))
    trunc = _vp([f["ms"], f["rem_s"], f["sum_sq"], np.ones(m, dtype=np.uint64)], rms_trunc_terms(n_real), trunc_ch)
    r_out = _draw(rng, _lg(m * d))
    out = _vp([x, _rows(f["rstd"], m, d), w, f["raw"], f["out"], f["rem_out"], np.ones(m * d, dtype=np.uint64)],
              RMS_OUT_TERMS, r_out)
    rem_split_ch = _draw(rng, _lg(m * d))
    rem_split = _vp([f["rem_out"], f["rem_lo"], f["rem_hi"]], REM_SPLIT_TERMS, rem_split_ch)
    return ("RmsNorm", trunc, out, rem_split, trunc_ch, r_out, rem_split_ch), f


def _rope_halves(v, m, d):
    """extract_first / extract_second (rope.rs:47-71): [m, heads, d] split into
    its two d/2 halves, each [m, heads, d/2] flattened."""
    v = o.u64(v).reshape(m, -1, d)
    return np.ascontiguousarray(v[:, :, :d // 2]).reshape(-1), np.ascontiguousarray(v[:, :, d // 2:]).reshape(-1)


def _rope_pair(table, m, d, heads):
    """broadcast_pair (rope.rs:73-85): [m, d/2] repeated over the heads."""
    return np.repeat(o.u64(table).reshape(m, 1, d // 2), heads, axis=1).reshape(-1)


def rope_forward(x, cos, sin, m, d, shift):
    """rope.rs:87-124 -> (out, rem_f, rem_s): rotate-half in wrapping i64,
    each product rounded by 2^shift, remainders offset by 2^(shift-1)."""
    heads = o.u64(x).size // (m * d)
    xf, xs = (to_i64(h).reshape(m, heads, d // 2) for h in _rope_halves(x, m, d))
    c = to_i64(cos).reshape(m, 1, d // 2)
    sn = to_i64(sin).reshape(m, 1, d // 2)
    with np.errstate(over="ignore"):
        raw_f = xf * c - xs * sn
        raw_s = xs * c + xf * sn
        of = round_div(raw_f.reshape(-1), 1 << shift).reshape(raw_f.shape)
        os_ = round_div(raw_s.reshape(-1), 1 << shift).reshape(raw_s.shape)
        rem_f = from_i64((raw_f - of * (1 << shift) + (1 << (shift - 1))).reshape(-1))
        rem_s = from_i64((raw_s - os_ * (1 << shift) + (1 << (shift - 1))).reshape(-1))
    out = np.concatenate([from_i64(of.reshape(-1)).reshape(m, heads, d // 2),
                          from_i64(os_.reshape(-1)).reshape(m, heads, d // 2)], axis=2).reshape(-1)
    return out, rem_f, rem_s


def rope_terms(shift, second):
    two, half = 1 << shift, 1 << (shift - 1)
    return [(1, [0, 1]), ((1 if second else NEG), [2, 3]), (NEG * two % P, [4]), (NEG, [5]), (half, [6])]


def prove_rope(x, cos, sin, out, m, d, shift, rng):
    """rope.rs:126-196 -> (("RoPE", first, second, r_first, r_second, r_out),
    rem_f, rem_s)."""
    heads = o.u64(x).size // (m * d)
    _, rem_f, rem_s = rope_forward(x, cos, sin, m, d, shift)
    x_f, x_s = _rope_halves(x, m, d)
    o_f, o_s = _rope_halves(out, m, d)
    cos_b, sin_b = _rope_pair(cos, m, d, heads), _rope_pair(sin, m, d, heads)
    n = m * heads * (d // 2)
    ones = np.ones(n, dtype=np.uint64)
    r_f = _draw(rng, _lg(n))
    first = _vp([x_f, cos_b, x_s, sin_b, o_f, rem_f, ones], rope_terms(shift, False), r_f)
    r_s = _draw(rng, _lg(n))
    second = _vp([x_s, cos_b, x_f, sin_b, o_s, rem_s, ones], rope_terms(shift, True), r_s)
    r_out = _draw(rng, _lg(o.u64(out).size))
    return ("RoPE", first, second, r_f, r_s, r_out), rem_f, rem_s


def scatter_forward(sel, m, n):
    """scatter.rs:12-25 -> (token_id, expert_of) in expert-major order."""
    s = (o.u64(sel).reshape(m, n) == 1)
    e_idx, t_idx = np.nonzero(s.T)
    return t_idx.astype(np.uint32), e_idx.astype(np.uint32)


def _perm_num_den(values, alpha):
    """build_perm_num_den (logup_gkr.rs:807-820): num 1, den alpha - value,
    padded to max(next power of two, 32) with 0 / alpha."""
    v = o.u64(values).reshape(-1)
    total = max(1 << max(v.size - 1, 0).bit_length(), 32)
    num = np.zeros(total, dtype=np.uint64)
    den = np.full(total, int(alpha) % P, dtype=np.uint64)
    num[:v.size] = 1
    den[:v.size] = o.vec_sub(np.full(v.size, int(alpha) % P, dtype=np.uint64), v)
    return num, den


def prove_permutation(a, b, rng):
    """logup_gkr.rs:822-840 -> (a_side, b_side, alpha, a, b)."""
    alpha = rng.field()
    na, da = _perm_num_den(a, alpha)
    nb, db = _perm_num_den(b, alpha)
    a_side = prove_fractional(na, da, rng)
    b_side = prove_fractional(nb, db, rng)
    return (a_side, b_side, int(alpha), o.u64(a).reshape(-1).copy(), o.u64(b).reshape(-1).copy())


def prove_scatter(sel, token_id, expert_of, m, n, rng):
    """scatter.rs:39-55: the source encodings t n + e in token-major order
    against token_id n + expert_of, as a permutation."""
    s = (o.u64(sel).reshape(m, n) == 1)
    t_idx, e_idx = np.nonzero(s)
    a = (t_idx * n + e_idx).astype(np.uint64)
    b = np.asarray(token_id, dtype=np.uint64) * np.uint64(n) + np.asarray(expert_of, dtype=np.uint64)
    return ("Scatter", prove_permutation(a, b, rng))


def gather_forward(weighted, token_id, gate, m, h):
    """gather.rs:36-52: out[t] = sum over positions routed to t of
    weighted[pos] gate[pos] (field)."""
    tid = np.asarray(token_id, dtype=np.int64)
    wg = o.vec_mul(o.u64(weighted).reshape(-1), np.repeat(o.u64(gate).reshape(-1), h))
    out = np.zeros(m * h, dtype=np.uint64)
    for pos, t in enumerate(tid):
        out[t * h:(t + 1) * h] = o.vec_add(out[t * h:(t + 1) * h], wg[pos * h:(pos + 1) * h])
    return out


def _pow2(n):
    return 1 << max(int(n) - 1, 0).bit_length()


def prove_scatter_add(weighted, token_id, gate, out, m, h, rng):
    """gather.rs:54-157 -> ("Gather", source_side, target_side, alpha, gamma,
    num_source, den_source, num_target, den_target, prod_source, prod_target,
    r_prod_source, r_prod_target, weighted, gate, out, token_id)."""
    weighted, gate, out = (o.u64(v).reshape(-1) for v in (weighted, gate, out))
    tid = np.asarray(token_id, dtype=np.uint64)
    s = tid.size
    alpha = int(rng.field()) % P
    gamma = _draw(rng, h)
    st, tt = _pow2(s * h), _pow2(m * h)
    gamma_s = np.zeros(st, dtype=np.uint64)
    gamma_s[:s * h] = np.tile(gamma, s)
    gate_b = np.zeros(st, dtype=np.uint64)
    gate_b[:s * h] = np.repeat(gate, h)
    w_pad = np.zeros(st, dtype=np.uint64)
    w_pad[:s * h] = weighted
    num_s = o.vec_mul(o.vec_mul(gamma_s, w_pad), gate_b)
    den_s = np.full(st, alpha, dtype=np.uint64)
    den_s[:s * h] = o.vec_sub(den_s[:s * h], np.repeat(tid, h))
    gamma_t = np.zeros(tt, dtype=np.uint64)
    gamma_t[:m * h] = np.tile(gamma, m)
    o_pad = np.zeros(tt, dtype=np.uint64)
    o_pad[:m * h] = out
    num_t = o.vec_mul(gamma_t, o_pad)
    den_t = np.full(tt, alpha, dtype=np.uint64)
    den_t[:m * h] = o.vec_sub(den_t[:m * h], np.repeat(np.arange(m, dtype=np.uint64), h))
    source_side = prove_fractional(num_s, den_s, rng)
    target_side = prove_fractional(num_t, den_t, rng)
    r_ps = _draw(rng, _lg(st))
    prod_source = _vp([o.eq_evals(r_ps), num_s, gamma_s, w_pad, gate_b], SCATTER_ADD_SOURCE_TERMS, r_ps)
    r_pt = _draw(rng, _lg(tt))
    prod_target = _vp([o.eq_evals(r_pt), num_t, gamma_t, o_pad], SCATTER_ADD_TARGET_TERMS, r_pt)
    return ("Gather", source_side, target_side, alpha, gamma, num_s, den_s, num_t, den_t, prod_source, prod_target,
            r_ps, r_pt, weighted.copy(), gate.copy(), out.copy(), tid.astype(np.uint32))


SCATTER_ADD_SOURCE_TERMS = [(1, [0, 1]), (NEG, [0, 2, 3, 4])]
SCATTER_ADD_TARGET_TERMS = [(1, [0, 1]), (NEG, [0, 2, 3])]
BMM_TERMS = [(1, [0, 1, 2])]


def batched_matmul_forward(a, w, s, k, n):
    """batched_matmul.rs:112-134: g[pos] = a[pos] w[pos] (field), w S x K x N."""
    a, w = o.u64(a).reshape(s, k), o.u64(w).reshape(s, k, n)
    return np.concatenate([o.matmul_field(a[p:p + 1], w[p]).reshape(-1) for p in range(s)])


def prove_batched_matmul(a, w, g, s, k, n, u, v, ch):
    """batched_matmul.rs:51-83 -> (claimed, (rounds, finals)): the eq-selector
    sumcheck over [a, w contracted with eq(v), eq(u) per row]."""
    w_v = o.mle_partial_eval(o.u64(w).reshape(-1), v)
    eq_b = np.repeat(o.eq_evals(u), k)
    claimed = o.mle_eval(g, np.concatenate([v, u]))
    return (int(claimed), _vp([a, w_v, eq_b], BMM_TERMS, ch))


def verify_batched_matmul(p, s, k):
    """batched_matmul.rs:85-110."""
    _, (claimed, (rounds, finals)), u, _, ch = p
    eq_final = o.mle_eval(np.repeat(o.eq_evals(u), k), ch)
    fin = np.array([int(finals[0]), int(finals[1]), int(eq_final)], dtype=np.uint64)
    return o.virtual_verify(rounds, BMM_TERMS, claimed, ch, fin)


def gather_matmul_forward(seg, expert_of, w_all, s, k, n, n_experts):
    """batched_matmul.rs:331-357: g[pos] = seg[pos] W_all[expert_of[pos]] (field)."""
    seg = o.u64(seg).reshape(s, k)
    w_all = o.u64(w_all).reshape(n_experts, k, n)
    g = np.zeros((s, n), dtype=np.uint64)
    e_of = np.asarray(expert_of, dtype=np.int64)
    for e in np.unique(e_of):
        rows = np.nonzero(e_of == e)[0]
        g[rows] = o.matmul_field(seg[rows], w_all[e])
    return g.reshape(-1)


def prove_gather_matmul(seg, expert_of, w_all, g, s, k, n, n_experts, u, v, ch):
    """batched_matmul.rs:359-390 (prove_streaming) and :469-494 -> (claimed,
    (rounds, finals), counts, table): the eq-selector sumcheck over [seg,
    w_v, eq(u) per row], w_v the experts' weights contracted with eq(v)."""
    w_all = o.u64(w_all).reshape(n_experts, k, n)
    e_of = np.asarray(expert_of, dtype=np.int64)
    eq_v = o.eq_evals(v)
    wv = np.stack([o.matmul_field(w_all[e], eq_v.reshape(n, 1)).reshape(-1) for e in range(n_experts)])
    w_v = wv[e_of].reshape(-1)
    eq_b = np.repeat(o.eq_evals(u), k)
    claimed = o.mle_eval(g, np.concatenate([v, u]))
    sc = _vp([seg, w_v, eq_b], BMM_TERMS, ch)
    kb = _lg(k)
    eq_pos = o.eq_evals(ch[kb:])
    counts = np.zeros(n_experts, dtype=np.uint64)
    for pos, e in enumerate(e_of):
        counts[e] = (int(counts[e]) + int(eq_pos[pos])) % P
    table = np.array([int(o.mle_eval(wv[e], ch[:kb])) for e in range(n_experts)], dtype=np.uint64)
    return (int(claimed), sc, counts, table)


# ---- op arms -----------------------------------------------------------------------------
def _vp(mles, terms, ch):
    """prove_virtual -> (rounds, finals)."""
    return o.virtual_prove([o.u64(t).reshape(-1) for t in mles], terms, ch)


def prove_layer_norm_centered(x, w, b, table, m, d, n_real, rng):
    """layer_norm_centered.rs:122-245.  The two reduction sumchecks whose
    proofs the reference discards (:153-159, :193-201) only advance the
    challenge source here; they contribute nothing to the proof."""
    f = layer_norm_forward(x, w, b, table, m, d, n_real)
    lm, lmd = _lg(m), _lg(m * d)
    df, half_d = n_real % P, (n_real // 2) % P
    r_mean = _draw(rng, lm)
    _draw(rng, lmd)  # mean_ch of the discarded mean reduction
    m_ch = _draw(rng, lm)
    ones_m = np.ones(m, dtype=np.uint64)
    trunc_terms = [(df, [0]), (1, [1]), (NEG, [2]), (NEG * half_d % P, [3])]
    mean = _vp([f["mean"], f["rem_mean"], f["sum_mean"], ones_m], trunc_terms, m_ch)
    centered_r = _draw(rng, lmd)
    centered = _vp([x, _rows(f["mean"], m, d), f["centered"]], [(1, [2]), (NEG, [0]), (1, [1])], centered_r)
    r_var = _draw(rng, lm)
    _draw(rng, lmd)  # var_ch of the discarded variance reduction
    v_ch = _draw(rng, lm)
    var = _vp([f["var"], f["rem_var"], f["sum_var"], ones_m], trunc_terms, v_ch)
    r_out = _draw(rng, lmd)
    two32, half32 = 1 << 32, 1 << 31
    out_terms = [(1, [0, 1, 2]), (NEG, [4]), (1, [4]), (NEG * two32 % P, [5]), (two32, [3]), (NEG, [6]),
                 (half32, [7])]
    out = _vp([f["centered"], _rows(f["rstd"], m, d), w, b, f["raw"], f["out"], f["rem_out"],
               np.ones(m * d, dtype=np.uint64)], out_terms, r_out)
    proof = ("LayerNormCentered", mean, centered, var, out, r_mean, m_ch, centered_r, r_var, v_ch, r_out)
    return proof, f["s_index"], f["rstd"]


def prove_layernorm_chain(x, w, b, table, m, d, rng):
    """layernorm_chain.rs:24-93."""
    f = layernorm_forward(x, w, b, table, m, d)
    r_mean = _draw(rng, _lg(m))
    eq_b = _rows(o.eq_evals(r_mean), m, d)
    mean_claim = o.mle_eval(f["mean_sq"], r_mean)
    mean_ch = _draw(rng, _lg(m * d))
    mean_sq = _vp([eq_b, x], [(1, [0, 1, 1])], mean_ch)
    r_out = _draw(rng, _lg(m * d))
    out = _vp([x, f["scale"], b, f["out"]], [(1, [0, 1]), (1, [2]), (NEG, [3])], r_out)
    return ("Layernorm", mean_sq, out, r_mean, mean_ch, r_out, mean_claim), f["idx"], f["rsqrt"]


def prove_softmax_rounded(idx, e, out, table, m, n, rng):
    """softmax_scaled.rs:42-108."""
    s = o.row_sums(e, m, n, n)
    r_sum = _draw(rng, _lg(m))
    eq_b = _rows(o.eq_evals(r_sum), m, n)
    sum_ch = _draw(rng, _lg(m * n))
    claimed = o.mle_eval(s, r_sum)
    row_sum = _vp([eq_b, e], [(1, [0, 1])], sum_ch)
    sum_b = _rows(s, m, n)
    with np.errstate(over="ignore"):
        rem = from_i64(to_i64(e) * (1 << 16) - to_i64(out) * to_i64(sum_b))
    r_scale = _draw(rng, _lg(m * n))
    rescale = _vp([out, e, sum_b, rem], [(1, [0, 2]), (NEG * (1 << 16) % P, [1]), (1, [3])], r_scale)
    return ("Softmax", row_sum, rescale, r_sum, sum_ch, r_scale, claimed)


def prove_same_poly(f, claims, rng):
    """same_poly.rs:13-45 -> (coeffs, (rounds, finals), merged_point, merged_eval)."""
    t = _lg(len(f))
    coeffs = _draw(rng, len(claims))
    eqs = [o.eq_evals(pt) for pt, _ in claims]
    terms = [(int(c), [0, i + 1]) for i, c in enumerate(coeffs)]
    merged = _draw(rng, t)
    rounds, finals = o.virtual_prove([f] + eqs, terms, merged)
    return (coeffs, (rounds, finals), merged, int(finals[0]))


def prove_fractional(num, den, rng):
    """logup_gkr.rs:71-81 -> (layers, final_num, final_den, full_r); layer =
    (r, c, rounds, finals)."""
    lg = _lg(len(num))
    full_r, cs = _draw(rng, lg), _draw(rng, lg)
    rounds, finals, fnum, fden = o.fractional_prove(num, den, full_r, cs)
    layers = tuple((full_r[:lg - l - 1].copy(), int(cs[l]), rounds[l], finals[l]) for l in range(lg))
    return (layers, fnum, fden, full_r)


def fractional_leaf(proof):
    layers, _, _, full_r = proof
    top = int(full_r[-1])
    fe = [int(v) for v in layers[0][3]]
    one_m = (1 - top) % P
    return full_r.copy(), (one_m * fe[3] + top * fe[4]) % P, (one_m * fe[5] + top * fe[6]) % P


def merge_multiplicity(xs, t):
    m = np.zeros(t, dtype=np.uint64)
    for x in xs:
        x = np.asarray(x, dtype=np.int64)
        if x.size and x.max() >= t:
            raise IndexError("lookup index outside the table")
        m += np.bincount(x, minlength=t).astype(np.uint64)
    return m


def prove_lookup_witness_batch_columns(xs, ys, alpha, beta, rng):
    x = np.concatenate([np.asarray(v, dtype=np.uint32) for v in xs]) if xs else np.zeros(0, np.uint32)
    y = np.concatenate([o.u64(v).reshape(-1) for v in ys]) if ys else np.zeros(0, np.uint64)
    num, den = o.lookup_num_den(x, y, None, None, 2, alpha, beta)
    x_flat = np.zeros(num.size, dtype=np.uint64)
    y_flat = np.zeros(num.size, dtype=np.uint64)
    x_flat[:x.size] = x
    y_flat[:y.size] = y
    return prove_fractional(num, den, rng), x_flat, y_flat, num


def prove_lookup_table(m, table, alpha, beta, rng):
    num, den = o.lookup_num_den(None, None, table, m, 3, alpha, beta)
    return prove_fractional(num, den, rng)


# ---- shard (compose.rs:1602-2091, 2276-2346) -------------------------------------------------
ADD_TERMS = [(1, [2]), (NEG, [0]), (NEG, [1])]
# the arms with no proof of their own (compose.rs:1623-1723)
MARKER_KINDS = ("Transpose", "Scale", "SoftmaxIndex", "GeluIndex", "StableSoftmaxIndex", "ScaleVec", "IdxBroadcast",
                "CombineIdx", "PadIdx", "BroadcastScale", "ScaleGate", "Relu")


def prove_shard_precomputed(store, ops, boundary, rng):
    """-> dict(ops, bound, binds, claims, witness_columns, table_columns)."""
    g = store.get
    claims, op_proofs, lookups = [], [], {}

    def claim(t, pt):
        pt = o.u64(pt).reshape(-1)
        claims.append((t, pt, o.mle_eval(g(t), pt)))

    for op in ops:
        k = op.kind
        if k in MARKER_KINDS:
            op_proofs.append((k,))
        elif k == "MatMul":
            r = o.op_matmul_prove(g(op.a).reshape(op.m, op.k), g(op.b).reshape(op.k, op.n),
                                  g(op.c).reshape(op.m, op.n), op.m, op.k, op.n, rng)
            fe = [int(v) for v in r["finals"]]
            pts = [np.concatenate([r["ch"], r["u"]]), np.concatenate([r["v"], r["ch"]]),
                   np.concatenate([r["v"], r["u"]])]
            for t, pt, ev in zip((op.a, op.b, op.c), pts, r["claims"]):
                claims.append((t, o.u64(pt), int(ev)))
            op_proofs.append(("MatMul", r["claimed"], r["rounds"], fe[0], fe[1], r["u"], r["v"], r["ch"]))
        elif k == "Projection":
            p = o.projection_prove(g(op.x), g(op.w), g(op.bias), g(op.out), g(op.rem), op.m, op.k, op.n,
                                   op.shift, rng)
            claim(op.x, np.concatenate([p["ch"], p["u"]]))
            claim(op.w, np.concatenate([p["v"], p["ch"]]))
            claim(op.out, p["pt"])
            claims.append((op.bias, o.u64(p["pt"]), int(p["affine_finals"][4])))
            lg = len(p["full_r"])
            layers = tuple((p["full_r"][:lg - l - 1].copy(), int(p["cs"][l]), p["frac_rounds"][l],
                            p["frac_finals"][l]) for l in range(lg))
            frac = (layers, p["final_num"], p["final_den"], p["full_r"])
            mm = (p["claimed"], p["mm_rounds"], int(p["mm_finals"][0]), int(p["mm_finals"][1]))
            op_proofs.append(("Projection", mm, (p["affine_rounds"], p["affine_finals"]), frac, p["alpha"],
                              p["beta"], p["pt"], p["u"], p["v"], p["ch"]))
        elif k == "Add":
            r = _draw(rng, _lg(len(g(op.c))))
            proof = _vp([g(op.a), g(op.b), g(op.c)], ADD_TERMS, r)
            for t in (op.a, op.b, op.c):
                claim(t, r)
            op_proofs.append(("Add", proof, r))
        elif k == "Lookup":
            lookups.setdefault(op.table, []).append((store.idx[op.idx], g(op.out)))
            op_proofs.append(("Lookup",))
        elif k == "Softmax":
            p = prove_softmax_rounded(store.idx[op.idx], g(op.e), g(op.out), g(op.table), op.m, op.n, rng)
            claim(op.out, p[5])
            lookups.setdefault(op.table, []).append((store.idx[op.idx], g(op.e)))
            op_proofs.append(p)
        elif k == "Layernorm":
            p, ridx, rvals = prove_layernorm_chain(g(op.x), g(op.w), g(op.b), g(op.rsqrt_table), op.m, op.d, rng)
            lookups.setdefault(op.rsqrt_table, []).append((ridx, rvals))
            for t in (op.out, op.w, op.b):
                claim(t, p[5])
            op_proofs.append(p)
        elif k == "LayerNormCentered":
            p, ridx, rvals = prove_layer_norm_centered(g(op.x), g(op.w), g(op.b), g(op.rsqrt_table), op.m,
                                                       op.d, op.n_real, rng)
            lookups.setdefault(op.rsqrt_table, []).append((ridx, rvals))
            claim(op.x, p[7])
            for t in (op.out, op.w, op.b):
                claim(t, p[10])
            op_proofs.append(p)
        elif k == "Scatter":  # compose.rs:1632-1648
            op_proofs.append(prove_scatter(g(op.sel), store.idx[op.token_id], store.idx[op.expert_of], op.m, op.n,
                                           rng))
        elif k == "Gather":  # :1649-1667
            op_proofs.append(prove_scatter_add(g(op.weighted), store.idx[op.token_id], g(op.gate), g(op.out), op.m,
                                               op.h, rng))
        elif k == "BatchedMatMul":  # :1668-1681
            u, v, ch = _draw(rng, _lg(op.s)), _draw(rng, _lg(op.n)), _draw(rng, _lg(op.s * op.k))
            p = prove_batched_matmul(g(op.a), g(op.w), g(op.c), op.s, op.k, op.n, u, v, ch)
            claim(op.a, ch)
            claim(op.w, np.concatenate([v, ch]))
            claim(op.c, np.concatenate([v, u]))
            op_proofs.append(("BatchedMatMul", p, u, v, ch))
        elif k == "GatherMatMul":  # :1682-1705
            u, v, ch = _draw(rng, _lg(op.s)), _draw(rng, _lg(op.n)), _draw(rng, _lg(op.s * op.k))
            p = prove_gather_matmul(g(op.a), store.idx[op.expert_of], g(op.w), g(op.c), op.s, op.k, op.n,
                                    op.n_experts, u, v, ch)
            claims.append((op.a, ch.copy(), int(p[1][1][0])))
            claims.append((op.c, np.concatenate([v, u]), p[0]))
            op_proofs.append(("GatherMatMul", p, u, v, ch))
        elif k == "RmsNorm":  # :1898-1934
            p, f = prove_rms_norm(g(op.x), g(op.w), g(op.rsqrt_table), op.m, op.d, op.n_real, rng)
            lookups.setdefault(op.rsqrt_table, []).append((f["s_index"], f["rstd"]))
            for part in ("rem_lo", "rem_hi"):
                lookups.setdefault(op.limb_table, []).append((o.to_i32_indices(f[part]), f[part]))
            claim(op.out, p[5])
            claim(op.w, p[5])
            op_proofs.append(p)
        elif k == "RoPE":  # :1935-1967
            p, rem_f, rem_s = prove_rope(g(op.x), g(op.cos), g(op.sin), g(op.out), op.m, op.d, op.shift, rng)
            for rem in (rem_f, rem_s):
                lookups.setdefault(op.range_table, []).append((o.to_i32_indices(rem), rem))
            claim(op.out, p[5])
            op_proofs.append(p)
        elif k in ("TopKSelect", "Argmax"):
            args = (g(op.x), g(op.sel), g(op.thr), g(op.gate), g(op.d1), g(op.d2))
            if k == "TopKSelect":  # compose.rs:1968-1996 (range_bits 22)
                p = prove_topk(*args, op.m, op.n, op.k, 22, rng)
                tk = p
            else:  # :1997-2025 (range_bits 16)
                p = prove_argmax(*args, store.idx[op.out], op.m, op.n, 16, rng)
                tk = p[1]
            for t in (op.x, op.sel, op.gate):
                claim(t, tk[8])
            op_proofs.append(p)
        else:
            raise ValueError(f"op {k} is not restated")

    by_tensor = {}
    for t, pt, ev in claims:
        by_tensor.setdefault(t, []).append((pt, ev))
    bound, binds = [], []
    for t in sorted(by_tensor):
        cs = by_tensor[t]
        if t in set(boundary) or len(cs) < 2:
            continue
        binds.append(prove_same_poly(g(t), cs, rng))
        bound.append(t)

    witness_columns, table_columns = [], []
    for table in sorted(lookups):
        alpha, beta = rng.field(), rng.field()
        xs = [x for x, _ in lookups[table]]
        ys = [y for _, y in lookups[table]]
        proof, x_flat, y_flat, num = prove_lookup_witness_batch_columns(xs, ys, alpha, beta, rng)
        point, nl, dl = fractional_leaf(proof)
        m = merge_multiplicity(xs, len(g(table)))
        tproof = prove_lookup_table(m, g(table), alpha, beta, rng)
        tpoint, tnl, tdl = fractional_leaf(tproof)
        witness_columns.append((proof, x_flat, y_flat, num, point, nl, dl, alpha, beta, table))
        table_columns.append((tproof, table, m, alpha, beta, tpoint, tnl, tdl))
    return dict(ops=op_proofs, bound=bound, binds=binds, claims=claims, witness_columns=witness_columns,
                table_columns=table_columns)


def prove_shard(store, ops, boundary, rng):
    forward_ops(store, ops)
    return prove_shard_precomputed(store, ops, boundary, rng)


def shard_ranges(op_count, ops_per_shard):
    ops_per_shard = max(ops_per_shard, 1)
    return [(s, min(s + ops_per_shard, op_count)) for s in range(0, op_count, ops_per_shard)]


def master_transcript(ops, ops_per_shard):
    """Transcript::new("zkie-shard-dag-v1") with absorb_statement (compose.rs:2276-2287)."""
    t = o.OracleTranscript(b"zkie-shard-dag-v1")
    t.absorb_u64(ops_per_shard)
    t.absorb_u64(len(ops))
    for op in ops:
        for i in op.reads():
            t.absorb_u64(i)
        for i in op.writes():
            t.absorb_u64(i)
    return t


def prove_shard_dag(store, ops, ops_per_shard):
    """compose.rs:2289-2346 -> dict(shards, cross_tensors, cross_binds)."""
    forward_ops(store, ops)
    master = master_transcript(ops, ops_per_shard)
    shards = []
    for si, (s, e) in enumerate(shard_ranges(len(ops), ops_per_shard)):
        child = o.OracleTranscript(raw=master.t)
        child.absorb_u64(si)
        shards.append(prove_shard_precomputed(store, ops[s:e], [], child))
    by_tensor, owners = {}, {}
    for si, sh in enumerate(shards):
        for t, pt, ev in sh["claims"]:
            by_tensor.setdefault(t, []).append((pt, ev))
            owners.setdefault(t, set()).add(si)
    cross_tensors, cross_binds = [], []
    for t in sorted(by_tensor):
        if len(owners[t]) > 1:
            cross_binds.append(prove_same_poly(store.get(t), by_tensor[t], master))
            cross_tensors.append(t)
    return dict(shards=shards, cross_tensors=cross_tensors, cross_binds=cross_binds)


# ---- verify_shard_precomputed (compose.rs:2103-2239) ------------------------------------------
def _verify_virtual(vp, terms, claimed, ch):
    rounds, finals = vp
    return o.virtual_verify(rounds, terms, claimed, ch, finals)


def _chain_core(frac):
    layers, _, _, full_r = frac
    cs = [c for _, c, _, _ in layers]
    return o.fractional_chain_core(full_r, cs, [r for _, _, r, _ in layers], [f for _, _, _, f in layers])


def verify_lookup_split(wp, tp):
    """logup_gkr.rs verify_lookup_split: both chains sound and the two sides'
    fractional sums equal (cross-multiplied)."""
    return (_chain_core(wp) and _chain_core(tp)
            and (wp[1] * tp[2] - tp[1] * wp[2]) % P == 0)


def verify_layer_norm_centered(p, n_real):
    """layer_norm_centered.rs:247-310."""
    _, mean, centered, var, out, _, mean_ch, centered_r, _, var_ch, r_out = p
    trunc = [(n_real % P, [0]), (1, [1]), (NEG, [2]), (NEG * (n_real // 2) % P, [3])]
    two32 = 1 << 32
    out_terms = [(1, [0, 1, 2]), (NEG, [4]), (1, [4]), (NEG * two32 % P, [5]), (two32, [3]), (NEG, [6]),
                 (1 << 31, [7])]
    return (_verify_virtual(mean, trunc, 0, mean_ch)
            and _verify_virtual(centered, [(1, [2]), (NEG, [0]), (1, [1])], 0, centered_r)
            and _verify_virtual(var, trunc, 0, var_ch)
            and _verify_virtual(out, out_terms, 0, r_out))


def verify_layernorm_chain(p):
    """layernorm_chain.rs:95-115."""
    _, mean_sq, out, _, mean_ch, r_out, mean_claim = p
    return (_verify_virtual(mean_sq, [(1, [0, 1, 1])], mean_claim, mean_ch)
            and _verify_virtual(out, [(1, [0, 1]), (1, [2]), (NEG, [3])], 0, r_out))


def verify_softmax_rounded(p):
    """softmax_scaled.rs:110-135."""
    _, row_sum, rescale, _, sum_ch, r_scale, claimed = p
    return (_verify_virtual(row_sum, [(1, [0, 1])], claimed, sum_ch)
            and _verify_virtual(rescale, [(1, [0, 2]), (NEG * (1 << 16) % P, [1]), (1, [3])], 0, r_scale))


def verify_lookup_fractional_chain(frac):
    """logup_gkr.rs:450-452: the chain sound and the fraction sum zero."""
    return _chain_core(frac) and int(frac[1]) % P == 0


def verify_range_decomp(p):
    """topk.rs:450-470."""
    return (all(verify_lookup_fractional_chain(f) for f in p[:3])
            and _verify_virtual(p[3], RECOMPOSE_TERMS, 0, p[10]))


def verify_topk(p, k):
    """topk.rs:178-240."""
    _, gate_rel, d1_rel, d2_rel, row_sum, sel_range, d1_range, d2_decomp, r = p[:9]
    return (_verify_virtual(gate_rel, GATE_TERMS, 0, r) and _verify_virtual(d1_rel, D1_TERMS, 0, r)
            and _verify_virtual(d2_rel, D2_TERMS, 0, r) and _verify_virtual(row_sum, ROW_SUM_TERMS, k % P, r)
            and verify_lookup_fractional_chain(sel_range) and verify_lookup_fractional_chain(d1_range)
            and verify_range_decomp(d2_decomp))


def verify_argmax(p, m, n):
    """topk.rs:320-343: the top-1 proof, then sel = 1 at every row's output
    position."""
    _, tk, out, sel_evals = p
    if not verify_topk(tk, 1):
        return False
    sel = tk[15]
    for i in range(m):
        j = int(out[i])
        if j >= n:
            return False
        v = int(sel_evals[i]) if len(sel_evals) else int(sel[i * n + j])
        if v != 1:
            return False
    return True


def verify_rms_norm(p, n_real):
    """rms_norm.rs:176-222."""
    _, trunc, out, rem_split, trunc_ch, r_out, rem_split_ch = p
    return (_verify_virtual(trunc, rms_trunc_terms(n_real), 0, trunc_ch)
            and _verify_virtual(out, RMS_OUT_TERMS, 0, r_out)
            and _verify_virtual(rem_split, REM_SPLIT_TERMS, 0, rem_split_ch))


def verify_rope(p, shift):
    """rope.rs:198-230."""
    _, first, second, r_f, r_s, _ = p
    return (_verify_virtual(first, rope_terms(shift, False), 0, r_f)
            and _verify_virtual(second, rope_terms(shift, True), 0, r_s))


def verify_scatter(p):
    """scatter.rs:57-59 / logup_gkr.rs:842-844."""
    a_side, b_side = p[1][0], p[1][1]
    return verify_lookup_split(a_side, b_side)


def verify_scatter_add(p):
    """gather.rs:159-186."""
    return (verify_lookup_split(p[1], p[2])
            and _verify_virtual(p[9], SCATTER_ADD_SOURCE_TERMS, 0, p[11])
            and _verify_virtual(p[10], SCATTER_ADD_TARGET_TERMS, 0, p[12]))


def verify_gather_matmul(p, s, k):
    """batched_matmul.rs:496-513: the sumcheck with the public eq(u) selector's
    final value recomputed, then the weight claim against sum_e counts table."""
    _, (claimed, (rounds, finals), counts, table), u, _, ch = p
    eq_final = o.mle_eval(np.repeat(o.eq_evals(u), k), ch)
    fin = np.array([int(finals[0]), int(finals[1]), int(eq_final)], dtype=np.uint64)
    if not o.virtual_verify(rounds, BMM_TERMS, claimed, ch, fin):
        return False
    return int(finals[1]) % P == sum(int(c) * int(t) for c, t in zip(counts, table)) % P


def verify_same_poly(sp, claims):
    """same_poly.rs:46-70: the merged evaluation, or None."""
    coeffs, vp, merged, merged_eval = sp
    terms = [(int(c), [0, i + 1]) for i, c in enumerate(coeffs)]
    claimed = sum(int(c) * int(y) for c, (_, y) in zip(coeffs, claims)) % P
    return merged_eval if _verify_virtual(vp, terms, claimed, merged) else None


def verify_shard(ops, proof):
    """verify_shard_precomputed over the proof layout of prove_shard_precomputed."""
    if len(proof["ops"]) != len(ops) or len(proof["bound"]) != len(proof["binds"]):
        return False
    wcols = {c[9]: c for c in proof["witness_columns"]}
    tcols = {c[1]: c for c in proof["table_columns"]}
    for op, p in zip(ops, proof["ops"]):
        k = op.kind
        if p[0] != k:
            return False
        if k == "MatMul":
            _, claimed, rounds, f, h, _, _, ch = p
            ok = o.sumcheck_verify(rounds, claimed, ch, f, h)
        elif k == "Projection":
            _, mm, aff, frac, alpha, beta, pt, u, v, ch = p
            lg = len(frac[3])
            ok = o.projection_verify(dict(claimed=mm[0], mm_rounds=mm[1], mm_finals=[mm[2], mm[3]], ch=ch,
                                          affine_rounds=aff[0], affine_finals=aff[1], pt=pt, full_r=frac[3],
                                          cs=[l[1] for l in frac[0]], frac_rounds=[l[2] for l in frac[0]],
                                          frac_finals=[l[3] for l in frac[0]], final_num=frac[1]),
                                     op.shift) if lg else False
        elif k == "Add":
            ok = _verify_virtual(p[1], ADD_TERMS, 0, p[2])
        elif k == "Lookup":
            w, t = wcols.get(op.table), tcols.get(op.table)
            ok = w is not None and t is not None and verify_lookup_split(w[0], t[0])
        elif k == "Softmax":
            ok = verify_softmax_rounded(p)
        elif k == "Layernorm":
            ok = verify_layernorm_chain(p)
        elif k == "LayerNormCentered":
            ok = verify_layer_norm_centered(p, op.n_real)
        elif k == "RmsNorm":
            ok = verify_rms_norm(p, op.n_real)
        elif k == "RoPE":
            ok = verify_rope(p, op.shift)
        elif k == "Scatter":
            ok = verify_scatter(p)
        elif k == "Gather":
            ok = verify_scatter_add(p)
        elif k == "GatherMatMul":
            ok = verify_gather_matmul(p, op.s, op.k)
        elif k == "BatchedMatMul":
            ok = verify_batched_matmul(p, op.s, op.k)
        elif k == "TopKSelect":
            ok = verify_topk(p, op.k)
        elif k == "Argmax":
            ok = verify_argmax(p, op.m, op.n)
        else:
            ok = k in MARKER_KINDS
        if not ok:
            return False
    by_tensor = {}
    for t, pt, ev in proof["claims"]:
        by_tensor.setdefault(t, []).append((pt, ev))
    for t, sp in zip(proof["bound"], proof["binds"]):
        cs = by_tensor.get(t, [])
        if len(cs) < 2 or verify_same_poly(sp, cs) is None:
            return False
    return True
