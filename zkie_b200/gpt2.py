"""GPT-2 op graphs for the shard prover, with synthetic weights.

- ``build_gpt2_layer``: the reference's random single-layer builder
  (crates/zkie-ops/src/compose.rs:4237-4470, Layernorm + SoftmaxIndex arms),
  drawing every weight from the caller's XorShift64 in the reference's order;
  ``reference_layer_roundtrip_case`` replays the store its test
  ``build_gpt2_layer_roundtrip`` (:6211-6259) builds.
- ``gpt2_layer``: one layer of the GPT-2 graph (models/gpt2/src/lib.rs
  build_layer, :48-319: LayerNormCentered, 12 heads of Projection / Scale /
  Transpose / MatMul / StableSoftmaxIndex / Softmax, the head sum, the FFN
  with GeluIndex + Lookup, 176 ops) over a store laid out as build_gpt2
  (:321-372) lays it out, minus the embedding: the layer input, then the exp,
  rsqrt and gelu tables and the causal mask.  The model's weight files are
  not in the tree; the weights are drawn from an XorShift64 with the value
  ranges of the random builder (weights in [0, 50), biases in [-5, 5), norm
  scales in [1, 6)) at the real extents (768 wide, FFN 3072) and zero-padded
  to the graph's powers of two (1024, 4096), as the model's export pads them.
- the lookup tables, from the formulas of the reference's table scripts
  (scripts/extract_exp_table.py, extract_rsqrt_piecewise.py,
  extract_gpt2.py:136-144): exp of [-32, 0] and gelu at scale 2^16, the
  piecewise rsqrt table, and ``causal_mask`` (compose.rs:834-846).

Builders take any store with ``push`` / ``push_idx`` taking numpy arrays (the
device Store, or a host store for the CPU checker).
"""
import ctypes as C
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import lib
from .gkr import XorShift64
from .compose import (Add, Argmax, GeluIndex, Layernorm, LayerNormCentered, Lookup, MatMul, Projection, Scale, Softmax,
                      SoftmaxIndex, StableSoftmaxIndex, Transpose)

P = 0xFFFFFFFF00000001
SCALE = 65536.0


def xorshift_fill(rng, n: int, mod: int, offset: int = 0) -> np.ndarray:
    """n draws ``from_i64((rng.next_u64() % mod) + offset)`` from a product
    XorShift64 (advanced in place)."""
    out = np.zeros(max(n, 1), dtype=np.uint64)
    st = _lib.u64(rng.c.xorshift_state)
    lib.zkie2_xorshift_fill(C.byref(st), n, mod, offset, out.ctypes.data_as(_lib.pu64))
    rng.c.xorshift_state = st.value
    return out[:n]


def from_i64(a) -> np.ndarray:
    a = np.asarray(a, dtype=np.int64)
    u = a.astype(np.uint64)
    neg = a < 0
    u[neg] = np.uint64(P) - (np.uint64(0) - u[neg])
    return u


# ---- tables ----------------------------------------------------------------------------------
def exp_table(bits: int = 21) -> np.ndarray:
    """exp(x) at scale 2^16 for x = (j - 2^bits) / 2^16, j < 2^bits (the
    reference's table: bits = 21, x in [-32, 0))."""
    j = np.arange(1 << bits, dtype=np.float64)
    t = np.clip(np.round(np.exp((j - (1 << bits)) / SCALE) * SCALE), 0, 2 ** 31 - 1).astype(np.int64)
    return from_i64(t)


def gelu_table(bits: int = 24) -> np.ndarray:
    """gelu_new(x) at scale 2^16 for x = (j - 2^(bits-1)) / 2^16."""
    x = (np.arange(1 << bits, dtype=np.float64) - (1 << (bits - 1))) / SCALE
    g = 0.5 * x * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (x + 0.044715 * x ** 3)))
    return from_i64(np.clip(np.round(g * SCALE), -(2 ** 31), 2 ** 31 - 1).astype(np.int64))


RSQRT_TABLE_LEN = (1 << 20) + (1 << 22) + (1 << 21)


def rsqrt_table(length: int = RSQRT_TABLE_LEN) -> np.ndarray:
    """The piecewise rsqrt table (2^20 entries at index scale 2^14, then 2^22
    at step 2^8, then 2^21 at step 2^16), 1/sqrt(var + 1e-6) at scale 2^16;
    its first ``length`` entries."""
    fine, coarse, coarse2 = 1 << 20, 1 << 22, 1 << 21
    raw = np.concatenate([np.arange(fine, dtype=np.float64),
                          fine + np.arange(coarse, dtype=np.float64) * (1 << 8),
                          fine + coarse * (1 << 8) + np.arange(coarse2, dtype=np.float64) * (1 << 16)])[:length]
    t = np.clip(np.round(1.0 / np.sqrt(raw / (1 << 14) + 1e-6) * SCALE), 0, 2 ** 31 - 1).astype(np.int64)
    return from_i64(t)


def causal_mask(m: int) -> np.ndarray:
    """-(2^30) above the diagonal, 0 elsewhere (compose.rs:834-846)."""
    i, j = np.meshgrid(np.arange(m), np.arange(m), indexing="ij")
    return from_i64(np.where(j > i, -(1 << 30), 0).reshape(-1))


# ---- the reference's random builder (compose.rs:4237-4470) -------------------------------------
def build_gpt2_layer(store, x, heads, m, d, ffn, shift, exp_t, gelu_t, rsqrt_t, rng):
    """-> (ops, out): Layernorm, per head three Projections, Transpose,
    MatMul, SoftmaxIndex (256), Softmax, MatMul, Projection; the head sum and
    the residual; Layernorm, the FFN with SoftmaxIndex (64) + Lookup."""
    dh = d // heads
    ops = []
    draw = lambda n, mod, off=0: xorshift_fill(rng, n, mod, off)  # noqa: E731
    ln1_w = store.push(draw(m * d, 5, 1))
    ln1_b = store.push(draw(m * d, 10, -5))
    h = store.push(None)
    ops.append(Layernorm(x, ln1_w, ln1_b, h, rsqrt_t, m, d))
    head_outs = []
    for _ in range(heads):
        wq, wk, wv = (store.push(draw(d * dh, 50)) for _ in range(3))
        wo = store.push(draw(dh * d, 50))
        bq, bk, bv = (store.push(draw(m * dh, 10, -5)) for _ in range(3))
        bo = store.push(draw(m * d, 10, -5))
        q, k, v, qr, kr, vr, kt, scores = (store.push(None) for _ in range(8))
        idx = store.push_idx(None)
        e, probs, attn, out_h, out_h_rem = (store.push(None) for _ in range(5))
        ops += [Projection(h, wq, bq, q, qr, m, d, dh, shift), Projection(h, wk, bk, k, kr, m, d, dh, shift),
                Projection(h, wv, bv, v, vr, m, d, dh, shift), Transpose(k, kt, m, dh),
                MatMul(q, kt, scores, m, dh, m), SoftmaxIndex(scores, idx, 1 << 8),
                Softmax(idx, e, probs, exp_t, m, m), MatMul(probs, v, attn, m, m, dh),
                Projection(attn, wo, bo, out_h, out_h_rem, m, dh, d, shift)]
        head_outs.append(out_h)
    acc = head_outs[0]
    for ho in head_outs[1:]:
        s = store.push(None)
        ops.append(Add(acc, ho, s))
        acc = s
    x2 = store.push(None)
    ops.append(Add(x, acc, x2))
    ln2_w = store.push(draw(m * d, 5, 1))
    ln2_b = store.push(draw(m * d, 10, -5))
    h2 = store.push(None)
    ops.append(Layernorm(x2, ln2_w, ln2_b, h2, rsqrt_t, m, d))
    fc_w = store.push(draw(d * ffn, 50))
    fc_b = store.push(draw(m * ffn, 10, -5))
    proj_w = store.push(draw(ffn * d, 50))
    proj_b = store.push(draw(m * d, 10, -5))
    fc, fc_rem = store.push(None), store.push(None)
    gelu_idx = store.push_idx(None)
    act, proj2, proj2_rem = (store.push(None) for _ in range(3))
    ops += [Projection(h2, fc_w, fc_b, fc, fc_rem, m, d, ffn, shift), SoftmaxIndex(fc, gelu_idx, 64),
            Lookup(gelu_idx, act, gelu_t), Projection(act, proj_w, proj_b, proj2, proj2_rem, m, ffn, d, shift)]
    out = store.push(None)
    ops.append(Add(x2, proj2, out))
    return ops, out


def reference_layer_roundtrip_case(store, rng_cls):
    """The store and ops of build_gpt2_layer_roundtrip (compose.rs:6211-6259):
    XorShift64(0x1D1D), (m, d, ffn, heads, shift) = (4, 8, 16, 2, 8), tables
    of 256 / 64 / 256 entries.  Returns (ops, out, rng) with rng positioned
    where the test's prove_shard draws from it."""
    rng = rng_cls(0x1D1D)
    m, d, ffn, heads, shift = 4, 8, 16, 2, 8
    x = store.push(xorshift_fill(rng, m * d, 50))
    exp_t = store.push(from_i64(np.arange(256) % 255 + 1))
    gelu_t = store.push(from_i64(np.arange(64) ** 2 % 1000))
    rsqrt_t = store.push(from_i64(np.arange(256) % 255 + 1))
    ops, out = build_gpt2_layer(store, x, heads, m, d, ffn, shift, exp_t, gelu_t, rsqrt_t, rng)
    return ops, out, rng


# ---- one layer of the GPT-2 graph (models/gpt2/src/lib.rs:48-319) --------------------------
@dataclass
class LayerShape:
    m: int = 512            # sequence length
    d: int = 1024           # D (768 real)
    d_real: int = 768
    heads: int = 12
    dh: int = 64
    ffn: int = 4096         # FFN (3072 real)
    ffn_real: int = 3072
    shift: int = 16
    exp_bits: int = 21      # StableSoftmaxIndex offset / table length 2^21
    gelu_bits: int = 24     # GeluIndex offset 2^23, table 2^24
    rsqrt_len: int = RSQRT_TABLE_LEN
    vocab: int = 65536      # the padded vocabulary of the tied embedding / lm_head (50257 real)
    vocab_real: int = 50257


GPT2_SMALL = LayerShape()


def _pad2(a, rows, cols):
    out = np.zeros((rows, cols), dtype=np.uint64)
    out[:a.shape[0], :a.shape[1]] = a
    return out


def _pad1(a, n):
    out = np.zeros(n, dtype=np.uint64)
    out[:a.size] = a
    return out


def synthetic_layer_weights(rng, s: LayerShape):
    """Weights of one layer at the real extents, zero-padded: q/k/v/o
    (d_real x d_real), their biases, ln1/ln2 scale and shift, fc (d_real x
    ffn_real), proj (ffn_real x d_real) and their biases, in that order."""
    dr, fr = s.d_real, s.ffn_real
    w = {}
    for name in ("q_w", "k_w", "v_w", "o_w"):
        w[name] = _pad2(xorshift_fill(rng, dr * dr, 50).reshape(dr, dr), s.d, s.d)
    for name in ("q_b", "k_b", "v_b", "o_b"):
        w[name] = _pad1(xorshift_fill(rng, dr, 10, -5), s.d)
    for name in ("ln1", "ln2"):
        w[name + "_w"] = _pad1(xorshift_fill(rng, dr, 5, 1), s.d)
        w[name + "_b"] = _pad1(xorshift_fill(rng, dr, 10, -5), s.d)
    w["fc_w"] = _pad2(xorshift_fill(rng, dr * fr, 50).reshape(dr, fr), s.d, s.ffn)
    w["fc_b"] = _pad1(xorshift_fill(rng, fr, 10, -5), s.ffn)
    w["proj_w"] = _pad2(xorshift_fill(rng, fr * dr, 50).reshape(fr, dr), s.ffn, s.d)
    w["proj_b"] = _pad1(xorshift_fill(rng, dr, 10, -5), s.d)
    return w


def gpt2_layer(store, s: LayerShape, seed: int = 0x6B2):
    """A store holding one GPT-2 layer's inputs and the layer's ops:
    (ops, x, out).  The layer input x is drawn in [0, 50) on the real
    columns (zero padding), then the weights (synthetic_layer_weights)."""
    return gpt2_layers(store, s, 1, seed)


def gpt2_layers(store, s: LayerShape, layers: int, seed: int = 0x6B2):
    """``layers`` GPT-2 layers chained as build_gpt2 chains them (the output
    of layer l is the input of layer l + 1; models/gpt2/src/lib.rs:367-372),
    sharing the tables and the mask: (ops, x, out).  The input x is drawn
    first, then each layer's weights as the layer is built."""
    rng = XorShift64(seed)
    m = s.m
    x_host = _pad2(xorshift_fill(rng, m * s.d_real, 50).reshape(m, s.d_real), m, s.d).reshape(-1)
    x = store.push(x_host)
    exp_t = store.push(exp_table(s.exp_bits))
    rsqrt_t = store.push(rsqrt_table(s.rsqrt_len))
    gelu_t = store.push(gelu_table(s.gelu_bits))
    mask_t = store.push(causal_mask(m))
    ops, cur = [], x
    for _ in range(layers):
        layer_ops, cur = build_layer(store, s, cur, synthetic_layer_weights(rng, s), exp_t, rsqrt_t, gelu_t, mask_t)
        ops += layer_ops
    return ops, x, cur


def build_layer(store, s: LayerShape, x, w, exp_t, rsqrt_t, gelu_t, mask_t):
    """models/gpt2/src/lib.rs build_layer (:48-319) over weights w
    (synthetic_layer_weights): -> (ops, out)."""
    m, D, DH = s.m, s.d, s.dh
    bc = lambda v: np.tile(v, m)  # noqa: E731  broadcast a row vector over m rows
    ops = []
    ln1_w, ln1_b = store.push(bc(w["ln1_w"])), store.push(bc(w["ln1_b"]))
    h = store.push(None)
    ops.append(LayerNormCentered(x, ln1_w, ln1_b, h, rsqrt_t, m, D, s.d_real))
    head_outs = []
    for head in range(s.heads):
        cols = slice(head * DH, (head + 1) * DH)
        qh = store.push(np.ascontiguousarray(w["q_w"][:, cols]).reshape(-1))
        kh = store.push(np.ascontiguousarray(w["k_w"][:, cols]).reshape(-1))
        vh = store.push(np.ascontiguousarray(w["v_w"][:, cols]).reshape(-1))
        oh = store.push(np.ascontiguousarray(w["o_w"][cols, :]).reshape(-1))
        qb, kb, vb = (store.push(bc(w[n][cols])) for n in ("q_b", "k_b", "v_b"))
        ob = store.push(np.zeros(m * D, dtype=np.uint64))
        q, k, v, q_s, k_s, qr, kr, vr, kt, scores, scores_16 = (store.push(None) for _ in range(11))
        idx = store.push_idx(None)
        e, probs, attn, attn_16, out_h, out_rem = (store.push(None) for _ in range(6))
        ops += [Projection(h, qh, qb, q, qr, m, D, DH, s.shift), Projection(h, kh, kb, k, kr, m, D, DH, s.shift),
                Projection(h, vh, vb, v, vr, m, D, DH, s.shift), Scale(q, q_s, 23170, 16),
                Scale(k, k_s, 23170, 16), Transpose(k_s, kt, m, DH), MatMul(q_s, kt, scores, m, DH, m),
                Scale(scores, scores_16, 1, 16),
                StableSoftmaxIndex(scores_16, mask_t, idx, 1 << s.exp_bits, 1 << s.exp_bits, m, m),
                Softmax(idx, e, probs, exp_t, m, m), MatMul(probs, v, attn, m, m, DH), Scale(attn, attn_16, 1, 16),
                Projection(attn_16, oh, ob, out_h, out_rem, m, DH, D, s.shift)]
        head_outs.append(out_h)
    acc = head_outs[0]
    for ho in head_outs[1:]:
        t = store.push(None)
        ops.append(Add(acc, ho, t))
        acc = t
    o_b = store.push(bc(w["o_b"]))
    attn_biased = store.push(None)
    ops.append(Add(acc, o_b, attn_biased))
    x2 = store.push(None)
    ops.append(Add(x, attn_biased, x2))
    ln2_w, ln2_b = store.push(bc(w["ln2_w"])), store.push(bc(w["ln2_b"]))
    h2 = store.push(None)
    ops.append(LayerNormCentered(x2, ln2_w, ln2_b, h2, rsqrt_t, m, D, s.d_real))
    fc_w, fc_b = store.push(w["fc_w"].reshape(-1)), store.push(bc(w["fc_b"]))
    proj_w, proj_b = store.push(w["proj_w"].reshape(-1)), store.push(bc(w["proj_b"]))
    fc, fc_rem = store.push(None), store.push(None)
    gelu_idx = store.push_idx(None)
    act, proj2, proj2_rem = (store.push(None) for _ in range(3))
    ops += [Projection(h2, fc_w, fc_b, fc, fc_rem, m, D, s.ffn, s.shift),
            GeluIndex(fc, gelu_idx, 1 << (s.gelu_bits - 1), 1 << s.gelu_bits), Lookup(gelu_idx, act, gelu_t),
            Projection(act, proj_w, proj_b, proj2, proj2_rem, m, s.ffn, D, s.shift)]
    out = store.push(None)
    ops.append(Add(x2, proj2, out))
    return ops, out


def gpt2_model(store, s: LayerShape, layers: int = 12, seed: int = 0x6B2):
    """The GPT-2 graph of build_gpt2 (models/gpt2/src/lib.rs:321-436): the
    token embedding as a Lookup into the tied lm_head table (emb_idx[i D + d]
    = d vocab + token_i) plus the position embedding, ``layers`` layers, the
    final LayerNormCentered, the lm_head MatMul, the vocabulary mask Add and
    the Argmax over the masked logits (the next token of every position, a
    public index tensor).  Synthetic inputs: the tokens (below vocab_real),
    the position embedding, the lm_head weights (d_real x vocab_real,
    zero-padded) and the final norm's scale and shift, drawn after the
    layers' weights.  Returns (ops, tokens index id, argmax index id)."""
    rng = XorShift64(seed)
    m, D, V = s.m, s.d, s.vocab
    tokens = np.array([int(t) % s.vocab_real for t in xorshift_fill(rng, m, 1 << 30)], dtype=np.uint32)
    lm_w = _pad2(xorshift_fill(rng, s.d_real * s.vocab_real, 50).reshape(s.d_real, s.vocab_real), D, V)
    pos = _pad2(xorshift_fill(rng, m * s.d_real, 50).reshape(m, s.d_real), m, D).reshape(-1)
    tok_t = store.push_idx(tokens)
    emb_idx = (np.arange(D, dtype=np.uint64)[None, :] * V + tokens.astype(np.uint64)[:, None]).reshape(-1)
    emb_t = store.push_idx(emb_idx.astype(np.uint32))
    wte = store.push(lm_w.reshape(-1))
    token_emb = store.push(None)
    ops = [Lookup(emb_t, token_emb, wte)]
    pos_t = store.push(pos)
    x0 = store.push(None)
    ops.append(Add(token_emb, pos_t, x0))
    exp_t = store.push(exp_table(s.exp_bits))
    rsqrt_t = store.push(rsqrt_table(s.rsqrt_len))
    gelu_t = store.push(gelu_table(s.gelu_bits))
    mask_t = store.push(causal_mask(m))
    cur = x0
    for _ in range(layers):
        layer_ops, cur = build_layer(store, s, cur, synthetic_layer_weights(rng, s), exp_t, rsqrt_t, gelu_t, mask_t)
        ops += layer_ops
    bc = lambda v: np.tile(v, m)  # noqa: E731
    lnf_w = store.push(bc(_pad1(xorshift_fill(rng, s.d_real, 5, 1), D)))
    lnf_b = store.push(bc(_pad1(xorshift_fill(rng, s.d_real, 10, -5), D)))
    h_final = store.push(None)
    ops.append(LayerNormCentered(cur, lnf_w, lnf_b, h_final, rsqrt_t, m, D, s.d_real))
    lm_t = store.push(lm_w.reshape(-1))
    logits = store.push(None)
    ops.append(MatMul(h_final, lm_t, logits, m, D, V))
    vmask = from_i64(np.where(np.arange(V) < s.vocab_real, 0, -(1 << 41)))
    mask_v = store.push(np.tile(vmask, m))
    logits_masked = store.push(None)
    ops.append(Add(logits, mask_v, logits_masked))
    sel, thr, gate, d1, d2 = (store.push(None) for _ in range(5))
    out = store.push_idx(None)
    ops.append(Argmax(logits_masked, sel, thr, gate, d1, d2, out, m, V))
    return ops, tok_t, out
