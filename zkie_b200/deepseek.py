"""A DeepSeek-V2-Lite-shaped MoE layer as an op graph (models/deepseek-v2-lite/
src/lib.rs: build_attention :57-250, build_moe :252-470 and one layer of the
loop in build_deepseek :620-672), with synthetic weights in place of the
reference's weight files.

Shapes follow the reference: hidden 2048, MLA with 16 heads (q/k nope 128,
rope 64, v 128, kv_lora 512), 64 routed experts (top 6, expert FFN padded to
2048 with 1408 real columns) plus the shared experts (4096 padded, 2816 real),
sequence 512, shift 16.  The routed experts run expert-major as in the
reference: TopKSelect over the router's softmax, Scatter into expert order,
per-expert GatherMatMul for gate / up / down, SiLU by lookup, the gate
values gathered back by (token, expert), and Gather (scatter-add) into token
order.  The tables are the reference's kinds: exp (2^21), the piecewise rsqrt,
the 2^16 limb range, SiLU at scale 2^16 over 2^24 points, the causal mask and
RoPE's cos / sin at scale 2^16.
"""
from dataclasses import dataclass

import numpy as np

from .compose import (Add, BroadcastScale, CombineIdx, Gather, GatherMatMul, GeluIndex, IdxBroadcast, Lookup,
                      MatMul, PadIdx, Projection, RmsNorm, RoPE, Scale, ScaleVec, Scatter, Softmax, StableSoftmaxIndex,
                      TopKSelect, Transpose)
from .gkr import XorShift64
from .gpt2 import RSQRT_TABLE_LEN, SCALE, _pad2, causal_mask, exp_table, from_i64, rsqrt_table, xorshift_fill


@dataclass(frozen=True)
class MoeShape:
    m: int = 512            # sequence length
    h: int = 2048           # hidden
    heads: int = 16
    qk_nope: int = 128
    qk_rope: int = 64
    v_head: int = 128
    kv_lora: int = 512
    n_routed: int = 64
    top_k: int = 6
    moe: int = 2048         # routed expert FFN, padded (1408 real)
    moe_real: int = 1408
    shared: int = 4096      # shared experts' FFN, padded (2816 real)
    shared_real: int = 2816
    shift: int = 16
    exp_bits: int = 21
    silu_bits: int = 24
    rsqrt_len: int = RSQRT_TABLE_LEN
    w_mod: int = 50          # weights drawn in [0, w_mod)
    router_mod: int = 1 << 10  # router weights in [-router_mod / 2, router_mod / 2): routing spread over the experts


DSV2_LITE = MoeShape()


def silu_table(bits: int = 24) -> np.ndarray:
    """silu(x) = x sigmoid(x) at scale 2^16 for x = (j - 2^(bits-1)) / 2^16."""
    x = (np.arange(1 << bits, dtype=np.float64) - (1 << (bits - 1))) / SCALE
    y = x / (1.0 + np.exp(-np.clip(x, -700, 700)))
    return from_i64(np.clip(np.round(y * SCALE), -(2 ** 31), 2 ** 31 - 1).astype(np.int64))


def rope_tables(m: int, rope: int, base: float = 10000.0):
    """cos / sin (m x rope/2) of p theta_i, theta_i = base^(-2 i / rope), at scale 2^16."""
    half = rope // 2
    ang = np.arange(m, dtype=np.float64)[:, None] * base ** (-2.0 * np.arange(half) / rope)[None, :]
    q = lambda a: from_i64(np.round(a * SCALE).astype(np.int64).reshape(-1))  # noqa: E731
    return q(np.cos(ang)), q(np.sin(ang))


def _draw(rng, n, mod, off=0):
    return xorshift_fill(rng, n, mod, off)


def _norm_weights(rng, n):
    """RMSNorm scales near 1.0 at scale 2^16 (1 +- 2^-5), so the normalised
    activations keep the 2^16 scale the projections' shift assumes."""
    return _draw(rng, n, 1 << 12, (1 << 16) - (1 << 11))


def _cols(mat, cols, c0, c1):
    return np.ascontiguousarray(mat.reshape(-1, cols)[:, c0:c1]).reshape(-1)


def _rows(mat, cols, r0, r1):
    return np.ascontiguousarray(mat.reshape(-1, cols)[r0:r1]).reshape(-1)


def build_attention(store, ops, x, s: MoeShape, t, rng):
    """build_attention (lib.rs:57-250): the shared kv latent (Projection to
    kv_lora, RmsNorm) and the MQA rope key (Projection, RoPE, Transpose), then
    per head the q nope / rope, k nope and v Projections, RoPE on q rope, the
    two score MatMuls, Scale (7519 / 2^32), StableSoftmaxIndex, Softmax, the
    value MatMul, Scale (2^-16) and the output Projection; the head sum."""
    m, H, nope, rp, vh, kvl = s.m, s.h, s.qk_nope, s.qk_rope, s.v_head, s.kv_lora
    zeros = lambda n: np.zeros(n, dtype=np.uint64)  # noqa: E731
    wm = s.w_mod
    qnope_w = _draw(rng, H * s.heads * nope, wm)
    qpe_w = _draw(rng, H * s.heads * rp, wm)
    kvlora_w = _draw(rng, H * kvl, wm)
    kpe_w = _draw(rng, H * rp, wm)
    kva_ln = _norm_weights(rng, kvl)
    knope_w = _draw(rng, kvl * s.heads * nope, wm)
    v_w = _draw(rng, kvl * s.heads * vh, wm)
    o_w = _draw(rng, s.heads * vh * H, wm)
    kvlora_w_t, kpe_w_t = store.push(kvlora_w), store.push(kpe_w)
    kv_b, kpe_b = store.push(zeros(m * kvl)), store.push(zeros(m * rp))
    kvlora, kvlora_rem, kpe, kpe_rem = (store.push(None) for _ in range(4))
    ops.append(Projection(x, kvlora_w_t, kv_b, kvlora, kvlora_rem, m, H, kvl, s.shift))
    ops.append(Projection(x, kpe_w_t, kpe_b, kpe, kpe_rem, m, H, rp, s.shift))
    kva_ln_t = store.push(np.tile(kva_ln, m))
    kvlora_n = store.push(None)
    ops.append(RmsNorm(kvlora, kva_ln_t, kvlora_n, t["rsqrt"], t["limb"], m, kvl, kvl))
    kpe_rot = store.push(None)
    ops.append(RoPE(kpe, t["cos"], t["sin"], kpe_rot, t["limb"], m, rp, s.shift))
    kt = store.push(None)
    ops.append(Transpose(kpe_rot, kt, m, rp))
    head_outs = []
    for hd in range(s.heads):
        qn_w = store.push(_cols(qnope_w, s.heads * nope, hd * nope, (hd + 1) * nope))
        qp_w = store.push(_cols(qpe_w, s.heads * rp, hd * rp, (hd + 1) * rp))
        kn_w = store.push(_cols(knope_w, s.heads * nope, hd * nope, (hd + 1) * nope))
        vh_w = store.push(_cols(v_w, s.heads * vh, hd * vh, (hd + 1) * vh))
        oh = store.push(_rows(o_w, H, hd * vh, (hd + 1) * vh))
        qn, qn_rem, qp, qp_rem, kn, kn_rem, vv, vv_rem = (store.push(None) for _ in range(8))
        ops.append(Projection(x, qn_w, store.push(zeros(m * nope)), qn, qn_rem, m, H, nope, s.shift))
        ops.append(Projection(x, qp_w, store.push(zeros(m * rp)), qp, qp_rem, m, H, rp, s.shift))
        ops.append(Projection(kvlora_n, kn_w, store.push(zeros(m * nope)), kn, kn_rem, m, kvl, nope, s.shift))
        ops.append(Projection(kvlora_n, vh_w, store.push(zeros(m * vh)), vv, vv_rem, m, kvl, vh, s.shift))
        qp_rot = store.push(None)
        ops.append(RoPE(qp, t["cos"], t["sin"], qp_rot, t["limb"], m, rp, s.shift))
        knt = store.push(None)
        ops.append(Transpose(kn, knt, m, nope))
        s_nope, s_rope, sc, s16 = (store.push(None) for _ in range(4))
        idx = store.push_idx(None)
        e, probs, attn, attn16, out_h, out_rem = (store.push(None) for _ in range(6))
        ops += [MatMul(qn, knt, s_nope, m, nope, m), MatMul(qp_rot, kt, s_rope, m, rp, m), Add(s_nope, s_rope, sc),
                Scale(sc, s16, 7519, 32),
                StableSoftmaxIndex(s16, t["mask"], idx, 1 << s.exp_bits, 1 << s.exp_bits, m, m),
                Softmax(idx, e, probs, t["exp"], m, m), MatMul(probs, vv, attn, m, m, vh), Scale(attn, attn16, 1, 16)]
        ops.append(Projection(attn16, oh, store.push(zeros(m * H)), out_h, out_rem, m, vh, H, s.shift))
        head_outs.append(out_h)
    acc = head_outs[0]
    for ho in head_outs[1:]:
        nxt = store.push(None)
        ops.append(Add(acc, ho, nxt))
        acc = nxt
    return acc


def build_moe(store, ops, x, s: MoeShape, t, rng):
    """build_moe (lib.rs:252-470): router MatMul, Scale, StableSoftmaxIndex,
    Softmax, TopKSelect (6 of 64); Scatter into expert order, PadIdx to a
    power of two, the token rows gathered by Lookup and zeroed past the real
    positions (BroadcastScale); gate / up GatherMatMuls with Scale, SiLU by
    GeluIndex + Lookup, ScaleVec, the down GatherMatMul with Scale; the gate
    values by CombineIdx + Lookup, BroadcastScale, Scale and Gather back to
    token order; the shared experts as Projections with SiLU; the sum."""
    m, H, E, F, wm = s.m, s.h, s.n_routed, s.moe, s.w_mod
    zeros = lambda n: np.zeros(n, dtype=np.uint64)  # noqa: E731
    router_t = store.push(_draw(rng, H * E, s.router_mod, -(s.router_mod // 2)))
    logits, logits_16 = store.push(None), store.push(None)
    ops += [MatMul(x, router_t, logits, m, H, E), Scale(logits, logits_16, 1, 16)]
    zero_mask = store.push(zeros(m * E))
    scores_idx = store.push_idx(None)
    ops.append(StableSoftmaxIndex(logits_16, zero_mask, scores_idx, 1 << s.exp_bits, 1 << s.exp_bits, m, E))
    scores_e, scores = store.push(None), store.push(None)
    ops.append(Softmax(scores_idx, scores_e, scores, t["exp"], m, E))
    sel, thr, gate, d1, d2 = (store.push(None) for _ in range(5))
    ops.append(TopKSelect(scores, sel, thr, gate, d1, d2, m, E, s.top_k))
    shared_g = _pad2(_draw(rng, H * s.shared_real, wm).reshape(H, s.shared_real), H, s.shared).reshape(-1)
    shared_u = _pad2(_draw(rng, H * s.shared_real, wm).reshape(H, s.shared_real), H, s.shared).reshape(-1)
    shared_d = _pad2(_draw(rng, s.shared_real * H, wm).reshape(s.shared_real, H), s.shared, H).reshape(-1)
    experts = lambda k, n, kr, nr: np.stack([_pad2(_draw(rng, kr * nr, wm).reshape(kr, nr), k, n)  # noqa: E731
                                             for _ in range(E)]).reshape(-1)
    eg, eu = experts(H, F, H, s.moe_real), experts(H, F, H, s.moe_real)
    ed = experts(F, H, s.moe_real, H)
    n_pos = s.top_k * m
    s_pad = 1 << max(n_pos - 1, 0).bit_length()
    token_id, expert_of = store.push_idx(None), store.push_idx(None)
    ops.append(Scatter(sel, token_id, expert_of, m, E))
    token_id_pad, expert_of_pad = store.push_idx(None), store.push_idx(None)
    ops += [PadIdx(token_id, token_id_pad, s_pad), PadIdx(expert_of, expert_of_pad, s_pad)]
    idx_seg = store.push_idx(None)
    ops.append(IdxBroadcast(token_id_pad, idx_seg, H))
    seg = store.push(None)
    ops.append(Lookup(idx_seg, seg, x))
    pos_mask = zeros(s_pad)
    pos_mask[:n_pos] = 1
    mask_t = store.push(pos_mask)
    seg_z = store.push(None)
    ops.append(BroadcastScale(seg, mask_t, seg_z, H))
    eg_full, eu_full, ed_full = store.push(eg), store.push(eu), store.push(ed)
    g_raw, g = store.push(None), store.push(None)
    ops += [GatherMatMul(seg_z, expert_of_pad, eg_full, g_raw, s_pad, H, F, E), Scale(g_raw, g, 1, 16)]
    u_raw, u = store.push(None), store.push(None)
    ops += [GatherMatMul(seg_z, expert_of_pad, eu_full, u_raw, s_pad, H, F, E), Scale(u_raw, u, 1, 16)]
    silu_idx = store.push_idx(None)
    silu, act = store.push(None), store.push(None)
    ops += [GeluIndex(g, silu_idx, 1 << (s.silu_bits - 1), 1 << s.silu_bits), Lookup(silu_idx, silu, t["silu"]),
            ScaleVec(silu, u, act, 16)]
    d_raw, dd = store.push(None), store.push(None)
    ops += [GatherMatMul(act, expert_of_pad, ed_full, d_raw, s_pad, F, H, E), Scale(d_raw, dd, 1, 16)]
    idx_gate = store.push_idx(None)
    ops.append(CombineIdx(token_id_pad, expert_of_pad, idx_gate, E))
    gate_pos = store.push(None)
    ops.append(Lookup(idx_gate, gate_pos, gate))
    weighted_raw, weighted = store.push(None), store.push(None)
    ops += [BroadcastScale(dd, gate_pos, weighted_raw, H), Scale(weighted_raw, weighted, 1, 16)]
    gate_ones = store.push(np.ones(s_pad, dtype=np.uint64))
    out = store.push(None)
    ops.append(Gather(weighted, token_id_pad, gate_ones, out, m, H))
    sg_w, su_w, sd_w = store.push(shared_g), store.push(shared_u), store.push(shared_d)
    sg, sg_rem, su, su_rem = (store.push(None) for _ in range(4))
    ss_idx = store.push_idx(None)
    ss, sa, sd, sd_rem = (store.push(None) for _ in range(4))
    ops += [Projection(x, sg_w, store.push(zeros(m * s.shared)), sg, sg_rem, m, H, s.shared, s.shift),
            Projection(x, su_w, store.push(zeros(m * s.shared)), su, su_rem, m, H, s.shared, s.shift),
            GeluIndex(sg, ss_idx, 1 << (s.silu_bits - 1), 1 << s.silu_bits), Lookup(ss_idx, ss, t["silu"]),
            ScaleVec(ss, su, sa, 16),
            Projection(sa, sd_w, store.push(zeros(m * H)), sd, sd_rem, m, s.shared, H, s.shift)]
    total = store.push(None)
    ops.append(Add(out, sd, total))
    return total


def moe_layer(store, s: MoeShape = DSV2_LITE, seed: int = 0xD5E):
    """One MoE layer (a layer >= 1 of build_deepseek, lib.rs:620-672) over a
    synthetic input: (ops, x, out).  The input x (m x hidden, drawn in [0,
    2^12)) comes first, then the tables, then the weights as the layer is
    built."""
    rng = XorShift64(seed)
    m, H = s.m, s.h
    x = store.push(_draw(rng, m * H, 1 << 12))
    cos, sin = rope_tables(m, s.qk_rope)
    t = {"exp": store.push(exp_table(s.exp_bits)), "rsqrt": store.push(rsqrt_table(s.rsqrt_len)),
         "limb": store.push(np.arange(1 << 16, dtype=np.uint64)), "silu": store.push(silu_table(s.silu_bits)),
         "mask": store.push(causal_mask(m)), "cos": store.push(cos), "sin": store.push(sin)}
    ops = []
    in_norm = store.push(np.tile(_norm_weights(rng, H), m))
    hn = store.push(None)
    ops.append(RmsNorm(x, in_norm, hn, t["rsqrt"], t["limb"], m, H, H))
    attn = build_attention(store, ops, hn, s, t, rng)
    x2 = store.push(None)
    ops.append(Add(x, attn, x2))
    post_norm = store.push(np.tile(_norm_weights(rng, H), m))
    h2 = store.push(None)
    ops.append(RmsNorm(x2, post_norm, h2, t["rsqrt"], t["limb"], m, H, H))
    ff = build_moe(store, ops, h2, s, t, rng)
    x3 = store.push(None)
    ops.append(Add(x2, ff, x3))
    return ops, x, x3

