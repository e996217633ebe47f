"""The CPU restatement of the MLA / MoE arms (oracle/compose_oracle.py), no
GPU: the reference's own roundtrip tests of rms_norm.rs, rope.rs, scatter.rs,
gather.rs and common/batched_matmul.rs replayed (same seeds and inputs), each
forward against a direct restatement of its definition, and tampered proofs
rejected."""
import copy

import numpy as np
import pytest

from oracle import compose_oracle as co
from oracle import oracle as o

P = co.P


def _fe(vals):
    return co.from_i64(np.asarray(vals, dtype=np.int64))


def test_reference_rms_norm_roundtrip():
    """rms_norm.rs tests::rms_norm_roundtrip (:228-248): seed 0x12345678, m 4,
    d 8, n_real 5, a constant rsqrt table."""
    m, d, n_real = 4, 8, 5
    x = _fe([(i % 97) - 48 for i in range(m * d)])
    w = _fe([(i % 13) + 1 for i in range(m * d)])
    table = _fe([65536] * 64)
    p, f = co.prove_rms_norm(x, w, table, m, d, n_real, o.XorShift64(0x12345678))
    assert co.verify_rms_norm(p, n_real)
    xi = co.to_i64(x).reshape(m, d)
    for r in range(m):  # ms = round(sum of squares over n_real / n_real)
        s = sum(int(v) * int(v) for v in xi[r, :n_real])
        q, rem = divmod(s, n_real)
        assert int(co.to_i64(f["ms"][r:r + 1])[0]) == q + (1 if 2 * rem >= n_real else 0)
    ro = co.to_i64(f["rem_out"])
    assert ((0 <= ro) & (ro < (1 << 32))).all()
    assert np.array_equal(co.to_i64(f["rem_lo"]) + (co.to_i64(f["rem_hi"]) << 16), ro)
    bad = copy.deepcopy(p)
    bad[2][1][4] = (int(bad[2][1][4]) + 1) % P  # out (raw appears with coefficient -1 + 1)
    assert not co.verify_rms_norm(bad, n_real)


def test_reference_rope_roundtrip():
    """rope.rs tests::rope_roundtrip (:242-261): seed 0x0D0D0001, m 4, 2 heads,
    d 8, cos 1.0 and sin 0 (the identity rotation), plus a real rotation
    checked against the rotate-half definition."""
    m, heads, d, shift = 4, 2, 8, 16
    x = _fe([(i % 97) - 48 for i in range(m * heads * d)])
    cos, sin = _fe([65536] * (m * d // 2)), _fe([0] * (m * d // 2))
    out, _, _ = co.rope_forward(x, cos, sin, m, d, shift)
    assert np.array_equal(out, x)
    p, _, _ = co.prove_rope(x, cos, sin, out, m, d, shift, o.XorShift64(0x0D0D0001))
    assert co.verify_rope(p, shift)
    rng = np.random.default_rng(3)
    cos = _fe(rng.integers(-65536, 65536, size=m * d // 2))
    sin = _fe(rng.integers(-65536, 65536, size=m * d // 2))
    x = _fe(rng.integers(-(1 << 20), 1 << 20, size=m * heads * d))
    out, rem_f, rem_s = co.rope_forward(x, cos, sin, m, d, shift)
    xi, ci, si, oi = (co.to_i64(v) for v in (x, cos, sin, out))
    h = d // 2
    for pp in range(m):
        for hh in range(heads):
            for i in range(h):
                xf, xs = int(xi[(pp * heads + hh) * d + i]), int(xi[(pp * heads + hh) * d + h + i])
                c, s = int(ci[pp * h + i]), int(si[pp * h + i])
                for raw, got in ((xf * c - xs * s, oi[(pp * heads + hh) * d + i]),
                                 (xs * c + xf * s, oi[(pp * heads + hh) * d + h + i])):
                    q, r = divmod(raw, 1 << shift)
                    assert int(got) == q + (1 if 2 * r >= (1 << shift) else 0)
    assert (co.to_i64(rem_f) >= 0).all() and (co.to_i64(rem_s) < (1 << shift)).all()
    p, _, _ = co.prove_rope(x, cos, sin, out, m, d, shift, o.XorShift64(5))
    assert co.verify_rope(p, shift)
    assert not co.verify_rope(p, shift - 1)


def _two_hot(m, n):
    sel = np.zeros(m * n, dtype=np.uint64)
    for t in range(m):
        sel[t * n + (t % n)] = 1
        sel[t * n + ((t + 1) % n)] = 1
    return sel


def test_reference_scatter_roundtrip():
    """scatter.rs tests::scatter_roundtrip (:65-78): seed 0x4242, 4 tokens each
    routed to experts t and t + 1 of 4; a wrong token order fails."""
    m, n = 4, 4
    sel = _two_hot(m, n)
    tid, eof = co.scatter_forward(sel, m, n)
    assert tid.size == 2 * m
    assert list(eof) == sorted(eof)  # expert-major
    p = co.prove_scatter(sel, tid, eof, m, n, o.XorShift64(0x4242))
    assert co.verify_scatter(p)
    bad = tid.copy()
    bad[0] = (bad[0] + 1) % m
    assert not co.verify_scatter(co.prove_scatter(sel, bad, eof, m, n, o.XorShift64(0x4242)))


@pytest.mark.parametrize("seed,gate", [(0x777, [1, 1, 1, 1]), (0x888, [2, 3, 5, 7])])
def test_reference_scatter_add_roundtrips(seed, gate):
    """gather.rs tests::scatter_add_roundtrip (:191-213) and
    scatter_add_weighted_roundtrip (:217-242): token_id [0, 2, 1, 2], h 2."""
    m, h = 4, 2
    tid = np.array([0, 2, 1, 2], dtype=np.uint32)
    gate = np.array(gate, dtype=np.uint64)
    weighted = np.array([(i % 5) + 1 for i in range(tid.size * h)], dtype=np.uint64)
    out = co.gather_forward(weighted, tid, gate, m, h)
    expect = np.zeros(m * h, dtype=np.uint64)
    for pos, t in enumerate(tid):
        for dd in range(h):
            expect[t * h + dd] = (int(expect[t * h + dd]) + int(weighted[pos * h + dd]) * int(gate[pos])) % P
    assert np.array_equal(out, expect)
    p = co.prove_scatter_add(weighted, tid, gate, out, m, h, o.XorShift64(seed))
    assert co.verify_scatter_add(p)
    wrong = out.copy()
    wrong[0] = (int(wrong[0]) + 1) % P
    assert not co.verify_scatter_add(co.prove_scatter_add(weighted, tid, gate, wrong, m, h, o.XorShift64(seed)))


def test_reference_gather_matmul_self_contained():
    """batched_matmul.rs gather_matmul_proof_tests (:519-546): seed 0x7171,
    s 8, k 4, n 2, 4 experts; a tampered weight claim fails."""
    s, k, n, ne = 8, 4, 2, 4
    w_all = np.array([(i % 7) + 1 for i in range(ne * k * n)], dtype=np.uint64)
    e_of = np.array([i % ne for i in range(s)], dtype=np.uint32)
    seg = np.array([(i % 11) + 1 for i in range(s * k)], dtype=np.uint64)
    g = co.gather_matmul_forward(seg, e_of, w_all, s, k, n, ne)
    want = np.zeros(s * n, dtype=np.uint64)
    for pos in range(s):
        for j in range(n):
            want[pos * n + j] = sum(int(seg[pos * k + dd]) * int(w_all[int(e_of[pos]) * k * n + dd * n + j])
                                    for dd in range(k)) % P
    assert np.array_equal(g, want)
    rng = o.XorShift64(0x7171)
    u, v, ch = rng.fields(3), rng.fields(1), rng.fields(5)
    p = co.prove_gather_matmul(seg, e_of, w_all, g, s, k, n, ne, u, v, ch)
    op_proof = ("GatherMatMul", p, u, v, ch)
    assert co.verify_gather_matmul(op_proof, s, k)
    claimed, (rounds, finals), counts, table = p
    assert int(finals[0]) == int(o.mle_eval(seg, ch))
    bad_f = finals.copy()
    bad_f[1] = (int(bad_f[1]) + 1) % P
    assert not co.verify_gather_matmul(("GatherMatMul", (claimed, (rounds, bad_f), counts, table), u, v, ch), s, k)


def test_reference_expert_major_bmm_closure():
    """gather.rs moe_bmm::expert_major_bmm_closure (:309-391): scatter, the
    per-expert matmul and the scatter-add equal the dense top-2 MoE."""
    m, n, h, pdim = 4, 4, 4, 2
    sel = _two_hot(m, n)
    gate = np.array([(i % 3) + 1 for i in range(m * n)], dtype=np.uint64)
    x = np.array([(i % 7) + 1 for i in range(m * h)], dtype=np.uint64)
    eg_all = np.array([(i % 5) + 1 for i in range(n * h * pdim)], dtype=np.uint64)
    tid, eof = co.scatter_forward(sel, m, n)
    s = tid.size
    seg = x.reshape(m, h)[tid.astype(np.int64)].reshape(-1)
    g = co.gather_matmul_forward(seg, eof, eg_all, s, h, pdim, n)
    weighted = o.vec_mul(g, np.repeat(gate.reshape(m, n)[tid.astype(np.int64), eof.astype(np.int64)], pdim))
    out = co.gather_forward(weighted, tid, np.ones(s, dtype=np.uint64), m, pdim)
    ref = np.zeros(m * pdim, dtype=np.uint64)
    for t in range(m):
        for e in range(n):
            if sel[t * n + e] == 1:
                for j in range(pdim):
                    acc = sum(int(x[t * h + dd]) * int(eg_all[e * h * pdim + dd * pdim + j]) for dd in range(h))
                    ref[t * pdim + j] = (int(ref[t * pdim + j]) + acc * int(gate[t * n + e])) % P
    assert np.array_equal(out, ref)
    rng = o.XorShift64(0x1234)
    assert co.verify_scatter(co.prove_scatter(sel, tid, eof, m, n, rng))
    assert co.verify_scatter_add(co.prove_scatter_add(weighted, tid, np.ones(s, dtype=np.uint64), out, m, pdim,
                                                      rng))


SMALL = dict(m=8, h=16, heads=2, qk_nope=4, qk_rope=4, v_head=4, kv_lora=8, n_routed=8, top_k=2, moe=8, moe_real=6,
             shared=16, shared_real=12, exp_bits=8, silu_bits=12, rsqrt_len=1 << 12, w_mod=1 << 12, router_mod=1 << 10)


def test_moe_layer_shard_verifies():
    """A DeepSeek-V2-Lite-shaped MoE layer (zkie_b200.deepseek.moe_layer) at
    a small shape through prove_shard: every arm's proof and every same_poly
    binding accepted; the routing uses more than top_k experts; the layer's
    output differs from its residual input (the experts contribute)."""
    from zkie_b200 import deepseek as ds
    shape = ds.MoeShape(**SMALL)
    st = co.HostStore()
    ops, x, out = ds.moe_layer(st, shape)
    kinds = {op.kind for op in ops}
    assert {"RmsNorm", "RoPE", "Scatter", "Gather", "GatherMatMul", "TopKSelect", "ScaleVec", "BroadcastScale",
            "IdxBroadcast", "CombineIdx", "PadIdx"} <= kinds
    proof = co.prove_shard(st, ops, [], o.XorShift64(9))
    assert co.verify_shard(ops, proof)
    sel = next(op for op in ops if op.kind == "TopKSelect")
    assert int((st.v[sel.sel].reshape(shape.m, shape.n_routed).sum(axis=0) > 0).sum()) > shape.top_k
    res = next(op for op in ops if op.kind == "Add" and op.c == out)
    assert not np.array_equal(st.v[out], st.v[res.a])
    assert proof["bound"], "no tensor was bound by same_poly"


def test_reference_batched_matmul_roundtrip():
    """batched_matmul.rs tests::batched_matmul_roundtrip (:164-215): seed
    0xbeef, s 4, k 4, n 2, the weights gathered from 3 experts; the endpoint
    evaluations are a at ch and w contracted with eq(v) at ch; a tampered
    claim fails."""
    s, k, n, ne = 4, 4, 2, 3
    w_all = np.array([(i % 7) + 1 for i in range(ne * k * n)], dtype=np.uint64).reshape(ne, k, n)
    e_of = np.array([i % ne for i in range(s)])
    w = w_all[e_of].reshape(-1)
    seg = np.array([(i % 11) + 1 for i in range(s * k)], dtype=np.uint64)
    g = co.batched_matmul_forward(seg, w, s, k, n)
    assert np.array_equal(g, co.gather_matmul_forward(seg, e_of.astype(np.uint32), w_all.reshape(-1), s, k, n, ne))
    rng = o.XorShift64(0xbeef)
    u, v, ch = rng.fields(2), rng.fields(1), rng.fields(4)
    p = co.prove_batched_matmul(seg, w, g, s, k, n, u, v, ch)
    assert co.verify_batched_matmul(("BatchedMatMul", p, u, v, ch), s, k)
    claimed, (rounds, finals) = p
    assert int(finals[0]) == int(o.mle_eval(seg, ch))
    assert int(finals[1]) == int(o.mle_eval(o.mle_partial_eval(w, v), ch))
    assert not co.verify_batched_matmul(("BatchedMatMul", ((claimed + 1) % P, (rounds, finals)), u, v, ch), s, k)


def relu_gate_bmm_shard(C, store, s=8, k=16, n=4, m=2, h=8):
    """Relu, ScaleGate and BatchedMatMul chained (the arms of the Gemma /
    TimesFM graphs): -> ops."""
    rng = np.random.default_rng(s + k)
    x = store.push(co.from_i64(rng.integers(-(1 << 20), 1 << 20, size=s * k)))
    w = store.push(co.from_i64(rng.integers(-(1 << 12), 1 << 12, size=s * k * n)))
    gate = store.push(co.from_i64(rng.integers(-(1 << 16), 1 << 16, size=m * n)))
    r, c, sg = store.push(None), store.push(None), store.push(None)
    return [C.Relu(x, r), C.BatchedMatMul(r, w, c, s, k, n), C.ScaleGate(c, gate, 1, sg, m, n, (s * n) // m, 8)]


def test_relu_scale_gate_batched_matmul_shard_verifies():
    from zkie_b200 import compose as C
    st = co.HostStore()
    ops = relu_gate_bmm_shard(C, st)
    proof = co.prove_shard(st, ops, [], o.XorShift64(4))
    assert co.verify_shard(ops, proof)
    xi = co.to_i64(st.v[ops[0].x])
    assert np.array_equal(co.to_i64(st.v[ops[0].out]), np.maximum(xi, 0))
