"""The CPU restatement of the op-layer shard prover (oracle/compose_oracle.py),
no GPU: its fixed-point helpers against the reference's semantics, its proofs
against its restatement of the reference's verifier (verify_shard_precomputed,
compose.rs:2103-2239), the reference's own layer test replayed
(build_gpt2_layer_roundtrip, compose.rs:6211-6259), and the identity the
device same_poly relies on."""
import copy

import numpy as np
import pytest

from oracle import compose_oracle as co
from oracle import oracle as o
from zkie_b200 import gpt2
from zkie_b200.gkr import XorShift64

P = co.P


def _oracle_rng(product_rng):
    r = o.XorShift64(0)
    r.s.value = product_rng.c.xorshift_state
    return r


def test_round_div_matches_rust_semantics():
    # div_euclid / rem_euclid, plus one when 2 r >= b
    cases = [(7, 2, 4), (-7, 2, -3), (5, 2, 3), (-5, 2, -2), (6, 4, 2), (-6, 4, -1), (7, -2, -2), (-7, -2, 5),
             (0, 3, 0), (1, 3, 0), (2, 3, 1), (-1, 3, 0), (-2, 3, -1)]
    for a, b, want in cases:
        assert int(co.round_div(np.array([a]), b)[0]) == want, (a, b)
    with pytest.raises(ZeroDivisionError):
        co.round_div(np.array([1]), 0)


def test_fixed_point_roundtrip_and_rsqrt_index():
    x = np.array([0, 1, -1, 2 ** 40, -(2 ** 40), 2 ** 62, -(2 ** 62)], dtype=np.int64)
    assert np.array_equal(co.to_i64(co.from_i64(x)), x)
    assert int(co.from_i64(np.array([-1]))[0]) == P - 1
    # rsqrt_index: round(var / 2^18), then steps of 2^8 above 2^20, 2^16 above 2^20 + 2^30
    var = np.array([0, 1 << 17, (1 << 18) - 1, (1 << 38), (1 << 38) + (300 << 18), ((1 << 20) + (1 << 30)) << 18,
                    -5], dtype=np.int64)
    got = [int(v) for v in co.rsqrt_index(var)]
    assert got == [0, 1, 1, 1 << 20, (1 << 20) + 1, (1 << 20) + (1 << 22), 0]


def test_xorshift_fill_matches_the_reference_draws():
    """from_i64((next_u64() % mod) + offset), next_u64 of common/field.rs:17-36."""
    rng = XorShift64(0x1D1D)
    got = gpt2.xorshift_fill(rng, 50, 10, -5)
    ref = o.XorShift64(0x1D1D)
    want = [int(co.from_i64(np.array([ref.next_u64() % 10 - 5]))[0]) for _ in range(50)]
    assert [int(v) for v in got] == want
    assert rng.c.xorshift_state == ref.s.value


def test_same_poly_as_one_product():
    """prove_same_poly's virtual polynomial sum_i c_i f eq_i has the round
    messages of f E, E = sum_i c_i eq_i (the device builds E)."""
    rng = o.XorShift64(11)
    t = 7
    f = rng.fields(1 << t)
    pts = [rng.fields(t) for _ in range(5)]
    cs = [rng.field() for _ in range(5)]
    merged = rng.fields(t)
    eqs = [o.eq_evals(p) for p in pts]
    r1, f1 = o.virtual_prove([f] + eqs, [(c, [0, i + 1]) for i, c in enumerate(cs)], merged)
    E = np.zeros(1 << t, dtype=np.uint64)
    for c, e in zip(cs, eqs):
        E = o.vec_add(E, o.vec_mul(np.full(1 << t, c, dtype=np.uint64), e))
    r2, f2 = o.virtual_prove([f, E], [(1, [0, 1])], merged)
    assert np.array_equal(r1, r2) and f1[0] == f2[0]


@pytest.fixture(scope="module")
def reference_case():
    st = co.HostStore()
    ops, out, rng = gpt2.reference_layer_roundtrip_case(st, XorShift64)
    proof = co.prove_shard(st, ops, [out], _oracle_rng(rng))
    return st, ops, out, proof


def test_reference_layer_roundtrip(reference_case):
    """build_gpt2_layer_roundtrip: prove_shard then verify_shard accept."""
    st, ops, out, proof = reference_case
    assert len(ops) == 27
    assert [p[0] for p in proof["ops"]][:5] == ["Layernorm", "Projection", "Projection", "Projection", "Transpose"]
    assert co.verify_shard(ops, proof)
    assert out not in proof["bound"]
    assert [c[9] for c in proof["witness_columns"]] == sorted({op.table for op in ops if op.kind in
                                                                ("Lookup", "Softmax")} | {ops[0].rsqrt_table})


@pytest.mark.parametrize("where", ["bind", "projection", "softmax", "layernorm", "lookup", "add"])
def test_verify_rejects_tampering(reference_case, where):
    _, ops, _, proof = reference_case
    bad = copy.deepcopy(proof)
    kinds = [p[0] for p in bad["ops"]]

    def bump(a, i=0):
        a.reshape(-1)[i] = (int(a.reshape(-1)[i]) + 1) % P

    if where == "bind":
        bump(bad["binds"][0][1][0])
    elif where == "projection":
        bump(bad["ops"][kinds.index("Projection")][2][0], 1)
    elif where == "softmax":
        bump(bad["ops"][kinds.index("Softmax")][2][0])
    elif where == "layernorm":
        bump(bad["ops"][kinds.index("Layernorm")][2][0])
    elif where == "lookup":
        # the table an Op::Lookup reads (the reference's verifier checks the
        # logUp split for Lookup arms; Softmax's exp lookup is not re-checked there)
        table = next(op.table for op in ops if op.kind == "Lookup")
        col = next(c for c in bad["table_columns"] if c[1] == table)
        bump(col[0][0][0][2])
    else:
        bump(bad["ops"][kinds.index("Add")][1][0])
    assert not co.verify_shard(ops, bad)


SMALL = gpt2.LayerShape(m=8, d=16, d_real=12, heads=2, dh=4, ffn=32, ffn_real=24, shift=16, exp_bits=8,
                        gelu_bits=10, rsqrt_len=256)


def test_gpt2_layer_graph_shape():
    """176 ops at the GPT-2 head count, in build_layer's order."""
    st = co.HostStore()
    s = gpt2.LayerShape(m=4, d=16, d_real=12, heads=12, dh=1, ffn=32, ffn_real=24, exp_bits=6, gelu_bits=8,
                        rsqrt_len=64)
    ops, x, out = gpt2.gpt2_layer(st, s)
    assert len(ops) == 176
    kinds = [op.kind for op in ops]
    assert kinds[0] == "LayerNormCentered" and kinds[-1] == "Add"
    assert kinds[1:14] == ["Projection"] * 3 + ["Scale"] * 2 + ["Transpose", "MatMul", "Scale", "StableSoftmaxIndex",
                                                              "Softmax", "MatMul", "Scale", "Projection"]
    assert kinds.count("Projection") == 12 * 4 + 2 and kinds.count("Add") == 11 + 3
    assert x == 0 and out == len(st.v) - 1


def test_gpt2_layer_shard_dag_verifies():
    """One GPT-2-shaped layer as one shard of prove_shard_dag, and split into
    shards of 12 ops (cross-shard bindings), both accepted."""
    for ops_per_shard in (176, 12):
        st = co.HostStore()
        ops, _, _ = gpt2.gpt2_layer(st, SMALL)
        dag = co.prove_shard_dag(st, ops, ops_per_shard)
        ranges = co.shard_ranges(len(ops), ops_per_shard)
        assert len(dag["shards"]) == len(ranges)
        for (s, e), sh in zip(ranges, dag["shards"]):
            assert co.verify_shard(ops[s:e], sh)
        if ops_per_shard == 176:
            assert dag["cross_tensors"] == []
        else:
            assert dag["cross_tensors"]
            by = {}
            for sh in dag["shards"]:
                for t, pt, ev in sh["claims"]:
                    by.setdefault(t, []).append((pt, ev))
            for t, sp in zip(dag["cross_tensors"], dag["cross_binds"]):
                assert co.verify_same_poly(sp, by[t]) is not None


def _topk_rows(x, m, n, k):
    """The top-k order restated independently: per row a Python sort on
    (-value, position)."""
    xi = co.to_i64(x).reshape(m, n)
    sel = np.zeros((m, n), dtype=np.uint64)
    thr = np.zeros(m, dtype=np.int64)
    for t in range(m):
        order = sorted(range(n), key=lambda e: (-int(xi[t, e]), e))
        sel[t, order[:k]] = 1
        thr[t] = xi[t, order[k - 1]]
    return sel.reshape(-1), thr


@pytest.mark.parametrize("m,n,k", [(4, 8, 3), (4, 8, 1), (2, 64, 6), (8, 16, 16)])
def test_topk_forward_order_and_ties(m, n, k):
    """topk_forward (topk.rs:41-80): ties broken by position, d1 and d2 the
    signed distances to the threshold on either side."""
    rng = np.random.default_rng(m * n + k)
    vals = rng.integers(-4, 4, size=m * n)  # many ties
    vals[::5] = rng.integers(-(1 << 40), 1 << 40, size=vals[::5].size)
    x = co.from_i64(vals)
    thr, sel, gate, d1, d2 = co.topk_forward(x, m, n, k)
    want_sel, want_thr = _topk_rows(x, m, n, k)
    assert np.array_equal(sel, want_sel) and np.array_equal(co.to_i64(thr), want_thr)
    assert (sel.reshape(m, n).sum(axis=1) == k).all()
    s = sel.astype(bool)
    xi, ti = co.to_i64(x), np.repeat(want_thr, n)
    assert np.array_equal(co.to_i64(gate), np.where(s, xi, 0))
    assert np.array_equal(co.to_i64(d1), np.where(s, xi - ti, 0)) and (co.to_i64(d1) >= 0).all()
    assert np.array_equal(co.to_i64(d2), np.where(s, 0, ti - xi)) and (co.to_i64(d2) >= 0).all()


def test_reference_topk_roundtrip():
    """topk.rs tests::topk_roundtrip (:247-259): seed 0x7777, x_i = (i mod 53)
    - 26 over 4 x 8, k 3, range_bits 16; a corrupted sel-range leaf fails."""
    m, n, k = 4, 8, 3
    x = co.from_i64(np.array([(i % 53) - 26 for i in range(m * n)]))
    thr, sel, gate, d1, d2 = co.topk_forward(x, m, n, k)
    p = co.prove_topk(x, sel, thr, gate, d1, d2, m, n, k, 16, o.XorShift64(0x7777))
    assert co.verify_topk(p, k)
    bad = copy.deepcopy(p)
    layers, fnum, fden, full_r = bad[5]
    l0 = list(layers[0])
    l0[3] = l0[3].copy()
    l0[3][3] = (int(l0[3][3]) + 1) % P
    bad = bad[:5] + (((tuple(l0),) + tuple(layers[1:]), fnum, fden, full_r),) + bad[6:]
    assert not co.verify_topk(bad, k)
    assert not co.verify_topk(p, k + 1)  # the row-sum claim is k


def test_reference_argmax_roundtrip():
    """topk.rs argmax_tests::argmax_roundtrip (:347-369): seed 0x9999; the
    output positions are each row's first maximum, the proof verifies, and a
    moved output position fails the index binding."""
    m, n = 4, 8
    x = co.from_i64(np.array([(i % 53) - 26 for i in range(m * n)]))
    thr, sel, gate, d1, d2, out = co.argmax_forward(x, m, n)
    xi = co.to_i64(x).reshape(m, n)
    for i in range(m):
        best = 0
        for j in range(1, n):
            if xi[i, j] > xi[i, best]:
                best = j
        assert out[i] == best and sel[i * n + best] == 1
    p = co.prove_argmax(x, sel, thr, gate, d1, d2, out, m, n, 16, o.XorShift64(0x9999))
    assert co.verify_argmax(p, m, n)
    moved = out.copy()
    moved[0] = (moved[0] + 1) % n
    assert not co.verify_argmax((p[0], p[1], moved, p[3]), m, n)


def test_range_decomp_wide_differences():
    """prove_range_decomp (topk.rs:391-448) over 48-bit values verifies; a
    value of 2^48 loses its top bits in the limbs and fails the
    recomposition."""
    vals = np.array([0, 1, 0xFFFF, 0x10000, (1 << 48) - 1, 12345678901, 7, 1 << 47], dtype=np.int64)
    p = co.prove_range_decomp(co.from_i64(vals), o.XorShift64(3))
    assert co.verify_range_decomp(p)
    vals[3] = 1 << 48
    assert not co.verify_range_decomp(co.prove_range_decomp(co.from_i64(vals), o.XorShift64(3)))


def test_topk_and_argmax_shard_verifies():
    """Op::TopKSelect (range_bits 22) and Op::Argmax (16) inside
    prove_shard_precomputed: claims of x, sel and gate at the gate relation's
    point, bound to x's other claim (an Add producing it) by same_poly."""
    m, n = 4, 16
    st = co.HostStore()
    rng = np.random.default_rng(5)
    a = st.push(co.from_i64(rng.integers(-1000, 1000, size=m * n)))
    b = st.push(co.from_i64(rng.integers(-1000, 1000, size=m * n)))
    x = st.push(None)
    ts = [st.push(None) for _ in range(10)]
    out = st.push_idx(None)
    ops = [co_op("Add", a=a, b=b, c=x),
           co_op("TopKSelect", x=x, sel=ts[0], thr=ts[1], gate=ts[2], d1=ts[3], d2=ts[4], m=m, n=n, k=3),
           co_op("Argmax", x=x, sel=ts[5], thr=ts[6], gate=ts[7], d1=ts[8], d2=ts[9], out=out, m=m, n=n)]
    proof = co.prove_shard(st, ops, [], o.XorShift64(11))
    assert co.verify_shard(ops, proof)
    assert x in proof["bound"]
    assert np.array_equal(st.idx[out], co.to_i64(st.v[x]).reshape(m, n).argmax(axis=1))


def co_op(kind, **fields):
    """An op object of the product's op classes (read by duck typing)."""
    from zkie_b200 import compose as C
    return getattr(C, kind)(**fields)
