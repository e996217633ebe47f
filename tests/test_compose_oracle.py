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
