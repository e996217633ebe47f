"""The MLA / MoE arms on the device (zkie_b200/csrc/moe.cu, the RmsNorm,
RoPE, Scatter, Gather, GatherMatMul and index arms of zkie_b200/compose.py)
against the CPU restatement: a DeepSeek-V2-Lite-shaped MoE layer's forward
witness tensor for tensor, and its shard proof value for value."""
import numpy as np
import pytest

from oracle import compose_oracle as co
from oracle import oracle as o

pytestmark = pytest.mark.gpu

SMALL = dict(m=8, h=16, heads=2, qk_nope=4, qk_rope=4, v_head=4, kv_lora=8, n_routed=8, top_k=2, moe=8, moe_real=6,
             shared=16, shared_real=12, exp_bits=8, silu_bits=12, rsqrt_len=1 << 12, w_mod=1 << 12, router_mod=1 << 10)
MEDIUM = dict(m=32, h=256, heads=2, qk_nope=16, qk_rope=8, v_head=16, kv_lora=32, n_routed=16, top_k=3, moe=64,
              moe_real=48, shared=128, shared_real=96, exp_bits=12, silu_bits=16, rsqrt_len=1 << 16, w_mod=1 << 8,
              router_mod=1 << 10)


def _stores(zk, shape):
    from zkie_b200 import deepseek as ds
    host = co.HostStore()
    ops, x, out = ds.moe_layer(host, ds.MoeShape(**shape))
    dev = zk.compose.Store()
    for v in host.v:
        dev.push(None if v is None else v.copy())
    for i in host.idx:
        dev.push_idx(None if i is None else i.copy())
    return host, dev, ops, out


def _assert_same(a, b, path="proof"):
    if isinstance(a, dict):
        assert a.keys() == b.keys(), path
        for k in a:
            _assert_same(a[k], b[k], f"{path}.{k}")
    elif isinstance(a, (list, tuple)):
        assert isinstance(b, (list, tuple)) and len(a) == len(b), f"{path}: {len(a)} vs {len(b)}"
        for i, (x, y) in enumerate(zip(a, b)):
            _assert_same(x, y, f"{path}[{i}]")
    elif isinstance(a, np.ndarray) or isinstance(b, np.ndarray):
        x, y = np.asarray(a, dtype=np.uint64), np.asarray(b, dtype=np.uint64)
        assert x.shape == y.shape and np.array_equal(x, y), f"{path}: arrays differ"
    elif isinstance(a, str):
        assert a == b, f"{path}: {a} vs {b}"
    else:
        assert int(a) % co.P == int(b) % co.P, f"{path}: {a} vs {b}"


@pytest.mark.parametrize("shape", [SMALL, MEDIUM], ids=["small", "medium"])
def test_moe_layer_forward_matches_oracle(zk, shape):
    host, dev, ops, out = _stores(zk, shape)
    zk.compose.forward_ops(dev, ops)
    co.forward_ops(host, ops)
    for t, v in enumerate(host.v):
        if v is not None:
            assert np.array_equal(dev.get(t).cpu().numpy(), v), f"tensor {t}"
    for t, v in enumerate(host.idx):
        if v is not None:
            assert np.array_equal(dev.get_idx(t).cpu().numpy(), v), f"index tensor {t}"
    assert np.count_nonzero(host.v[out])


@pytest.mark.parametrize("shape", [SMALL, MEDIUM], ids=["small", "medium"])
def test_moe_layer_shard_matches_oracle(zk, shape):
    host, dev, ops, _ = _stores(zk, shape)
    zk.compose.forward_ops(dev, ops)
    got = zk.compose.prove_shard_precomputed(dev, ops, [], zk.gkr.XorShift64(33)).canonical()
    want = co.prove_shard(host, ops, [], o.XorShift64(33))
    _assert_same(got, want)
    assert co.verify_shard(ops, want)


def test_moe_layer_graph_replay(zk):
    """The MoE layer's proof recorded once as a CUDA graph and replayed: the
    eager proof's digest."""
    from zkie_b200 import dag
    host, dev, ops, _ = _stores(zk, MEDIUM)
    C = zk.compose
    C.forward_ops(dev, ops)
    master = C.master_transcript(ops, len(ops))

    def make_rng():
        c = master.clone()
        c.absorb_u64(0)
        return c
    eager = dag.digest(C.prove_shard_precomputed(dev, ops, [], make_rng()).canonical())
    gp = C.GraphShardProver(dev, ops, [], make_rng)
    gp.replay()
    assert dag.digest(gp.prove().canonical()) == eager


def test_gather_token_outside_is_an_error(zk):
    import torch
    C = zk.compose
    st = C.Store()
    w = st.push(np.arange(8, dtype=np.uint64))
    tid = st.push_idx(np.array([0, 5], dtype=np.uint32))  # 5 >= m
    g = st.push(np.ones(2, dtype=np.uint64))
    out = st.push(None)
    with pytest.raises(ValueError, match="lookup index"):
        C.forward_ops(st, [C.Gather(w, tid, g, out, 4, 4)])
    torch.cuda.synchronize()


def test_index_and_scale_ops_edge_cases(zk):
    """The no-proof arms against the CPU restatement where the reference's
    semantics bite: PadIdx truncating (len below the base's length),
    IdxBroadcast and CombineIdx wrapping in u32, ScaleVec with a scale
    shorter than x (cycled) and negative products, BroadcastScale over rows."""
    C = zk.compose
    host = co.HostStore()
    rng = np.random.default_rng(7)
    base = host.push_idx(rng.integers(0, 1 << 32, size=12, dtype=np.uint64).astype(np.uint32))
    bb = host.push_idx(rng.integers(0, 1 << 32, size=12, dtype=np.uint32))
    x = host.push(co.from_i64(rng.integers(-(1 << 30), 1 << 30, size=24)))
    sv = host.push(co.from_i64(rng.integers(-(1 << 20), 1 << 20, size=5)))
    rows = host.push(co.from_i64(rng.integers(-1000, 1000, size=6)))
    outs = [host.push_idx(None) for _ in range(4)] + [host.push(None), host.push(None)]
    ops = [C.PadIdx(base, outs[0], 7), C.PadIdx(base, outs[1], 20), C.IdxBroadcast(base, outs[2], 3000),
           C.CombineIdx(base, bb, outs[3], 1 << 20), C.ScaleVec(x, sv, outs[4], 7),
           C.BroadcastScale(x, rows, outs[5], 4)]
    dev = zk.compose.Store()
    for v in host.v:
        dev.push(None if v is None else v.copy())
    for i in host.idx:
        dev.push_idx(None if i is None else i.copy())
    C.forward_ops(dev, ops)
    co.forward_ops(host, ops)
    for t in outs[:4]:
        assert np.array_equal(dev.get_idx(t).cpu().numpy(), host.idx[t]), t
    for t in outs[4:]:
        assert np.array_equal(dev.get(t).cpu().numpy(), host.v[t]), t
    assert host.idx[outs[0]].size == 7 and host.idx[outs[1]].size == 20


def test_relu_scale_gate_batched_matmul_shard_matches_oracle(zk):
    """The arms only the Gemma / TimesFM graphs use (Relu, ScaleGate,
    BatchedMatMul): forward and shard proof equal to the CPU restatement's."""
    C = zk.compose
    host = co.HostStore()
    s, k, n, m = 16, 64, 32, 4
    rng = np.random.default_rng(s + k)
    x = host.push(co.from_i64(rng.integers(-(1 << 20), 1 << 20, size=s * k)))
    w = host.push(co.from_i64(rng.integers(-(1 << 12), 1 << 12, size=s * k * n)))
    gate = host.push(co.from_i64(rng.integers(-(1 << 16), 1 << 16, size=m * n)))
    r, c, sg = host.push(None), host.push(None), host.push(None)
    ops = [C.Relu(x, r), C.BatchedMatMul(r, w, c, s, k, n), C.ScaleGate(c, gate, 1, sg, m, n, (s * n) // m, 8)]
    dev = C.Store()
    for v in host.v:
        dev.push(None if v is None else v.copy())
    C.forward_ops(dev, ops)
    got = C.prove_shard_precomputed(dev, ops, [], zk.gkr.XorShift64(8)).canonical()
    want = co.prove_shard(host, ops, [], o.XorShift64(8))
    for op in ops:
        t = op.writes()[0]
        assert np.array_equal(dev.get(t).cpu().numpy(), host.v[t]), op.kind
    _assert_same(got, want)
    assert co.verify_shard(ops, want)
