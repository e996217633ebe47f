"""The op-layer shard prover on the GPU against its CPU restatement, bit for
bit: every forward tensor, every proof field, every claim, every binding and
every lookup column, for the reference's own layer test
(build_gpt2_layer_roundtrip, compose.rs:6211-6259) and for GPT-2-shaped
layers (models/gpt2/src/lib.rs build_layer) as prove_shard_dag shards; the
device proofs are also accepted by the restated verifier."""
import numpy as np
import pytest
import torch

from oracle import compose_oracle as co
from oracle import oracle as o

pytestmark = pytest.mark.gpu

P = co.P


def assert_same(a, b, path="proof"):
    if isinstance(a, dict):
        assert isinstance(b, dict) and a.keys() == b.keys(), path
        for k in a:
            assert_same(a[k], b[k], f"{path}.{k}")
    elif isinstance(a, (list, tuple)) and not isinstance(a, np.ndarray):
        assert isinstance(b, (list, tuple)) and len(a) == len(b), f"{path}: {len(a)} vs {len(b)}"
        for i, (x, y) in enumerate(zip(a, b)):
            assert_same(x, y, f"{path}[{i}]")
    elif isinstance(a, np.ndarray) or isinstance(b, np.ndarray):
        x, y = np.asarray(a, dtype=np.uint64), np.asarray(b, dtype=np.uint64)
        assert x.shape == y.shape and np.array_equal(x, y), f"{path}: arrays differ"
    elif isinstance(a, str):
        assert a == b, f"{path}: {a} vs {b}"
    else:
        assert int(a) % P == int(b) % P, f"{path}: {a} vs {b}"


def _device_store(zk, host):
    st = zk.compose.Store()
    for v in host.v:
        st.push(None if v is None else v.copy())
    for i in host.idx:
        st.push_idx(None if i is None else i.copy())
    return st


def _host_copy(host):
    c = co.HostStore()
    c.v = [None if v is None else v.copy() for v in host.v]
    c.idx = [None if i is None else i.copy() for i in host.idx]
    return c


def _reference_case(zk):
    from zkie_b200 import gpt2
    from zkie_b200.gkr import XorShift64
    host = co.HostStore()
    ops, out, rng = gpt2.reference_layer_roundtrip_case(host, XorShift64)
    orng = o.XorShift64(0)
    orng.s.value = rng.c.xorshift_state
    return host, ops, out, rng, orng


def test_forward_matches_oracle_reference_case(zk):
    host, ops, _, _, _ = _reference_case(zk)
    dev = _device_store(zk, host)
    zk.compose.forward_ops(dev, ops)
    co.forward_ops(host, ops)
    for i, v in enumerate(host.v):
        assert np.array_equal(dev.v[i].cpu().numpy(), v), f"tensor {i}"
    for i, v in enumerate(host.idx):
        assert np.array_equal(dev.idx[i].cpu().numpy(), v), f"index tensor {i}"


def test_prove_shard_matches_oracle_reference_case(zk):
    """The reference's layer test: prove_shard(store, ops, [out], rng) with the
    XorShift64 that drew the weights."""
    host, ops, out, rng, orng = _reference_case(zk)
    dev = _device_store(zk, host)
    got = zk.compose.prove_shard(dev, ops, [out], rng).canonical()
    want = co.prove_shard(host, ops, [out], orng)
    assert_same(got, want)
    assert co.verify_shard(ops, got)
    assert rng.c.xorshift_state == orng.s.value


def _layer(zk, shape):
    from zkie_b200 import gpt2
    host = co.HostStore()
    ops, x, out = gpt2.gpt2_layer(host, shape)
    return host, ops


@pytest.mark.parametrize("name,ops_per_shard", [("small", 176), ("small", 12), ("medium", 176)])
def test_gpt2_layer_shard_dag_matches_oracle(zk, name, ops_per_shard):
    from zkie_b200 import gpt2
    shape = {"small": gpt2.LayerShape(m=8, d=16, d_real=12, heads=2, dh=4, ffn=32, ffn_real=24, exp_bits=8,
                                      gelu_bits=10, rsqrt_len=256),
             "medium": gpt2.LayerShape(m=64, d=128, d_real=96, heads=6, dh=16, ffn=512, ffn_real=384, exp_bits=12,
                                       gelu_bits=14, rsqrt_len=4096)}[name]
    host, ops = _layer(zk, shape)
    dev = _device_store(zk, host)
    ref = _host_copy(host)
    got = zk.compose.prove_shard_dag(dev, ops, ops_per_shard).canonical()
    want = co.prove_shard_dag(ref, ops, ops_per_shard)
    for i, v in enumerate(ref.v):
        assert np.array_equal(dev.v[i].cpu().numpy(), v), f"forward tensor {i}"
    assert_same(got, want)
    for (s, e), sh in zip(co.shard_ranges(len(ops), ops_per_shard), got["shards"]):
        assert co.verify_shard(ops[s:e], sh)


def test_lookup_outside_table_is_an_error(zk):
    """An index past the table end raises on the host (the reference panics);
    the kernel bounds-checks every read."""
    C = zk.compose
    st = C.Store()
    x = st.push(np.array([1, 2, 3, 70], dtype=np.uint64))
    idx = st.push_idx(None)
    table = st.push(np.arange(64, dtype=np.uint64))
    out = st.push(None)
    ops = [C.SoftmaxIndex(x, idx, 1 << 8), C.Lookup(idx, out, table)]
    with pytest.raises(ValueError, match="outside its table"):
        C.forward_ops(st, ops)
    torch.cuda.synchronize()


def test_graph_prover_replays_for_a_new_witness(zk):
    """GraphShardProver: the recorded prove equals the eager one, and after
    new input values go into the same buffers (forward in place), a replay
    proves the new witness exactly as the CPU restatement does."""
    from zkie_b200 import gpt2
    C = zk.compose
    shape = gpt2.LayerShape(m=16, d=32, d_real=24, heads=3, dh=8, ffn=64, ffn_real=48, exp_bits=9, gelu_bits=11,
                            rsqrt_len=512)
    host = co.HostStore()
    ops, x, out = gpt2.gpt2_layer(host, shape)
    dev = _device_store(zk, host)
    C.forward_ops(dev, ops)
    master = C.master_transcript(ops, len(ops))

    def make_rng():
        c = master.clone()
        c.absorb_u64(0)
        return c
    gp = C.GraphShardProver(dev, ops, [], make_rng)
    eager = C.prove_shard_precomputed(dev, ops, [], make_rng()).canonical()
    assert_same(gp.prove().canonical(), eager)
    # a new layer input in the same buffer
    g = np.random.default_rng(5)
    new_x = np.zeros((shape.m, shape.d), dtype=np.uint64)
    new_x[:, :shape.d_real] = g.integers(0, 50, size=(shape.m, shape.d_real)).astype(np.uint64)
    dev.v[x].copy_(torch.from_numpy(new_x.reshape(-1)).cuda())
    C.forward_ops(dev, ops)
    got = gp.prove().canonical()
    ref = _host_copy(host)
    ref.v[x] = new_x.reshape(-1)
    co.forward_ops(ref, ops)
    om = co.master_transcript(ops, len(ops))
    child = o.OracleTranscript(raw=om.t)
    child.absorb_u64(0)
    assert_same(got, co.prove_shard_precomputed(ref, ops, [], child))


@pytest.mark.parametrize("graph", [False, True])
def test_dag_ranks_device_matches_oracle(zk, graph):
    """The shard-DAG orchestration (zkie_b200/dag.py) over the device prover,
    eager and with recorded graphs, on a three-layer stack: the DAG digest of
    the CPU restatement's prove_shard_dag."""
    from zkie_b200 import dag, gpt2
    shape = gpt2.LayerShape(m=8, d=16, d_real=12, heads=2, dh=4, ffn=32, ffn_real=24, exp_bits=8, gelu_bits=10,
                            rsqrt_len=256)
    host = co.HostStore()
    ops, _, _ = gpt2.gpt2_layers(host, shape, 3)
    dev = _device_store(zk, host)
    zk.compose.forward_ops(dev, ops)
    per = len(ops) // 3
    provers = dag.device_provers(summary="digest", graph=graph)
    got = dag.prove_dag_ranks(dev, ops, per, provers)
    if graph:  # a second pass replays the recorded graphs
        got = dag.prove_dag_ranks(dev, ops, per, provers)
        assert len(provers.graphs) == 3
    co.forward_ops(host, ops)
    full = co.prove_shard_dag(host, ops, per)
    consts = o.p2_constants(1)
    roots = [o.whir_commit(consts, host.get(t))[1] for t in full["cross_tensors"]]
    assert got.digest == dag.dag_digest(full["shards"], full["cross_tensors"], full["cross_binds"], roots)
    assert len(got.boundary_roots) == len(full["cross_tensors"])


def test_gpt2_model_dag_device_matches_oracle(zk):
    """The GPT-2 model graph (embedding lookup into the tied table, two small
    layers, final LayerNorm, lm_head, vocabulary mask, Argmax) as a DAG of 35-op
    shards on the device: the CPU restatement's DAG digest."""
    from zkie_b200 import dag, gpt2
    shape = gpt2.LayerShape(m=8, d=16, d_real=12, heads=2, dh=4, ffn=32, ffn_real=24, exp_bits=8, gelu_bits=10,
                            rsqrt_len=256, vocab=64, vocab_real=50)
    host = co.HostStore()
    ops, _, _ = gpt2.gpt2_model(host, shape, 2)
    dev = _device_store(zk, host)
    zk.compose.forward_ops(dev, ops)
    got = dag.prove_dag_ranks(dev, ops, 35, dag.device_provers(summary="digest", graph=True))
    co.forward_ops(host, ops)
    full = co.prove_shard_dag(host, ops, 35)
    consts = o.p2_constants(1)
    roots = [o.whir_commit(consts, host.get(t))[1] for t in full["cross_tensors"]]
    assert got.digest == dag.dag_digest(full["shards"], full["cross_tensors"], full["cross_binds"], roots)


def _topk_case(m, n, seed, wide=False):
    rng = np.random.default_rng(seed)
    vals = rng.integers(-4, 4, size=m * n)  # ties in every row
    if wide:
        vals[::3] = rng.integers(-(1 << 41), 1 << 30, size=vals[::3].size)
    return co.from_i64(vals)


@pytest.mark.parametrize("m,n,k", [(4, 8, 1), (4, 8, 3), (8, 64, 6), (2, 4096, 5), (3, 1 << 17, 1), (16, 16, 16)])
def test_topk_forward_matches_oracle(zk, m, n, k):
    """zkie2_op_topk against topk_forward / argmax_forward: the k-th entry,
    the one-hot selection (ties by position), gate, d1, d2 and the Argmax
    output positions."""
    x = _topk_case(m, n, m + n + k, wide=True)
    host = co.HostStore()
    xi = host.push(x)
    ts = [host.push(None) for _ in range(5)]
    out = host.push_idx(None)
    C = zk.compose
    op = (C.Argmax(xi, *ts, out, m, n) if k == 1 else C.TopKSelect(xi, *ts, m, n, k))
    dev = _device_store(zk, host)
    C.forward_ops(dev, [op])
    co.forward_ops(host, [op])
    for t in ts:
        assert np.array_equal(dev.get(t).cpu().numpy(), host.v[t]), t
    if k == 1:
        assert np.array_equal(dev.get_idx(out).cpu().numpy(), host.idx[out])


def test_topk_rejects_unsupported_k(zk):
    from zkie_b200.device import to_dev
    x = to_dev(_topk_case(2, 8, 1))
    bufs = [torch.empty(16, dtype=torch.uint64, device="cuda") for _ in range(5)]
    lib = zk.lib
    for k in (0, 9):
        assert lib.zkie2_op_topk(x.data_ptr(), 2, 8, k, *[b.data_ptr() for b in bufs], None, 0) != 0


@pytest.mark.parametrize("n", [16, 1024])
def test_topk_argmax_shard_matches_oracle(zk, n):
    """Op::TopKSelect (range_bits 22) and Op::Argmax (16) in one shard on the
    device prover: the CPU restatement's proof, value for value, and it
    verifies."""
    C = zk.compose
    host, ops = _topk_shard(C, 4, n, 1000)
    dev = _device_store(zk, host)
    C.forward_ops(dev, ops)
    got = C.prove_shard_precomputed(dev, ops, [], zk.gkr.XorShift64(21)).canonical()
    want = co.prove_shard(host, ops, [], o.XorShift64(21))
    assert_same(got, want)
    assert co.verify_shard(ops, want)


def _topk_shard(C, m, n, spread):
    """x = a + b with a quarter of the entries 2^40 below the rest (never
    among the top 6: d2 needs all three 16-bit limbs); the others within
    +-spread, so the selected entries' distances d1 stay below 2^22 when
    spread is small."""
    host = co.HostStore()
    rng = np.random.default_rng(n + spread)
    a = host.push(co.from_i64(rng.integers(-spread, spread, size=m * n)))
    bv = rng.integers(-1000, 1000, size=m * n)
    bv[::4] = -(1 << 40)
    b = host.push(co.from_i64(bv))
    x = host.push(None)
    ts = [host.push(None) for _ in range(10)]
    out = host.push_idx(None)
    return host, [C.Add(a, b, x), C.TopKSelect(x, *ts[:5], m, n, 6), C.Argmax(x, *ts[5:], out, m, n)]


def test_topk_selected_spread_outside_the_range_table(zk):
    """Selected entries further than 2^22 from the threshold: d1 falls
    outside TopKSelect's range table, where the reference's multiplicity
    count would panic; the device prover reports the lookup error and the
    CPU restatement raises."""
    C = zk.compose
    host, ops = _topk_shard(C, 2, 16, 1 << 30)
    dev = _device_store(zk, host)
    C.forward_ops(dev, ops)
    with pytest.raises(ValueError, match="lookup index"):
        C.prove_shard_precomputed(dev, ops, [], zk.gkr.XorShift64(1))
    with pytest.raises(IndexError):
        co.prove_shard(host, ops, [], o.XorShift64(1))


def test_graph_forward_replays_new_witnesses_and_falls_back(zk):
    """GraphForward: the forward of a GPT-2-shaped layer whose wide products
    take the tensor path, recorded once; a new witness in the same buffers
    replays to the CPU restatement's forward, and a witness whose FFN weights
    outgrow the recorded byte planes is detected on the device and recomputed
    eagerly, again equal to the restatement."""
    from zkie_b200 import gpt2
    from zkie_b200.device import to_dev
    shape = gpt2.LayerShape(m=256, d=512, d_real=384, heads=8, dh=64, ffn=2048, ffn_real=1536, exp_bits=16,
                            gelu_bits=18, rsqrt_len=1 << 16)
    host, ops = _layer(zk, shape)
    dev = _device_store(zk, host)
    gf = zk.compose.GraphForward(dev, ops)
    assert any(int(h[0]) == 0 for _, h in gf.plan.steps), "no product took the tensor path"
    x = ops[0].x
    rng = np.random.default_rng(3)
    for step in range(2):
        if step == 0:
            new = np.zeros((shape.m, shape.d), dtype=np.uint64)
            new[:, :shape.d_real] = rng.integers(0, 50, size=(shape.m, shape.d_real)).astype(np.uint64)
            t = x
        else:  # the FFN weights past 16 bits
            t = next(op for op in ops if op.kind == "Projection" and op.n == shape.ffn).w
            new = co.from_i64(rng.integers(-(1 << 20), 1 << 20, size=host.v[t].size))
        host.v[t] = new.reshape(-1)
        dev.get(t).copy_(to_dev(host.v[t]).reshape(-1))
        gf.run()
        co.forward_ops(host, ops)
        for i, v in enumerate(host.v):
            if v is not None:
                assert np.array_equal(dev.get(i).cpu().numpy(), v), f"step {step}: tensor {i}"
        assert gf.fallbacks == step
