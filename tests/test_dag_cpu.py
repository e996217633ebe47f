"""The shard-DAG split over ranks (zkie_b200/dag.py), no GPU: the orchestration
driven by the CPU restatement's shard prover, in one process and as world-size
2 and 3 gloo process groups, against the restatement's own prove_shard_dag
(compose.rs:2289-2346) over a stack of small GPT-2-shaped layers."""
import os
import pickle
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from oracle import compose_oracle as co
from oracle import oracle as o
from zkie_b200 import dag, gpt2

SHAPE = gpt2.LayerShape(m=8, d=16, d_real=12, heads=2, dh=4, ffn=32, ffn_real=24, exp_bits=8, gelu_bits=10,
                        rsqrt_len=256)


def oracle_provers():
    def child(m, si):
        c = o.OracleTranscript(raw=m.t)
        c.absorb_u64(si)
        return c
    consts = o.p2_constants(1)
    return dag.DagProvers(
        master=co.master_transcript, child=child,
        prove=lambda store, ops, rng: co.prove_shard_precomputed(store, ops, [], rng),
        claims=lambda p: p["claims"], summary=lambda p: p,
        same_poly=lambda store, t, cs, m: co.prove_same_poly(store.get(t), cs, m),
        commit=lambda store, t: o.whir_commit(consts, store.get(t))[1])


def stack(layers):
    st = co.HostStore()
    ops, x, out = gpt2.gpt2_layers(st, SHAPE, layers)
    co.forward_ops(st, ops)
    return st, ops


def _want(layers, ops_per_shard):
    st, ops = stack(layers)
    full = co.prove_shard_dag(st, ops, ops_per_shard)
    consts = o.p2_constants(1)
    roots = [o.whir_commit(consts, st.get(t))[1] for t in full["cross_tensors"]]
    return dag.dag_digest(full["shards"], full["cross_tensors"], full["cross_binds"], roots), full


def test_layers_chain():
    """Layer l + 1 reads layer l's output; the tables and the mask are shared."""
    st = co.HostStore()
    ops, x, out = gpt2.gpt2_layers(st, SHAPE, 3)
    per = len(ops) // 3
    assert len(ops) == 3 * per
    assert ops[per].kind == "LayerNormCentered" and ops[per].x == ops[per - 1].c
    assert ops[2 * per].rsqrt_table == ops[0].rsqrt_table
    assert out == ops[-1].c


@pytest.mark.parametrize("layers,ops_per_shard", [(3, None), (2, 20)])
def test_dag_single_process_matches_prove_shard_dag(layers, ops_per_shard):
    st, ops = stack(layers)
    ops_per_shard = ops_per_shard or len(ops) // layers
    res = dag.prove_dag_ranks(st, ops, ops_per_shard, oracle_provers())
    want, full = _want(layers, ops_per_shard)
    assert res.digest == want
    assert res.cross_tensors == full["cross_tensors"] and res.cross_tensors
    for (s, e), sh in zip(dag.shard_ranges(len(ops), ops_per_shard), res.shards):
        assert co.verify_shard(ops[s:e], sh)
    by = {}
    for sh in res.shards:
        for t, pt, ev in sh["claims"]:
            by.setdefault(t, []).append((pt, ev))
    for t, sp in zip(res.cross_tensors, res.cross_binds):
        assert co.verify_same_poly(sp, by[t]) is not None


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, layers, out_dir):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    o.set_threads(1)  # one core per rank: the ranks share the host
    try:
        st, ops = stack(layers)
        res = dag.prove_dag_ranks(st, ops, len(ops) // layers, oracle_provers(), rank, world, dag.torch_gather())
        with open(os.path.join(out_dir, f"dag{rank}.pkl"), "wb") as f:
            pickle.dump(None if res is None else (res.digest, res.cross_tensors), f)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_dag_ranks(tmp_path, world):
    """Shards si % world on each rank, claims gathered to rank 0, cross-shard
    bindings there: the same DAG proof as one process."""
    layers = 3
    mp.start_processes(_rank_main, args=(world, _free_port(), layers, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    with open(tmp_path / "dag0.pkl", "rb") as f:
        digest, cross = pickle.load(f)
    want, full = _want(layers, len(stack(layers)[1]) // layers)
    assert digest == want and cross == full["cross_tensors"]
    for r in range(1, world):
        with open(tmp_path / f"dag{r}.pkl", "rb") as f:
            assert pickle.load(f) is None


def test_gpt2_model_graph_shard_dag():
    """The model graph (embedding Lookup into the tied table, the layers, the
    final LayerNorm, the lm_head MatMul, the vocabulary mask, the Argmax):
    13 shards of 176 ops at GPT-2's 12 layers; here 2 small layers in shards
    of 35 ops, each shard and each cross-shard binding accepted, and the
    Argmax output the first maximum of every masked-logit row."""
    small = gpt2.LayerShape(m=8, d=16, d_real=12, heads=2, dh=4, ffn=32, ffn_real=24, exp_bits=8, gelu_bits=10,
                            rsqrt_len=256, vocab=64, vocab_real=50)
    st = co.HostStore()
    ops, tokens, nxt = gpt2.gpt2_model(st, small, 2)
    assert [o.kind for o in ops[:2]] == ["Lookup", "Add"] and [o.kind for o in ops[-4:]] == [
        "LayerNormCentered", "MatMul", "Add", "Argmax"]
    assert st.v[ops[0].table].size == small.d * small.vocab == st.v[ops[-3].b].size
    assert max(st.idx[tokens]) < small.vocab_real
    full_ops = 2 + 12 * 176 + 4
    assert len(dag.shard_ranges(full_ops, 176)) == 13
    co.forward_ops(st, ops)
    logits = co.to_i64(st.v[ops[-1].x]).reshape(small.m, small.vocab)
    assert (st.idx[nxt] == logits.argmax(axis=1)).all() and (st.idx[nxt] < small.vocab_real).all()
    res = dag.prove_dag_ranks(st, ops, 35, oracle_provers())
    for (s, e), sh in zip(dag.shard_ranges(len(ops), 35), res.shards):
        assert co.verify_shard(ops[s:e], sh)
    by = {}
    for sh in res.shards:
        for t, pt, ev in sh["claims"]:
            by.setdefault(t, []).append((pt, ev))
    assert res.cross_tensors
    for t, sp in zip(res.cross_tensors, res.cross_binds):
        assert co.verify_same_poly(sp, by[t]) is not None


def test_projection_groups_follow_the_data_dependencies():
    """The forward's wide products: Projections that read the same input with
    weights and biases no op writes at or after the first of them form one
    group at that first op; a Projection whose weight is produced later, or
    whose input or shape differs, stays on its own."""
    from zkie_b200 import compose as C
    P_ = C.Projection
    ops = [P_(0, 1, 2, 10, 11, 4, 8, 4, 16),      # x 0: the group's first
           C.Add(3, 3, 12),                        # writes 12
           P_(0, 5, 6, 13, 14, 4, 8, 8, 16),       # x 0, constant weights: joins
           P_(0, 12, 6, 15, 16, 4, 8, 4, 16),      # weight 12 written after op 0: alone
           P_(7, 1, 2, 17, 18, 4, 8, 4, 16),       # another input
           P_(0, 1, 2, 19, 20, 4, 16, 4, 16)]      # same x, another k
    assert C._projection_groups(ops) == {0: [0, 2]}
    st = co.HostStore()
    lops, _, _ = gpt2.gpt2_layer(st, gpt2.LayerShape(m=8, d=16, d_real=12, heads=3, dh=4, ffn=32, ffn_real=24,
                                                     exp_bits=8, gelu_bits=10, rsqrt_len=256))
    groups = C._projection_groups(lops)
    assert [len(g) for g in groups.values()] == [9]  # q, k, v of every head read the first LayerNorm's output
    assert all(lops[j].x == lops[i].x for i, g in groups.items() for j in g)
