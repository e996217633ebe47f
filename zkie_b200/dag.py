"""prove_shard_dag (crates/zkie-ops/src/compose.rs:2289-2346) with its shards
spread over ranks, one process per GPU.

The reference proves the shards of a DAG in parallel on one host
(`ranges.par_iter()`, :2305-2313): every shard's challenges come from its own
child transcript (the master transcript over the statement, plus the shard
index), so shards are independent once the witness exists, and only the
tensors claimed by more than one shard are bound afterwards, with the master
transcript (:2315-2345).  The split here is the same one, across GPUs: rank r
proves the shards si with si % world == r (each rank holds the whole witness:
the forward pass is cheap next to the proof), rank 0 gathers every shard's
claims and proves the cross-shard bindings.  No collective touches the data
path; the gather carries claims (points and values) and each shard's proof
summary.

The orchestration is host logic over a few callables, so the same code runs
the device prover (``prove_dag_ranks`` with ``device_provers``) and, in the
CPU tests, the CPU restatement under a gloo process group.
"""
import hashlib
from dataclasses import dataclass
from typing import Callable, List

import numpy as np


def shard_ranges(op_count: int, ops_per_shard: int):
    """compose.rs:2264-2274."""
    ops_per_shard = max(ops_per_shard, 1)
    return [(s, min(s + ops_per_shard, op_count)) for s in range(0, op_count, ops_per_shard)]


def shard_owner(si: int, world: int) -> int:
    return si % world


def digest(canon) -> str:
    """SHA-256 (first 16 hex digits) over every value of a canonical proof
    form: dict keys sorted, sequence lengths, arrays as little-endian u64."""
    h = hashlib.sha256()

    def walk(v):
        if isinstance(v, dict):
            for k in sorted(v):
                h.update(str(k).encode())
                walk(v[k])
        elif isinstance(v, (list, tuple)):
            h.update(b"[%d" % len(v))
            for x in v:
                walk(x)
        elif isinstance(v, np.ndarray):
            h.update(np.ascontiguousarray(v, dtype=np.uint64).tobytes())
        elif isinstance(v, str):
            h.update(v.encode())
        else:
            h.update(int(v).to_bytes(8, "little"))
    walk(canon)
    return h.hexdigest()[:16]


@dataclass
class DagProvers:
    """What the orchestration needs from a prover: the master transcript of a
    statement, a shard's child, a shard proof (store, ops, rng) -> proof, the
    proof's raw claims [(tensor, point, value)], its summary for the gather
    (the canonical form, or a digest of it), and the same_poly binding of one
    tensor's claims with the master transcript."""
    master: Callable
    child: Callable
    prove: Callable
    claims: Callable
    summary: Callable
    same_poly: Callable
    commit: Callable = None  # (store, tensor) -> the WHIR base commitment's root (8 values)
    # optional split of prove: start(store, ops, rng) enqueues and returns a
    # handle, finish(handle) returns the proof; all of a rank's shards are
    # started before the first is finished
    start: Callable = None
    finish: Callable = None


@dataclass
class DagResult:
    """Rank 0's view: every shard's summary in shard order, the cross-shard
    tensors and their bindings (canonical), the roots of the cross-shard
    tensors' WHIR base commitments (when the provers commit), and the DAG
    digest."""
    shards: List
    cross_tensors: List[int]
    cross_binds: List
    digest: str
    boundary_roots: List = None


def dag_digest(shard_summaries, cross_tensors, cross_binds, boundary_roots=None) -> str:
    parts = [s if isinstance(s, str) or s is None else digest(s) for s in shard_summaries]
    parts = ["" if s is None else s for s in parts]
    body = [parts, list(cross_tensors), [b for b in cross_binds]]
    if boundary_roots is not None:
        body.append([np.asarray(r, dtype=np.uint64) for r in boundary_roots])
    return digest(body)


def prove_dag_ranks(store, ops, ops_per_shard: int, provers: DagProvers, rank: int = 0, world: int = 1,
                    gather=None):
    """Prove the shards this rank owns; rank 0 returns the DagResult (other
    ranks None).  ``gather(obj)`` returns every rank's obj (in rank order) on
    rank 0 and None elsewhere; with world 1 it is not needed."""
    ranges = shard_ranges(len(ops), ops_per_shard)
    master = provers.master(ops, ops_per_shard)
    mine = []
    owned = [si for si in range(len(ranges)) if shard_owner(si, world) == rank]

    def record(si, proof):
        claims = [(int(t), np.asarray(pt, dtype=np.uint64), int(v)) for t, pt, v in provers.claims(proof)]
        mine.append((si, claims, provers.summary(proof)))
    if provers.start is not None:
        handles = [(si, provers.start(store, ops[ranges[si][0]:ranges[si][1]], provers.child(master, si)))
                   for si in owned]
        for si, h in handles:
            record(si, provers.finish(h))
    else:
        for si in owned:
            s, e = ranges[si]
            record(si, provers.prove(store, ops[s:e], provers.child(master, si)))
    everyone = gather(mine) if world > 1 else [mine]
    if rank != 0:
        return None
    by_shard = sorted((x for part in everyone for x in part), key=lambda x: x[0])
    assert [x[0] for x in by_shard] == list(range(len(ranges))), "a shard is missing from the gather"
    by_tensor, owners = {}, {}
    for si, claims, _ in by_shard:
        for t, pt, v in claims:
            by_tensor.setdefault(t, []).append((pt, v))
            owners.setdefault(t, set()).add(si)
    cross = [t for t in sorted(by_tensor) if len(owners[t]) > 1]
    binds = [provers.same_poly(store, t, by_tensor[t], master) for t in cross]
    summaries = [x[2] for x in by_shard]
    # prove_committed_shard_dag (compose.rs:2796-2806) commits every
    # cross-shard tensor with Whir::with_params(arity, 90, 17); its openings
    # (committed_cross_bind) are not part of this prover
    roots = [provers.commit(store, t) for t in cross] if provers.commit else None
    return DagResult(summaries, cross, binds, dag_digest(summaries, cross, binds, roots), roots)


def torch_gather(group=None):
    """gather over torch.distributed (gather_object to rank 0)."""
    import torch.distributed as dist

    def gather(obj):
        out = [None] * dist.get_world_size(group) if dist.get_rank(group) == 0 else None
        dist.gather_object(obj, out, dst=0, group=group)
        return out
    return gather


# ---- the device prover -----------------------------------------------------------------------
def device_provers(summary: str = "digest", graph: bool = False, streams: int = 8, graphs=None) -> DagProvers:
    """DagProvers over zkie_b200.compose.  summary "digest" keeps each shard's
    proof on its rank (only claims and a digest of the proof travel; the
    digest downloads the proof's lookup columns, hundreds of MB per GPT-2
    layer), "canonical" gathers the whole canonical form (small statements),
    "none" only the claims.  graph=True records each shard's prove as a CUDA
    graph and replays it; the recorded graphs live in ``graphs`` (a dict,
    shared between provers when given) and on the returned object."""
    from . import compose as C

    def master(ops, ops_per_shard):
        return C.master_transcript(ops, ops_per_shard)

    def child(m, si):
        c = m.clone()
        c.absorb_u64(si)
        return c

    graphs = {} if graphs is None else graphs

    def recorded(store, shard_ops, rng):
        key = (shard_ops[0].__class__.__name__, id(shard_ops[0]), len(shard_ops))
        gp = graphs.get(key)
        if gp is None:
            state = rng.clone()
            gp = C.GraphShardProver(store, shard_ops, [], lambda: state.clone(), streams)
            graphs[key] = gp
        return gp

    def prove(store, shard_ops, rng):
        if not graph:
            return C.OpShardProver(store, rng, streams).prove(shard_ops, [])
        return recorded(store, shard_ops, rng).prove()

    def start(store, shard_ops, rng):
        gp = recorded(store, shard_ops, rng)
        gp.start()
        return gp

    def finish(gp):
        return gp.finish()

    def claims(proof):
        return proof.claims

    def summ(proof):
        if summary == "none":
            return None
        can = proof.canonical()
        return digest(can) if summary == "digest" else can

    def same_poly(store, t, cs, m):
        pr = C.OpShardProver(store, m, streams=1)
        b = pr.same_poly(store.get(t), cs)
        pr.pend.fetch()
        return b().canonical()

    def commit(store, t):
        from .commit import Whir
        v = store.get(t)
        return Whir.with_params(v.numel().bit_length() - 1, 90, 17).commit(v).root

    p = DagProvers(master, child, prove, claims, summ, same_poly, commit,
                   start if graph else None, finish if graph else None)
    p.graphs = graphs
    return p
