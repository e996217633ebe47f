"""Timed cases for the kernel families of libzkie_b200: the reproduction recipe
of the profiles (run from the repository root).

    python perfcases.py sumcheck --log-size 24
    python perfcases.py mle --log-size 24
    python perfcases.py matmul --m 512 --k 1024 --n 4096
    python perfcases.py commit --log-size 16 --polys 256 --lg-blowup 1
    python perfcases.py virtual --log-size 21
    python perfcases.py logup --log-size 24
    python perfcases.py grind --log-size 24
    python perfcases.py fixed --m 512 --k 1024 --n 4096
    python perfcases.py cache --log-size 25
    python perfcases.py sop --log-size 20 --polys 4
    python perfcases.py shard --m 16 --k 1024 --n 1024
    python perfcases.py split --log-size 18 --polys 32 --gpus 4
    python perfcases.py sweep
    python perfcases.py coset --log-size 20 --polys 256 --gpus 8
    python perfcases.py projection --m 512 --k 1024 --n 4096
    python perfcases.py layer --trace
    python perfcases.py model
    python perfcases.py moe [--cpu | --trace]

Each case prints one JSON line (the sweep one per configuration-2 case):
time per call (CUDA events on the launching stream, after warm-up) and,
where meaningful, the algorithmic HBM bytes per call.  Inputs are synthetic,
uniform canonical field elements.
"""
import argparse
import json
import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from zkie_b200 import _lib  # noqa: E402
from zkie_b200._lib import check, lib  # noqa: E402

P = 0xFFFFFFFF00000001


def _rand(n, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    hi = torch.randint(0, 1 << 32, (n,), generator=g, device="cuda", dtype=torch.int64)
    lo = torch.randint(0, 1 << 32, (n,), generator=g, device="cuda", dtype=torch.int64)
    x = (hi << 32) | lo
    x = torch.where((x < 0) & (x >= -(1 << 32) + 1), x + ((1 << 32) - 1), x)
    return x.view(torch.uint64)


def _time(fn, iters, warmup=2):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(iters):
        fn()
    e1.record(s)
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def _p(a):
    return a.ctypes.data_as(_lib.pu64)


def case_sumcheck(a):
    t = a.log_size
    f, h = _rand(1 << t, 1), _rand(1 << t, 2)
    ch = np.arange(1, t + 1, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15 % P)
    rounds = np.zeros((max(t, 1), 3), dtype=np.uint64)
    finals = np.zeros(2, dtype=np.uint64)
    scr = torch.empty(lib.zkie2_sumcheck_scratch_elems(t), dtype=torch.uint64, device="cuda")
    st = torch.cuda.current_stream().cuda_stream

    def run():
        check(lib.zkie2_sumcheck_prove(f.data_ptr(), h.data_ptr(), t, _p(ch), _p(rounds), _p(finals),
                                       scr.data_ptr(), st), "sumcheck")
    ms = _time(run, a.iters)
    return {"case": "sumcheck", "log_size": t, "ms": ms, "bytes": 16 << t,
            "gbs": (16 << t) / (ms / 1e3) / 1e9}


def case_mle(a):
    t = a.log_size
    v = _rand(1 << t, 3)
    pt = (np.arange(1, t + 1, dtype=np.uint64) * np.uint64(12345)).astype(np.uint64)
    out = _lib.u64(0)
    scr = torch.empty(lib.zkie2_mle_scratch_elems(t), dtype=torch.uint64, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    import ctypes as C

    def run():
        check(lib.zkie2_mle_eval(v.data_ptr(), t, _p(pt), C.byref(out), scr.data_ptr(), st), "mle_eval")
    ms = _time(run, a.iters)
    return {"case": "mle_eval", "log_size": t, "ms": ms, "bytes": 8 << t, "gbs": (8 << t) / (ms / 1e3) / 1e9}


def case_matmul(a):
    m, k, n = a.m, a.k, a.n
    A, B, Cm = _rand(m * k, 4), _rand(k * n, 5), _rand(m * n, 6)
    scr = torch.empty(lib.zkie2_op_matmul_scratch_elems(m, k, n), dtype=torch.uint64, device="cuda")
    lm, lk, ln = m.bit_length() - 1, k.bit_length() - 1, n.bit_length() - 1
    outs = [np.zeros(max(x, 1), dtype=np.uint64) for x in (lm, ln, lk)]
    rounds = np.zeros((max(lk, 1), 3), dtype=np.uint64)
    fin, cl = np.zeros(2, dtype=np.uint64), np.zeros(3, dtype=np.uint64)
    claimed = _lib.u64(0)
    st = torch.cuda.current_stream().cuda_stream
    import ctypes as C

    def run():
        chal = _lib.Challenger()
        lib.zkie2_challenger_xorshift(C.byref(chal), 7)
        check(lib.zkie2_op_matmul_prove(A.data_ptr(), B.data_ptr(), Cm.data_ptr(), m, k, n, C.byref(chal),
                                        _p(outs[0]), _p(outs[1]), _p(outs[2]), C.byref(claimed), _p(rounds),
                                        _p(fin), _p(cl), scr.data_ptr(), st), "op_matmul_prove")
    ms = _time(run, a.iters)
    byts = 8 * (m * k + k * n + m * n)
    return {"case": "op_matmul_prove", "m": m, "k": k, "n": n, "ms": ms, "bytes": byts,
            "gbs": byts / (ms / 1e3) / 1e9}


def case_virtual(a):
    """prove_virtual with the Projection-affine term shape (6 MLEs, 5 degree-2 terms)."""
    import ctypes as C
    t = a.log_size
    mles = [_rand(1 << t, 20 + j) for j in range(6)]
    neg = lambda x: (P - x) % P  # noqa: E731
    terms = [(1, [0, 1]), (neg(1), [0, 2]), (1 << 16, [0, 3]), (neg(1 << 16), [0, 4]), (neg(1 << 15), [0, 5])]
    coeffs = np.array([c for c, _ in terms], dtype=np.uint64)
    off = np.array([0, 2, 4, 6, 8, 10], dtype=np.uint32)
    idx = np.array([j for _, ids in terms for j in ids], dtype=np.uint32)
    ch = np.arange(1, t + 1, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15 % P)
    ptrs = (C.c_void_p * 6)(*[m.data_ptr() for m in mles])
    rounds = np.zeros((max(t, 1), 3), dtype=np.uint64)
    finals = np.zeros(6, dtype=np.uint64)
    scr = torch.empty(lib.zkie2_virtual_scratch_elems(6, t), dtype=torch.uint64, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    pu32 = _lib.pu32

    def run():
        check(lib.zkie2_virtual_prove(ptrs, 6, t, _p(coeffs), off.ctypes.data_as(pu32), idx.ctypes.data_as(pu32),
                                      5, _p(ch), _p(rounds), _p(finals), scr.data_ptr(), st), "virtual")
    ms = _time(run, a.iters)
    return {"case": "virtual_affine6", "log_size": t, "ms": ms, "bytes": 48 << t,
            "gbs": (48 << t) / (ms / 1e3) / 1e9}


def case_logup(a):
    """The logUp fraction tree (prove_fractional_with_challenges) over 2^log_size
    fractions, and the merged lookup columns of 2^(log_size-1) samples into a
    2^(log_size-1) table.  Algorithmic bytes of the tree: every layer of N_l
    fractions reads num and den once and writes the N_l / 2 next fractions
    (24 N_l bytes), about 48 N over all layers."""
    lg = a.log_size
    n = 1 << lg
    num, den = _rand(n, 40), _rand(n, 41)
    full_r = np.arange(1, lg + 1, dtype=np.uint64) * np.uint64(0x9E3779B97F4A7C15 % P)
    cs = np.arange(1, lg + 1, dtype=np.uint64) * np.uint64(0x5851F42D4C957F2D % P)
    rounds = np.zeros(max(2 * lg * (lg - 1), 1), dtype=np.uint64)
    finals = np.zeros(max(7 * lg, 1), dtype=np.uint64)
    fnd = np.zeros(2, dtype=np.uint64)
    scr = torch.empty(lib.zkie2_fractional_scratch_elems(lg), dtype=torch.uint64, device="cuda")
    st = torch.cuda.current_stream().cuda_stream

    def run():
        check(lib.zkie2_fractional_prove(num.data_ptr(), den.data_ptr(), lg, _p(full_r), _p(cs), _p(rounds),
                                         _p(finals), _p(fnd), scr.data_ptr(), st), "fractional")
    ms = _time(run, a.iters)
    half = n // 2
    x = torch.from_numpy(np.random.default_rng(43).integers(0, half, size=half).astype(np.uint32)).cuda()
    table, y = _rand(half, 42), _rand(half, 44)
    onum = torch.empty(n, dtype=torch.uint64, device="cuda")
    oden = torch.empty(n, dtype=torch.uint64, device="cuda")
    lscr = torch.empty(lib.zkie2_lookup_scratch_elems(half), dtype=torch.uint64, device="cuda")

    def cols():
        check(lib.zkie2_lookup_num_den(x.data_ptr(), y.data_ptr(), half, table.data_ptr(), None, half, 0, 3, 5,
                                       onum.data_ptr(), oden.data_ptr(), lscr.data_ptr(), st), "lookup columns")
    ms_cols = _time(cols, a.iters)
    alg = 48 * n
    return {"case": "logup_fraction_tree", "log_size": lg, "ms": ms, "bytes": alg, "gbs": alg / (ms / 1e3) / 1e9,
            "lookup_columns_ms": ms_cols}


def case_grind(a):
    """PoW grinding (zkie2_grind) at --log-size bits from a fixed challenger
    state; the candidate count is data-dependent, so the rate is reported per
    candidate tried (the smallest witness + 1, one permutation each)."""
    from zkie_b200.pow import grind
    sponge = [(0x9E3779B97F4A7C15 * (i + 1)) % P for i in range(16)]
    w = {}

    def run():
        w["w"] = grind(sponge, [5, 6, 7], a.log_size)
    ms = _time(run, a.iters)
    perms = w["w"] + 1
    return {"case": "grind", "bits": a.log_size, "ms": ms, "witness": w["w"],
            "gperm_s_tried": perms / (ms / 1e3) / 1e9}


def case_fixed(a):
    """The fixed-point forward matmul (zkie2_matmul_fixed) on m x k @ k x n with
    16-bit entries, against the exact field kernel on the same inputs;
    tensor-core work = 4 m n k u8 MACs (three GEMMs, the middle one over 2k)."""
    import ctypes as C
    m, k, n = a.m, a.k, a.n
    g = torch.Generator(device="cuda")
    g.manual_seed(3)

    def fx(cnt):
        return _fx_field(torch.randint(-(1 << 15), 1 << 15, (cnt,), generator=g, device="cuda", dtype=torch.int64))
    da, db = fx(m * k), fx(k * n)
    dc = torch.empty(m * n, dtype=torch.uint64, device="cuda")
    dc2 = torch.empty(m * n, dtype=torch.uint64, device="cuda")
    scr = torch.empty(lib.zkie2_matmul_fixed_scratch_elems(m, k, n), dtype=torch.uint64, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    path = C.c_uint32(9)

    def tc():
        check(lib.zkie2_matmul_fixed(da.data_ptr(), db.data_ptr(), m, k, n, dc.data_ptr(), 0, C.byref(path),
                                     scr.data_ptr(), st), "matmul_fixed")

    def field():
        check(lib.zkie2_matmul_field(da.data_ptr(), db.data_ptr(), m, k, n, dc2.data_ptr(), st), "matmul_field")
    ms_tc = _time(tc, a.iters)
    ms_f = _time(field, a.iters)
    same = bool(torch.equal(dc.view(torch.int64), dc2.view(torch.int64)))
    macs = 4 * m * n * k
    return {"case": "matmul_fixed", "m": m, "k": k, "n": n, "path": int(path.value), "ms": ms_tc,
            "field_kernel_ms": ms_f, "equal": same, "tops_u8": macs * 2 / (ms_tc / 1e3) / 1e12}


def _fx_field(x):
    """int64 values in (-2^62, 2^62) -> field elements (from_i64) as uint64 on the
    device: p + x for x < 0 is x + 1 - 2^32 in 64-bit two's complement."""
    return torch.where(x < 0, x + 1 - (1 << 32), x).view(torch.uint64)


def case_cache(a):
    """The ZKIEBCH2 cache file of a WHIR commit of 2^log_size evaluations,
    written from and read back into device buffers (a temporary file)."""
    import os
    import tempfile
    import time

    from zkie_b200.cache import BatchCacheMetadata, read_cache, write_cache
    from zkie_b200.commit import Whir
    n = a.log_size
    com = Whir(n).commit(_rand(1 << n, 50))
    rows = com.lde.numel() // 32
    meta = BatchCacheMetadata("model", "group", ["w"], n, 1, 90, 32, bytes(32))
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "batch.zkc")
        write_cache(path, meta, com.root, com.lde, 32, com.layers)
        t0 = time.perf_counter()
        for _ in range(a.iters):
            write_cache(path, meta, com.root, com.lde, 32, com.layers)
        tw = (time.perf_counter() - t0) / a.iters
        size = os.path.getsize(path)
        t0 = time.perf_counter()
        for _ in range(a.iters):
            read_cache(path, rows, 32)
        tr = (time.perf_counter() - t0) / a.iters
    return {"case": "cache", "log_size": n, "bytes": size, "write_ms": 1e3 * tw, "read_ms": 1e3 * tr,
            "write_gbs": size / tw / 1e9, "read_gbs": size / tr / 1e9}


def case_sop(a):
    """prove_sum_of_products over `polys` table pairs of 2^log_size."""
    t, n = a.log_size, a.polys
    w, v = _rand(n << t, 30), _rand(n << t, 31)
    ch = np.arange(1, t + 1, dtype=np.uint64) * np.uint64(12345)
    rounds = np.zeros((max(t, 1), 3), dtype=np.uint64)
    be = _lib.u64(0)
    scr = torch.empty(lib.zkie2_sum_of_products_scratch_elems(n, t), dtype=torch.uint64, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    import ctypes as C

    def run():
        check(lib.zkie2_sum_of_products_prove(w.data_ptr(), v.data_ptr(), n, t, _p(ch), _p(rounds), C.byref(be),
                                              scr.data_ptr(), st), "sum_of_products")
    ms = _time(run, a.iters)
    byts = 16 * (n << t)
    return {"case": "sum_of_products", "tables": n, "log_size": t, "ms": ms, "bytes": byts,
            "gbs": byts / (ms / 1e3) / 1e9}


def case_shard(a):
    """zkie2_shard_prove_matmul at BASELINE configuration 1 (16 x 1024 x 1024,
    entries uniform in [-2^15, 2^15) embedded in the field)."""
    from zkie_b200.gkr import ShardProver
    m, k, n = a.m, a.k, a.n
    g = np.random.default_rng(5)

    def fx(shape):
        x = g.integers(-(1 << 15), 1 << 15, size=shape, dtype=np.int64)
        return x.astype(np.uint64) + np.where(x < 0, np.uint64(P), np.uint64(0))
    A = torch.from_numpy(fx(m * k)).cuda()
    W = torch.from_numpy(fx(k * n)).cuda()
    prover = ShardProver(m, k, n)

    def run():
        prover.prove(A, W)
    ms = _time(run, a.iters)
    return {"case": "shard_prove_matmul", "m": m, "k": k, "n": n, "ms": ms}


def case_split(a):
    """The split commit over `gpus` ranks emulated on this one GPU (every
    rank's coset LDE, leaf hashes, digest interleave and subtree in turn)."""
    from zkie_b200.multigpu import split_commit_emulated
    lg_l, w, lb, G = a.log_size, a.polys, a.lg_blowup, a.gpus
    d_in = _rand((1 << lg_l) * w, 8)

    def run():
        split_commit_emulated(d_in, lg_l, lb, w, G)
    ms = _time(run, a.iters)
    return {"case": "split_commit_emulated", "log_size": lg_l, "polys": w, "blowup": 1 << lb, "ranks": G, "ms": ms}


def case_coset(a):
    """One coset of the LDE rows as one rank of a `gpus`-way split computes it
    (zkie2_lde_coset: the twist of the replicated input, folded when the rank
    count exceeds the blowup, then the sub-LDE)."""
    lg_l, w, lb, G = a.log_size, a.polys, a.lg_blowup, a.gpus
    lg_g = G.bit_length() - 1
    d_in = _rand((1 << lg_l) * w, 8)
    rows = 1 << (lg_l + lb - lg_g)
    out = torch.empty(rows * w, dtype=torch.uint64, device="cuda")
    scr = torch.empty(max(lib.zkie2_lde_coset_scratch_elems(lg_l, lb, w, lg_g), 2), dtype=torch.uint64,
                      device="cuda")
    s = torch.cuda.current_stream().cuda_stream

    def run():
        check(lib.zkie2_lde_coset(d_in.data_ptr(), out.data_ptr(), scr.data_ptr(), lg_l, lb, w, lg_g, G - 1, s),
              "lde_coset")
    ms = _time(run, a.iters)
    return {"case": "lde_coset", "log_size": lg_l, "polys": w, "blowup": 1 << lb, "ranks": G, "ms": ms,
            "algorithmic_bytes": 8 * w * ((1 << lg_l) + rows)}


def case_projection(a):
    """prove_projection (the projection block) of x (m x k) @ W (k x n),
    16-bit fixed-point inputs, shift 16, inputs and witness resident."""
    from zkie_b200.gkr import XorShift64, matmul_fixed
    from zkie_b200.projection import projection_witness, prove_projection
    m, k, n, shift = a.m, a.k, a.n, 16
    g = np.random.default_rng(11)

    def fx(size, lim):
        x = g.integers(-lim, lim, size=size, dtype=np.int64)
        return torch.from_numpy(x.astype(np.uint64) + np.where(x < 0, np.uint64(P), np.uint64(0))).cuda()
    x, w, b = fx(m * k, 1 << 15), fx(k * n, 1 << 15), fx(m * n, 1 << 20)
    h, _ = matmul_fixed(x, w, m, k, n)
    out, rem, idx = projection_witness(h, b, shift)

    def run():
        prove_projection(x, w, b, out, rem, m, k, n, shift, XorShift64(3))
    ms = _time(run, a.iters)
    return {"case": "prove_projection", "m": m, "k": k, "n": n, "shift": shift, "ms": ms}


def case_layer(a):
    """One GPT-2-small layer shard (zkie_b200.gpt2.GPT2_SMALL, 176 ops) proven
    by a recorded CUDA graph: the replay's device time, and with --trace the
    kernels of one replay (torch.profiler / CUPTI: launches, the sum of kernel
    times against the replay's span, the top kernels by total time)."""
    from zkie_b200 import compose as C
    from zkie_b200 import gpt2
    st = C.Store()
    ops, _, _ = gpt2.gpt2_layer(st, gpt2.GPT2_SMALL)
    C.forward_ops(st, ops)
    master = C.master_transcript(ops, len(ops))

    def make_rng():
        c = master.clone()
        c.absorb_u64(0)
        return c
    gp = C.GraphShardProver(st, ops, [], make_rng, a.streams)
    ms = _time(gp.replay, a.iters)
    res = {"case": "layer_shard_replay", "ops": len(ops), "streams": a.streams, "ms": ms}
    if a.trace:
        res.update(_trace(gp.replay))
        res["forward"] = _trace(lambda: C.forward_ops(st, ops))
    return res


def _trace(fn, top_n=12):
    """The kernels of one call of fn (torch.profiler / CUPTI): launches, the
    span first start -> last end, the sum of kernel durations, the top
    kernels by total time."""
    import collections

    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        fn()
        torch.cuda.synchronize()
    evs = [e for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA]
    iv = sorted((e.time_range.start, e.time_range.end) for e in evs)
    span = iv[-1][1] - iv[0][0]
    total = sum(e - s for s, e in iv)
    agg = collections.defaultdict(lambda: [0, 0.0])
    for e in evs:
        name = e.name.replace("void ", "").replace("zk::(anonymous namespace)::", "").split("(")[0]
        agg[name][0] += 1
        agg[name][1] += e.time_range.end - e.time_range.start
    top = sorted(agg.items(), key=lambda kv: -kv[1][1])[:top_n]
    return {"launches": len(evs), "span_ms": span / 1e3, "kernel_time_sum_ms": total / 1e3,
            "mean_concurrency": total / max(span, 1),
            "top": [[k, n, round(t / 1e3, 3), round(t / total, 4)] for k, (n, t) in top]}


def case_model(a):
    """BASELINE configuration 4 on one GPU: the GPT-2-small graph (embedding
    lookup to Argmax) proven as a DAG of 176-op shards by recorded graphs
    (the bench's cfg4 case)."""
    import bench
    import zkie_b200 as zk
    return {"case": "gpt2_model_dag", **bench.cfg4_case(zk, torch.device("cuda", 0), 0, 1)}


def case_moe(a):
    """BASELINE configuration 5 on one GPU: the DeepSeek-V2-Lite-shaped MoE
    layer proven as one shard by a recorded graph (the bench's cfg5 case);
    with --cpu also the CPU restatement of the same shard."""
    import bench
    import zkie_b200 as zk
    if a.trace:
        from zkie_b200 import compose as C
        from zkie_b200 import deepseek
        st = C.Store()
        ops, _, _ = deepseek.moe_layer(st, deepseek.DSV2_LITE)
        C.forward_ops(st, ops)
        fwd = _trace(lambda: C.forward_ops(st, ops))
        master = C.master_transcript(ops, len(ops))

        def make_rng():
            c = master.clone()
            c.absorb_u64(0)
            return c
        gp = C.GraphShardProver(st, ops, [], make_rng, a.streams)
        gp.replay()
        return {"case": "moe_layer_trace", "streams": a.streams, "replay_ms": _time(gp.replay, a.iters),
                "forward": fwd, "prove_replay": _trace(gp.replay)}
    return {"case": "moe_layer_shard", **bench.moe_case(zk, torch.device("cuda", 0), a.cpu, a.iters)}


def case_sweep(a):
    """batches of 1, 16, 256 polynomials of 2^16,
    2^20, 2^24 coefficients at blowup 2 and 4.  One JSON line per case that
    fits this GPU's free memory (input + LDE + NTT scratch + digest layers),
    commit time with inputs resident."""
    free, _ = torch.cuda.mem_get_info()
    out = []
    for lg_l in (16, 20, 24):
        for w in (1, 16, 256):
            for lb in (1, 2):
                L, H = 1 << lg_l, 1 << (lg_l + lb)
                need = 8 * (L * w + 2 * H * w) + 64 * 2 * H
                case = {"case": "cfg2_commit", "log_size": lg_l, "polys": w, "blowup": 1 << lb}
                if need > 0.9 * free:
                    case["skipped"] = f"needs {need / 2**30:.1f} GiB of {free / 2**30:.1f} GiB free (one GPU)"
                    print(json.dumps(case), flush=True)
                    continue
                d_in = _rand(L * w, 7)
                d_lde = torch.empty(H * w, dtype=torch.uint64, device="cuda")
                d_layers = torch.empty(lib.zkie2_merkle_total_digests(H) * 8, dtype=torch.uint64, device="cuda")
                d_scr = torch.empty(max(lib.zkie2_commit_scratch_elems(lg_l, lb, w), 1), dtype=torch.uint64,
                                    device="cuda")
                st = torch.cuda.current_stream().cuda_stream

                def run():
                    check(lib.zkie2_commit(d_in.data_ptr(), lg_l, lb, w, d_lde.data_ptr(), d_layers.data_ptr(),
                                           d_scr.data_ptr(), st), "commit")
                iters = max(1, min(a.iters, int(2e9 // (H * max(w, 8)))))
                ms = _time(run, iters, warmup=1)
                case.update({"ms": round(ms, 4), "melem_s": round(L * w / (ms / 1e3) / 1e6, 1),
                             "lde_melem_s": round(H * w / (ms / 1e3) / 1e6, 1),
                             "root0": hex(int(d_layers[-8:].cpu().view(torch.int64)[0].item()) & (2**64 - 1))})
                print(json.dumps(case), flush=True)
                del d_in, d_lde, d_layers, d_scr
                torch.cuda.empty_cache()
    return {"case": "cfg2_sweep", "done": True}


def case_commit(a):
    lg_l, w, lb = a.log_size, a.polys, a.lg_blowup
    L, H = 1 << lg_l, 1 << (lg_l + lb)
    d_in = _rand(L * w, 7)
    d_lde = torch.empty(H * w, dtype=torch.uint64, device="cuda")
    d_layers = torch.empty(lib.zkie2_merkle_total_digests(H) * 8, dtype=torch.uint64, device="cuda")
    d_scr = torch.empty(max(lib.zkie2_commit_scratch_elems(lg_l, lb, w), 1), dtype=torch.uint64, device="cuda")
    st = torch.cuda.current_stream().cuda_stream

    def run():
        check(lib.zkie2_commit(d_in.data_ptr(), lg_l, lb, w, d_lde.data_ptr(), d_layers.data_ptr(),
                               d_scr.data_ptr(), st), "commit")
    ms = _time(run, a.iters)
    return {"case": "commit", "log_size": lg_l, "polys": w, "blowup": 1 << lb, "ms": ms,
            "melem_s": L * w / (ms / 1e3) / 1e6}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["sumcheck", "mle", "matmul", "commit", "virtual", "sop", "shard", "split", "sweep",
                                         "logup", "grind", "fixed", "cache", "coset", "projection", "layer",
                                         "model", "moe"])
    ap.add_argument("--gpus", type=int, default=4, help="ranks of the emulated split commit")
    ap.add_argument("--log-size", type=int, default=20)
    ap.add_argument("--polys", type=int, default=16)
    ap.add_argument("--lg-blowup", type=int, default=1)
    ap.add_argument("--m", type=int, default=16)
    ap.add_argument("--k", type=int, default=1024)
    ap.add_argument("--n", type=int, default=1024)
    ap.add_argument("--iters", type=int, default=5)
    ap.add_argument("--trace", action="store_true", help="layer: list one replay's kernels")
    ap.add_argument("--cpu", action="store_true", help="moe: also time the CPU restatement")
    ap.add_argument("--streams", type=int, default=8, help="layer / moe --trace: the prover's streams")
    a = ap.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("perfcases needs a CUDA device")
    check(lib.zkie2_p2_init_default(), "constants")
    res = {"sumcheck": case_sumcheck, "mle": case_mle, "matmul": case_matmul, "commit": case_commit,
           "virtual": case_virtual, "logup": case_logup, "grind": case_grind, "fixed": case_fixed, "cache": case_cache, "sop": case_sop, "shard": case_shard, "split": case_split,
           "sweep": case_sweep, "coset": case_coset, "projection": case_projection, "layer": case_layer,
           "model": case_model, "moe": case_moe}[a.case](a)
    print(json.dumps({k: (round(v, 4) if isinstance(v, float) else v) for k, v in res.items()}), flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
