"""Split commit over several ranks (zkie_b200.multigpu) on CPU: the coset-LDE
math against the oracle's full LDE, the all-to-all / interleave layout by
emulation, and the orchestration itself as world-size 2 and 4 gloo process
groups with oracle-backed compute.  Every case must give the single-device
root."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from tests.mgpu_ops import OracleOps

P = 0xFFFFFFFF00000001


def coeffs(seed, L, w):
    g = np.random.default_rng(seed)
    v = g.integers(0, 2 ** 64, size=(L, w), dtype=np.uint64)
    return np.where(v >= np.uint64(P), v - np.uint64(P), v)


@pytest.mark.parametrize("lg_l,lg_b,w,G", [(5, 1, 3, 2), (5, 1, 3, 4), (4, 2, 2, 4), (4, 1, 5, 8), (6, 2, 1, 2)])
def test_coset_rows_are_lde_rows(orc, consts, lg_l, lg_b, w, G):
    x = coeffs(lg_l * 10 + G, 1 << lg_l, w)
    full = orc.lde(x, lg_b)
    ops = OracleOps(orc, consts)
    lg_g = G.bit_length() - 1
    for g in range(G):
        rows = ops.lde_coset(torch.from_numpy(x.reshape(-1)), lg_l, lg_b, w, lg_g, g).numpy()
        assert np.array_equal(rows.reshape(-1, w), full[g::G]), (g, G)


@pytest.mark.parametrize("lg_l,lg_b,w,G", [(5, 1, 3, 2), (5, 1, 9, 4), (4, 2, 2, 4), (5, 1, 2, 8)])
def test_emulated_split_root(orc, consts, lg_l, lg_b, w, G):
    from zkie_b200.multigpu import split_commit_emulated
    x = coeffs(lg_l + 100 * G, 1 << lg_l, w)
    _, want = orc.merkle_tree(consts, orc.lde(x, lg_b))
    root, _ = split_commit_emulated(torch.from_numpy(x.reshape(-1)), lg_l, lg_b, w, G, ops=OracleOps(orc, consts))
    assert np.array_equal(root, want)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, lg_l, lg_b, w, out_dir):
    import torch.distributed as dist

    from oracle import oracle as orc
    from zkie_b200.multigpu import split_commit
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x = coeffs(77, 1 << lg_l, w)
        res = split_commit(torch.from_numpy(x.reshape(-1)), lg_l, lg_b, w,
                           ops=OracleOps(orc, orc.p2_constants(1)))
        np.save(os.path.join(out_dir, f"root{rank}.npy"), res.root)
        np.save(os.path.join(out_dir, f"lde{rank}.npy"), res.lde.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_gloo_split_commit(orc, consts, tmp_path, world):
    lg_l, lg_b, w = 5, 1, 3
    mp.start_processes(_rank_main, args=(world, _free_port(), lg_l, lg_b, w, str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    x = coeffs(77, 1 << lg_l, w)
    full = orc.lde(x, lg_b)
    _, want = orc.merkle_tree(consts, full)
    for r in range(world):
        assert np.array_equal(np.load(tmp_path / f"root{r}.npy"), want), r
        assert np.array_equal(np.load(tmp_path / f"lde{r}.npy").reshape(-1, w), full[r::world]), r


def _sc_rank_main(rank, world, port, t, out_dir):
    import torch.distributed as dist

    from oracle import oracle as orc
    from tests.mgpu_ops import OracleSumcheckOps
    from zkie_b200.multigpu import split_sumcheck
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        f, h, ch = coeffs(5, 1 << t, 1).reshape(-1), coeffs(6, 1 << t, 1).reshape(-1), coeffs(7, t, 1).reshape(-1)
        n = (1 << t) // world
        rounds, fe, he = split_sumcheck(f[rank * n:(rank + 1) * n], h[rank * n:(rank + 1) * n], t, ch,
                                        ops=OracleSumcheckOps(orc), device=torch.device("cpu"))
        np.save(os.path.join(out_dir, f"sc{rank}.npy"),
                np.concatenate([rounds.reshape(-1), np.array([fe, he], dtype=np.uint64)]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,t", [(2, 9), (4, 10), (4, 2)])
def test_gloo_split_sumcheck(orc, tmp_path, world, t):
    """Hypercube split by the high variables: local rounds, one all-reduce of
    the round messages (32-bit limbs), last log2(world) rounds on every rank."""
    mp.start_processes(_sc_rank_main, args=(world, _free_port(), t, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    f, h, ch = coeffs(5, 1 << t, 1).reshape(-1), coeffs(6, 1 << t, 1).reshape(-1), coeffs(7, t, 1).reshape(-1)
    rounds, finals = orc.sumcheck_prove(f, h, ch)
    want = np.concatenate([np.asarray(rounds, dtype=np.uint64).reshape(-1), np.asarray(finals, dtype=np.uint64)])
    for r in range(world):
        assert np.array_equal(np.load(tmp_path / f"sc{r}.npy"), want), r
