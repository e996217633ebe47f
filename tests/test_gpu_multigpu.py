"""Split commit on the GPU: zkie2_lde_coset against the full zkie2_lde, the
whole split path emulated on one device (all G ranks in turn) against the
single-device commit root, and, when the box has two or more GPUs, the real
NCCL split over two ranks."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

P = 0xFFFFFFFF00000001
pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _constants(zk):
    zk.check(zk.lib.zkie2_p2_init_default(), "constants")


def coeffs(seed, L, w):
    g = np.random.default_rng(seed)
    v = g.integers(0, 2 ** 64, size=(L, w), dtype=np.uint64)
    return np.where(v >= np.uint64(P), v - np.uint64(P), v)


@pytest.mark.parametrize("lg_l,lg_b,w,G", [(4, 1, 3, 2), (10, 1, 8, 2), (10, 1, 8, 8), (12, 2, 5, 4),
                                          (12, 1, 16, 16), (16, 1, 32, 8), (18, 1, 4, 2)])
def test_lde_coset_rows(zk, lg_l, lg_b, w, G):
    from zkie_b200.multigpu import DeviceOps
    x = torch.from_numpy(coeffs(lg_l + G, 1 << lg_l, w).reshape(-1)).cuda()
    full = zk.commit(x.reshape(1 << lg_l, w), lg_b).lde.reshape(-1, w)
    ops = DeviceOps()
    lg_g = G.bit_length() - 1
    for g in range(G):
        rows = ops.lde_coset(x, lg_l, lg_b, w, lg_g, g).reshape(-1, w)
        assert torch.equal(rows.view(torch.int64), full.view(torch.int64)[g::G]), (g, G)


def test_lde_coset_matches_oracle(zk, orc):
    from zkie_b200.multigpu import DeviceOps
    lg_l, lg_b, w, G = 8, 1, 4, 4
    x = coeffs(3, 1 << lg_l, w)
    full = orc.lde(x, lg_b)
    for g in range(G):
        rows = DeviceOps().lde_coset(torch.from_numpy(x.reshape(-1)).cuda(), lg_l, lg_b, w, 2, g)
        assert np.array_equal(rows.cpu().numpy().reshape(-1, w), full[g::G])


@pytest.mark.parametrize("lg_l,lg_b,w,G", [(10, 1, 16, 2), (12, 1, 32, 4), (14, 1, 32, 8), (16, 2, 8, 8)])
def test_split_commit_emulated_root(zk, lg_l, lg_b, w, G):
    from zkie_b200.multigpu import split_commit_emulated
    x = torch.from_numpy(coeffs(lg_l * G, 1 << lg_l, w).reshape(-1)).cuda()
    want = zk.commit(x.reshape(1 << lg_l, w), lg_b).root
    root, _ = split_commit_emulated(x, lg_l, lg_b, w, G)
    assert np.array_equal(root, np.asarray(want, dtype=np.uint64))


def test_split_committer_run_host_single_rank(zk):
    """SplitCommitter.run_host without a process group (one rank): pinned
    input slice in, the LDE downloaded on a side stream while the rows are
    hashed, the digest layers back; two calls in a row, each equal to the
    device commit."""
    from zkie_b200.multigpu import SplitCommitter
    lg_l, lg_b, w = 14, 1, 32
    x = coeffs(77, 1 << lg_l, w)
    want = zk.commit(torch.from_numpy(x).cuda(), lg_b)
    want_lde = want.lde.reshape(-1).view(torch.int64).cpu()
    want_layers = want.layers.view(torch.int64).cpu()
    H = 1 << (lg_l + lg_b)
    sc = SplitCommitter(lg_l, lg_b, w)
    h_part = torch.from_numpy(x.view(np.int64).reshape(-1).copy()).pin_memory()
    h_lde = torch.empty(H * w, dtype=torch.int64).pin_memory()
    h_layers = torch.empty(zk.lib.zkie2_merkle_total_digests(H) * 8, dtype=torch.int64).pin_memory()
    for call in range(2):
        h_lde.zero_()
        h_layers.zero_()
        phases = [] if call else None  # the second call also records its phase times
        root = sc.run_host(h_part, h_lde, h_layers, phases)
        if call:
            ph = phases[0]
            assert set(ph) == {"upload", "allgather", "lde_done", "commit", "lde_download", "layers_download"}
            assert 0 <= ph["upload"] <= ph["allgather"] <= ph["lde_done"] <= ph["commit"] <= ph["layers_download"]
            assert ph["lde_done"] <= ph["lde_download"]
        assert torch.equal(h_lde, want_lde)
        assert torch.equal(h_layers, want_layers)
        assert np.array_equal(np.asarray(root).view(np.uint64), np.asarray(want.root, dtype=np.uint64))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _nccl_rank(rank, world, port, lg_l, lg_b, w, out_dir):
    import datetime

    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        import zkie_b200 as zk
        from zkie_b200.multigpu import split_commit
        zk.check(zk.lib.zkie2_p2_init_default(), "constants")
        x = torch.from_numpy(coeffs(91, 1 << lg_l, w).reshape(-1)).cuda()
        res = split_commit(x, lg_l, lg_b, w)
        torch.cuda.synchronize()
        np.save(os.path.join(out_dir, f"root{rank}.npy"), res.root)
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_split_commit_nccl_two_ranks(zk, tmp_path):
    lg_l, lg_b, w = 14, 1, 32
    mp.start_processes(_nccl_rank, args=(2, _free_port(), lg_l, lg_b, w, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    x = torch.from_numpy(coeffs(91, 1 << lg_l, w).reshape(-1)).cuda()
    want = np.asarray(zk.commit(x.reshape(1 << lg_l, w), lg_b).root, dtype=np.uint64)
    for r in range(2):
        assert np.array_equal(np.load(tmp_path / f"root{r}.npy"), want), r


@pytest.mark.parametrize("G,t", [(2, 12), (4, 20), (8, 16)])
def test_split_sumcheck_math_on_one_gpu(zk, orc, G, t):
    """The split-sumcheck combination on one device: local proofs of the G
    high-variable chunks, round messages summed mod p, the last log2(G) rounds
    over the gathered folded values -- equal to the single-device proof."""
    from zkie_b200.multigpu import DeviceSumcheckOps
    f, h = coeffs(t, 1 << t, 1).reshape(-1), coeffs(t + 1, 1 << t, 1).reshape(-1)
    ch = coeffs(t + 2, t, 1).reshape(-1)
    lg_g = G.bit_length() - 1
    n = (1 << t) // G
    ops = DeviceSumcheckOps()
    loc = [ops.sumcheck(f[g * n:(g + 1) * n], h[g * n:(g + 1) * n], ch[:t - lg_g]) for g in range(G)]
    summed = np.array([[sum(int(p[0][r][c]) for p in loc) % P for c in range(3)] for r in range(t - lg_g)],
                      dtype=np.uint64)
    tail, fe, he = ops.sumcheck(np.array([p[1] for p in loc], dtype=np.uint64),
                                np.array([p[2] for p in loc], dtype=np.uint64), ch[t - lg_g:])
    rounds, finals = orc.sumcheck_prove(f, h, ch)
    assert np.array_equal(np.concatenate([summed, tail]), rounds)
    assert (fe, he) == (int(finals[0]), int(finals[1]))


def _nccl_sumcheck_rank(rank, world, port, t, out_dir):
    import datetime

    import torch.distributed as dist
    torch.cuda.set_device(rank)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from zkie_b200.multigpu import split_sumcheck
        f, h = coeffs(31, 1 << t, 1).reshape(-1), coeffs(32, 1 << t, 1).reshape(-1)
        ch = coeffs(33, t, 1).reshape(-1)
        n = (1 << t) // world
        df = torch.from_numpy(f[rank * n:(rank + 1) * n].copy()).cuda()
        dh = torch.from_numpy(h[rank * n:(rank + 1) * n].copy()).cuda()
        rounds, fe, he = split_sumcheck(df, dh, t, ch)
        np.save(os.path.join(out_dir, f"sc{rank}.npy"),
                np.concatenate([rounds.reshape(-1), np.array([fe, he], dtype=np.uint64)]))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_split_sumcheck_nccl_two_ranks(orc, tmp_path):
    t = 20
    mp.start_processes(_nccl_sumcheck_rank, args=(2, _free_port(), t, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    f, h = coeffs(31, 1 << t, 1).reshape(-1), coeffs(32, 1 << t, 1).reshape(-1)
    rounds, finals = orc.sumcheck_prove(f, h, coeffs(33, t, 1).reshape(-1))
    want = np.concatenate([np.asarray(rounds, dtype=np.uint64).reshape(-1), np.asarray(finals, dtype=np.uint64)])
    for r in range(2):
        assert np.array_equal(np.load(tmp_path / f"sc{r}.npy"), want), r


# ---- the C-ABI multi-GPU context (zkie2_mg_*) ------------------------------------------------
MG_COMMIT_CASES = [(14, 1, 32), (12, 2, 9), (12, 0, 8), (10, 1, 256), (11, 1, 200)]


def _mg_check_rank(zk, ctx, rank, world):
    """Split commits and split sumchecks through the C ABI on this rank,
    each compared with the single-device result on this rank's GPU."""
    import ctypes as C
    lib = zk.lib
    s = torch.cuda.current_stream().cuda_stream
    ok = []
    for lg_l, lg_b, w in MG_COMMIT_CASES:
        H = 1 << (lg_l + lg_b)
        x = torch.from_numpy(coeffs(lg_l * 7 + w, 1 << lg_l, w).reshape(-1)).cuda()
        n_local = H // world
        lde = torch.empty(n_local * w, dtype=torch.uint64, device="cuda")
        layers = torch.empty(lib.zkie2_merkle_total_digests(n_local) * 8, dtype=torch.uint64, device="cuda")
        top = torch.empty(lib.zkie2_mg_top_digests(world) * 8, dtype=torch.uint64, device="cuda")
        scr = torch.empty(lib.zkie2_mg_split_commit_scratch_elems(lg_l, lg_b, w, world), dtype=torch.uint64,
                          device="cuda")
        root = np.zeros(8, dtype=np.uint64)
        for _ in range(2):  # two calls in a row on the same buffers
            rc = lib.zkie2_mg_split_commit(ctx, x.data_ptr(), lg_l, lg_b, w, lde.data_ptr(), layers.data_ptr(),
                                           top.data_ptr(), scr.data_ptr(), root.ctypes.data_as(C.POINTER(C.c_uint64)),
                                           s)
            assert rc == 0, rc
        want = zk.commit(x.reshape(1 << lg_l, w), lg_b)
        want_rows = want.lde.reshape(H, w)[rank::world].reshape(-1)
        ok.append(bool(np.array_equal(root, np.asarray(want.root, dtype=np.uint64))))
        ok.append(bool(torch.equal(lde.view(torch.int64), want_rows.view(torch.int64))))
        # the host-buffer form: this rank's input rows in, LDE rows, subtree layers and root out
        rows = (1 << lg_l) // world
        h_part = x.view(torch.int64)[rank * rows * w:(rank + 1) * rows * w].cpu().pin_memory()
        h_lde = torch.zeros(n_local * w, dtype=torch.int64).pin_memory()
        h_layers = torch.zeros(layers.numel(), dtype=torch.int64).pin_memory()
        hscr = torch.empty(lib.zkie2_mg_split_commit_host_scratch_elems(lg_l, lg_b, w, world), dtype=torch.uint64,
                           device="cuda")
        for _ in range(2):
            root2 = np.zeros(8, dtype=np.uint64)
            rc = lib.zkie2_mg_split_commit_host(ctx, h_part.data_ptr(), lg_l, lg_b, w, h_lde.data_ptr(),
                                                h_layers.data_ptr(), root2.ctypes.data_as(C.POINTER(C.c_uint64)),
                                                hscr.data_ptr())
            assert rc == 0, rc
            ok.append(bool(np.array_equal(root2, root)))
        ok.append(bool(torch.equal(h_lde, want_rows.view(torch.int64).cpu())))
        ok.append(bool(torch.equal(h_layers, layers.view(torch.int64).cpu())))
    for t in (20, world.bit_length() - 1, 9):
        f, h = coeffs(40 + t, 1 << t, 1).reshape(-1), coeffs(50 + t, 1 << t, 1).reshape(-1)
        ch = coeffs(60 + t, max(t, 1), 1).reshape(-1)[:t].copy()
        n = (1 << t) // world
        df = torch.from_numpy(f[rank * n:(rank + 1) * n].copy()).cuda()
        dh = torch.from_numpy(h[rank * n:(rank + 1) * n].copy()).cuda()
        scr = torch.empty(lib.zkie2_mg_split_sumcheck_scratch_elems(t, world), dtype=torch.uint64, device="cuda")
        rounds = np.zeros((max(t, 1), 3), dtype=np.uint64)
        fin = np.zeros(2, dtype=np.uint64)
        P64 = C.POINTER(C.c_uint64)
        rc = lib.zkie2_mg_split_sumcheck(ctx, df.data_ptr(), dh.data_ptr(), t, ch.ctypes.data_as(P64),
                                         rounds.ctypes.data_as(P64), fin.ctypes.data_as(P64), scr.data_ptr(), s)
        assert rc == 0, rc
        want = zk.sumcheck_prove(f, h, 0, ch)
        ok.append(bool(np.array_equal(rounds[:t], want.rounds)))
        ok.append((int(fin[0]), int(fin[1])) == (want.f_eval, want.h_eval))
    return ok


def test_mg_context_single_rank(zk):
    """zkie2_mg_* with a one-rank communicator: the split commit and split
    sumcheck entry points reduce to the single-device results."""
    import ctypes as C
    lib = zk.lib
    assert lib.zkie2_mg_available() == 1
    uid = C.create_string_buffer(128)
    assert lib.zkie2_mg_unique_id(uid) == 0
    ctx = C.c_void_p()
    assert lib.zkie2_mg_init(uid, 1, 0, C.byref(ctx)) == 0
    try:
        assert (lib.zkie2_mg_rank(ctx), lib.zkie2_mg_size(ctx)) == (0, 1)
        assert all(_mg_check_rank(zk, ctx, 0, 1))
    finally:
        assert lib.zkie2_mg_destroy(ctx) == 0


def _mg_rank(rank, world, out_dir):
    import ctypes as C
    import time
    torch.cuda.set_device(rank)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    import zkie_b200 as zk
    lib = zk.lib
    path = os.path.join(out_dir, "uid.bin")
    uid = C.create_string_buffer(128)
    if rank == 0:
        assert lib.zkie2_mg_unique_id(uid) == 0
        with open(path + ".tmp", "wb") as fh:
            fh.write(uid.raw)
        os.replace(path + ".tmp", path)
    else:
        t0 = time.time()
        while not os.path.exists(path):
            assert time.time() - t0 < 60, "rank 0 never wrote the NCCL id"
            time.sleep(0.05)
        uid = C.create_string_buffer(open(path, "rb").read(), 128)
    ctx = C.c_void_p()
    assert lib.zkie2_mg_init(uid, world, rank, C.byref(ctx)) == 0
    try:
        ok = _mg_check_rank(zk, ctx, rank, world)
        np.save(os.path.join(out_dir, f"mg{rank}.npy"), np.array(ok))
    finally:
        lib.zkie2_mg_destroy(ctx)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_mg_context_two_ranks(zk, tmp_path):
    """zkie2_mg_split_commit / zkie2_mg_split_sumcheck over a two-rank NCCL
    communicator made by the library (zkie2_mg_unique_id + zkie2_mg_init):
    every rank's root, LDE rows and proof equal the single-device ones."""
    mp.start_processes(_mg_rank, args=(2, str(tmp_path)), nprocs=2, join=True, start_method="spawn")
    for r in range(2):
        ok = np.load(tmp_path / f"mg{r}.npy")
        assert ok.all(), (r, ok)
