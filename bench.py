#!/usr/bin/env python3
"""Commit throughput of the zkIE shard-commit hot path on B200.

Metric: "shard prove s; commit Melem/s (NTT+Merkle) at 1/2/4/8
B200 vs host CPU".  The value reported is commit throughput in input field
elements per second (Melem/s) on BASELINE configuration 2 (raw commit sweep),
case: 256 polynomials of 2^20 coefficients each, blowup 2 -- an LDE of
2^21 x 256 Goldilocks elements, then the Poseidon2-16 Merkle tree over its
2^21 rows.  One step = one full commit (LDE NTT + leaf hashing + tree).

  value: inputs resident in HBM, device-side timing (CUDA events on the stream
         the kernels run on), max over ranks.
  e2e:   the same commit through the host-buffer C-ABI call zkie2_commit_host
         (pinned coefficients in, LDE + all digest layers + root out).

N > 1: one process per GPU, and ONE commit of the same workload split over
the N GPUs (strong scaling): each GPU computes a coset of the LDE rows and
hashes them, one NCCL all-to-all of 64-byte leaf digests gives each GPU a
contiguous leaf block, and an all-gather of the N subtree roots finishes the
tree.  The root is checked against the single-GPU commit of the same input.

--impl reference times the reference algorithm on the host cores (the C
restatement under oracle/, OpenMP over all cores -- the reference itself is
Rust and cannot be built in this image) on bounded samples of the same
workload.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "shard prove s; commit Melem/s (NTT+Merkle) at 1/2/4/8 B200 vs host CPU"
UNIT = "Melem/s"
P = 0xFFFFFFFF00000001
LG_L, W, LG_B = 20, 256, 1
HBM_FALLBACK_GBS = 6650.0
CPU_LABEL = "C restatement, not the reference binary"
MULS_PER_PERM = 8 * 16 * 4 + 22 * 4 + 22
# ALU-pipe thread instructions per Poseidon2 permutation of k_leaf_rows:
# sm__inst_executed_pipe_alu.sum (1,428,619,264 warp instructions) x 32 over the
# 4,194,304 permutations of one ncu capture (2^21 rows x 16 columns).
ALU_INST_PER_PERM = 1428619264 * 32 / 4194304
ALU_WARP_INST_PER_SM_CYCLE = 2  # integer ALU pipe: 16 lanes per cycle in each of 4 sub-partitions


def alu_pipe_roofline(dev, perm_rate, clocks):
    """The leaf kernel against the integer ALU pipe's issue peak (the pipe ncu
    shows binding): achieved ALU thread-instructions per second = permutations
    per second x ALU instructions per permutation (from the capture); peak =
    SMs x 64 lanes x the SM clock sampled under load (else the max clock)."""
    import torch
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    mhz = (clocks or {}).get("sm_mhz") or (clocks or {}).get("sm_max_mhz") or 1965.0
    peak = sms * ALU_WARP_INST_PER_SM_CYCLE * 32 * mhz * 1e6
    ach = perm_rate * ALU_INST_PER_PERM
    return {"achieved": round(ach / 1e12, 3), "peak": round(peak / 1e12, 3), "unit": "T ALU thread-instr/s",
            "frac": round(ach / peak, 4), "inst_per_perm": round(ALU_INST_PER_PERM, 1), "sm_mhz": mhz,
            "source": "sm__inst_executed_pipe_alu.sum of one ncu capture of k_leaf_rows / its permutations; "
                      "peak = 2 warp instructions per SM per cycle"}


def workload_config(lg_l, w, lg_b, n_gpus):
    return {
        "workload": f"cfg2 raw commit: {w} polys x 2^{lg_l} coeffs, blowup {1 << lg_b}, LDE NTT + Poseidon2-16 Merkle over rows",
        "polys": w, "log_size": lg_l, "blowup": 1 << lg_b,
        "lde_rows": 1 << (lg_l + lg_b),
        "bytes_in_per_rank": 8 * w << lg_l,
        "l2_policy": "inputs (2 GiB) and LDE (4 GiB) per step exceed the 126 MB L2; no flush",
        "parallelism": "single GPU" if n_gpus == 1 else
                       f"one commit split over {n_gpus} GPUs: coset rows per GPU, NCCL all-to-all of leaf digests, "
                       "all-gather of subtree roots",
    }


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="zkie_b200", choices=["zkie_b200", "reference"])
    ap.add_argument("--lg-size", type=int, default=LG_L)
    ap.add_argument("--polys", type=int, default=W)
    ap.add_argument("--lg-blowup", type=int, default=LG_B)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-big", action="store_true", help="skip the 256 x 2^24 and expert-stack commits")
    ap.add_argument("--no-cfg4", action="store_true", help="skip the 12-layer GPT-2 shard DAG")
    ap.add_argument("--no-moe", action="store_true", help="skip the DeepSeek-V2-Lite-shaped MoE layer shard")
    ap.add_argument("--cpu-moe", action="store_true", help="also time the MoE layer on the CPU restatement (minutes)")
    return ap.parse_args()


# ---- CPU side (oracle) --------------------------------------------------------------------
def host_threads():
    """Cores this process may run on (torch.distributed.run sets
    OMP_NUM_THREADS=1 for its ranks; the CPU baseline sets its own count)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_commit_rate(lg_rows, w, lg_b, seed=7):
    """Oracle LDE + Merkle commit of a (2^lg_rows x w) sample on every host
    thread; returns (Melem/s, seconds)."""
    import numpy as np
    from oracle import oracle as orc
    orc.set_threads(host_threads())
    consts = orc.p2_constants(1)
    m = np.random.default_rng(seed).integers(0, P, size=(1 << lg_rows, w), dtype=np.uint64)
    t0 = time.perf_counter()
    lde = orc.lde(m, lg_b)
    orc.merkle_tree(consts, lde)
    dt = time.perf_counter() - t0
    return m.size / dt / 1e6, dt


def cpu_sample_rows(w, lg_b, target_s):
    """Sample height (log2) for about target_s seconds, from the rate of a
    2^12-row probe (large enough that the per-call setup does not set it)."""
    rate, _ = cpu_commit_rate(12, w, lg_b)
    rows = max(1, int(target_s * rate * 1e6 / w))
    return min(max(8, rows.bit_length() - 1), 19)


def cpu_lanes():
    """SIMD lanes of the oracle's packed field loops on this host (8 with
    AVX-512F, 4 with AVX2, 0 scalar)."""
    from oracle import oracle as orc
    return orc.set_lanes(-1)


def cpu_baseline(w, lg_b, target_s=10.0):
    lg_rows = cpu_sample_rows(w, lg_b, target_s)
    rate, dt = cpu_commit_rate(lg_rows, w, lg_b)
    return {"value": round(rate, 3), "unit": UNIT, "cores": host_threads(), "kind": "port", "label": CPU_LABEL,
            "sample": f"oracle/zkie_oracle.c LDE + Merkle of {w} polys x 2^{lg_rows} coeffs (blowup {1 << lg_b}), "
                      f"OpenMP over {host_threads()} host threads, {cpu_lanes()} SIMD lanes per field op, {dt:.1f} s"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    lg_rows = cpu_sample_rows(args.polys, args.lg_blowup, target_s=3.0)
    for _ in range(args.warmup):
        cpu_commit_rate(max(8, lg_rows - 2), args.polys, args.lg_blowup)
    times = []
    for s in range(args.steps):
        _, dt = cpu_commit_rate(lg_rows, args.polys, args.lg_blowup, seed=100 + s)
        times.append(dt)
    elems = args.polys << lg_rows
    value = elems * len(times) / sum(times) / 1e6
    cfg = workload_config(args.lg_size, args.polys, args.lg_blowup, args.gpus)
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(1e3 * sum(times) / len(times), 3), "higher_is_better": True,
        "scaling": "weak" if args.gpus == 1 else "strong", "vs_baseline": None, "dtype": "u64 (Goldilocks)",
        "data": "synthetic", "impl": "reference", "config": cfg,
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": host_threads(), "kind": "port", "label": CPU_LABEL,
                         "sample": f"{args.polys} polys x 2^{lg_rows} coeffs per step (bounded sample of the "
                                   f"workload), oracle/zkie_oracle.c on all host threads, {cpu_lanes()} SIMD "
                                   f"lanes per field op"},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---- clocks ------------------------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi samples (every 50 ms) of the ONE GPU this rank runs on,
    matched by UUID or PCI bus id; the median SM clock is taken over the
    samples inside the timed region in which that GPU was busy."""
    FIELDS = ("timestamp,uuid,pci.bus_id,utilization.gpu,clocks.sm,clocks.max.sm,power.draw,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
    PERIOD_MS = 50  # a split step at N = 8 takes about 10 ms: several samples even in a 0.1 s region

    def __init__(self, ident):
        self.uuid, self.bus = ident
        self.proc = None
        self.rows = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", str(self.PERIOD_MS)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True)
        except OSError:
            self.proc = None
            return
        self.th = threading.Thread(target=self._read, daemon=True)
        self.th.start()

    def _read(self):
        import datetime
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 11:
                try:
                    ts = datetime.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                except ValueError:
                    ts = time.time()
                self.rows.append([ts] + parts[1:])

    def window(self, t0, t1):
        self.t0, self.t1 = t0, t1

    def _mine(self, row):
        uuid, bus = row[1].lower(), row[2].upper()
        if self.uuid and uuid.endswith(self.uuid):
            return True
        return bool(self.bus) and bus.endswith(self.bus)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "gpu_match": "nvidia-smi unavailable"}
        time.sleep(0.3)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        mine = [r for r in self.rows if self._mine(r)]
        if not mine:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "gpu_match": "unmatched",
                    "gpu": {"uuid": self.uuid, "pci_bus_id": self.bus}}
        t0, t1 = getattr(self, "t0", 0.0), getattr(self, "t1", 1e30)
        inside = [r for r in mine if t0 - 0.1 <= r[0] <= t1 + 0.1]

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        busy = [r for r in inside if (num(r[3]) or 0) > 0]
        if not busy:  # a region shorter than the sampling period: the busy samples next to it
            busy = [r for r in mine if t0 - 1.0 <= r[0] <= t1 + 1.0 and (num(r[3]) or 0) > 0]
        use = busy or inside or mine
        sm = [v for v in (num(r[4]) for r in use) if v is not None]
        mx = [v for v in (num(r[5]) for r in use) if v is not None]
        reasons = sorted({self.REASONS[i] for r in use for i in range(4) if r[7 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples_in_timed_region": len(inside), "samples_busy": len(busy),
                "samples": len(use), "gpu_match": "uuid/pci", "gpu": {"uuid": self.uuid, "pci_bus_id": self.bus}}


# ---- GPU side -------------------------------------------------------------------------------------
def synth_device(n, seed, device):
    """Uniform canonical Goldilocks elements generated on the device."""
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    hi = torch.randint(0, 1 << 32, (n,), generator=g, device=device, dtype=torch.int64)
    lo = torch.randint(0, 1 << 32, (n,), generator=g, device=device, dtype=torch.int64)
    x = (hi << 32) | lo                       # bit pattern of a u64
    big = (x < 0) & (x >= -(1 << 32) + 1)     # u64 >= p  <=>  signed in [p - 2^64, 0)
    x = torch.where(big, x + ((1 << 32) - 1), x)  # x - p mod 2^64
    return x.view(torch.uint64)


def synth_into(out, seed):
    """synth_device into a preallocated uint64 tensor in chunks of 2^26
    elements, so that a 32 GiB input needs no 100 GiB of temporaries."""
    import torch
    n, chunk = out.numel(), 1 << 26
    v = out.view(torch.int64)
    for i, c0 in enumerate(range(0, n, chunk)):
        c1 = min(n, c0 + chunk)
        v[c0:c1].copy_(synth_device(c1 - c0, seed * 7919 + i, out.device).view(torch.int64))
    return out


def ntt_passes(lg):
    """Launches of k_ntt_pass per LDE (the plan in zkie_b200/csrc/ntt.cu)."""
    return 1 if lg <= 10 else (2 if lg <= 22 else 3)


def int_peaks(zk, dev):
    """Integer-pipe peak of this GPU, measured now: Goldilocks multiplications
    per second of independent register-resident chains (no memory traffic),
    and the Poseidon2 permutation rate without memory traffic (the ceiling of
    the hash code)."""
    import torch
    lib, check = zk.lib, zk.check
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream
    n_thr, iters = 148 * 16 * 128, 2048
    st = synth_device(n_thr * 16, 99, dev)
    check(lib.zkie2_gl_mul_probe(st.data_ptr(), n_thr, 16, sh), "mul probe warmup")
    pe0, pe1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    pe0.record(stream)
    check(lib.zkie2_gl_mul_probe(st.data_ptr(), n_thr, iters, sh), "mul probe")
    pe1.record(stream)
    torch.cuda.synchronize()
    mul_peak = n_thr * 8 * iters / (pe0.elapsed_time(pe1) / 1e3)
    check(lib.zkie2_p2_permute(st.data_ptr(), n_thr, 1, sh), "permute warmup")
    pe0.record(stream)
    check(lib.zkie2_p2_permute(st.data_ptr(), n_thr, 16, sh), "permute")
    pe1.record(stream)
    torch.cuda.synchronize()
    return mul_peak, n_thr * 16 / (pe0.elapsed_time(pe1) / 1e3)


def hbm_peak_gbs():
    peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(peaks_path):
        try:
            return float(json.load(open(peaks_path))["hbm_gbs"]), "MEASURED_PEAKS.json hbm_gbs (measured)"
        except Exception:
            pass
    return HBM_FALLBACK_GBS, "fallback 6.65 TB/s"


def gpu_ident(dev):
    """(uuid, PCI bus id) of this rank's GPU in nvidia-smi's forms: torch's
    pci_bus_id is the bus NUMBER, so the "DDDDDDDD:BB:DD.0" string is built
    from the domain, bus and device numbers."""
    import torch
    props = torch.cuda.get_device_properties(dev)
    uuid = str(getattr(props, "uuid", "") or "").lower()
    try:
        bus = "%08X:%02X:%02X.0" % (int(props.pci_domain_id), int(props.pci_bus_id), int(props.pci_device_id))
    except (AttributeError, TypeError, ValueError):
        bus = ""
    return uuid, bus


def gpu_local_cpus(dev):
    """(host CPUs close to the GPU, how they were found), or (None, why not):
    the NUMA node of the GPU's PCI function in sysfs, else NVML's CPU
    affinity of the device (a read-only query)."""
    import torch
    allowed = os.sched_getaffinity(0)
    try:
        props = torch.cuda.get_device_properties(dev)
        dom, bus, devn = int(props.pci_domain_id), int(props.pci_bus_id), int(props.pci_device_id)
    except (AttributeError, TypeError, ValueError):
        return None, "no PCI id"
    try:
        node = int(open("/sys/bus/pci/devices/%04x:%02x:%02x.0/numa_node" % (dom, bus, devn)).read().strip())
        if node >= 0:
            cpus = set()
            for part in open(f"/sys/devices/system/node/node{node}/cpulist").read().strip().split(","):
                lo, _, hi = part.partition("-")
                cpus.update(range(int(lo), int(hi or lo) + 1))
            if cpus & allowed:
                return cpus & allowed, f"sysfs NUMA node {node}"
    except (OSError, ValueError):
        pass
    try:
        import pynvml
        pynvml.nvmlInit()
        try:
            h = pynvml.nvmlDeviceGetHandleByPciBusId(("%08X:%02X:%02X.0" % (dom, bus, devn)).encode())
            words = (os.cpu_count() + 63) // 64
            masks = pynvml.nvmlDeviceGetCpuAffinity(h, words)
            cpus = {64 * i + b for i, m in enumerate(masks) for b in range(64) if (int(m) >> b) & 1}
            if cpus & allowed and cpus & allowed != allowed:
                return cpus & allowed, "NVML CPU affinity"
        finally:
            pynvml.nvmlShutdown()
    except Exception:  # NVML absent or the query unsupported on this box
        pass
    return None, "no NUMA locality reported (sysfs numa_node -1, NVML affinity = all CPUs)"


class NumaLocal:
    """Context manager: the calling thread runs on the CPUs of the GPU's own
    NUMA node while the end-to-end path allocates its pinned host buffers and
    copies, so those pages sit in that node's memory (first touch) and the
    PCIe transfers do not cross the socket interconnect; the previous CPU set
    comes back on exit (the CPU-baseline legs keep every host thread).  A
    host-thread setting only: nothing on the GPU changes."""

    def __init__(self, dev):
        self.local, self.how = gpu_local_cpus(dev)
        self.prev = None

    def __enter__(self):
        if self.local:
            self.prev = os.sched_getaffinity(0)
            os.sched_setaffinity(0, self.local)
        return self

    def __exit__(self, *exc):
        if self.prev:
            os.sched_setaffinity(0, self.prev)
        return False

    def describe(self):
        if self.local:
            return f"pinned buffers allocated on {len(self.local)} CPUs close to the GPU ({self.how})"
        return f"default placement: {self.how}"


def max_over_ranks(x, dev):
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(x)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main_split(args, zk, dev, world, rank):
    """N > 1: ONE commit of the workload split over the N ranks (strong
    scaling): rank g computes the LDE rows g, g + N, ... (coset LDE, no data
    exchange), hashes them, one all-to-all of 64-byte leaf digests gives each
    rank a contiguous leaf block, each rank builds its subtree, and an
    all-gather of the N subtree roots plus log2(N) compressions give the root
    (zkie_b200/multigpu.py)."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from zkie_b200.multigpu import SplitCommitter
    lib, check = zk.lib, zk.check
    lg_l, w, lg_b = args.lg_size, args.polys, args.lg_blowup
    L, H = 1 << lg_l, 1 << (lg_l + lg_b)
    n_in = L * w
    check(lib.zkie2_p2_init_default(), "init constants")
    d_in = synth_device(n_in, 1234, dev)  # the same coefficients on every rank (replicated input)
    sc = SplitCommitter(lg_l, lg_b, w)
    stream = torch.cuda.current_stream()
    for _ in range(args.warmup):
        sc.run(d_in)
    torch.cuda.synchronize()
    sampler = ClockSampler(gpu_ident(dev))
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(5)] for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist.barrier()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.5)
    host_t0 = time.time()
    t_start.record(stream)
    for s in range(args.steps):
        evs[s][0].record(stream)
        sc.run(d_in, evs[s][1:])
    t_end.record(stream)
    torch.cuda.synchronize()
    sampler.window(host_t0, time.time())
    clocks = sampler.stop()
    dist.barrier()
    ms_per_step = max_over_ranks(t_start.elapsed_time(t_end), dev) / args.steps
    phase = [sum(e[i].elapsed_time(e[i + 1]) for e in evs) / args.steps for i in range(4)]
    ntt_ms, leaf_ms, exch_ms, tree_ms = phase
    value = n_in / (ms_per_step / 1e3) / 1e6
    root = sc.root()
    # the split root must equal the single-device commit root of the same input
    if rank == 0:
        full = zk.commit(d_in.reshape(L, w), lg_b)
        root_ok = bool((np.asarray(full.root, dtype=np.uint64) == root).all())
        del full
    else:
        root_ok = None
    torch.cuda.empty_cache()

    mul_peak, perm_ceiling = int_peaks(zk, dev)
    perms_leaf = sc.n_local * ((w + 7) // 8)
    leaf_rate = perms_leaf / (leaf_ms / 1e3)
    hbm_peak, hbm_src = hbm_peak_gbs()
    ntt_bytes = 8 * w * (L + sc.n_local)
    ntt_gbs = ntt_bytes / (ntt_ms / 1e3) / 1e9

    # e2e through the C-ABI context (the headline host-buffer path), then the
    # torch-orchestrated one with per-phase times: each rank copies its 1/N
    # row slice of the pinned host input in, the full input is all-gathered
    # over NVLink, and each rank copies its LDE rows and subtree layers back
    ctx = mg_context(zk, rank, world)
    e2e, e2e_torch = None, None
    if not args.no_e2e:
        rows = L // world
        numa = NumaLocal(dev)
        e2e = e2e_mg(zk, dev, ctx, rank, world, lg_l, lg_b, w, d_in, root, numa, args.warmup, args.steps)
        with numa:
            h_part = torch.empty(rows * w, dtype=torch.uint64, pin_memory=True)
            h_part.view(torch.int64).copy_(d_in.view(torch.int64)[rank * rows * w:(rank + 1) * rows * w])
            h_lde = torch.empty(sc.n_local * w, dtype=torch.uint64, pin_memory=True)
            h_layers = torch.empty(sc.layers.numel(), dtype=torch.uint64, pin_memory=True)
            for _ in range(max(1, args.warmup)):
                sc.run_host(h_part, h_lde, h_layers)
            k_e2e = max(1, min(args.steps, 5))
            dist.barrier()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for _ in range(k_e2e):
                r = sc.run_host(h_part, h_lde, h_layers)
            e2e_s = max_over_ranks((time.perf_counter() - t0) / k_e2e, dev)
            assert (r == root).all(), "host-path root differs from the device-path root"
            phases = []
            sc.run_host(h_part, h_lde, h_layers, phases)   # one more call with phase events (not in the timing)
        ph = {k: round(max_over_ranks(v, dev), 3) for k, v in phases[0].items()}
        lde_b, lay_b, part_b = 8 * sc.n_local * w, 8 * sc.layers.numel(), 8 * rows * w
        e2e_torch = {"value": round(n_in / e2e_s / 1e6, 3), "unit": UNIT, "ms_per_step": round(1e3 * e2e_s, 3),
               "h2d_bytes_per_step": 8 * n_in, "d2h_bytes_per_step": 8 * H * w + 8 * world * sc.layers.numel(),
               "call": "SplitCommitter.run_host (per rank: pinned 1/N input slice in, NVLink all-gather, "
                       "split commit, LDE rows + subtree layers back to pinned host; not pipelined)",
               "host_memory": numa.describe(),
               "phases_ms_from_start_max_over_ranks": ph,
               "per_rank_gbs": {"upload": round(part_b / max(ph["upload"], 1e-3) / 1e6, 1),
                                "lde_download": round(lde_b / max(ph["lde_download"] - ph["lde_done"], 1e-3) / 1e6, 1),
                                "layers_download": round(lay_b / max(ph["layers_download"] - ph["commit"], 1e-3)
                                                         / 1e6, 1)}}
        del h_part, h_lde, h_layers

    lg_local = lg_l + lg_b - sc.lg_g
    launches = (1 + ntt_passes(lg_local)) + 1 + 1 + (lib.zkie2_merkle_num_layers(sc.n_local) - 1) + \
        (lib.zkie2_merkle_num_layers(world) - 1)
    n_local = sc.n_local
    del sc, d_in
    torch.cuda.empty_cache()

    # configuration 1 as replicas: every rank proves its own shard (shards
    # are independent until the cross-shard binding); max over ranks
    dist.barrier()
    shard = shard_prove_ms(zk, dev)
    shard.pop("inputs")
    shard_ms = max_over_ranks(shard["ms"], dev)
    shard_dev_ms = max_over_ranks(shard["device_ms"], dev)
    shard.update({"ms": round(shard_ms, 3), "device_ms": round(shard_dev_ms, 3), "replicas": world,
                  "value": round(world / (shard_ms / 1e3), 1), "unit": "shards/s (all GPUs)",
                  "parallelism": f"replicas: one independent shard per GPU, max over {world} ranks"})
    shard["roofline"] = shard_roofline(zk, dev, shard_dev_ms, perm_ceiling)
    big = big_commits(zk, dev, rank, world) if not args.no_big else {}
    split_sc = sumcheck_case(zk, dev, rank, world)
    mg = mg_case(zk, dev, ctx, rank, world, lg_l, lg_b, w, root)
    lib.zkie2_mg_destroy(ctx)
    cfg4 = cfg4_case(zk, dev, rank, world) if not args.no_cfg4 else None
    cfg = workload_config(lg_l, w, lg_b, world)
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 3), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "u64 (Goldilocks mod-p integer)", "data": "synthetic",
        "config": cfg,
        "roofline": {
            "bound": "int", "kernel": f"k_leaf_rows (Poseidon2 leaf sponge, {(w + 7) // 8} permutations per row, "
                                      f"{n_local} rows per rank)",
            "achieved": round(leaf_rate * MULS_PER_PERM / 1e9, 2), "peak": round(mul_peak / 1e9, 2),
            "unit": "G Goldilocks mul/s (per GPU)", "frac": round(leaf_rate * MULS_PER_PERM / mul_peak, 4),
            "traffic": None,
            "work_per_unit": f"{MULS_PER_PERM} field multiplications per Poseidon2-16 permutation",
            "peak_source": "measured live: zkie2_gl_mul_probe, independent register-resident multiply chains",
            "perm_rate_gperm_s": round(leaf_rate / 1e9, 4), "perm_ceiling_gperm_s": round(perm_ceiling / 1e9, 4),
            "ms_per_launch": round(leaf_ms, 4), "share_of_step": round(leaf_ms / ms_per_step, 4),
            "alu_pipe": alu_pipe_roofline(dev, leaf_rate, clocks),
        },
        "roofline_ntt": {
            "bound": "hbm", "kernel": f"k_coset_twist + k_ntt_pass2 x{ntt_passes(lg_local)} (coset LDE, "
                                      f"2^{lg_local} rows per rank)",
            "achieved": round(ntt_gbs, 1), "peak": hbm_peak, "unit": "GB/s (per GPU)",
            "frac": round(ntt_gbs / hbm_peak, 4), "traffic": None,
            "algorithmic_bytes": ntt_bytes, "peak_source": hbm_src,
            "ms_per_step": round(ntt_ms, 4), "share_of_step": round(ntt_ms / ms_per_step, 4),
        },
        "exchange_ms_per_step": round(exch_ms, 4),
        "exchange_bytes_per_rank": 64 * n_local * (world - 1) // world,
        "nodes_ms_per_step": round(tree_ms, 4),
        "gpu_launches": launches * args.steps,
        "clocks": clocks,
        "root_rank0": [hex(int(x)) for x in root[:2]],
        "root_matches_single_gpu_commit": root_ok,
    }
    if e2e:
        line["e2e"] = e2e
    if e2e_torch:
        line["e2e_torch_split"] = e2e_torch
    line["shard_prove"] = shard
    line.update(big)
    line["split_sumcheck"] = split_sc
    line["mg_c_abi"] = mg
    if cfg4:
        line["cfg4_gpt2_model"] = cfg4
    if rank == 0:
        print(json.dumps(line), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    return 0


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)

    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    dev = torch.device("cuda", torch.cuda.current_device())

    try:
        import zkie_b200 as zk
    except ImportError:
        import importlib.util
        spec = importlib.util.spec_from_file_location("_b", os.path.join(ROOT, "zkie_b200", "build.py"))
        b = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(b)
        b.build()
        import zkie_b200 as zk
    lib, check = zk.lib, zk.check
    if world > 1:
        return main_split(args, zk, dev, world, rank)

    lg_l, w, lg_b = args.lg_size, args.polys, args.lg_blowup
    L, H = 1 << lg_l, 1 << (lg_l + lg_b)
    lg = lg_l + lg_b
    n_in = L * w
    check(lib.zkie2_p2_init_default(), "init constants")
    d_in = synth_device(n_in, 1234, dev)
    d_lde = torch.empty(H * w, dtype=torch.uint64, device=dev)
    total_dig = lib.zkie2_merkle_total_digests(H)
    d_layers = torch.empty(total_dig * 8, dtype=torch.uint64, device=dev)
    d_scr = torch.empty(max(lib.zkie2_commit_scratch_elems(lg_l, lg_b, w), 1), dtype=torch.uint64, device=dev)
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream

    def step(evs=None):
        if evs:
            evs[0].record(stream)
        check(lib.zkie2_lde(d_in.data_ptr(), d_lde.data_ptr(), d_scr.data_ptr(), lg_l, lg_b, w, sh), "lde")
        if evs:
            evs[1].record(stream)
        check(lib.zkie2_merkle_leaves(d_lde.data_ptr(), H, w, d_layers.data_ptr(), sh), "leaves")
        if evs:
            evs[2].record(stream)
        check(lib.zkie2_merkle_tree_from_leaves(H, d_layers.data_ptr(), sh), "tree")
        if evs:
            evs[3].record(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    sampler = ClockSampler(gpu_ident(dev))

    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler.start()
    time.sleep(0.5)  # let nvidia-smi start sampling before the timed region
    host_t0 = time.time()
    t_start.record(stream)
    for s in range(args.steps):
        step(evs[s])
    t_end.record(stream)
    torch.cuda.synchronize()
    sampler.window(host_t0, time.time())
    clocks = sampler.stop()
    if world > 1:
        dist.barrier()
    elapsed_ms = t_start.elapsed_time(t_end)
    ntt_ms = sum(e[0].elapsed_time(e[1]) for e in evs) / args.steps
    leaf_ms = sum(e[1].elapsed_time(e[2]) for e in evs) / args.steps
    node_ms = sum(e[2].elapsed_time(e[3]) for e in evs) / args.steps
    if world > 1:
        t = torch.tensor([elapsed_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed_ms = float(t.item())
    ms_per_step = elapsed_ms / args.steps
    value = world * n_in / (ms_per_step / 1e3) / 1e6
    root = d_layers[-8:].cpu().numpy()

    mul_peak, perm_ceiling = int_peaks(zk, dev)
    perms_leaf = H * ((w + 7) // 8)
    leaf_rate = perms_leaf / (leaf_ms / 1e3)
    hbm_peak, hbm_src = hbm_peak_gbs()
    ntt_bytes = 8 * w * (L + H)
    ntt_gbs = ntt_bytes / (ntt_ms / 1e3) / 1e9

    # ---- e2e through the host-buffer C-ABI call ----
    e2e = None
    numa = NumaLocal(dev)
    if not args.no_e2e:
        with numa:
            h_in = torch.empty(n_in, dtype=torch.uint64, pin_memory=True)
            h_in.copy_(d_in)
            h_lde = torch.empty(H * w, dtype=torch.uint64, pin_memory=True)
            h_layers = torch.empty(total_dig * 8, dtype=torch.uint64, pin_memory=True)
            h_root = torch.empty(8, dtype=torch.uint64, pin_memory=True)
            for _ in range(max(1, args.warmup)):
                check(lib.zkie2_commit_host(h_in.data_ptr(), lg_l, lg_b, w, h_lde.data_ptr(), h_layers.data_ptr(),
                                            h_root.data_ptr()), "commit_host")
            k_e2e = max(1, min(args.steps, 5))
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for _ in range(k_e2e):
                check(lib.zkie2_commit_host(h_in.data_ptr(), lg_l, lg_b, w, h_lde.data_ptr(), h_layers.data_ptr(),
                                            h_root.data_ptr()), "commit_host")
            e2e_s = (time.perf_counter() - t0) / k_e2e
            if world > 1:
                t = torch.tensor([e2e_s], dtype=torch.float64, device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                e2e_s = float(t.item())
            assert (h_root.numpy() == root).all(), "host-path root differs from the device-path root"
            e2e = {"value": round(world * n_in / e2e_s / 1e6, 3), "unit": UNIT, "ms_per_step": round(1e3 * e2e_s, 3),
                   "h2d_bytes_per_step": 8 * n_in, "d2h_bytes_per_step": 8 * H * w + 64 * total_dig,
                   "call": "zkie2_commit_host (pinned input; LDE + every digest layer + root back to pinned host)",
                   "host_memory": numa.describe()}
            del h_in, h_lde, h_layers

    # ---- MatMul shard prove (inputs resident) ----
    shard = shard_prove_ms(zk, dev)
    sa, sw = shard.pop("inputs")
    shard["roofline"] = shard_roofline(zk, dev, shard["device_ms"], perm_ceiling)
    if not args.no_cpu:
        shard["cpu_baseline"] = shard_cpu_baseline(sa, sw)
    # ---- the next rows: logUp fraction tree and WHIR PoW grinding ----
    extra = next_rows(want_cpu=not args.no_cpu)
    extra["projection"] = projection_case(zk, dev, want_cpu=not args.no_cpu)
    extra["layer_shard"] = layer_case(zk, dev, want_cpu=not args.no_cpu)
    if not args.no_moe:
        extra["cfg5_moe_layer"] = moe_case(zk, dev, want_cpu=args.cpu_moe)
    if not args.no_cfg4:
        extra["cfg4_gpt2_model"] = cfg4_case(zk, dev, 0, 1)
    # ---- configurations 2 (256 x 2^24) and 5 (expert stack); the 2^28 sumcheck ----
    del d_in, d_lde, d_layers, d_scr
    torch.cuda.empty_cache()
    big = big_commits(zk, dev, rank, world) if not args.no_big else {}
    sumcheck = sumcheck_case(zk, dev, rank, world)

    launches_per_step = ntt_passes(lg) + 1 + (lib.zkie2_merkle_num_layers(H) - 1)
    traffic = measured_traffic(lg_l, w, lg_b, world)
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_per_step, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "u64 (Goldilocks mod-p integer)", "data": "synthetic",
        "config": workload_config(lg_l, w, lg_b, world),
        "roofline": {
            "bound": "int", "kernel": f"k_leaf_rows (Poseidon2 leaf sponge, {(w + 7) // 8} permutations per row)",
            "achieved": round(leaf_rate * MULS_PER_PERM / 1e9, 2), "peak": round(mul_peak / 1e9, 2),
            "unit": "G Goldilocks mul/s", "frac": round(leaf_rate * MULS_PER_PERM / mul_peak, 4),
            "traffic": traffic["leaf"], "traffic_unit": "DRAM bytes per launch", "traffic_source": traffic["src"],
            "work_per_unit": f"{MULS_PER_PERM} field multiplications per Poseidon2-16 permutation "
                             "(8x16 + 22 S-boxes x^7 at 4 each, 22 diagonal products)",
            "peak_source": "measured live: zkie2_gl_mul_probe, independent register-resident multiply chains",
            "perm_rate_gperm_s": round(leaf_rate / 1e9, 4),
            "perm_ceiling_gperm_s": round(perm_ceiling / 1e9, 4),
            "ms_per_launch": round(leaf_ms, 4), "share_of_step": round(leaf_ms / ms_per_step, 4),
            "alu_pipe": alu_pipe_roofline(dev, leaf_rate, clocks),
        },
        "roofline_ntt": {
            "bound": "hbm", "kernel": f"k_ntt_pass2 x{ntt_passes(lg)} (register-radix passes, LDE 2^{lg_l} -> 2^{lg})",
            "achieved": round(ntt_gbs, 1), "peak": hbm_peak, "unit": "GB/s", "frac": round(ntt_gbs / hbm_peak, 4),
            "traffic": traffic["ntt"], "traffic_unit": "DRAM bytes per LDE (both passes)",
            "algorithmic_bytes": ntt_bytes, "peak_source": hbm_src,
            "ms_per_step": round(ntt_ms, 4), "share_of_step": round(ntt_ms / ms_per_step, 4),
        },
        "nodes_ms_per_step": round(node_ms, 4),
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
        "root_rank0": [hex(int(x)) for x in root[:2]],
    }
    if e2e:
        line["e2e"] = e2e
    if shard:
        line["shard_prove"] = shard
    if extra:
        line.update(extra)
    line.update(big)
    line["sumcheck_2^28"] = sumcheck
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(w, lg_b)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def measured_traffic(lg_l, w, lg_b, world):
    """dram__bytes_read.sum + dram__bytes_write.sum of the dominant launches,
    from one single-pass ncu capture of this exact workload; null for other
    workloads."""
    if (lg_l, w, lg_b, world) == (20, 256, 1, 1):
        return {"leaf": 4310624256 + 131658752, "ntt": 2149098240 + 4298085632 + 4295429120 + 4260205056,
                "src": "dram__bytes_read.sum + dram__bytes_write.sum from one single-pass ncu capture of this "
                       "workload (a constant of that capture, not measured in this run)"}
    return {"leaf": None, "ntt": None, "src": None}


def next_rows(want_cpu, lg_frac=22, grind_bits=24):
    """The logUp fraction tree (prove_fractional_with_challenges, 2^22
    fractions, inputs resident) and PoW grinding (24 bits) on the device, each
    with the CPU oracle port timed beside it on a bounded sample (a
    2^18-fraction tree on every host thread; a 16-bit grind on one)."""
    import types

    from perfcases import case_fixed, case_grind, case_logup
    lg = case_logup(types.SimpleNamespace(log_size=lg_frac, iters=5))
    gr = case_grind(types.SimpleNamespace(log_size=grind_bits, iters=3))
    fm = case_fixed(types.SimpleNamespace(m=512, k=1024, n=4096, iters=5))
    out = {
        "logup": {"config": f"prove_fractional_with_challenges over 2^{lg_frac} fractions (every layer on the device)",
                  "ms": round(lg["ms"], 4), "value": round((1 << lg_frac) / (lg["ms"] / 1e3) / 1e6, 3),
                  "unit": "Mfractions/s", "lookup_columns_ms": round(lg["lookup_columns_ms"], 4)},
        "grind": {"config": f"WHIR PoW grind, {grind_bits} bits, DuplexChallenger<Goldilocks, Poseidon2-16, 16, 8>",
                  "ms": round(gr["ms"], 4), "witness": gr["witness"], "value": round(gr["gperm_s_tried"] * 1e3, 3),
                  "unit": "M candidates/s"},
        "forward_matmul": {"config": "par::mm_par_fixed, 512 x 1024 @ 1024 x 4096 (a GPT-2 layer's FFN shape), "
                                     "16-bit fixed-point entries, u8 x u8 -> s32 tcgen05 GEMMs",
                           "ms": round(fm["ms"], 4), "path": "tensor cores" if fm["path"] == 0 else "field kernel",
                           "field_kernel_ms": round(fm["field_kernel_ms"], 4), "equal_to_field_kernel": fm["equal"],
                           "value": round(512 * 1024 * 4096 / (fm["ms"] / 1e3) / 1e9, 3), "unit": "G MAC/s"},
    }
    if want_cpu:
        import numpy as np

        from oracle import oracle as orc
        g = np.random.default_rng(1)
        n = 1 << 18
        num, den = g.integers(0, P, size=n, dtype=np.uint64), g.integers(1, P, size=n, dtype=np.uint64)
        orc.set_threads(host_threads())
        t0 = time.perf_counter()
        orc.fractional_prove(num, den, list(range(3, 21)), list(range(5, 23)))
        s_frac = time.perf_counter() - t0
        out["logup"]["cpu_baseline"] = {"value": round(n / s_frac / 1e6, 4), "unit": "Mfractions/s",
                                        "cores": host_threads(),
                                        "kind": "port", "label": CPU_LABEL, "sample": "2^18-fraction tree, oracle/zkie_oracle.c"}
        consts = orc.p2_constants(1)
        sponge = [(0x9E3779B97F4A7C15 * (i + 1)) % P for i in range(16)]
        t0 = time.perf_counter()
        w = orc.grind(consts, sponge, [5, 6, 7], 16)
        s_grind = time.perf_counter() - t0
        out["grind"]["cpu_baseline"] = {"value": round((w + 1) / s_grind / 1e6, 4), "unit": "M candidates/s",
                                        "cores": 1, "kind": "port", "label": CPU_LABEL,
                                        "sample": f"16-bit grind from the same state ({w + 1} candidates)"}
        a = g.integers(-(1 << 15), 1 << 15, size=(16, 1024), dtype=np.int64)
        b = g.integers(-(1 << 15), 1 << 15, size=(1024, 4096), dtype=np.int64)
        fa = a.astype(np.uint64) + np.where(a < 0, np.uint64(P), np.uint64(0))
        fb = b.astype(np.uint64) + np.where(b < 0, np.uint64(P), np.uint64(0))
        orc.set_threads(host_threads())
        t0 = time.perf_counter()
        orc.matmul_field(fa, fb)
        s_mm = time.perf_counter() - t0
        out["forward_matmul"]["cpu_baseline"] = {"value": round(16 * 1024 * 4096 / s_mm / 1e9, 4), "unit": "G MAC/s",
                                                 "cores": host_threads(), "kind": "port", "label": CPU_LABEL,
                                                 "sample": "16 x 1024 @ 1024 x 4096, oracle field matmul (OpenMP)"}
    return out


def shard_prove_ms(zk, dev, iters=5):
    """A 16x768 and W 768x768 (entries uniform in [-2^15, 2^15),
    zero-padded to 16x1024 / 1024x1024), forward C = A @ W, WHIR commits of W
    (n = 20) and of the shard boundary A, C (n = 14), and the MatMul GKR proof
    with challenges from the shard-DAG child transcript."""
    import numpy as np
    import torch

    from zkie_b200.device import to_dev
    m, k, n = 16, 1024, 1024
    g = np.random.default_rng(5)

    def fx(shape):
        # signed fixed-point embedding x < 0 -> p - |x| (common/fixed_point.rs:53-59)
        x = g.integers(-(1 << 15), 1 << 15, size=shape, dtype=np.int64)
        return x.astype(np.uint64) + np.where(x < 0, np.uint64(P), np.uint64(0))

    a = np.zeros((m, k), dtype=np.uint64)
    wt = np.zeros((k, n), dtype=np.uint64)
    a[:, :768] = fx((m, 768))
    wt[:768, :768] = fx((768, 768))
    d_a, d_w = to_dev(a), to_dev(wt)
    prover = zk.ShardProver(m, k, n)
    times, dev_times = [], []
    stream = torch.cuda.current_stream()
    for it in range(iters + 2):
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        e0.record(stream)
        res = prover.prove(d_a, d_w, op_ids=(0, 1, 2), ops_per_shard=1, shard_index=0)
        e1.record(stream)
        torch.cuda.synchronize()
        if it >= 2:
            times.append(time.perf_counter() - t0)
            dev_times.append(e0.elapsed_time(e1))
    return {"config": "cfg1: MatMul 16x1024x1024 (768 real) shard: forward + WHIR commits W(n=20), A, C(n=14) "
                      "+ 10-round GKR sumcheck, one zkie2_shard_prove_matmul call (four streams)",
            "ms": round(1e3 * statistics.median(times), 3),
            "device_ms": round(statistics.median(dev_times), 3),
            "claimed": hex(res.proof.proof.claimed), "root_w": hex(int(res.roots[0][0])),
            "inputs": (a, wt)}


def projection_case(zk, dev, want_cpu, m=512, k=1024, n=4096, shift=16, iters=5):
    """The projection block (crates/zkie-ops/src/projection.rs prove_projection)
    at a GPT-2 layer's FFN up-projection shape, 16-bit fixed-point x and W
    (scale 2^16), bias within 2^20: the whole prove (forward h = x W on the
    tensor cores, MatMul GKR, affine virtual sumcheck, logUp range check into
    the 2^16 table) with inputs resident; the proof alone (h given) beside it."""
    import numpy as np
    import torch

    from zkie_b200.projection import projection_witness, prove_projection
    g = np.random.default_rng(11)

    def fx(size, lim):
        x = g.integers(-lim, lim, size=size, dtype=np.int64)
        return torch.from_numpy(x.astype(np.uint64) + np.where(x < 0, np.uint64(P), np.uint64(0))).to(dev)
    x, w, b = fx(m * k, 1 << 15), fx(k * n, 1 << 15), fx(m * n, 1 << 20)
    h, path = zk.matmul_fixed(x, w, m, k, n)
    out, rem, idx = projection_witness(h, b, shift)
    whole, proof_only = [], []
    for it in range(iters + 2):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        prove_projection(x, w, b, out, rem, m, k, n, shift, zk.XorShift64(3))
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        p = prove_projection(x, w, b, out, rem, m, k, n, shift, zk.XorShift64(3), h=h)
        torch.cuda.synchronize()
        t2 = time.perf_counter()
        if it >= 2:
            whole.append(t1 - t0)
            proof_only.append(t2 - t1)
    ms, ms_p = 1e3 * statistics.median(whole), 1e3 * statistics.median(proof_only)
    lg = (m * n + (1 << shift) - 1).bit_length()
    # bytes the proof reads at least once: x, W, h (GKR); rem, h, out, bias
    # (affine; eq and ones are generated); the lookup columns num / den of
    # 2^lg fractions written and read once
    proof_bytes = 8 * (m * k + k * n + m * n) + 8 * 4 * m * n + 2 * 16 * (1 << lg)
    hbm_peak, hbm_src = hbm_peak_gbs()
    out_d = {"config": f"prove_projection, x {m}x{k} @ W {k}x{n} (a GPT-2 layer's FFN up-projection), shift {shift}, "
                       "16-bit fixed-point inputs, inputs resident",
             "ms": round(ms, 3), "proof_only_ms": round(ms_p, 3), "forward_path": "tensor cores" if path == 0 else
             "field kernel", "value": round(m * n / (ms / 1e3) / 1e6, 3), "unit": "M outputs/s",
             "claimed": hex(p.matmul.claimed), "lookup_fractions": 1 << lg,
             "roofline": {"bound": "hbm", "achieved": round(proof_bytes / (ms_p / 1e3) / 1e9, 1), "peak": hbm_peak,
                          "unit": "GB/s", "frac": round(proof_bytes / (ms_p / 1e3) / 1e9 / hbm_peak, 4),
                          "algorithmic_bytes": proof_bytes, "peak_source": hbm_src,
                          "note": "proof part (h given); the logUp tree's ~2 lg serial rounds per layer make it "
                                  "latency-bound, see logup"}}
    if want_cpu:
        from oracle import oracle as orc
        orc.set_threads(host_threads())
        xs, ws, bs, os_, rs = (t.cpu().numpy() for t in (x, w, b, out, rem))
        t0 = time.perf_counter()
        orc.projection_prove(xs, ws, bs, os_, rs, m, k, n, shift, orc.XorShift64(3))
        dt = time.perf_counter() - t0
        out_d["cpu_baseline"] = {"value": round(1e3 * dt, 1), "unit": "ms per projection", "cores": host_threads(),
                                 "kind": "port", "label": CPU_LABEL,
                                 "sample": "the same projection once by oracle/zkie_oracle.c (fixed-point matmul, "
                                           "sumcheck rounds and fraction layers on every host thread)"}
    del x, w, b, h, out, rem, idx
    torch.cuda.empty_cache()
    return out_d


def layer_case(zk, dev, want_cpu, iters=5):
    """Configuration 3: one GPT-2-small layer (models/gpt2 build_layer: 176 ops,
    m 512, D 1024 with 768 real, 12 heads x 64, FFN 4096 with 3072 real; the
    exp 2^21, rsqrt 7.3 M and gelu 2^24 tables) proven as one shard of
    prove_shard_dag: the forward witness, then the shard proof (every arm,
    53 same_poly bindings, the three tables' logUp)."""
    from zkie_b200 import gpt2
    return shard_case(zk, lambda st: gpt2.gpt2_layer(st, gpt2.GPT2_SMALL),
                      "GPT-2-small layer shard (models/gpt2/src/lib.rs build_layer, 176 ops: m 512, D 1024 (768 real), "
                      "12 heads x 64, FFN 4096 (3072 real), shift 16; synthetic weights in the random builder's ranges; "
                      "exp 2^21 / rsqrt 7.3M / gelu 2^24 tables), one shard of prove_shard_dag, inputs resident",
                      want_cpu, iters)


def moe_case(zk, dev, want_cpu, iters=3):
    """Configuration 5: one DeepSeek-V2-Lite-shaped MoE layer
    (models/deepseek-v2-lite build_attention + build_moe, zkie_b200.deepseek:
    hidden 2048, MLA with 16 heads, kv_lora 512, 64 routed experts top-6 with
    the expert FFN 2048 (1408 real), the shared experts 4096 (2816 real),
    sequence 512) proven as one shard.  The CPU restatement of this layer
    takes minutes, so it runs only on request (--cpu-moe)."""
    from zkie_b200 import deepseek
    return shard_case(zk, lambda st: deepseek.moe_layer(st, deepseek.DSV2_LITE),
                      "DeepSeek-V2-Lite-shaped MoE layer shard (models/deepseek-v2-lite/src/lib.rs build_attention + "
                      "build_moe as one layer: hidden 2048, MLA 16 heads (nope 128, rope 64, v 128, kv_lora 512), "
                      "64 routed experts top-6 (FFN 2048, 1408 real) expert-major via Scatter / GatherMatMul / Gather, "
                      "shared experts 4096 (2816 real), m 512, shift 16; synthetic weights; exp 2^21 / rsqrt 7.3M / "
                      "SiLU 2^24 / limb 2^16 tables), one shard, inputs resident",
                      want_cpu, iters)


def shard_case(zk, build, config, want_cpu, iters):
    """One op-graph shard on one GPU: the forward witness, then the shard
    proof, recorded once as a CUDA graph (its challenges and launch shapes
    depend on the statement only) and replayed; the eager proof (host
    orchestration of every launch) is reported beside it, with its digest."""
    import torch

    from zkie_b200 import compose as C
    from zkie_b200.dag import digest as _proof_digest
    st = C.Store()
    t0 = time.perf_counter()
    ops, x, out = build(st)
    build_s = time.perf_counter() - t0
    # the forward recorded as a CUDA graph where the graph allows it (no
    # routing read back to the host), else eager
    t0 = time.perf_counter()
    gf = None if any(op.kind in ("Scatter", "GatherMatMul") for op in ops) else C.GraphForward(st, ops)
    fwd_capture_s = time.perf_counter() - t0
    forward = gf.run if gf is not None else (lambda: C.forward_ops(st, ops))
    fwd = []
    for it in range(iters + 2):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        forward()
        torch.cuda.synchronize()
        if it >= 2:
            fwd.append(time.perf_counter() - t0)
    master = C.master_transcript(ops, len(ops))

    def make_rng():
        c = master.clone()
        c.absorb_u64(0)
        return c
    eager = []
    for it in range(3):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        p_eager = C.prove_shard_precomputed(st, ops, [], make_rng())
        torch.cuda.synchronize()
        if it >= 1:
            eager.append(time.perf_counter() - t0)
    t0 = time.perf_counter()
    gp = C.GraphShardProver(st, ops, [], make_rng)
    capture_s = time.perf_counter() - t0
    stream = torch.cuda.current_stream()
    replay, collect, whole = [], [], []
    for it in range(iters + 1):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        forward()
        e0.record(stream)
        gp.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        t1 = time.perf_counter()
        proof = gp.prover.collect()
        t2 = time.perf_counter()
        if it >= 1:
            replay.append(e0.elapsed_time(e1))
            collect.append(t2 - t1)
            whole.append(t2 - t0)
    digest = _proof_digest(proof.canonical())
    eager_digest = _proof_digest(p_eager.canonical())
    sh = proof
    traffic = gp.prover.traffic
    prove_ms = statistics.median(replay)
    hbm_peak, hbm_src = hbm_peak_gbs()
    out_d = {
        "config": config,
        "ms": round(1e3 * statistics.median(whole), 3), "unit": "ms per layer shard (forward + prove + proof to host)",
        "forward_ms": round(1e3 * statistics.median(fwd), 3),
        "forward": ("CUDA graph (GraphForward, recorded in %.0f ms)" % (1e3 * fwd_capture_s)) if gf is not None
                   else "eager (routing read back to the host)",
        "prove_ms": round(prove_ms, 3),
        "collect_ms": round(1e3 * statistics.median(collect), 3),
        "eager_prove_ms": round(1e3 * statistics.median(eager), 3), "capture_ms": round(1e3 * capture_s, 1),
        "build_s": round(build_s, 2), "ops": len(ops), "same_poly_binds": len(sh.binds), "claims": len(sh.claims),
        "lookup_tables": len(sh.table_columns), "proof_digest": digest, "replay_equals_eager": digest == eager_digest,
        "roofline": {"bound": "hbm", "achieved": round(traffic / (prove_ms / 1e3) / 1e9, 1), "peak": hbm_peak,
                     "unit": "GB/s", "frac": round(traffic / (prove_ms / 1e3) / 1e9 / hbm_peak, 4),
                     "algorithmic_bytes": int(traffic), "peak_source": hbm_src,
                     "note": "every table each sub-proof reads, once, over the graph replay's device time; "
                             "the sumchecks' serial rounds (thousands of short dependent launches over 8 streams) "
                             "keep it latency-bound"},
    }
    if want_cpu:
        from oracle import compose_oracle as co
        from oracle import oracle as orc
        orc.set_threads(host_threads())
        host = co.HostStore()
        build(host)
        t0 = time.perf_counter()
        co.forward_ops(host, ops)
        t1 = time.perf_counter()
        om = co.master_transcript(ops, len(ops))
        child = orc.OracleTranscript(raw=om.t)
        child.absorb_u64(0)
        cpu_proof = co.prove_shard_precomputed(host, ops, [], child)
        t2 = time.perf_counter()
        out_d["cpu_baseline"] = {"value": round(1e3 * (t2 - t0), 1), "unit": "ms per layer shard",
                                 "cores": host_threads(), "kind": "port", "label": CPU_LABEL,
                                 "forward_ms": round(1e3 * (t1 - t0), 1), "prove_ms": round(1e3 * (t2 - t1), 1),
                                 "proof_digest": _proof_digest(cpu_proof),
                                 "sample": "the same layer shard once (forward + prove) by oracle/compose_oracle.py "
                                           "over oracle/zkie_oracle.c (OpenMP loops on every host thread)"}
        out_d["proof_matches_cpu"] = out_d["cpu_baseline"]["proof_digest"] == digest
    del st, gp
    torch.cuda.empty_cache()
    return out_d


def cfg4_case(zk, dev, rank, world, layers=12):
    """Configuration 4: the GPT-2-small graph of build_gpt2 (models/gpt2/src/
    lib.rs:321-436: the embedding lookup into the tied 1024 x 65536 table,
    12 layers, the final LayerNorm, the lm_head matmul, the vocabulary mask,
    the Argmax) proven as a shard DAG of 176-op shards (13 shards, as the reference's
    GPT-2 512 proof; compose.rs prove_shard_dag :2289-2346): rank r proves
    the shards si % world == r, each recorded once as a CUDA graph and
    replayed; rank 0 gathers the claims, binds the tensors claimed by two
    shards with the master transcript and commits each of them as
    prove_committed_shard_dag does (Whir::with_params(arity, 90, 17)).  Every
    rank holds the whole witness (the forward pass of the whole graph).  Not
    built: the WHIR openings of the committed path."""
    import torch
    import torch.distributed as dist

    from zkie_b200 import compose as C
    from zkie_b200 import dag, gpt2
    t0 = time.perf_counter()
    st = C.Store()
    ops, _, _ = gpt2.gpt2_model(st, gpt2.GPT2_SMALL, layers)
    build_s = time.perf_counter() - t0
    gf = C.GraphForward(st, ops)  # the whole graph's forward, recorded once
    fwd = []
    for _ in range(3):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        gf.run()
        torch.cuda.synchronize()
        fwd.append(time.perf_counter() - t0)
    per = 176
    gather = dag.torch_gather() if world > 1 else None
    # timed passes gather only the claims; the digests come from one more
    # replay afterwards (they download every shard's lookup columns)
    provers = dag.device_provers(summary="none", graph=True)
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    dag.prove_dag_ranks(st, ops, per, provers, rank, world, gather)
    torch.cuda.synchronize()
    record_s = time.perf_counter() - t0
    times = []
    for _ in range(3):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        res = dag.prove_dag_ranks(st, ops, per, provers, rank, world, gather)
        torch.cuda.synchronize()
        times.append(time.perf_counter() - t0)
    ms = 1e3 * statistics.median(times)
    fwd_ms = 1e3 * fwd[-1]
    if world > 1:
        ms = max_over_ranks(ms, dev)
        fwd_ms = max_over_ranks(fwd_ms, dev)
    if world > 1:
        dist.barrier()
    res = dag.prove_dag_ranks(st, ops, per, dag.device_provers(summary="digest", graph=True, graphs=provers.graphs),
                              rank, world, gather)
    out_d = None
    if rank == 0:
        check = dag.prove_dag_ranks(st, ops, per, dag.device_provers(summary="digest", graph=False))
        out_d = {
            "config": f"cfg4: GPT-2-small graph of models/gpt2 build_gpt2 ({len(ops)} ops: embedding lookup into "
                      f"the tied 1024 x 65536 table, {layers} layers (m 512, D 1024, FFN 4096, 12 heads), final "
                      f"LayerNorm, lm_head, vocabulary mask, Argmax over the 65536 logits of every position; "
                      f"synthetic weights and tokens), ops_per_shard {per}, shards round-robin over {world} GPU(s)",
            "ms": round(ms, 3), "unit": "ms per DAG proof (every shard + cross-shard bindings), max over ranks",
            "layers_per_s": round(layers / (ms / 1e3), 2), "forward_ms": round(fwd_ms, 3), "ops": len(ops),
            "record_ms": round(1e3 * record_s, 1), "build_s": round(build_s, 2),
            "shards": len(res.shards), "max_shards_per_gpu": -(-len(res.shards) // world),
            "cross_tensors": len(res.cross_tensors),
            "boundary_commits": f"{len(res.boundary_roots)} WHIR base commits of the cross-shard tensors "
                                "(prove_committed_shard_dag's boundary commitments; their openings are not built)",
            "digest": res.digest,
            "digest_matches_eager_one_gpu": res.digest == check.digest,
        }
    del st, provers
    torch.cuda.empty_cache()
    return out_d


def shard_roofline(zk, dev, device_ms, perm_ceiling):
    """Floor of the configuration-1 shard: the larger of (a) its dependency
    chain, W's 4 leaf absorptions (32 columns, rate 8) then 16 tree levels, one
    permutation each, at the measured latency of one permutation (one thread
    per permutation where a launch has more than 2^14 states, four lanes per
    permutation below), and (b) its permutation count at the measured
    permutation throughput (the NTT, matmul and GKR bytes add < 10 us at HBM
    speed).  Kernel-launch gaps between the dependent steps are not in the
    floor."""
    import torch
    lib = zk.lib
    st = synth_device(16, 77, dev)
    reps = 4096
    zk.check(lib.zkie2_p2_permute(st.data_ptr(), 1, 16, 0), "permute warmup")
    s = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    zk.check(lib.zkie2_p2_permute(st.data_ptr(), 1, reps, s.cuda_stream), "permute latency")
    e1.record(s)
    torch.cuda.synchronize()
    lat_us = 1e3 * e0.elapsed_time(e1) / reps
    # launches of at most 2^14 states run each permutation on four lanes: the
    # latency of that form from one row of 8 * 256 columns (256 dependent
    # absorptions in one four-lane group)
    absorb = 256
    row = synth_device(8 * absorb, 78, dev)
    dig = torch.empty(8, dtype=torch.uint64, device=dev)
    zk.check(lib.zkie2_merkle_leaves(row.data_ptr(), 1, 8 * absorb, dig.data_ptr(), s.cuda_stream), "warmup")
    e0.record(s)
    zk.check(lib.zkie2_merkle_leaves(row.data_ptr(), 1, 8 * absorb, dig.data_ptr(), s.cuda_stream), "x4 latency")
    e1.record(s)
    torch.cuda.synchronize()
    lat4_us = 1e3 * e0.elapsed_time(e1) / absorb
    perms = 0
    for n in (20, 14, 14):  # W, A, C
        H = 1 << (n - 4)
        perms += H * 4 + (lib.zkie2_merkle_total_digests(H) - H)
    # W's chain: 4 absorptions of 2^16 rows and the 2^15-node level (one lane
    # per permutation), then 15 levels of at most 2^14 nodes (four lanes)
    chain = 4 + 16
    chain_ms = ((4 + 1) * lat_us + 15 * lat4_us) / 1e3
    thr_ms = perms / perm_ceiling * 1e3
    floor = max(chain_ms, thr_ms)
    return {"bound": "latency" if chain_ms >= thr_ms else "int", "achieved_ms": device_ms, "floor_ms": round(floor, 4),
            "frac": round(floor / device_ms, 4), "unit": "ms",
            "chain_floor_ms": round(chain_ms, 4), "chain_permutations": chain,
            "permutation_latency_us": round(lat_us, 3), "permutation_latency_x4_us": round(lat4_us, 3),
            "throughput_floor_ms": round(thr_ms, 4), "permutations": perms,
            "perm_rate_gperm_s": round(perm_ceiling / 1e9, 4)}


def shard_cpu_baseline(a, wt, m=16, k=1024, n=1024):
    """The configuration-1 shard on the host cores: forward C = A W (field
    matmul, OpenMP), the three WHIR commits (LDE + Merkle, OpenMP) and the
    Op::MatMul proof with the shard's child transcript (single thread)."""
    from oracle import oracle as orc
    orc.set_threads(host_threads())
    consts = orc.p2_constants(1)
    t0 = time.perf_counter()
    c = orc.matmul_field(a, wt)
    for t in (wt, a, c):
        orc.whir_commit(consts, t.reshape(-1))
    orc.op_matmul_prove(a, wt, c, m, k, n, orc.shard_dag_child([[0, 1, 2]], 1, 0))
    dt = time.perf_counter() - t0
    return {"value": round(1e3 * dt, 3), "unit": "ms per shard", "cores": host_threads(), "kind": "port",
            "label": CPU_LABEL, "sample": "the whole configuration-1 shard (forward, three WHIR commits, MatMul GKR) "
                                          "by oracle/zkie_oracle.c, once"}


# ---- the commits larger than one GPU's plain commit, and the split sumcheck --------------
EXTRA_WARMUP, EXTRA_STEPS = 1, 2
BIG_CASES = [
    # name, lg_l, lg_blowup, w, description
    ("cfg5_expert_stack", 23, 1, 32,
     "cfg5: DeepSeek-V2-Lite routed-expert stack, N_ROUTED x H x MOE_PAD = 64 x 2048 x 2048 = 2^28 evaluations, "
     "one WHIR base commit (group size 1: arity 28 > 26): 2^23 x 32 at blowup 2"),
    ("cfg2_256x2^24_b2", 24, 1, 256, "cfg2: 256 polys x 2^24 coeffs, blowup 2 (LDE 64 GiB)"),
    ("cfg2_256x2^24_b4", 24, 2, 256, "cfg2: 256 polys x 2^24 coeffs, blowup 4 (LDE 128 GiB)"),
]


def _timed(fn, stream, dev, world):
    """EXTRA_WARMUP untimed calls, then EXTRA_STEPS calls between CUDA events on
    the launching stream; ms per call, max over ranks."""
    import torch
    import torch.distributed as dist
    for _ in range(EXTRA_WARMUP):
        fn()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(EXTRA_STEPS):
        fn()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / EXTRA_STEPS
    return max_over_ranks(ms, dev) if world > 1 else ms


def _hex_root(root):
    return [hex(int(x)) for x in root[:2]]


def big_commits(zk, dev, rank, world):
    """BASELINE configurations 2 (256 x 2^24, blowup 2 and 4) and 5 (the
    routed-expert stack).  N = 1: the expert stack through the plain WHIR
    commit (LDE kept), the 2^24 cases through zkie2_commit_cosets (LDE one
    coset of rows at a time; 164 / 296 GiB would not fit otherwise).  N > 1:
    every case as one commit split over the ranks (SplitCommitter), blowup 4 at
    N >= 4 (at N = 2 a rank would hold 32 GiB of input plus 2 x 64 GiB).  Each
    root is checked on rank 0 against a single-GPU commit of the same input
    taken by another path: the plain commit for the expert stack, the coset
    commit with a different coset count for the 2^24 cases."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from zkie_b200.device import empty
    from zkie_b200.multigpu import SplitCommitter
    lib, check = zk.lib, zk.check
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream
    lg_g = world.bit_length() - 1
    out = {}
    for idx, (name, lg_l, lg_b, w, desc) in enumerate(BIG_CASES):
        if world == 2 and lg_b == 2:
            continue
        L, H = 1 << lg_l, 1 << (lg_l + lg_b)
        torch.cuda.empty_cache()
        d_in = synth_into(torch.empty(L * w, dtype=torch.uint64, device=dev), 4242 + idx)
        total = lib.zkie2_merkle_total_digests(H)
        if world > 1:
            sc = SplitCommitter(lg_l, lg_b, w)
            ms = _timed(lambda: sc.run(d_in), stream, dev, world)
            root = sc.root()
            path = (f"split over {world} GPUs (coset LDE rows per rank, NCCL all-to-all of leaf digests, "
                    "all-gather of subtree roots)")
            del sc
        elif name.startswith("cfg5"):
            lde, layers = empty(H * w), empty(total * 8)
            scr = empty(max(lib.zkie2_whir_scratch_elems(lg_l + 5), 1))
            ms = _timed(lambda: check(lib.zkie2_whir_commit(d_in.data_ptr(), lg_l + 5, lde.data_ptr(),
                                                            layers.data_ptr(), scr.data_ptr(), sh), "whir_commit"),
                        stream, dev, world)
            root = layers[-8:].cpu().numpy()
            path = "zkie2_whir_commit on one GPU (LDE kept resident)"
            del lde, layers, scr
        else:
            lg_c = 2 if lg_b == 1 else 3
            layers = empty(total * 8)
            scr = empty(lib.zkie2_commit_cosets_scratch_elems(lg_l, lg_b, w, lg_c))
            ms = _timed(lambda: check(lib.zkie2_commit_cosets(d_in.data_ptr(), lg_l, lg_b, w, lg_c, layers.data_ptr(),
                                                              scr.data_ptr(), sh), "commit_cosets"),
                        stream, dev, world)
            root = layers[-8:].cpu().numpy()
            path = f"zkie2_commit_cosets on one GPU ({1 << lg_c} cosets of LDE rows, LDE not kept)"
            del layers, scr
        torch.cuda.empty_cache()
        root_ok, check_path = None, None
        if rank == 0:
            if name.startswith("cfg5") and world > 1:
                ref = zk.Whir.with_params(lg_l + 5, 90, 17).commit(d_in)
                exp, check_path = np.asarray(ref.root, dtype=np.uint64), "zkie2_whir_commit on one GPU"
                del ref
            else:
                lg_c = (lg_g + 1) if world > 1 else (2 if lg_b == 1 else 3) + 1
                exp, layers = zk.commit_cosets(d_in, lg_b, lg_c, w=w)
                check_path = f"zkie2_commit_cosets on one GPU with {1 << lg_c} cosets"
                del layers
            root_ok = bool((exp == root).all())
            torch.cuda.empty_cache()
        if world > 1:
            dist.barrier()
        del d_in
        torch.cuda.empty_cache()
        perms = H * ((w + 7) // 8) + (total - H)
        out[name] = {"config": desc, "path": path, "ms": round(ms, 3), "steps": EXTRA_STEPS, "warmup": EXTRA_WARMUP,
                     "value": round(L * w / (ms / 1e3) / 1e6, 3), "unit": "Melem/s (input elements, all GPUs)",
                     "lde_melem_s": round(H * w / (ms / 1e3) / 1e6, 3),
                     "gperm_s_per_gpu": round(perms / world / (ms / 1e3) / 1e9, 4),
                     "root": _hex_root(root), "root_check": check_path, "root_ok": root_ok}
    return out


def mg_context(zk, rank, world):
    """The library's multi-GPU context over a communicator it makes from an
    NCCL id that rank 0 creates and torch.distributed broadcasts."""
    import ctypes as C

    import torch.distributed as dist
    uid = C.create_string_buffer(128)
    if rank == 0:
        zk.check(zk.lib.zkie2_mg_unique_id(uid), "mg unique id")
    box = [uid.raw if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    uid = C.create_string_buffer(box[0], 128)
    ctx = C.c_void_p()
    zk.check(zk.lib.zkie2_mg_init(uid, world, rank, C.byref(ctx)), "mg init")
    return ctx


def e2e_mg(zk, dev, ctx, rank, world, lg_l, lg_b, w, d_in, want_root, numa, warmup, steps):
    """The end-to-end split commit through the C-ABI context
    (zkie2_mg_split_commit_host): per rank, its pinned 1/N row slice of the
    input in, column blocks pipelined (upload, NVLink all-gather of the
    block, coset LDE and leaf absorption, download of the block's LDE rows),
    its LDE rows and subtree layers back to pinned host memory."""
    import ctypes as C

    import numpy as np
    import torch
    import torch.distributed as dist
    lib = zk.lib
    L, H = 1 << lg_l, 1 << (lg_l + lg_b)
    rows, n_local = L // world, H // world
    with numa:
        h_part = torch.empty(rows * w, dtype=torch.uint64, pin_memory=True)
        h_part.view(torch.int64).copy_(d_in.view(torch.int64)[rank * rows * w:(rank + 1) * rows * w])
        h_lde = torch.empty(n_local * w, dtype=torch.uint64, pin_memory=True)
        n_lay = lib.zkie2_merkle_total_digests(n_local) * 8
        h_layers = torch.empty(n_lay, dtype=torch.uint64, pin_memory=True)
        scr = torch.empty(lib.zkie2_mg_split_commit_host_scratch_elems(lg_l, lg_b, w, world), dtype=torch.uint64,
                          device=dev)
        root = np.zeros(8, dtype=np.uint64)
        rp = root.ctypes.data_as(C.POINTER(C.c_uint64))

        def call():
            zk.check(lib.zkie2_mg_split_commit_host(ctx, h_part.data_ptr(), lg_l, lg_b, w, h_lde.data_ptr(),
                                                    h_layers.data_ptr(), rp, scr.data_ptr()), "mg split commit host")
        for _ in range(max(1, warmup)):
            call()
        k_e2e = max(1, min(steps, 5))
        dist.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(k_e2e):
            call()
        e2e_s = max_over_ranks((time.perf_counter() - t0) / k_e2e, dev)
        assert (root == want_root).all(), "host-path root differs from the device-path root"
    del h_part, h_lde, h_layers, scr
    torch.cuda.empty_cache()
    return {"value": round(L * w / e2e_s / 1e6, 3), "unit": UNIT, "ms_per_step": round(1e3 * e2e_s, 3),
            "h2d_bytes_per_step": 8 * L * w, "d2h_bytes_per_step": 8 * H * w + 8 * world * n_lay,
            "call": "zkie2_mg_split_commit_host (per rank: pinned 1/N row slice in, column blocks pipelined: "
                    "upload, NVLink all-gather, coset LDE + leaf absorption, LDE rows down; subtree layers back "
                    "to pinned host)",
            "host_memory": numa.describe()}


def mg_case(zk, dev, ctx, rank, world, lg_l, lg_b, w, want_root, t=28):
    """The same split commit and a 2^t split sumcheck through the library's
    own multi-GPU context (zkie2_mg_split_commit, zkie2_mg_split_sumcheck):
    the path a non-Python host drives.  ms per call
    (CUDA events around the synchronous calls, max over ranks); the root is
    compared with the torch-orchestrated split above, the proof with the
    single-GPU sumcheck on rank 0."""
    import ctypes as C

    import numpy as np
    import torch
    import torch.distributed as dist
    lib, check = zk.lib, zk.check
    P64 = C.POINTER(C.c_uint64)
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream
    out = {}
    L, H = 1 << lg_l, 1 << (lg_l + lg_b)
    n_local = H // world
    d_in = synth_device(L * w, 1234, dev)
    lde = torch.empty(n_local * w, dtype=torch.uint64, device=dev)
    layers = torch.empty(lib.zkie2_merkle_total_digests(n_local) * 8, dtype=torch.uint64, device=dev)
    top = torch.empty(lib.zkie2_mg_top_digests(world) * 8, dtype=torch.uint64, device=dev)
    scr = torch.empty(lib.zkie2_mg_split_commit_scratch_elems(lg_l, lg_b, w, world), dtype=torch.uint64,
                      device=dev)
    root = np.zeros(8, dtype=np.uint64)

    def commit():
        check(lib.zkie2_mg_split_commit(ctx, d_in.data_ptr(), lg_l, lg_b, w, lde.data_ptr(), layers.data_ptr(),
                                        top.data_ptr(), scr.data_ptr(), root.ctypes.data_as(P64), sh),
              "mg split commit")
    ms = _timed(commit, stream, dev, world)
    out["split_commit"] = {"ms": round(ms, 3), "value": round(L * w / (ms / 1e3) / 1e6, 3),
                           "unit": "Melem/s (input elements, all GPUs)",
                           "root_matches_torch_split": bool((root == want_root).all())}
    del d_in, lde, layers, top, scr
    torch.cuda.empty_cache()
    n_loc = (1 << t) // world
    f = synth_into(torch.empty(n_loc, dtype=torch.uint64, device=dev), 500 + rank)
    h = synth_into(torch.empty(n_loc, dtype=torch.uint64, device=dev), 600 + rank)
    ch = np.array([(0x9E3779B97F4A7C15 * (i + 1)) % P for i in range(t)], dtype=np.uint64)
    scr = torch.empty(lib.zkie2_mg_split_sumcheck_scratch_elems(t, world), dtype=torch.uint64, device=dev)
    rounds, fin = np.zeros((t, 3), dtype=np.uint64), np.zeros(2, dtype=np.uint64)

    def sumcheck():
        check(lib.zkie2_mg_split_sumcheck(ctx, f.data_ptr(), h.data_ptr(), t, ch.ctypes.data_as(P64),
                                          rounds.ctypes.data_as(P64), fin.ctypes.data_as(P64), scr.data_ptr(),
                                          sh), "mg split sumcheck")
    ms = _timed(sumcheck, stream, dev, world)
    ok = None
    if rank == 0:
        F = torch.empty(1 << t, dtype=torch.uint64, device=dev)
        G = torch.empty(1 << t, dtype=torch.uint64, device=dev)
        for r in range(world):
            synth_into(F[r * n_loc:(r + 1) * n_loc], 500 + r)
            synth_into(G[r * n_loc:(r + 1) * n_loc], 600 + r)
        ref = zk.sumcheck_prove(F, G, 0, ch)
        ok = bool(np.array_equal(rounds, ref.rounds) and (int(fin[0]), int(fin[1])) == (ref.f_eval, ref.h_eval))
        del F, G
    dist.barrier()
    hbm_peak, _ = hbm_peak_gbs()
    gbs = 16 * n_loc / (ms / 1e3) / 1e9
    out["split_sumcheck"] = {"config": f"sumcheck::prove, f and h of 2^{t} elements split over {world} GPUs",
                             "ms": round(ms, 4), "value": round((1 << t) / (ms / 1e3) / 1e6, 3),
                             "unit": "Melem/s", "rounds_match": ok,
                             "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm_peak,
                                          "unit": "GB/s per GPU", "frac": round(gbs / hbm_peak, 4)}}
    del f, h, scr
    torch.cuda.empty_cache()
    return out


def sumcheck_case(zk, dev, rank, world, t=28):
    """sumcheck::prove of f, h of 2^t elements, split over the ranks by the
    high variables (zkie_b200.multigpu.split_sumcheck: local rounds, ONE
    all-reduce of every local round message, an all-gather of the folded
    values, the last log2 N rounds on every rank); at N = 1 the plain
    single-GPU proof.  Rounds and finals are checked on rank 0 against the
    single-GPU proof of the whole vectors."""
    import numpy as np
    import torch

    from zkie_b200.multigpu import split_sumcheck
    n_loc = (1 << t) // world
    f = synth_into(torch.empty(n_loc, dtype=torch.uint64, device=dev), 500 + rank)
    h = synth_into(torch.empty(n_loc, dtype=torch.uint64, device=dev), 600 + rank)
    ch = np.array([(0x9E3779B97F4A7C15 * (i + 1)) % P for i in range(t)], dtype=np.uint64)
    for _ in range(2):
        split_sumcheck(f, h, t, ch)
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    reps = 5
    t0 = time.perf_counter()
    for _ in range(reps):
        rounds, fe, he = split_sumcheck(f, h, t, ch)
    torch.cuda.synchronize()
    ms = 1e3 * (time.perf_counter() - t0) / reps
    if world > 1:
        ms = max_over_ranks(ms, dev)
    ok = None
    if rank == 0:
        if world > 1:
            F = torch.empty(1 << t, dtype=torch.uint64, device=dev)
            G = torch.empty(1 << t, dtype=torch.uint64, device=dev)
            for r in range(world):
                synth_into(F[r * n_loc:(r + 1) * n_loc], 500 + r)
                synth_into(G[r * n_loc:(r + 1) * n_loc], 600 + r)
            ref = zk.sumcheck_prove(F, G, 0, ch)
            ok = bool(np.array_equal(np.asarray(rounds).reshape(-1, 3), ref.rounds)
                      and (fe, he) == (ref.f_eval, ref.h_eval))
            del F, G
        else:
            ok = True
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    del f, h
    torch.cuda.empty_cache()
    hbm_peak, _ = hbm_peak_gbs()
    gbs = 16 * n_loc / (ms / 1e3) / 1e9
    return {"config": f"sumcheck::prove, f and h of 2^{t} elements" +
                      (f" split over {world} GPUs by the high variables" if world > 1 else " on one GPU"),
            "ms": round(ms, 4), "value": round((1 << t) / (ms / 1e3) / 1e6, 3), "unit": "Melem/s",
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm_peak, "unit": "GB/s per GPU",
                         "frac": round(gbs / hbm_peak, 4),
                         "note": "16 bytes per element (f and h read once), whole call incl. host round trips"},
            "rounds_match": ok}


if __name__ == "__main__":
    sys.exit(main())
