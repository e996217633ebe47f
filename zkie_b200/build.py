"""Build libzkie_b200.so in-tree with nvcc for sm_100a.

Every .cu / .cpp under zkie_b200/csrc is compiled to an object under
zkie_b200/_build (incrementally, in parallel) and linked with the static CUDA
runtime into zkie_b200/libzkie_b200.so.  The shared object travels with the
source tree; nothing is JIT-compiled at import time.
"""
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libzkie_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def cutlass_include() -> list:
    """-I flags of the CUTLASS/CuTe header tree (the tensor-core GEMM of the
    fixed-point forward matmul instantiates its sm100 templates): the tree
    vendored with the flashinfer package, or $CUTLASS_DIR."""
    cands = []
    if os.environ.get("CUTLASS_DIR"):
        cands.append(os.environ["CUTLASS_DIR"])
    try:
        import site
        for sp in site.getsitepackages():
            cands.append(os.path.join(sp, "flashinfer", "data", "cutlass"))
    except Exception:
        pass
    for c in cands:
        if os.path.exists(os.path.join(c, "include", "cutlass", "gemm", "collective", "collective_builder.hpp")):
            return ["-I" + os.path.join(c, "include"), "-I" + os.path.join(c, "tools", "util", "include")]
    raise RuntimeError("CUTLASS headers not found (set CUTLASS_DIR to a CUTLASS 4.x checkout)")


NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "-diag-suppress", "550,20012",
                     "--expt-relaxed-constexpr", "-I" + INCLUDE]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _headers():
    hs = []
    for d in (CSRC, INCLUDE):
        for f in os.listdir(d):
            if f.endswith((".h", ".cuh", ".hpp")):
                hs.append(os.path.join(d, f))
    return hs


def _compile(src: str, obj: str, verbose_ptxas: bool) -> str:
    cmd = [nvcc()] + NVCC_FLAGS + (cutlass_include() if src.endswith("_tc.cu") else []) + ["-c", src, "-o", obj]
    if verbose_ptxas and src.endswith(".cu"):
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stderr}")
    return res.stderr


def build(force: bool = False, verbose_ptxas: bool = False, jobs: int = 8) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))
    hdr_mtime = max(os.path.getmtime(h) for h in _headers())
    todo, objs = [], []
    for s in srcs:
        obj = os.path.join(BUILD, os.path.basename(s) + ".o")
        objs.append(obj)
        if force or not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(s), hdr_mtime):
            todo.append((s, obj))
    logs = []
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
            futs = {ex.submit(_compile, s, o, verbose_ptxas): s for s, o in todo}
            for f in cf.as_completed(futs):
                logs.append((futs[f], f.result()))
    need_link = force or todo or not os.path.exists(LIB) or \
        os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs)
    if need_link:
        tmp = LIB + ".tmp"
        cmd = [nvcc()] + ARCH + ["-shared", "--cudart", "static", "-o", tmp] + objs + ["-ldl"]
        subprocess.check_call(cmd)
        os.replace(tmp, LIB)
    if verbose_ptxas:
        for s, log in logs:
            sys.stderr.write(f"== {os.path.basename(s)}\n{log}")
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv))
