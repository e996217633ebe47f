"""Build recipe for oracle/_ref/libzkie_ref.so: the reference's OWN CUDA kernels.

TEST INFRASTRUCTURE, never part of the product.  The two CUDA files of the
reference's GPU backend (crates/zkie-core/cuda/goldilocks_ntt.cu and
poseidon2_merkle.cu) are compiled where they lie in the reference checkout,
unmodified, with nvcc for sm_100a, into oracle/_ref/libzkie_ref.so.  They
export the same seven C symbols as libzkie_b200.so (the seam of
crates/zkie-core/src/pcs/cuda_ffi.rs:2-46), so the GPU parity tests can run
the reference kernels and this library's kernels on the same inputs,
constants and twiddle tables and compare every output bit for bit.

The files include three names from sppark 0.1.15, which is not in the
reference tree: goldilocks::fr_t (<ff/goldilocks.hpp>), CUDA_OK / cuda_error
(<util/exception.cuh>) and ngpus() (<util/gpu_t.cuh>).  oracle/ref_shim/
holds a from-scratch stand-in for exactly those names (a canonical Goldilocks
field element; a throwing error check; the device count).

The reference checkout is taken from $ZKIE_REFERENCE_DIR, else the directory
"reference" beside this repository.  Without it, nothing is built and the
tests that need the library skip; a library built earlier is kept (it travels
with the tree to a machine that has no reference checkout).
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SHIM = os.path.join(HERE, "ref_shim")
OUT_DIR = os.path.join(HERE, "_ref")
OUT = os.path.join(OUT_DIR, "libzkie_ref.so")
FILES = ("goldilocks_ntt.cu", "poseidon2_merkle.cu")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def reference_dir() -> str:
    env = os.environ.get("ZKIE_REFERENCE_DIR")
    if env:
        return env
    return os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")


def sources():
    cuda = os.path.join(reference_dir(), "crates", "zkie-core", "cuda")
    srcs = [os.path.join(cuda, f) for f in FILES]
    return srcs if all(os.path.exists(s) for s in srcs) else None


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def build(force: bool = False):
    """Build the library if the reference sources are present; returns its
    path, or None when neither the sources nor an earlier build exist."""
    srcs = sources()
    if srcs is None:
        return OUT if os.path.exists(OUT) else None
    shim = [os.path.join(d, f) for d, _, fs in os.walk(SHIM) for f in fs]
    newest = max(os.path.getmtime(p) for p in srcs + shim + [os.path.abspath(__file__)])
    if not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= newest:
        return OUT
    os.makedirs(OUT_DIR, exist_ok=True)
    objs = []
    for s in srcs:
        obj = os.path.join(OUT_DIR, os.path.basename(s) + ".o")
        subprocess.check_call([_nvcc()] + ARCH + ["-O3", "-std=c++17", "-Xcompiler", "-fPIC", "-I" + SHIM,
                                                 "-diag-suppress", "186", "-c", s, "-o", obj])
        objs.append(obj)
    subprocess.check_call([_nvcc()] + ARCH + ["-shared", "--cudart", "static", "-o", OUT + ".tmp"] + objs)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
