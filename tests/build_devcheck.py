"""Build tests/_build/libdevcheck.so from tests/devcheck.cu (test infrastructure)."""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "devcheck.cu")
OUT = os.path.join(HERE, "_build", "libdevcheck.so")
HDRS = [os.path.join(HERE, "..", "zkie_b200", "csrc", f) for f in ("gl64.cuh", "poseidon2.cuh", "dft_reg.cuh")]


def build() -> str:
    os.makedirs(os.path.dirname(OUT), exist_ok=True)
    newest = max(os.path.getmtime(p) for p in [SRC] + HDRS)
    if os.path.exists(OUT) and os.path.getmtime(OUT) >= newest:
        return OUT
    nvcc = "/usr/local/cuda/bin/nvcc" if os.path.exists("/usr/local/cuda/bin/nvcc") else "nvcc"
    subprocess.check_call([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17",
                           "-Xcompiler", "-fPIC", "-shared", "--cudart", "static", "-diag-suppress", "550", "-o", OUT + ".tmp", SRC])
    os.replace(OUT + ".tmp", OUT)
    return OUT
