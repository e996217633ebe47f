"""Build recipe for the CPU oracle (test infrastructure, never part of the product).

Compiles oracle/zkie_oracle.c into oracle/liboracle.so with gcc + OpenMP.

The reference's host code is Rust, with no toolchain present, so this C
restatement is the CPU oracle.  The reference's two CUDA files are built
separately, against a stand-in for the three sppark names they include, by
``oracle/build_ref.py`` (the GPU parity tests run them beside this library).
"""
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "zkie_oracle.c")
OUT = os.path.join(HERE, "liboracle.so")


def build(force: bool = False) -> str:
    if (not force and os.path.exists(OUT)
            and os.path.getmtime(OUT) >= max(os.path.getmtime(os.path.join(HERE, f))
                                             for f in ("zkie_oracle.c", "zkie_oracle.h", "packed_field.h"))):
        return OUT
    # -fno-semantic-interposition: the exported field primitives (orc_add,
    # orc_mul, ...) are inlined into the library's own loops instead of being
    # called through the PLT; no -march: the library travels to other hosts
    cmd = ["gcc", "-O3", "-std=gnu11", "-fPIC", "-fno-semantic-interposition", "-shared", "-fopenmp", "-Wall",
           "-Wno-unknown-pragmas", "-o", OUT + ".tmp", SRC]
    subprocess.check_call(cmd)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
