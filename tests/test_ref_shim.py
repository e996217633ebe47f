"""The sppark stand-in under oracle/ref_shim/ (the field type the reference's
own CUDA kernels are compiled against for the GPU parity tests), checked on
the CPU against Python integer arithmetic modulo p: construction from any
u64 (non-canonical values included), +, -, *, sqr, [0] and the explicit
conversion, on edge values and random operands."""
import os
import random
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SHIM = os.path.join(ROOT, "oracle", "ref_shim")
P = 0xFFFFFFFF00000001

PROG = r"""
#include <cstdio>
#include <cinttypes>
#include <ff/goldilocks.hpp>
using gl = goldilocks::fr_t;
int main() {
    unsigned long long a, b;
    while (std::scanf("%llu %llu", &a, &b) == 2) {
        gl x(a), y(b);
        gl s = x + y, d = x - y, m = x * y, q = x;
        q.sqr();
        gl acc = x;
        acc += y;
        acc *= y;
        std::printf("%" PRIu64 " %" PRIu64 " %" PRIu64 " %" PRIu64 " %" PRIu64 " %" PRIu64 "\n",
                    static_cast<uint64_t>(x), s[0], d[0], m[0], static_cast<uint64_t>(q), acc[0]);
    }
    return 0;
}
"""


@pytest.mark.skipif(shutil.which("g++") is None, reason="g++ not available")
def test_shim_field_matches_integer_arithmetic(tmp_path):
    src, exe = tmp_path / "shim.cpp", tmp_path / "shim"
    src.write_text(PROG)
    subprocess.check_call(["g++", "-O2", "-std=c++17", "-D__host__=", "-D__device__=", "-I" + SHIM, str(src),
                           "-o", str(exe)])
    edge = [0, 1, 2, P - 1, P - 2, P, P + 1, 2 ** 64 - 1, 2 ** 32, 2 ** 32 - 1, 2 ** 63, (P + 1) // 2]
    rng = random.Random(7)
    pairs = [(a, b) for a in edge for b in edge] + [(rng.getrandbits(64), rng.getrandbits(64)) for _ in range(5000)]
    out = subprocess.run([str(exe)], input="\n".join(f"{a} {b}" for a, b in pairs), capture_output=True, text=True,
                         check=True).stdout.split("\n")
    for (a, b), line in zip(pairs, out):
        x, y = a % P, b % P
        exp = [x, (x + y) % P, (x - y) % P, x * y % P, x * x % P, (x + y) * y % P]
        assert [int(v) for v in line.split()] == exp, (a, b)
