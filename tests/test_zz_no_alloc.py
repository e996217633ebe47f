"""The allocation-free sumcheck entry point, zkie2_sumcheck_prove_noalloc.

It exists for callers that cannot allocate device memory (a prover living
next to a framework allocator that already holds the GPU's memory, or a
latency-critical caller that cannot take cudaFree's device-wide sync).  Its
scratch is a fixed array inside the library, shared by every call.  This test
calls it through the C ABI several times in a row, with different inputs each
time so stale contents from an earlier call would show, at sizes from no
variables to the largest the array holds, and checks every result bit-exactly
against the allocating entry point zkie2_sumcheck_prove.  It sits
in its own file so that pytest collects it last."""
import ctypes as C

import numpy as np
import pytest

P = 0xFFFFFFFF00000001
pytestmark = pytest.mark.gpu


def _fields(seed, n):
    g = np.random.default_rng(seed)
    v = g.integers(0, 2 ** 64, size=n, dtype=np.uint64)
    return np.where(v >= np.uint64(P), v - np.uint64(P), v).astype(np.uint64)


def _p(a):
    return a.ctypes.data_as(C.POINTER(C.c_uint64))


def test_noalloc_sumcheck_matches_allocating_entry_point(zk):
    import torch
    lib = zk.lib
    t_max = lib.zkie2_sumcheck_noalloc_max_vars()
    assert t_max == 24
    stream = torch.cuda.current_stream().cuda_stream
    # t_max fills the fixed array to its end (round polynomials and finals sit
    # last); t = 0 has no rounds, only the two canonicalised values
    for call, t in enumerate((18, 14, 0, t_max)):
        f = _fields(10 + call, 1 << t)
        h = _fields(20 + call, 1 << t)
        ch = _fields(30 + call, t)
        df, dh = torch.from_numpy(f).cuda(), torch.from_numpy(h).cuda()
        rounds = np.zeros((t, 3), dtype=np.uint64)
        finals = np.zeros(2, dtype=np.uint64)
        rc = lib.zkie2_sumcheck_prove_noalloc(df.data_ptr(), dh.data_ptr(), t, _p(ch), _p(rounds), _p(finals),
                                              stream)
        assert rc == 0, f"call {call}: cudaError {rc}"
        ref = zk.sumcheck_prove(df, dh, 0, ch)   # allocating entry point, scratch from torch
        assert np.array_equal(rounds, ref.rounds), f"call {call}: round polynomials differ"
        assert (int(finals[0]), int(finals[1])) == (ref.f_eval, ref.h_eval), f"call {call}: finals differ"


def test_noalloc_sumcheck_rejects_oversize(zk):
    import torch
    t = zk.lib.zkie2_sumcheck_noalloc_max_vars() + 1
    d = torch.zeros(4, dtype=torch.uint64, device="cuda")
    ch = np.zeros(t, dtype=np.uint64)
    rounds = np.zeros((t, 3), dtype=np.uint64)
    finals = np.zeros(2, dtype=np.uint64)
    rc = zk.lib.zkie2_sumcheck_prove_noalloc(d.data_ptr(), d.data_ptr(), t, _p(ch), _p(rounds), _p(finals), None)
    assert rc != 0
