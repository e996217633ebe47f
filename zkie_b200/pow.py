"""PoW grinding of the WHIR prover on the device: ``challenger.grind(bits)``
(p3-whir src/pcs/prover/mod.rs:240-245, 355-358) for the transcript's
DuplexChallenger<Goldilocks, Poseidon2-16, 16, 8> (crates/zkie-core/src/pcs/whir.rs:42).

The challenger itself stays with the caller: ``grind`` takes its sponge state
and buffered inputs, returns the smallest valid witness, and the caller then
replays ``check_witness(bits, witness)`` on its own challenger (one
permutation), as the reference does after its parallel search.
"""
import numpy as np

from ._lib import check, lib
from .device import stream_handle
from .gkr import _p


def grind(sponge_state, input_buffer, bits: int) -> int:
    """Smallest w < p with observe(w); sample_bits(bits) == 0 for the
    challenger (16-element sponge state, fewer than 8 buffered inputs)."""
    sp = np.ascontiguousarray(np.asarray(sponge_state, dtype=np.uint64).reshape(-1))
    inp = np.ascontiguousarray(np.asarray(list(input_buffer) or [0], dtype=np.uint64).reshape(-1))
    n_in = len(input_buffer)
    if sp.size != 16 or n_in >= 8:
        raise ValueError("grind: a 16-element sponge state and fewer than 8 buffered inputs")
    w = np.zeros(1, dtype=np.uint64)
    check(lib.zkie2_grind(_p(sp), _p(inp), n_in, bits, _p(w), stream_handle()), "zkie2_grind")
    return int(w[0])
