"""bincode 1.3.3 bytes of the proofs this library produces, in the layout the
reference's serde derives give them (little-endian, fixed-width integers, u64
sequence lengths, struct fields in declaration order, each Goldilocks as its
u64 word), so a Rust caller can deserialize them with its own types:

- ``SumcheckProof { rounds: Vec<RoundPoly{c0,c1,c2}>, f_eval, h_eval }``  <- common/sumcheck.rs:10-29
- ``MatmulProof { claimed, sumcheck: SumcheckProof }``                     <- common/matmul.rs:11-15
- ``SumcheckProofBatch { rounds: Vec<RoundPoly>, b_eval }``                <- common/sumcheck.rs:236-240
- ``VirtualProof { rounds: Vec<Vec<Goldilocks>>, final_evals }``          <- common/sumcheck.rs:373-377
- ``FractionalProof { layers: Vec<FractionalLayer{r, c, proof}>, final_num, final_den, full_r }``
                                                                          <- common/logup_gkr.rs:7-18

The device emits canonical field elements; p3 serializes its internal word,
which is non-canonical only for values it holds in [p, 2^64) (about 2^-32 of
results), so canonical bytes deserialize to the same field elements.
"""
import struct

import numpy as np

from .gkr import MatmulProof, SumcheckProof, SumcheckProofBatch, VirtualProof
from .logup import FractionalLayer, FractionalProof

P = 0xFFFFFFFF00000001


class _W:
    def __init__(self):
        self.parts = []

    def u64(self, v):
        self.parts.append(struct.pack("<Q", int(v)))

    def fe(self, v):
        self.u64(int(v) % P)

    def vec_fe(self, vals):
        vals = [int(x) for x in np.asarray(vals, dtype=np.uint64).reshape(-1)]
        self.u64(len(vals))
        self.parts.append(struct.pack(f"<{len(vals)}Q", *[v % P for v in vals]))

    def bytes(self):
        return b"".join(self.parts)


class _R:
    def __init__(self, data):
        self.data, self.pos = data, 0

    def u64(self):
        if self.pos + 8 > len(self.data):
            raise ValueError("proof bytes: truncated")
        v = struct.unpack_from("<Q", self.data, self.pos)[0]
        self.pos += 8
        return v

    def vec_fe(self):
        n = self.u64()
        if self.pos + 8 * n > len(self.data):
            raise ValueError("proof bytes: truncated")
        v = np.frombuffer(self.data, dtype="<u8", count=n, offset=self.pos).astype(np.uint64)
        self.pos += 8 * n
        return v


def _rounds3(w, rounds):
    r = np.asarray(rounds, dtype=np.uint64).reshape(-1, 3)
    w.u64(r.shape[0])
    for c0, c1, c2 in r:
        w.fe(c0), w.fe(c1), w.fe(c2)


def _read_rounds3(r):
    n = r.u64()
    return np.array([[r.u64(), r.u64(), r.u64()] for _ in range(n)], dtype=np.uint64).reshape(n, 3)


def _virtual(w, p: VirtualProof):
    rounds = np.asarray(p.rounds, dtype=np.uint64)
    w.u64(rounds.shape[0])
    for row in rounds:
        w.vec_fe(row)
    w.vec_fe(p.final_evals)


def _read_virtual(r) -> VirtualProof:
    n = r.u64()
    rows = [r.vec_fe() for _ in range(n)]
    width = rows[0].size if rows else 0
    if any(x.size != width for x in rows):
        raise ValueError("proof bytes: ragged round messages")
    rounds = np.stack(rows) if rows else np.zeros((0, 0), dtype=np.uint64)
    return VirtualProof(rounds, r.vec_fe())


def to_bincode(proof) -> bytes:
    """bincode bytes of a SumcheckProof, MatmulProof, SumcheckProofBatch,
    VirtualProof or FractionalProof."""
    w = _W()
    if isinstance(proof, MatmulProof):
        w.fe(proof.claimed)
        proof = proof.sumcheck
    if isinstance(proof, SumcheckProof):
        _rounds3(w, proof.rounds)
        w.fe(proof.f_eval), w.fe(proof.h_eval)
    elif isinstance(proof, SumcheckProofBatch):
        _rounds3(w, proof.rounds)
        w.fe(proof.b_eval)
    elif isinstance(proof, VirtualProof):
        _virtual(w, proof)
    elif isinstance(proof, FractionalProof):
        w.u64(len(proof.layers))
        for layer in proof.layers:
            w.vec_fe(layer.r)
            w.fe(layer.c)
            _virtual(w, layer.proof)
        w.fe(proof.final_num), w.fe(proof.final_den)
        w.vec_fe(proof.full_r)
    else:
        raise TypeError(f"no bincode layout for {type(proof).__name__}")
    return w.bytes()


def from_bincode(kind, data: bytes):
    """Decode bytes written by ``to_bincode`` (or by the reference) as ``kind``,
    one of the proof classes above; the whole input must be consumed."""
    r = _R(data)
    if kind is MatmulProof:
        claimed = r.u64()
        rounds = _read_rounds3(r)
        out = MatmulProof(claimed, SumcheckProof(rounds, r.u64(), r.u64()))
    elif kind is SumcheckProof:
        rounds = _read_rounds3(r)
        out = SumcheckProof(rounds, r.u64(), r.u64())
    elif kind is SumcheckProofBatch:
        rounds = _read_rounds3(r)
        out = SumcheckProofBatch(rounds, r.u64())
    elif kind is VirtualProof:
        out = _read_virtual(r)
    elif kind is FractionalProof:
        layers = []
        for _ in range(r.u64()):
            rr = r.vec_fe()
            c = r.u64()
            layers.append(FractionalLayer(rr, c, _read_virtual(r)))
        fn, fd = r.u64(), r.u64()
        out = FractionalProof(layers, fn, fd, r.vec_fe())
    else:
        raise TypeError(f"no bincode layout for {kind}")
    if r.pos != len(data):
        raise ValueError("proof bytes: trailing data")
    return out
