"""Host-side mirror of zkIE's commit seam, backed by libzkie_b200.so.

- ``CudaDft.dft_batch``      <- crates/zkie-core/src/pcs/dft_cuda.rs:121-222
- ``CudaMerkleTreeMmcs.commit`` <- crates/zkie-core/src/pcs/merkle_cuda.rs:132-393
- ``Whir.commit / commit_batch`` (commit geometry only)
                              <- crates/zkie-core/src/pcs/whir.rs:296-359, 438-519
- ``commit`` (LDE at any blowup + Merkle; the BASELINE raw-commit sweep)

Like the reference these raise on bad shapes; unlike it they never fall back
to a CPU implementation: any CUDA error raises ``ZkieError``.
"""
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib
from ._lib import check, lib
from .device import empty, ptr, stream_handle, to_dev, to_host

DIGEST_ELEMS = 8
MERKLE_ARITY = 2


def _lg(h: int) -> int:
    lg = h.bit_length() - 1
    if h != 1 << lg:
        raise ValueError("height must be a power of two")
    return lg


def padded_len(raw_len: int, n: int = MERKLE_ARITY) -> int:
    """p3-merkle-tree padded_len (vendor/p3-merkle-tree/src/merkle_tree.rs:577-585)."""
    if raw_len <= 1:
        return raw_len
    if raw_len >= n:
        return -(-raw_len // n) * n
    return n


def merkle_layer_lengths(h: int):
    lens = [padded_len(h)]
    while lens[-1] > 1:
        lens.append(padded_len(lens[-1] // MERKLE_ARITY))
    return lens


def split_layers(flat: np.ndarray, h: int):
    out, off = [], 0
    for ln in merkle_layer_lengths(h):
        out.append(flat[off:off + ln])
        off += ln
    return out


def p2_default_constants(seed: int = 1):
    """Round constants of Perm::new_from_rng_128(SmallRng::seed_from_u64(seed))
    (pcs/merkle_cuda.rs:54-85): (rc_init 4x16, rc_final 4x16, rc_internal 22, diag15)."""
    ri = np.zeros(64, dtype=np.uint64)
    rf = np.zeros(64, dtype=np.uint64)
    rp = np.zeros(22, dtype=np.uint64)
    d15 = _lib.u64(0)
    check(lib.zkie2_p2_default_constants(seed, _np_ptr(ri), _np_ptr(rf), _np_ptr(rp), _lib.C.byref(d15)),
          "zkie2_p2_default_constants")
    return ri.reshape(4, 16), rf.reshape(4, 16), rp, int(d15.value)


def _np_ptr(a: np.ndarray):
    assert a.dtype == np.uint64 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(_lib.pu64)


def upload_constants(rc_init, rc_final, rc_internal, diag15):
    """zkie_p2_upload_constants on the current device."""
    ri = np.ascontiguousarray(np.asarray(rc_init, dtype=np.uint64).reshape(-1))
    rf = np.ascontiguousarray(np.asarray(rc_final, dtype=np.uint64).reshape(-1))
    rp = np.ascontiguousarray(np.asarray(rc_internal, dtype=np.uint64).reshape(-1))
    check(lib.zkie_p2_upload_constants(_np_ptr(ri), _np_ptr(rf), _np_ptr(rp), int(diag15)),
          "zkie_p2_upload_constants")


def init_default_constants():
    check(lib.zkie2_p2_init_default(), "zkie2_p2_init_default")


def make_twiddles(lg: int) -> np.ndarray:
    """Concatenated per-stage DIT twiddles (pcs/dft_cuda.rs:44-59): stage s at
    offset 2^(s-1) - 1 holds TWO_ADIC_GENERATORS[s]^j, j < 2^(s-1)."""
    out = np.zeros(max((1 << lg) - 1, 1), dtype=np.uint64)
    check(lib.zkie2_dft_twiddles(lg, _np_ptr(out)), "zkie2_dft_twiddles")
    return out


class CudaDft:
    """TwoAdicSubgroupDft<Goldilocks>::dft_batch through the reference entry
    point zkie_ntt_forward_goldilocks."""

    def __init__(self):
        self._tw = {}

    def _twiddles(self, lg):
        if lg not in self._tw:
            self._tw[lg] = to_dev(make_twiddles(lg))
        return self._tw[lg]

    def dft_batch(self, mat: np.ndarray) -> np.ndarray:
        mat = np.asarray(mat, dtype=np.uint64)
        h, w = mat.shape
        if h <= 1:
            return mat
        lg = _lg(h)
        d_mat = to_dev(mat)
        d_temp = empty(h * w)
        check(lib.zkie_ntt_forward_goldilocks(ptr(d_mat), ptr(d_temp), lg, w, ptr(self._twiddles(lg))),
              "zkie_ntt_forward_goldilocks")
        torch.cuda.synchronize()
        return to_host(d_mat).reshape(h, w)


@dataclass
class MerkleTree:
    """Digest layers of one matrix (layer 0 = leaves, last = [root])."""
    layers: list
    root: np.ndarray


class CudaMerkleTreeMmcs:
    """Mmcs<Goldilocks>::commit for a single matrix.

    ``commit`` runs the fused tree builder (zkie2_merkle_tree);
    ``commit_reference_sequence`` drives the reference symbols in exactly the
    order commit_gpu does (pcs/merkle_cuda.rs:227-285)."""

    def __init__(self, constants=None):
        if constants is None:
            init_default_constants()
        else:
            upload_constants(*constants)

    def commit(self, mat) -> MerkleTree:
        d_mat = to_dev(mat)
        h, w = (d_mat.shape[0], d_mat.shape[1]) if d_mat.dim() == 2 else (d_mat.shape[0], 1)
        tot = lib.zkie2_merkle_total_digests(h)
        d_layers = empty(tot * DIGEST_ELEMS)
        check(lib.zkie2_merkle_tree(ptr(d_mat), h, w, ptr(d_layers), stream_handle()), "zkie2_merkle_tree")
        flat = to_host(d_layers).reshape(-1, DIGEST_ELEMS)
        layers = split_layers(flat, h)
        return MerkleTree(layers, layers[-1][0].copy())

    def commit_reference_sequence(self, mat, ffi=None) -> MerkleTree:
        """``ffi``: another library exporting the same seven C symbols (the
        parity tests pass the reference's own kernels); default: this one."""
        lib_ = lib if ffi is None else ffi
        mat = np.asarray(mat, dtype=np.uint64)
        h, w = mat.shape
        lens = merkle_layer_lengths(h)
        d_mat = to_dev(mat)
        d_layers = [torch.zeros(n * DIGEST_ELEMS, dtype=torch.uint64, device=d_mat.device) for n in lens]
        batches = h // 8
        check(lib_.zkie_p2_leaf_batch(ptr(d_mat), ptr(d_layers[0]), h, w), "zkie_p2_leaf_batch")
        check(lib_.zkie_p2_leaf_scalar(ptr(d_mat), ptr(d_layers[0]), batches * 8, h, w), "zkie_p2_leaf_scalar")
        for i in range(len(lens) - 1):
            raw = lens[i] // MERKLE_ARITY
            check(lib_.zkie_p2_compress_batch(ptr(d_layers[i]), ptr(d_layers[i + 1]), raw, MERKLE_ARITY),
                  "zkie_p2_compress_batch")
            check(lib_.zkie_p2_compress_scalar(ptr(d_layers[i]), ptr(d_layers[i + 1]), raw // 8 * 8, raw,
                                              MERKLE_ARITY), "zkie_p2_compress_scalar")
        torch.cuda.synchronize()
        layers = [to_host(l).reshape(-1, DIGEST_ELEMS) for l in d_layers]
        return MerkleTree(layers, layers[-1][0].copy())


@dataclass
class Committed:
    """A committed matrix kept resident in HBM: the LDE (the tree's leaves),
    the flat digest layers and the root."""
    root: np.ndarray
    lde: torch.Tensor
    layers: torch.Tensor
    height: int
    width: int

    def layer_list(self):
        return split_layers(to_host(self.layers).reshape(-1, DIGEST_ELEMS), self.height)


def commit(coeffs, lg_blowup: int, stream=None) -> Committed:
    """LDE (zero-pad L -> L << lg_blowup rows, DFT per column, shift 1) of the
    L x w coefficient matrix, then the Merkle tree over the LDE rows."""
    d_in = to_dev(coeffs)
    L = d_in.shape[0]
    w = d_in.shape[1] if d_in.dim() == 2 else 1
    lg_l = _lg(L)
    H = L << lg_blowup
    d_lde = empty(H * w)
    d_layers = empty(lib.zkie2_merkle_total_digests(H) * DIGEST_ELEMS)
    ns = lib.zkie2_commit_scratch_elems(lg_l, lg_blowup, w)
    d_scr = empty(max(ns, 1))
    check(lib.zkie2_commit(ptr(d_in), lg_l, lg_blowup, w, ptr(d_lde), ptr(d_layers), ptr(d_scr),
                           stream_handle(stream)), "zkie2_commit")
    root = to_host(d_layers[-DIGEST_ELEMS:]).copy()
    return Committed(root, d_lde.view(H, w), d_layers, H, w)


def commit_cosets(coeffs, lg_blowup: int, lg_cosets: int, w: int = None, stream=None):
    """zkie2_commit_cosets: the commit of an L x w coefficient matrix (device
    tensor or host array) whose LDE need not fit in HBM, computed one coset of
    the LDE rows at a time.  Returns (root, flat digest layers on the device);
    same root and layers as ``commit``, the LDE is not kept."""
    d_in = to_dev(coeffs)
    if w is None:
        w = d_in.shape[1] if d_in.dim() == 2 else 1
    L = d_in.numel() // w
    lg_l = _lg(L)
    H = L << lg_blowup
    ns = lib.zkie2_commit_cosets_scratch_elems(lg_l, lg_blowup, w, lg_cosets)
    if ns == 0:
        raise ValueError("commit_cosets needs (2^lg_cosets)^2 <= LDE rows")
    d_layers = empty(lib.zkie2_merkle_total_digests(H) * DIGEST_ELEMS)
    d_scr = empty(ns)
    check(lib.zkie2_commit_cosets(ptr(d_in), lg_l, lg_blowup, w, lg_cosets, ptr(d_layers), ptr(d_scr),
                                  stream_handle(stream)), "zkie2_commit_cosets")
    del d_scr
    return to_host(d_layers[-DIGEST_ELEMS:]).copy(), d_layers


def commit_host(coeffs: np.ndarray, lg_blowup: int, want_lde=True, want_layers=True):
    """zkie2_commit_host: host buffers in and out (pinned buffers recommended)."""
    coeffs = np.ascontiguousarray(np.asarray(coeffs, dtype=np.uint64))
    L, w = coeffs.shape
    lg_l = _lg(L)
    H = L << lg_blowup
    lde = np.empty((H, w), dtype=np.uint64) if want_lde else None
    layers = np.empty((lib.zkie2_merkle_total_digests(H), DIGEST_ELEMS), dtype=np.uint64) if want_layers else None
    root = np.zeros(DIGEST_ELEMS, dtype=np.uint64)
    check(lib.zkie2_commit_host(coeffs.ctypes.data, lg_l, lg_blowup, w,
                                lde.ctypes.data if lde is not None else None,
                                layers.ctypes.data if layers is not None else None,
                                root.ctypes.data), "zkie2_commit_host")
    return root, lde, layers


class Whir:
    """Commit geometry of the WHIR wrapper (pcs/whir.rs): folding factor 5,
    starting_log_inv_rate 1.  Opening / verification stay on the CPU side of
    the reference and are not part of this path."""
    FOLDING_FACTOR = 5
    STARTING_LOG_INV_RATE = 1

    def __init__(self, num_variables: int, security_level: int = 90, pow_bits: int = 32):
        self.num_variables = num_variables
        self.security_level = security_level
        self.pow_bits = pow_bits

    @classmethod
    def new(cls, num_variables):
        return cls(num_variables, 90, 32)

    @classmethod
    def new_testing(cls, num_variables):
        return cls(num_variables, 32, 10)

    @classmethod
    def with_params(cls, num_variables, security_level, pow_bits):
        return cls(num_variables, security_level, pow_bits)

    def commit(self, evals, stream=None) -> Committed:
        """Whir::commit (pcs/whir.rs:438-469): 2^n evaluations as a 2^(n-5) x 32
        row-major matrix, blowup 2, DFT per column, Merkle over rows."""
        d = to_dev(evals).reshape(-1)
        n = _lg(d.numel())
        if n < self.FOLDING_FACTOR:
            raise ValueError("WHIR commit needs at least 2^5 evaluations")
        H = 1 << (n - 4)
        d_lde = empty(H * 32)
        d_layers = empty(lib.zkie2_merkle_total_digests(H) * DIGEST_ELEMS)
        d_scr = empty(max(lib.zkie2_whir_scratch_elems(n), 1))
        check(lib.zkie2_whir_commit(ptr(d), n, ptr(d_lde), ptr(d_layers), ptr(d_scr), stream_handle(stream)),
              "zkie2_whir_commit")
        root = to_host(d_layers[-DIGEST_ELEMS:]).copy()
        return Committed(root, d_lde.view(H, 32), d_layers, H, 32)

    def commit_batch(self, evals_batch, stream=None):
        """Whir::commit_batch (pcs/whir.rs:476-519): same-size tables stacked
        into one 2^total_num_vars witness, total_num_vars =
        ceil(log2(tables * 2^arity)).  The stacking order lives in the
        unvendored p3-sumcheck; tables are concatenated in order and
        zero-padded."""
        if len(evals_batch) == 0:
            raise ValueError("batch must not be empty")
        tabs = [to_dev(e).reshape(-1) for e in evals_batch]
        size = tabs[0].numel()
        if any(t.numel() != size for t in tabs):
            raise ValueError("all MLEs in a batch must have the same size")
        total = len(tabs) * size
        total_vars = (total - 1).bit_length() if total > 1 else 0
        stacked = torch.zeros(1 << total_vars, dtype=torch.uint64, device=tabs[0].device)
        stacked[:total] = torch.cat(tabs)
        batch_whir = Whir(total_vars, self.security_level, self.pow_bits)
        return batch_whir.commit(stacked, stream), batch_whir

    # ---- per-round commits of the WHIR prover -----------------------------------------
    MAX_NUM_VARIABLES_TO_SEND_COEFFS = 6

    @staticmethod
    def folding_schedule(num_variables: int, factor: int = FOLDING_FACTOR):
        """FoldingFactor::Constant(factor).compute_folding_schedule
        (vendor/p3-whir/src/parameters/folding.rs:88-104): fold `factor`
        variables per round until at most 6 remain."""
        if factor == 0:
            raise ValueError("zero folding factor")
        if factor > num_variables:
            raise ValueError("folding factor larger than the number of variables")
        remaining, schedule = num_variables, []
        while True:
            f = min(factor, remaining)
            schedule.append(f)
            remaining -= f
            if remaining <= Whir.MAX_NUM_VARIABLES_TO_SEND_COEFFS:
                return schedule

    def round_commits(self):
        """(num_variables, log_inv_rate) of each round's commit_extension:
        num_rounds = len(schedule) - 1 (folding.rs:177-184); round i commits
        the polynomial folded i + 1 times, at log_inv_rate 1 + (i + 1)(5 - 1)
        (round_log_inv_rates of pcs/whir.rs:298-304)."""
        sched = self.folding_schedule(self.num_variables)
        out, n, rate = [], self.num_variables, self.STARTING_LOG_INV_RATE
        for r in range(len(sched) - 1):
            n -= sched[r]
            rate += sched[r] - 1
            out.append((n, rate))
        return out

    @staticmethod
    def commit_extension(evals_ef, log_inv_rate: int, stream=None) -> Committed:
        """commit_extension (vendor/p3-whir/src/pcs/committer/writer.rs:21-86,
        Suffix order) of 2^n extension-field evaluations given as a (2^n, 2)
        array of base coefficients (c0, c1): the (2^(n-5) << log_inv_rate) x 32
        EF encoding, stored and hashed as 64 base columns per row."""
        d = to_dev(evals_ef).reshape(-1)
        n = _lg(d.numel() // 2)
        if d.numel() != 2 << n or n < 5:
            raise ValueError("commit_extension needs 2^n >= 32 EF elements (2 u64 each)")
        H = 1 << (n - 5 + log_inv_rate)
        d_lde = empty(H * 64)
        d_layers = empty(lib.zkie2_merkle_total_digests(H) * DIGEST_ELEMS)
        d_scr = empty(max(lib.zkie2_commit_extension_scratch_elems(n, log_inv_rate), 1))
        check(lib.zkie2_commit_extension(ptr(d), n, log_inv_rate, ptr(d_lde), ptr(d_layers), ptr(d_scr),
                                         stream_handle(stream)), "zkie2_commit_extension")
        root = to_host(d_layers[-DIGEST_ELEMS:]).copy()
        return Committed(root, d_lde.view(H, 64), d_layers, H, 64)
