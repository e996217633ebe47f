"""ctypes view of the CPU oracle (TEST INFRASTRUCTURE).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg import
this module, and only to check or time against the CUDA product.  Nothing in
``zkie_b200`` imports it.
"""
import ctypes as C
import os

import numpy as np

from . import build_oracle

P = 0xFFFFFFFF00000001

_u64 = C.c_uint64
_u32 = C.c_uint32
_pu64 = C.POINTER(C.c_uint64)
_pu32 = C.POINTER(C.c_uint32)


class P2Consts(C.Structure):
    _fields_ = [("ext_init", (_u64 * 16) * 4), ("ext_final", (_u64 * 16) * 4),
                ("internal", _u64 * 22), ("diag15", _u64)]

    def as_arrays(self):
        ei = np.array([[self.ext_init[r][i] for i in range(16)] for r in range(4)], dtype=np.uint64)
        ef = np.array([[self.ext_final[r][i] for i in range(16)] for r in range(4)], dtype=np.uint64)
        it = np.array([self.internal[i] for i in range(22)], dtype=np.uint64)
        return ei, ef, it, int(self.diag15)


class Transcript(C.Structure):
    _fields_ = [("state", C.c_uint8 * 32), ("counter", _u64)]


class Challenger(C.Structure):
    _fields_ = [("kind", C.c_int), ("xs_state", _u64), ("tr", Transcript)]


_lib = None


def lib():
    global _lib
    if _lib is None:
        path = build_oracle.build()
        L = C.CDLL(path)
        sig = {
            "orc_add": (_u64, [_u64, _u64]), "orc_sub": (_u64, [_u64, _u64]),
            "orc_mul": (_u64, [_u64, _u64]), "orc_pow": (_u64, [_u64, _u64]),
            "orc_inv": (_u64, [_u64]), "orc_from_i64": (_u64, [C.c_int64]),
            "orc_two_adic_generator": (_u64, [_u32]),
            "orc_xorshift_init": (_u64, [_u64]), "orc_xorshift_next": (_u64, [_pu64]),
            "orc_xorshift_field": (_u64, [_pu64]),
            "orc_sha256": (None, [C.c_char_p, C.c_size_t, C.c_char_p]),
            "orc_transcript_new": (None, [C.POINTER(Transcript), C.c_char_p, C.c_size_t]),
            "orc_transcript_absorb": (None, [C.POINTER(Transcript), C.c_char_p, C.c_size_t]),
            "orc_transcript_absorb_u64": (None, [C.POINTER(Transcript), _u64]),
            "orc_transcript_field": (_u64, [C.POINTER(Transcript)]),
            "orc_transcript_next_u64": (_u64, [C.POINTER(Transcript)]),
            "orc_dft_batch": (None, [_pu64, _u32, _u64]),
            "orc_dft_naive": (None, [_pu64, _pu64, _u32, _u64]),
            "orc_lde": (None, [_pu64, _pu64, _u32, _u32, _u64]),
            "orc_poly_eval_col": (_u64, [_pu64, _u64, _u64, _u64, _u64]),
            "orc_p2_derive_constants": (None, [_u64, C.POINTER(P2Consts)]),
            "orc_p2_permute": (None, [C.POINTER(P2Consts), _pu64]),
            "orc_p2_hash_row": (None, [C.POINTER(P2Consts), _pu64, _u64, _pu64]),
            "orc_p2_compress": (None, [C.POINTER(P2Consts), _pu64, _pu64, _pu64]),
            "orc_set_lanes": (C.c_int, [C.c_int]),
            "orc_padded_len": (_u64, [_u64, _u64]),
            "orc_merkle_num_layers": (_u32, [_u64]),
            "orc_merkle_total_digests": (_u64, [_u64]),
            "orc_merkle_leaves": (None, [C.POINTER(P2Consts), _pu64, _u64, _u64, _pu64, C.c_int]),
            "orc_merkle_tree": (None, [C.POINTER(P2Consts), _pu64, _u64, _u64, _pu64, _pu64, C.c_int]),
            "orc_merkle_root_from_leaves": (None, [C.POINTER(P2Consts), _pu64, _u64, _pu64]),
            "orc_whir_commit": (None, [C.POINTER(P2Consts), _pu64, _u32, _pu64, _pu64, C.c_int]),
            "orc_mle_eval": (_u64, [_pu64, _u32, _pu64]),
            "orc_mle_partial_eval": (None, [_pu64, _u32, _pu64, _u32, _pu64]),
            "orc_eq_evals": (None, [_pu64, _u32, _pu64]),
            "orc_sumcheck_prove": (None, [_pu64, _pu64, _u32, _pu64, _pu64, _pu64]),
            "orc_sumcheck_verify": (C.c_int, [_pu64, _u32, _u64, _pu64, _u64, _u64]),
            "orc_sumcheck3_prove": (None, [_pu64, _pu64, _pu64, _u32, _pu64, _pu64, _pu64]),
            "orc_sumcheck3_verify": (C.c_int, [_pu64, _u32, _u64, _pu64, _u64, _u64, _u64]),
            "orc_sum_of_products_prove": (None, [_pu64, _pu64, _u32, _u32, _pu64, _pu64, _pu64]),
            "orc_virtual_prove": (None, [_pu64, _u32, _u32, _pu64, _pu32, _pu32, _u32, _pu64, _pu64, _pu64]),
            "orc_virtual_verify": (C.c_int, [_pu64, _u32, _pu64, _pu32, _pu32, _u32, _u64, _pu64, _pu64]),
            "orc_matmul_prove": (None, [_pu64, _pu64, _pu64, _u64, _u64, _u64, _pu64, _pu64, _pu64,
                                        _pu64, _pu64, _pu64]),
            "orc_matmul_field": (None, [_pu64, _pu64, _u64, _u64, _u64, _pu64, C.c_int]),
            "orc_challenger_field": (_u64, [C.POINTER(Challenger)]),
            "orc_op_matmul_prove": (None, [_pu64, _pu64, _pu64, _u64, _u64, _u64, C.POINTER(Challenger),
                                           _pu64, _pu64, _pu64, _pu64, _pu64, _pu64, _pu64]),
            "orc_shard_dag_child": (None, [_pu64, _u32, _u64, _u64, C.POINTER(Transcript)]),
            "orc_set_threads": (None, [C.c_int]),
            "orc_check_witness": (C.c_int, [C.POINTER(P2Consts), _pu64, _pu64, _u32, _u32, _u64]),
            "orc_grind": (_u64, [C.POINTER(P2Consts), _pu64, _pu64, _u32, _u32, _u64, _u64]),
            "orc_fractional_prove": (None, [_pu64, _pu64, _u32, _pu64, _pu64, _pu64, _pu64, _pu64]),
            "orc_fractional_verify": (C.c_int, [_pu64, _pu64, _u32, _pu64, _pu64, _pu64, _u64, _u64, _u64]),
            "orc_fractional_chain_core": (C.c_int, [_u32, _pu64, _pu64, _pu64, _pu64]),
            "orc_lookup_len": (_u64, [_u64, _u64, _u32]),
            "orc_matmul_fixed": (None, [_pu64, _pu64, _u64, _u64, _u64, _pu64]),
            "orc_vec_add": (None, [_pu64, _pu64, _u64, _pu64]),
            "orc_vec_sub": (None, [_pu64, _pu64, _u64, _pu64]),
            "orc_vec_mul": (None, [_pu64, _pu64, _u64, _pu64]),
            "orc_row_sums": (None, [_pu64, _u64, _u64, _u64, _pu64]),
            "orc_lookup_num_den": (_u64, [_pu32, _pu64, _u64, _pu64, _pu64, _u64, _u32, _u64, _u64, _pu64,
                                          _pu64]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def ptr(a):
    assert a.flags["C_CONTIGUOUS"]
    if a.dtype == np.uint32:
        return a.ctypes.data_as(_pu32)
    assert a.dtype == np.uint64, a.dtype
    return a.ctypes.data_as(_pu64)


def u64(a):
    return np.ascontiguousarray(np.asarray(a, dtype=np.uint64))


# ---- field --------------------------------------------------------------------------
def add(a, b): return lib().orc_add(a, b)
def sub(a, b): return lib().orc_sub(a, b)
def mul(a, b): return lib().orc_mul(a, b)
def inv(a): return lib().orc_inv(a)
def from_i64(x): return lib().orc_from_i64(int(x))
def two_adic_generator(bits): return lib().orc_two_adic_generator(bits)


def _vec(fn, a, b):
    a, b = u64(a).reshape(-1), u64(b).reshape(-1)
    if a.size != b.size:
        raise ValueError("field vector lengths differ")
    out = np.zeros(a.size, dtype=np.uint64)
    if a.size:
        fn(ptr(a), ptr(b), a.size, ptr(out))
    return out


def vec_add(a, b): return _vec(lib().orc_vec_add, a, b)
def vec_sub(a, b): return _vec(lib().orc_vec_sub, a, b)
def vec_mul(a, b): return _vec(lib().orc_vec_mul, a, b)


def row_sums(x, m, d, ncols):
    """Field sums of the first ncols entries of each of the m rows (d wide)."""
    xx = u64(x).reshape(-1)
    out = np.zeros(m, dtype=np.uint64)
    if m:
        lib().orc_row_sums(ptr(xx), m, d, ncols, ptr(out))
    return out


# ---- PRNG / transcript --------------------------------------------------------------
class XorShift64:
    """common/field.rs:17-36."""

    def __init__(self, seed):
        self.s = _u64(lib().orc_xorshift_init(seed))

    def next_u64(self):
        return lib().orc_xorshift_next(C.byref(self.s))

    def field(self):
        return lib().orc_xorshift_field(C.byref(self.s))

    def fields(self, n):
        return np.array([self.field() for _ in range(n)], dtype=np.uint64)


def sha256(data: bytes) -> bytes:
    out = C.create_string_buffer(32)
    lib().orc_sha256(data, len(data), out)
    return out.raw


class OracleTranscript:
    """common/transcript.rs:21-80."""

    def __init__(self, domain: bytes = None, raw=None):
        self.t = Transcript()
        if raw is not None:
            C.memmove(C.byref(self.t), C.byref(raw), C.sizeof(Transcript))
        else:
            lib().orc_transcript_new(C.byref(self.t), domain, len(domain))

    def absorb(self, data: bytes):
        lib().orc_transcript_absorb(C.byref(self.t), data, len(data))

    def absorb_u64(self, x):
        lib().orc_transcript_absorb_u64(C.byref(self.t), x)

    def field(self):
        return lib().orc_transcript_field(C.byref(self.t))

    def next_u64(self):
        return lib().orc_transcript_next_u64(C.byref(self.t))

    def state(self):
        return bytes(self.t.state), int(self.t.counter)


# ---- DFT ----------------------------------------------------------------------------
def dft_batch(mat):
    m = u64(mat).copy()
    h = m.shape[0]
    lg = h.bit_length() - 1
    assert h == 1 << lg
    w = m.shape[1] if m.ndim == 2 else 1
    lib().orc_dft_batch(ptr(m), lg, w)
    return m


def dft_naive(mat):
    m = u64(mat)
    h = m.shape[0]
    lg = h.bit_length() - 1
    w = m.shape[1] if m.ndim == 2 else 1
    out = np.zeros_like(m)
    lib().orc_dft_naive(ptr(m), ptr(out), lg, w)
    return out


def lde_rows(coeffs, rows, H):
    """Rows i of the H-row LDE of the L x w coefficient matrix, by Horner."""
    m = u64(coeffs)
    L, w = m.shape
    lg = H.bit_length() - 1
    wH = two_adic_generator(lg)
    out = np.zeros((len(rows), w), dtype=np.uint64)
    for a, i in enumerate(rows):
        x = lib().orc_pow(wH, int(i))
        for c in range(w):
            out[a, c] = lib().orc_poly_eval_col(ptr(m), L, w, c, x)
    return out


def lde(mat, lg_blowup):
    m = u64(mat)
    L = m.shape[0]
    w = m.shape[1]
    out = np.zeros((L << lg_blowup, w), dtype=np.uint64)
    lib().orc_lde(ptr(m), ptr(out), L.bit_length() - 1, lg_blowup, w)
    return out


# ---- Poseidon2 / Merkle -------------------------------------------------------------
def p2_constants(seed=1):
    c = P2Consts()
    lib().orc_p2_derive_constants(seed, C.byref(c))
    return c


def p2_permute(consts, state):
    st = u64(state).copy()
    lib().orc_p2_permute(C.byref(consts), ptr(st))
    return st


def p2_hash_row(consts, row):
    r = u64(row)
    out = np.zeros(8, dtype=np.uint64)
    lib().orc_p2_hash_row(C.byref(consts), ptr(r), r.size, ptr(out))
    return out


def p2_compress(consts, left, right):
    out = np.zeros(8, dtype=np.uint64)
    lib().orc_p2_compress(C.byref(consts), ptr(u64(left)), ptr(u64(right)), ptr(out))
    return out


def set_lanes(lanes=-1):
    """SIMD lanes of the packed DFT and Merkle loops (8 AVX-512F, 4 AVX2, 0
    scalar only; -1 the widest the CPU has); returns the lanes now in use."""
    return int(lib().orc_set_lanes(int(lanes)))


def padded_len(raw, n=2): return lib().orc_padded_len(raw, n)


def merkle_leaves(consts, mat, threads=0):
    m = u64(mat)
    h, w = m.shape
    d = np.zeros((h, 8), dtype=np.uint64)
    lib().orc_merkle_leaves(C.byref(consts), ptr(m), h, w, ptr(d), threads)
    return d


def merkle_tree(consts, mat, threads=0):
    """Returns (list of layers as (len, 8) arrays, root)."""
    m = u64(mat)
    h, w = m.shape
    tot = lib().orc_merkle_total_digests(h)
    layers = np.zeros((tot, 8), dtype=np.uint64)
    root = np.zeros(8, dtype=np.uint64)
    lib().orc_merkle_tree(C.byref(consts), ptr(m), h, w, ptr(layers), ptr(root), threads)
    out, off, ln = [], 0, padded_len(h)
    while True:
        out.append(layers[off:off + ln])
        off += ln
        if ln <= 1:
            break
        ln = padded_len(ln // 2)
    return out, root


def merkle_root_from_leaves(consts, leaves):
    lv = u64(leaves)
    root = np.zeros(8, dtype=np.uint64)
    lib().orc_merkle_root_from_leaves(C.byref(consts), ptr(lv), lv.shape[0], ptr(root))
    return root


def whir_commit(consts, evals, threads=0):
    e = u64(evals)
    n = e.size.bit_length() - 1
    lde_out = np.zeros((1 << (n - 4), 32), dtype=np.uint64)
    root = np.zeros(8, dtype=np.uint64)
    lib().orc_whir_commit(C.byref(consts), ptr(e), n, ptr(lde_out), ptr(root), threads)
    return lde_out, root


def ef_dft_naive(evals_ef, H):
    """The H-point DFT of an extension-field column zero-padded from len(evals)
    to H entries, in extension arithmetic: out[k] = sum_j e_j * W_H^(jk),
    with e_j = (c0, c1) in F[X]/(X^2 - 7) and W_H in F (scalar
    multiplication of both coefficients).  O(H * len), small cases only."""
    e = u64(evals_ef).reshape(-1, 2)
    lg = H.bit_length() - 1
    wh = two_adic_generator(lg)
    out = np.zeros((H, 2), dtype=np.uint64)
    for k in range(H):
        wk = lib().orc_pow(wh, k)
        x, acc0, acc1 = 1, 0, 0
        for j in range(e.shape[0]):
            acc0 = add(acc0, mul(int(e[j, 0]), x))
            acc1 = add(acc1, mul(int(e[j, 1]), x))
            x = mul(x, wk)
        out[k] = (acc0, acc1)
    return out


def commit_extension(consts, evals_ef, log_inv_rate, threads=0):
    """commit_extension (vendor/p3-whir/src/pcs/committer/writer.rs:21-86,
    Suffix order): 2^n EF evaluations (rows of (c0, c1)) fill the first
    2^(n-5) rows of the (2^(n-5) << log_inv_rate) x 32 EF matrix, each EF
    column is DFT'd (dft_algebra_batch: coefficient-wise, the twiddles being
    base-field elements), and the tree hashes each row's 64 base coefficients
    (ExtensionMmcs over FlatMatrixView).  Returns (encoding as H x 64, root)."""
    e = u64(evals_ef).reshape(-1)
    n = (e.size // 2).bit_length() - 1
    mat = e.reshape(1 << (n - 5), 64)
    enc = lde(mat, log_inv_rate)
    _, root = merkle_tree(consts, enc, threads)
    return enc, root


# ---- MLE / sumcheck -----------------------------------------------------------------
def mle_eval(values, point):
    v, pt = u64(values), u64(point)
    return lib().orc_mle_eval(ptr(v), pt.size, ptr(pt) if pt.size else None)


def mle_partial_eval(values, fix):
    v, fx = u64(values), u64(fix)
    t = v.size.bit_length() - 1
    out = np.zeros(v.size >> fx.size, dtype=np.uint64)
    lib().orc_mle_partial_eval(ptr(v), t, ptr(fx) if fx.size else None, fx.size, ptr(out))
    return out


def eq_evals(r):
    rr = u64(r)
    out = np.zeros(1 << rr.size, dtype=np.uint64)
    lib().orc_eq_evals(ptr(rr) if rr.size else None, rr.size, ptr(out))
    return out


def sumcheck_prove(f, h, ch):
    f, h, ch = u64(f), u64(h), u64(ch)
    t = ch.size
    rounds = np.zeros((max(t, 1), 3), dtype=np.uint64)
    finals = np.zeros(2, dtype=np.uint64)
    lib().orc_sumcheck_prove(ptr(f), ptr(h), t, ptr(ch) if t else None, ptr(rounds), ptr(finals))
    return rounds[:t], finals


def sumcheck_verify(rounds, claimed, ch, f_eval, h_eval):
    r, ch = u64(rounds).reshape(-1, 3), u64(ch)
    return bool(lib().orc_sumcheck_verify(ptr(r), ch.size, claimed, ptr(ch) if ch.size else None, f_eval, h_eval))


def sumcheck3_prove(f, g, h, ch):
    f, g, h, ch = u64(f), u64(g), u64(h), u64(ch)
    rounds = np.zeros((max(ch.size, 1), 4), dtype=np.uint64)
    finals = np.zeros(3, dtype=np.uint64)
    lib().orc_sumcheck3_prove(ptr(f), ptr(g), ptr(h), ch.size, ptr(ch), ptr(rounds), ptr(finals))
    return rounds[:ch.size], finals


def sumcheck3_verify(rounds, claimed, ch, fe, ge, he):
    r, ch = u64(rounds).reshape(-1, 4), u64(ch)
    return bool(lib().orc_sumcheck3_verify(ptr(r), ch.size, claimed, ptr(ch), fe, ge, he))


def sum_of_products_prove(weights, values, ch):
    w, v, ch = u64(weights), u64(values), u64(ch)
    nt = w.shape[0]
    rounds = np.zeros((max(ch.size, 1), 3), dtype=np.uint64)
    be = _u64(0)
    lib().orc_sum_of_products_prove(ptr(w), ptr(v), nt, ch.size, ptr(ch), ptr(rounds), C.byref(be))
    return rounds[:ch.size], be.value


def _terms(terms):
    coeffs = u64([c for c, _ in terms])
    off = [0]
    idx = []
    for _, ids in terms:
        idx.extend(ids)
        off.append(len(idx))
    return coeffs, np.array(off, dtype=np.uint32), np.array(idx if idx else [0], dtype=np.uint32)


def virtual_prove(mles, terms, ch):
    m = u64(mles)
    ch = u64(ch)
    coeffs, off, idx = _terms(terms)
    max_deg = max((len(ids) for _, ids in terms), default=0)
    rounds = np.zeros((max(ch.size, 1), max_deg + 1), dtype=np.uint64)
    finals = np.zeros(m.shape[0], dtype=np.uint64)
    lib().orc_virtual_prove(ptr(m), m.shape[0], ch.size, ptr(coeffs), ptr(off), ptr(idx), len(terms),
                            ptr(ch), ptr(rounds), ptr(finals))
    return rounds[:ch.size], finals


def virtual_verify(rounds, terms, claimed, ch, finals):
    r, ch, fin = u64(rounds), u64(ch), u64(finals)
    coeffs, off, idx = _terms(terms)
    return bool(lib().orc_virtual_verify(ptr(np.ascontiguousarray(r)), ch.size, ptr(coeffs), ptr(off), ptr(idx),
                                         len(terms), claimed, ptr(ch), ptr(fin)))


def matmul_field(a, b):
    a, b = u64(a), u64(b)
    m, k = a.shape
    n = b.shape[1]
    c = np.zeros((m, n), dtype=np.uint64)
    lib().orc_matmul_field(ptr(a), ptr(b), m, k, n, ptr(c), 0)
    return c


def matmul_fixed(a, b):
    """par::mm_par_fixed: the same field product as matmul_field, in i64 when it fits."""
    a, b = u64(a), u64(b)
    m, k = a.shape
    n = b.shape[1]
    c = np.zeros((m, n), dtype=np.uint64)
    lib().orc_matmul_fixed(ptr(a), ptr(b), m, k, n, ptr(c))
    return c


def matmul_prove(at, b, c, m, k, n, u, v, ch):
    at, b, c, u, v, ch = map(u64, (at, b, c, u, v, ch))
    claimed = _u64(0)
    rounds = np.zeros((max(ch.size, 1), 3), dtype=np.uint64)
    finals = np.zeros(2, dtype=np.uint64)
    lib().orc_matmul_prove(ptr(at), ptr(b), ptr(c), m, k, n, ptr(u) if u.size else None,
                           ptr(v) if v.size else None, ptr(ch) if ch.size else None,
                           C.byref(claimed), ptr(rounds), ptr(finals))
    return claimed.value, rounds[:ch.size], finals


def op_matmul_prove(a, b, c, m, k, n, challenger):
    """Op::MatMul arm.  challenger: XorShift64 or OracleTranscript (advanced in place)."""
    a, b, c = u64(a), u64(b), u64(c)
    ch_obj = Challenger()
    if isinstance(challenger, XorShift64):
        ch_obj.kind = 0
        ch_obj.xs_state = challenger.s.value
    else:
        ch_obj.kind = 1
        C.memmove(C.byref(ch_obj.tr), C.byref(challenger.t), C.sizeof(Transcript))
    lm, lk, ln = (m.bit_length() - 1, k.bit_length() - 1, n.bit_length() - 1)
    u = np.zeros(max(lm, 1), dtype=np.uint64)
    v = np.zeros(max(ln, 1), dtype=np.uint64)
    chv = np.zeros(max(lk, 1), dtype=np.uint64)
    claimed = _u64(0)
    rounds = np.zeros((max(lk, 1), 3), dtype=np.uint64)
    finals = np.zeros(2, dtype=np.uint64)
    claims = np.zeros(3, dtype=np.uint64)
    lib().orc_op_matmul_prove(ptr(a), ptr(b), ptr(c), m, k, n, C.byref(ch_obj), ptr(u), ptr(v), ptr(chv),
                              C.byref(claimed), ptr(rounds), ptr(finals), ptr(claims))
    if isinstance(challenger, XorShift64):
        challenger.s.value = ch_obj.xs_state
    else:
        C.memmove(C.byref(challenger.t), C.byref(ch_obj.tr), C.sizeof(Transcript))
    return dict(u=u[:lm], v=v[:ln], ch=chv[:lk], claimed=claimed.value, rounds=rounds[:lk],
                finals=finals, claims=claims)


def shard_dag_child(op_ids, ops_per_shard, shard_index):
    ids = u64(op_ids).reshape(-1)
    t = OracleTranscript(b"x")
    lib().orc_shard_dag_child(ptr(ids), ids.size // 3, ops_per_shard, shard_index, C.byref(t.t))
    return t


# ---- logUp GKR fraction tree (logup_gkr.rs:29-164, 210-301) ---------------------------
def fractional_prove(num, den, full_r, cs):
    """-> (rounds: list of (t_l, 4) arrays, finals: (lg, 7), final_num, final_den)."""
    nm, dn, fr, c = u64(num), u64(den), u64(full_r), u64(cs)
    lg = nm.size.bit_length() - 1
    rounds = np.zeros(max(2 * lg * (lg - 1), 1), dtype=np.uint64)
    finals = np.zeros(max(7 * lg, 1), dtype=np.uint64)
    fnd = np.zeros(2, dtype=np.uint64)
    lib().orc_fractional_prove(ptr(nm), ptr(dn), lg, ptr(fr) if fr.size else None, ptr(c) if c.size else None,
                               ptr(rounds), ptr(finals), ptr(fnd))
    out, off = [], 0
    for layer in range(lg):
        t = lg - layer - 1
        out.append(rounds[off:off + 4 * t].reshape(t, 4).copy())
        off += 4 * t
    return out, finals[:7 * lg].reshape(lg, 7).copy(), int(fnd[0]), int(fnd[1])


def _flat_rounds(rounds):
    parts = [np.asarray(r, dtype=np.uint64).reshape(-1) for r in rounds]
    flat = np.concatenate(parts) if parts else np.zeros(0, dtype=np.uint64)
    return np.ascontiguousarray(flat if flat.size else np.zeros(1, dtype=np.uint64))


def fractional_verify(num, den, full_r, cs, rounds, final_num, final_den, claimed):
    nm, dn, fr, c = u64(num), u64(den), u64(full_r), u64(cs)
    lg = nm.size.bit_length() - 1
    rf = _flat_rounds(rounds)
    return bool(lib().orc_fractional_verify(ptr(nm), ptr(dn), lg, ptr(fr) if fr.size else None,
                                            ptr(c) if c.size else None, ptr(rf), final_num, final_den, claimed))


def fractional_chain_core(full_r, cs, rounds, finals):
    fr, c = u64(full_r), u64(cs)
    fin = np.ascontiguousarray(np.asarray(finals, dtype=np.uint64).reshape(-1))
    rf = _flat_rounds(rounds)
    return bool(lib().orc_fractional_chain_core(fr.size, ptr(fr) if fr.size else None, ptr(c) if c.size else None,
                                                ptr(rf), ptr(fin) if fin.size else None))


def lookup_num_den(x, y, table, m, mode, alpha, beta):
    """mode 0 merged, 1 witness, 2 witness columns, 3 table; None if an index
    is outside the table."""
    xx = np.ascontiguousarray(np.asarray(x if x is not None else [], dtype=np.uint32).reshape(-1))
    yy, tb = u64(y if y is not None else []), u64(table if table is not None else [])
    mm = u64(m if m is not None else [])
    n = xx.size if mode != 3 else 0
    total = lib().orc_lookup_len(n, tb.size, mode)
    num = np.zeros(total, dtype=np.uint64)
    den = np.zeros(total, dtype=np.uint64)
    got = lib().orc_lookup_num_den(xx.ctypes.data_as(_pu32) if xx.size else None, ptr(yy) if yy.size else None, n,
                                   ptr(tb) if tb.size else None, ptr(mm) if mm.size else None, tb.size, mode,
                                   int(alpha) % P, int(beta) % P, ptr(num), ptr(den))
    return (num, den) if got else None


# ---- projection block (crates/zkie-ops/src/projection.rs) -------------------------------
def to_i64(v):
    """fixed_point.rs to_i64."""
    v = int(v) % P
    return v if v <= 0x7FFFFFFFFFFFFFFF else -(P - v)


def to_i32_index(v):
    """to_i32(v) as u32 (fixed_point.rs): the low 32 bits of (P - v), negated."""
    v = int(v) % P
    if v <= 0x7FFFFFFF:
        return v
    return (-((P - v) & 0xFFFFFFFF)) & 0xFFFFFFFF


def to_i32_indices(v):
    """to_i32_index over an array (numpy, u32)."""
    v = u64(v).reshape(-1) % np.uint64(P)
    small = v <= np.uint64(0x7FFFFFFF)
    low = ((np.uint64(P) - v) & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    return np.where(small, v.astype(np.uint32), (np.uint32(0) - low).astype(np.uint32)).astype(np.uint32)


def projection_terms(shift):
    """prove_projection's terms over [eq, rem_off, h, out, bias, ones] (:71-81)."""
    two, half, neg = 1 << shift, 1 << (shift - 1), P - 1
    return [(1, [0, 1]), (neg, [0, 2]), (two, [0, 3]), (neg * two % P, [0, 4]), (neg * half % P, [0, 5])]


def projection_witness(h, bias, shift):
    """out and rem_off as the reference's tests build them (:136-176):
    out = div_round(to_i64(h), 2^shift) + to_i64(bias), rem_off = h - (out - bias)
    2^shift + 2^(shift-1), with div_round = floor plus one at remainder >= half."""
    out, rem = [], []
    for hv, bv in zip(np.asarray(h, dtype=np.uint64).reshape(-1), np.asarray(bias, dtype=np.uint64).reshape(-1)):
        a, b = to_i64(hv), to_i64(bv)
        q, r = divmod(a, 1 << shift)
        if 2 * r >= (1 << shift):
            q += 1
        o = q + b
        out.append(from_i64(o))
        rem.append(from_i64(a - (o - b) * (1 << shift) + (1 << (shift - 1))))
    return np.array(out, dtype=np.uint64), np.array(rem, dtype=np.uint64)


def projection_prove(x, w, bias, out, rem_off, m, k, n, shift, challenger):
    """prove_projection (projection.rs:44-101) over the oracle's parts: h = x w,
    matmul::prove(x^T, w, h) with u, v, ch drawn in that order (the Op::MatMul
    draw order), prove_virtual over [eq(v||u), rem_off, h, out, bias, ones],
    then alpha, beta and prove_lookup_fractional of (to_i32(rem_off) as u32,
    rem_off) into the table 0 .. 2^shift - 1 (full_r then cs per variable)."""
    x = u64(x).reshape(m, k)
    w = u64(w).reshape(k, n)
    h = matmul_fixed(x, w).reshape(-1)
    op = op_matmul_prove(x, w, h.reshape(m, n), m, k, n, challenger)
    pt = np.concatenate([op["v"], op["u"]]).astype(np.uint64)
    eq = eq_evals(pt)
    ones = np.ones(m * n, dtype=np.uint64)
    rem = u64(rem_off).reshape(-1)
    a_rounds, a_finals = virtual_prove([eq, rem, h, u64(out).reshape(-1), u64(bias).reshape(-1), ones],
                                       projection_terms(shift), pt)
    alpha, beta = challenger.field(), challenger.field()
    table = np.arange(1 << shift, dtype=np.uint64)
    idx = to_i32_indices(rem)
    num, den = lookup_num_den(idx, rem, table, None, 0, alpha, beta)
    lg = num.size.bit_length() - 1
    full_r = [challenger.field() for _ in range(lg)]
    cs = [challenger.field() for _ in range(lg)]
    f_rounds, f_finals, fnum, fden = fractional_prove(num, den, full_r, cs)
    return dict(h=h, claimed=op["claimed"], mm_rounds=op["rounds"], mm_finals=op["finals"], u=op["u"], v=op["v"],
                ch=op["ch"], pt=pt, affine_rounds=a_rounds, affine_finals=a_finals, alpha=alpha, beta=beta,
                full_r=np.array(full_r, dtype=np.uint64), cs=np.array(cs, dtype=np.uint64), frac_rounds=f_rounds,
                frac_finals=f_finals, final_num=fnum, final_den=fden)


def projection_verify(proof, shift):
    """verify_projection (projection.rs:102-128): the affine virtual sumcheck
    with h's final evaluation replaced by the matmul claim, the matmul
    sumcheck, and the lookup's fraction chain with claimed sum 0."""
    fe = np.array(proof["affine_finals"], dtype=np.uint64).copy()
    fe[2] = np.uint64(proof["claimed"])
    if not virtual_verify(proof["affine_rounds"], projection_terms(shift), 0, proof["pt"], fe):
        return False
    f_eval, h_eval = (int(v) for v in proof["mm_finals"])
    if not sumcheck_verify(proof["mm_rounds"], proof["claimed"], proof["ch"], f_eval, h_eval):
        return False
    return (fractional_chain_core(proof["full_r"], proof["cs"], proof["frac_rounds"], proof["frac_finals"])
            and proof["final_num"] == 0)


# ---- PoW grinding (DuplexChallenger<Goldilocks, Poseidon2-16, 16, 8>) --------------------
def check_witness(consts, sponge, inputs, bits, w):
    sp, inp = u64(sponge), u64(inputs if len(inputs) else [0])
    return bool(lib().orc_check_witness(C.byref(consts), ptr(sp), ptr(inp), len(inputs), bits, w))


def grind(consts, sponge, inputs, bits, start=0, limit=1 << 40):
    """Smallest valid witness >= start (None if none below start + limit)."""
    sp, inp = u64(sponge), u64(inputs if len(inputs) else [0])
    w = lib().orc_grind(C.byref(consts), ptr(sp), ptr(inp), len(inputs), bits, start, limit)
    return None if w == 0xFFFFFFFFFFFFFFFF else int(w)


def set_threads(n):
    """OpenMP threads of the oracle's parallel loops."""
    lib().orc_set_threads(int(n))
