"""ctypes binding of libzkie_b200.so: every symbol declared in include/*.h.

The shared object is built in-tree by zkie_b200/build.py.  There is no
fallback: if it is missing or fails to load, importing this module raises.
"""
import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libzkie_b200.so")

u64, u32, i32, i64 = C.c_uint64, C.c_uint32, C.c_int32, C.c_int
s64 = C.c_int64
pu64 = C.POINTER(C.c_uint64)
pu32 = C.POINTER(C.c_uint32)
vp = C.c_void_p  # device pointers and streams travel as integers
sz = C.c_size_t


class Transcript(C.Structure):
    _fields_ = [("state", C.c_uint8 * 32), ("counter", C.c_uint64)]


class Challenger(C.Structure):
    _fields_ = [("kind", C.c_int32), ("xorshift_state", C.c_uint64), ("transcript", Transcript)]


PTr = C.POINTER(Transcript)
PCh = C.POINTER(Challenger)

# name -> (restype, argtypes); one entry per declaration in include/*.h
SIGNATURES = {
    # include/zkie_goldilocks_cuda.h (reference symbols)
    "zkie_cuda_device_count": (i64, []),
    "zkie_ntt_forward_goldilocks": (i64, [vp, vp, u32, u64, vp]),
    "zkie_p2_upload_constants": (i64, [pu64, pu64, pu64, u64]),
    "zkie_p2_leaf_batch": (i64, [vp, vp, u32, u32]),
    "zkie_p2_leaf_scalar": (i64, [vp, vp, u32, u32, u32]),
    "zkie_p2_compress_batch": (i64, [vp, vp, u32, u32]),
    "zkie_p2_compress_scalar": (i64, [vp, vp, u32, u32, u32]),
    # include/zkie2.h
    "zkie2_p2_default_constants": (i64, [u64, pu64, pu64, pu64, pu64]),
    "zkie2_p2_init_default": (i64, []),
    "zkie2_p2_permute": (i64, [vp, u64, u32, vp]),
    "zkie2_gl_mul_probe": (i64, [vp, u64, u32, vp]),
    "zkie2_lde_scratch_elems": (u64, [u32, u32, u64]),
    "zkie2_lde": (i64, [vp, vp, vp, u32, u32, u64, vp]),
    "zkie2_dft_twiddles": (i64, [u32, pu64]),
    "zkie2_dft": (i64, [vp, vp, vp, u32, u64, vp]),
    "zkie2_lde_coset_scratch_elems": (u64, [u32, u32, u64, u32]),
    "zkie2_lde_coset": (i64, [vp, vp, vp, u32, u32, u64, u32, u64, vp]),
    "zkie2_merkle_total_digests": (u64, [u64]),
    "zkie2_merkle_num_layers": (u32, [u64]),
    "zkie2_merkle_leaves": (i64, [vp, u64, u64, vp, vp]),
    "zkie2_merkle_tree": (i64, [vp, u64, u64, vp, vp]),
    "zkie2_merkle_tree_from_leaves": (i64, [u64, vp, vp]),
    "zkie2_digests_interleave": (i64, [vp, u64, u64, vp, vp]),
    "zkie2_commit_scratch_elems": (u64, [u32, u32, u64]),
    "zkie2_commit": (i64, [vp, u32, u32, u64, vp, vp, vp, vp]),
    "zkie2_whir_scratch_elems": (u64, [u32]),
    "zkie2_whir_commit": (i64, [vp, u32, vp, vp, vp, vp]),
    "zkie2_commit_extension_scratch_elems": (u64, [u32, u32]),
    "zkie2_commit_extension": (i64, [vp, u32, u32, vp, vp, vp, vp]),
    "zkie2_commit_cosets_scratch_elems": (u64, [u32, u32, u64, u32]),
    "zkie2_commit_cosets": (i64, [vp, u32, u32, u64, u32, vp, vp, vp]),
    "zkie2_commit_host": (i64, [vp, u32, u32, u64, vp, vp, vp]),
    "zkie2_sha256": (None, [C.c_char_p, sz, C.c_char_p]),
    "zkie2_transcript_new": (None, [PTr, C.c_char_p, sz]),
    "zkie2_transcript_absorb": (None, [PTr, C.c_char_p, sz]),
    "zkie2_transcript_absorb_u64": (None, [PTr, u64]),
    "zkie2_transcript_field": (u64, [PTr]),
    "zkie2_transcript_next_u64": (u64, [PTr]),
    "zkie2_challenger_xorshift": (None, [PCh, u64]),
    "zkie2_challenger_field": (u64, [PCh]),
    "zkie2_shard_dag_child": (None, [pu64, u32, u64, u64, PCh]),
    "zkie2_eq_evals": (i64, [pu64, u32, vp, vp]),
    "zkie2_mle_scratch_elems": (u64, [u32]),
    "zkie2_mle_partial_eval": (i64, [vp, u32, pu64, u32, vp, vp, vp]),
    "zkie2_mle_eval": (i64, [vp, u32, pu64, pu64, vp, vp]),
    "zkie2_sumcheck_scratch_elems": (u64, [u32]),
    "zkie2_sumcheck_prove": (i64, [vp, vp, u32, pu64, pu64, pu64, vp, vp]),
    "zkie2_sumcheck_noalloc_max_vars": (u32, []),
    "zkie2_sumcheck_prove_noalloc": (i64, [vp, vp, u32, pu64, pu64, pu64, vp]),
    "zkie2_matmul_scratch_elems": (u64, [u64, u64, u64]),
    "zkie2_matmul_prove": (i64, [vp, vp, vp, u64, u64, u64, pu64, pu64, pu64, pu64, pu64, pu64, vp, vp]),
    "zkie2_op_matmul_scratch_elems": (u64, [u64, u64, u64]),
    "zkie2_op_matmul_prove": (i64, [vp, vp, vp, u64, u64, u64, PCh, pu64, pu64, pu64, pu64, pu64, pu64,
                                    pu64, vp, vp]),
    "zkie2_matmul_field": (i64, [vp, vp, u64, u64, u64, vp, vp]),
    "zkie2_matmul_fixed_scratch_elems": (u64, [u64, u64, u64]),
    "zkie2_projection_witness": (i64, [vp, vp, u64, u32, vp, vp, vp, vp]),
    "zkie2_lookup_index_i32": (i64, [vp, u64, vp, vp]),
    "zkie2_projection_lookup_vars": (u32, [u64, u64, u32]),
    "zkie2_projection_scratch_elems": (u64, [u64, u64, u64, u32]),
    "zkie2_projection_prove": (i64, [vp, vp, vp, vp, vp, vp, u64, u64, u64, u32, PCh, pu64, pu64, pu64, pu64, pu64,
                                     pu64, pu64, pu64, pu64, pu64, pu64, pu64, pu64, pu64, vp, vp]),
    "zkie2_matmul_fixed": (i64, [vp, vp, u64, u64, u64, vp, u32, pu32, vp, vp]),
    "zkie2_shard_prove_matmul_scratch_elems": (u64, [u64, u64, u64]),
    "zkie2_shard_prove_matmul": (i64, [vp, vp, u64, u64, u64, pu64, u64, u64, vp, pu64, pu64, pu64, pu64, pu64,
                                       vp, vp]),
    "zkie2_sum_of_products_scratch_elems": (u64, [u32, u32]),
    "zkie2_sum_of_products_prove": (i64, [vp, vp, u32, u32, pu64, pu64, pu64, vp, vp]),
    "zkie2_virtual_scratch_elems": (u64, [u32, u32]),
    "zkie2_virtual_prove": (i64, [C.POINTER(vp), u32, u32, pu64, pu32, pu32, u32, pu64, pu64, pu64, vp, vp]),
    "zkie2_grind_batch": (u64, [u32]),
    "zkie2_grind": (i64, [pu64, pu64, u32, u32, pu64, vp]),
    "zkie2_cache_header": (u64, [C.c_char_p, C.c_char_p, C.POINTER(C.c_char_p), u32, u32, u32, u32, C.c_char_p, pu64,
                                  C.c_char_p, u64]),
    "zkie2_cache_write": (i64, [C.c_char_p, C.c_char_p, u64, vp, u64, u64, vp, vp]),
    "zkie2_cache_read": (i64, [C.c_char_p, u64, u64, u64, vp, vp, vp]),
    "zkie2_fractional_scratch_elems": (u64, [u32]),
    "zkie2_fractional_prove": (i64, [vp, vp, u32, pu64, pu64, pu64, pu64, pu64, vp, vp]),
    "zkie2_lookup_len": (u64, [u64, u64, u32]),
    "zkie2_lookup_scratch_elems": (u64, [u64]),
    "zkie2_lookup_num_den": (i64, [vp, vp, u64, vp, vp, u64, u32, u64, u64, vp, vp, vp, vp]),
    "zkie2_xorshift_fill": (None, [pu64, u64, u64, s64, pu64]),
    "zkie2_mle_eval_async": (i64, [vp, u32, pu64, vp, vp, vp]),
    "zkie2_mle_eval_many_scratch_elems": (u64, [u32]),
    "zkie2_mle_eval_many": (i64, [C.POINTER(vp), pu32, pu64, u32, vp, vp, vp]),
    "zkie2_challenger_fields": (None, [PCh, u64, pu64]),
    "zkie2_transcript_fields": (None, [PTr, u64, pu64]),
    "zkie2_op_matmul_prove_async": (i64, [vp, vp, vp, u64, u64, u64, pu64, pu64, pu64, vp, vp, vp]),
    "zkie2_projection_proof_elems": (u64, [u64, u64, u64, u32]),
    "zkie2_projection_prove_async": (i64, [vp, vp, vp, vp, vp, vp, u64, u64, u64, u32, pu64, pu64, pu64, u64, u64,
                                           pu64, pu64, vp, vp, vp, vp]),
    "zkie2_virtual_prove_async": (i64, [C.POINTER(vp), u32, u32, pu64, pu32, pu32, u32, pu64, vp, vp, vp, vp]),
    "zkie2_fractional_proof_elems": (u64, [u32]),
    "zkie2_fractional_prove_async": (i64, [vp, vp, u32, pu64, pu64, vp, vp, vp]),
    "zkie2_lookup_num_den_async": (i64, [vp, vp, u64, vp, vp, u64, u32, u64, u64, vp, vp, vp, vp, vp]),
    "zkie2_lookup_multiplicity": (i64, [vp, u64, u64, vp, i64, vp, vp]),
    "zkie2_op_add": (i64, [vp, vp, u64, vp, vp]),
    "zkie2_op_scale": (i64, [vp, u64, s64, u32, vp, vp]),
    "zkie2_op_transpose": (i64, [vp, u64, u64, vp, vp]),
    "zkie2_op_softmax_index": (i64, [vp, u64, u64, vp, vp]),
    "zkie2_op_gelu_index": (i64, [vp, u64, s64, u64, vp, vp]),
    "zkie2_op_stable_softmax_index": (i64, [vp, vp, u64, u64, s64, u64, vp, vp]),
    "zkie2_op_lookup": (i64, [vp, u64, vp, u64, vp, vp, vp]),
    "zkie2_op_softmax": (i64, [vp, vp, u64, u64, u64, vp, vp, vp, vp, vp]),
    "zkie2_op_softmax_rem": (i64, [vp, vp, vp, u64, u64, vp, vp, vp]),
    "zkie2_op_layer_norm_centered": (i64, [vp, vp, vp, vp, u64, u64, u64, u64, C.POINTER(vp), vp, vp, vp]),
    "zkie2_op_layernorm": (i64, [vp, vp, vp, vp, u64, u64, u64, vp, vp, vp, vp, vp, vp]),
    "zkie2_op_row_broadcast": (i64, [vp, u64, u64, vp, vp]),
    "zkie2_op_row_sums": (i64, [vp, u64, u64, u64, vp, vp]),
    "zkie2_op_fill": (i64, [vp, u64, u64, vp]),
    "zkie2_op_iota": (i64, [vp, u64, vp]),
    "zkie2_op_topk": (i64, [vp, u64, u64, u64, vp, vp, vp, vp, vp, vp, vp]),
    "zkie2_op_topk_limbs": (i64, [vp, vp, vp, u64, vp, vp, vp, vp, vp]),
    "zkie2_op_rms_norm": (i64, [vp, vp, vp, u64, u64, u64, u64, vp, vp, vp, vp]),
    "zkie2_op_scale_vec": (i64, [vp, u64, vp, u64, u32, vp, vp]),
    "zkie2_matmul_fixed_runs_scratch_elems": (u64, [u64, u64, u64]),
    "zkie2_matmul_fixed_ex": (i64, [vp, vp, u64, u64, u64, vp, u32, pu32, vp, vp]),
    "zkie2_matmul_fixed_planned": (i64, [vp, vp, u64, u64, u64, vp, pu32, vp, vp, vp]),
    "zkie2_matmul_fixed_runs": (i64, [vp, vp, u64, u64, u64, pu64, u64, vp, vp, vp]),
    "zkie2_op_scale_gate": (i64, [vp, u64, vp, u64, u64, u64, u64, u32, vp, vp]),
    "zkie2_op_relu": (i64, [vp, u64, vp, vp]),
    "zkie2_op_batched_matmul": (i64, [vp, vp, u64, u64, u64, vp, vp]),
    "zkie2_op_broadcast_scale": (i64, [vp, u64, vp, u64, u64, vp, vp]),
    "zkie2_op_idx_broadcast": (i64, [vp, u64, u32, vp, vp]),
    "zkie2_op_combine_idx": (i64, [vp, vp, u64, u32, vp, vp]),
    "zkie2_op_pad_idx": (i64, [vp, u64, u64, vp, vp]),
    "zkie2_op_rope": (i64, [vp, u64, vp, vp, u64, u64, u32, vp, vp]),
    "zkie2_op_rope_columns": (i64, [vp, vp, u64, vp, vp, u64, u64, u32, vp, vp]),
    "zkie2_op_sel_counts": (i64, [vp, u64, u64, u32, vp, vp]),
    "zkie2_op_scatter": (i64, [vp, u64, u64, vp, vp, vp, vp, vp]),
    "zkie2_op_scatter_encodings": (i64, [vp, u64, u64, vp, vp, vp, u64, vp, vp, vp, vp, vp]),
    "zkie2_perm_num_den": (i64, [vp, u64, u64, u64, vp, vp, vp]),
    "zkie2_op_gather_scratch_u32": (u64, [u64, u64]),
    "zkie2_op_gather": (i64, [vp, vp, vp, u64, u64, u64, vp, vp, vp, vp]),
    "zkie2_scatter_add_columns": (i64, [vp, vp, vp, vp, u64, u64, u64, u64, vp, vp]),
    "zkie2_expert_rows": (i64, [vp, vp, u64, u64, u64, vp, vp, vp]),
    "zkie2_expert_open": (i64, [vp, u64, vp, vp, u64, vp, u64, vp, vp, vp]),
    "zkie2_eq_combine_scratch_elems": (u64, [u32, u32]),
    "zkie2_eq_combine": (i64, [pu64, pu64, u32, u32, vp, vp, vp]),
    "zkie2_mg_available": (i64, []),
    "zkie2_mg_unique_id": (i64, [C.c_char_p]),
    "zkie2_mg_init": (i64, [C.c_char_p, i64, i64, C.POINTER(vp)]),
    "zkie2_mg_init_comm": (i64, [vp, C.POINTER(vp)]),
    "zkie2_mg_destroy": (i64, [vp]),
    "zkie2_mg_rank": (i64, [vp]),
    "zkie2_mg_size": (i64, [vp]),
    "zkie2_mg_split_commit_scratch_elems": (u64, [u32, u32, u64, i64]),
    "zkie2_mg_top_digests": (u64, [i64]),
    "zkie2_mg_split_commit": (i64, [vp, vp, u32, u32, u64, vp, vp, vp, vp, pu64, vp]),
    "zkie2_mg_split_commit_host_scratch_elems": (u64, [u32, u32, u64, i64]),
    "zkie2_mg_split_commit_host": (i64, [vp, vp, u32, u32, u64, vp, vp, pu64, vp]),
    "zkie2_mg_split_sumcheck_scratch_elems": (u64, [u32, i64]),
    "zkie2_mg_split_sumcheck": (i64, [vp, vp, vp, u32, pu64, pu64, pu64, vp, vp]),
}

if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is missing: build it with `python -m zkie_b200.build` "
                      "(there is no CPU fallback)")

lib = C.CDLL(LIB_PATH)
for _name, (_res, _args) in SIGNATURES.items():
    _f = getattr(lib, _name)
    _f.restype = _res
    _f.argtypes = _args


class ZkieError(RuntimeError):
    pass


def check(rc: int, what: str):
    if rc != 0:
        raise ZkieError(f"{what} failed with CUDA error {rc}")
