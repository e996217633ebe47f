"""zkie_b200: the zkIE prover hot path (shard commit + matmul GKR sumcheck)
as hand-written sm_100a CUDA kernels behind a C ABI (libzkie_b200.so).

The package is a thin host-side mirror of the reference's Rust interface; all
compute runs in the shared object.  Importing fails if the shared object is
missing -- there is no CPU fallback.
"""
from ._lib import LIB_PATH, ZkieError, check, lib  # noqa: F401
from .commit import (  # noqa: F401
    Committed, CudaDft, CudaMerkleTreeMmcs, MerkleTree, Whir, commit, commit_cosets, commit_host, init_default_constants,
    make_twiddles, merkle_layer_lengths, p2_default_constants, padded_len, split_layers, upload_constants)
from .device import P  # noqa: F401
from .gkr import (  # noqa: F401
    MatmulProof, OpMatMulProof, SumcheckProof, SumcheckProofBatch, Transcript, VirtualProof, XorShift64, eq_evals,
    matmul_field, matmul_fixed, matmul_prove, mle_eval, mle_partial_eval, op_matmul_prove, prove_sum_of_products, prove_virtual,
    sha256, shard_dag_child, sumcheck_prove)
from .gkr import ShardMatMulProof, ShardProver  # noqa: F401
from .cache import BatchCacheMetadata, header_bytes, read_cache, read_header, write_cache  # noqa: F401
from .pow import grind  # noqa: F401
from .proofbytes import from_bincode, to_bincode  # noqa: F401
from .logup import (  # noqa: F401
    FractionalLayer, FractionalProof, build_lookup_num_den, build_lookup_table_num_den, build_lookup_witness_num_den,
    fractional_leaf, lookup_multiplicity, merge_multiplicity, pad_table, prove_fractional,
    prove_fractional_with_challenges, prove_lookup_fractional, prove_lookup_fractional_batch,
    prove_lookup_fractional_columns, prove_lookup_table, prove_lookup_witness, prove_lookup_witness_batch,
    prove_lookup_witness_batch_columns)
from . import compose, gpt2, projection  # noqa: F401,E402
