/*
 * zkie2.h -- additive entry points of libzkie_b200.so (sm_100a).
 *
 * Conventions (same as zkie_goldilocks_cuda.h unless stated): plain pointers
 * and sizes; d_* are device pointers owned by the caller, h_* host pointers;
 * every int-returning call returns a cudaError_t (0 = success) and never
 * falls back to a CPU path; work is enqueued on the explicit stream argument
 * (NULL = legacy default stream) on the current device.  Scratch buffers are
 * supplied by the caller, sized by the matching *_scratch_elems() query (in
 * u64 elements).  Outputs are canonical Goldilocks elements.
 *
 * Reference functions replaced are cited as file:line of trustless-ai/zkIE.
 */
#ifndef ZKIE2_H
#define ZKIE2_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

struct CUstream_st;
typedef struct CUstream_st *zkie_stream_t; /* ABI-identical to cudaStream_t */

/* ---- Poseidon2 constants ---------------------------------------------------- */

/* Round constants of Perm::new_from_rng_128(SmallRng::seed_from_u64(seed)) as
 * derived by crates/zkie-core/src/pcs/merkle_cuda.rs:54-85 (host only). */
int zkie2_p2_default_constants(uint64_t seed, uint64_t *rc_init, uint64_t *rc_final,
                               uint64_t *rc_internal, uint64_t *diag15);
/* Upload the seed-1 constants to the current device unless constants were
 * already uploaded there (by this call or zkie_p2_upload_constants). */
int zkie2_p2_init_default(void);
/* reps full permutations of each of n 16-element states, in place. */
int zkie2_p2_permute(uint64_t *d_states, uint64_t n, uint32_t reps, zkie_stream_t stream);
/* Measurement helper: n threads each run 8 independent chains of iters
 * Goldilocks multiplications on d_buf[16 * i .. 16 * i + 16) (x *= y), in
 * registers; the peak field-multiplication rate of the integer pipes. */
int zkie2_gl_mul_probe(uint64_t *d_buf, uint64_t n, uint32_t iters, zkie_stream_t stream);

/* ---- NTT / LDE -------------------------------------------------------------- */

/* Zero-padded LDE of every column: d_in is L x w row-major (L = 2^lg_l),
 * d_out is (L << lg_blowup) x w, out[i] = sum_j in[j] W^(ij) with W the
 * generator of order L << lg_blowup (TWO_ADIC_GENERATORS).  Same contract as
 * the pad + dft_batch of vendor/p3-whir/src/pcs/committer/writer.rs:73-82 and
 * crates/zkie-core/src/pcs/dft_cuda.rs:161-221. */
uint64_t zkie2_lde_scratch_elems(uint32_t lg_l, uint32_t lg_blowup, uint64_t w);
int zkie2_lde(const uint64_t *d_in, uint64_t *d_out, uint64_t *d_scratch, uint32_t lg_l,
              uint32_t lg_blowup, uint64_t w, zkie_stream_t stream);
/* Host-side builder of the twiddle table zkie_ntt_forward_goldilocks consumes
 * (the make_twiddles of crates/zkie-core/src/pcs/dft_cuda.rs:44-59): h_out
 * receives 2^lg - 1 entries, stage s at offset 2^(s-1) - 1. */
int zkie2_dft_twiddles(uint32_t lg, uint64_t *h_out);
/* Out-of-place DFT of every column (h = 2^lg_h); scratch as zkie2_lde(lg_h, 0, w). */
int zkie2_dft(const uint64_t *d_in, uint64_t *d_out, uint64_t *d_scratch, uint32_t lg_h, uint64_t w,
              zkie_stream_t stream);
/* One coset of the zero-padded LDE, for commits split over G = 2^lg_g GPUs:
 * d_out ((H/G) x w, H = L << lg_blowup) receives rows g, g + G, g + 2G, ...
 * of the zkie2_lde output, computed by one H/G-point DFT of the twisted (and,
 * when G > 2^lg_blowup, folded) input.  No reference counterpart: the
 * reference commits on one device. */
uint64_t zkie2_lde_coset_scratch_elems(uint32_t lg_l, uint32_t lg_blowup, uint64_t w, uint32_t lg_g);
int zkie2_lde_coset(const uint64_t *d_in, uint64_t *d_out, uint64_t *d_scratch, uint32_t lg_l,
                    uint32_t lg_blowup, uint64_t w, uint32_t lg_g, uint64_t g, zkie_stream_t stream);

/* ---- Merkle ----------------------------------------------------------------- */

/* Layer geometry of one h-row matrix (pcs/merkle_cuda.rs:203-209): layer 0 has
 * padded_len(h, 2) digests, each next layer padded_len(prev / 2, 2), down to
 * one root.  Layers are stored back to back, 8 u64 per digest. */
uint64_t zkie2_merkle_total_digests(uint64_t h);
uint32_t zkie2_merkle_num_layers(uint64_t h);
/* Leaf digests of all h rows (PaddingFreeSponge<Perm,16,8,8>). */
int zkie2_merkle_leaves(const uint64_t *d_mat, uint64_t h, uint64_t w, uint64_t *d_digests,
                        zkie_stream_t stream);
/* All layers (CudaMerkleTreeMmcs::commit_gpu, pcs/merkle_cuda.rs:177-312);
 * the root is the last digest. */
int zkie2_merkle_tree(const uint64_t *d_mat, uint64_t h, uint64_t w, uint64_t *d_layers,
                      zkie_stream_t stream);
/* Layers 1.. of the tree whose h leaf digests are already in d_layers[0 .. 8h)
 * (the compression loop of pcs/merkle_cuda.rs:250-280). */
int zkie2_merkle_tree_from_leaves(uint64_t h, uint64_t *d_layers, zkie_stream_t stream);
/* Split commit over g GPUs: after the all-to-all of leaf digests a rank holds,
 * per source rank r, the n digests of rows r, r + g, r + 2g, ... of its leaf
 * block (source-major); d_out receives them in row order:
 * d_out[c*g + r] = d_in[r*n + c] (64-byte digests; d_in != d_out). */
int zkie2_digests_interleave(const uint64_t *d_in, uint64_t g, uint64_t n, uint64_t *d_out,
                             zkie_stream_t stream);

/* ---- commit (LDE + Merkle) ---------------------------------------------------- */

uint64_t zkie2_commit_scratch_elems(uint32_t lg_l, uint32_t lg_blowup, uint64_t w);
/* LDE of d_coeffs into d_lde ((L << lg_blowup) x w), then every Merkle layer
 * of its rows into d_layers (zkie2_merkle_total_digests(L << lg_blowup) x 8). */
int zkie2_commit(const uint64_t *d_coeffs, uint32_t lg_l, uint32_t lg_blowup, uint64_t w,
                 uint64_t *d_lde, uint64_t *d_layers, uint64_t *d_scratch, zkie_stream_t stream);
/* WHIR base commit of 2^n evaluations (n >= 5): a 2^(n-5) x 32 row-major
 * matrix at blowup 2 (pcs/whir.rs:296-359,438-469).  d_lde is 2^(n-4) x 32. */
uint64_t zkie2_whir_scratch_elems(uint32_t n);
int zkie2_whir_commit(const uint64_t *d_evals, uint32_t n, uint64_t *d_lde, uint64_t *d_layers,
                      uint64_t *d_scratch, zkie_stream_t stream);
/* WHIR round commit of a folded extension-field polynomial (commit_extension,
 * vendor/p3-whir/src/pcs/committer/writer.rs:21-86, Suffix order): d_evals
 * holds 2^n EF elements (degree-2 binomial extension, c0 then c1 per
 * element), n >= 5; the encoding is (2^(n-5) << log_inv_rate) rows x 32 EF,
 * stored in d_lde as 64 base columns per row, and the tree hashes those
 * 64-element rows (ExtensionMmcs).  d_layers as zkie2_merkle_total_digests of
 * the row count. */
uint64_t zkie2_commit_extension_scratch_elems(uint32_t n, uint32_t log_inv_rate);
int zkie2_commit_extension(const uint64_t *d_evals, uint32_t n, uint32_t log_inv_rate, uint64_t *d_lde,
                           uint64_t *d_layers, uint64_t *d_scratch, zkie_stream_t stream);
/* Commit (root and every digest layer, as zkie2_commit) of a matrix whose LDE
 * need not fit in HBM: the LDE rows are computed one coset of 2^lg_c at a time
 * (rows c, c + 2^lg_c, ...; 2 lg_c <= lg_l + lg_blowup), each coset hashed
 * and its LDE buffer reused, and the leaf digests put in row order before the
 * tree.  The LDE is not kept.  d_scratch holds
 * zkie2_commit_cosets_scratch_elems u64 (0 = unsupported shape).  No reference
 * counterpart: the reference keeps the whole LDE on one device. */
uint64_t zkie2_commit_cosets_scratch_elems(uint32_t lg_l, uint32_t lg_blowup, uint64_t w, uint32_t lg_c);
int zkie2_commit_cosets(const uint64_t *d_coeffs, uint32_t lg_l, uint32_t lg_blowup, uint64_t w, uint32_t lg_c,
                        uint64_t *d_layers, uint64_t *d_scratch, zkie_stream_t stream);
/* Host-buffer commit (the drop-in path of CudaDft::dft_batch followed by
 * CudaMerkleTreeMmcs::commit): h_coeffs L x w in, root (8 u64) out, plus the
 * LDE ((L << lg_blowup) x w) and all digest layers when those pointers are
 * non-null.  Synchronous.  Allocates its device buffers from a memory pool
 * the library creates for the current device on the first call (freed blocks
 * stay cached in that pool for the next call; the device's default pool is
 * left as it was).  Calls on one device are serialised inside the library:
 * a second host thread blocks until the first call has returned. */
int zkie2_commit_host(const uint64_t *h_coeffs, uint32_t lg_l, uint32_t lg_blowup, uint64_t w,
                      uint64_t *h_lde, uint64_t *h_layers, uint64_t *h_root);

/* ---- Fiat-Shamir (host) ---------------------------------------------------------- */

/* Transcript of crates/zkie-core/src/common/transcript.rs:21-80. */
typedef struct {
    uint8_t state[32];
    uint64_t counter;
} zkie2_transcript;

#define ZKIE2_CHALLENGER_XORSHIFT 0
#define ZKIE2_CHALLENGER_TRANSCRIPT 1
/* A ChallengeSource (common/field.rs:58-76): XorShift64 (common/field.rs:17-36)
 * or Transcript. */
typedef struct {
    int32_t kind;
    uint64_t xorshift_state;
    zkie2_transcript transcript;
} zkie2_challenger;

void zkie2_sha256(const uint8_t *data, size_t len, uint8_t *out32);
void zkie2_transcript_new(zkie2_transcript *t, const uint8_t *domain, size_t len);
void zkie2_transcript_absorb(zkie2_transcript *t, const uint8_t *data, size_t len);
void zkie2_transcript_absorb_u64(zkie2_transcript *t, uint64_t x);
uint64_t zkie2_transcript_field(zkie2_transcript *t);
uint64_t zkie2_transcript_next_u64(zkie2_transcript *t);
void zkie2_challenger_xorshift(zkie2_challenger *c, uint64_t seed);
/* n XorShift64 draws from *state (advanced), each stored as
 * from_i64((draw % mod) + offset): the weight draws of the reference's random
 * model builders.  mod > 0. */
void zkie2_xorshift_fill(uint64_t *state, uint64_t n, uint64_t mod, int64_t offset, uint64_t *out);
uint64_t zkie2_challenger_field(zkie2_challenger *c);
/* n successive draws of zkie2_challenger_field / zkie2_transcript_field into out. */
void zkie2_challenger_fields(zkie2_challenger *c, uint64_t n, uint64_t *out);
void zkie2_transcript_fields(zkie2_transcript *t, uint64_t n, uint64_t *out);
/* Child transcript of shard `shard_index` in prove_shard_dag
 * (zkie-ops/src/compose.rs:2276-2311) for a statement of MatMul ops given as
 * (a, b, c) tensor-id triples. */
void zkie2_shard_dag_child(const uint64_t *op_ids, uint32_t n_ops, uint64_t ops_per_shard,
                           uint64_t shard_index, zkie2_challenger *child);

/* ---- MLE / sumcheck / matmul GKR ------------------------------------------------- */

/* eq(r, x) for every x < 2^d (common/mle.rs:44-55). */
int zkie2_eq_evals(const uint64_t *h_r, uint32_t d, uint64_t *d_out, zkie_stream_t stream);
uint64_t zkie2_mle_scratch_elems(uint32_t t);
/* partial_eval (common/mle.rs:25-38): fix the first f of t variables. */
int zkie2_mle_partial_eval(const uint64_t *d_values, uint32_t t, const uint64_t *h_fix, uint32_t f,
                           uint64_t *d_out, uint64_t *d_scratch, zkie_stream_t stream);
/* eval (common/mle.rs:8-23); synchronous, result to *h_out. */
int zkie2_mle_eval(const uint64_t *d_values, uint32_t t, const uint64_t *h_point, uint64_t *h_out,
                   uint64_t *d_scratch, zkie_stream_t stream);
/* The same with the value left in *d_out on the device (no synchronization). */
int zkie2_mle_eval_async(const uint64_t *d_values, uint32_t t, const uint64_t *h_point, uint64_t *d_out,
                         uint64_t *d_scratch, zkie_stream_t stream);
/* count evaluations in one call: table i (2^ts[i] values at d_values[i]) at
 * the next ts[i] values of h_points, into d_out[i]; d_scratch holds
 * zkie2_mle_eval_many_scratch_elems(max ts[i]) u64.  No synchronization. */
uint64_t zkie2_mle_eval_many_scratch_elems(uint32_t max_t);
int zkie2_mle_eval_many(const uint64_t *const *d_values, const uint32_t *ts, const uint64_t *h_points,
                        uint32_t count, uint64_t *d_out, uint64_t *d_scratch, zkie_stream_t stream);
/* sumcheck::prove (common/sumcheck.rs:33-79) over f, h of length 2^t with the
 * t challenges h_ch: h_rounds gets (c0, c1, c2) per round, h_finals (f, h)
 * after the last fold.  Synchronous. */
uint64_t zkie2_sumcheck_scratch_elems(uint32_t t);
int zkie2_sumcheck_prove(const uint64_t *d_f, const uint64_t *d_h, uint32_t t, const uint64_t *h_ch,
                         uint64_t *h_rounds, uint64_t *h_finals, uint64_t *d_scratch,
                         zkie_stream_t stream);
/* Allocation-free variant of zkie2_sumcheck_prove; it has no counterpart in
 * the reference.  It is for callers that cannot allocate device memory: a
 * prover embedded in a process whose framework allocator (PyTorch's caching
 * allocator, an inference server's pool) has already reserved the GPU's
 * memory, so a cudaMalloc fails or fragments that pool, and latency-critical
 * callers that cannot afford the device-wide synchronization cudaFree
 * implies.  The caller still passes f, h (device), the challenges and the
 * host outputs; the scratch is a fixed array inside the library (about
 * 1.9 MB, held on every GPU that loads the library until exit), so this call
 * allocates nothing.  Limit: t <= zkie2_sumcheck_noalloc_max_vars() (24);
 * larger t returns cudaErrorInvalidValue.  The first call on a device looks
 * up the array's device address (once per device), so make that first call
 * before any stream capture.  All calls share the one array: calls that
 * overlap on the GPU (other threads or streams) race and must be serialized
 * by the caller.  Synchronous, same outputs as zkie2_sumcheck_prove. */
uint32_t zkie2_sumcheck_noalloc_max_vars(void);
int zkie2_sumcheck_prove_noalloc(const uint64_t *d_f, const uint64_t *d_h, uint32_t t,
                                 const uint64_t *h_ch, uint64_t *h_rounds, uint64_t *h_finals,
                                 zkie_stream_t stream);
/* matmul::prove (common/matmul.rs:17-46): d_at = A^T (k x m), d_b (k x n),
 * d_c (m x n), powers of two.  Synchronous. */
uint64_t zkie2_matmul_scratch_elems(uint64_t m, uint64_t k, uint64_t n);
int zkie2_matmul_prove(const uint64_t *d_at, const uint64_t *d_b, const uint64_t *d_c, uint64_t m,
                       uint64_t k, uint64_t n, const uint64_t *h_u, const uint64_t *h_v,
                       const uint64_t *h_ch, uint64_t *h_claimed, uint64_t *h_rounds,
                       uint64_t *h_finals, uint64_t *d_scratch, zkie_stream_t stream);
/* Op::MatMul arm (zkie-ops/src/compose.rs:1724-1747): draws u, v, ch from src,
 * proves C = A @ B with d_a (m x k) as stored, returns the draws, the proof and
 * the claims eval(A, ch||u), eval(B, v||ch), eval(C, v||u).  Synchronous. */
uint64_t zkie2_op_matmul_scratch_elems(uint64_t m, uint64_t k, uint64_t n);
int zkie2_op_matmul_prove(const uint64_t *d_a, const uint64_t *d_b, const uint64_t *d_c, uint64_t m,
                          uint64_t k, uint64_t n, zkie2_challenger *src, uint64_t *out_u,
                          uint64_t *out_v, uint64_t *out_ch, uint64_t *out_claimed,
                          uint64_t *out_rounds, uint64_t *out_finals, uint64_t *out_claims,
                          uint64_t *d_scratch, zkie_stream_t stream);
/* The same with u, v, ch from the caller and claimed | rounds (3 log2 k) |
 * finals (2) left in d_proof on the device; no synchronization (the claims
 * are left to zkie2_mle_eval_async). */
int zkie2_op_matmul_prove_async(const uint64_t *d_a, const uint64_t *d_b, const uint64_t *d_c, uint64_t m,
                                uint64_t k, uint64_t n, const uint64_t *h_u, const uint64_t *h_v,
                                const uint64_t *h_ch, uint64_t *d_proof, uint64_t *d_scratch, zkie_stream_t stream);
/* C = A @ B over the field (the forward witness of Op::MatMul,
 * zkie-ops/src/compose.rs:1327-1331, zkie-ops/src/par.rs:41-89). */
int zkie2_matmul_field(const uint64_t *d_a, const uint64_t *d_b, uint64_t m, uint64_t k, uint64_t n,
                       uint64_t *d_c, zkie_stream_t stream);
/* The forward witness of a fixed-point matmul (par::mm_par_fixed, zkie-ops/src/par.rs:41-89):
 * d_c (m x n) = d_a (m x k) times d_b (k x n), row-major field elements, exactly as
 * zkie2_matmul_field.  When every input lies in [-2^23, 2^23) (to_i64 of the field element)
 * and k % 16 == 0, n % 4 == 0 (and k < 2^17 once an operand needs 24 bits), the products run
 * on the tensor cores (u8 x u8 -> s32 tcgen05 GEMMs over two or three byte planes per operand,
 * two where its values lie in [-2^15, 2^15), offset to unsigned and recombined exactly);
 * otherwise the exact field kernel
 * runs, as the reference falls back to its field matmul.  policy 0: the field kernel also
 * below 2^27 multiply-adds, where it is faster; policy 1: the tensor cores whenever the inputs
 * allow.  *h_path (optional) = 0 tensor cores, 1 field kernel.  The tensor path reads two
 * range flags back (synchronizes the stream). */
uint64_t zkie2_matmul_fixed_scratch_elems(uint64_t m, uint64_t k, uint64_t n);
int zkie2_matmul_fixed(const uint64_t *d_a, const uint64_t *d_b, uint64_t m, uint64_t k, uint64_t n,
                       uint64_t *d_c, uint32_t policy, uint32_t *h_path, uint64_t *d_scratch,
                       zkie_stream_t stream);
/* zkie2_matmul_fixed reporting its choices: h_plan = {path (0 tensor cores, 1 field kernel),
 * planes of A, planes of B}. */
int zkie2_matmul_fixed_ex(const uint64_t *d_a, const uint64_t *d_b, uint64_t m, uint64_t k, uint64_t n,
                          uint64_t *d_c, uint32_t policy, uint32_t *h_plan, uint64_t *d_scratch,
                          zkie_stream_t stream);
/* The product with the choices of an earlier call fixed (h_plan as above),
 * no read-back and no synchronization, so it can be recorded in a CUDA graph:
 * the operands' widths are still checked on the device, and operands that
 * need more planes than planned (or more than 24 bits) set bit 3 (value 4) of
 * *d_err, in which case d_c is not the product and the caller recomputes it
 * with zkie2_matmul_fixed. */
int zkie2_matmul_fixed_planned(const uint64_t *d_a, const uint64_t *d_b, uint64_t m, uint64_t k, uint64_t n,
                               uint64_t *d_c, const uint32_t *h_plan, uint64_t *d_scratch, uint32_t *d_err,
                               zkie_stream_t stream);
/* The same product for runs of rows that each multiply one block of a
 * stack (GatherMatMul's forward, batched_matmul.rs:331-357, with the
 * positions of one expert consecutive): h_runs holds n_runs triples
 * (expert e, first row r0, rows), consecutive from row 0; rows r0 .. r0 +
 * rows - 1 of d_a (k columns) times block e of d_w (n_experts x k x n) into
 * the same rows of d_c (n columns).  One range pass over all rows and the
 * whole stack and one read-back, then per run the tensor path (or the field
 * kernel for runs below 2^27 multiply-adds or operands past 24 bits) with no
 * further synchronization.  Scratch: zkie2_matmul_fixed_runs_scratch_elems
 * of the longest run. */
uint64_t zkie2_matmul_fixed_runs_scratch_elems(uint64_t rows, uint64_t k, uint64_t n);
int zkie2_matmul_fixed_runs(const uint64_t *d_a, const uint64_t *d_w, uint64_t n_experts, uint64_t k, uint64_t n,
                            const uint64_t *h_runs, uint64_t n_runs, uint64_t *d_c, uint64_t *d_scratch,
                            zkie_stream_t stream);
/* The projection block's witness columns (crates/zkie-ops/src/projection.rs, the
 * out / rem_off construction of its tests, :136-176): for each of n elements,
 * with a = to_i64(h) (h = x @ W) and b = to_i64(bias),
 *   out = div_round(a, 2^shift) + b      (floor, plus one when the remainder >= 2^(shift-1)),
 *   rem_off = a - (out - b) 2^shift + 2^(shift-1)   (in [0, 2^shift)),
 * as field elements (from_i64), and, when d_idx is non-null, the lookup index
 * to_i32(rem_off) as u32 of prove_projection (:94).  1 <= shift <= 30. */
int zkie2_projection_witness(const uint64_t *d_h, const uint64_t *d_bias, uint64_t n, uint32_t shift,
                             uint64_t *d_out, uint64_t *d_rem_off, uint32_t *d_idx, zkie_stream_t stream);
/* to_i32(v) as u32 of n field elements (the lookup indices of a fixed-point
 * column, fixed_point.rs to_i32). */
int zkie2_lookup_index_i32(const uint64_t *d_v, uint64_t n, uint32_t *d_idx, zkie_stream_t stream);
/* prove_projection (crates/zkie-ops/src/projection.rs:44-101) in one call, for
 * x (m x k), W (k x n), bias, out, rem_off (m x n) on the device, m, k, n
 * powers of two, 1 <= shift <= 30: h = x W (zkie2_matmul_fixed; pass d_h to
 * reuse an h already computed, else NULL), the MatMul GKR with u, v, ch drawn
 * from src, prove_virtual over [eq(v||u), rem_off, h, out, bias, ones] with
 * the five affine terms, alpha and beta from src, and the logUp range check
 * of (to_i32(rem_off) as u32, rem_off) into the table 0 .. 2^shift - 1 with
 * full_r then cs drawn from src (lg = zkie2_projection_lookup_vars of each).
 * Host outputs: claimed (1), mm_rounds (log2 k x 3), mm_finals (2), u (log2 m),
 * v (log2 n), ch (log2 k), aff_rounds (log2(m n) x 3), aff_finals (6),
 * alpha_beta (2), full_r, cs (lg each), frac_rounds (2 lg (lg - 1)),
 * frac_finals (7 lg), frac_nd (2): the fields of the reference's
 * ProjectionProof.  d_scratch: zkie2_projection_scratch_elems.  Synchronous. */
uint32_t zkie2_projection_lookup_vars(uint64_t m, uint64_t n, uint32_t shift);
uint64_t zkie2_projection_scratch_elems(uint64_t m, uint64_t k, uint64_t n, uint32_t shift);
int zkie2_projection_prove(const uint64_t *d_x, const uint64_t *d_w, const uint64_t *d_bias, const uint64_t *d_out,
                           const uint64_t *d_rem_off, const uint64_t *d_h, uint64_t m, uint64_t k, uint64_t n,
                           uint32_t shift, zkie2_challenger *src, uint64_t *h_claimed, uint64_t *h_mm_rounds,
                           uint64_t *h_mm_finals, uint64_t *h_u, uint64_t *h_v, uint64_t *h_ch,
                           uint64_t *h_aff_rounds, uint64_t *h_aff_finals, uint64_t *h_alpha_beta,
                           uint64_t *h_full_r, uint64_t *h_cs, uint64_t *h_frac_rounds, uint64_t *h_frac_finals,
                           uint64_t *h_frac_nd, uint64_t *d_scratch, zkie_stream_t stream);
/* The same with every challenge from the caller (u, v, ch, alpha, beta,
 * full_r, cs) and the proof fields left on the device in d_proof
 * (zkie2_projection_proof_elems u64: claimed | mm_rounds | mm_finals |
 * aff_rounds | aff_finals | frac_rounds | frac_finals | frac_nd); a lookup
 * index outside the table sets bit 1 of the device word *d_err.  No
 * synchronization; d_scratch as above. */
uint64_t zkie2_projection_proof_elems(uint64_t m, uint64_t k, uint64_t n, uint32_t shift);
int zkie2_projection_prove_async(const uint64_t *d_x, const uint64_t *d_w, const uint64_t *d_bias,
                                 const uint64_t *d_out, const uint64_t *d_rem_off, const uint64_t *d_h, uint64_t m,
                                 uint64_t k, uint64_t n, uint32_t shift, const uint64_t *h_u, const uint64_t *h_v,
                                 const uint64_t *h_ch, uint64_t alpha, uint64_t beta, const uint64_t *h_full_r,
                                 const uint64_t *h_cs, uint64_t *d_proof, uint32_t *d_err, uint64_t *d_scratch,
                                 zkie_stream_t stream);
/* One MatMul shard in one call: C = A W into d_c
 * (m x n), WHIR base commits of W (k*n evaluations), A (m*k) and C (m*n)
 * (pcs/whir.rs:438-469, each >= 32 evaluations), and the Op::MatMul proof
 * with challenges from the shard's child transcript (zkie2_shard_dag_child
 * of op_ids = {a, b, c}, one op).  The stages run concurrently on four
 * streams; one synchronization at the end.  h_roots gets 3 x 8 u64 (W, A, C),
 * the rest as zkie2_op_matmul_prove.  The LDEs and digest layers stay in
 * d_scratch (zkie2_shard_prove_matmul_scratch_elems u64).  Synchronous. */
uint64_t zkie2_shard_prove_matmul_scratch_elems(uint64_t m, uint64_t k, uint64_t n);
int zkie2_shard_prove_matmul(const uint64_t *d_a, const uint64_t *d_w, uint64_t m, uint64_t k, uint64_t n,
                             const uint64_t *op_ids, uint64_t ops_per_shard, uint64_t shard_index,
                             uint64_t *d_c, uint64_t *h_roots, uint64_t *h_claimed, uint64_t *h_rounds,
                             uint64_t *h_finals, uint64_t *h_claims, uint64_t *d_scratch,
                             zkie_stream_t stream);
/* prove_sum_of_products (common/sumcheck.rs:243-286): the batch-opening
 * sumcheck of sum_x sum_i w_i(x) v_i(x) over n_tables pairs of 2^t tables,
 * stored row-major: table i of d_weights / d_values starts at element i * 2^t.
 * h_rounds gets (c0, c1, c2) per round, h_b_eval = sum_i w_i(r) v_i(r).
 * Synchronous. */
uint64_t zkie2_sum_of_products_scratch_elems(uint32_t n_tables, uint32_t t);
int zkie2_sum_of_products_prove(const uint64_t *d_weights, const uint64_t *d_values, uint32_t n_tables,
                                uint32_t t, const uint64_t *h_ch, uint64_t *h_rounds, uint64_t *h_b_eval,
                                uint64_t *d_scratch, zkie_stream_t stream);
/* prove_virtual (common/sumcheck.rs:378-438): sum over {0,1}^t of
 * sum_i coeffs[i] * prod_{j in term i} f_j, over n_mles (<= 16) device tables
 * of 2^t values (d_mles is a host array of device pointers).  Term i has the
 * factors idx[idx_off[i] .. idx_off[i+1]) (at most 8 per term, 64 in all,
 * n_terms <= 32, idx_off[0] = 0).  h_rounds gets t x (d + 1) evaluations,
 * d = the largest term size; h_finals the n_mles folded values.
 * Synchronous. */
uint64_t zkie2_virtual_scratch_elems(uint32_t n_mles, uint32_t t);
int zkie2_virtual_prove(const uint64_t *const *d_mles, uint32_t n_mles, uint32_t t, const uint64_t *coeffs,
                        const uint32_t *idx_off, const uint32_t *idx, uint32_t n_terms, const uint64_t *h_ch,
                        uint64_t *h_rounds, uint64_t *h_finals, uint64_t *d_scratch, zkie_stream_t stream);
/* The same with the rounds and finals left in device memory (d_rounds: t x
 * (d + 1), d_finals: n_mles); no synchronization. */
int zkie2_virtual_prove_async(const uint64_t *const *d_mles, uint32_t n_mles, uint32_t t, const uint64_t *coeffs,
                              const uint32_t *idx_off, const uint32_t *idx, uint32_t n_terms, const uint64_t *h_ch,
                              uint64_t *d_rounds, uint64_t *d_finals, uint64_t *d_scratch, zkie_stream_t stream);

/* PoW grinding of the WHIR prover (challenger.grind, p3-whir src/pcs/prover/mod.rs:240-245,
 * 355-358) on the transcript's DuplexChallenger<Goldilocks, Poseidon2-16, 16, 8>
 * (pcs/whir.rs:42): the smallest w < p with check_witness(bits, w), i.e. observe(w) then
 * sample_bits(bits) == 0, for the challenger whose sponge state is h_sponge (16 values)
 * with len < 8 inputs h_input buffered.  The reference searches with find_any and keeps
 * any valid witness; every valid witness verifies.  The caller then replays
 * check_witness on its own challenger (one permutation), as the reference does.
 * Batches of zkie2_grind_batch(bits) candidates per launch.  Synchronous. */
uint64_t zkie2_grind_batch(uint32_t bits);
int zkie2_grind(const uint64_t *h_sponge, const uint64_t *h_input, uint32_t len, uint32_t bits,
                uint64_t *h_witness, zkie_stream_t stream);

/* ---- ZKIEBCH2 weight cache --------------------------------------------------------- */
/* The weight-cache file of a committed batch: header = bincode 1.3.3 of (b"ZKIEBCH2",
 * BatchCacheMetadata, MerkleCap of the root) (pcs/cache.rs:7-70); then the committed
 * matrix (Whir::serialize_batch_prover_data_into, pcs/whir.rs:542-559: u64 count 1,
 * u64 width, u64 value count, values); then the digest layers (p3-merkle-tree
 * write_digest_layers: u64 layer count, u64 per layer length, u64 arity 2 per step,
 * digests).  All integers little-endian.  zkie2_cache_header returns the header length
 * and writes it to out when out_cap is large enough (0 on a null argument). */
uint64_t zkie2_cache_header(const char *model_id, const char *group_id, const char *const *table_ids,
                            uint32_t num_tables, uint32_t table_arity, uint32_t security_level, uint32_t pow_bits,
                            const uint8_t *source_digest, const uint64_t *root, uint8_t *out, uint64_t out_cap);
/* Write the file: the header bytes, then the rows x width matrix d_lde and every digest
 * layer of its rows-row tree (d_layers, the layout of zkie2_merkle_tree) streamed from the
 * device through pinned staging buffers.  Synchronous. */
int zkie2_cache_write(const char *path, const uint8_t *header, uint64_t header_len, const uint64_t *d_lde,
                      uint64_t rows, uint64_t width, const uint64_t *d_layers, zkie_stream_t stream);
/* Read the matrix and the digest layers of such a file (after its header_len header bytes)
 * into device buffers, checking every count against rows x width.  Synchronous. */
int zkie2_cache_read(const char *path, uint64_t header_len, uint64_t rows, uint64_t width, uint64_t *d_lde,
                     uint64_t *d_layers, zkie_stream_t stream);

/* ---- logUp GKR fraction tree (common/logup_gkr.rs) ------------------------------------ */
/* prove_fractional_with_challenges (logup_gkr.rs:29-69) over device tables
 * num, den of 2^lg_n values (read only), with lg_n challenges full_r and cs
 * (host).  Layer l = 0 .. lg_n-1 is a prove_virtual over seven tables with
 * lg_n - l - 1 rounds of 4 evaluations: h_rounds gets every layer's rounds
 * concatenated (2 lg_n (lg_n - 1) values), h_finals 7 final evaluations per
 * layer, h_final_nd the last layer's (num, den).  Synchronous. */
uint64_t zkie2_fractional_scratch_elems(uint32_t lg_n);
int zkie2_fractional_prove(const uint64_t *d_num, const uint64_t *d_den, uint32_t lg_n, const uint64_t *h_full_r,
                           const uint64_t *h_cs, uint64_t *h_rounds, uint64_t *h_finals, uint64_t *h_final_nd,
                           uint64_t *d_scratch, zkie_stream_t stream);
/* The same with rounds | finals | final (num, den) left in d_proof
 * (zkie2_fractional_proof_elems u64); no synchronization. */
uint64_t zkie2_fractional_proof_elems(uint32_t lg_n);
int zkie2_fractional_prove_async(const uint64_t *d_num, const uint64_t *d_den, uint32_t lg_n,
                                 const uint64_t *h_full_r, const uint64_t *h_cs, uint64_t *d_proof,
                                 uint64_t *d_scratch, zkie_stream_t stream);
/* Lookup columns num, den of zkie2_lookup_len(n, t, mode) values (device):
 * mode 0 build_lookup_num_den (logup_gkr.rs:210-240: witness fractions, then
 * the table with -multiplicity, multiplicities counted on the device;
 * cudaErrorInvalidValue if some x >= t), 1 build_lookup_witness_num_den
 * (:261-277), 2 the witness columns of prove_lookup_witness_batch_columns
 * (:340-370: at least 32 rows, padding den = alpha), 3
 * build_lookup_table_num_den (:285-301, multiplicities d_m from the caller).
 * d_x is u32.  Mode 0 synchronizes on the stream to report a bad index. */
uint64_t zkie2_lookup_len(uint64_t n, uint64_t t, uint32_t mode);
uint64_t zkie2_lookup_scratch_elems(uint64_t t);
int zkie2_lookup_num_den(const uint32_t *d_x, const uint64_t *d_y, uint64_t n, const uint64_t *d_table,
                         const uint64_t *d_m, uint64_t t, uint32_t mode, uint64_t alpha, uint64_t beta,
                         uint64_t *d_num, uint64_t *d_den, uint64_t *d_scratch, zkie_stream_t stream);
/* The same without synchronization: in mode 0 an index at or past t sets
 * bit 1 of the device word *d_err. */
int zkie2_lookup_num_den_async(const uint32_t *d_x, const uint64_t *d_y, uint64_t n, const uint64_t *d_table,
                               const uint64_t *d_m, uint64_t t, uint32_t mode, uint64_t alpha, uint64_t beta,
                               uint64_t *d_num, uint64_t *d_den, uint64_t *d_scratch, uint32_t *d_err,
                               zkie_stream_t stream);
/* merge_multiplicity (logup_gkr.rs:251-260) on the device: d_m[j] (u64, t
 * values) += the count of j in d_x[0 .. n) (zeroed first unless
 * accumulate); an index at or past t sets bit 1 of *d_err. */
int zkie2_lookup_multiplicity(const uint32_t *d_x, uint64_t n, uint64_t t, uint64_t *d_m, int accumulate,
                              uint32_t *d_err, zkie_stream_t stream);

/* ---- the op layer (crates/zkie-ops/src/compose.rs) ----------------------------------- */
/* The forward witness of the op arms a GPT-2 layer uses (forward_ops,
 * compose.rs:1174-1583) and the columns their proofs read.  Tensors are flat
 * row-major device arrays of field elements (u64) or of u32 lookup indices.
 * Fixed-point values are the field embedding of fixed_point.rs (to_i64 /
 * from_i64), with the reference's wrapping i64 arithmetic.  Where the
 * reference panics on data (an index outside a table, a zero softmax row
 * sum), the kernels set a bit in the device word *d_err (1: index, 2:
 * division) and carry on.  None of these synchronizes. */
/* Op::Add: out = a + b over the field */
int zkie2_op_add(const uint64_t *d_a, const uint64_t *d_b, uint64_t n, uint64_t *d_out, zkie_stream_t stream);
/* Op::Scale: out = from_i64(round_div(to_i64(x) * factor, 2^shift)), shift <= 62 */
int zkie2_op_scale(const uint64_t *d_x, uint64_t n, int64_t factor, uint32_t shift, uint64_t *d_out,
                   zkie_stream_t stream);
/* Op::Transpose: x (m x k) -> out (k x m) */
int zkie2_op_transpose(const uint64_t *d_x, uint64_t m, uint64_t k, uint64_t *d_out, zkie_stream_t stream);
/* Op::SoftmaxIndex: idx = (max(to_i64(x), 0) as u64) % table_len */
int zkie2_op_softmax_index(const uint64_t *d_x, uint64_t n, uint64_t table_len, uint32_t *d_idx,
                           zkie_stream_t stream);
/* Op::GeluIndex: idx = clamp(to_i64(x) + offset, 0, table_len - 1) */
int zkie2_op_gelu_index(const uint64_t *d_x, uint64_t n, int64_t offset, uint64_t table_len, uint32_t *d_idx,
                        zkie_stream_t stream);
/* Op::StableSoftmaxIndex: masked = x + mask, idx = clamp(to_i64(masked) -
 * max over the row of to_i64(masked) + offset, 0, table_len - 1); m rows of n */
int zkie2_op_stable_softmax_index(const uint64_t *d_x, const uint64_t *d_mask, uint64_t m, uint64_t n,
                                  int64_t offset, uint64_t table_len, uint32_t *d_idx, zkie_stream_t stream);
/* Op::Lookup: out = table[idx] */
int zkie2_op_lookup(const uint32_t *d_idx, uint64_t n, const uint64_t *d_table, uint64_t t, uint64_t *d_out,
                    uint32_t *d_err, zkie_stream_t stream);
/* Op::Softmax: e = table[idx], sum = each row's field sum (into d_sum, m
 * values, when non-null), out = from_i64(round_div(to_i64(e) 2^16, to_i64(sum))) */
int zkie2_op_softmax(const uint32_t *d_idx, const uint64_t *d_table, uint64_t t, uint64_t m, uint64_t n,
                     uint64_t *d_e, uint64_t *d_out, uint64_t *d_sum, uint32_t *d_err, zkie_stream_t stream);
/* prove_softmax_rounded's columns (softmax_scaled.rs:69-80): sum_b = the row
 * sum broadcast over its row, rem = from_i64(to_i64(e) 2^16 - to_i64(out) to_i64(sum_b)) */
int zkie2_op_softmax_rem(const uint64_t *d_e, const uint64_t *d_out, const uint64_t *d_sum, uint64_t m, uint64_t n,
                         uint64_t *d_sum_b, uint64_t *d_rem, zkie_stream_t stream);
/* layer_norm_forward (layer_norm_centered.rs:42-120) of m rows of d values,
 * the first n_real real, with rsqrt_index (compose.rs:884-896) into the
 * table of t values.  d_outs (host array of 11 device pointers): mean (m),
 * centered (m d), var (m), rstd (m), raw = centered rstd w (m d), out (m d),
 * rem_out (m d), sum_mean (m), rem_mean (m), sum_var (m), rem_var (m);
 * d_s_index (m u32). */
int zkie2_op_layer_norm_centered(const uint64_t *d_x, const uint64_t *d_w, const uint64_t *d_b,
                                 const uint64_t *d_table, uint64_t t, uint64_t m, uint64_t d, uint64_t n_real,
                                 uint64_t *const *d_outs, uint32_t *d_s_index, uint32_t *d_err, zkie_stream_t stream);
/* The Layernorm arm's forward (compose.rs:1467-1496): mean_sq (m), idx (m
 * u32), rsqrt (m), scale (m d), out (m d) */
int zkie2_op_layernorm(const uint64_t *d_x, const uint64_t *d_w, const uint64_t *d_b, const uint64_t *d_table,
                       uint64_t t, uint64_t m, uint64_t d, uint64_t *d_mean_sq, uint32_t *d_idx, uint64_t *d_rsqrt,
                       uint64_t *d_scale, uint64_t *d_out, zkie_stream_t stream);
/* out[r n + j] = v[r] (m rows of n) */
int zkie2_op_row_broadcast(const uint64_t *d_v, uint64_t m, uint64_t n, uint64_t *d_out, zkie_stream_t stream);
/* out[r] = the field sum of x[r d .. r d + ncols) */
int zkie2_op_row_sums(const uint64_t *d_x, uint64_t m, uint64_t d, uint64_t ncols, uint64_t *d_out,
                      zkie_stream_t stream);
/* out[i] = value */
int zkie2_op_fill(uint64_t *d_out, uint64_t n, uint64_t value, zkie_stream_t stream);
/* out[i] = i (the range tables of the top-k proofs) */
int zkie2_op_iota(uint64_t *d_out, uint64_t n, zkie_stream_t stream);
/* The TopKSelect / Argmax arms' forward (topk.rs:41-80 topk_forward,
 * :272-297 argmax_forward; compose.rs:1543-1583): x is m rows of n; per row
 * the entries ordered by to_i64 value descending, ties by position
 * ascending; thr (m) = the k-th, sel (m n) = 1 on the first k, gate = x sel,
 * d1 = sel (x - thr), d2 = (1 - sel) (thr - x) (wrapping i64).  d_out (m
 * u32, Argmax only, k = 1) receives each row's first position of its
 * maximum.  k = 1 takes any n < 2^32; k > 1 needs n <= 4096 (the row is
 * ranked in shared memory); k = 0 or k > n is rejected, as the reference
 * would panic. */
int zkie2_op_topk(const uint64_t *d_x, uint64_t m, uint64_t n, uint64_t k, uint64_t *d_thr, uint64_t *d_sel,
                  uint64_t *d_gate, uint64_t *d_d1, uint64_t *d_d2, uint32_t *d_out, zkie_stream_t stream);
/* ---- the arms of an MLA attention / MoE layer (compose.rs:1193-1293, rms_norm.rs,
 * rope.rs, scatter.rs, gather.rs, zkie-core common/batched_matmul.rs) ---- */
/* The RmsNorm arm's forward (rms_norm.rs:37-95) over m rows of d, the first
 * n_real of each averaged: d_outs = {ms (m), rstd (m), raw, out, rem_out,
 * rem_lo, rem_hi (m d each), sum_sq (m), rem_s (m)}; d_s_index (m u32).  An
 * rsqrt index at or past t sets bit 1 of *d_err. */
int zkie2_op_rms_norm(const uint64_t *d_x, const uint64_t *d_w, const uint64_t *d_table, uint64_t t, uint64_t m,
                      uint64_t d, uint64_t n_real, uint64_t *const *d_outs, uint32_t *d_s_index, uint32_t *d_err,
                      zkie_stream_t stream);
/* ScaleVec (compose.rs:1193-1212): out[i] = from_i64(round_div(to_i64(x[i])
 * to_i64(scale[i % len]), 2^shift)), wrapping i64, shift <= 62. */
int zkie2_op_scale_vec(const uint64_t *d_x, uint64_t n, const uint64_t *d_scale, uint64_t len, uint32_t shift,
                       uint64_t *d_out, zkie_stream_t stream);
/* BroadcastScale (:1284-1293): out[i] = x[i] scale[i / h] (field); scale
 * holds len >= ceil(n / h) values. */
int zkie2_op_broadcast_scale(const uint64_t *d_x, uint64_t n, const uint64_t *d_scale, uint64_t len, uint64_t h,
                             uint64_t *d_out, zkie_stream_t stream);
/* ScaleGate (:1294-1318): out[i] = from_i64(round_div(to_i64(x[i])
 * to_i64(gate[(i / h) n + col]), 2^shift)); gate holds gate_len values. */
int zkie2_op_scale_gate(const uint64_t *d_x, uint64_t len, const uint64_t *d_gate, uint64_t gate_len, uint64_t col,
                        uint64_t n, uint64_t h, uint32_t shift, uint64_t *d_out, zkie_stream_t stream);
/* Relu (:1319-1326): x where to_i64(x) > 0, else 0. */
int zkie2_op_relu(const uint64_t *d_x, uint64_t n, uint64_t *d_out, zkie_stream_t stream);
/* BatchedMatMul's forward (batched_matmul.rs:112-134): c[pos] (n values) =
 * a[pos] (k values) times w[pos] (k x n), s positions, field arithmetic. */
int zkie2_op_batched_matmul(const uint64_t *d_a, const uint64_t *d_w, uint64_t s, uint64_t k, uint64_t n,
                            uint64_t *d_c, zkie_stream_t stream);
/* IdxBroadcast (:1258-1267): out[i b + j] = base[i] b + j (u32, wrapping). */
int zkie2_op_idx_broadcast(const uint32_t *d_base, uint64_t nb, uint32_t b, uint32_t *d_out, zkie_stream_t stream);
/* CombineIdx (:1268-1278): out[i] = a[i] scale + b[i] (u32, wrapping). */
int zkie2_op_combine_idx(const uint32_t *d_a, const uint32_t *d_b, uint64_t n, uint32_t scale, uint32_t *d_out,
                         zkie_stream_t stream);
/* PadIdx (:1279-1283): out = base resized to len (zeros past nb). */
int zkie2_op_pad_idx(const uint32_t *d_base, uint64_t nb, uint64_t len, uint32_t *d_out, zkie_stream_t stream);
/* RoPE forward (rope.rs:87-124): x is m x heads x d (n values, d even), cos /
 * sin m x d/2; rotate-half in wrapping i64, rounded by 2^shift. */
int zkie2_op_rope(const uint64_t *d_x, uint64_t n, const uint64_t *d_cos, const uint64_t *d_sin, uint64_t m,
                  uint64_t d, uint32_t shift, uint64_t *d_out, zkie_stream_t stream);
/* The columns prove_rope reads (rope.rs:126-150), n / 2 values each:
 * d_cols = {x_f, x_s, out_f, out_s, cos_b, sin_b, rem_f, rem_s}. */
int zkie2_op_rope_columns(const uint64_t *d_x, const uint64_t *d_out, uint64_t n, const uint64_t *d_cos,
                          const uint64_t *d_sin, uint64_t m, uint64_t d, uint32_t shift, uint64_t *const *d_cols,
                          zkie_stream_t stream);
/* Ones of the m x n one-hot sel (field value 1) per token row (by_token, m
 * counts) or per expert column (n counts), u32.  Here and in the two scatter
 * entries below, m and n must be below 2^32 (ids and counts are u32): larger
 * sizes return cudaErrorInvalidValue. */
int zkie2_op_sel_counts(const uint64_t *d_sel, uint64_t m, uint64_t n, uint32_t by_token, uint32_t *d_cnt,
                        zkie_stream_t stream);
/* scatter_forward (scatter.rs:12-25): for each expert in order, the tokens
 * routed to it; d_expert_cnt from zkie2_op_sel_counts(by_token = 0); the
 * outputs hold sum(d_expert_cnt) entries; d_scratch: n u64. */
int zkie2_op_scatter(const uint64_t *d_sel, uint64_t m, uint64_t n, const uint32_t *d_expert_cnt,
                     uint32_t *d_token_id, uint32_t *d_expert_of, uint64_t *d_scratch, zkie_stream_t stream);
/* prove_scatter's multisets (scatter.rs:27-55): d_a (room for m n values) =
 * the source encodings t n + e in token-major order (d_token_cnt from
 * sel_counts(by_token = 1)), d_b[pos] = token_id[pos] n + expert_of[pos] for
 * s positions; d_scratch: m u64.  Ones in sel other than s set bit 1 of
 * *d_err (the reference asserts equal lengths). */
int zkie2_op_scatter_encodings(const uint64_t *d_sel, uint64_t m, uint64_t n, const uint32_t *d_token_cnt,
                               const uint32_t *d_token_id, const uint32_t *d_expert_of, uint64_t s, uint64_t *d_a,
                               uint64_t *d_b, uint64_t *d_scratch, uint32_t *d_err, zkie_stream_t stream);
/* build_perm_num_den (common/logup_gkr.rs:807-820) into total entries: num 1,
 * den alpha - v for i < len, then 0 / alpha. */
int zkie2_perm_num_den(const uint64_t *d_v, uint64_t len, uint64_t total, uint64_t alpha, uint64_t *d_num,
                       uint64_t *d_den, zkie_stream_t stream);
/* gather_forward (gather.rs:36-52): out[t] (h values) = the field sum over
 * the positions routed to t of weighted[pos] gate[pos]; s positions, m
 * tokens; scratch zkie2_op_gather_scratch_u32(s, m) u32 values.  A token id
 * at or past m sets bit 1 of *d_err.  s and m must be below 2^32 (the
 * offsets are u32): larger sizes return cudaErrorInvalidValue. */
uint64_t zkie2_op_gather_scratch_u32(uint64_t s, uint64_t m);
int zkie2_op_gather(const uint64_t *d_weighted, const uint32_t *d_token_id, const uint64_t *d_gate, uint64_t s,
                    uint64_t m, uint64_t h, uint64_t *d_out, uint32_t *d_scratch_u32, uint32_t *d_err,
                    zkie_stream_t stream);
/* prove_scatter_add's columns (gather.rs:70-141) into total entries: with
 * token ids and gate (the source side, rows = s positions) num = gamma[d]
 * vals gate[pos], den = alpha - token_id[pos]; without (the target side,
 * rows = m tokens) num = gamma[d] vals, den = alpha - t; then 0 / alpha.
 * d_cols = {num, den, gamma_b, gate_b (source side only), vals_pad}. */
int zkie2_scatter_add_columns(const uint64_t *d_vals, const uint64_t *d_gate, const uint32_t *d_token_id,
                              const uint64_t *d_gamma, uint64_t rows, uint64_t h, uint64_t total, uint64_t alpha,
                              uint64_t *const *d_cols, zkie_stream_t stream);
/* gather_w_v's gather step (batched_matmul.rs:219-245): out[pos k + d] =
 * wv[expert_of[pos] k + d] with wv the experts' weights contracted with
 * eq(v) (zkie2_mle_partial_eval); an expert id at or past n_experts sets bit
 * 1 of *d_err. */
int zkie2_expert_rows(const uint64_t *d_wv, const uint32_t *d_expert_of, uint64_t s, uint64_t k, uint64_t n_experts,
                      uint64_t *d_out, uint32_t *d_err, zkie_stream_t stream);
/* expert_counts and expert_table_evals (batched_matmul.rs:247-277):
 * counts[e] = sum over positions of expert e of eq_pos[pos]; table[e] = sum_d
 * eq_d[d] wv[e k + d]. */
int zkie2_expert_open(const uint32_t *d_expert_of, uint64_t s, const uint64_t *d_eq_pos, const uint64_t *d_wv,
                      uint64_t k, const uint64_t *d_eq_d, uint64_t n_experts, uint64_t *d_counts, uint64_t *d_table,
                      zkie_stream_t stream);
/* The lookup columns of prove_topk (topk.rs:141-154) and prove_range_decomp
 * (:395-419) over n entries: to_i32(sel) and to_i32(d1) as u32 indices, and
 * the 16-bit limbs c0, c1, c2 of to_i64(d2) as u64, each as field values
 * (d_limbs, 3 n: limb c at c n) and as u32 indices (d_limb_idx, 3 n). */
int zkie2_op_topk_limbs(const uint64_t *d_sel, const uint64_t *d_d1, const uint64_t *d_d2, uint64_t n,
                        uint32_t *d_sel_idx, uint32_t *d_d1_idx, uint64_t *d_limbs, uint32_t *d_limb_idx,
                        zkie_stream_t stream);
/* prove_same_poly (common/same_poly.rs:13-45) as one degree-2 virtual
 * polynomial: every term of the reference's is c_i f eq(r_i, .), so its
 * round messages are those of f E with E = sum_i c_i eq(r_i, .).  This
 * builds E (2^t values) from c points r_i (h_points, c x t, t <= 40) and
 * coefficients; the points travel as kernel parameters (no host copy, so the
 * call can be recorded in a CUDA graph). */
uint64_t zkie2_eq_combine_scratch_elems(uint32_t c, uint32_t t);
int zkie2_eq_combine(const uint64_t *h_points, const uint64_t *h_coeffs, uint32_t c, uint32_t t, uint64_t *d_out,
                     uint64_t *d_scratch, zkie_stream_t stream);

/* ---- multi-GPU context (NCCL) ------------------------------------------------------- */
/* One split commit and one split sumcheck over an NCCL communicator, one
 * process (or host thread) per GPU, G = a power of two ranks.  No reference
 * counterpart: the reference commits and proves on one device.  NCCL is
 * loaded at run time (libnccl.so.2); without it these calls return
 * cudaErrorSharedObjectInitFailed and the rest of the library is unaffected.
 * NCCL failures return ZKIE2_MG_NCCL_ERROR_BASE + the ncclResult_t.  Every
 * rank calls the collective entry points in the same order with the same
 * shapes; each call synchronizes its stream before returning. */
#define ZKIE2_MG_NCCL_ERROR_BASE 10000
#define ZKIE2_MG_UNIQUE_ID_BYTES 128
typedef struct zkie2_mg_ctx zkie2_mg_ctx;
/* 1 if NCCL could be loaded. */
int zkie2_mg_available(void);
/* ncclGetUniqueId into h_id (128 bytes), on one rank; the caller hands it to
 * every rank (its own transport). */
int zkie2_mg_unique_id(uint8_t *h_id);
/* A context with a new communicator of nranks ranks (this process = rank) on
 * the current device (the zkie2_mg_init(ncclComm_t[]) of the survey's
 * additive entry points, per rank). */
int zkie2_mg_init(const uint8_t *h_id, int nranks, int rank, zkie2_mg_ctx **out);
/* A context around a communicator the caller created (an ncclComm_t, e.g.
 * from its own NCCL binding); not destroyed by zkie2_mg_destroy. */
int zkie2_mg_init_comm(void *nccl_comm, zkie2_mg_ctx **out);
int zkie2_mg_destroy(zkie2_mg_ctx *ctx);
int zkie2_mg_rank(const zkie2_mg_ctx *ctx);
int zkie2_mg_size(const zkie2_mg_ctx *ctx);
/* Split commit of the L x w coefficient matrix d_coeffs (replicated on every
 * rank, L = 2^lg_l) at blowup 2^lg_blowup, H = L << lg_blowup rows,
 * G^2 <= H: rank g leaves with its LDE rows g, g + G, ... in d_lde
 * ((H/G) x w), the digest layers of its contiguous leaf block
 * [g H/G, (g+1) H/G) in d_layers (zkie2_merkle_total_digests(H/G) x 8), the
 * layers above the G subtree roots in d_top (zkie2_mg_top_digests(G) x 8) and
 * the root of the single-device commit (zkie2_commit) in h_root (8 u64).
 * d_scratch: zkie2_mg_split_commit_scratch_elems (0 = unsupported shape). */
uint64_t zkie2_mg_split_commit_scratch_elems(uint32_t lg_l, uint32_t lg_blowup, uint64_t w, int nranks);
uint64_t zkie2_mg_top_digests(int nranks);
int zkie2_mg_split_commit(zkie2_mg_ctx *ctx, const uint64_t *d_coeffs, uint32_t lg_l, uint32_t lg_blowup, uint64_t w,
                          uint64_t *d_lde, uint64_t *d_layers, uint64_t *d_top, uint64_t *d_scratch,
                          uint64_t *h_root, zkie_stream_t stream);
/* The same split commit from host buffers (the end-to-end path of a rank):
 * h_part holds this rank's rows [g L/G, (g+1) L/G) of the L x w coefficient
 * matrix (pinned host memory for overlap); the root (8 u64) comes back in
 * h_root, this rank's LDE rows g, g + G, ... in h_lde ((H/G) x w) and its
 * subtree's digest layers in h_layers (zkie2_merkle_total_digests(H/G) x 8)
 * when those are non-null.  Pipelined over about four column blocks on the
 * context's own streams: the upload of block j + 1, the NVLink all-gather of
 * block j's rows from every rank, its coset LDE and leaf-sponge absorption,
 * and the download of its LDE rows overlap.  Synchronous; d_scratch:
 * zkie2_mg_split_commit_host_scratch_elems (0 = unsupported shape). */
uint64_t zkie2_mg_split_commit_host_scratch_elems(uint32_t lg_l, uint32_t lg_blowup, uint64_t w, int nranks);
int zkie2_mg_split_commit_host(zkie2_mg_ctx *ctx, const uint64_t *h_part, uint32_t lg_l, uint32_t lg_blowup,
                               uint64_t w, uint64_t *h_lde, uint64_t *h_layers, uint64_t *h_root,
                               uint64_t *d_scratch);
/* sumcheck::prove (common/sumcheck.rs:33-79) of f, h of 2^t elements split
 * over the G ranks by the high variables: rank g passes its 2^t / G
 * contiguous elements [g 2^t/G, (g+1) 2^t/G) of each; h_ch the t challenges
 * (host, the same on every rank).  Every rank receives the single-device
 * proof: h_rounds (t x 3), h_finals (f_eval, h_eval).  log2 G <= t. */
uint64_t zkie2_mg_split_sumcheck_scratch_elems(uint32_t t, int nranks);
int zkie2_mg_split_sumcheck(zkie2_mg_ctx *ctx, const uint64_t *d_f, const uint64_t *d_h, uint32_t t,
                            const uint64_t *h_ch, uint64_t *h_rounds, uint64_t *h_finals, uint64_t *d_scratch,
                            zkie_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif
