/*
 * zkie_goldilocks_cuda.h -- the reference-facing GPU seam of zkIE, re-implemented
 * for sm_100a in libzkie_b200.so.
 *
 * These are exactly the symbols the reference's Rust FFI binds
 * (crates/zkie-core/src/pcs/cuda_ffi.rs:2-46), with the same signatures and
 * semantics as its CUDA sources:
 *
 *   - all pointers are device pointers owned by the caller;
 *   - work is enqueued asynchronously on the legacy default stream, so the
 *     caller's cudaMemcpy / cudaMemset / cudaDeviceSynchronize order it;
 *   - every call returns a cudaError_t as int (0 = success);
 *   - outputs are canonical Goldilocks elements (< p = 2^64 - 2^32 + 1);
 *     inputs may be any u64 (taken mod p).
 *
 * Differences, all on inputs the reference does not handle: a null pointer
 * with non-empty work returns cudaErrorInvalidValue (the reference would
 * fault on the device); hashing before zkie_p2_upload_constants returns
 * cudaErrorInitializationError (the reference would hash with zero constants).
 */
#ifndef ZKIE_GOLDILOCKS_CUDA_H
#define ZKIE_GOLDILOCKS_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Number of visible CUDA devices, 0 if CUDA is unusable.
 * Replaces crates/zkie-core/cuda/poseidon2_merkle.cu:315-318. */
int zkie_cuda_device_count(void);

/* Forward DFT of every column of the row-major h x w matrix d_mat
 * (h = 2^lg_h), in place, natural order, w = TWO_ADIC_GENERATORS[lg_h].
 * d_temp: h*w u64 of scratch.  d_tw: concatenated per-stage twiddles, stage s
 * (1..lg_h) at offset 2^(s-1) - 1 holding TWO_ADIC_GENERATORS[s]^j,
 * j < 2^(s-1) (the table built by crates/zkie-core/src/pcs/dft_cuda.rs:44-59).
 * lg_h == 0 or w == 0 is a no-op.
 * Replaces crates/zkie-core/cuda/goldilocks_ntt.cu:105-137. */
int zkie_ntt_forward_goldilocks(uint64_t *d_mat, uint64_t *d_temp, uint32_t lg_h, uint64_t w,
                                const uint64_t *d_tw);

/* Upload the Poseidon2-16 round constants to the current device:
 * rc_init / rc_final are 4 x 16 (initial / terminal external rounds),
 * rc_internal 22 values, diag15 entry 15 of the internal diagonal.
 * Replaces crates/zkie-core/cuda/poseidon2_merkle.cu:252-264. */
int zkie_p2_upload_constants(const uint64_t *rc_init, const uint64_t *rc_final,
                             const uint64_t *rc_internal, uint64_t diag15);

/* Leaf digests (PaddingFreeSponge<Perm,16,8,8>, 8 u64 each) of rows
 * [0, (h/8)*8) of the row-major h x w matrix mat into digests[row*8 ..].
 * Replaces crates/zkie-core/cuda/poseidon2_merkle.cu:266-275. */
int zkie_p2_leaf_batch(const uint64_t *mat, uint64_t *digests, uint32_t h, uint32_t w);

/* Leaf digests of rows [start_row, h).
 * Replaces crates/zkie-core/cuda/poseidon2_merkle.cu:277-287. */
int zkie_p2_leaf_scalar(const uint64_t *mat, uint64_t *digests, uint32_t start_row, uint32_t h,
                        uint32_t w);

/* Nodes [0, (next_len/8)*8) of the next layer: next[i] =
 * TruncatedPermutation(prev[step*i], prev[step*i+1] if step == 2, zero-padded).
 * Replaces crates/zkie-core/cuda/poseidon2_merkle.cu:289-299. */
int zkie_p2_compress_batch(const uint64_t *prev, uint64_t *next, uint32_t next_len, uint32_t step);

/* Nodes [from, to) of the next layer.
 * Replaces crates/zkie-core/cuda/poseidon2_merkle.cu:301-311. */
int zkie_p2_compress_scalar(const uint64_t *prev, uint64_t *next, uint32_t from, uint32_t to,
                            uint32_t step);

#ifdef __cplusplus
}
#endif
#endif
