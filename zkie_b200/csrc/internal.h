// internal.h -- host-side launch API shared between the translation units of
// libzkie_b200 (not exported).
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

namespace zk {

// ---- Poseidon2 / Merkle (poseidon2.cu) --------------------------------------
// Constants must be present on the current device before any hashing launch.
bool p2_constants_ready();
int p2_upload(const uint64_t* rc_init, const uint64_t* rc_final, const uint64_t* rc_internal,
              uint64_t diag15);
// Derive the reference's default constants (SmallRng seed 1) and upload them
// to the current device if nothing was uploaded there yet.
int p2_ensure_default();

int launch_leaf_rows(const uint64_t* mat, uint64_t* digests, uint64_t row0, uint64_t row_end,
                     uint64_t w, cudaStream_t s);
int launch_compress(const uint64_t* prev, uint64_t* next, uint64_t from, uint64_t to,
                    uint32_t step, cudaStream_t s);
// Leaf sponge over columns [c0, c0 + cn) of each of h rows (row stride ld,
// c0 a multiple of 8); per-row states (16 u64) carried in `states` between
// column blocks; the last block writes the digests.
int launch_leaf_absorb(const uint64_t* mat, uint64_t ld, uint64_t c0, uint64_t cn, uint64_t h, uint64_t* states,
                       uint64_t* digests, bool first, bool last, cudaStream_t s);

// Merkle layer geometry of one matrix of h rows (pcs/merkle_cuda.rs:203-209).
struct MerkleGeom {
    std::vector<uint64_t> len;     // padded length of each layer
    std::vector<uint64_t> offset;  // digest offset of each layer in the flat buffer
    uint64_t total = 0;            // total digests
};
MerkleGeom merkle_geometry(uint64_t h);
// Hash every row and build every layer into `layers` (flat, geometry above).
int merkle_build(const uint64_t* mat, uint64_t h, uint64_t w, uint64_t* layers, cudaStream_t s);
// Build layers 1.. from a leaf layer already in layers[0 .. h).
int merkle_build_from_leaves(uint64_t h, uint64_t* layers, cudaStream_t s);

// ---- NTT (ntt.cu) ------------------------------------------------------------
// Zero-padded LDE of every column: in is L x w (L = 2^lg_l), out is
// (L << lg_blowup) x w, scratch holds (L << lg_blowup) * w u64.
int lde_launch(const uint64_t* in, uint64_t* out, uint64_t* scratch, uint32_t lg_l,
               uint32_t lg_blowup, uint64_t w, cudaStream_t s);
// The same on w columns of wider matrices: in, out and scratch all have row
// stride ld (e.g. a column block, pointers offset to its first column).
int lde_launch_ld(const uint64_t* in, uint64_t* out, uint64_t* scratch, uint32_t lg_l, uint32_t lg_blowup,
                  uint64_t w, uint64_t ld, cudaStream_t s);
uint64_t lde_scratch_elems(uint32_t lg_l, uint32_t lg_blowup, uint64_t w);

// ---- commit / GKR pieces used by the fused shard prove (shard.cu) ------------------
int commit_device(const uint64_t* d_in, uint32_t lg_l, uint32_t lg_blowup, uint64_t w, uint64_t* d_lde,
                  uint64_t* d_layers, uint64_t* d_scratch, cudaStream_t s);
int matmul_field_dev(const uint64_t* d_a, const uint64_t* d_b, uint64_t m, uint64_t k, uint64_t n,
                     uint64_t* d_c, cudaStream_t s);
uint64_t op_matmul_scratch_elems(uint64_t m, uint64_t k, uint64_t n);
int op_matmul_enqueue(const uint64_t* d_a, const uint64_t* d_b, const uint64_t* d_c, uint64_t m, uint64_t k,
                      uint64_t n, const uint64_t* u, const uint64_t* v, const uint64_t* ch, uint64_t* d_scratch,
                      uint64_t** d_out, cudaStream_t s);

// ---- virtual sumcheck and MLE pieces used by the LogUp fraction tree (logup.cu) -----
uint64_t virtual_plan_elems(uint32_t n_mles, uint32_t t);
int virtual_enqueue(const uint64_t* const* d_mles, uint32_t n_mles, uint32_t t, const uint64_t* coeffs,
                    const uint32_t* idx_off, const uint32_t* idx, uint32_t n_terms, const uint64_t* h_ch,
                    uint64_t* d_rounds, uint64_t* d_finals, uint32_t* deg_out, uint64_t* d_scratch,
                    cudaStream_t stream, bool tree_layer = false);
int eq_table_dev(const uint64_t* h_r, uint32_t d, uint64_t* d_out, cudaStream_t s);
// prove_fractional_with_challenges enqueued (logup.cu), outputs left in d_scratch
int fractional_enqueue(const uint64_t* d_num, const uint64_t* d_den, uint32_t lg_n, const uint64_t* h_full_r,
                       const uint64_t* h_cs, uint64_t* d_scratch, cudaStream_t stream, uint64_t** d_rounds,
                       uint64_t** d_finals, uint64_t** d_nd, uint64_t* n_rounds);

// ---- host-side primitives (host.cpp) -------------------------------------------
void p2_derive_constants_host(uint64_t seed, uint64_t rc_init[64], uint64_t rc_final[64],
                              uint64_t rc_internal[22], uint64_t* diag15);
uint64_t gl_mul_host(uint64_t a, uint64_t b);
uint64_t gl_add_host(uint64_t a, uint64_t b);
uint64_t gl_sub_host(uint64_t a, uint64_t b);
uint64_t gl_pow_host(uint64_t a, uint64_t e);
uint64_t two_adic_generator_host(uint32_t bits);

}  // namespace zk
