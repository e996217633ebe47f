// poseidon2.cu -- Poseidon2 Merkle hashing kernels and the reference-facing
// zkie_p2_* entry points (crates/zkie-core/cuda/poseidon2_merkle.cu:252-318).
//
// Hash configuration (pcs/merkle_cuda.rs:39-45): Poseidon2Goldilocks<16>,
// leaves PaddingFreeSponge<Perm,16,8,8>, nodes TruncatedPermutation<Perm,2,8,16>,
// binary tree, 8-element digests.
//
// Design: one thread per row (leaf) or per node; the 16-element state stays
// in registers, the round constants in __constant__ memory.  Unlike the
// reference (one thread serially hashing 8 rows), every thread hashes one
// row, so a launch exposes 8x more parallelism and the integer pipes stay fed.
#include <mutex>

#include "../../include/zkie_goldilocks_cuda.h"
#include "../../include/zkie2.h"
#include "common.cuh"
#include "internal.h"
#include "poseidon2.cuh"

namespace zk {

__constant__ P2Const c_p2;

namespace {
std::mutex g_p2_mu;
bool g_p2_ready[kMaxDevices];

constexpr int kHashThreads = 128;
// Up to this many states per launch the four-threads-per-state kernels run:
// such a launch is bound by one permutation's latency, which the
// cooperative form cuts by about 3x.  Larger launches take one thread per
// state (fewer instructions per permutation).  Measured on the bench's tree
// and the configuration-1 shard: the crossover lies between 2^12 and 2^14
// states (2^16 was 13 % slower on the shard, whose 2^16-row leaf launch is
// throughput-bound).
constexpr uint64_t kX4MaxStates = 1ull << 14;
// Up to this many states the sixteen-threads-per-state kernels run (a
// quarter of the four-thread form's latency per permutation).
constexpr uint64_t kX16MaxStates = 1ull << 11;

// Leaf digests of rows [row0, row_end): sponge with rate 8, overwrite mode,
// one permutation per full 8-block and one after a partial tail
// (poseidon2_merkle.cu:161-184).  Row r starts at mat + r*w.
__global__ void __launch_bounds__(kHashThreads)
    k_leaf_rows(const uint64_t* __restrict__ mat, uint64_t* __restrict__ digests, uint64_t row0,
                uint64_t row_end, uint64_t w) {
    const uint64_t row = row0 + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= row_end) return;
    const uint64_t* src = mat + row * w;
    uint64_t s[16];
#pragma unroll
    for (int i = 0; i < 16; i++) s[i] = 0;
    const uint64_t nblk = (w + 7) >> 3;
    const bool vec = ((w & 1) == 0) && ((reinterpret_cast<uintptr_t>(mat) & 15) == 0);
    for (uint64_t b = 0; b < nblk; b++) {
        const uint64_t base = b << 3;
        const uint64_t n = (w - base) < 8 ? (w - base) : 8;
        if (n == 8 && vec) {
            const ulonglong2* p = reinterpret_cast<const ulonglong2*>(src + base);
#pragma unroll
            for (int q = 0; q < 4; q++) {
                ulonglong2 v = __ldg(p + q);
                s[2 * q] = v.x;
                s[2 * q + 1] = v.y;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 8; i++)
                if ((uint64_t)i < n) s[i] = __ldg(src + base + i);
        }
        p2_permute(s, c_p2);
    }
    ulonglong2* dst = reinterpret_cast<ulonglong2*>(digests + row * 8);
#pragma unroll
    for (int q = 0; q < 4; q++) dst[q] = make_ulonglong2(gl_canon(s[2 * q]), gl_canon(s[2 * q + 1]));
}

// Node i of the next layer: state = [prev[step*i], prev[step*i+1] (if step
// is 2), zeros], permute, keep state[0..8] (poseidon2_merkle.cu:212-225).
__global__ void __launch_bounds__(kHashThreads)
    k_compress(const uint64_t* __restrict__ prev, uint64_t* __restrict__ next, uint64_t from,
               uint64_t to, uint32_t step) {
    const uint64_t i = from + (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= to) return;
    const ulonglong2* src = reinterpret_cast<const ulonglong2*>(prev + (uint64_t)step * i * 8);
    uint64_t s[16];
#pragma unroll
    for (int q = 0; q < 4; q++) {
        ulonglong2 v = __ldg(src + q);
        s[2 * q] = v.x;
        s[2 * q + 1] = v.y;
    }
    if (step >= 2) {
#pragma unroll
        for (int q = 0; q < 4; q++) {
            ulonglong2 v = __ldg(src + 4 + q);
            s[8 + 2 * q] = v.x;
            s[8 + 2 * q + 1] = v.y;
        }
    } else {
#pragma unroll
        for (int i2 = 8; i2 < 16; i2++) s[i2] = 0;
    }
    p2_permute(s, c_p2);
    ulonglong2* dst = reinterpret_cast<ulonglong2*>(next + i * 8);
#pragma unroll
    for (int q = 0; q < 4; q++) dst[q] = make_ulonglong2(gl_canon(s[2 * q]), gl_canon(s[2 * q + 1]));
}

// The leaf sponge over one block of columns [c0, c0 + cn) of every row (rows
// of stride ld), so hashing can run while later column blocks are still
// being uploaded and transformed.  c0 is a multiple of 8, so block
// boundaries are absorption boundaries and the result equals k_leaf_rows.
// The 16-element state of each row waits in `states` between blocks; the
// first block starts from zeros, the last writes the digest.
__global__ void __launch_bounds__(kHashThreads)
    k_leaf_absorb(const uint64_t* __restrict__ mat, uint64_t ld, uint64_t c0, uint64_t cn, uint64_t h,
                  uint64_t* __restrict__ states, uint64_t* __restrict__ digests, int first, int last) {
    const uint64_t row = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= h) return;
    uint64_t s[16];
    ulonglong2* sp = reinterpret_cast<ulonglong2*>(states + row * 16);
    if (first) {
#pragma unroll
        for (int i = 0; i < 16; i++) s[i] = 0;
    } else {
#pragma unroll
        for (int q = 0; q < 8; q++) {
            const ulonglong2 v = sp[q];
            s[2 * q] = v.x;
            s[2 * q + 1] = v.y;
        }
    }
    const uint64_t* src = mat + row * ld + c0;
    const uint64_t nblk = (cn + 7) >> 3;
    for (uint64_t b = 0; b < nblk; b++) {
        const uint64_t base = b << 3;
        const uint64_t n = (cn - base) < 8 ? (cn - base) : 8;
#pragma unroll
        for (int i = 0; i < 8; i++)
            if ((uint64_t)i < n) s[i] = __ldg(src + base + i);
        p2_permute(s, c_p2);
    }
    if (last) {
        ulonglong2* dst = reinterpret_cast<ulonglong2*>(digests + row * 8);
#pragma unroll
        for (int q = 0; q < 4; q++) dst[q] = make_ulonglong2(gl_canon(s[2 * q]), gl_canon(s[2 * q + 1]));
    } else {
#pragma unroll
        for (int q = 0; q < 8; q++) sp[q] = make_ulonglong2(s[2 * q], s[2 * q + 1]);
    }
}

// Latency-bound shapes (few rows or nodes): the same leaf sponge and
// compression with four threads per state (p2_permute_x4).  Lane g of each
// aligned 4-lane group holds state lanes 4g..4g+3; g = 0, 1 hold the rate and
// the digest.  Groups past the end still run the permutation (the shuffles
// need every lane) but load zeros and store nothing.
__global__ void __launch_bounds__(kHashThreads)
    k_leaf_rows_x4(const uint64_t* __restrict__ mat, uint64_t* __restrict__ digests, uint64_t row0,
                   uint64_t row_end, uint64_t w) {
    const uint64_t row = row0 + (((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 2);
    const uint32_t g = threadIdx.x & 3;
    const bool ok = row < row_end;
    const uint64_t* src = mat + (ok ? row : row0) * w;
    uint64_t v[4] = {0, 0, 0, 0};
    const uint64_t nblk = (w + 7) >> 3;
    for (uint64_t b = 0; b < nblk; b++) {
        const uint64_t base = b << 3;
        const uint64_t n = (w - base) < 8 ? (w - base) : 8;
        if (ok && g < 2) {
#pragma unroll
            for (int j = 0; j < 4; j++)
                if (4 * g + j < n) v[j] = __ldg(src + base + 4 * g + j);
        }
        p2_permute_x4(v, g, c_p2);
    }
    if (ok && g < 2) {
        ulonglong2* dst = reinterpret_cast<ulonglong2*>(digests + row * 8 + 4 * g);
        dst[0] = make_ulonglong2(gl_canon(v[0]), gl_canon(v[1]));
        dst[1] = make_ulonglong2(gl_canon(v[2]), gl_canon(v[3]));
    }
}

__global__ void __launch_bounds__(kHashThreads)
    k_compress_x4(const uint64_t* __restrict__ prev, uint64_t* __restrict__ next, uint64_t from, uint64_t to,
                  uint32_t step) {
    const uint64_t i = from + (((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 2);
    const uint32_t g = threadIdx.x & 3;
    const bool ok = i < to;
    uint64_t v[4] = {0, 0, 0, 0};
    if (ok && (g < 2 || step >= 2)) {
        const ulonglong2* src = reinterpret_cast<const ulonglong2*>(prev + ((uint64_t)step * i * 8 + 4 * g));
        const ulonglong2 a = __ldg(src), b = __ldg(src + 1);
        v[0] = a.x;
        v[1] = a.y;
        v[2] = b.x;
        v[3] = b.y;
    }
    p2_permute_x4(v, g, c_p2);
    if (ok && g < 2) {
        ulonglong2* dst = reinterpret_cast<ulonglong2*>(next + i * 8 + 4 * g);
        dst[0] = make_ulonglong2(gl_canon(v[0]), gl_canon(v[1]));
        dst[1] = make_ulonglong2(gl_canon(v[2]), gl_canon(v[3]));
    }
}

// The same with sixteen threads per state (p2_permute_x16): lane l of each
// aligned 16-lane group holds state element l; lanes 0-7 are the rate and the
// digest.  Groups past the end still run the permutation (full-mask
// shuffles) but load zeros and store nothing.  Each lane loads one element
// per absorbed block, so a group reads 64 consecutive bytes of its row.
__global__ void __launch_bounds__(kHashThreads)
    k_leaf_rows_x16(const uint64_t* __restrict__ mat, uint64_t* __restrict__ digests, uint64_t row0,
                    uint64_t row_end, uint64_t w) {
    const uint64_t row = row0 + (((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 4);
    const uint32_t l = threadIdx.x & 15;
    const bool ok = row < row_end;
    const uint64_t* src = mat + (ok ? row : row0) * w;
    uint64_t x = 0;
    const uint64_t nblk = (w + 7) >> 3;
    for (uint64_t b = 0; b < nblk; b++) {
        const uint64_t base = b << 3;
        const uint64_t n = (w - base) < 8 ? (w - base) : 8;
        if (ok && l < n) x = __ldg(src + base + l);  // overwrite the rate; a partial tail keeps stale lanes
        x = p2_permute_x16(x, l, c_p2);
    }
    if (ok && l < 8) digests[row * 8 + l] = gl_canon(x);
}

__global__ void __launch_bounds__(kHashThreads)
    k_compress_x16(const uint64_t* __restrict__ prev, uint64_t* __restrict__ next, uint64_t from, uint64_t to,
                   uint32_t step) {
    const uint64_t i = from + (((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 4);
    const uint32_t l = threadIdx.x & 15;
    const bool ok = i < to;
    // state [left(8), right(8)] (step 2) or [child(8), 0(8)] (step 1): the
    // children are consecutive digests, so lane l reads element l of them
    uint64_t x = (ok && l < 8 * step) ? __ldg(prev + (uint64_t)step * i * 8 + l) : 0;
    x = p2_permute_x16(x, l, c_p2);
    if (ok && l < 8) next[i * 8 + l] = gl_canon(x);
}

// Full permutations of a batch of 16-element states (tests and the
// permutation throughput probe used for the integer-pipe roofline).
__global__ void __launch_bounds__(kHashThreads)
    k_permute(uint64_t* __restrict__ states, uint64_t n, uint32_t reps) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint64_t s[16];
#pragma unroll
    for (int q = 0; q < 16; q++) s[q] = states[i * 16 + q];
    for (uint32_t r = 0; r < reps; r++) p2_permute(s, c_p2);
#pragma unroll
    for (int q = 0; q < 16; q++) states[i * 16 + q] = gl_canon(s[q]);
}

// Peak Goldilocks multiplication throughput: 8 independent multiply chains
// per thread in registers, no memory traffic in the loop.  The measured rate
// is the denominator of the hashing kernels' integer roofline.
__global__ void __launch_bounds__(kHashThreads) k_gl_mul_probe(uint64_t* __restrict__ buf, uint64_t n,
                                                              uint32_t iters) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint64_t x[8], y[8];
#pragma unroll
    for (int q = 0; q < 8; q++) {
        x[q] = buf[i * 16 + q];
        y[q] = buf[i * 16 + 8 + q];
    }
    for (uint32_t it = 0; it < iters; it++) {
#pragma unroll
        for (int q = 0; q < 8; q++) x[q] = gl_mul(x[q], y[q]);
    }
#pragma unroll
    for (int q = 0; q < 8; q++) buf[i * 16 + q] = gl_canon(x[q]);
}

// out digest c*G + r = in digest r*n + c (a G x n -> n x G transpose of
// 64-byte digests), one thread per u64 word.
__global__ void k_digest_interleave(const uint64_t* __restrict__ in, uint64_t G, uint64_t n,
                                    uint64_t* __restrict__ out) {
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= G * n * 8) return;
    const uint64_t d = idx >> 3, c = d / G, r = d - c * G;
    out[idx] = __ldg(in + ((r * n + c) << 3) + (idx & 7));
}

// PoW grinding (challenger.grind in the WHIR prover, p3-whir
// src/pcs/prover/mod.rs:240-245, 355-358) on the transcript's
// DuplexChallenger<Goldilocks, Poseidon2-16, 16, 8> (pcs/whir.rs:42).
// check_witness(bits, w) = observe(w); sample_bits(bits) == 0.  With len < 8
// inputs already buffered, observing w and sampling is one duplexing: the
// sponge lanes [0, len) take the buffered inputs, lane len takes w, the other
// lanes keep the sponge state, the state is permuted, and sample() pops the
// last of the eight outputs, lane 7.  `b` is that state with lane len to be
// replaced; w is valid when the canonical lane 7 has its low `bits` bits
// clear.  The smallest valid w of [start, start + count) lands in *found
// (atomicMin); a thread stops once a smaller witness is known.
struct GrindBase {
    uint64_t s[16];
};
__global__ void __launch_bounds__(kHashThreads)
    k_grind(GrindBase b, uint32_t len, uint64_t mask, uint64_t start, uint64_t count,
            unsigned long long* __restrict__ found) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += stride) {
        const uint64_t w = start + i;
        if (w >= *reinterpret_cast<volatile unsigned long long*>(found)) break;
        uint64_t s[16];
#pragma unroll
        for (int q = 0; q < 16; q++) s[q] = (uint32_t)q == len ? w : b.s[q];
        p2_permute(s, c_p2);
        if ((gl_canon(s[7]) & mask) == 0) atomicMin(found, (unsigned long long)w);
    }
}

uint64_t canon_host(uint64_t x) { return x >= GL_P ? x - GL_P : x; }

}  // namespace

bool p2_constants_ready() {
    int d = current_device();
    if (d < 0 || d >= kMaxDevices) return false;
    std::lock_guard<std::mutex> g(g_p2_mu);
    return g_p2_ready[d];
}

int p2_upload(const uint64_t* rc_init, const uint64_t* rc_final, const uint64_t* rc_internal,
              uint64_t diag15) {
    if (!rc_init || !rc_final || !rc_internal) return (int)cudaErrorInvalidValue;
    P2Const h;
    for (int r = 0; r < 4; r++)
        for (int i = 0; i < 16; i++) {
            h.ext[r][i] = canon_host(rc_init[r * 16 + i]);
            h.ext[4 + r][i] = canon_host(rc_final[r * 16 + i]);
        }
    for (int r = 0; r < 22; r++) h.internal[r] = canon_host(rc_internal[r]);
    h.diag15 = canon_host(diag15);
    int d = current_device();
    if (d < 0 || d >= kMaxDevices) return (int)cudaErrorInvalidDevice;
    ZK_TRY(cudaMemcpyToSymbol(c_p2, &h, sizeof(P2Const)));
    std::lock_guard<std::mutex> g(g_p2_mu);
    g_p2_ready[d] = true;
    return 0;
}

int p2_ensure_default() {
    if (p2_constants_ready()) return 0;
    uint64_t ri[64], rf[64], rp[22], d15;
    p2_derive_constants_host(1, ri, rf, rp, &d15);
    return p2_upload(ri, rf, rp, d15);
}

int launch_leaf_rows(const uint64_t* mat, uint64_t* digests, uint64_t row0, uint64_t row_end,
                     uint64_t w, cudaStream_t s) {
    if (row_end <= row0) return 0;
    if (!digests || (!mat && w != 0)) return (int)cudaErrorInvalidValue;
    const uint64_t n = row_end - row0;
    if (n <= kX16MaxStates)
        k_leaf_rows_x16<<<(unsigned)ceil_div(16 * n, kHashThreads), kHashThreads, 0, s>>>(mat, digests, row0,
                                                                                       row_end, w);
    else if (n <= kX4MaxStates)
        k_leaf_rows_x4<<<(unsigned)ceil_div(4 * n, kHashThreads), kHashThreads, 0, s>>>(mat, digests, row0, row_end,
                                                                                     w);
    else
        k_leaf_rows<<<(unsigned)ceil_div(n, kHashThreads), kHashThreads, 0, s>>>(mat, digests, row0, row_end, w);
    ZK_LAUNCH_CHECK();
    return 0;
}

int launch_leaf_absorb(const uint64_t* mat, uint64_t ld, uint64_t c0, uint64_t cn, uint64_t h, uint64_t* states,
                       uint64_t* digests, bool first, bool last, cudaStream_t s) {
    if (h == 0) return 0;
    if (!mat || !states || !digests || (c0 & 7) || cn == 0) return (int)cudaErrorInvalidValue;
    k_leaf_absorb<<<(unsigned)ceil_div(h, kHashThreads), kHashThreads, 0, s>>>(mat, ld, c0, cn, h, states, digests,
                                                                              first ? 1 : 0, last ? 1 : 0);
    ZK_LAUNCH_CHECK();
    return 0;
}

int launch_compress(const uint64_t* prev, uint64_t* next, uint64_t from, uint64_t to, uint32_t step,
                    cudaStream_t s) {
    if (to <= from) return 0;
    if (!prev || !next || step < 1 || step > 2) return (int)cudaErrorInvalidValue;
    const uint64_t n = to - from;
    if (n <= kX16MaxStates)
        k_compress_x16<<<(unsigned)ceil_div(16 * n, kHashThreads), kHashThreads, 0, s>>>(prev, next, from, to,
                                                                                        step);
    else if (n <= kX4MaxStates)
        k_compress_x4<<<(unsigned)ceil_div(4 * n, kHashThreads), kHashThreads, 0, s>>>(prev, next, from, to, step);
    else
        k_compress<<<(unsigned)ceil_div(n, kHashThreads), kHashThreads, 0, s>>>(prev, next, from, to, step);
    ZK_LAUNCH_CHECK();
    return 0;
}

static uint64_t padded_len(uint64_t raw, uint64_t n) {
    if (raw <= 1) return raw;
    if (raw >= n) return (raw + n - 1) / n * n;
    return n;
}

MerkleGeom merkle_geometry(uint64_t h) {
    MerkleGeom g;
    uint64_t len = padded_len(h, 2), off = 0;
    g.len.push_back(len);
    g.offset.push_back(off);
    off += len;
    while (len > 1) {
        len = padded_len(len / 2, 2);
        g.len.push_back(len);
        g.offset.push_back(off);
        off += len;
    }
    g.total = off;
    return g;
}

int merkle_build_from_leaves(uint64_t h, uint64_t* layers, cudaStream_t s) {
    MerkleGeom g = merkle_geometry(h);
    // Padding slots hold the default (zero) digest.
    if (g.len[0] > h) ZK_TRY(cudaMemsetAsync(layers + 8 * h, 0, 64 * (g.len[0] - h), s));
    for (size_t i = 0; i + 1 < g.len.size(); i++) {
        uint64_t raw = g.len[i] / 2;
        uint64_t* prev = layers + 8 * g.offset[i];
        uint64_t* next = layers + 8 * g.offset[i + 1];
        if (g.len[i + 1] > raw) ZK_TRY(cudaMemsetAsync(next + 8 * raw, 0, 64 * (g.len[i + 1] - raw), s));
        int rc = launch_compress(prev, next, 0, raw, 2, s);
        if (rc) return rc;
    }
    return 0;
}

int merkle_build(const uint64_t* mat, uint64_t h, uint64_t w, uint64_t* layers, cudaStream_t s) {
    if (h == 0) return (int)cudaErrorInvalidValue;
    int rc = launch_leaf_rows(mat, layers, 0, h, w, s);
    if (rc) return rc;
    return merkle_build_from_leaves(h, layers, s);
}

}  // namespace zk

using namespace zk;

// ============================================================================
// Reference-facing entry points (same names, signatures and semantics as
// crates/zkie-core/cuda/poseidon2_merkle.cu:252-318, bound in
// crates/zkie-core/src/pcs/cuda_ffi.rs:19-45).  Default stream, asynchronous;
// return the CUDA error code.  Where the reference would dereference a null
// pointer on the device, these return cudaErrorInvalidValue instead.
// ============================================================================
extern "C" {

int zkie_p2_upload_constants(const uint64_t* rc_init, const uint64_t* rc_final,
                             const uint64_t* rc_internal, uint64_t diag15) {
    return p2_upload(rc_init, rc_final, rc_internal, diag15);
}

int zkie_p2_leaf_batch(const uint64_t* mat, uint64_t* digests, uint32_t h, uint32_t w) {
    uint64_t rows = (uint64_t)(h / 8) * 8;
    if (rows == 0) return 0;
    if (!p2_constants_ready()) return (int)cudaErrorInitializationError;
    return launch_leaf_rows(mat, digests, 0, rows, w, 0);
}

int zkie_p2_leaf_scalar(const uint64_t* mat, uint64_t* digests, uint32_t start_row, uint32_t h,
                        uint32_t w) {
    if (start_row >= h) return 0;
    if (!p2_constants_ready()) return (int)cudaErrorInitializationError;
    return launch_leaf_rows(mat, digests, start_row, h, w, 0);
}

int zkie_p2_compress_batch(const uint64_t* prev, uint64_t* next, uint32_t next_len, uint32_t step) {
    uint64_t n = (uint64_t)(next_len / 8) * 8;
    if (n == 0) return 0;
    if (!p2_constants_ready()) return (int)cudaErrorInitializationError;
    return launch_compress(prev, next, 0, n, step, 0);
}

int zkie_p2_compress_scalar(const uint64_t* prev, uint64_t* next, uint32_t from, uint32_t to,
                            uint32_t step) {
    if (from >= to) return 0;
    if (!p2_constants_ready()) return (int)cudaErrorInitializationError;
    return launch_compress(prev, next, from, to, step, 0);
}

int zkie_cuda_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return n;
}

// ---- new entry points --------------------------------------------------------
int zkie2_p2_default_constants(uint64_t seed, uint64_t* rc_init, uint64_t* rc_final,
                               uint64_t* rc_internal, uint64_t* diag15) {
    if (!rc_init || !rc_final || !rc_internal || !diag15) return (int)cudaErrorInvalidValue;
    p2_derive_constants_host(seed, rc_init, rc_final, rc_internal, diag15);
    return 0;
}

int zkie2_p2_init_default(void) { return p2_ensure_default(); }

int zkie2_p2_permute(uint64_t* d_states, uint64_t n, uint32_t reps, cudaStream_t stream) {
    if (n == 0) return 0;
    if (!d_states) return (int)cudaErrorInvalidValue;
    if (!p2_constants_ready()) return (int)cudaErrorInitializationError;
    k_permute<<<(unsigned)ceil_div(n, kHashThreads), kHashThreads, 0, stream>>>(d_states, n, reps);
    ZK_LAUNCH_CHECK();
    return 0;
}

uint64_t zkie2_grind_batch(uint32_t bits) {
    const uint32_t lg = bits + 2 < 16 ? 16 : (bits + 2 > 26 ? 26 : bits + 2);
    return 1ull << lg;
}

int zkie2_grind(const uint64_t* h_sponge, const uint64_t* h_input, uint32_t len, uint32_t bits, uint64_t* h_witness,
                cudaStream_t stream) {
    if (!h_sponge || !h_witness || len >= 8 || (len && !h_input) || bits >= 63) return (int)cudaErrorInvalidValue;
    int rc = p2_ensure_default();
    if (rc) return rc;
    GrindBase b{};
    for (int q = 0; q < 16; q++) b.s[q] = gl_canon(h_sponge[q]);
    for (uint32_t q = 0; q < len; q++) b.s[q] = gl_canon(h_input[q]);
    const uint64_t mask = (1ull << bits) - 1;
    unsigned long long* d_found = nullptr;
    ZK_TRY(cudaMallocAsync((void**)&d_found, 8, stream));
    // One wave of resident blocks: the grid-stride loop then walks the
    // candidates in increasing order across all threads at once, so the
    // search stops close to the smallest witness instead of finishing the
    // ranges of the first resident blocks while later blocks wait.
    int dev = 0, sms = 0, per_sm = 0;
    ZK_TRY(cudaGetDevice(&dev));
    ZK_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    ZK_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_grind, kHashThreads, 0));
    const uint64_t resident = (uint64_t)(sms > 0 ? sms : 1) * (uint64_t)(per_sm > 0 ? per_sm : 1);
    const uint64_t batch = zkie2_grind_batch(bits);
    const uint64_t none = ~0ull;
    uint64_t got = none;
    // batches in increasing order: the first batch holding a witness yields the smallest one
    for (uint64_t start = 0; !rc && got == none && start < GL_P; start += batch) {
        const uint64_t count = GL_P - start < batch ? GL_P - start : batch;
        rc = (int)cudaMemcpyAsync(d_found, &none, 8, cudaMemcpyHostToDevice, stream);
        if (!rc) {
            const uint64_t blocks = ceil_div(count, kHashThreads);
            k_grind<<<(unsigned)(blocks < resident ? blocks : resident), kHashThreads, 0, stream>>>(b, len, mask, start,
                                                                                            count, d_found);
            rc = (int)cudaGetLastError();
        }
        if (!rc) rc = (int)cudaMemcpyAsync(&got, d_found, 8, cudaMemcpyDeviceToHost, stream);
        if (!rc) rc = (int)cudaStreamSynchronize(stream);
    }
    cudaFreeAsync(d_found, stream);
    if (rc) return rc;
    if (got == none) return (int)cudaErrorInvalidValue;  // no witness in the field (not for bits < 63)
    *h_witness = got;
    return 0;
}

int zkie2_gl_mul_probe(uint64_t* d_buf, uint64_t n, uint32_t iters, cudaStream_t stream) {
    if (n == 0) return 0;
    if (!d_buf) return (int)cudaErrorInvalidValue;
    k_gl_mul_probe<<<(unsigned)ceil_div(n, kHashThreads), kHashThreads, 0, stream>>>(d_buf, n, iters);
    ZK_LAUNCH_CHECK();
    return 0;
}

uint64_t zkie2_merkle_total_digests(uint64_t h) { return h ? merkle_geometry(h).total : 0; }

uint32_t zkie2_merkle_num_layers(uint64_t h) { return h ? (uint32_t)merkle_geometry(h).len.size() : 0; }

int zkie2_merkle_leaves(const uint64_t* d_mat, uint64_t h, uint64_t w, uint64_t* d_digests,
                        cudaStream_t stream) {
    if (!p2_constants_ready()) return (int)cudaErrorInitializationError;
    return launch_leaf_rows(d_mat, d_digests, 0, h, w, stream);
}

int zkie2_merkle_tree(const uint64_t* d_mat, uint64_t h, uint64_t w, uint64_t* d_layers,
                      cudaStream_t stream) {
    if (!p2_constants_ready()) return (int)cudaErrorInitializationError;
    if (!d_layers) return (int)cudaErrorInvalidValue;
    return merkle_build(d_mat, h, w, d_layers, stream);
}

int zkie2_merkle_tree_from_leaves(uint64_t h, uint64_t* d_layers, cudaStream_t stream) {
    if (!p2_constants_ready()) return (int)cudaErrorInitializationError;
    if (!d_layers || h == 0) return (int)cudaErrorInvalidValue;
    return merkle_build_from_leaves(h, d_layers, stream);
}

// Split commit: after the all-to-all of leaf digests a rank holds, for each of
// the G source ranks r, the n digests of rows r, r + G, r + 2G, ... of its
// leaf block; this puts them in row order (d_out[c*G + r] = d_in[r*n + c]).
int zkie2_digests_interleave(const uint64_t* d_in, uint64_t g, uint64_t n, uint64_t* d_out, cudaStream_t stream) {
    if (!d_in || !d_out || d_in == d_out) return (int)cudaErrorInvalidValue;
    const uint64_t words = g * n * 8;
    if (words == 0) return 0;
    k_digest_interleave<<<(unsigned)ceil_div(words, 256), 256, 0, stream>>>(d_in, g, n, d_out);
    ZK_LAUNCH_CHECK();
    return 0;
}

}  // extern "C"
