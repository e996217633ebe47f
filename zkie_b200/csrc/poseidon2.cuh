// poseidon2.cuh -- Poseidon2-16 permutation over Goldilocks, one thread per
// permutation (the state lives in 32 registers).
//
// Structure (crates/zkie-core/cuda/poseidon2_merkle.cu:37-155, the generic
// p3-poseidon2 permutation): initial light MDS; 4 external rounds (add round
// constants, x^7 on all 16 lanes, light MDS); 22 internal rounds (add constant
// and x^7 on lane 0, then state <- (1 + diag(V)) * state); 4 external rounds.
//
// Cost shape on sm_100a: the integer ALU pipe (additions, carry folding) is
// the bottleneck, the multiply pipe has headroom.  So the S-box squares and
// multiplies with products whose cross terms are multiply-add carry chains
// (gl_sqr, gl_mul_madc: additions moved onto the multiply pipe), the linear layers add
// into 96-bit accumulators (3 instructions per addition) and reduce each
// output once, instead of reducing after every modular addition; and the
// eight external rounds share one loop body, the internal rounds nested after
// the fourth, to keep the code small enough for the instruction cache.
#pragma once
#include "gl64.cuh"

namespace zk {

constexpr uint64_t kInv2Pow32 = 0xFFFFFFFE00000002ull;  // 1/2^32 mod p

struct P2Const {
    uint64_t ext[8][16];  // rounds 0-3: initial external, 4-7: terminal external
    uint64_t internal[22];
    uint64_t diag15;
};

ZK_HD uint64_t p2_sbox(uint64_t x) {
    const uint64_t x2 = gl_sqr(x);
    const uint64_t x3 = gl_mul_madc(x2, x);
    const uint64_t x4 = gl_sqr(x2);
    return gl_mul_madc(x3, x4);
}

// [2 3 1 1; 1 2 3 1; 1 1 2 3; 3 1 1 2] on one 4-lane block, unreduced
// (every output is a sum of 7 inputs, below 7 * 2^64).
ZK_HD void p2_mat4_acc(uint64_t x0, uint64_t x1, uint64_t x2, uint64_t x3, Acc y[4]) {
    const Acc t01 = acc_sum(x0, x1);
    const Acc t23 = acc_sum(x2, x3);
    const Acc t0123 = acc_add(t01, t23);
    const Acc t01123 = acc_add(t0123, x1);
    const Acc t01233 = acc_add(t0123, x3);
    y[3] = acc_add(acc_add(t01233, x0), x0);  // 3x0 + x1 + x2 + 2x3
    y[1] = acc_add(acc_add(t01123, x2), x2);  // x0 + 2x1 + 3x2 + x3
    y[0] = acc_add(t01123, t01);              // 2x0 + 3x1 + x2 + x3
    y[2] = acc_add(t01233, t23);              // x0 + x1 + 2x2 + 3x3
}

// Reduced form of one block (tests and the reference-shaped helpers).
ZK_HD void p2_mat4(uint64_t& x0, uint64_t& x1, uint64_t& x2, uint64_t& x3) {
    Acc y[4];
    p2_mat4_acc(x0, x1, x2, x3, y);
    x0 = acc_reduce(y[0]);
    x1 = acc_reduce(y[1]);
    x2 = acc_reduce(y[2]);
    x3 = acc_reduce(y[3]);
}

// Light external MDS: 4x4 block on each chunk, then add the per-residue
// column sums.  Outputs are below 35 * 2^64 before the single reduction.
ZK_HD void p2_mds_light(uint64_t s[16]) {
    Acc y[16];
#pragma unroll
    for (int j = 0; j < 16; j += 4) p2_mat4_acc(s[j], s[j + 1], s[j + 2], s[j + 3], y + j);
    Acc sum[4];
#pragma unroll
    for (int k = 0; k < 4; k++) sum[k] = acc_add(acc_add(y[k], y[4 + k]), acc_add(y[8 + k], y[12 + k]));
#pragma unroll
    for (int i = 0; i < 16; i++) s[i] = acc_reduce(acc_add(y[i], sum[i & 3]));
}

// sum - V s for V in {2, 3, 4}, given vs = V s: (V + 1) p exceeds V s, so
// sum + (V + 1) p - V s is a non-negative accumulator below (V + 2) 2^64.
template <int V>
ZK_HD uint64_t p2_sum_minus(uint64_t sum, Acc vs) {
    const Acc c = acc_add(Acc{(uint64_t)0 - (uint64_t)(V + 1) * GL_EPS, (uint32_t)V}, sum);
    return acc_reduce(acc_sub(c, vs));
}

// Internal linear layer: s_i <- sum + V_i * s_i with
// V = [-2, 1, 2, 1/2, 3, 4, -1/2, -3, -4, 1/2^3, 1/2^4, 1/2^5, -1/2^3,
//      -1/2^4, -1/2^5, diag15] (poseidon2_merkle.cu:111-142).
ZK_HD void p2_internal_linear(uint64_t s[16], uint64_t diag15) {
    // the sum over the 32-bit halves (3-input additions), then recombined
    uint64_t lo = 0, hi = 0;
#pragma unroll
    for (int i = 0; i < 16; i++) {
        lo += (uint32_t)s[i];
        hi += s[i] >> 32;
    }
    // lo, hi < 2^36: lo + hi 2^32 < 2^69
    const Acc acc = acc_add(Acc{hi << 32, (uint32_t)(hi >> 32)}, lo);
    // canonical, so that sum + x needs a single carry fold (gl_add_c)
    const uint64_t sum = gl_canon(acc_reduce(acc));
    // integer V: one accumulator expression and one reduction per lane
    s[0] = p2_sum_minus<2>(sum, acc_shl<1>(s[0]));
    s[1] = gl_add_c(s[1], sum);
    s[2] = acc_reduce(acc_add(acc_shl<1>(s[2]), sum));
    s[3] = gl_add_c(gl_div_pow2<1>(s[3]), sum);
    s[4] = acc_reduce(acc_add(acc_add(acc_sum(sum, s[4]), s[4]), s[4]));
    s[5] = acc_reduce(acc_add(acc_shl<2>(s[5]), sum));
    s[6] = gl_sub(sum, gl_div_pow2<1>(s[6]));
    s[7] = p2_sum_minus<3>(sum, acc_add(acc_shl<1>(s[7]), s[7]));
    s[8] = p2_sum_minus<4>(sum, acc_shl<2>(s[8]));
    s[9] = gl_add_c(gl_div_pow2<3>(s[9]), sum);
    s[10] = gl_add_c(gl_div_pow2<4>(s[10]), sum);
    s[11] = gl_add_c(gl_div_pow2<5>(s[11]), sum);
    s[12] = gl_sub(sum, gl_div_pow2<3>(s[12]));
    s[13] = gl_sub(sum, gl_div_pow2<4>(s[13]));
    s[14] = gl_sub(sum, gl_div_pow2<5>(s[14]));
    // V_15 = 1/2^32 for the reference's constants: a division, not a product
    s[15] = gl_add_c(diag15 == kInv2Pow32 ? gl_div_pow2<32>(s[15]) : gl_mul(s[15], diag15), sum);
}

ZK_HD void p2_internal_round(uint64_t s[16], uint64_t rc, uint64_t diag15) {
    s[0] = p2_sbox(gl_add_c(s[0], rc));
    p2_internal_linear(s, diag15);
}

ZK_HD void p2_external_round(uint64_t s[16], const uint64_t rc[16]) {
#pragma unroll
    for (int i = 0; i < 16; i++) s[i] = p2_sbox(gl_add_c(s[i], rc[i]));
    p2_mds_light(s);
}

ZK_HD void p2_permute(uint64_t s[16], const P2Const& c) {
    p2_mds_light(s);
#pragma unroll 1
    for (int r = 0; r < 8; r++) {
        p2_external_round(s, c.ext[r]);
        if (r == 3) {
#pragma unroll 1
            for (int q = 0; q < 22; q++) p2_internal_round(s, c.internal[q], c.diag15);
        }
    }
}

#if defined(__CUDACC__)
// ---- four threads per permutation ---------------------------------------------------
// For latency-bound hashing (few rows or tree nodes), an aligned group of four
// lanes shares one state: lane g (= lane & 3) holds state lanes 4g .. 4g+3,
// which is exactly one 4x4 block of the external MDS.  Per external round a
// thread does its four S-boxes and its block locally; the per-residue column
// sums are two xor-shuffle steps.  Per internal round lane 0's S-box runs on
// g = 0, the full-state sum is a local sum plus two shuffle steps, and each
// thread applies its four diagonal entries as multiplications by the
// constants V_i.  The values equal the one-thread permutation's modulo p; the
// critical path is about a third as long.  Every lane of the warp must call
// this (the shuffles use the full mask).

// V_i of the internal layer as field elements (1/2^k = p - (p-1)/2^k).
__device__ __forceinline__ uint64_t p2_vdiag(uint32_t i, uint64_t diag15) {
    switch (i) {
        case 0: return GL_P - 2;
        case 1: return 1;
        case 2: return 2;
        case 3: return GL_P - (GL_P - 1) / 2;
        case 4: return 3;
        case 5: return 4;
        case 6: return (GL_P - 1) / 2;
        case 7: return GL_P - 3;
        case 8: return GL_P - 4;
        case 9: return GL_P - (GL_P - 1) / 8;
        case 10: return GL_P - (GL_P - 1) / 16;
        case 11: return GL_P - (GL_P - 1) / 32;
        case 12: return (GL_P - 1) / 8;
        case 13: return (GL_P - 1) / 16;
        case 14: return (GL_P - 1) / 32;
        default: return diag15;
    }
}

__device__ __forceinline__ uint64_t p2x4_group_sum(uint64_t x) {
    x = gl_add(x, __shfl_xor_sync(0xffffffffu, x, 1));
    return gl_add(x, __shfl_xor_sync(0xffffffffu, x, 2));
}

__device__ __forceinline__ void p2x4_mds_light(uint64_t v[4]) {
    Acc y[4];
    p2_mat4_acc(v[0], v[1], v[2], v[3], y);
#pragma unroll
    for (int k = 0; k < 4; k++) v[k] = acc_reduce(acc_add(y[k], p2x4_group_sum(acc_reduce(y[k]))));
}

__device__ __forceinline__ void p2_permute_x4(uint64_t v[4], uint32_t g, const P2Const& c) {
    uint64_t vd[4];
#pragma unroll
    for (int j = 0; j < 4; j++) vd[j] = p2_vdiag(4 * g + j, c.diag15);
    p2x4_mds_light(v);
#pragma unroll 1
    for (int r = 0; r < 8; r++) {
#pragma unroll
        for (int j = 0; j < 4; j++) v[j] = p2_sbox(gl_add_c(v[j], c.ext[r][4 * g + j]));
        p2x4_mds_light(v);
        if (r == 3) {
#pragma unroll 1
            for (int q = 0; q < 22; q++) {
                // Lane 0's S-box and the sum of the other fifteen lanes are
                // independent: every thread computes the S-box of its v[0]
                // (only group lane g = 0's is used; the warp issues it either
                // way) while the partial sum's shuffles run, then lane 0's
                // result is broadcast and added.
                const uint64_t t = p2_sbox(gl_add_c(v[0], c.internal[q]));
                const Acc a = acc_add(acc_add(acc_sum(v[1], v[2]), v[3]), g ? v[0] : 0ull);
                const uint64_t part = p2x4_group_sum(acc_reduce(a));
                const uint64_t t0 = __shfl_sync(0xffffffffu, t, 0, 4);
                const uint64_t sum = gl_canon(gl_add(part, t0));
                if (g == 0) v[0] = t;
#pragma unroll
                for (int j = 0; j < 4; j++) v[j] = gl_add_c(gl_mul(v[j], vd[j]), sum);
            }
        }
    }
}

// ---- sixteen threads per permutation ------------------------------------------------
// For the most latency-bound launches (the top levels of a tree, a few rows):
// lane l (= lane & 15) of an aligned 16-lane group holds state element l.  An
// external round is one S-box per lane, the 4x4 block row of the lane's
// position from three in-block shuffles, and the per-residue column sum from
// two xor-shuffle steps; an internal round is lane 0's S-box, a four-step
// xor-shuffle sum and one product by the lane's diagonal entry V_l.  The
// values equal the one-thread permutation's modulo p; the critical path is
// about a quarter of the four-thread form's.  Every lane of the warp must
// call this (full-mask shuffles, width 16).
__device__ __forceinline__ uint64_t p2x16_mds_light(uint64_t x, uint32_t l) {
    // block row of position k: out_k = 2 x_k + 3 x_{k+1} + x_{k+2} + x_{k+3} (circulant [2 3 1 1])
    const uint32_t base = l & ~3u, k = l & 3u;
    const uint64_t x1 = __shfl_sync(0xffffffffu, x, base | ((k + 1) & 3u), 16);
    const uint64_t x2 = __shfl_sync(0xffffffffu, x, base | ((k + 2) & 3u), 16);
    const uint64_t x3 = __shfl_sync(0xffffffffu, x, base | ((k + 3) & 3u), 16);
    const Acc y = acc_add(acc_add(acc_add(acc_add(acc_add(acc_sum(x, x), x1), x1), x1), x2), x3);  // < 7 2^64
    uint64_t c = acc_reduce(y);
    c = gl_add(c, __shfl_xor_sync(0xffffffffu, c, 4, 16));
    c = gl_add(c, __shfl_xor_sync(0xffffffffu, c, 8, 16));
    return acc_reduce(acc_add(y, c));
}

__device__ __forceinline__ uint64_t p2_permute_x16(uint64_t x, uint32_t l, const P2Const& c) {
    const uint64_t vd = p2_vdiag(l, c.diag15);
    x = p2x16_mds_light(x, l);
#pragma unroll 1
    for (int r = 0; r < 8; r++) {
        x = p2x16_mds_light(p2_sbox(gl_add_c(x, c.ext[r][l])), l);
        if (r == 3) {
#pragma unroll 1
            for (int q = 0; q < 22; q++) {
                // lane 0's S-box overlaps the shuffle sum of lanes 1-15 (as in
                // the four-thread form), then is broadcast into the sum
                const uint64_t t = p2_sbox(gl_add_c(x, c.internal[q]));
                uint64_t part = l ? x : 0ull;
                part = gl_add(part, __shfl_xor_sync(0xffffffffu, part, 1, 16));
                part = gl_add(part, __shfl_xor_sync(0xffffffffu, part, 2, 16));
                part = gl_add(part, __shfl_xor_sync(0xffffffffu, part, 4, 16));
                part = gl_add(part, __shfl_xor_sync(0xffffffffu, part, 8, 16));
                const uint64_t sum = gl_canon(gl_add(part, __shfl_sync(0xffffffffu, t, 0, 16)));
                x = gl_add_c(gl_mul(l ? x : t, vd), sum);
            }
        }
    }
    return x;
}
#endif

}  // namespace zk
