// poseidon2.cuh -- Poseidon2-16 permutation over Goldilocks, one thread per
// permutation (the state lives in 32 registers).
//
// Structure (crates/zkie-core/cuda/poseidon2_merkle.cu:37-155, the generic
// p3-poseidon2 permutation): initial light MDS; 4 external rounds (add round
// constants, x^7 on all 16 lanes, light MDS); 22 internal rounds (add constant
// and x^7 on lane 0, then state <- (1 + diag(V)) * state); 4 external rounds.
//
// Round constants live in __constant__ memory of the including translation
// unit (every warp reads the same constant: a broadcast).
#pragma once
#include "gl64.cuh"

namespace zk {

struct P2Const {
    uint64_t ext_init[4][16];
    uint64_t ext_final[4][16];
    uint64_t internal[22];
    uint64_t diag15;
};

ZK_HD uint64_t p2_sbox(uint64_t x) {
    uint64_t x2 = gl_sqr(x);
    uint64_t x3 = gl_mul(x2, x);
    uint64_t x4 = gl_sqr(x2);
    return gl_mul(x3, x4);
}

// [2 3 1 1; 1 2 3 1; 1 1 2 3; 3 1 1 2] on one 4-lane block.
ZK_HD void p2_mat4(uint64_t& x0, uint64_t& x1, uint64_t& x2, uint64_t& x3) {
    uint64_t t01 = gl_add(x0, x1);
    uint64_t t23 = gl_add(x2, x3);
    uint64_t t0123 = gl_add(t01, t23);
    uint64_t t01123 = gl_add(t0123, x1);
    uint64_t t01233 = gl_add(t0123, x3);
    uint64_t d0 = gl_add(x0, x0);
    uint64_t d2 = gl_add(x2, x2);
    x3 = gl_add(t01233, d0);
    x1 = gl_add(t01123, d2);
    x0 = gl_add(t01123, t01);
    x2 = gl_add(t01233, t23);
}

// Light external MDS: 4x4 block on each chunk, then add per-residue column sums.
ZK_HD void p2_mds_light(uint64_t s[16]) {
#pragma unroll
    for (int j = 0; j < 16; j += 4) p2_mat4(s[j], s[j + 1], s[j + 2], s[j + 3]);
    uint64_t sum[4];
#pragma unroll
    for (int k = 0; k < 4; k++) sum[k] = gl_add(gl_add(s[k], s[4 + k]), gl_add(s[8 + k], s[12 + k]));
#pragma unroll
    for (int i = 0; i < 16; i++) s[i] = gl_add(s[i], sum[i & 3]);
}

// Internal linear layer: s_i <- sum + V_i * s_i with
// V = [-2, 1, 2, 1/2, 3, 4, -1/2, -3, -4, 1/2^3, 1/2^4, 1/2^5, -1/2^3,
//      -1/2^4, -1/2^5, diag15] (poseidon2_merkle.cu:111-142).
ZK_HD void p2_internal_linear(uint64_t s[16], uint64_t diag15) {
    uint64_t sum = s[0];
#pragma unroll
    for (int i = 1; i < 16; i++) sum = gl_add(sum, s[i]);
    uint64_t t;
    s[0] = gl_sub(sum, gl_add(s[0], s[0]));
    s[1] = gl_add(sum, s[1]);
    s[2] = gl_add(sum, gl_add(s[2], s[2]));
    s[3] = gl_add(sum, gl_div_pow2<1>(s[3]));
    t = gl_add(s[4], s[4]);
    s[4] = gl_add(sum, gl_add(t, s[4]));
    t = gl_add(s[5], s[5]);
    s[5] = gl_add(sum, gl_add(t, t));
    s[6] = gl_sub(sum, gl_div_pow2<1>(s[6]));
    t = gl_add(s[7], s[7]);
    s[7] = gl_sub(sum, gl_add(t, s[7]));
    t = gl_add(s[8], s[8]);
    s[8] = gl_sub(sum, gl_add(t, t));
    s[9] = gl_add(sum, gl_div_pow2<3>(s[9]));
    s[10] = gl_add(sum, gl_div_pow2<4>(s[10]));
    s[11] = gl_add(sum, gl_div_pow2<5>(s[11]));
    s[12] = gl_sub(sum, gl_div_pow2<3>(s[12]));
    s[13] = gl_sub(sum, gl_div_pow2<4>(s[13]));
    s[14] = gl_sub(sum, gl_div_pow2<5>(s[14]));
    s[15] = gl_add(sum, gl_mul(s[15], diag15));
}

ZK_HD void p2_permute(uint64_t s[16], const P2Const& c) {
    p2_mds_light(s);
#pragma unroll 1
    for (int r = 0; r < 4; r++) {
#pragma unroll
        for (int i = 0; i < 16; i++) s[i] = p2_sbox(gl_add_c(s[i], c.ext_init[r][i]));
        p2_mds_light(s);
    }
    const uint64_t diag15 = c.diag15;
#pragma unroll 1
    for (int r = 0; r < 22; r++) {
        s[0] = p2_sbox(gl_add_c(s[0], c.internal[r]));
        p2_internal_linear(s, diag15);
    }
#pragma unroll 1
    for (int r = 0; r < 4; r++) {
#pragma unroll
        for (int i = 0; i < 16; i++) s[i] = p2_sbox(gl_add_c(s[i], c.ext_final[r][i]));
        p2_mds_light(s);
    }
}

}  // namespace zk
