// devcheck.cu -- test-side self-check of the device arithmetic (TEST INFRASTRUCTURE).
//
// Runs the product's Goldilocks primitives and Poseidon2 stages (from
// zkie_b200/csrc/*.cuh) element-wise on the device and, from the same source,
// on the host, so a test can compare the two on identical inputs.  The host
// path is itself checked against the CPU oracle.  Constants are passed by
// value (kernel parameter), independent of the product's __constant__ upload.
#include <cuda_runtime.h>

#include <cstdint>

#include "../zkie_b200/csrc/dft_reg.cuh"
#include "../zkie_b200/csrc/poseidon2.cuh"

using namespace zk;

namespace {

ZK_HD uint64_t scalar_op(int op, uint64_t a, uint64_t b) {
    switch (op) {
        case 0: return gl_add(a, b);
        case 1: return gl_add_c(a, gl_canon(b));
        case 2: return gl_sub(a, b);
        case 3: return gl_mul(a, b);
        case 4: return gl_sqr(a);
        case 5: return gl_div_pow2<1>(a);
        case 6: return gl_div_pow2<3>(a);
        case 7: return gl_div_pow2<4>(a);
        case 8: return gl_div_pow2<5>(a);
        case 9: return gl_div_pow2<32>(a);
        case 10: return gl_canon(a);
        case 11: return p2_sbox(a);
        case 12: return mul_hi(a, b);
        case 13: return gl_reduce128(a, b);
        case 14: {
            Acc160 s = acc160_zero();
            acc160_mac(s, a, b);
            acc160_mac(s, a, a);
            acc160_mac(s, b, b);
            acc160_mac(s, a ^ b, ~a);
            return acc160_reduce(s);
        }
        case 15: {
            Acc160 s = acc160_zero();
            for (uint64_t k = 0; k <= (b & 1023); k++) acc160_mac(s, a, a);
            return acc160_reduce(s);
        }
        case 16: return gl_mul_pow2<1>(a);
        case 17: return gl_mul_pow2<33>(a);
        case 18: return gl_mul_pow2<63>(a);
        case 19: return gl_mul_pow2<64>(a);
        case 20: return gl_mul_pow2<95>(a);
        case 21: return gl_mul_pow2<96>(a);
        case 22: return gl_mul_pow2<120>(a);
        case 23: return gl_mul_pow2<156>(a);
        case 24: return gl_mul_pow2<191>(a);
        case 25: return gl_mul_pow2<39>(a);
        default: return 0;
    }
}

// Stage ops on 16-element states.
ZK_HD void state_op(int op, uint64_t s[16], const P2Const& c) {
    switch (op) {
        case 100: p2_mds_light(s); break;
        case 101:
            p2_external_round(s, c.ext[0]);
            break;
        case 102: p2_internal_linear(s, c.diag15); break;
        case 103:
            p2_internal_round(s, c.internal[0], c.diag15);
            break;
        case 104: p2_permute(s, c); break;
        case 105: {
            uint64_t a = s[0], b = s[1], x = s[2], d = s[3];
            p2_mat4(a, b, x, d);
            s[0] = a; s[1] = b; s[2] = x; s[3] = d;
            break;
        }
        // in-register DFTs of the NTT passes: plain and lazy forms, radix 16
        // (also with the upper half of the input zero), 8, 4 and 2 on
        // consecutive groups of the state
        case 110: dft_reg<4>(s); break;
        case 111: dft_reg_lazy<4>(s); break;
        case 112: dft_reg_half<4>(s); break;
        case 113: dft_reg_half_lazy<4>(s); break;
        case 114: dft_reg<3>(s); dft_reg<3>(s + 8); break;
        case 115: dft_reg_lazy<3>(s); dft_reg_lazy<3>(s + 8); break;
        case 116: for (int g = 0; g < 16; g += 4) dft_reg<2>(s + g); break;
        case 117: for (int g = 0; g < 16; g += 4) dft_reg_lazy<2>(s + g); break;
        case 118: for (int g = 0; g < 16; g += 2) dft_reg<1>(s + g); break;
        case 119: for (int g = 0; g < 16; g += 2) dft_reg_lazy<1>(s + g); break;
        // radix 16 with only the first 4, 2 or 1 inputs nonzero
        case 120: dft_reg_zero_lazy<4, 2>(s); break;
        case 121: dft_reg_zero_lazy<4, 3>(s); break;
        case 122: dft_reg_zero_lazy<4, 4>(s); break;
        default: break;
    }
}

__global__ void k_scalar(int op, const uint64_t* a, const uint64_t* b, uint64_t* out, uint64_t n) {
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = scalar_op(op, a[i], b[i]);
}

__global__ void k_state(int op, uint64_t* st, uint64_t n, P2Const c) {
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint64_t s[16];
    for (int q = 0; q < 16; q++) s[q] = st[i * 16 + q];
    state_op(op, s, c);
    for (int q = 0; q < 16; q++) st[i * 16 + q] = s[q];
}

// The four-threads-per-state permutation: group i of four lanes permutes
// state i (every lane of the grid runs it; groups past n use zeros).
__global__ void k_permute_x4(uint64_t* st, uint64_t n, P2Const c) {
    const uint64_t i = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 2;
    const uint32_t g = threadIdx.x & 3;
    uint64_t v[4] = {0, 0, 0, 0};
    if (i < n)
        for (int j = 0; j < 4; j++) v[j] = st[i * 16 + 4 * g + j];
    p2_permute_x4(v, g, c);
    if (i < n)
        for (int j = 0; j < 4; j++) st[i * 16 + 4 * g + j] = v[j];
}

P2Const consts_from151(const uint64_t* h) {
    P2Const c;
    for (int r = 0; r < 4; r++)
        for (int i = 0; i < 16; i++) {
            c.ext[r][i] = h[r * 16 + i];
            c.ext[4 + r][i] = h[64 + r * 16 + i];
        }
    for (int i = 0; i < 22; i++) c.internal[i] = h[128 + i];
    c.diag15 = h[150];
    return c;
}

}  // namespace

extern "C" {

int devcheck_permute_x4(uint64_t* d_states, uint64_t n, const uint64_t* h_consts151) {
    k_permute_x4<<<(unsigned)((4 * n + 127) / 128), 128>>>(d_states, n, consts_from151(h_consts151));
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    return (int)e;
}

// Device: out[i] = op(a[i], b[i]) for device arrays of n u64.
int devcheck_scalar(int op, const uint64_t* d_a, const uint64_t* d_b, uint64_t* d_out, uint64_t n) {
    k_scalar<<<(unsigned)((n + 127) / 128), 128>>>(op, d_a, d_b, d_out, n);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    return (int)e;
}

int devcheck_state(int op, uint64_t* d_states, uint64_t n, const uint64_t* h_consts151) {
    P2Const c;
    for (int r = 0; r < 4; r++)
        for (int i = 0; i < 16; i++) {
            c.ext[r][i] = h_consts151[r * 16 + i];
            c.ext[4 + r][i] = h_consts151[64 + r * 16 + i];
        }
    for (int i = 0; i < 22; i++) c.internal[i] = h_consts151[128 + i];
    c.diag15 = h_consts151[150];
    k_state<<<(unsigned)((n + 127) / 128), 128>>>(op, d_states, n, c);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    return (int)e;
}

// Host: the same functions compiled for the CPU.
void hostcheck_scalar(int op, const uint64_t* a, const uint64_t* b, uint64_t* out, uint64_t n) {
    for (uint64_t i = 0; i < n; i++) out[i] = scalar_op(op, a[i], b[i]);
}

void hostcheck_state(int op, uint64_t* states, uint64_t n, const uint64_t* h_consts151) {
    P2Const c;
    for (int r = 0; r < 4; r++)
        for (int i = 0; i < 16; i++) {
            c.ext[r][i] = h_consts151[r * 16 + i];
            c.ext[4 + r][i] = h_consts151[64 + r * 16 + i];
        }
    for (int i = 0; i < 22; i++) c.internal[i] = h_consts151[128 + i];
    c.diag15 = h_consts151[150];
    for (uint64_t i = 0; i < n; i++) state_op(op, states + 16 * i, c);
}

}  // extern "C"
