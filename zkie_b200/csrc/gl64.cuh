// gl64.cuh -- Goldilocks (p = 2^64 - 2^32 + 1) arithmetic for sm_100a.
//
// Values are kept "partially reduced": any u64 in [0, 2^64) that is congruent
// to the field element.  Every operation accepts partially reduced inputs and
// returns a partially reduced output; gl_canon() maps to [0, p) and is applied
// once, where a value leaves the device as a result.  This is the same value
// contract as the reference's gl64_t (crates/zkie-core/cuda/goldilocks_ntt.cu:
// 13-15: "values stay partially reduced between stages; the final scatter
// canonicalizes").
//
// Carry handling is written with PTX add/sub-with-carry so the 64-bit
// operations map onto 32-bit carry chains without 128-bit emulation.
#pragma once
#include <cstdint>

namespace zk {

constexpr uint64_t GL_P = 0xFFFFFFFF00000001ull;
constexpr uint64_t GL_EPS = 0xFFFFFFFFull;  // 2^64 mod p

__device__ __forceinline__ uint64_t gl_canon(uint64_t x) { return x >= GL_P ? x - GL_P : x; }

// a + b mod p.  2^64 == EPS, so a carry out of bit 63 is folded back as +EPS;
// a second carry is only possible when both inputs are >= 2^64 - 2^32.
__device__ __forceinline__ uint64_t gl_add(uint64_t a, uint64_t b) {
    uint64_t s;
    uint32_t c;
    asm("add.cc.u64 %0, %2, %3;\n\t"
        "addc.u32 %1, 0, 0;"
        : "=l"(s), "=r"(c)
        : "l"(a), "l"(b));
    uint64_t fix = (uint64_t)(0u - c) & GL_EPS;  // EPS if carry
    uint64_t t;
    asm("add.cc.u64 %0, %2, %3;\n\t"
        "addc.u32 %1, 0, 0;"
        : "=l"(t), "=r"(c)
        : "l"(s), "l"(fix));
    return t + ((uint64_t)(0u - c) & GL_EPS);
}

// a + b where b < p (canonical): at most one fold is needed.
__device__ __forceinline__ uint64_t gl_add_c(uint64_t a, uint64_t b_canon) {
    uint64_t s;
    uint32_t c;
    asm("add.cc.u64 %0, %2, %3;\n\t"
        "addc.u32 %1, 0, 0;"
        : "=l"(s), "=r"(c)
        : "l"(a), "l"(b_canon));
    return s + ((uint64_t)(0u - c) & GL_EPS);
}

// a - b mod p.  A borrow means the wrapped result is 2^64 too large, i.e.
// EPS too large modulo p; a second borrow can only occur for b >= 2^64 - 2^32.
__device__ __forceinline__ uint64_t gl_sub(uint64_t a, uint64_t b) {
    uint64_t d;
    uint32_t br;
    asm("sub.cc.u64 %0, %2, %3;\n\t"
        "subc.u32 %1, 0, 0;"
        : "=l"(d), "=r"(br)
        : "l"(a), "l"(b));
    uint64_t fix = (uint64_t)br & GL_EPS;  // br is 0 or 0xFFFFFFFF
    uint64_t t;
    asm("sub.cc.u64 %0, %2, %3;\n\t"
        "subc.u32 %1, 0, 0;"
        : "=l"(t), "=r"(br)
        : "l"(d), "l"(fix));
    return t - ((uint64_t)br & GL_EPS);
}

// Reduce hi*2^64 + lo.  With hi = hh*2^32 + hl: 2^64 == 2^32 - 1 and
// 2^96 == -1, so the value is lo - hh + hl*(2^32 - 1).
__device__ __forceinline__ uint64_t gl_reduce128(uint64_t lo, uint64_t hi) {
    uint32_t hh = (uint32_t)(hi >> 32);
    uint32_t hl = (uint32_t)hi;
    uint64_t t0;
    uint32_t br;
    asm("sub.cc.u64 %0, %2, %3;\n\t"
        "subc.u32 %1, 0, 0;"
        : "=l"(t0), "=r"(br)
        : "l"(lo), "l"((uint64_t)hh));
    t0 -= (uint64_t)br & GL_EPS;             // borrow: +p == -EPS (mod 2^64), no underflow
    uint64_t t1 = ((uint64_t)hl << 32) - hl;  // hl * (2^32 - 1) < 2^64
    uint64_t t2;
    uint32_t c;
    asm("add.cc.u64 %0, %2, %3;\n\t"
        "addc.u32 %1, 0, 0;"
        : "=l"(t2), "=r"(c)
        : "l"(t0), "l"(t1));
    return t2 + ((uint64_t)(0u - c) & GL_EPS);  // cannot carry again
}

__device__ __forceinline__ uint64_t gl_mul(uint64_t a, uint64_t b) {
    return gl_reduce128(a * b, __umul64hi(a, b));
}

__device__ __forceinline__ uint64_t gl_sqr(uint64_t a) { return gl_mul(a, a); }

// x / 2^k mod p for 1 <= k <= 32.  p == 1 (mod 2^k), so with
// m = (-x) mod 2^k the sum x + m*p is divisible by 2^k and
// (x + m*p) / 2^k = (x >> k) + [x mod 2^k != 0] + m*2^(64-k) - m*2^(32-k),
// which is below 2^64 for every x < 2^64.
template <int K>
__device__ __forceinline__ uint64_t gl_div_pow2(uint64_t x) {
    static_assert(K >= 1 && K <= 32, "k in [1, 32]");
    const uint64_t mask = (K == 32) ? 0xFFFFFFFFull : ((1ull << K) - 1);
    uint64_t m = (0ull - x) & mask;
    uint64_t r = (x >> K) + (m != 0 ? 1ull : 0ull);
    r += (m << (64 - K)) - (m << (32 - K));
    return r;
}

__device__ __forceinline__ uint64_t gl_neg(uint64_t a) { return gl_sub(0, a); }

__device__ __forceinline__ uint64_t gl_pow(uint64_t a, uint64_t e) {
    uint64_t r = 1;
    while (e) {
        if (e & 1) r = gl_mul(r, a);
        a = gl_mul(a, a);
        e >>= 1;
    }
    return r;
}

}  // namespace zk
