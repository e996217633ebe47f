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
// On the device the carry handling is PTX add/sub-with-carry, so the 64-bit
// operations map onto 32-bit carry chains without 128-bit emulation.  The
// same functions compile for the host (portable C), which lets the kernel-side
// permutation and NTT logic be unit-tested on a CPU.
#pragma once
#include <cstdint>

#if defined(__CUDACC__)
#define ZK_HD __host__ __device__ __forceinline__
#else
#define ZK_HD inline
#endif

namespace zk {

constexpr uint64_t GL_P = 0xFFFFFFFF00000001ull;
constexpr uint64_t GL_EPS = 0xFFFFFFFFull;  // 2^64 mod p

ZK_HD uint64_t gl_canon(uint64_t x) { return x >= GL_P ? x - GL_P : x; }

// s = a + b (mod 2^64) and the carry out of bit 63.
ZK_HD uint64_t add_carry(uint64_t a, uint64_t b, uint32_t& c) {
#if defined(__CUDA_ARCH__)
    uint64_t s;
    asm("add.cc.u64 %0, %2, %3;\n\t"
        "addc.u32 %1, 0, 0;"
        : "=l"(s), "=r"(c)
        : "l"(a), "l"(b));
    return s;
#else
    uint64_t s = a + b;
    c = s < a ? 1u : 0u;
    return s;
#endif
}

// d = a - b (mod 2^64) and the borrow as a mask (0 or 0xFFFFFFFF).
ZK_HD uint64_t sub_borrow(uint64_t a, uint64_t b, uint32_t& mask) {
#if defined(__CUDA_ARCH__)
    uint64_t d;
    asm("sub.cc.u64 %0, %2, %3;\n\t"
        "subc.u32 %1, 0, 0;"
        : "=l"(d), "=r"(mask)
        : "l"(a), "l"(b));
    return d;
#else
    mask = a < b ? 0xFFFFFFFFu : 0u;
    return a - b;
#endif
}

ZK_HD uint64_t pack64(uint32_t lo, uint32_t hi) { return ((uint64_t)hi << 32) | lo; }

// a + b mod p.  2^64 == EPS, so a carry out of bit 63 is folded back as +EPS;
// a second carry is only possible when both inputs are >= 2^64 - 2^32.
// (Measured on sm_100a: this carry-mask form issues fewer instructions than
// folding the carry with multiply-adds or leaving the carries to the
// compiler.)
ZK_HD uint64_t gl_add(uint64_t a, uint64_t b) {
    uint32_t c;
    uint64_t s = add_carry(a, b, c);
    s = add_carry(s, (uint64_t)(0u - c) & GL_EPS, c);
    return s + ((uint64_t)(0u - c) & GL_EPS);
}

// a + b where b < p (canonical): at most one fold is needed.
ZK_HD uint64_t gl_add_c(uint64_t a, uint64_t b_canon) {
    uint32_t c;
    const uint64_t s = add_carry(a, b_canon, c);
    return s + ((uint64_t)(0u - c) & GL_EPS);
}

// a - b mod p.  A borrow means the wrapped result is 2^64 too large, i.e.
// EPS too large modulo p; a second borrow can only occur for b >= 2^64 - 2^32.
ZK_HD uint64_t gl_sub(uint64_t a, uint64_t b) {
    uint32_t br;
    uint64_t d = sub_borrow(a, b, br);
    d = sub_borrow(d, (uint64_t)br & GL_EPS, br);
    return d - ((uint64_t)br & GL_EPS);
}

// 32 x 32 -> 64 product (one wide IMAD on the device).
ZK_HD uint64_t mul_wide32(uint32_t a, uint32_t b) {
#if defined(__CUDA_ARCH__)
    uint64_t r;
    asm("mul.wide.u32 %0, %1, %2;" : "=l"(r) : "r"(a), "r"(b));
    return r;
#else
    return (uint64_t)a * b;
#endif
}

// Reduce hi*2^64 + lo.  With hi = hh*2^32 + hl: 2^64 == 2^32 - 1 and
// 2^96 == -1, so the value is lo - hh + hl*(2^32 - 1).
ZK_HD uint64_t gl_reduce128(uint64_t lo, uint64_t hi) {
    const uint32_t hh = (uint32_t)(hi >> 32);
    const uint32_t hl = (uint32_t)hi;
    uint32_t br;
    uint64_t t0 = sub_borrow(lo, (uint64_t)hh, br);
    t0 -= (uint64_t)br & GL_EPS;                      // borrow: +p == -EPS (mod 2^64), no underflow
    const uint64_t t1 = mul_wide32(hl, 0xFFFFFFFFu);  // hl * (2^32 - 1) < 2^64
    uint32_t c;
    const uint64_t t2 = add_carry(t0, t1, c);
    return t2 + ((uint64_t)(0u - c) & GL_EPS);  // cannot carry again
}

// Full 64 x 64 -> 128 product.  On the device: schoolbook over 32-bit limbs
// as one multiply-add carry chain (the integer-multiply pipe does nearly all
// of it, leaving the ALU pipe to the additions).
ZK_HD void mul_wide64(uint64_t a, uint64_t b, uint64_t& lo, uint64_t& hi) {
#if defined(__CUDA_ARCH__)
    const uint32_t a0 = (uint32_t)a, a1 = (uint32_t)(a >> 32);
    const uint32_t b0 = (uint32_t)b, b1 = (uint32_t)(b >> 32);
    uint32_t r0, r1, r2, r3;
    asm("mul.lo.u32     %0, %4, %6;\n\t"
        "mul.hi.u32     %1, %4, %6;\n\t"
        "mad.lo.cc.u32  %1, %4, %7, %1;\n\t"
        "madc.hi.u32    %2, %4, %7, 0;\n\t"
        "mad.lo.cc.u32  %1, %5, %6, %1;\n\t"
        "madc.hi.cc.u32 %2, %5, %6, %2;\n\t"
        "madc.hi.u32    %3, %5, %7, 0;\n\t"
        "mad.lo.cc.u32  %2, %5, %7, %2;\n\t"
        "addc.u32       %3, %3, 0;"
        : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
        : "r"(a0), "r"(a1), "r"(b0), "r"(b1));
    lo = ((uint64_t)r1 << 32) | r0;
    hi = ((uint64_t)r3 << 32) | r2;
#else
    const unsigned __int128 p = (unsigned __int128)a * b;
    lo = (uint64_t)p;
    hi = (uint64_t)(p >> 64);
#endif
}

ZK_HD uint64_t mul_hi(uint64_t a, uint64_t b) {
    uint64_t lo, hi;
    mul_wide64(a, b, lo, hi);
    return hi;
}

ZK_HD uint64_t gl_mul(uint64_t a, uint64_t b) {
    uint64_t lo, hi;
    mul_wide64(a, b, lo, hi);
    return gl_reduce128(lo, hi);
}

// ---- lazy accumulation ---------------------------------------------------------------
// A non-negative integer below 2^96 held as lo + hi * 2^64.  Sums of a few
// dozen partially reduced elements fit; each addition is a 3-instruction
// carry chain instead of a modular add, and the sum is reduced once.
struct Acc {
    uint64_t lo;
    uint32_t hi;
};

ZK_HD Acc acc_of(uint64_t x) { return Acc{x, 0u}; }

// a + x
ZK_HD Acc acc_add(Acc a, uint64_t x) {
#if defined(__CUDA_ARCH__)
    asm("add.cc.u64 %0, %0, %2;\n\t"
        "addc.u32 %1, %1, 0;"
        : "+l"(a.lo), "+r"(a.hi)
        : "l"(x));
    return a;
#else
    const uint64_t s = a.lo + x;
    return Acc{s, a.hi + (s < x ? 1u : 0u)};
#endif
}

// a + b
ZK_HD Acc acc_add(Acc a, Acc b) {
#if defined(__CUDA_ARCH__)
    asm("add.cc.u64 %0, %0, %2;\n\t"
        "addc.u32 %1, %1, %3;"
        : "+l"(a.lo), "+r"(a.hi)
        : "l"(b.lo), "r"(b.hi));
    return a;
#else
    const uint64_t s = a.lo + b.lo;
    return Acc{s, a.hi + b.hi + (s < b.lo ? 1u : 0u)};
#endif
}

// a - b, for a >= b
ZK_HD Acc acc_sub(Acc a, Acc b) {
#if defined(__CUDA_ARCH__)
    asm("sub.cc.u64 %0, %0, %2;\n\t"
        "subc.u32 %1, %1, %3;"
        : "+l"(a.lo), "+r"(a.hi)
        : "l"(b.lo), "r"(b.hi));
    return a;
#else
    return Acc{a.lo - b.lo, a.hi - b.hi - (a.lo < b.lo ? 1u : 0u)};
#endif
}

// x * 2^K as an accumulator, 1 <= K <= 31
template <int K>
ZK_HD Acc acc_shl(uint64_t x) {
    return Acc{x << K, (uint32_t)(x >> (64 - K))};
}

// x + y of two partially reduced elements, as an accumulator
ZK_HD Acc acc_sum(uint64_t x, uint64_t y) { return acc_add(acc_of(x), y); }

// lo + hi * 2^64 == lo + hi * (2^32 - 1) (mod p); hi * (2^32 - 1) < 2^64 and
// after a carry the sum is below hi * (2^32 - 1), so one fold suffices.
ZK_HD uint64_t acc_reduce(Acc a) {
    uint32_t c;
    const uint64_t s = add_carry(a.lo, mul_wide32(a.hi, 0xFFFFFFFFu), c);
    return s + ((uint64_t)(0u - c) & GL_EPS);
}

// ---- lazy sums of products -------------------------------------------------------------
// A non-negative integer below 2^160 in five 32-bit limbs (little-endian).
// Sums of up to 2^32 full 64 x 64 -> 128 products fit, so a dot product
// accumulates every product exactly and reduces once at the end instead of
// reducing each product and adding modulo p.
struct Acc160 {
    uint32_t w[5];
};

ZK_HD Acc160 acc160_zero() { return Acc160{{0u, 0u, 0u, 0u, 0u}}; }

// a += x * y: the four 32 x 32 partial products as three multiply-add carry
// chains (x0*y0 and x1*y1 on the even diagonals, then x0*y1 and x1*y0).
ZK_HD void acc160_mac(Acc160& a, uint64_t x, uint64_t y) {
#if defined(__CUDA_ARCH__)
    const uint32_t x0 = (uint32_t)x, x1 = (uint32_t)(x >> 32);
    const uint32_t y0 = (uint32_t)y, y1 = (uint32_t)(y >> 32);
    asm("mad.lo.cc.u32  %0, %5, %7, %0;\n\t"
        "madc.hi.cc.u32 %1, %5, %7, %1;\n\t"
        "madc.lo.cc.u32 %2, %6, %8, %2;\n\t"
        "madc.hi.cc.u32 %3, %6, %8, %3;\n\t"
        "addc.u32       %4, %4, 0;\n\t"
        "mad.lo.cc.u32  %1, %5, %8, %1;\n\t"
        "madc.hi.cc.u32 %2, %5, %8, %2;\n\t"
        "addc.cc.u32    %3, %3, 0;\n\t"
        "addc.u32       %4, %4, 0;\n\t"
        "mad.lo.cc.u32  %1, %6, %7, %1;\n\t"
        "madc.hi.cc.u32 %2, %6, %7, %2;\n\t"
        "addc.cc.u32    %3, %3, 0;\n\t"
        "addc.u32       %4, %4, 0;"
        : "+r"(a.w[0]), "+r"(a.w[1]), "+r"(a.w[2]), "+r"(a.w[3]), "+r"(a.w[4])
        : "r"(x0), "r"(x1), "r"(y0), "r"(y1));
#else
    const unsigned __int128 p = (unsigned __int128)x * y;
    const unsigned __int128 lo = ((unsigned __int128)a.w[1] << 32 | a.w[0]) |
                                 ((unsigned __int128)((uint64_t)a.w[3] << 32 | a.w[2]) << 64);
    const unsigned __int128 s = lo + p;
    a.w[4] += s < p ? 1u : 0u;
    a.w[0] = (uint32_t)s;
    a.w[1] = (uint32_t)(s >> 32);
    a.w[2] = (uint32_t)(s >> 64);
    a.w[3] = (uint32_t)(s >> 96);
#endif
}

// a += x
ZK_HD void acc160_add(Acc160& a, uint64_t x) {
#if defined(__CUDA_ARCH__)
    asm("add.cc.u32  %0, %0, %5;\n\t"
        "addc.cc.u32 %1, %1, %6;\n\t"
        "addc.cc.u32 %2, %2, 0;\n\t"
        "addc.cc.u32 %3, %3, 0;\n\t"
        "addc.u32    %4, %4, 0;"
        : "+r"(a.w[0]), "+r"(a.w[1]), "+r"(a.w[2]), "+r"(a.w[3]), "+r"(a.w[4])
        : "r"((uint32_t)x), "r"((uint32_t)(x >> 32)));
#else
    uint64_t carry = x;
    for (int i = 0; i < 5 && carry; i++) {
        const uint64_t s = (uint64_t)a.w[i] + (uint32_t)carry;
        a.w[i] = (uint32_t)s;
        carry = (carry >> 32) + (s >> 32);
    }
#endif
}

// lo + mid * 2^64 + hi * 2^128 with 2^128 == -2^32 (mod p); hi * 2^32 < p.
ZK_HD uint64_t acc160_reduce(const Acc160& a) {
    const uint64_t r = gl_reduce128(pack64(a.w[0], a.w[1]), pack64(a.w[2], a.w[3]));
    return gl_sub(r, (uint64_t)a.w[4] << 32);
}

// a^2 = a0^2 + 2 a0 a1 2^32 + a1^2 2^64: the two squares as wide products and
// the doubled cross term as two multiply-add carry chains.  Three fewer
// multiplies than gl_mul and most of the additions on the multiply pipe
// (the ALU pipe is the one that binds the Poseidon2 S-box).
ZK_HD uint64_t gl_sqr(uint64_t a) {
#if defined(__CUDA_ARCH__)
    const uint32_t a0 = (uint32_t)a, a1 = (uint32_t)(a >> 32);
    const uint64_t ll = mul_wide32(a0, a0), hh = mul_wide32(a1, a1);
    uint32_t r0 = (uint32_t)ll, r1 = (uint32_t)(ll >> 32), r2 = (uint32_t)hh, r3 = (uint32_t)(hh >> 32);
    asm("mad.lo.cc.u32  %0, %3, %4, %0;\n\t"
        "madc.hi.cc.u32 %1, %3, %4, %1;\n\t"
        "addc.u32       %2, %2, 0;\n\t"
        "mad.lo.cc.u32  %0, %3, %4, %0;\n\t"
        "madc.hi.cc.u32 %1, %3, %4, %1;\n\t"
        "addc.u32       %2, %2, 0;"
        : "+r"(r1), "+r"(r2), "+r"(r3)
        : "r"(a0), "r"(a1));
    return gl_reduce128(pack64(r0, r1), pack64(r2, r3));
#else
    return gl_mul(a, a);
#endif
}

// a * b with the diagonal products as wide multiplies and the two cross
// products as multiply-add carry chains: fewer ALU instructions than gl_mul
// (whose single carry chain suits the NTT better), for the S-box.
ZK_HD uint64_t gl_mul_madc(uint64_t a, uint64_t b) {
#if defined(__CUDA_ARCH__)
    const uint32_t a0 = (uint32_t)a, a1 = (uint32_t)(a >> 32);
    const uint32_t b0 = (uint32_t)b, b1 = (uint32_t)(b >> 32);
    const uint64_t ll = mul_wide32(a0, b0), hh = mul_wide32(a1, b1);
    uint32_t r0 = (uint32_t)ll, r1 = (uint32_t)(ll >> 32), r2 = (uint32_t)hh, r3 = (uint32_t)(hh >> 32);
    asm("mad.lo.cc.u32  %0, %3, %6, %0;\n\t"
        "madc.hi.cc.u32 %1, %3, %6, %1;\n\t"
        "addc.u32       %2, %2, 0;\n\t"
        "mad.lo.cc.u32  %0, %4, %5, %0;\n\t"
        "madc.hi.cc.u32 %1, %4, %5, %1;\n\t"
        "addc.u32       %2, %2, 0;"
        : "+r"(r1), "+r"(r2), "+r"(r3)
        : "r"(a0), "r"(a1), "r"(b0), "r"(b1));
    return gl_reduce128(pack64(r0, r1), pack64(r2, r3));
#else
    return gl_mul(a, b);
#endif
}

// x / 2^k mod p for 1 <= k <= 32.  p == 1 (mod 2^k), so with
// m = (-x) mod 2^k the sum x + m*p is divisible by 2^k and
// (x + m*p) / 2^k = (x >> k) + [x mod 2^k != 0] + t*(2^32 - 1), t = m*2^(32-k),
// which is below 2^64 for every x < 2^64.  t < 2^32 is formed as a 32-bit
// value and widened with one 32x32->64 multiply: the equivalent 64-bit shift
// form (m << (64-k)) - (m << (32-k)) produced wrong high bits on sm_100a
// with nvcc 12.9 (caught by tests/test_devcheck.py).
template <int K>
ZK_HD uint64_t gl_div_pow2(uint64_t x) {
    static_assert(K >= 1 && K <= 32, "k in [1, 32]");
    const uint32_t mask = (K == 32) ? 0xFFFFFFFFu : ((1u << (K & 31)) - 1u);
    const uint32_t m = (0u - (uint32_t)x) & mask;
    const uint32_t t = m << (32 - K);  // K == 32: t = m
    return (x >> K) + (m != 0u ? 1ull : 0ull) + (uint64_t)t * GL_EPS;
}

ZK_HD uint64_t gl_neg(uint64_t a) { return gl_sub(0, a); }

// x * 2^K for 0 <= K < 192 without a multiplication, as t with the sign
// separate (x * 2^K = neg ? -t : t): 2^96 = -1, so K = 96 + K' flips the
// sign; for 0 < K' < 64 the 128-bit shift x * 2^K' is reduced once; for
// 64 <= K' < 96, 2^K' = -2^-(96-K') is a division by a power of two.
template <int K>
struct GlPow2 {
    static_assert(K >= 0 && K < 192, "exponent in [0, 192)");
    static constexpr int Kp = K % 96;
    static constexpr bool neg = (K >= 96) != (Kp >= 64);
    ZK_HD static uint64_t mag(uint64_t x) {
        if constexpr (Kp == 0) return x;
        else if constexpr (Kp < 64) return gl_reduce128(x << Kp, x >> (64 - Kp));
        else return gl_div_pow2<96 - Kp>(x);
    }
};

template <int K>
ZK_HD uint64_t gl_mul_pow2(uint64_t x) {
    const uint64_t t = GlPow2<K>::mag(x);
    return GlPow2<K>::neg ? gl_neg(t) : t;
}

ZK_HD uint64_t gl_pow(uint64_t a, uint64_t e) {
    uint64_t r = 1;
    while (e) {
        if (e & 1) r = gl_mul(r, a);
        a = gl_mul(a, a);
        e >>= 1;
    }
    return r;
}

}  // namespace zk
