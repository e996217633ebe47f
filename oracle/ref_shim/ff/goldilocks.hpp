// Stand-in for the one sppark 0.1.15 name the reference's CUDA files use from
// <ff/goldilocks.hpp>: goldilocks::fr_t, a Goldilocks field element
// (p = 2^64 - 2^32 + 1) with the operators those files call (+, -, *, +=, *=,
// sqr(), zero(), [0], and an explicit conversion to a canonical uint64_t).
//
// TEST INFRASTRUCTURE: only the parity tests' build of the reference kernels
// (oracle/build_ref.py) includes it.  sppark itself is not in the reference
// tree.  Field arithmetic is exact modulo p, so any correct representation
// gives the same canonical results: this type keeps every value canonical
// (< p) at all times, which makes [0] (sppark's raw limb access) canonical
// too.  The reduction of a 128-bit product uses 2^64 = 2^32 - 1 (mod p) and
// 2^96 = -1 (mod p), written independently of the library under test.
#pragma once
#include <cstddef>
#include <cstdint>

namespace goldilocks {

class fr_t {
    uint64_t v;

    static constexpr uint64_t P = 0xFFFFFFFF00000001ull;
    static constexpr uint64_t EPS = 0xFFFFFFFFull;  // 2^64 mod p

    __host__ __device__ static inline uint64_t canon(uint64_t x) { return x >= P ? x - P : x; }

    __host__ __device__ static inline uint64_t add_c(uint64_t a, uint64_t b) {
        uint64_t s = a + b;
        if (s < a) s += EPS;  // wrapped past 2^64: subtract p = add 2^64 - p
        return canon(s);
    }
    __host__ __device__ static inline uint64_t sub_c(uint64_t a, uint64_t b) {
        uint64_t d = a - b;
        if (a < b) d -= EPS;  // borrowed 2^64: add p = subtract 2^64 - p
        return d;
    }
    __host__ __device__ static inline uint64_t mul_c(uint64_t a, uint64_t b) {
#ifdef __CUDA_ARCH__
        const uint64_t lo = a * b, hi = __umul64hi(a, b);
#else
        const unsigned __int128 t = (unsigned __int128)a * b;
        const uint64_t lo = (uint64_t)t, hi = (uint64_t)(t >> 64);
#endif
        // lo + 2^64 (hl + 2^32 hh) = lo + (2^32 - 1) hl - hh  (mod p)
        const uint64_t hh = hi >> 32, hl = hi & 0xFFFFFFFFull;
        uint64_t t0 = lo - hh;
        if (lo < hh) t0 -= EPS;
        const uint64_t t1 = hl * EPS;  // < 2^64
        uint64_t r = t0 + t1;
        if (r < t0) r += EPS;
        return canon(r);
    }

public:
    __host__ __device__ fr_t() : v(0) {}
    __host__ __device__ fr_t(uint64_t x) : v(canon(x)) {}

    __host__ __device__ inline void zero() { v = 0; }
    __host__ __device__ inline uint64_t operator[](size_t) const { return v; }
    __host__ __device__ explicit inline operator uint64_t() const { return v; }

    __host__ __device__ inline fr_t& operator+=(const fr_t& b) { v = add_c(v, b.v); return *this; }
    __host__ __device__ inline fr_t& operator-=(const fr_t& b) { v = sub_c(v, b.v); return *this; }
    __host__ __device__ inline fr_t& operator*=(const fr_t& b) { v = mul_c(v, b.v); return *this; }
    __host__ __device__ inline fr_t& sqr() { v = mul_c(v, v); return *this; }

    __host__ __device__ friend inline fr_t operator+(fr_t a, const fr_t& b) { return a += b; }
    __host__ __device__ friend inline fr_t operator-(fr_t a, const fr_t& b) { return a -= b; }
    __host__ __device__ friend inline fr_t operator*(fr_t a, const fr_t& b) { return a *= b; }
};

}  // namespace goldilocks
