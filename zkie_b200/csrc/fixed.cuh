// fixed.cuh -- signed fixed-point values embedded in the Goldilocks field, on
// the device: fixed_point.rs to_i64 / from_i64 / to_i32 (:32-70) and the
// rounding division of the op layer (compose.rs round_div, :103-111).  The
// reference does this arithmetic in i64 in a release build, where overflow
// wraps; every product and sum here wraps the same way (through uint64_t).
#pragma once
#include <cstdint>

namespace zk {

constexpr uint64_t kFixP = 0xFFFFFFFF00000001ull;

// v if v <= i64::MAX, else -(p - v)  (v reduced first)
__device__ __forceinline__ int64_t fx_to_i64(uint64_t v) {
    v = v >= kFixP ? v - kFixP : v;
    return v <= 0x7FFFFFFFFFFFFFFFull ? (int64_t)v : -(int64_t)(kFixP - v);
}

// x if x >= 0, else p - |x|  (|x| = 2^63 included)
__device__ __forceinline__ uint64_t fx_from_i64(int64_t x) {
    return x >= 0 ? (uint64_t)x : kFixP - (0ull - (uint64_t)x);
}

// to_i32(v) as u32: v if v <= i32::MAX, else the negation of (p - v)
// truncated to 32 bits
__device__ __forceinline__ uint32_t fx_to_i32_index(uint64_t v) {
    v = v >= kFixP ? v - kFixP : v;
    if (v <= 0x7FFFFFFFull) return (uint32_t)v;
    return 0u - (uint32_t)(kFixP - v);
}

__device__ __forceinline__ int64_t fx_wadd(int64_t a, int64_t b) { return (int64_t)((uint64_t)a + (uint64_t)b); }
__device__ __forceinline__ int64_t fx_wsub(int64_t a, int64_t b) { return (int64_t)((uint64_t)a - (uint64_t)b); }
__device__ __forceinline__ int64_t fx_wmul(int64_t a, int64_t b) { return (int64_t)((uint64_t)a * (uint64_t)b); }

// round_div(a, 2^s): floor division, plus one when 2 * remainder >= 2^s
// (0 <= s <= 62)
__device__ __forceinline__ int64_t fx_round_div_pow2(int64_t a, uint32_t s) {
    const uint64_t r = (uint64_t)a & ((1ull << s) - 1);
    return fx_wadd(a >> s, (r << 1) >= (1ull << s) ? 1 : 0);
}

// round_div(a, b) for any b != 0: the Euclidean quotient q and remainder
// 0 <= r < |b|, plus one when 2 r >= b (always when b < 0).  Returns false
// where the reference panics: b == 0, or i64::MIN / -1.
__device__ __forceinline__ bool fx_round_div(int64_t a, int64_t b, int64_t* out) {
    if (b == 0 || (b == -1 && a == INT64_MIN)) return false;
    int64_t q = a / b, r = a % b;
    if (r < 0) {
        if (b > 0) {
            q -= 1;
            r += b;
        } else {
            q += 1;
            r -= b;
        }
    }
    *out = fx_wmul(r, 2) >= b ? fx_wadd(q, 1) : q;
    return true;
}

}  // namespace zk
