// host.cpp -- host-side field helpers and Poseidon2 constant derivation.
#include <cstdint>

#include "internal.h"

namespace zk {

namespace {
constexpr uint64_t P = 0xFFFFFFFF00000001ull;
}

uint64_t gl_add_host(uint64_t a, uint64_t b) {
    a = a >= P ? a - P : a;
    b = b >= P ? b - P : b;
    uint64_t s = a + b;
    if (s < a) return s + 0xFFFFFFFFull;
    return s >= P ? s - P : s;
}

uint64_t gl_sub_host(uint64_t a, uint64_t b) {
    a = a >= P ? a - P : a;
    b = b >= P ? b - P : b;
    return a >= b ? a - b : a - b + P;
}

uint64_t gl_mul_host(uint64_t a, uint64_t b) {
    unsigned __int128 x = (unsigned __int128)a * b;
    return (uint64_t)(x % P);
}

uint64_t gl_pow_host(uint64_t a, uint64_t e) {
    uint64_t r = 1;
    while (e) {
        if (e & 1) r = gl_mul_host(r, a);
        a = gl_mul_host(a, a);
        e >>= 1;
    }
    return r;
}

// TWO_ADIC_GENERATORS[bits] of p3-goldilocks, consumed by the reference's
// twiddle builder (crates/zkie-core/src/pcs/dft_cuda.rs:44-59): the element of
// order 2^bits given by g^(2^(32-bits)) with g = 7^((p-1)/2^32).
uint64_t two_adic_generator_host(uint32_t bits) {
    uint64_t g = gl_pow_host(7, (P - 1) >> 32);
    for (uint32_t i = bits; i < 32; i++) g = gl_mul_host(g, g);
    return g;
}

namespace {
uint64_t splitmix64(uint64_t* s) {
    *s += 0x9e3779b97f4a7c15ull;
    uint64_t z = *s;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

inline uint64_t rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

struct Xoshiro256pp {
    uint64_t s[4];
    explicit Xoshiro256pp(uint64_t seed) {
        uint64_t sm = seed;
        for (int i = 0; i < 4; i++) s[i] = splitmix64(&sm);
    }
    uint64_t next() {
        uint64_t result = rotl(s[0] + s[3], 23) + s[0];
        uint64_t t = s[1] << 17;
        s[2] ^= s[0];
        s[3] ^= s[1];
        s[1] ^= s[2];
        s[0] ^= s[3];
        s[2] ^= t;
        s[3] = rotl(s[3], 45);
        return result;
    }
    // p3-goldilocks StandardUniform sampling: reject draws >= p.
    uint64_t field() {
        for (;;) {
            uint64_t v = next();
            if (v < P) return v;
        }
    }
};
}  // namespace

// Poseidon2 round constants as derived by
// crates/zkie-core/src/pcs/merkle_cuda.rs:54-85 (Perm::new_from_rng_128 on
// SmallRng::seed_from_u64(seed)): 4 initial external rounds of 16, 4 terminal
// external rounds of 16, then 22 internal constants, drawn in that order.
// SmallRng is taken as xoshiro256++ seeded by SplitMix64.  diag15 is entry 15
// of the width-16 internal diagonal, 2^-32 mod p.
void p2_derive_constants_host(uint64_t seed, uint64_t rc_init[64], uint64_t rc_final[64],
                              uint64_t rc_internal[22], uint64_t* diag15) {
    Xoshiro256pp rng(seed);
    for (int i = 0; i < 64; i++) rc_init[i] = rng.field();
    for (int i = 0; i < 64; i++) rc_final[i] = rng.field();
    for (int i = 0; i < 22; i++) rc_internal[i] = rng.field();
    *diag15 = gl_pow_host(gl_pow_host(2, 32), P - 2);
}

}  // namespace zk
