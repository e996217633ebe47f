// transcript.cpp -- host-side Fiat-Shamir challenge sources of the prover:
// the SHA-256 chained Transcript (crates/zkie-core/src/common/transcript.rs:
// 21-80) and the XorShift64 test source (common/field.rs:17-36), plus the
// shard-DAG child transcript (zkie-ops/src/compose.rs:2276-2311).
//
// Challenges never depend on device data in the matmul GKR (they are drawn
// before the proof is computed), so these run on the host while the device
// works.
#include <array>
#include <cstring>
#include <vector>

#include "../../include/zkie2.h"

namespace {

constexpr uint64_t kP = 0xFFFFFFFF00000001ull;

// SHA-256 (FIPS 180-4).  The round constants are computed from their
// definition: the first 32 fractional bits of the cube roots (K) and square
// roots (H0) of the first primes.
class Sha256 {
   public:
    Sha256() {
        static const Tables& t = tables();
        std::memcpy(h_, t.h0, sizeof h_);
    }
    void update(const uint8_t* p, size_t n) {
        total_ += n;
        while (n > 0) {
            size_t take = 64 - fill_;
            if (take > n) take = n;
            std::memcpy(buf_ + fill_, p, take);
            fill_ += take;
            p += take;
            n -= take;
            if (fill_ == 64) {
                block(buf_);
                fill_ = 0;
            }
        }
    }
    void finish(uint8_t out[32]) {
        const uint64_t bits = total_ * 8;
        const uint8_t one = 0x80, zero = 0;
        update(&one, 1);
        while (fill_ != 56) update(&zero, 1);
        uint8_t len[8];
        for (int i = 0; i < 8; i++) len[i] = (uint8_t)(bits >> (56 - 8 * i));
        update(len, 8);
        for (int i = 0; i < 8; i++)
            for (int b = 0; b < 4; b++) out[4 * i + b] = (uint8_t)(h_[i] >> (24 - 8 * b));
    }

   private:
    struct Tables {
        uint32_t k[64];
        uint32_t h0[8];
    };
    static unsigned __int128 root(unsigned __int128 n, int deg) {
        unsigned __int128 x = 0;
        for (int b = 42; b >= 0; b--) {
            unsigned __int128 y = x | ((unsigned __int128)1 << b);
            unsigned __int128 p = deg == 3 ? y * y * y : y * y;
            if (p <= n) x = y;
        }
        return x;
    }
    static const Tables& tables() {
        static Tables t = [] {
            Tables tt{};
            std::vector<int> primes;
            for (int c = 2; primes.size() < 64; c++) {
                bool ok = true;
                for (int d = 2; d * d <= c; d++)
                    if (c % d == 0) ok = false;
                if (ok) primes.push_back(c);
            }
            for (int i = 0; i < 64; i++) tt.k[i] = (uint32_t)root((unsigned __int128)primes[i] << 96, 3);
            for (int i = 0; i < 8; i++) tt.h0[i] = (uint32_t)root((unsigned __int128)primes[i] << 64, 2);
            return tt;
        }();
        return t;
    }
    static uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }
    void block(const uint8_t* p) {
        const Tables& t = tables();
        uint32_t w[64];
        for (int i = 0; i < 16; i++)
            w[i] = (uint32_t)p[4 * i] << 24 | (uint32_t)p[4 * i + 1] << 16 | (uint32_t)p[4 * i + 2] << 8 |
                   (uint32_t)p[4 * i + 3];
        for (int i = 16; i < 64; i++) {
            uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
            uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
            w[i] = w[i - 16] + s0 + w[i - 7] + s1;
        }
        uint32_t v[8];
        std::memcpy(v, h_, sizeof v);
        for (int i = 0; i < 64; i++) {
            uint32_t e = v[4], a = v[0];
            uint32_t t1 = v[7] + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & v[5]) ^ (~e & v[6])) + t.k[i] + w[i];
            uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & v[1]) ^ (a & v[2]) ^ (v[1] & v[2]));
            for (int j = 7; j > 0; j--) v[j] = v[j - 1];
            v[4] += t1;
            v[0] = t1 + t2;
        }
        for (int i = 0; i < 8; i++) h_[i] += v[i];
    }
    uint32_t h_[8];
    uint8_t buf_[64];
    size_t fill_ = 0;
    uint64_t total_ = 0;
};

uint64_t draw(zkie2_transcript* t) {
    Sha256 h;
    h.update(t->state, 32);
    uint8_t c[8];
    for (int i = 0; i < 8; i++) c[i] = (uint8_t)(t->counter >> (8 * i));
    h.update(c, 8);
    t->counter += 1;
    uint8_t d[32];
    h.finish(d);
    uint64_t v = 0;
    for (int i = 0; i < 8; i++) v |= (uint64_t)d[i] << (8 * i);
    return v;
}

}  // namespace

extern "C" {

void zkie2_sha256(const uint8_t* data, size_t len, uint8_t* out32) {
    Sha256 h;
    h.update(data, len);
    h.finish(out32);
}

void zkie2_transcript_new(zkie2_transcript* t, const uint8_t* domain, size_t len) {
    zkie2_sha256(domain, len, t->state);
    t->counter = 0;
}

void zkie2_transcript_absorb(zkie2_transcript* t, const uint8_t* data, size_t len) {
    Sha256 h;
    h.update(t->state, 32);
    h.update(data, len);
    h.finish(t->state);
}

void zkie2_transcript_absorb_u64(zkie2_transcript* t, uint64_t x) {
    uint8_t b[8];
    for (int i = 0; i < 8; i++) b[i] = (uint8_t)(x >> (8 * i));
    zkie2_transcript_absorb(t, b, 8);
}

uint64_t zkie2_transcript_field(zkie2_transcript* t) {
    for (;;) {
        uint64_t c = draw(t);
        if (c < kP) return c;
    }
}

uint64_t zkie2_transcript_next_u64(zkie2_transcript* t) { return draw(t); }

uint64_t zkie2_challenger_field(zkie2_challenger* c) {
    if (c->kind == ZKIE2_CHALLENGER_XORSHIFT) {
        uint64_t x = c->xorshift_state;
        x ^= x << 13;
        x ^= x >> 7;
        x ^= x << 17;
        c->xorshift_state = x;
        return x >= kP ? x - kP : x;  // Goldilocks::from_u64
    }
    return zkie2_transcript_field(&c->transcript);
}

void zkie2_challenger_xorshift(zkie2_challenger* c, uint64_t seed) {
    std::memset(c, 0, sizeof *c);
    c->kind = ZKIE2_CHALLENGER_XORSHIFT;
    c->xorshift_state = seed + 0x9e3779b97f4a7c15ull;
}

// Master transcript of prove_shard_dag + the child of shard `shard_index`
// (compose.rs:2276-2311) for a statement made of MatMul ops given as
// (a, b, c) tensor-id triples: absorb ops_per_shard, ops.len(), then each op's
// reads (a, b) and writes (c); the child absorbs the shard index.
void zkie2_shard_dag_child(const uint64_t* op_ids, uint32_t n_ops, uint64_t ops_per_shard,
                           uint64_t shard_index, zkie2_challenger* child) {
    static const char kDomain[] = "zkie-shard-dag-v1";
    std::memset(child, 0, sizeof *child);
    child->kind = ZKIE2_CHALLENGER_TRANSCRIPT;
    zkie2_transcript* t = &child->transcript;
    zkie2_transcript_new(t, (const uint8_t*)kDomain, sizeof(kDomain) - 1);
    zkie2_transcript_absorb_u64(t, ops_per_shard);
    zkie2_transcript_absorb_u64(t, n_ops);
    for (uint32_t i = 0; i < n_ops; i++)
        for (int j = 0; j < 3; j++) zkie2_transcript_absorb_u64(t, op_ids[3 * i + j]);
    zkie2_transcript_absorb_u64(t, shard_index);
}

// n draws of XorShift64::next_u64 (common/field.rs:17-36) from *state (advanced
// in place), each mapped to from_i64((draw % mod) + offset): the fixed-point
// weight draws of the reference's random model builders (e.g. compose.rs
// build_gpt2_layer, `from_i64((rng.next_u64() % 50) as i64)`).
void zkie2_xorshift_fill(uint64_t* state, uint64_t n, uint64_t mod, int64_t offset, uint64_t* out) {
    uint64_t x = *state;
    for (uint64_t i = 0; i < n; i++) {
        x ^= x << 13;
        x ^= x >> 7;
        x ^= x << 17;
        const int64_t v = (int64_t)(x % mod) + offset;
        out[i] = v >= 0 ? (uint64_t)v : kP - (0ull - (uint64_t)v);
    }
    *state = x;
}

// n successive field draws of a challenge source into out (the reference's
// `(0..n).map(|_| rng.field())`).
void zkie2_challenger_fields(zkie2_challenger* c, uint64_t n, uint64_t* out) {
    for (uint64_t i = 0; i < n; i++) out[i] = zkie2_challenger_field(c);
}

void zkie2_transcript_fields(zkie2_transcript* t, uint64_t n, uint64_t* out) {
    for (uint64_t i = 0; i < n; i++) out[i] = zkie2_transcript_field(t);
}

}  // extern "C"
