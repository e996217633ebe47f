/*
 * zkie_oracle.c -- CPU restatement of the zkIE prover hot path (TEST INFRASTRUCTURE).
 *
 * Parity checker only: loaded by tests/, __graft_entry__.smoke() and bench.py's
 * CPU baseline.  The product (zkie_b200/) never links or calls this file.
 * See zkie_oracle.h for the parity status of each part.
 *
 * Reference paths below are relative to the trustless-ai/zkIE project root.
 */
#include "zkie_oracle.h"

#include <stdlib.h>
#include <string.h>
#if defined(__x86_64__)
#include <immintrin.h>
#endif
#ifdef _OPENMP
#include <omp.h>
#endif

typedef unsigned __int128 u128;
#define EPS 0xFFFFFFFFULL /* 2^64 mod p */

/* ============================================================================
 * Goldilocks field, canonical representation.
 * Semantics of p3-goldilocks `Goldilocks` (re-exported at
 * crates/zkie-core/src/common/field.rs:10-14).
 * ========================================================================== */
/* a + b and a - b of canonical inputs, canonical; the conditions are masks,
 * not branches (they are coin flips on random data). */
uint64_t orc_add(uint64_t a, uint64_t b)
{
    uint64_t s = a + b;
    const uint64_t wrapped = 0 - (uint64_t)(s < a); /* +2^64 == +EPS, result < p */
    s += EPS & wrapped;
    return s - (ORC_P & ~wrapped & (0 - (uint64_t)(s >= ORC_P)));
}

uint64_t orc_sub(uint64_t a, uint64_t b)
{
    return a - b + (ORC_P & (0 - (uint64_t)(a < b)));
}

/* x mod p for any 128-bit x: 2^64 = EPS and 2^96 = -1 (mod p).  Written
 * without data-dependent branches (the conditions become masks). */
static inline uint64_t reduce128(u128 x)
{
    uint64_t lo = (uint64_t)x, hi = (uint64_t)(x >> 64);
    uint64_t hh = hi >> 32, hl = hi & 0xFFFFFFFFULL;
    uint64_t t0 = lo - hh;
    t0 -= EPS & (0 - (uint64_t)(lo < hh));
    uint64_t t1 = hl * EPS;
    uint64_t t2 = t0 + t1;
    t2 += EPS & (0 - (uint64_t)(t2 < t1));
    return t2 - (ORC_P & (0 - (uint64_t)(t2 >= ORC_P)));
}

uint64_t orc_mul(uint64_t a, uint64_t b) { return reduce128((u128)a * b); }

uint64_t orc_pow(uint64_t a, uint64_t e)
{
    uint64_t r = 1;
    while (e) {
        if (e & 1) r = orc_mul(r, a);
        a = orc_mul(a, a);
        e >>= 1;
    }
    return r;
}

uint64_t orc_inv(uint64_t a) { return orc_pow(a, ORC_P - 2); }

/* fixed_point::from_i64 (crates/zkie-core/src/common/fixed_point.rs:53-59). */
uint64_t orc_from_i64(int64_t x)
{
    if (x >= 0) return ((uint64_t)x) % ORC_P;
    uint64_t mag = (uint64_t)(-(x + 1)) + 1; /* |x| without overflow */
    return ORC_P - mag;
}

static uint64_t canon(uint64_t x) { return x >= ORC_P ? x - ORC_P : x; }

/* TWO_ADIC_GENERATORS[bits]: the order-2^bits element g^(2^(32-bits)) with
 * g = 7^((p-1)/2^32), 7 generating the multiplicative group.  The reference
 * twiddle builder consumes this table (crates/zkie-core/src/pcs/dft_cuda.rs:44-59). */
uint64_t orc_two_adic_generator(uint32_t bits)
{
    uint64_t g = orc_pow(7, (ORC_P - 1) >> 32);
    for (uint32_t i = bits; i < 32; i++) g = orc_mul(g, g);
    return g;
}

/* ============================================================================
 * XorShift64 (crates/zkie-core/src/common/field.rs:17-36).
 * ========================================================================== */
uint64_t orc_xorshift_init(uint64_t seed) { return seed + 0x9e3779b97f4a7c15ULL; }

uint64_t orc_xorshift_next(uint64_t *state)
{
    uint64_t x = *state;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    *state = x;
    return x;
}

/* `Goldilocks::from_u64(next_u64())`: the value mod p. */
uint64_t orc_xorshift_field(uint64_t *state) { return canon(orc_xorshift_next(state)); }

/* ============================================================================
 * SHA-256 (FIPS 180-4).  Round constants are derived from their definition
 * (fractional bits of square / cube roots of the first primes).
 * ========================================================================== */
static uint32_t K256[64], H256[8];
static int sha_ready = 0;

static u128 iroot(u128 n, int k)
{
    u128 x = 0;
    for (int b = 42; b >= 0; b--) {
        u128 y = x | ((u128)1 << b);
        u128 p = y * y;
        if (k == 3) p *= y;
        if (p <= n) x = y;
    }
    return x;
}

static void sha_init_consts(void)
{
    if (sha_ready) return;
    int primes[64], np = 0;
    for (int c = 2; np < 64; c++) {
        int ok = 1;
        for (int d = 2; d * d <= c; d++)
            if (c % d == 0) { ok = 0; break; }
        if (ok) primes[np++] = c;
    }
    for (int i = 0; i < 64; i++) K256[i] = (uint32_t)iroot((u128)primes[i] << 96, 3);
    for (int i = 0; i < 8; i++) H256[i] = (uint32_t)iroot((u128)primes[i] << 64, 2);
    sha_ready = 1;
}

#define ROR(x, n) (((x) >> (n)) | ((x) << (32 - (n))))

static void sha_block(uint32_t h[8], const uint8_t *p)
{
    uint32_t w[64];
    for (int i = 0; i < 16; i++)
        w[i] = ((uint32_t)p[4 * i] << 24) | ((uint32_t)p[4 * i + 1] << 16) |
               ((uint32_t)p[4 * i + 2] << 8) | p[4 * i + 3];
    for (int i = 16; i < 64; i++) {
        uint32_t s0 = ROR(w[i - 15], 7) ^ ROR(w[i - 15], 18) ^ (w[i - 15] >> 3);
        uint32_t s1 = ROR(w[i - 2], 17) ^ ROR(w[i - 2], 19) ^ (w[i - 2] >> 10);
        w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], hh = h[7];
    for (int i = 0; i < 64; i++) {
        uint32_t S1 = ROR(e, 6) ^ ROR(e, 11) ^ ROR(e, 25);
        uint32_t ch = (e & f) ^ (~e & g);
        uint32_t t1 = hh + S1 + ch + K256[i] + w[i];
        uint32_t S0 = ROR(a, 2) ^ ROR(a, 13) ^ ROR(a, 22);
        uint32_t mj = (a & b) ^ (a & c) ^ (b & c);
        uint32_t t2 = S0 + mj;
        hh = g; g = f; f = e; e = d + t1; d = c; c = b; b = a; a = t1 + t2;
    }
    h[0] += a; h[1] += b; h[2] += c; h[3] += d;
    h[4] += e; h[5] += f; h[6] += g; h[7] += hh;
}

void orc_sha256(const uint8_t *data, size_t len, uint8_t out[32])
{
    sha_init_consts();
    uint32_t h[8];
    memcpy(h, H256, sizeof h);
    size_t full = len / 64;
    for (size_t i = 0; i < full; i++) sha_block(h, data + 64 * i);
    uint8_t tail[128];
    size_t rem = len - 64 * full;
    memset(tail, 0, sizeof tail);
    memcpy(tail, data + 64 * full, rem);
    tail[rem] = 0x80;
    size_t tl = rem + 1 + 8 <= 64 ? 64 : 128;
    uint64_t bits = (uint64_t)len * 8;
    for (int i = 0; i < 8; i++) tail[tl - 1 - i] = (uint8_t)(bits >> (8 * i));
    sha_block(h, tail);
    if (tl == 128) sha_block(h, tail + 64);
    for (int i = 0; i < 8; i++) {
        out[4 * i] = (uint8_t)(h[i] >> 24);
        out[4 * i + 1] = (uint8_t)(h[i] >> 16);
        out[4 * i + 2] = (uint8_t)(h[i] >> 8);
        out[4 * i + 3] = (uint8_t)h[i];
    }
}

/* ============================================================================
 * Transcript (crates/zkie-core/src/common/transcript.rs:21-80).
 * ========================================================================== */
void orc_transcript_new(orc_transcript *t, const uint8_t *domain, size_t len)
{
    orc_sha256(domain, len, t->state);
    t->counter = 0;
}

void orc_transcript_absorb(orc_transcript *t, const uint8_t *data, size_t len)
{
    uint8_t *buf = (uint8_t *)malloc(32 + len);
    memcpy(buf, t->state, 32);
    if (len) memcpy(buf + 32, data, len);
    orc_sha256(buf, 32 + len, t->state);
    free(buf);
}

void orc_transcript_absorb_u64(orc_transcript *t, uint64_t x)
{
    uint8_t b[8];
    for (int i = 0; i < 8; i++) b[i] = (uint8_t)(x >> (8 * i));
    orc_transcript_absorb(t, b, 8);
}

static uint64_t transcript_draw(orc_transcript *t)
{
    uint8_t buf[40], d[32];
    memcpy(buf, t->state, 32);
    for (int i = 0; i < 8; i++) buf[32 + i] = (uint8_t)(t->counter >> (8 * i));
    t->counter += 1;
    orc_sha256(buf, 40, d);
    uint64_t v = 0;
    for (int i = 0; i < 8; i++) v |= (uint64_t)d[i] << (8 * i);
    return v;
}

uint64_t orc_transcript_field(orc_transcript *t)
{
    for (;;) {
        uint64_t c = transcript_draw(t);
        if (c < ORC_P) return c;
    }
}

uint64_t orc_transcript_next_u64(orc_transcript *t) { return transcript_draw(t); }

/* ============================================================================
 * Packed lanes (oracle/packed_field.h): the DFT runs blocks of adjacent
 * columns and the Merkle loops groups of rows / pairs one per SIMD lane, the
 * lane count chosen once per process from what the CPU offers (8 with
 * AVX-512F, 4 with AVX2, else 0: the scalar forms), the remainder through
 * the scalar forms.
 * ========================================================================== */
#if defined(__x86_64__) && defined(__GNUC__)
#define PW 8
#define PTGT __attribute__((target("avx512f")))
#define PMUL32(a, b) ((pv_x8)_mm512_mul_epu32((__m512i)(a), (__m512i)(b)))
#define PSUF _x8
#define PADD_IF_LT(x, a, b, c) \
    ((pv_x8)_mm512_mask_add_epi64((__m512i)(x), _mm512_cmplt_epu64_mask((__m512i)(a), (__m512i)(b)), \
                                  (__m512i)(x), (__m512i)(c)))
#define PSUB_IF_LT(x, a, b, c) \
    ((pv_x8)_mm512_mask_sub_epi64((__m512i)(x), _mm512_cmplt_epu64_mask((__m512i)(a), (__m512i)(b)), \
                                  (__m512i)(x), (__m512i)(c)))
#define PSUB_IF_GE(x, a, b, c) \
    ((pv_x8)_mm512_mask_sub_epi64((__m512i)(x), _mm512_cmpge_epu64_mask((__m512i)(a), (__m512i)(b)), \
                                  (__m512i)(x), (__m512i)(c)))
#include "packed_field.h"
#undef PW
#undef PTGT
#undef PMUL32
#undef PSUF
#undef PADD_IF_LT
#undef PSUB_IF_LT
#undef PSUB_IF_GE

#define PW 4
#define PTGT __attribute__((target("avx2")))
#define PMUL32(a, b) ((pv_x4)_mm256_mul_epu32((__m256i)(a), (__m256i)(b)))
#define PSUF _x4
#include "packed_field.h"
#undef PW
#undef PTGT
#undef PMUL32
#undef PSUF
#define ORC_HAVE_PACKED 1
#endif

static int g_lanes; /* 0 = scalar */

static int best_lanes(void)
{
#ifdef ORC_HAVE_PACKED
    __builtin_cpu_init();
    if (__builtin_cpu_supports("avx512f")) return 8;
    if (__builtin_cpu_supports("avx2")) return 4;
#endif
    return 0;
}

__attribute__((constructor)) static void init_lanes(void) { g_lanes = best_lanes(); }

int orc_set_lanes(int lanes)
{
    const int best = best_lanes();
    if (lanes < 0 || lanes > best) lanes = best;
    if (lanes != 0 && lanes != 4 && lanes != 8) lanes = best;
    g_lanes = lanes;
    return lanes;
}

/* ============================================================================
 * DFT.  Contract of p3 `TwoAdicSubgroupDft::dft_batch`, restated at
 * crates/zkie-core/cuda/goldilocks_ntt.cu:1-23: out[i] = sum_j x[j] w^(ij),
 * w = TWO_ADIC_GENERATORS[lg h], natural order in and out, canonical output.
 * ========================================================================== */
static uint32_t bitrev(uint32_t x, uint32_t bits)
{
    uint32_t r = 0;
    for (uint32_t b = 0; b < bits; b++) {
        r = (r << 1) | (x & 1);
        x >>= 1;
    }
    return r;
}

/* tw = the twiddles of every stage, stage s (half = 2^(s-1)) at offset
 * half - 1: w_{2^s}^j for j < half (2^lg - 1 values in all). */
static uint64_t *dft_twiddles(uint32_t lg)
{
    uint64_t *tw = (uint64_t *)malloc(sizeof(uint64_t) * ((1ULL << lg) > 1 ? (1ULL << lg) : 2));
    for (uint32_t s = 1; s <= lg; s++) {
        uint64_t half = 1ULL << (s - 1), root = orc_two_adic_generator(s);
        uint64_t *t = tw + half - 1;
        t[0] = 1;
        for (uint64_t j = 1; j < half; j++) t[j] = orc_mul(t[j - 1], root);
    }
    return tw;
}

/* Radix-2 decimation in time on one column, natural order in and out; rev
 * = the bit-reversal permutation of lg bits. */
static void dft_column(uint64_t *v, uint32_t lg, const uint64_t *tw_all, const uint32_t *rev)
{
    uint64_t n = 1ULL << lg;
    for (uint64_t i = 0; i < n; i++) {
        uint64_t j = rev[i];
        if (j > i) {
            uint64_t t = v[i];
            v[i] = v[j];
            v[j] = t;
        }
    }
    for (uint32_t s = 1; s <= lg; s++) {
        uint64_t half = 1ULL << (s - 1);
        const uint64_t *tw = tw_all + half - 1;
        for (uint64_t base = 0; base < n; base += 2 * half)
            for (uint64_t j = 0; j < half; j++) {
                uint64_t u = v[base + j];
                uint64_t x = orc_mul(v[base + j + half], tw[j]);
                v[base + j] = orc_add(u, x);
                v[base + j + half] = orc_sub(u, x);
            }
    }
}

/* Columns go through in blocks: with packed lanes, `lanes` adjacent columns
 * per block as one vector per row (dft_block, one lane per column); the
 * columns past the last full block, or all of them without lanes, in blocks
 * of eight (one 64-byte line of a row holds a block's values), each column
 * gathered into a contiguous buffer, transformed and scattered back.  The
 * twiddles and the bit-reversal are built once. */
#define DFT_BLOCK 8
static void dft_packed_columns(int lanes, uint64_t *mat, uint64_t w, uint64_t c0, uint32_t lg,
                               const uint64_t *tw, const uint32_t *rev, void *buf)
{
#ifdef ORC_HAVE_PACKED
    if (lanes == 8) {
        dft_columns_x8(mat, w, c0, lg, tw, rev, (pv_x8 *)buf);
        return;
    }
    if (lanes == 4) {
        dft_columns_x4(mat, w, c0, lg, tw, rev, (pv_x4 *)buf);
        return;
    }
#endif
    (void)lanes, (void)mat, (void)w, (void)c0, (void)lg, (void)tw, (void)rev, (void)buf;
}

void orc_dft_batch(uint64_t *mat, uint32_t lg_h, uint64_t w)
{
    if (lg_h == 0 || w == 0) {
        for (uint64_t i = 0; i < (w << lg_h); i++) mat[i] = canon(mat[i]);
        return;
    }
    uint64_t h = 1ULL << lg_h;
    uint64_t *tw = dft_twiddles(lg_h);
    uint32_t *rev = (uint32_t *)malloc(sizeof(uint32_t) * h);
    for (uint64_t i = 0; i < h; i++) rev[i] = bitrev((uint32_t)i, lg_h);
    const int lanes = g_lanes;
    const int64_t packed = lanes ? (int64_t)(w / (uint64_t)lanes) : 0;
    const uint64_t c_rest = (uint64_t)packed * (uint64_t)lanes;
    int64_t blocks = (int64_t)((w - c_rest + DFT_BLOCK - 1) / DFT_BLOCK);
#pragma omp parallel
    {
        if (packed) {
            void *buf = aligned_alloc(64, 64 * h);
#pragma omp for schedule(dynamic, 1) nowait
            for (int64_t blk = 0; blk < packed; blk++)
                dft_packed_columns(lanes, mat, w, (uint64_t)blk * (uint64_t)lanes, lg_h, tw, rev, buf);
            free(buf);
        }
        uint64_t *col = blocks ? (uint64_t *)malloc(sizeof(uint64_t) * h * DFT_BLOCK) : NULL;
#pragma omp for schedule(dynamic, 1)
        for (int64_t blk = 0; blk < blocks; blk++) {
            uint64_t c0 = c_rest + (uint64_t)blk * DFT_BLOCK, nc = w - c0 < DFT_BLOCK ? w - c0 : DFT_BLOCK;
            for (uint64_t i = 0; i < h; i++)
                for (uint64_t c = 0; c < nc; c++) col[c * h + i] = canon(mat[i * w + c0 + c]);
            for (uint64_t c = 0; c < nc; c++) dft_column(col + c * h, lg_h, tw, rev);
            for (uint64_t i = 0; i < h; i++)
                for (uint64_t c = 0; c < nc; c++) mat[i * w + c0 + c] = col[c * h + i];
        }
        free(col);
    }
    free(tw);
    free(rev);
}

void orc_dft_naive(const uint64_t *in, uint64_t *out, uint32_t lg_h, uint64_t w)
{
    uint64_t h = 1ULL << lg_h;
    uint64_t omega = orc_two_adic_generator(lg_h);
    for (uint64_t c = 0; c < w; c++)
        for (uint64_t i = 0; i < h; i++) {
            uint64_t wi = orc_pow(omega, i), acc = 0, pw = 1;
            for (uint64_t j = 0; j < h; j++) {
                acc = orc_add(acc, orc_mul(canon(in[j * w + c]), pw));
                pw = orc_mul(pw, wi);
            }
            out[i * w + c] = acc;
        }
}

uint64_t orc_poly_eval_col(const uint64_t *mat, uint64_t L, uint64_t w, uint64_t col, uint64_t x)
{
    uint64_t acc = 0;
    for (uint64_t j = L; j-- > 0;) acc = orc_add(orc_mul(acc, x), canon(mat[j * w + col]));
    return acc;
}

/* Zero-pad L rows to L << lg_blowup rows, then dft_batch: the Suffix-order
 * pad + DFT of vendor/p3-whir/src/pcs/committer/writer.rs:73-82 and the
 * BASELINE raw-commit sweep (shift 1). */
void orc_lde(const uint64_t *in, uint64_t *out, uint32_t lg_l, uint32_t lg_blowup, uint64_t w)
{
    uint64_t L = 1ULL << lg_l, H = L << lg_blowup;
    memcpy(out, in, sizeof(uint64_t) * L * w);
    memset(out + L * w, 0, sizeof(uint64_t) * (H - L) * w);
    orc_dft_batch(out, lg_l + lg_blowup, w);
}

/* ============================================================================
 * Poseidon2-16 over Goldilocks.  Structure restated from
 * crates/zkie-core/cuda/poseidon2_merkle.cu:37-155 (p3-poseidon2 generic
 * permutation, x^7 S-box, light external MDS, width-16 internal diffusion).
 * ========================================================================== */
static uint64_t sbox7(uint64_t x)
{
    uint64_t x2 = orc_mul(x, x), x3 = orc_mul(x2, x), x4 = orc_mul(x2, x2);
    return orc_mul(x3, x4);
}

/* [2 3 1 1; 1 2 3 1; 1 1 2 3; 3 1 1 2] (poseidon2_merkle.cu:61-76) on one
 * 4-lane block of canonical inputs, unreduced: each output is a sum of seven
 * inputs, below 7 p < 2^67, so the sums run in 128 bits. */
static inline void mat4_acc(const uint64_t *x, u128 *y)
{
    u128 a = x[0], b = x[1], c = x[2], d = x[3];
    y[0] = 2 * a + 3 * b + c + d;
    y[1] = a + 2 * b + 3 * c + d;
    y[2] = a + b + 2 * c + 3 * d;
    y[3] = 3 * a + b + c + 2 * d;
}

/* mds_light16 (poseidon2_merkle.cu:78-97): the 4x4 block on each chunk, then
 * the per-residue column sums added; one reduction per output. */
static void mds_light16(uint64_t *st)
{
    u128 y[16];
    for (int j = 0; j < 16; j += 4) mat4_acc(st + j, y + j);
    u128 sums[4];
    for (int k = 0; k < 4; k++) sums[k] = y[k] + y[4 + k] + y[8 + k] + y[12 + k];
    for (int i = 0; i < 16; i++) st[i] = reduce128(y[i] + sums[i & 3]);
}

/* Internal diagonal V (matrix 1 + diag(V)), poseidon2_merkle.cu:111-142:
 * V = [-2, 1, 2, 1/2, 3, 4, -1/2, -3, -4, 1/2^3, 1/2^4, 1/2^5,
 *      -1/2^3, -1/2^4, -1/2^5, diag15]. */
static uint64_t V_BASE[15];

__attribute__((constructor)) static void init_internal_diag(void)
{
    uint64_t inv2 = orc_inv(2);
    uint64_t i8 = orc_pow(inv2, 3), i16 = orc_pow(inv2, 4), i32 = orc_pow(inv2, 5);
    uint64_t V[15] = {ORC_P - 2, 1, 2, inv2, 3, 4, ORC_P - inv2, ORC_P - 3, ORC_P - 4,
                      i8, i16, i32, ORC_P - i8, ORC_P - i16, ORC_P - i32};
    memcpy(V_BASE, V, sizeof V);
}

void orc_p2_permute(const orc_p2_consts *c, uint64_t st[16])
{
    uint64_t V[16];
    memcpy(V, V_BASE, sizeof V_BASE);
    V[15] = c->diag15;
    for (int i = 0; i < 16; i++) st[i] = canon(st[i]);
    mds_light16(st);
    for (int r = 0; r < 4; r++) {
        for (int i = 0; i < 16; i++) st[i] = sbox7(orc_add(st[i], c->ext_init[r][i]));
        mds_light16(st);
    }
    for (int r = 0; r < 22; r++) {
        st[0] = sbox7(orc_add(st[0], c->internal[r]));
        u128 acc = 0;
        for (int i = 0; i < 16; i++) acc += st[i];
        const uint64_t sum = reduce128(acc);
        /* sum + V_i st_i, reduced once (the product and the sum in 128 bits) */
        for (int i = 0; i < 16; i++) st[i] = reduce128((u128)V[i] * st[i] + sum);
    }
    for (int r = 0; r < 4; r++) {
        for (int i = 0; i < 16; i++) st[i] = sbox7(orc_add(st[i], c->ext_final[r][i]));
        mds_light16(st);
    }
}

static void p2_diag(const orc_p2_consts *c, uint64_t diag[16])
{
    memcpy(diag, V_BASE, sizeof V_BASE);
    diag[15] = c->diag15;
}

/* rows [0, h) of a row-major h x w matrix hashed into digests; `lanes`
 * states per group, the rows past the last full group one by one */
static void p2_hash_group(int lanes, const orc_p2_consts *c, const uint64_t *diag, const uint64_t *rows,
                          uint64_t w, uint64_t *digests)
{
#ifdef ORC_HAVE_PACKED
    if (lanes == 8) {
        p2_hash_rows_x8(c, diag, rows, w, digests);
        return;
    }
    if (lanes == 4) {
        p2_hash_rows_x4(c, diag, rows, w, digests);
        return;
    }
#endif
    (void)c, (void)diag, (void)rows, (void)w, (void)digests, (void)lanes;
}

static void p2_compress_group(int lanes, const orc_p2_consts *c, const uint64_t *diag, const uint64_t *prev,
                              uint64_t *next)
{
#ifdef ORC_HAVE_PACKED
    if (lanes == 8) {
        p2_compress_pairs_x8(c, diag, prev, next);
        return;
    }
    if (lanes == 4) {
        p2_compress_pairs_x4(c, diag, prev, next);
        return;
    }
#endif
    (void)c, (void)diag, (void)prev, (void)next, (void)lanes;
}

/* --- round-constant derivation (pcs/merkle_cuda.rs:54-85) ------------------
 * rand 0.10 `SmallRng::seed_from_u64` is restated as xoshiro256++ whose state
 * is filled by SplitMix64 (the published algorithms); p3-goldilocks samples a
 * `Goldilocks` from `StandardUniform` by rejecting next_u64() >= p.  The crates
 * are absent here, so these constants are UNPINNED. */
static uint64_t splitmix64(uint64_t *s)
{
    *s += 0x9e3779b97f4a7c15ULL;
    uint64_t z = *s;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

static uint64_t rotl64(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

static uint64_t xoshiro_next(uint64_t s[4])
{
    uint64_t result = rotl64(s[0] + s[3], 23) + s[0];
    uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl64(s[3], 45);
    return result;
}

static uint64_t sample_field(uint64_t s[4])
{
    for (;;) {
        uint64_t v = xoshiro_next(s);
        if (v < ORC_P) return v;
    }
}

void orc_p2_derive_constants(uint64_t seed, orc_p2_consts *c)
{
    uint64_t sm = seed, s[4];
    for (int i = 0; i < 4; i++) s[i] = splitmix64(&sm);
    /* ExternalLayerConstants::new_from_rng(8, rng): 4 initial [F;16], then 4
     * terminal [F;16]; then 22 internal constants. */
    for (int r = 0; r < 4; r++)
        for (int i = 0; i < 16; i++) c->ext_init[r][i] = sample_field(s);
    for (int r = 0; r < 4; r++)
        for (int i = 0; i < 16; i++) c->ext_final[r][i] = sample_field(s);
    for (int r = 0; r < 22; r++) c->internal[r] = sample_field(s);
    /* MATRIX_DIAG_16_GOLDILOCKS[15] = 2^-32 mod p (poseidon2_merkle.cu:34,141). */
    c->diag15 = orc_inv(orc_pow(2, 32));
}

/* PaddingFreeSponge<Perm, 16, 8, 8>: overwrite the rate, permute per full
 * block and once after a partial tail; digest = state[0..8]. */
void orc_p2_hash_row(const orc_p2_consts *c, const uint64_t *row, uint64_t w, uint64_t out[8])
{
    uint64_t st[16] = {0};
    uint64_t nb = w >> 3, rem = w & 7;
    for (uint64_t b = 0; b < nb; b++) {
        for (int i = 0; i < 8; i++) st[i] = canon(row[8 * b + i]);
        orc_p2_permute(c, st);
    }
    if (rem) {
        for (uint64_t i = 0; i < rem; i++) st[i] = canon(row[8 * nb + i]);
        orc_p2_permute(c, st);
    }
    memcpy(out, st, 64);
}

void orc_p2_compress(const orc_p2_consts *c, const uint64_t l[8], const uint64_t r[8], uint64_t out[8])
{
    uint64_t st[16];
    memcpy(st, l, 64);
    memcpy(st + 8, r, 64);
    orc_p2_permute(c, st);
    memcpy(out, st, 64);
}

/* ============================================================================
 * Merkle geometry for one matrix: vendor/p3-merkle-tree/src/merkle_tree.rs
 * (first_digest_layer :372-442, compress :594-642, padded_len :577-585) as
 * driven by pcs/merkle_cuda.rs:203-280.
 * ========================================================================== */
uint64_t orc_padded_len(uint64_t raw_len, uint64_t n)
{
    if (raw_len <= 1) return raw_len;
    if (raw_len >= n) return (raw_len + n - 1) / n * n;
    return n;
}

uint32_t orc_merkle_num_layers(uint64_t h)
{
    uint64_t len = orc_padded_len(h, 2);
    uint32_t n = 1;
    while (len > 1) {
        len = orc_padded_len(len / 2, 2);
        n++;
    }
    return n;
}

uint64_t orc_merkle_total_digests(uint64_t h)
{
    uint64_t len = orc_padded_len(h, 2), tot = len;
    while (len > 1) {
        len = orc_padded_len(len / 2, 2);
        tot += len;
    }
    return tot;
}

void orc_merkle_leaves(const orc_p2_consts *c, const uint64_t *mat, uint64_t h, uint64_t w,
                       uint64_t *digests, int threads)
{
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#endif
    const int lanes = g_lanes;
    const uint64_t groups = lanes ? h / (uint64_t)lanes : 0, done = groups * (uint64_t)lanes;
    uint64_t diag[16];
    p2_diag(c, diag);
#ifdef _OPENMP
#pragma omp parallel num_threads(threads)
#endif
    {
#ifdef _OPENMP
#pragma omp for schedule(static) nowait
#endif
        for (int64_t g = 0; g < (int64_t)groups; g++) {
            const uint64_t r = (uint64_t)g * (uint64_t)lanes;
            p2_hash_group(lanes, c, diag, mat + r * w, w, digests + 8 * r);
        }
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
        for (int64_t r = (int64_t)done; r < (int64_t)h; r++)
            orc_p2_hash_row(c, mat + (uint64_t)r * w, w, digests + 8 * r);
    }
    (void)threads;
}

static void build_layers(const orc_p2_consts *c, uint64_t *layers, uint64_t h, uint64_t root[8])
{
    uint64_t diag[16];
    p2_diag(c, diag);
    uint64_t len = orc_padded_len(h, 2);
    for (uint64_t i = h; i < len; i++) memset(layers + 8 * i, 0, 64);
    uint64_t *prev = layers;
    while (len > 1) {
        uint64_t raw = len / 2, next_len = orc_padded_len(raw, 2);
        uint64_t *next = prev + 8 * len;
        memset(next, 0, 64 * next_len);
        const int lanes = g_lanes;
        const uint64_t groups = lanes ? raw / (uint64_t)lanes : 0, done = groups * (uint64_t)lanes;
#pragma omp parallel for schedule(static) if (groups > 512)
        for (int64_t g = 0; g < (int64_t)groups; g++) {
            const uint64_t i = (uint64_t)g * (uint64_t)lanes;
            p2_compress_group(lanes, c, diag, prev + 16 * i, next + 8 * i);
        }
        for (uint64_t i = done; i < raw; i++) orc_p2_compress(c, prev + 16 * i, prev + 16 * i + 8, next + 8 * i);
        prev = next;
        len = next_len;
    }
    memcpy(root, prev, 64);
}

void orc_merkle_tree(const orc_p2_consts *c, const uint64_t *mat, uint64_t h, uint64_t w,
                     uint64_t *layers, uint64_t root[8], int threads)
{
    orc_merkle_leaves(c, mat, h, w, layers, threads);
    build_layers(c, layers, h, root);
}

void orc_merkle_root_from_leaves(const orc_p2_consts *c, const uint64_t *leaves, uint64_t h,
                                 uint64_t root[8])
{
    uint64_t *layers = (uint64_t *)malloc(sizeof(uint64_t) * 8 * orc_merkle_total_digests(h));
    memcpy(layers, leaves, 64 * h);
    build_layers(c, layers, h, root);
    free(layers);
}

/* ============================================================================
 * WHIR base commit (pcs/whir.rs:438-469; committer/writer.rs:73-82 layout):
 * 2^n evaluations viewed row-major with width 2^5, zero-padded to twice the
 * height (starting_log_inv_rate 1), DFT per column, Merkle over rows.
 * ========================================================================== */
void orc_whir_commit(const orc_p2_consts *c, const uint64_t *evals, uint32_t n, uint64_t *lde_out,
                     uint64_t root[8], int threads)
{
    uint32_t lg_rows = n - 5;
    orc_lde(evals, lde_out, lg_rows, 1, 32);
    uint64_t H = 2ULL << lg_rows;
    uint64_t *layers = (uint64_t *)malloc(sizeof(uint64_t) * 8 * orc_merkle_total_digests(H));
    orc_merkle_tree(c, lde_out, H, 32, layers, root, threads);
    free(layers);
}

/* ============================================================================
 * MLE (crates/zkie-core/src/common/mle.rs:8-64).  Variable 0 = LSB.
 * ========================================================================== */
uint64_t orc_mle_eval(const uint64_t *values, uint32_t t, const uint64_t *point)
{
    uint64_t n = 1ULL << t;
    uint64_t *buf = (uint64_t *)malloc(sizeof(uint64_t) * n);
    for (uint64_t i = 0; i < n; i++) buf[i] = canon(values[i]);
    uint64_t size = n;
    for (uint32_t r = 0; r < t; r++) {
        uint64_t half = size / 2;
        for (uint64_t i = 0; i < half; i++) {
            uint64_t a = buf[2 * i], b = buf[2 * i + 1];
            buf[i] = orc_add(a, orc_mul(point[r], orc_sub(b, a)));
        }
        size = half;
    }
    uint64_t out = buf[0];
    free(buf);
    return out;
}

void orc_mle_partial_eval(const uint64_t *values, uint32_t t, const uint64_t *fix, uint32_t f,
                          uint64_t *out)
{
    uint64_t n = 1ULL << t;
    uint64_t *buf = (uint64_t *)malloc(sizeof(uint64_t) * n);
    for (uint64_t i = 0; i < n; i++) buf[i] = canon(values[i]);
    uint64_t size = n;
    for (uint32_t r = 0; r < f; r++) {
        uint64_t half = size / 2;
        for (uint64_t i = 0; i < half; i++) {
            uint64_t a = buf[2 * i], b = buf[2 * i + 1];
            buf[i] = orc_add(a, orc_mul(fix[r], orc_sub(b, a)));
        }
        size = half;
    }
    memcpy(out, buf, sizeof(uint64_t) * size);
    free(buf);
}

void orc_eq_evals(const uint64_t *r, uint32_t d, uint64_t *out)
{
    /* doubling, variable j on bit j: entries with bit j set take r_j, the
     * others 1 - r_j (mle.rs eq_evals) */
    out[0] = 1;
    uint64_t size = 1;
    for (uint32_t j = 0; j < d; j++) {
        const uint64_t rj = canon(r[j]), om = orc_sub(1, rj);
#pragma omp parallel for schedule(static) if (size >= 4096)
        for (int64_t i = 0; i < (int64_t)size; i++) {
            const uint64_t v = out[i];
            out[i + size] = orc_mul(v, rj);
            out[i] = orc_mul(v, om);
        }
        size <<= 1;
    }
}

/* ============================================================================
 * Sumchecks (crates/zkie-core/src/common/sumcheck.rs).
 * ========================================================================== */
static const uint64_t INV2 = ORC_P / 2 + 1;

static void fold_vec(uint64_t *buf, uint64_t len, uint64_t r)
{
    for (uint64_t i = 0; i < len / 2; i++) {
        uint64_t a = buf[2 * i], b = buf[2 * i + 1];
        buf[i] = orc_add(a, orc_mul(r, orc_sub(b, a)));
    }
}

/* prove (:33-79) + fold (:81-89). */
void orc_sumcheck_prove(const uint64_t *f, const uint64_t *h, uint32_t t, const uint64_t *ch,
                        uint64_t *rounds, uint64_t finals[2])
{
    uint64_t n = 1ULL << t;
    uint64_t *fb = (uint64_t *)malloc(8 * n), *hb = (uint64_t *)malloc(8 * n);
    for (uint64_t i = 0; i < n; i++) {
        fb[i] = canon(f[i]);
        hb[i] = canon(h[i]);
    }
    uint64_t len = n;
    for (uint32_t r = 0; r < t; r++) {
        uint64_t y0 = 0, y1 = 0, y2 = 0;
        for (uint64_t s = 0; s < len / 2; s++) {
            uint64_t f0 = fb[2 * s], f1 = fb[2 * s + 1], h0 = hb[2 * s], h1 = hb[2 * s + 1];
            y0 = orc_add(y0, orc_mul(f0, h0));
            y1 = orc_add(y1, orc_mul(f1, h1));
            uint64_t f2 = orc_sub(orc_add(f1, f1), f0), h2 = orc_sub(orc_add(h1, h1), h0);
            y2 = orc_add(y2, orc_mul(f2, h2));
        }
        uint64_t c0 = y0;
        uint64_t c1 = orc_mul(orc_sub(orc_sub(orc_mul(4, y1), y2), orc_mul(3, y0)), INV2);
        uint64_t c2 = orc_mul(orc_add(orc_sub(y2, orc_add(y1, y1)), y0), INV2);
        rounds[3 * r] = c0;
        rounds[3 * r + 1] = c1;
        rounds[3 * r + 2] = c2;
        fold_vec(fb, len, ch[r]);
        fold_vec(hb, len, ch[r]);
        len /= 2;
    }
    finals[0] = fb[0];
    finals[1] = hb[0];
    free(fb);
    free(hb);
}

/* verify (:91-111). */
int orc_sumcheck_verify(const uint64_t *rounds, uint32_t t, uint64_t claimed, const uint64_t *ch,
                        uint64_t f_eval, uint64_t h_eval)
{
    uint64_t prev = claimed;
    for (uint32_t r = 0; r < t; r++) {
        uint64_t c0 = rounds[3 * r], c1 = rounds[3 * r + 1], c2 = rounds[3 * r + 2];
        uint64_t p1 = orc_add(orc_add(c0, c1), c2);
        if (orc_add(c0, p1) != prev) return 0;
        uint64_t x = ch[r];
        prev = orc_add(orc_add(c0, orc_mul(c1, x)), orc_mul(orc_mul(c2, x), x));
    }
    return prev == orc_mul(f_eval, h_eval);
}

static uint64_t eval_at(uint64_t f0, uint64_t f1, uint64_t t) { return orc_add(f0, orc_mul(orc_sub(f1, f0), t)); }

/* prove3 (:162-209) with interpolate_cubic (:144-159). */
void orc_sumcheck3_prove(const uint64_t *f, const uint64_t *g, const uint64_t *h, uint32_t t,
                         const uint64_t *ch, uint64_t *rounds, uint64_t finals[3])
{
    uint64_t n = 1ULL << t;
    uint64_t *fb = (uint64_t *)malloc(8 * n), *gb = (uint64_t *)malloc(8 * n), *hb = (uint64_t *)malloc(8 * n);
    for (uint64_t i = 0; i < n; i++) {
        fb[i] = canon(f[i]);
        gb[i] = canon(g[i]);
        hb[i] = canon(h[i]);
    }
    uint64_t inv2 = orc_inv(2), inv3 = orc_inv(3), inv6 = orc_inv(6);
    uint64_t len = n;
    for (uint32_t r = 0; r < t; r++) {
        uint64_t p0 = 0, p1 = 0, p2 = 0, p3 = 0;
        for (uint64_t s = 0; s < len / 2; s++) {
            uint64_t f0 = fb[2 * s], f1 = fb[2 * s + 1], g0 = gb[2 * s], g1 = gb[2 * s + 1];
            uint64_t h0 = hb[2 * s], h1 = hb[2 * s + 1];
            p0 = orc_add(p0, orc_mul(orc_mul(f0, g0), h0));
            p1 = orc_add(p1, orc_mul(orc_mul(f1, g1), h1));
            p2 = orc_add(p2, orc_mul(orc_mul(eval_at(f0, f1, 2), eval_at(g0, g1, 2)), eval_at(h0, h1, 2)));
            p3 = orc_add(p3, orc_mul(orc_mul(eval_at(f0, f1, 3), eval_at(g0, g1, 3)), eval_at(h0, h1, 3)));
        }
        uint64_t d1_0 = orc_sub(p1, p0), d1_1 = orc_sub(p2, p1), d1_2 = orc_sub(p3, p2);
        uint64_t d2_0 = orc_sub(d1_1, d1_0), d2_1 = orc_sub(d1_2, d1_1);
        uint64_t d3_0 = orc_sub(d2_1, d2_0);
        rounds[4 * r] = p0;
        rounds[4 * r + 1] = orc_add(orc_sub(d1_0, orc_mul(d2_0, inv2)), orc_mul(d3_0, inv3));
        rounds[4 * r + 2] = orc_sub(orc_mul(d2_0, inv2), orc_mul(d3_0, inv2));
        rounds[4 * r + 3] = orc_mul(d3_0, inv6);
        fold_vec(fb, len, ch[r]);
        fold_vec(gb, len, ch[r]);
        fold_vec(hb, len, ch[r]);
        len /= 2;
    }
    finals[0] = fb[0];
    finals[1] = gb[0];
    finals[2] = hb[0];
    free(fb);
    free(gb);
    free(hb);
}

/* verify3 (:211-232). */
int orc_sumcheck3_verify(const uint64_t *rounds, uint32_t t, uint64_t claimed, const uint64_t *ch,
                         uint64_t f_eval, uint64_t g_eval, uint64_t h_eval)
{
    uint64_t prev = claimed;
    for (uint32_t r = 0; r < t; r++) {
        const uint64_t *c = rounds + 4 * r;
        uint64_t p1 = orc_add(orc_add(c[0], c[1]), orc_add(c[2], c[3]));
        if (orc_add(c[0], p1) != prev) return 0;
        uint64_t x = ch[r], x2 = orc_mul(x, x), x3 = orc_mul(x2, x);
        prev = orc_add(orc_add(c[0], orc_mul(c[1], x)), orc_add(orc_mul(c[2], x2), orc_mul(c[3], x3)));
    }
    return prev == orc_mul(orc_mul(f_eval, g_eval), h_eval);
}

/* prove_sum_of_products (:243-286). */
void orc_sum_of_products_prove(const uint64_t *weights, const uint64_t *values, uint32_t n_tables,
                               uint32_t t, const uint64_t *ch, uint64_t *rounds, uint64_t *b_eval)
{
    uint64_t n = 1ULL << t;
    uint64_t *wb = (uint64_t *)malloc(8 * n * n_tables), *vb = (uint64_t *)malloc(8 * n * n_tables);
    for (uint64_t i = 0; i < n * n_tables; i++) {
        wb[i] = canon(weights[i]);
        vb[i] = canon(values[i]);
    }
    uint64_t len = n;
    for (uint32_t r = 0; r < t; r++) {
        uint64_t p0 = 0, p1 = 0, p2 = 0;
        for (uint32_t i = 0; i < n_tables; i++) {
            const uint64_t *w = wb + i * n, *v = vb + i * n;
            for (uint64_t s = 0; s < len / 2; s++) {
                uint64_t w0 = w[2 * s], w1 = w[2 * s + 1], v0 = v[2 * s], v1 = v[2 * s + 1];
                p0 = orc_add(p0, orc_mul(w0, v0));
                p1 = orc_add(p1, orc_mul(w1, v1));
                p2 = orc_add(p2, orc_mul(orc_sub(orc_add(w1, w1), w0), orc_sub(orc_add(v1, v1), v0)));
            }
        }
        rounds[3 * r] = p0;
        rounds[3 * r + 1] = orc_mul(orc_sub(orc_sub(orc_mul(4, p1), p2), orc_mul(3, p0)), INV2);
        rounds[3 * r + 2] = orc_mul(orc_add(orc_sub(p2, orc_add(p1, p1)), p0), INV2);
        for (uint32_t i = 0; i < n_tables; i++) {
            fold_vec(wb + i * n, len, ch[r]);
            fold_vec(vb + i * n, len, ch[r]);
        }
        len /= 2;
    }
    uint64_t acc = 0;
    for (uint32_t i = 0; i < n_tables; i++) acc = orc_add(acc, orc_mul(wb[i * n], vb[i * n]));
    *b_eval = acc;
    free(wb);
    free(vb);
}

/* prove_virtual (:378-438).  Round message = evaluations at t = 0..max_deg via
 * k*f1 - (k-1)*f0; fold (1-r)*f0 + r*f1.  As the reference's rayon loops, the
 * pairs of a round are summed in parallel (field addition is associative, so
 * the message does not depend on the split) and the fold writes a second
 * buffer. */
#define ORC_VMAX_DEG 16
void orc_virtual_prove(const uint64_t *mles, uint32_t n_mles, uint32_t t, const uint64_t *coeffs,
                       const uint32_t *idx_off, const uint32_t *idx, uint32_t n_terms,
                       const uint64_t *ch, uint64_t *rounds, uint64_t *finals)
{
    uint64_t n = 1ULL << t;
    uint32_t max_deg = 0;
    for (uint32_t i = 0; i < n_terms; i++)
        if (idx_off[i + 1] - idx_off[i] > max_deg) max_deg = idx_off[i + 1] - idx_off[i];
    if (max_deg > ORC_VMAX_DEG) max_deg = ORC_VMAX_DEG;
    uint64_t nm = n_mles ? n_mles : 1;
    uint64_t *cur = (uint64_t *)malloc(8 * n * nm), *nxt = (uint64_t *)malloc(8 * (n / 2 ? n / 2 : 1) * nm);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)(n * n_mles); i++) cur[i] = canon(mles[i]);
    uint64_t kf[ORC_VMAX_DEG + 1], km1[ORC_VMAX_DEG + 1];
    uint64_t *cf = (uint64_t *)malloc(8 * (n_terms ? n_terms : 1));
    for (uint32_t k = 0; k <= max_deg; k++) {
        kf[k] = orc_from_i64((int64_t)k);
        km1[k] = orc_from_i64((int64_t)k - 1);
    }
    for (uint32_t ti = 0; ti < n_terms; ti++) cf[ti] = canon(coeffs[ti]);
    uint64_t len = n;
    for (uint32_t r = 0; r < t; r++) {
        uint64_t *p = rounds + (uint64_t)r * (max_deg + 1);
        uint64_t acc[ORC_VMAX_DEG + 1] = {0};
        const uint64_t half = len / 2;
#pragma omp parallel
        {
            uint64_t loc[ORC_VMAX_DEG + 1] = {0};
#pragma omp for schedule(static)
            for (int64_t s = 0; s < (int64_t)half; s++)
                for (uint32_t ti = 0; ti < n_terms; ti++)
                    for (uint32_t k = 0; k <= max_deg; k++) {
                        uint64_t prod = cf[ti];
                        for (uint32_t q = idx_off[ti]; q < idx_off[ti + 1]; q++) {
                            const uint64_t *b = cur + (uint64_t)idx[q] * len;
                            uint64_t fk = orc_sub(orc_mul(kf[k], b[2 * s + 1]), orc_mul(km1[k], b[2 * s]));
                            prod = orc_mul(prod, fk);
                        }
                        loc[k] = orc_add(loc[k], prod);
                    }
#pragma omp critical
            for (uint32_t k = 0; k <= max_deg; k++) acc[k] = orc_add(acc[k], loc[k]);
        }
        for (uint32_t k = 0; k <= max_deg; k++) p[k] = acc[k];
        uint64_t rr = ch[r], om = orc_sub(1, rr);
#pragma omp parallel for schedule(static) collapse(2)
        for (uint32_t j = 0; j < n_mles; j++)
            for (int64_t s = 0; s < (int64_t)half; s++) {
                const uint64_t *b = cur + (uint64_t)j * len;
                nxt[(uint64_t)j * half + s] = orc_add(orc_mul(om, b[2 * s]), orc_mul(rr, b[2 * s + 1]));
            }
        uint64_t *tmp = cur;
        cur = nxt;
        nxt = tmp;
        len = half;
    }
    for (uint32_t j = 0; j < n_mles; j++) finals[j] = cur[(uint64_t)j * len];
    free(cur);
    free(nxt);
    free(cf);
}

/* interpolate (:439-453) + verify_virtual (:454-484). */
static uint64_t lagrange(const uint64_t *vals, uint64_t x, uint32_t d)
{
    uint64_t out = 0;
    for (uint32_t k = 0; k <= d; k++) {
        uint64_t term = vals[k];
        for (uint32_t j = 0; j <= d; j++) {
            if (j == k) continue;
            uint64_t num = orc_sub(x, orc_from_i64(j));
            uint64_t den = orc_sub(orc_from_i64(k), orc_from_i64(j));
            term = orc_mul(orc_mul(term, num), orc_inv(den));
        }
        out = orc_add(out, term);
    }
    return out;
}

int orc_virtual_verify(const uint64_t *rounds, uint32_t t, const uint64_t *coeffs,
                       const uint32_t *idx_off, const uint32_t *idx, uint32_t n_terms,
                       uint64_t claimed, const uint64_t *ch, const uint64_t *finals)
{
    uint32_t max_deg = 0;
    for (uint32_t i = 0; i < n_terms; i++)
        if (idx_off[i + 1] - idx_off[i] > max_deg) max_deg = idx_off[i + 1] - idx_off[i];
    uint64_t cur = claimed;
    for (uint32_t r = 0; r < t; r++) {
        const uint64_t *p = rounds + (uint64_t)r * (max_deg + 1);
        if (orc_add(p[0], p[1]) != cur) return 0;
        cur = lagrange(p, ch[r], max_deg);
    }
    uint64_t fv = 0;
    for (uint32_t ti = 0; ti < n_terms; ti++) {
        uint64_t prod = canon(coeffs[ti]);
        for (uint32_t q = idx_off[ti]; q < idx_off[ti + 1]; q++) prod = orc_mul(prod, finals[idx[q]]);
        fv = orc_add(fv, prod);
    }
    return cur == fv;
}

/* ============================================================================
 * Matmul GKR (crates/zkie-core/src/common/matmul.rs:17-46).
 * ========================================================================== */
static uint32_t tz(uint64_t x)
{
    uint32_t r = 0;
    while (x > 1 && !(x & 1)) {
        x >>= 1;
        r++;
    }
    return r;
}

void orc_matmul_prove(const uint64_t *at, const uint64_t *b, const uint64_t *c, uint64_t m,
                      uint64_t k, uint64_t n, const uint64_t *u, const uint64_t *v,
                      const uint64_t *ch, uint64_t *claimed, uint64_t *rounds, uint64_t finals[2])
{
    uint32_t lm = tz(m), lk = tz(k), ln = tz(n);
    uint64_t *ar = (uint64_t *)malloc(8 * k), *br = (uint64_t *)malloc(8 * k);
    orc_mle_partial_eval(at, lk + lm, u, lm, ar);
    orc_mle_partial_eval(b, lk + ln, v, ln, br);
    uint64_t *cp = (uint64_t *)malloc(8 * (ln + lm + 1));
    memcpy(cp, v, 8 * ln);
    memcpy(cp + ln, u, 8 * lm);
    *claimed = orc_mle_eval(c, ln + lm, cp);
    orc_sumcheck_prove(ar, br, lk, ch, rounds, finals);
    free(ar);
    free(br);
    free(cp);
}

void orc_matmul_field(const uint64_t *a, const uint64_t *b, uint64_t m, uint64_t k, uint64_t n,
                      uint64_t *c, int threads)
{
#ifdef _OPENMP
    if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel for num_threads(threads)
#endif
    for (int64_t i = 0; i < (int64_t)m; i++)
        for (uint64_t j = 0; j < n; j++) {
            uint64_t acc = 0;
            for (uint64_t q = 0; q < k; q++) acc = orc_add(acc, orc_mul(canon(a[i * k + q]), canon(b[q * n + j])));
            c[i * n + j] = acc;
        }
    (void)threads;
}

static int64_t to_i64_c(uint64_t v)
{
    v = canon(v);
    return v <= (uint64_t)INT64_MAX ? (int64_t)v : -(int64_t)(ORC_P - v);
}

/* par::mm_par_fixed (crates/zkie-ops/src/par.rs:41-89): the field product,
 * accumulated exactly in i64 (row-parallel, i-k-j order) when max|a| max|b| k
 * < 2^63, else the field matmul. */
void orc_matmul_fixed(const uint64_t *a, const uint64_t *b, uint64_t m, uint64_t k, uint64_t n, uint64_t *c)
{
    uint64_t max_a = 0, max_b = 0;
    for (uint64_t i = 0; i < m * k; i++) {
        const int64_t v = to_i64_c(a[i]);
        const uint64_t u = v < 0 ? 0ULL - (uint64_t)v : (uint64_t)v;
        if (u > max_a) max_a = u;
    }
    for (uint64_t i = 0; i < k * n; i++) {
        const int64_t v = to_i64_c(b[i]);
        const uint64_t u = v < 0 ? 0ULL - (uint64_t)v : (uint64_t)v;
        if (u > max_b) max_b = u;
    }
    if ((u128)max_a * max_b * k >= ((u128)1 << 63)) {
        orc_matmul_field(a, b, m, k, n, c, 0);
        return;
    }
    int64_t *bi = (int64_t *)malloc(8 * (k * n != 0 ? k * n : 1));
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)(k * n); i++) bi[i] = to_i64_c(b[i]);
#pragma omp parallel
    {
        int64_t *row = (int64_t *)malloc(8 * (n ? n : 1));
#pragma omp for schedule(static)
        for (int64_t i = 0; i < (int64_t)m; i++) {
            for (uint64_t j = 0; j < n; j++) row[j] = 0;
            for (uint64_t q = 0; q < k; q++) {
                const int64_t av = to_i64_c(a[i * k + q]);
                const int64_t *br = bi + q * n;
                for (uint64_t j = 0; j < n; j++) row[j] += av * br[j];
            }
            for (uint64_t j = 0; j < n; j++) c[i * n + j] = orc_from_i64(row[j]);
        }
        free(row);
    }
    free(bi);
}

uint64_t orc_challenger_field(orc_challenger *s)
{
    if (s->kind == 0) return orc_xorshift_field(&s->xs_state);
    return orc_transcript_field(&s->tr);
}

/* Op::MatMul arm (zkie-ops/src/compose.rs:1724-1747) with transpose (:52-60). */
void orc_op_matmul_prove(const uint64_t *a, const uint64_t *b, const uint64_t *c, uint64_t m,
                         uint64_t k, uint64_t n, orc_challenger *src, uint64_t *out_u,
                         uint64_t *out_v, uint64_t *out_ch, uint64_t *claimed, uint64_t *rounds,
                         uint64_t finals[2], uint64_t claims[3])
{
    uint32_t lm = tz(m), lk = tz(k), ln = tz(n);
    uint64_t *at = (uint64_t *)malloc(8 * m * k);
    for (uint64_t i = 0; i < m; i++)
        for (uint64_t q = 0; q < k; q++) at[q * m + i] = a[i * k + q];
    for (uint32_t i = 0; i < lm; i++) out_u[i] = orc_challenger_field(src);
    for (uint32_t i = 0; i < ln; i++) out_v[i] = orc_challenger_field(src);
    for (uint32_t i = 0; i < lk; i++) out_ch[i] = orc_challenger_field(src);
    orc_matmul_prove(at, b, c, m, k, n, out_u, out_v, out_ch, claimed, rounds, finals);
    uint64_t *pt = (uint64_t *)malloc(8 * (lm + lk + ln + 1));
    memcpy(pt, out_ch, 8 * lk);
    memcpy(pt + lk, out_u, 8 * lm);
    claims[0] = orc_mle_eval(a, lk + lm, pt);
    memcpy(pt, out_v, 8 * ln);
    memcpy(pt + ln, out_ch, 8 * lk);
    claims[1] = orc_mle_eval(b, ln + lk, pt);
    memcpy(pt, out_v, 8 * ln);
    memcpy(pt + ln, out_u, 8 * lm);
    claims[2] = orc_mle_eval(c, ln + lm, pt);
    free(pt);
    free(at);
}

/* prove_shard_dag master/child transcript (compose.rs:2276-2311):
 * Transcript::new("zkie-shard-dag-v1"), absorb ops_per_shard, ops.len(), then
 * for each op its reads (a, b) and writes (c); the child absorbs the shard index. */
void orc_shard_dag_child(const uint64_t *op_ids, uint32_t n_ops, uint64_t ops_per_shard,
                         uint64_t shard_index, orc_transcript *child)
{
    static const char dom[] = "zkie-shard-dag-v1";
    orc_transcript_new(child, (const uint8_t *)dom, sizeof(dom) - 1);
    orc_transcript_absorb_u64(child, ops_per_shard);
    orc_transcript_absorb_u64(child, n_ops);
    for (uint32_t i = 0; i < n_ops; i++) {
        orc_transcript_absorb_u64(child, op_ids[3 * i]);
        orc_transcript_absorb_u64(child, op_ids[3 * i + 1]);
        orc_transcript_absorb_u64(child, op_ids[3 * i + 2]);
    }
    orc_transcript_absorb_u64(child, shard_index);
}

/* ============================================================================
 * logUp GKR fraction tree (crates/zkie-core/src/common/logup_gkr.rs).
 * Round messages of all layers are concatenated: layer l has lg - l - 1
 * rounds of 4 evaluations; finals hold 7 evaluations per layer.
 * ========================================================================== */

/* build_terms (:19-28) over [eq, next_num, next_den, num_lo, num_hi, den_lo, den_hi] */
static void frac_terms(uint64_t c, uint64_t coeffs[5], uint32_t off[6], uint32_t idx[13])
{
    static const uint32_t o[6] = {0, 2, 5, 8, 10, 13};
    static const uint32_t ix[13] = {0, 1, 0, 3, 6, 0, 4, 5, 0, 2, 0, 5, 6};
    uint64_t neg = orc_from_i64(-1);
    coeffs[0] = 1;
    coeffs[1] = neg;
    coeffs[2] = neg;
    coeffs[3] = canon(c);
    coeffs[4] = orc_mul(neg, canon(c));
    memcpy(off, o, sizeof(o));
    memcpy(idx, ix, sizeof(ix));
}

/* Layer tables of one fraction-tree step (:43-58): mles = 7 x half, contiguous. */
static void frac_layer_tables(const uint64_t *num, const uint64_t *den, uint64_t half, const uint64_t *r,
                              uint32_t t, uint64_t *mles)
{
    uint64_t *eq = mles, *nn = mles + half, *nd = mles + 2 * half;
#pragma omp parallel for schedule(static)
    for (int64_t s = 0; s < (int64_t)half; s++) {
        nn[s] = orc_add(orc_mul(num[s], den[half + s]), orc_mul(num[half + s], den[s]));
        nd[s] = orc_mul(den[s], den[half + s]);
    }
    orc_eq_evals(r, t, eq);
    memcpy(mles + 3 * half, num, 8 * half);
    memcpy(mles + 4 * half, num + half, 8 * half);
    memcpy(mles + 5 * half, den, 8 * half);
    memcpy(mles + 6 * half, den + half, 8 * half);
}

/* prove_fractional_with_challenges (:29-69). */
void orc_fractional_prove(const uint64_t *num, const uint64_t *den, uint32_t lg, const uint64_t *full_r,
                          const uint64_t *cs, uint64_t *rounds, uint64_t *finals, uint64_t final_nd[2])
{
    uint64_t n = 1ULL << lg;
    uint64_t *cn = (uint64_t *)malloc(8 * n), *cd = (uint64_t *)malloc(8 * n);
    uint64_t *mles = (uint64_t *)malloc(8 * 7 * (n / 2 ? n / 2 : 1));
    for (uint64_t i = 0; i < n; i++) {
        cn[i] = canon(num[i]);
        cd[i] = canon(den[i]);
    }
    uint64_t roff = 0;
    for (uint32_t l = 0; l < lg; l++) {
        uint64_t half = n >> (l + 1);
        uint32_t t = lg - l - 1;
        uint64_t coeffs[5];
        uint32_t off[6], idx[13];
        frac_terms(cs[l], coeffs, off, idx);
        frac_layer_tables(cn, cd, half, full_r, t, mles);
        orc_virtual_prove(mles, 7, t, coeffs, off, idx, 5, full_r, rounds + roff, finals + 7ULL * l);
        roff += 4ULL * t;
        memcpy(cn, mles + half, 8 * half);
        memcpy(cd, mles + 2 * half, 8 * half);
    }
    final_nd[0] = cn[0];
    final_nd[1] = cd[0];
    free(cn);
    free(cd);
    free(mles);
}

/* verify_fractional (:83-134): every layer's sumcheck against final
 * evaluations recomputed from the tables, then final_num == claimed * final_den. */
int orc_fractional_verify(const uint64_t *num, const uint64_t *den, uint32_t lg, const uint64_t *full_r,
                          const uint64_t *cs, const uint64_t *rounds, uint64_t final_num, uint64_t final_den,
                          uint64_t claimed)
{
    uint64_t n = 1ULL << lg;
    uint64_t *cn = (uint64_t *)malloc(8 * n), *cd = (uint64_t *)malloc(8 * n);
    uint64_t *mles = (uint64_t *)malloc(8 * 7 * (n / 2 ? n / 2 : 1));
    for (uint64_t i = 0; i < n; i++) {
        cn[i] = canon(num[i]);
        cd[i] = canon(den[i]);
    }
    int ok = 1;
    uint64_t roff = 0;
    for (uint32_t l = 0; ok && l < lg; l++) {
        uint64_t half = n >> (l + 1);
        uint32_t t = lg - l - 1;
        uint64_t coeffs[5], fe[7];
        uint32_t off[6], idx[13];
        frac_terms(cs[l], coeffs, off, idx);
        frac_layer_tables(cn, cd, half, full_r, t, mles);
        for (int j = 0; j < 7; j++) fe[j] = orc_mle_eval(mles + (uint64_t)j * half, t, full_r);
        ok = orc_virtual_verify(rounds + roff, t, coeffs, off, idx, 5, 0, full_r, fe);
        roff += 4ULL * t;
        memcpy(cn, mles + half, 8 * half);
        memcpy(cd, mles + 2 * half, 8 * half);
    }
    free(cn);
    free(cd);
    free(mles);
    return ok && canon(final_num) == orc_mul(canon(claimed), canon(final_den));
}

/* verify_fractional_chain_core (:136-164): each layer's sumcheck against its
 * own stored final evaluations, and the folding link between layers. */
int orc_fractional_chain_core(uint32_t lg, const uint64_t *full_r, const uint64_t *cs, const uint64_t *rounds,
                              const uint64_t *finals)
{
    uint64_t roff = 0;
    for (uint32_t l = 0; l < lg; l++) {
        uint32_t t = lg - l - 1;
        uint64_t coeffs[5];
        uint32_t off[6], idx[13];
        frac_terms(cs[l], coeffs, off, idx);
        if (!orc_virtual_verify(rounds + roff, t, coeffs, off, idx, 5, 0, full_r, finals + 7ULL * l)) return 0;
        roff += 4ULL * t;
    }
    for (uint32_t l = 0; l + 1 < lg; l++) {
        const uint64_t *prev = finals + 7ULL * l, *curr = finals + 7ULL * (l + 1);
        uint32_t tp = lg - l - 1; /* prev.r = full_r[..tp] */
        uint64_t rk = canon(full_r[tp - 1]), om = orc_sub(1, rk);
        uint64_t fold_num = orc_add(orc_mul(om, curr[3]), orc_mul(rk, curr[4]));
        uint64_t fold_den = orc_add(orc_mul(om, curr[5]), orc_mul(rk, curr[6]));
        if (canon(prev[1]) != fold_num || canon(prev[2]) != fold_den) return 0;
    }
    return 1;
}

/* Lookup columns.  mode 0: build_lookup_num_den (:210-240); 1:
 * build_lookup_witness_num_den (:261-277); 2: the columns of
 * prove_lookup_witness_batch_columns (:340-370); 3: build_lookup_table_num_den
 * (:285-301) with caller multiplicities m.  Returns the column length, or 0 if
 * an index is out of the table (mode 0). */
static uint64_t next_pow2_u64(uint64_t x)
{
    uint64_t p = 1;
    while (p < x) p <<= 1;
    return p;
}

uint64_t orc_lookup_len(uint64_t n, uint64_t t, uint32_t mode)
{
    switch (mode) {
    case 0: return next_pow2_u64(n + t);
    case 1: return next_pow2_u64(n);
    case 2: { uint64_t l = next_pow2_u64(n); return l < 32 ? 32 : l; }
    case 3: return next_pow2_u64(t);
    default: return 0;
    }
}

uint64_t orc_lookup_num_den(const uint32_t *x, const uint64_t *y, uint64_t n, const uint64_t *table,
                            const uint64_t *m, uint64_t t, uint32_t mode, uint64_t alpha, uint64_t beta,
                            uint64_t *num, uint64_t *den)
{
    uint64_t total = orc_lookup_len(n, t, mode);
    if (mode == 3) {
        for (uint64_t j = 0; j < total; j++) {
            uint64_t tj = j < t ? canon(table[j]) : 0;
            num[j] = j < t ? canon(m[j]) : 0;
            den[j] = orc_add(orc_add(canon(alpha), canon(j)), orc_mul(canon(beta), tj));
        }
        return total;
    }
    for (uint64_t i = 0; i < total; i++) {
        num[i] = 0;
        den[i] = mode == 2 ? canon(alpha) : 1;
    }
    for (uint64_t i = 0; i < n; i++) {
        num[i] = 1;
        den[i] = orc_add(orc_add(canon(alpha), x[i]), orc_mul(canon(beta), canon(y[i])));
    }
    if (mode == 0) {
        uint64_t *cnt = (uint64_t *)calloc(t ? t : 1, 8);
        for (uint64_t i = 0; i < n; i++) {
            if (x[i] >= t) {
                free(cnt);
                return 0;
            }
            cnt[x[i]]++;
        }
        for (uint64_t j = 0; j < t; j++) {
            num[n + j] = orc_from_i64(-(int64_t)cnt[j]);
            den[n + j] = orc_add(orc_add(canon(alpha), canon(j)), orc_mul(canon(beta), canon(table[j])));
        }
        free(cnt);
    }
    return total;
}

/* ============================================================================
 * PoW grinding on DuplexChallenger<Goldilocks, Poseidon2-16, 16, 8>
 * (pcs/whir.rs:42; grind called at p3-whir src/pcs/prover/mod.rs:240-245).
 * p3-challenger 0.7.0 is not vendored; restated from its published duplex
 * sponge: observe(v) clears the outputs and buffers v (a full rate of 8
 * inputs duplexes at once); sample() duplexes when inputs are buffered or no
 * output is left and pops the last output; a duplexing overwrites lanes
 * [0, len) with the buffered inputs, permutes, and keeps lanes [0, 8) as
 * outputs; sample_bits(b) = canonical(sample()) & (2^b - 1);
 * check_witness(b, w) = observe(w); sample_bits(b) == 0.
 * ========================================================================== */
int orc_check_witness(const orc_p2_consts *c, const uint64_t sponge[16], const uint64_t *input, uint32_t len,
                      uint32_t bits, uint64_t w)
{
    uint64_t st[16];
    for (int i = 0; i < 16; i++) st[i] = canon(sponge[i]);
    for (uint32_t i = 0; i < len; i++) st[i] = canon(input[i]);
    st[len] = canon(w);
    orc_p2_permute(c, st);
    return (canon(st[7]) & ((1ULL << bits) - 1)) == 0;
}

/* The smallest valid witness in [start, start + limit), or UINT64_MAX. */
uint64_t orc_grind(const orc_p2_consts *c, const uint64_t sponge[16], const uint64_t *input, uint32_t len,
                   uint32_t bits, uint64_t start, uint64_t limit)
{
    for (uint64_t w = start; w - start < limit && w < ORC_P; w++)
        if (orc_check_witness(c, sponge, input, len, bits, w)) return w;
    return ~0ULL;
}

/* Thread count of the OpenMP loops above (a launcher may have set
 * OMP_NUM_THREADS=1 for its ranks; the CPU baseline wants every core). */
void orc_set_threads(int n)
{
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

/* ============================================================================
 * Elementwise field operations and row sums for the op-layer restatement
 * (the Goldilocks +, -, * of crates/zkie-ops/src/compose.rs's forward and
 * prove arms, over whole tensors).
 * ========================================================================== */
void orc_vec_add(const uint64_t *a, const uint64_t *b, uint64_t n, uint64_t *out)
{
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; i++) out[i] = orc_add(canon(a[i]), canon(b[i]));
}

void orc_vec_sub(const uint64_t *a, const uint64_t *b, uint64_t n, uint64_t *out)
{
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; i++) out[i] = orc_sub(canon(a[i]), canon(b[i]));
}

void orc_vec_mul(const uint64_t *a, const uint64_t *b, uint64_t n, uint64_t *out)
{
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < (int64_t)n; i++) out[i] = orc_mul(a[i], b[i]);
}

/* out[r] = sum_{j < ncols} x[r * d + j] over the field, r < m */
void orc_row_sums(const uint64_t *x, uint64_t m, uint64_t d, uint64_t ncols, uint64_t *out)
{
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < (int64_t)m; r++) {
        uint64_t s = 0;
        for (uint64_t j = 0; j < ncols; j++) s = orc_add(s, canon(x[r * d + j]));
        out[r] = s;
    }
}
