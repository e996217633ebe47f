/*
 * packed_field.h -- Goldilocks arithmetic on PW lanes at once, and on it the
 * Poseidon2-16 permutation of PW independent states (one lane per state) and
 * the radix-2 DFT of PW adjacent columns (one lane per column).  TEST
 * INFRASTRUCTURE: part of the CPU oracle and of the CPU baseline it times.
 *
 * zkie_oracle.c includes this file once per instruction set, with
 *   PW      lanes per vector (8 for AVX-512, 4 for AVX2),
 *   PTGT    the function attribute that enables that instruction set,
 *   PMUL32  the lane product of the low 32 bits of two vectors (vpmuludq),
 *   PSUF    the suffix of every name defined here,
 * and optionally PADD_IF_LT(x, a, b, c) = x + (a < b ? c : 0) and
 * PSUB_IF_LT / PSUB_IF_GE (x - (a < b ? c : 0), x - (a >= b ? c : 0)) per
 * lane, unsigned, as mask-register forms (AVX-512); the default forms use
 * the all-ones lane masks of vector comparisons.
 * The permutation is orc_p2_permute's and the DFT dft_column's, lane by
 * lane: same steps, same constants, same canonical results (tests hold each
 * bit-identical to the scalar form).  They exist because zkIE's own CPU path
 * runs p3's packed field (PackedGoldilocksAVX2 / AVX512): MerkleTreeMmcs
 * hashes with the packed Poseidon2 and Radix2DFTSmallBatch transforms
 * packed columns, so a scalar-only baseline would understate the
 * reference's CPU speed.
 *
 * Field arithmetic on lanes (all values canonical, < p):
 *   a + b   one 64-bit add, the carry out folded back as 2^64 = 2^32 - 1,
 *   a * b   four 32x32 -> 64 products (the schoolbook 128-bit product), then
 *           the reduction x = lo + 2^64 hi_lo + 2^96 hi_hi
 *                       = lo + (2^32 - 1) hi_lo - hi_hi (mod p).
 */

#define PCAT_(a, b) a##b
#define PCAT(a, b) PCAT_(a, b)
#define PN(name) PCAT(name, PSUF)

typedef uint64_t PN(pv) __attribute__((vector_size(8 * PW)));
#define PV PN(pv)
#define PINL static inline __attribute__((always_inline)) PTGT

#ifndef PADD_IF_LT
#define PADD_IF_LT(x, a, b, c) ((x) + ((c) & (PV)((a) < (b))))
#define PSUB_IF_LT(x, a, b, c) ((x) - ((c) & (PV)((a) < (b))))
#define PSUB_IF_GE(x, a, b, c) ((x) - ((c) & (PV)((a) >= (b))))
#define PCOND_DEFAULT 1
#endif

PINL PV PN(bc)(uint64_t x) { return (PV){0} + x; }

PINL PV PN(canon)(PV x) { return PSUB_IF_GE(x, x, PN(bc)(ORC_P), PN(bc)(ORC_P)); }

/* a + b: a carry out of 64 bits is 2^64 = 2^32 - 1 (the sum is then below
 * p already), else one conditional subtraction of p */
PINL PV PN(add)(PV a, PV b)
{
    PV s = a + b;
    s = PADD_IF_LT(s, s, a, PN(bc)(EPS));
    return PSUB_IF_GE(s, s, PN(bc)(ORC_P), PN(bc)(ORC_P));
}

PINL PV PN(sub)(PV a, PV b) { return PADD_IF_LT(a - b, a, b, PN(bc)(ORC_P)); }

/* (hi, lo) mod p for any 128-bit value: reduce128 on lanes */
PINL PV PN(reduce)(PV lo, PV hi)
{
    const PV hh = hi >> 32, hl = hi & PN(bc)(0xFFFFFFFFULL);
    PV t0 = lo - hh;
    t0 = PSUB_IF_LT(t0, lo, hh, PN(bc)(EPS));
    const PV t1 = (hl << 32) - hl;
    PV t2 = t0 + t1;
    t2 = PADD_IF_LT(t2, t2, t1, PN(bc)(EPS));
    return PSUB_IF_GE(t2, t2, PN(bc)(ORC_P), PN(bc)(ORC_P));
}

/* the 128-bit product a * b + c (c < 2^64), as (lo, hi); never overflows
 * for canonical a, b since (p - 1)^2 + 2^64 < 2^128 */
PINL void PN(mul_wide)(PV a, PV b, PV c, PV *lo_out, PV *hi_out)
{
    const PV ah = a >> 32, bh = b >> 32;
    const PV ll = PMUL32(a, b), lh = PMUL32(a, bh), hl = PMUL32(ah, b), hh = PMUL32(ah, bh);
    const PV mid = lh + hl;
    PV hi = hh + (mid >> 32);
    hi = PADD_IF_LT(hi, mid, lh, PN(bc)(1ULL << 32));    /* carry of mid into bit 96 */
    const PV lo = ll + (mid << 32);
    hi = PADD_IF_LT(hi, lo, ll, PN(bc)(1));
    const PV lo2 = lo + c;
    hi = PADD_IF_LT(hi, lo2, lo, PN(bc)(1));
    *lo_out = lo2;
    *hi_out = hi;
}

PINL PV PN(mul)(PV a, PV b)
{
    PV lo, hi;
    PN(mul_wide)(a, b, (PV){0}, &lo, &hi);
    return PN(reduce)(lo, hi);
}

PINL PV PN(sbox7)(PV x)
{
    const PV x2 = PN(mul)(x, x), x3 = PN(mul)(x2, x), x4 = PN(mul)(x2, x2);
    return PN(mul)(x3, x4);
}

PINL PV PN(dbl)(PV x) { return PN(add)(x, x); }

/* x * 2^-k for 1 <= k <= 32: x = q 2^k + r gives x 2^-k = q + r 2^-k, and
 * 2^-k = -2^(96-k) (2^96 = -1 mod p), so x 2^-k = q - r 2^(32-k) 2^64
 * = q - r 2^(32-k) (2^32 - 1); that product is below p, so one modular
 * subtraction finishes it */
PINL PV PN(div2k)(PV x, int k)
{
    const PV hl = (x & PN(bc)((1ULL << k) - 1)) << (32 - k);
    return PN(sub)(x >> k, (hl << 32) - hl);
}

/* [2 3 1 1; 1 2 3 1; 1 1 2 3; 3 1 1 2] on one 4-lane block, canonical adds */
PINL void PN(mat4)(PV *x)
{
    const PV t01 = PN(add)(x[0], x[1]), t23 = PN(add)(x[2], x[3]);
    const PV t0123 = PN(add)(t01, t23);
    const PV t01123 = PN(add)(t0123, x[1]), t01233 = PN(add)(t0123, x[3]);
    const PV y0 = PN(add)(t01123, t01);
    const PV y1 = PN(add)(t01123, PN(add)(x[2], x[2]));
    const PV y2 = PN(add)(t01233, t23);
    const PV y3 = PN(add)(t01233, PN(add)(x[0], x[0]));
    x[0] = y0;
    x[1] = y1;
    x[2] = y2;
    x[3] = y3;
}

PINL void PN(mds_light16)(PV *st)
{
    for (int j = 0; j < 16; j += 4) PN(mat4)(st + j);
    PV sums[4];
    for (int k = 0; k < 4; k++) sums[k] = PN(add)(PN(add)(st[k], st[4 + k]), PN(add)(st[8 + k], st[12 + k]));
    for (int i = 0; i < 16; i++) st[i] = PN(add)(st[i], sums[i & 3]);
}

/* the permutation on PW states held transposed: st[i] lane j is element i
 * of state j; inputs canonical.  The internal layer's diagonal is the fixed
 * V = [-2, 1, 2, 1/2, 3, 4, -1/2, -3, -4, 1/2^3, 1/2^4, 1/2^5, -1/2^3,
 * -1/2^4, -1/2^5, diag[15]] of orc_p2_permute: its first fifteen entries are
 * applied as adds and shifts, diag[15] as a general product. */
PTGT static void PN(p2_permute)(const orc_p2_consts *c, const uint64_t *diag, PV *st)
{
    PN(mds_light16)(st);
    for (int r = 0; r < 4; r++) {
        for (int i = 0; i < 16; i++) st[i] = PN(sbox7)(PN(add)(st[i], PN(bc)(c->ext_init[r][i])));
        PN(mds_light16)(st);
    }
    for (int r = 0; r < 22; r++) {
        st[0] = PN(sbox7)(PN(add)(st[0], PN(bc)(c->internal[r])));
        /* the state's sum in 128 bits (16 canonical values < 2^68), reduced once */
        PV lo = st[0], hi = (PV){0};
        for (int i = 1; i < 16; i++) {
            const PV s = lo + st[i];
            hi = PADD_IF_LT(hi, s, lo, PN(bc)(1));
            lo = s;
        }
        const PV sum = PN(reduce)(lo, hi);
        /* st_i = sum + V_i st_i */
        st[0] = PN(sub)(sum, PN(dbl)(st[0]));
        st[1] = PN(add)(sum, st[1]);
        st[2] = PN(add)(sum, PN(dbl)(st[2]));
        st[3] = PN(add)(sum, PN(div2k)(st[3], 1));
        st[4] = PN(add)(sum, PN(add)(PN(dbl)(st[4]), st[4]));
        st[5] = PN(add)(sum, PN(dbl)(PN(dbl)(st[5])));
        st[6] = PN(sub)(sum, PN(div2k)(st[6], 1));
        st[7] = PN(sub)(sum, PN(add)(PN(dbl)(st[7]), st[7]));
        st[8] = PN(sub)(sum, PN(dbl)(PN(dbl)(st[8])));
        st[9] = PN(add)(sum, PN(div2k)(st[9], 3));
        st[10] = PN(add)(sum, PN(div2k)(st[10], 4));
        st[11] = PN(add)(sum, PN(div2k)(st[11], 5));
        st[12] = PN(sub)(sum, PN(div2k)(st[12], 3));
        st[13] = PN(sub)(sum, PN(div2k)(st[13], 4));
        st[14] = PN(sub)(sum, PN(div2k)(st[14], 5));
        PV plo, phi;
        PN(mul_wide)(PN(bc)(diag[15]), st[15], sum, &plo, &phi);
        st[15] = PN(reduce)(plo, phi);
    }
    for (int r = 0; r < 4; r++) {
        for (int i = 0; i < 16; i++) st[i] = PN(sbox7)(PN(add)(st[i], PN(bc)(c->ext_final[r][i])));
        PN(mds_light16)(st);
    }
}

/* orc_p2_hash_row on PW consecutive rows of a row-major h x w matrix: the
 * sponge overwrites the rate with each block of 8 (a partial tail block
 * keeps the old state beyond it), digest = state[0..8] */
PTGT static void PN(p2_hash_rows)(const orc_p2_consts *c, const uint64_t *diag, const uint64_t *rows,
                                   uint64_t w, uint64_t *digests)
{
    PV st[16];
    for (int i = 0; i < 16; i++) st[i] = (PV){0};
    const uint64_t nb = w >> 3, rem = w & 7;
    uint64_t blk[8][PW] __attribute__((aligned(64)));
    for (uint64_t b = 0; b <= nb; b++) {
        const uint64_t cnt = b < nb ? 8 : rem;
        if (cnt == 0) break;
        for (int j = 0; j < PW; j++) {
            const uint64_t *src = rows + (uint64_t)j * w + 8 * b;
            for (uint64_t i = 0; i < cnt; i++) blk[i][j] = src[i];
        }
        for (uint64_t i = 0; i < cnt; i++) {
            PV v;
            memcpy(&v, blk[i], sizeof v);
            st[i] = PN(canon)(v);
        }
        PN(p2_permute)(c, diag, st);
    }
    uint64_t out[8][PW] __attribute__((aligned(64)));
    for (int i = 0; i < 8; i++) memcpy(out[i], &st[i], sizeof st[i]);
    for (int j = 0; j < PW; j++)
        for (int i = 0; i < 8; i++) digests[8 * j + i] = out[i][j];
}

/* PW compressions of consecutive pairs: next[k] = compress(prev[2k], prev[2k+1]) */
PTGT static void PN(p2_compress_pairs)(const orc_p2_consts *c, const uint64_t *diag, const uint64_t *prev,
                                        uint64_t *next)
{
    uint64_t blk[16][PW] __attribute__((aligned(64)));
    for (int j = 0; j < PW; j++)
        for (int i = 0; i < 16; i++) blk[i][j] = prev[16 * j + i];
    PV st[16];
    for (int i = 0; i < 16; i++) {
        memcpy(&st[i], blk[i], sizeof st[i]);
        st[i] = PN(canon)(st[i]);
    }
    PN(p2_permute)(c, diag, st);
    uint64_t out[8][PW] __attribute__((aligned(64)));
    for (int i = 0; i < 8; i++) memcpy(out[i], &st[i], sizeof st[i]);
    for (int j = 0; j < PW; j++)
        for (int i = 0; i < 8; i++) next[8 * j + i] = out[i][j];
}

/* dft_column on PW adjacent columns at once: v[i] holds row i of the block
 * (canonical); radix-2 decimation in time, natural order in and out */
PTGT static void PN(dft_block)(PV *v, uint32_t lg, const uint64_t *tw_all, const uint32_t *rev)
{
    const uint64_t n = 1ULL << lg;
    for (uint64_t i = 0; i < n; i++) {
        const uint64_t j = rev[i];
        if (j > i) {
            const PV t = v[i];
            v[i] = v[j];
            v[j] = t;
        }
    }
    for (uint32_t s = 1; s <= lg; s++) {
        const uint64_t half = 1ULL << (s - 1);
        const uint64_t *tw = tw_all + half - 1;
        for (uint64_t base = 0; base < n; base += 2 * half)
            for (uint64_t j = 0; j < half; j++) {
                const PV u = v[base + j];
                const PV x = PN(mul)(v[base + j + half], PN(bc)(tw[j]));
                v[base + j] = PN(add)(u, x);
                v[base + j + half] = PN(sub)(u, x);
            }
    }
}

/* columns [c0, c0 + PW) of a row-major h x w matrix through dft_block, in
 * place; buf holds h vectors */
PTGT static void PN(dft_columns)(uint64_t *mat, uint64_t w, uint64_t c0, uint32_t lg, const uint64_t *tw_all,
                                  const uint32_t *rev, PV *buf)
{
    const uint64_t h = 1ULL << lg;
    for (uint64_t i = 0; i < h; i++) {
        PV x;
        memcpy(&x, mat + i * w + c0, sizeof x);
        buf[i] = PN(canon)(x);
    }
    PN(dft_block)(buf, lg, tw_all, rev);
    for (uint64_t i = 0; i < h; i++) memcpy(mat + i * w + c0, &buf[i], sizeof buf[i]);
}

#ifdef PCOND_DEFAULT
#undef PADD_IF_LT
#undef PSUB_IF_LT
#undef PSUB_IF_GE
#undef PCOND_DEFAULT
#endif
#undef PV
#undef PINL
#undef PN
#undef PCAT
#undef PCAT_
