// dft_reg.cuh -- in-register 2^L-point DFTs over Goldilocks (L <= 4), the
// radix steps of the NTT passes.  Every twiddle inside such a DFT is a power
// of W_16 or smaller, i.e. a power of two in Goldilocks
// (W_{2^s} = 2^(39 * 2^(6-s) mod 192)), so the butterflies multiply by shifts
// (GlPow2).  Host and device compile the same code, so the host can check it.
#pragma once
#include <utility>

#include "gl64.cuh"

namespace zk {

template <int L>
ZK_HD constexpr int brev_c(int i) {
    int r = 0;
    for (int b = 0; b < L; b++)
        if ((i >> b) & 1) r |= 1 << (L - 1 - b);
    return r;
}

// Butterfly (a, b) <- (a + W b, a - W b) with W = 2^K.
template <int K>
ZK_HD void bfly_pow2(uint64_t& a, uint64_t& b) {
    const uint64_t t = GlPow2<K>::mag(b), u = a;
    if (GlPow2<K>::neg) {
        a = gl_sub(u, t);
        b = gl_add(u, t);
    } else {
        a = gl_add(u, t);
        b = gl_sub(u, t);
    }
}

// Butterfly I of DIT stage S (1-based) of a 2^L-point transform on
// bit-reversed input: rows a, a + 2^(S-1), twiddle W_{2^S}^j.
template <int S, int I>
ZK_HD void dit_bfly(uint64_t* y) {
    constexpr int h = 1 << (S - 1), j = I % h, a = (I / h) * 2 * h + j;
    constexpr int K = ((39 << (6 - S)) * j) % 192;
    bfly_pow2<K>(y[a], y[a + h]);
}
template <int S, int... I>
ZK_HD void dit_stage(uint64_t* y, std::integer_sequence<int, I...>) {
    (dit_bfly<S, I>(y), ...);
}
template <int L, int... S>
ZK_HD void dit_stages(uint64_t* y, std::integer_sequence<int, S...>) {
    (dit_stage<S + 1>(y, std::make_integer_sequence<int, (1 << (L - 1))>{}), ...);
}
// x[e] <- sum_d x[d] W_{2^L}^(d e), natural order in and out.
template <int L>
ZK_HD void dft_reg(uint64_t* x) {
    constexpr int R = 1 << L;
    uint64_t y[R];
#pragma unroll
    for (int i = 0; i < R; i++) y[i] = x[brev_c<L>(i)];
    dit_stages<L>(y, std::make_integer_sequence<int, L>{});
#pragma unroll
    for (int i = 0; i < R; i++) x[i] = y[i];
}

template <int L, int... S>
ZK_HD void dit_stages_from2(uint64_t* y, std::integer_sequence<int, S...>) {
    (dit_stage<S + 2>(y, std::make_integer_sequence<int, (1 << (L - 1))>{}), ...);
}
// dft_reg for inputs whose upper half is zero: after the bit reversal those
// sit at the odd positions, so the first DIT stage (twiddle 1) is a copy.
template <int L>
ZK_HD void dft_reg_half(uint64_t* x) {
    constexpr int R = 1 << L;
    uint64_t y[R];
#pragma unroll
    for (int i = 0; i < R; i += 2) y[i] = y[i + 1] = x[brev_c<L>(i)];
    dit_stages_from2<L>(y, std::make_integer_sequence<int, L - 1>{});
#pragma unroll
    for (int i = 0; i < R; i++) x[i] = y[i];
}

// ---- lazy butterflies -----------------------------------------------------------------
// The same DIT network on 96-bit accumulators: a butterfly adds and subtracts
// without reducing, and only a value about to be multiplied by a shift
// twiddle (and only where the shifted value would not fit 128 bits), and
// each output, is reduced.  Values entering stage S are below
// B_S 2^64 with B_1 = 1 and B_(S+1) = 2 B_S + 1 (31 after four stages):
// a difference u - t is formed as u + c p - t with c p > t, namely
// c = B + 1 for an unreduced t < B 2^64 and c = 2 for a reduced t < 2^64.

// ceil(log2(x)) for x >= 1
ZK_HD constexpr int clog2_c(int x) {
    int r = 0;
    while ((1 << r) < x) r++;
    return r;
}

// c p as an accumulator, 1 <= c <= 2^31: (c - 1) 2^64 + (2^64 - c (2^32 - 1))
template <int C>
ZK_HD Acc acc_pmul() {
    return Acc{(uint64_t)0 - (uint64_t)C * GL_EPS, (uint32_t)(C - 1)};
}

template <int K, int B>
ZK_HD void bfly_lazy(Acc& a, Acc& b) {
    const Acc u = a;
    Acc s, d;
    if constexpr (K % 96 == 0) {
        s = acc_add(u, b);                              // below 2B
        d = acc_sub(acc_add(u, acc_pmul<B + 1>()), b);  // below 2B + 1
    } else {
        constexpr int Kp = K % 96;
        uint64_t t;
        if constexpr (Kp < 64 && Kp + clog2_c(B) <= 64) {
            // b 2^Kp as a 128-bit value: its high word, below B 2^Kp, fits
            t = gl_reduce128(b.lo << Kp, (b.lo >> (64 - Kp)) | ((uint64_t)b.hi << Kp));
        } else {
            t = GlPow2<K>::mag(acc_reduce(b));
        }
        s = acc_add(u, t);                                   // below B + 1
        d = acc_sub(acc_add(u, acc_pmul<2>()), Acc{t, 0u});  // below B + 2
    }
    if (GlPow2<K>::neg) {
        a = d;
        b = s;
    } else {
        a = s;
        b = d;
    }
}
template <int S, int B, int I>
ZK_HD void dit_bfly_lazy(Acc* y) {
    constexpr int h = 1 << (S - 1), j = I % h, a = (I / h) * 2 * h + j;
    constexpr int K = ((39 << (6 - S)) * j) % 192;
    bfly_lazy<K, B>(y[a], y[a + h]);
}
template <int S, int B, int... I>
ZK_HD void dit_stage_lazy(Acc* y, std::integer_sequence<int, I...>) {
    (dit_bfly_lazy<S, B, I>(y), ...);
}
template <int S, int L, int B>
ZK_HD void dit_stages_lazy(Acc* y) {
    if constexpr (S <= L) {
        dit_stage_lazy<S, B>(y, std::make_integer_sequence<int, (1 << (L - 1))>{});
        dit_stages_lazy<S + 1, L, 2 * B + 1>(y);
    }
}
// dft_reg on accumulators
template <int L>
ZK_HD void dft_reg_lazy(uint64_t* x) {
    constexpr int R = 1 << L;
    Acc y[R];
#pragma unroll
    for (int i = 0; i < R; i++) y[i] = acc_of(x[brev_c<L>(i)]);
    dit_stages_lazy<1, L, 1>(y);
#pragma unroll
    for (int i = 0; i < R; i++) x[i] = acc_reduce(y[i]);
}
// dft_reg_lazy for inputs e >= R / 2^Z all zero (1 <= Z <= L): after the bit
// reversal the nonzero inputs sit at the positions whose low Z bits are
// zero, and the first Z DIT stages spread each over its block of 2^Z (the
// DFT of a delta is constant), so they are copies.
template <int L, int Z>
ZK_HD void dft_reg_zero_lazy(uint64_t* x) {
    constexpr int R = 1 << L, S = 1 << Z;
    Acc y[R];
#pragma unroll
    for (int i = 0; i < R; i += S) {
        const Acc v = acc_of(x[brev_c<L>(i)]);
#pragma unroll
        for (int k = 0; k < S; k++) y[i + k] = v;
    }
    dit_stages_lazy<Z + 1, L, 1>(y);
#pragma unroll
    for (int i = 0; i < R; i++) x[i] = acc_reduce(y[i]);
}
// the upper half zero
template <int L>
ZK_HD void dft_reg_half_lazy(uint64_t* x) {
    dft_reg_zero_lazy<L, 1>(x);
}

}  // namespace zk
