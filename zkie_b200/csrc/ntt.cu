// ntt.cu -- Goldilocks DFT / zero-padded LDE of the columns of a row-major
// matrix, and the reference-facing zkie_ntt_forward_goldilocks
// (crates/zkie-core/cuda/goldilocks_ntt.cu:105-137).
//
// Contract (goldilocks_ntt.cu:1-23): for each column, out[i] = sum_j x[j] w^(ij)
// with w = TWO_ADIC_GENERATORS[lg h], natural order in and out, canonical
// output.
//
// Design: four-step decomposition of a 2^lg transform into 1 to 3 passes
// (2^lg = N1 * N2 [* N3], every factor <= 2^10).  A pass loads a tile of R
// consecutive "lanes" x C columns x M = 2^m rows of the strided sub-sequence
// into shared memory (one coalesced chunk of R*C u64 per row), runs m radix-2
// DIT stages there, multiplies the inter-pass twiddle and stores the tile with
// the next pass's layout.  Zero padding of an LDE is folded into the first
// pass (rows >= L read as zero, never fetched), so the HBM traffic is one read
// of the L input rows, one write + read of an intermediate per extra pass and
// one write of the H output rows -- instead of the reference's lg h + 2 full
// passes with one launch per radix-2 stage.
#include <mutex>
#include <utility>

#include "../../include/zkie_goldilocks_cuda.h"
#include "../../include/zkie2.h"
#include "common.cuh"
#include "dft_reg.cuh"
#include "gl64.cuh"
#include "internal.h"

namespace zk {

// Powers of the order-2^32 generator w32: lo[i] = w32^i, hi[i] = w32^(i*2^16).
__device__ uint64_t g_tw_lo[1 << 16];
__device__ uint64_t g_tw_hi[1 << 16];

namespace {

std::mutex g_tw_mu;
bool g_tw_ready[kMaxDevices];

int ensure_twiddles() {
    int d = current_device();
    if (d < 0 || d >= kMaxDevices) return (int)cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> g(g_tw_mu);
    if (g_tw_ready[d]) return 0;
    std::vector<uint64_t> lo(1 << 16), hi(1 << 16);
    uint64_t w32 = two_adic_generator_host(32);
    uint64_t w16 = gl_pow_host(w32, 1ull << 16);
    lo[0] = 1;
    hi[0] = 1;
    for (int i = 1; i < (1 << 16); i++) {
        lo[i] = gl_mul_host(lo[i - 1], w32);
        hi[i] = gl_mul_host(hi[i - 1], w16);
    }
    ZK_TRY(cudaMemcpyToSymbol(g_tw_lo, lo.data(), 8 * lo.size()));
    ZK_TRY(cudaMemcpyToSymbol(g_tw_hi, hi.data(), 8 * hi.size()));
    g_tw_ready[d] = true;
    return 0;
}

struct PassDesc {
    const uint64_t* in;
    uint64_t* out;
    uint64_t w;           // columns transformed
    uint64_t ld;          // row stride of in and out, in elements (>= w)
    uint64_t rows_valid;  // input rows >= rows_valid are zero (LDE padding)
    uint64_t F;           // lanes
    uint64_t fin, sin, jin;
    uint64_t fout, sout, kout;
    uint32_t m;       // log2 of the sub-DFT size M
    uint32_t logC;    // log2 of the tile columns C
    uint32_t logR;    // log2 of the tile lanes R (C * R = tile width)
    uint32_t tw_log;  // 0: no inter-pass twiddle; else multiply by W_{2^tw_log}^(f*k)
    uint32_t canon;   // canonicalize the output
    uint32_t cgroups;  // k_ntt_pass2: column groups of 2^logC columns (fastest-varying block index)
    uint32_t half_zero;  // k_ntt_pass2: inputs e >= 8 of every first-step group are padding rows
    // Twiddle source of the reference-facing entry: the caller's top-stage
    // table tab[e] = W_{2^tab_log}^e, e < 2^(tab_log-1).
    const uint64_t* tab;
    uint32_t tab_log;
};

template <bool kCallerTab>
__device__ __forceinline__ uint64_t root_pow(const PassDesc& d, uint32_t t, uint64_t e) {
    // W_{2^t}^e
    if (kCallerTab) {
        const uint64_t mask = (1ull << d.tab_log) - 1;
        const uint64_t x = (e << (d.tab_log - t)) & mask;
        const uint64_t half = 1ull << (d.tab_log - 1);
        return x < half ? __ldg(d.tab + x) : gl_neg(__ldg(d.tab + (x - half)));
    } else {
        const uint32_t E = (uint32_t)((e << (32 - t)) & 0xFFFFFFFFull);
        return gl_mul(__ldg(g_tw_lo + (E & 0xFFFF)), __ldg(g_tw_hi + (E >> 16)));
    }
}

__device__ __forceinline__ uint32_t brev_m(uint32_t j, uint32_t m) { return m ? (__brev(j) >> (32 - m)) : 0; }

constexpr int kNttThreads = 256;

// IdxT: uint32_t when every element offset of the matrices fits in 32 bits
// (fewer integer instructions for the address arithmetic), else uint64_t.
template <bool kCallerTab, typename IdxT>
__global__ void __launch_bounds__(kNttThreads) k_ntt_pass(PassDesc d) {
    extern __shared__ uint64_t sm[];
    const uint32_t m = d.m, M = 1u << m;
    const uint32_t logC = d.logC, logR = d.logR, logLW = logC + logR;
    const uint32_t C = 1u << logC, LW = 1u << logLW;
    uint64_t* data = sm;                         // [M][LW], row-major
    uint64_t* tws = sm + ((size_t)M << logLW);   // [M/2] powers of W_M

    const uint64_t tiles_f = d.F >> logR;
    const uint64_t s_idx = blockIdx.x / tiles_f;
    const uint64_t f0 = (blockIdx.x % tiles_f) << logR;
    const uint64_t c0 = (uint64_t)blockIdx.y << logC;
    const uint32_t ccur = (d.w - c0) < C ? (uint32_t)(d.w - c0) : C;
    const uint32_t tid = threadIdx.x;

    for (uint32_t i = tid; i < M / 2; i += kNttThreads) tws[i] = root_pow<kCallerTab>(d, m, i);

    // ---- load: element (j, lane fl, column c) of the tile is input row
    // (f0 + fl)*fin + s*sin + j*jin; stored at the bit-reversed position of j.
    const uint32_t total = M << logLW;
    // Each thread keeps one column c of the tile and walks the (lane, j) pairs.
    const uint32_t c = tid & (C - 1);
    const bool cok = c < ccur;
    const uint32_t nq = total >> logC, qstep = kNttThreads >> logC;
    const IdxT w = (IdxT)d.ld;  // row stride
    {
        const IdxT row0 = (IdxT)(f0 * d.fin + s_idx * d.sin);
        const IdxT fin = (IdxT)d.fin, jin = (IdxT)d.jin;
        const IdxT rows_valid = (IdxT)(d.rows_valid < (uint64_t)(IdxT)~(IdxT)0 ? d.rows_valid : (uint64_t)(IdxT)~(IdxT)0);
        const uint64_t* gin = d.in + c0 + c;
        const bool lane_major = d.jin != 1;  // consecutive lanes are consecutive rows
        for (uint32_t q = tid >> logC; q < nq; q += qstep) {
            uint32_t fl, j;
            if (lane_major) {
                fl = q & ((1u << logR) - 1);
                j = q >> logR;
            } else {
                j = q & (M - 1);
                fl = q >> m;
            }
            const IdxT row = row0 + (IdxT)fl * fin + (IdxT)j * jin;
            uint64_t v = 0;
            if (cok && row < rows_valid) v = __ldg(gin + row * w);
            data[(brev_m(j, m) << logLW) | (fl << logC) | c] = v;
        }
    }
    __syncthreads();

    // ---- DIT stages on bit-reversed input -> natural order.  Stage s pairs
    // rows at distance 2^(s-1) with twiddle W_{2^s}^(i mod 2^(s-1)).  Stages
    // run two at a time as radix-4 groups in registers (one shared-memory
    // round trip and one barrier per two stages); an odd first stage, whose
    // twiddle is 1, runs alone.
    uint32_t s = 1;
    if (m & 1) {
        const uint32_t nb = (M / 2) << logLW;
        for (uint32_t b = tid; b < nb; b += kNttThreads) {
            uint64_t* p = data + (((b >> logLW) << 1) << logLW) + (b & (LW - 1));
            const uint64_t u = p[0], v = p[LW];
            p[0] = gl_add(u, v);
            p[LW] = gl_sub(u, v);
        }
        s = 2;
        __syncthreads();
    }
    for (; s < m; s += 2) {
        const uint32_t hb = s - 1;
        const uint32_t h = 1u << hb;
        const uint32_t hs = h << logLW;  // distance between the group's rows, in elements
        const uint32_t nq = (M / 4) << logLW;
        for (uint32_t g = tid; g < nq; g += kNttThreads) {
            const uint32_t gg = g >> logLW;
            const uint32_t j0 = gg & (h - 1);
            const uint32_t i0 = ((gg >> hb) << (s + 1)) | j0;
            uint64_t* p = data + (i0 << logLW) + (g & (LW - 1));
            const uint64_t e0 = p[0], e1 = p[hs], e2 = p[2 * hs], e3 = p[3 * hs];
            const uint64_t w1 = tws[j0 << (m - s)];             // W_{2^s}^j0
            const uint64_t w2 = tws[j0 << (m - s - 1)];         // W_{2^(s+1)}^j0
            const uint64_t w3 = tws[(j0 + h) << (m - s - 1)];   // W_{2^(s+1)}^(j0 + h)
            uint64_t t = gl_mul(e1, w1);
            const uint64_t a0 = gl_add(e0, t), a1 = gl_sub(e0, t);
            t = gl_mul(e3, w1);
            const uint64_t a2 = gl_add(e2, t), a3 = gl_sub(e2, t);
            t = gl_mul(a2, w2);
            p[0] = gl_add(a0, t);
            p[2 * hs] = gl_sub(a0, t);
            t = gl_mul(a3, w3);
            p[hs] = gl_add(a1, t);
            p[3 * hs] = gl_sub(a1, t);
        }
        __syncthreads();
    }

    // ---- store: output k of lane fl goes to row (f0 + fl)*fout + s*sout + k*kout,
    // after the inter-pass twiddle W_{2^tw_log}^((f0 + fl) * k).
    {
        const IdxT row0 = (IdxT)(f0 * d.fout + s_idx * d.sout);
        const IdxT fout = (IdxT)d.fout, kout = (IdxT)d.kout;
        uint64_t* gout = d.out + c0 + c;
        const uint64_t emask = (1ull << d.tw_log) - 1;
        const bool lane_major = d.fout == 1;
        for (uint32_t q = tid >> logC; q < nq; q += qstep) {
            uint32_t fl, k;
            if (lane_major) {
                fl = q & ((1u << logR) - 1);
                k = q >> logR;
            } else {
                k = q & (M - 1);
                fl = q >> m;
            }
            uint64_t v = data[(k << logLW) | (fl << logC) | c];
            if (d.tw_log) v = gl_mul(v, root_pow<kCallerTab>(d, d.tw_log, ((f0 + fl) * k) & emask));
            if (d.canon) v = gl_canon(v);
            const IdxT row = row0 + (IdxT)fl * fout + (IdxT)k * kout;
            if (cok) gout[row * w] = v;
        }
    }
}

// ---- register-radix pass ------------------------------------------------------------
// The same pass contract (PassDesc) as k_ntt_pass, computed as a mixed-radix
// decimation in frequency over radix-2^L steps (L <= 4) held in registers.
// Step i takes each group of R_i elements at stride M_i/R_i inside its
// current sub-problem of M_i elements, does the R_i-point DFT in registers,
// multiplies output e by W_{M_i}^(j' e) (j' = the group's offset) and writes
// it back in place; the sub-problems of the next step are the contiguous
// blocks of M_i/R_i elements.  After the last step, position
// e_1 (M/R_1) + e_2 (M/(R_1 R_2)) + ... holds output k = e_1 + R_1 e_2 + ....
// Inside an R-point DFT every twiddle is a power of W_16 or smaller, i.e. a
// power of two in Goldilocks (W_{2^s} = 2^(39 * 2^(6-s) mod 192)), so those
// multiplications are shifts (GlPow2); only the inter-step twiddles are
// general multiplications, read from a shared-memory table of W_M powers.
// The first step loads from global memory and the last stores to it, so a
// pass makes (steps - 1) shared-memory round trips instead of one per stage
// pair.

constexpr int kN2Threads = 512;
constexpr int kN2Elems = 16;  // elements per thread per step

struct Sched {
    uint32_t n;       // steps
    uint32_t lg[4];   // log2 radix of each step
    uint32_t lgm[4];  // log2 of the sub-problem size M_i at step i
};

// Output index of the last step's group gam: the digit of step i sits at bits
// [lgm_i - lg_i, lgm_i) of the position and goes to bits
// [lg_0 + ... + lg_{i-1}, ...) of k; the last step's own digit is added by
// the caller.
__device__ __forceinline__ uint32_t n2_out_base(const Sched& sc, uint32_t gam, uint32_t lg_last) {
    const uint32_t pos = gam << lg_last;
    uint32_t k = 0, sh = 0;
#pragma unroll
    for (int i = 0; i < 3; i++) {
        if ((uint32_t)i + 1 < sc.n) {
            k |= ((pos >> (sc.lgm[i] - sc.lg[i])) & ((1u << sc.lg[i]) - 1)) << sh;
            sh += sc.lg[i];
        }
    }
    return k;
}

// One step with radix 2^L: the thread's 16 elements are G = 16 / 2^L groups.
// kIn / kOut: the step reads from global memory (first step) or shared
// memory, and writes to global memory (last step) or shared memory.
template <int L, bool kIn, bool kOut, typename IdxT, bool kHalf = false>
__device__ __forceinline__ void n2_step(const PassDesc& d, const Sched& sc, uint32_t lgm, uint64_t* data,
                                        const uint64_t* tws, const uint64_t* ptw, uint32_t q, uint32_t cc,
                                        uint32_t logC, bool cok, IdxT row_in0, IdxT row_out0, uint64_t col0) {
    constexpr int R = 1 << L, G = kN2Elems / R;
    const uint32_t m = d.m, lgs = lgm - L;  // stride M_i / R
    const IdxT w = (IdxT)d.ld;  // row stride
#pragma unroll
    for (int gi = 0; gi < G; gi++) {
        const uint32_t gam = q * G + gi;
        const uint32_t jp = gam & ((1u << lgs) - 1);
        const uint32_t base = ((gam >> lgs) << lgm) + jp;
        uint64_t x[R];
        if (kIn) {
            // rows row_in0 + (base + e 2^lgs) jin of column c0 + cc
            const IdxT rstep = (IdxT)d.jin << lgs;
            const IdxT row_b = row_in0 + (IdxT)base * (IdxT)d.jin;
            const uint64_t* g = d.in + col0 + cc + (uint64_t)row_b * w;
            const IdxT gstep = rstep * w;
#pragma unroll
            for (int e = 0; e < R; e++) {
                x[e] = 0;
                if ((!kHalf || e < R / 2) && cok && (uint64_t)(row_b + (IdxT)e * rstep) < d.rows_valid)
                    x[e] = __ldg(g + (IdxT)e * gstep);
            }
        } else {
            const uint64_t* p = data + (base << logC) + cc;
            const uint32_t st = 1u << (lgs + logC);
#pragma unroll
            for (int e = 0; e < R; e++) x[e] = p[e * st];
        }
        if (kHalf)
            dft_reg_half_lazy<L>(x);
        else
            dft_reg_lazy<L>(x);
        if (!kOut) {
            // W_{M_i}^(j' e) = W_M^(j' e 2^(m - lgm))
            const uint32_t tsh = m - lgm;
#pragma unroll
            for (int e = 1; e < R; e++) x[e] = gl_mul(x[e], tws[(jp * (uint32_t)e) << tsh]);
            uint64_t* p = data + (base << logC) + cc;
            const uint32_t st = 1u << (lgs + logC);
#pragma unroll
            for (int e = 0; e < R; e++) p[e * st] = x[e];
        } else {
            // the last step has M_i = R: lgs = 0, jp = 0, base = gam << L; output
            // k = kb + e 2^(m-L), row row_out0 + k kout
            const uint32_t kb = n2_out_base(sc, gam, L);
            if (d.tw_log) {
#pragma unroll
                for (int e = 0; e < R; e++) x[e] = gl_mul(x[e], ptw[kb | ((uint32_t)e << (m - L))]);
            }
            if (d.canon) {
#pragma unroll
                for (int e = 0; e < R; e++) x[e] = gl_canon(x[e]);
            }
            if (cok) {
                uint64_t* g = d.out + col0 + cc + (uint64_t)(row_out0 + (IdxT)kb * (IdxT)d.kout) * w;
                const IdxT gstep = ((IdxT)d.kout << (m - L)) * w;
#pragma unroll
                for (int e = 0; e < R; e++) g[(IdxT)e * gstep] = x[e];
            }
        }
    }
}

template <typename IdxT>
__global__ void __launch_bounds__(kN2Threads, 2) k_ntt_pass2(PassDesc d, Sched sc) {
    extern __shared__ uint64_t sm[];
    const uint32_t m = d.m, M = 1u << m, logC = d.logC;
    uint64_t* data = sm;                         // [M][C]
    uint64_t* tws = sm + ((size_t)M << logC);    // [M] powers of W_M
    uint64_t* ptw = tws + M;                     // [M] inter-pass twiddles (tw_log != 0)
    // Consecutive blocks take consecutive column groups of the same rows, so
    // the row segments that neighbouring blocks read share DRAM bursts in L2.
    const uint64_t cg = blockIdx.x % d.cgroups, bx = blockIdx.x / d.cgroups;
    const uint64_t col0 = cg << logC;
    const uint64_t f = bx % d.F;                 // one lane per block
    const uint64_t s_idx = bx / d.F;
    const uint32_t tid = threadIdx.x, cc = tid & ((1u << logC) - 1), q = tid >> logC;
    const bool cok = col0 + cc < d.w;
    for (uint32_t i = tid; i < M; i += blockDim.x) tws[i] = root_pow<false>(d, m, i);
    if (d.tw_log) {
        // W_{2^tw_log}^(f k) for this block's lane f and every output k, once
        // per block instead of once per element (the block's columns share them)
        const uint64_t emask = (1ull << d.tw_log) - 1;
        for (uint32_t i = tid; i < M; i += blockDim.x) ptw[i] = root_pow<false>(d, d.tw_log, (f * i) & emask);
    }
    __syncthreads();
    const IdxT row_in0 = (IdxT)(f * d.fin + s_idx * d.sin);
    const IdxT row_out0 = (IdxT)(f * d.fout + s_idx * d.sout);
    // The schedule (make_sched) is 4-bit steps with the remainder last, so
    // only the last step can have a radix below 16.
    if (sc.n == 1) {
        n2_step<4, true, true, IdxT>(d, sc, sc.lgm[0], data, tws, ptw, q, cc, logC, cok, row_in0, row_out0, col0);
        return;
    }
    if (d.half_zero)
        n2_step<4, true, false, IdxT, true>(d, sc, sc.lgm[0], data, tws, ptw, q, cc, logC, cok, row_in0, row_out0, col0);
    else
        n2_step<4, true, false, IdxT>(d, sc, sc.lgm[0], data, tws, ptw, q, cc, logC, cok, row_in0, row_out0, col0);
    __syncthreads();
    if (sc.n == 3) {
        n2_step<4, false, false, IdxT>(d, sc, sc.lgm[1], data, tws, ptw, q, cc, logC, cok, row_in0, row_out0, col0);
        __syncthreads();
    }
    const uint32_t lgm = sc.n == 3 ? sc.lgm[2] : sc.lgm[1];
    switch (lgm) {
        case 4: n2_step<4, false, true, IdxT>(d, sc, lgm, data, tws, ptw, q, cc, logC, cok, row_in0, row_out0, col0); break;
        case 3: n2_step<3, false, true, IdxT>(d, sc, lgm, data, tws, ptw, q, cc, logC, cok, row_in0, row_out0, col0); break;
        case 2: n2_step<2, false, true, IdxT>(d, sc, lgm, data, tws, ptw, q, cc, logC, cok, row_in0, row_out0, col0); break;
        default: n2_step<1, false, true, IdxT>(d, sc, lgm, data, tws, ptw, q, cc, logC, cok, row_in0, row_out0, col0); break;
    }
}

uint32_t floor_log2(uint64_t x) {
    uint32_t r = 0;
    while ((2ull << r) <= x) r++;
    return r;
}

// Radix schedule of an M = 2^m point sub-transform (m >= 4): steps of 4 bits,
// the remainder last.
Sched make_sched(uint32_t m) {
    Sched sc{};
    uint32_t rem = m;
    while (rem > 0) {
        const uint32_t l = rem >= 4 ? 4 : rem;
        sc.lg[sc.n] = l;
        sc.lgm[sc.n] = rem;
        sc.n++;
        rem -= l;
    }
    return sc;
}

// Register-radix pass: one lane per block, C = 2^logC columns, M/16 threads
// per column (at most 512 threads).
template <typename IdxT>
int run_pass2(PassDesc d, uint64_t S, cudaStream_t s) {
    const uint32_t m = d.m;
    uint32_t logC = floor_log2(d.w);
    const uint32_t maxC = floor_log2(kN2Threads) - (m - 4);  // (M/16) << logC <= 512
    if (logC > maxC) logC = maxC;
    d.logC = logC;
    d.logR = 0;
    const uint64_t blocks = d.F * S, cblocks = ceil_div(d.w, 1ull << logC);
    if (blocks * cblocks > 0x7FFFFFFFull) return (int)cudaErrorInvalidConfiguration;
    d.cgroups = (uint32_t)cblocks;
    const size_t smem = 8ull * ((1ull << m) << logC) + 8ull * (1ull << m) * (d.tw_log ? 2 : 1);
    if (smem > 48 * 1024)
        ZK_TRY(cudaFuncSetAttribute(k_ntt_pass2<IdxT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const Sched sc = make_sched(m);
    // first-step element e of a group reads row >= row_in0 + e 2^(m-4) jin, so
    // with 2^(m-1) jin >= rows_valid every element e >= 8 is a padding row
    d.half_zero = sc.n > 1 && (d.jin << (m - 1)) >= d.rows_valid ? 1u : 0u;
    const uint32_t threads = (1u << (m - 4)) << logC;
    k_ntt_pass2<IdxT><<<(unsigned)(blocks * cblocks), threads, smem, s>>>(d, sc);
    ZK_LAUNCH_CHECK();
    return 0;
}

// Tile width (C * R) for a sub-DFT of 2^m rows: keep M * C * R * 8 bytes
// around 64 KB of shared memory, between 4 and 32 u64 per row chunk.
uint32_t tile_log_width(uint32_t m) {
    int lw = 13 - (int)m;
    if (lw < 2) lw = 2;
    if (lw > 5) lw = 5;
    return (uint32_t)lw;
}

template <bool kCallerTab, typename IdxT>
int run_pass(PassDesc d, uint64_t S, cudaStream_t s) {
    const uint32_t logLW = tile_log_width(d.m);
    uint32_t logC = floor_log2(d.w);
    if (logC > logLW) logC = logLW;
    uint32_t logR = logLW - logC;
    uint32_t logF = floor_log2(d.F);
    if (logR > logF) logR = logF;  // a tile never spans more lanes than exist
    d.logC = logC;
    d.logR = logR;
    const uint64_t tiles = (d.F >> logR) * S;
    const uint64_t cblocks = ceil_div(d.w, 1ull << logC);
    if (tiles > 0x7FFFFFFFull || cblocks > 65535) return (int)cudaErrorInvalidConfiguration;
    const size_t smem = 8ull * (((uint64_t)1 << d.m) << (logC + logR)) + 8ull * ((1ull << d.m) / 2);
    if (smem > 48 * 1024)
        ZK_TRY(cudaFuncSetAttribute(k_ntt_pass<kCallerTab, IdxT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)smem));
    dim3 grid((unsigned)tiles, (unsigned)cblocks);
    k_ntt_pass<kCallerTab, IdxT><<<grid, kNttThreads, smem, s>>>(d);
    ZK_LAUNCH_CHECK();
    return 0;
}

// The register-radix kernel for sub-transforms of 2^4 .. 2^11 points on the
// library's own twiddles; the shared-memory radix-2/4 kernel for the rest and
// for the reference entry (which reads the caller's twiddle table).
template <bool kCallerTab, typename IdxT>
int run_pass_sel(PassDesc d, uint64_t S, cudaStream_t s) {
    if constexpr (!kCallerTab) {
        if (d.m >= 4 && d.m <= 11) return run_pass2<IdxT>(d, S, s);
    }
    return run_pass<kCallerTab, IdxT>(d, S, s);
}

// Full transform of size 2^lg over the w columns of `in` (row stride ld;
// rows >= rows_valid are zero) into `out` (row stride ld), using `scratch`
// (2^lg rows of stride ld) between passes.
template <bool kCallerTab, typename IdxT>
int dft_plan_t(const uint64_t* in, uint64_t* out, uint64_t* scratch, uint32_t lg, uint64_t w, uint64_t ld,
               uint64_t rows_valid, const uint64_t* tab, uint32_t tab_log, cudaStream_t s) {
    PassDesc base{};
    base.w = w;
    base.ld = ld;
    base.tab = tab;
    base.tab_log = tab_log;
    if (lg <= 10) {
        PassDesc d = base;
        d.in = in;
        d.out = out;
        d.rows_valid = rows_valid;
        d.F = 1;
        d.fin = 0; d.sin = 0; d.jin = 1;
        d.fout = 0; d.sout = 0; d.kout = 1;
        d.m = lg;
        d.tw_log = 0;
        d.canon = 1;
        return run_pass_sel<kCallerTab, IdxT>(d, 1, s);
    }
    if (lg <= 22) {
        const uint32_t a = (lg + 1) / 2, b = lg - a;  // N1 = 2^a, N2 = 2^b (<= 2^11 each)
        const uint64_t N1 = 1ull << a, N2 = 1ull << b;
        PassDesc A = base;
        A.in = in; A.out = scratch; A.rows_valid = rows_valid;
        A.F = N2; A.fin = 1; A.sin = 0; A.jin = N2;
        A.fout = 1; A.sout = 0; A.kout = N2;
        A.m = a; A.tw_log = lg; A.canon = 0;
        int rc = run_pass_sel<kCallerTab, IdxT>(A, 1, s);
        if (rc) return rc;
        PassDesc B = base;
        B.in = scratch; B.out = out; B.rows_valid = ~0ull;
        B.F = N1; B.fin = N2; B.sin = 0; B.jin = 1;
        B.fout = 1; B.sout = 0; B.kout = N1;
        B.m = b; B.tw_log = 0; B.canon = 1;
        return run_pass_sel<kCallerTab, IdxT>(B, 1, s);
    }
    if (lg <= 30) {
        const uint32_t a = (lg + 2) / 3, rest = lg - a, b = (rest + 1) / 2, c = rest - b;
        const uint64_t N1 = 1ull << a, N2 = 1ull << b, N3 = 1ull << c, N23 = N2 * N3;
        PassDesc A = base;
        A.in = in; A.out = scratch; A.rows_valid = rows_valid;
        A.F = N23; A.fin = 1; A.sin = 0; A.jin = N23;
        A.fout = 1; A.sout = 0; A.kout = N23;
        A.m = a; A.tw_log = lg; A.canon = 0;
        int rc = run_pass_sel<kCallerTab, IdxT>(A, 1, s);
        if (rc) return rc;
        PassDesc B1 = base;
        B1.in = scratch; B1.out = scratch; B1.rows_valid = ~0ull;
        B1.F = N3; B1.fin = 1; B1.sin = N23; B1.jin = N3;
        B1.fout = 1; B1.sout = N23; B1.kout = N3;
        B1.m = b; B1.tw_log = b + c; B1.canon = 0;
        rc = run_pass_sel<kCallerTab, IdxT>(B1, N1, s);
        if (rc) return rc;
        PassDesc B2 = base;
        B2.in = scratch; B2.out = out; B2.rows_valid = ~0ull;
        B2.F = N1; B2.fin = N23; B2.sin = N3; B2.jin = 1;
        B2.fout = 1; B2.sout = N1; B2.kout = N1 * N2;
        B2.m = c; B2.tw_log = 0; B2.canon = 1;
        return run_pass_sel<kCallerTab, IdxT>(B2, N2, s);
    }
    return (int)cudaErrorInvalidValue;
}

template <bool kCallerTab>
int dft_plan(const uint64_t* in, uint64_t* out, uint64_t* scratch, uint32_t lg, uint64_t w, uint64_t ld,
             uint64_t rows_valid, const uint64_t* tab, uint32_t tab_log, cudaStream_t s) {
    // 32-bit offsets when the whole 2^lg x ld matrix is addressable with them
    if (lg < 32 && (ld << lg) < (1ull << 32))
        return dft_plan_t<kCallerTab, uint32_t>(in, out, scratch, lg, w, ld, rows_valid, tab, tab_log, s);
    return dft_plan_t<kCallerTab, uint64_t>(in, out, scratch, lg, w, ld, rows_valid, tab, tab_log, s);
}

// Input of one coset of the LDE (the rows i = g + G*i' of the H-row output):
// y[j'][c] = sum_{m < nfold} x[j' + m*stride][c] * W_H^((j' + m*stride) * g)
// for j' < R.  Rows of x at or past L are zero.  Then the coset is the
// R-point DFT of y (zero-padded to H/G rows when R = L < H/G).
//
// The twist factor depends on the row only, so a block takes a tile of
// kTwistRows rows: it computes the tile's kTwistRows * nfold factors once in
// shared memory, then its threads walk the tile's (row, column) elements with
// consecutive threads on consecutive columns (coalesced rows of x and y).
// Each element costs nfold loads and one exact 160-bit dot product; the
// factors cost one table product per row and fold term instead of one per
// element.
constexpr int kTwistThreads = 256;
constexpr uint32_t kTwistRows = 8;
constexpr uint32_t kTwistMaxFold = 512;  // kTwistRows * kTwistMaxFold factors = 32 KB of shared memory

__device__ __forceinline__ uint64_t coset_factor(uint64_t j, uint64_t g, uint32_t lg_h) {
    // W_H^(j g) with W_H = w32^(2^(32 - lg_h)): exponent of w32 mod 2^32
    const uint32_t E = (uint32_t)(((j * g) << (32 - lg_h)) & 0xFFFFFFFFull);
    return gl_mul(__ldg(g_tw_lo + (E & 0xFFFF)), __ldg(g_tw_hi + (E >> 16)));
}

__global__ void __launch_bounds__(kTwistThreads)
    k_coset_twist(const uint64_t* __restrict__ x, uint64_t L, uint64_t w, uint32_t lg_h, uint64_t g, uint64_t R,
                  uint64_t stride, uint32_t nfold, uint64_t* __restrict__ y) {
    __shared__ uint64_t fac[kTwistRows * kTwistMaxFold];
    const uint64_t r0 = (uint64_t)blockIdx.x * kTwistRows;
    const uint32_t rows = (uint32_t)(R - r0 < kTwistRows ? R - r0 : kTwistRows);
    for (uint32_t i = threadIdx.x; i < rows * nfold; i += kTwistThreads) {
        const uint32_t r = i / nfold, m = i - r * nfold;
        const uint64_t j = r0 + r + (uint64_t)m * stride;
        fac[i] = j < L ? coset_factor(j, g, lg_h) : 0;
    }
    __syncthreads();
    // walk the tile's elements with the row / column pair advanced by the
    // stride (no division per element)
    uint32_t r = 0;
    uint64_t c = threadIdx.x;
    while (c >= w && r < rows) {
        c -= w;
        r++;
    }
    if (nfold == 1) {
        // no fold (G <= blowup): a pointwise twist; four elements per
        // iteration so that four reads are in flight per thread
        while (r < rows) {
            uint32_t rr[4];
            uint64_t cc[4], v[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                rr[u] = r;
                cc[u] = c;
                if (r < rows) {
                    const uint64_t j = r0 + r;
                    v[u] = j < L ? __ldg(x + j * w + c) : 0ull;
                    c += kTwistThreads;
                    while (c >= w && r < rows) {
                        c -= w;
                        r++;
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < 4; u++)
                if (rr[u] < rows) y[(r0 + rr[u]) * w + cc[u]] = gl_canon(gl_mul(v[u], fac[rr[u]]));
        }
        return;
    }
    for (; r < rows;) {
        const uint64_t jp = r0 + r;
        Acc160 acc = acc160_zero();
        // fold terms four at a time, their loads issued before the products
        // (several reads in flight per thread; rows at or past L read nothing)
        for (uint32_t m0 = 0; m0 < nfold; m0 += 4) {
            uint64_t v[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const uint64_t j = jp + (uint64_t)(m0 + u) * stride;
                v[u] = (m0 + u < nfold && j < L) ? __ldg(x + j * w + c) : 0ull;
            }
#pragma unroll
            for (int u = 0; u < 4; u++)
                if (m0 + u < nfold) acc160_mac(acc, v[u], fac[r * nfold + m0 + u]);
        }
        y[jp * w + c] = gl_canon(acc160_reduce(acc));
        c += kTwistThreads;
        while (c >= w && r < rows) {
            c -= w;
            r++;
        }
    }
}

// The same for fold counts above kTwistMaxFold (very many cosets per
// blowup): factors computed per element.
__global__ void __launch_bounds__(kTwistThreads)
    k_coset_twist_wide(const uint64_t* __restrict__ x, uint64_t L, uint64_t w, uint32_t lg_h, uint64_t g, uint64_t R,
                       uint64_t stride, uint32_t nfold, uint64_t* __restrict__ y) {
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= R * w) return;
    const uint64_t jp = idx / w, c = idx - jp * w;
    Acc160 acc = acc160_zero();
    for (uint32_t m = 0; m < nfold; m++) {
        const uint64_t j = jp + m * stride;
        if (j >= L) break;
        acc160_mac(acc, __ldg(x + j * w + c), coset_factor(j, g, lg_h));
    }
    y[idx] = gl_canon(acc160_reduce(acc));
}

}  // namespace

uint64_t lde_scratch_elems(uint32_t lg_l, uint32_t lg_blowup, uint64_t w) {
    const uint32_t lg = lg_l + lg_blowup;
    return lg <= 10 ? 0 : (w << lg);
}

int lde_launch_ld(const uint64_t* in, uint64_t* out, uint64_t* scratch, uint32_t lg_l, uint32_t lg_blowup,
                  uint64_t w, uint64_t ld, cudaStream_t s) {
    const uint32_t lg = lg_l + lg_blowup;
    if (w == 0) return 0;
    if (!in || !out || (lg > 10 && !scratch) || ld < w) return (int)cudaErrorInvalidValue;
    if (lg > 30) return (int)cudaErrorInvalidValue;
    int rc = ensure_twiddles();
    if (rc) return rc;
    return dft_plan<false>(in, out, scratch, lg, w, ld, 1ull << lg_l, nullptr, 0, s);
}

int lde_launch(const uint64_t* in, uint64_t* out, uint64_t* scratch, uint32_t lg_l,
               uint32_t lg_blowup, uint64_t w, cudaStream_t s) {
    return lde_launch_ld(in, out, scratch, lg_l, lg_blowup, w, w, s);
}

// Coset g of G = 2^lg_g of the LDE (H = 2^(lg_l + lg_blowup) rows): rows
// i = g + G*i', i' < H/G, in order.  Row i of the LDE is X(W_H^i), so the
// coset is the H/G-point DFT of x[j] W_H^(j g) with the input folded modulo
// H/G: when G <= blowup the L nonzero rows fit (twist, then an LDE of blowup
// 2^(lg_blowup - lg_g)); when G > blowup, G/blowup input rows land on each
// of the H/G DFT inputs.  Scratch: rows(y) * w for y, then the sub-LDE's.
uint64_t lde_coset_scratch_elems(uint32_t lg_l, uint32_t lg_blowup, uint64_t w, uint32_t lg_g) {
    const uint32_t lg_h = lg_l + lg_blowup;
    if (lg_g > lg_h) return 0;
    const uint32_t lg_y = lg_g <= lg_blowup ? lg_l : lg_h - lg_g;
    const uint32_t lg_sub = lg_h - lg_g;
    return (w << lg_y) + lde_scratch_elems(lg_sub, 0, w) + 2;
}

int lde_coset_launch(const uint64_t* in, uint64_t* out, uint64_t* scratch, uint32_t lg_l, uint32_t lg_blowup,
                     uint64_t w, uint32_t lg_g, uint64_t g, cudaStream_t s) {
    const uint32_t lg_h = lg_l + lg_blowup;
    if (w == 0) return 0;
    if (!in || !out || !scratch || lg_g > lg_h || lg_h > 30 || g >= (1ull << lg_g)) return (int)cudaErrorInvalidValue;
    int rc = ensure_twiddles();
    if (rc) return rc;
    const bool fold = lg_g > lg_blowup;
    const uint32_t lg_y = fold ? lg_h - lg_g : lg_l;
    const uint64_t R = 1ull << lg_y;
    uint64_t* y = scratch;
    uint64_t* sub = scratch + ((w << lg_y) + 1 & ~1ull);  // keep 16-byte alignment
    const uint64_t n = R * w;
    const uint32_t nfold = fold ? 1u << (lg_g - lg_blowup) : 1u;
    const uint64_t stride = 1ull << (lg_h - lg_g);
    if (nfold <= kTwistMaxFold && ceil_div(R, kTwistRows) <= 0x7FFFFFFFull)
        k_coset_twist<<<(unsigned)ceil_div(R, kTwistRows), kTwistThreads, 0, s>>>(in, 1ull << lg_l, w, lg_h, g, R,
                                                                                  stride, nfold, y);
    else
        k_coset_twist_wide<<<(unsigned)ceil_div(n, kTwistThreads), kTwistThreads, 0, s>>>(in, 1ull << lg_l, w, lg_h,
                                                                                           g, R, stride, nfold, y);
    ZK_LAUNCH_CHECK();
    if (fold) return dft_plan<false>(y, out, sub, lg_h - lg_g, w, w, ~0ull, nullptr, 0, s);
    return dft_plan<false>(y, out, sub, lg_h - lg_g, w, w, 1ull << lg_l, nullptr, 0, s);
}

}  // namespace zk

using namespace zk;

extern "C" {

// Reference-facing forward NTT (goldilocks_ntt.cu:105-137, bound in
// pcs/cuda_ffi.rs:3-9): d_mat (h x w, h = 2^lg_h, row-major) is overwritten
// in place with natural-order canonical evaluations; d_temp holds h*w u64 of
// scratch; d_tw holds the concatenated per-stage tables of
// pcs/dft_cuda.rs:44-59 (stage s at offset 2^(s-1) - 1, tw_s[j] =
// TWO_ADIC_GENERATORS[s]^j).  Every twiddle is read from the top stage
// s = lg_h of that table.  lg_h == 0 or w == 0 is a no-op.  Default stream.
int zkie_ntt_forward_goldilocks(uint64_t* d_mat, uint64_t* d_temp, uint32_t lg_h, uint64_t w,
                                const uint64_t* d_tw) {
    if (lg_h == 0 || w == 0) return 0;
    if (!d_mat || !d_tw || (lg_h > 10 && !d_temp)) return (int)cudaErrorInvalidValue;
    if (lg_h > 30) return (int)cudaErrorInvalidValue;
    const uint64_t* top = d_tw + ((1ull << (lg_h - 1)) - 1);
    return dft_plan<true>(d_mat, d_mat, d_temp, lg_h, w, w, ~0ull, top, lg_h, 0);
}

uint64_t zkie2_lde_scratch_elems(uint32_t lg_l, uint32_t lg_blowup, uint64_t w) {
    return lde_scratch_elems(lg_l, lg_blowup, w);
}

int zkie2_lde(const uint64_t* d_in, uint64_t* d_out, uint64_t* d_scratch, uint32_t lg_l,
              uint32_t lg_blowup, uint64_t w, cudaStream_t stream) {
    return lde_launch(d_in, d_out, d_scratch, lg_l, lg_blowup, w, stream);
}

// Host-side builder of the reference's concatenated per-stage DIT twiddles
// (pcs/dft_cuda.rs:44-59) for size 2^lg: stage s at offset 2^(s-1) - 1 holds
// TWO_ADIC_GENERATORS[s]^j for j < 2^(s-1); 2^lg - 1 entries in total.
int zkie2_dft_twiddles(uint32_t lg, uint64_t* h_out) {
    if (!h_out || lg > 32) return (int)cudaErrorInvalidValue;
    uint64_t off = 0;
    for (uint32_t s = 1; s <= lg; s++) {
        const uint64_t root = two_adic_generator_host(s);
        uint64_t acc = 1;
        for (uint64_t j = 0; j < (1ull << (s - 1)); j++) {
            h_out[off + j] = acc;
            acc = gl_mul_host(acc, root);
        }
        off += 1ull << (s - 1);
    }
    return 0;
}

int zkie2_dft(const uint64_t* d_in, uint64_t* d_out, uint64_t* d_scratch, uint32_t lg_h, uint64_t w,
              cudaStream_t stream) {
    return lde_launch(d_in, d_out, d_scratch, lg_h, 0, w, stream);
}

uint64_t zkie2_lde_coset_scratch_elems(uint32_t lg_l, uint32_t lg_blowup, uint64_t w, uint32_t lg_g) {
    return lde_coset_scratch_elems(lg_l, lg_blowup, w, lg_g);
}

int zkie2_lde_coset(const uint64_t* d_in, uint64_t* d_out, uint64_t* d_scratch, uint32_t lg_l, uint32_t lg_blowup,
                    uint64_t w, uint32_t lg_g, uint64_t g, cudaStream_t stream) {
    return lde_coset_launch(d_in, d_out, d_scratch, lg_l, lg_blowup, w, lg_g, g, stream);
}

}  // extern "C"
