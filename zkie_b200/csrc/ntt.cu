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

#include "../../include/zkie_goldilocks_cuda.h"
#include "../../include/zkie2.h"
#include "common.cuh"
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
    uint64_t w;           // row width of in and out
    uint64_t rows_valid;  // input rows >= rows_valid are zero (LDE padding)
    uint64_t F;           // lanes
    uint64_t fin, sin, jin;
    uint64_t fout, sout, kout;
    uint32_t m;       // log2 of the sub-DFT size M
    uint32_t logC;    // log2 of the tile columns C
    uint32_t logR;    // log2 of the tile lanes R (C * R = tile width)
    uint32_t tw_log;  // 0: no inter-pass twiddle; else multiply by W_{2^tw_log}^(f*k)
    uint32_t canon;   // canonicalize the output
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

template <bool kCallerTab>
__global__ void __launch_bounds__(kNttThreads) k_ntt_pass(PassDesc d) {
    extern __shared__ uint64_t sm[];
    const uint32_t M = 1u << d.m;
    const uint32_t C = 1u << d.logC, R = 1u << d.logR;
    const uint32_t LW = C * R;
    const uint32_t logLW = d.logC + d.logR;
    uint64_t* data = sm;                       // [M][LW]
    uint64_t* tws = sm + (uint64_t)M * LW;     // [M/2] powers of W_M

    const uint64_t tiles_f = d.F >> d.logR;
    const uint64_t tile = blockIdx.x;
    const uint64_t s_idx = tile / tiles_f;
    const uint64_t f0 = (tile % tiles_f) << d.logR;
    const uint64_t c0 = (uint64_t)blockIdx.y << d.logC;
    const uint64_t ccur = (d.w - c0) < C ? (d.w - c0) : C;
    const uint32_t tid = threadIdx.x;

    for (uint32_t i = tid; i < M / 2; i += kNttThreads) tws[i] = root_pow<kCallerTab>(d, d.m, i);

    const uint64_t sbase_in = s_idx * d.sin;
    const uint32_t total = M << logLW;
    if (d.jin == 1) {
        // j is the contiguous direction: c fastest, then j, then lane.
        for (uint32_t idx = tid; idx < total; idx += kNttThreads) {
            const uint32_t c = idx & (C - 1);
            const uint32_t j = (idx >> d.logC) & (M - 1);
            const uint32_t fl = idx >> (d.logC + d.m);
            const uint64_t row = (f0 + fl) * d.fin + sbase_in + j;
            uint64_t v = 0;
            if (row < d.rows_valid && c < ccur) v = __ldg(d.in + row * d.w + c0 + c);
            data[((uint64_t)brev_m(j, d.m) << logLW) + (fl << d.logC) + c] = v;
        }
    } else {
        // lanes are the contiguous direction: c fastest, then lane, then j.
        for (uint32_t idx = tid; idx < total; idx += kNttThreads) {
            const uint32_t c = idx & (C - 1);
            const uint32_t fl = (idx >> d.logC) & (R - 1);
            const uint32_t j = idx >> logLW;
            const uint64_t row = (f0 + fl) * d.fin + sbase_in + (uint64_t)j * d.jin;
            uint64_t v = 0;
            if (row < d.rows_valid && c < ccur) v = __ldg(d.in + row * d.w + c0 + c);
            data[((uint64_t)brev_m(j, d.m) << logLW) + (fl << d.logC) + c] = v;
        }
    }
    __syncthreads();

    // Radix-2 DIT stages on bit-reversed input -> natural-order output.
    const uint32_t nbf = (M / 2) << logLW;
    for (uint32_t s = 1; s <= d.m; s++) {
        const uint32_t hb = s - 1;
        for (uint32_t b = tid; b < nbf; b += kNttThreads) {
            const uint32_t lane = b & (LW - 1);
            const uint32_t bb = b >> logLW;
            const uint32_t jj = bb & ((1u << hb) - 1);
            const uint32_t i = ((bb >> hb) << s) | jj;
            const uint64_t tw = tws[jj << (d.m - s)];
            uint64_t* p = data + ((uint64_t)i << logLW) + lane;
            uint64_t* q = p + ((uint64_t)1 << (hb + logLW));
            const uint64_t u = *p;
            const uint64_t v = gl_mul(*q, tw);
            *p = gl_add(u, v);
            *q = gl_sub(u, v);
        }
        __syncthreads();
    }

    const uint64_t sbase_out = s_idx * d.sout;
    // Outputs: lanes contiguous (fout == 1) -> c fastest, then lane, then k.
    for (uint32_t idx = tid; idx < total; idx += kNttThreads) {
        uint32_t c, fl, k;
        if (d.fout == 1) {
            c = idx & (C - 1);
            fl = (idx >> d.logC) & (R - 1);
            k = idx >> logLW;
        } else {
            c = idx & (C - 1);
            k = (idx >> d.logC) & (M - 1);
            fl = idx >> (d.logC + d.m);
        }
        uint64_t v = data[((uint64_t)k << logLW) + (fl << d.logC) + c];
        if (d.tw_log) {
            const uint64_t e = ((f0 + fl) * (uint64_t)k) & ((1ull << d.tw_log) - 1);
            v = gl_mul(v, root_pow<kCallerTab>(d, d.tw_log, e));
        }
        if (d.canon) v = gl_canon(v);
        const uint64_t row = (f0 + fl) * d.fout + sbase_out + (uint64_t)k * d.kout;
        if (c < ccur) d.out[row * d.w + c0 + c] = v;
    }
}

uint32_t floor_log2(uint64_t x) {
    uint32_t r = 0;
    while ((2ull << r) <= x) r++;
    return r;
}

// Tile width (C * R) for a sub-DFT of 2^m rows: keep M * C * R * 8 bytes
// around 64 KB of shared memory, between 8 and 32 u64 per row chunk.
uint32_t tile_log_width(uint32_t m) {
    int lw = 13 - (int)m;
    if (lw < 3) lw = 3;
    if (lw > 5) lw = 5;
    return (uint32_t)lw;
}

template <bool kCallerTab>
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
        ZK_TRY(cudaFuncSetAttribute(k_ntt_pass<kCallerTab>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)smem));
    dim3 grid((unsigned)tiles, (unsigned)cblocks);
    k_ntt_pass<kCallerTab><<<grid, kNttThreads, smem, s>>>(d);
    ZK_LAUNCH_CHECK();
    return 0;
}

// Full transform of size 2^lg over the columns of `in` (rows >= rows_valid
// are zero) into `out`, using `scratch` (2^lg * w u64) between passes.
template <bool kCallerTab>
int dft_plan(const uint64_t* in, uint64_t* out, uint64_t* scratch, uint32_t lg, uint64_t w,
             uint64_t rows_valid, const uint64_t* tab, uint32_t tab_log, cudaStream_t s) {
    PassDesc base{};
    base.w = w;
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
        return run_pass<kCallerTab>(d, 1, s);
    }
    if (lg <= 20) {
        const uint32_t a = (lg + 1) / 2, b = lg - a;  // N1 = 2^a, N2 = 2^b
        const uint64_t N1 = 1ull << a, N2 = 1ull << b;
        PassDesc A = base;
        A.in = in; A.out = scratch; A.rows_valid = rows_valid;
        A.F = N2; A.fin = 1; A.sin = 0; A.jin = N2;
        A.fout = 1; A.sout = 0; A.kout = N2;
        A.m = a; A.tw_log = lg; A.canon = 0;
        int rc = run_pass<kCallerTab>(A, 1, s);
        if (rc) return rc;
        PassDesc B = base;
        B.in = scratch; B.out = out; B.rows_valid = ~0ull;
        B.F = N1; B.fin = N2; B.sin = 0; B.jin = 1;
        B.fout = 1; B.sout = 0; B.kout = N1;
        B.m = b; B.tw_log = 0; B.canon = 1;
        return run_pass<kCallerTab>(B, 1, s);
    }
    if (lg <= 30) {
        const uint32_t a = (lg + 2) / 3, rest = lg - a, b = (rest + 1) / 2, c = rest - b;
        const uint64_t N1 = 1ull << a, N2 = 1ull << b, N3 = 1ull << c, N23 = N2 * N3;
        PassDesc A = base;
        A.in = in; A.out = scratch; A.rows_valid = rows_valid;
        A.F = N23; A.fin = 1; A.sin = 0; A.jin = N23;
        A.fout = 1; A.sout = 0; A.kout = N23;
        A.m = a; A.tw_log = lg; A.canon = 0;
        int rc = run_pass<kCallerTab>(A, 1, s);
        if (rc) return rc;
        PassDesc B1 = base;
        B1.in = scratch; B1.out = scratch; B1.rows_valid = ~0ull;
        B1.F = N3; B1.fin = 1; B1.sin = N23; B1.jin = N3;
        B1.fout = 1; B1.sout = N23; B1.kout = N3;
        B1.m = b; B1.tw_log = b + c; B1.canon = 0;
        rc = run_pass<kCallerTab>(B1, N1, s);
        if (rc) return rc;
        PassDesc B2 = base;
        B2.in = scratch; B2.out = out; B2.rows_valid = ~0ull;
        B2.F = N1; B2.fin = N23; B2.sin = N3; B2.jin = 1;
        B2.fout = 1; B2.sout = N1; B2.kout = N1 * N2;
        B2.m = c; B2.tw_log = 0; B2.canon = 1;
        return run_pass<kCallerTab>(B2, N2, s);
    }
    return (int)cudaErrorInvalidValue;
}

}  // namespace

uint64_t lde_scratch_elems(uint32_t lg_l, uint32_t lg_blowup, uint64_t w) {
    const uint32_t lg = lg_l + lg_blowup;
    return lg <= 10 ? 0 : (w << lg);
}

int lde_launch(const uint64_t* in, uint64_t* out, uint64_t* scratch, uint32_t lg_l,
               uint32_t lg_blowup, uint64_t w, cudaStream_t s) {
    const uint32_t lg = lg_l + lg_blowup;
    if (w == 0) return 0;
    if (!in || !out || (lg > 10 && !scratch)) return (int)cudaErrorInvalidValue;
    if (lg > 30) return (int)cudaErrorInvalidValue;
    int rc = ensure_twiddles();
    if (rc) return rc;
    return dft_plan<false>(in, out, scratch, lg, w, 1ull << lg_l, nullptr, 0, s);
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
    return dft_plan<true>(d_mat, d_mat, d_temp, lg_h, w, ~0ull, top, lg_h, 0);
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

}  // extern "C"
