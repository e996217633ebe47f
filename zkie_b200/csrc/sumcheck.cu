// sumcheck.cu -- the matmul GKR reduction on the device: MLE eq-contractions
// (eval / partial_eval), the degree-2 sumcheck with all rounds run from
// challenges known up front, and the field matmul that produces the witness.
//
// Reference: crates/zkie-core/src/common/{mle.rs:8-64, sumcheck.rs:33-89,
// matmul.rs:17-46}.  Because the reference draws every challenge before it
// proves (sumcheck.rs:33-38, zkie-ops/src/compose.rs:1727-1735), no round needs
// a host round trip: one launch folds up to 11 rounds of a chunk in shared
// memory, so a 2^t-element sumcheck reads f and h from HBM once per 11 rounds.
//
// MLE evaluation by folding (a + r(b - a) per variable) and by contraction
// with the equality table (sum_x v[x] eq(r, x)) give the same field element;
// the contraction form reads each input once and needs no scratch writes.
#include <mutex>
#include <vector>

#include "../../include/zkie2.h"
#include "common.cuh"
#include "gl64.cuh"
#include "internal.h"

namespace zk {

namespace {

constexpr int kMaxVars = 48;
struct Point {
    uint64_t r[kMaxVars];
};

constexpr int kThreads = 256;

// eq(r, x) for x < 2^d: prod_j (bit_j(x) ? r_j : 1 - r_j)   (mle.rs:44-55)
__global__ void k_eq_table(Point p, uint32_t d, uint64_t* __restrict__ out) {
    const uint64_t x = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (x >= (1ull << d)) return;
    uint64_t acc = 1;
    for (uint32_t j = 0; j < d; j++) {
        const uint64_t rj = p.r[j];
        acc = gl_mul(acc, ((x >> j) & 1) ? rj : gl_sub(1, rj));
    }
    out[x] = gl_canon(acc);
}

__device__ __forceinline__ uint64_t warp_sum(uint64_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = gl_add(v, __shfl_down_sync(0xffffffffu, v, o));
    return v;
}

// out[y] = sum_{x < X} v[y*X + x] * eq[x], X >= 32: one warp per output.
__global__ void k_contract_warp(const uint64_t* __restrict__ v, const uint64_t* __restrict__ eq,
                                uint64_t X, uint64_t Y, uint64_t* __restrict__ out) {
    const uint64_t warp = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const uint32_t lane = threadIdx.x & 31;
    if (warp >= Y) return;
    const uint64_t* src = v + warp * X;
    uint64_t acc = 0;
    for (uint64_t x = lane; x < X; x += 32) acc = gl_add(acc, gl_mul(__ldg(src + x), __ldg(eq + x)));
    acc = warp_sum(acc);
    if (lane == 0) out[warp] = gl_canon(acc);
}

// Same contraction for X < 32: one thread per output.
__global__ void k_contract_thread(const uint64_t* __restrict__ v, const uint64_t* __restrict__ eq,
                                  uint64_t X, uint64_t Y, uint64_t* __restrict__ out) {
    const uint64_t y = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (y >= Y) return;
    const uint64_t* src = v + y * X;
    uint64_t acc = 0;
    for (uint64_t x = 0; x < X; x++) acc = gl_add(acc, gl_mul(__ldg(src + x), __ldg(eq + x)));
    out[y] = gl_canon(acc);
}

// out[c] = sum_{r < R} v[r*K + c] * eq[r]: contraction over the rows of an
// R x K row-major matrix, i.e. partial_eval of its transpose without
// materialising the transpose (zkie-ops/src/compose.rs:52-60 + mle.rs:25-38).
__global__ void k_contract_rows(const uint64_t* __restrict__ v, const uint64_t* __restrict__ eq,
                                uint64_t R, uint64_t K, uint64_t* __restrict__ out) {
    const uint64_t c = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= K) return;
    uint64_t acc = 0;
    for (uint64_t r = 0; r < R; r++) acc = gl_add(acc, gl_mul(__ldg(v + r * K + c), __ldg(eq + r)));
    out[c] = gl_canon(acc);
}

// Up to kMaxQ sumcheck rounds on one chunk of 2^q consecutive elements of f
// and h (sumcheck.rs:48-72): for each round the chunk's contributions to
// y0 = sum f0 h0, y1 = sum f1 h1, y2 = sum (2f1 - f0)(2h1 - h0) go to
// partials[chunk][round][3]; then both vectors fold with the round's challenge
// (a + r(b - a)).  The folded single values go to f_out/h_out[chunk].
constexpr int kMaxQ = 11;
struct Chal {
    uint64_t r[kMaxQ];
};

__device__ __forceinline__ void block_sum3(uint64_t& a, uint64_t& b, uint64_t& c, uint64_t* red) {
    a = warp_sum(a);
    b = warp_sum(b);
    c = warp_sum(c);
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) {
        red[3 * w] = a;
        red[3 * w + 1] = b;
        red[3 * w + 2] = c;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const int nw = blockDim.x >> 5;
        for (int i = 1; i < nw; i++) {
            a = gl_add(a, red[3 * i]);
            b = gl_add(b, red[3 * i + 1]);
            c = gl_add(c, red[3 * i + 2]);
        }
    }
}

__global__ void __launch_bounds__(kThreads)
    k_sumcheck_chunk(const uint64_t* __restrict__ f, const uint64_t* __restrict__ h, uint32_t q,
                     Chal ch, uint64_t* __restrict__ partials, uint64_t* __restrict__ f_out,
                     uint64_t* __restrict__ h_out) {
    __shared__ uint64_t sf[1 << kMaxQ], sh[1 << kMaxQ];
    __shared__ uint64_t red[3 * (kThreads / 32)];
    const uint32_t Q = 1u << q;
    const uint64_t base = (uint64_t)blockIdx.x << q;
    for (uint32_t i = threadIdx.x; i < Q; i += kThreads) {
        sf[i] = __ldg(f + base + i);
        sh[i] = __ldg(h + base + i);
    }
    __syncthreads();
    constexpr int kPer = (1 << kMaxQ) / 2 / kThreads;  // pairs per thread at most
    for (uint32_t rd = 0; rd < q; rd++) {
        const uint32_t pairs = (Q >> rd) >> 1;
        uint64_t y0 = 0, y1 = 0, y2 = 0;
        uint64_t nf[kPer > 0 ? kPer : 1], nh[kPer > 0 ? kPer : 1];
        const uint64_t r = ch.r[rd];
#pragma unroll
        for (int t = 0; t < (kPer > 0 ? kPer : 1); t++) {
            const uint32_t s = threadIdx.x + t * kThreads;
            if (s < pairs) {
                const uint64_t f0 = sf[2 * s], f1 = sf[2 * s + 1];
                const uint64_t h0 = sh[2 * s], h1 = sh[2 * s + 1];
                y0 = gl_add(y0, gl_mul(f0, h0));
                y1 = gl_add(y1, gl_mul(f1, h1));
                y2 = gl_add(y2, gl_mul(gl_sub(gl_add(f1, f1), f0), gl_sub(gl_add(h1, h1), h0)));
                nf[t] = gl_add(f0, gl_mul(r, gl_sub(f1, f0)));
                nh[t] = gl_add(h0, gl_mul(r, gl_sub(h1, h0)));
            }
        }
        block_sum3(y0, y1, y2, red);
        if (threadIdx.x == 0) {
            uint64_t* p = partials + ((uint64_t)blockIdx.x * kMaxQ + rd) * 3;
            p[0] = y0;
            p[1] = y1;
            p[2] = y2;
        }
        __syncthreads();
#pragma unroll
        for (int t = 0; t < (kPer > 0 ? kPer : 1); t++) {
            const uint32_t s = threadIdx.x + t * kThreads;
            if (s < pairs) {
                sf[s] = nf[t];
                sh[s] = nh[t];
            }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        f_out[blockIdx.x] = sf[0];
        h_out[blockIdx.x] = sh[0];
    }
}

// Sum the per-chunk partials of each round and turn (y0, y1, y2) into the
// round polynomial c0 = y0, c1 = (4y1 - y2 - 3y0)/2, c2 = (y2 - 2y1 + y0)/2
// (sumcheck.rs:65-68).  One block per round.
__global__ void k_sumcheck_reduce(const uint64_t* __restrict__ partials, uint64_t G, uint32_t q,
                                  uint64_t* __restrict__ rounds) {
    __shared__ uint64_t red[3 * (kThreads / 32)];
    const uint32_t rd = blockIdx.x;
    uint64_t y0 = 0, y1 = 0, y2 = 0;
    for (uint64_t g = threadIdx.x; g < G; g += kThreads) {
        const uint64_t* p = partials + (g * kMaxQ + rd) * 3;
        y0 = gl_add(y0, p[0]);
        y1 = gl_add(y1, p[1]);
        y2 = gl_add(y2, p[2]);
    }
    block_sum3(y0, y1, y2, red);
    if (threadIdx.x == 0) {
        const uint64_t inv2 = 0x7FFFFFFF80000001ull;  // (p + 1) / 2
        const uint64_t c1 = gl_mul(gl_sub(gl_sub(gl_mul(4, y1), y2), gl_mul(3, y0)), inv2);
        const uint64_t c2 = gl_mul(gl_add(gl_sub(y2, gl_add(y1, y1)), y0), inv2);
        uint64_t* o = rounds + 3ull * rd;
        o[0] = gl_canon(y0);
        o[1] = gl_canon(c1);
        o[2] = gl_canon(c2);
    }
}

// Field matmul C = A (m x k) @ B (k x n), the forward witness of Op::MatMul
// (zkie-ops/src/compose.rs:1327-1331; par.rs:41-89 computes the same field
// value through i64 when it cannot overflow).
__global__ void k_matmul_field(const uint64_t* __restrict__ a, const uint64_t* __restrict__ b,
                               uint64_t m, uint64_t k, uint64_t n, uint64_t* __restrict__ c) {
    const uint64_t j = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t i = blockIdx.y;
    if (j >= n || i >= m) return;
    uint64_t acc = 0;
    for (uint64_t q = 0; q < k; q++) acc = gl_add(acc, gl_mul(__ldg(a + i * k + q), __ldg(b + q * n + j)));
    c[i * n + j] = gl_canon(acc);
}

__global__ void k_canon_copy(const uint64_t* __restrict__ in, uint64_t* __restrict__ out, uint64_t n) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = gl_canon(in[i]);
}

int eq_table(const uint64_t* h_r, uint32_t d, uint64_t* d_out, cudaStream_t s) {
    if (d > kMaxVars) return (int)cudaErrorInvalidValue;
    Point p{};
    for (uint32_t j = 0; j < d; j++) p.r[j] = h_r[j];
    const uint64_t n = 1ull << d;
    k_eq_table<<<(unsigned)ceil_div(n, kThreads), kThreads, 0, s>>>(p, d, d_out);
    ZK_LAUNCH_CHECK();
    return 0;
}

int contract(const uint64_t* v, const uint64_t* eq, uint64_t X, uint64_t Y, uint64_t* out, cudaStream_t s) {
    if (Y == 0) return 0;
    if (X >= 32) {
        const uint64_t threads = Y * 32;
        k_contract_warp<<<(unsigned)ceil_div(threads, kThreads), kThreads, 0, s>>>(v, eq, X, Y, out);
    } else {
        k_contract_thread<<<(unsigned)ceil_div(Y, kThreads), kThreads, 0, s>>>(v, eq, X, Y, out);
    }
    ZK_LAUNCH_CHECK();
    return 0;
}

}  // namespace

// partial_eval(values (2^t), fix (f vars)) -> 2^(t-f) values in d_out.
// Scratch: 2^f u64 (the eq table).
int partial_eval_dev(const uint64_t* d_values, uint32_t t, const uint64_t* h_fix, uint32_t f,
                     uint64_t* d_out, uint64_t* d_scratch, cudaStream_t s) {
    if (f > t) return (int)cudaErrorInvalidValue;
    if (f == 0) {
        const uint64_t n = 1ull << t;
        k_canon_copy<<<(unsigned)ceil_div(n, kThreads), kThreads, 0, s>>>(d_values, d_out, n);
        ZK_LAUNCH_CHECK();
        return 0;
    }
    int rc = eq_table(h_fix, f, d_scratch, s);
    if (rc) return rc;
    return contract(d_values, d_scratch, 1ull << f, 1ull << (t - f), d_out, s);
}

uint64_t eval_scratch_elems(uint32_t t) {
    // eq table of at most 2^10 entries per level plus the intermediate vectors
    uint64_t tot = 1u << 10;
    uint32_t rest = t;
    while (rest > 0) {
        uint32_t f = rest < 10 ? rest : 10;
        rest -= f;
        tot += 1ull << rest;
    }
    return tot + 8;
}

// eval(values (2^t), point (t vars)) -> d_out[0], via successive 10-variable
// contractions.
int eval_dev(const uint64_t* d_values, uint32_t t, const uint64_t* h_point, uint64_t* d_out,
             uint64_t* d_scratch, cudaStream_t s) {
    if (t == 0) {
        k_canon_copy<<<1, 1, 0, s>>>(d_values, d_out, 1);
        ZK_LAUNCH_CHECK();
        return 0;
    }
    uint64_t* eq = d_scratch;
    uint64_t* buf = d_scratch + (1u << 10);
    const uint64_t* cur = d_values;
    uint32_t rest = t, used = 0;
    while (rest > 0) {
        const uint32_t f = rest < 10 ? rest : 10;
        rest -= f;
        uint64_t* dst = rest == 0 ? d_out : buf;
        int rc = eq_table(h_point + used, f, eq, s);
        if (rc) return rc;
        rc = contract(cur, eq, 1ull << f, 1ull << rest, dst, s);
        if (rc) return rc;
        used += f;
        cur = dst;
        buf += 1ull << rest;
    }
    return 0;
}

constexpr uint64_t sumcheck_scratch_elems_c(uint32_t t) {
    // two folded vectors per launch level (<= 2^(t-11) each) + partials
    return 4 * (t > kMaxQ ? (1ull << (t - kMaxQ)) : 1) + (t > kMaxQ ? (1ull << (t - kMaxQ)) : 1) * kMaxQ * 3 + 64;
}

uint64_t sumcheck_scratch_elems(uint32_t t) { return sumcheck_scratch_elems_c(t); }

// All t rounds of sumcheck::prove on device.  rounds (3t) and finals (2) are
// written to device memory d_rounds.
int sumcheck_dev(const uint64_t* d_f, const uint64_t* d_h, uint32_t t, const uint64_t* h_ch,
                 uint64_t* d_rounds, uint64_t* d_finals, uint64_t* d_scratch, cudaStream_t s) {
    const uint64_t chunks0 = t > kMaxQ ? (1ull << (t - kMaxQ)) : 1;
    uint64_t* fa = d_scratch;
    uint64_t* ha = fa + chunks0;
    uint64_t* fb = ha + chunks0;
    uint64_t* hb = fb + chunks0;
    uint64_t* partials = hb + chunks0;
    if (t == 0) {
        k_canon_copy<<<1, 1, 0, s>>>(d_f, d_finals, 1);
        k_canon_copy<<<1, 1, 0, s>>>(d_h, d_finals + 1, 1);
        ZK_LAUNCH_CHECK();
        return 0;
    }
    const uint64_t* cf = d_f;
    const uint64_t* chh = d_h;
    uint32_t done = 0;
    bool first = true;
    while (done < t) {
        const uint32_t rem = t - done;
        const uint32_t q = rem < (uint32_t)kMaxQ ? rem : (uint32_t)kMaxQ;
        const uint64_t G = 1ull << (rem - q);
        Chal ch{};
        for (uint32_t i = 0; i < q; i++) ch.r[i] = h_ch[done + i];
        uint64_t* of = (rem - q == 0) ? d_finals : (first ? fa : (cf == fa ? fb : fa));
        uint64_t* oh = (rem - q == 0) ? d_finals + 1 : (first ? ha : (chh == ha ? hb : ha));
        k_sumcheck_chunk<<<(unsigned)G, kThreads, 0, s>>>(cf, chh, q, ch, partials, of, oh);
        ZK_LAUNCH_CHECK();
        k_sumcheck_reduce<<<q, kThreads, 0, s>>>(partials, G, q, d_rounds + 3ull * done);
        ZK_LAUNCH_CHECK();
        cf = of;
        chh = oh;
        done += q;
        first = false;
    }
    if (t > 0) {
        // finals were written by the last chunk launch without canonicalization
        k_canon_copy<<<1, 2, 0, s>>>(d_finals, d_finals, 2);
        ZK_LAUNCH_CHECK();
    }
    return 0;
}

int matmul_field_dev(const uint64_t* d_a, const uint64_t* d_b, uint64_t m, uint64_t k, uint64_t n,
                     uint64_t* d_c, cudaStream_t s) {
    if (m == 0 || n == 0) return 0;
    if (m > 65535) return (int)cudaErrorInvalidValue;
    dim3 grid((unsigned)ceil_div(n, kThreads), (unsigned)m);
    k_matmul_field<<<grid, kThreads, 0, s>>>(d_a, d_b, m, k, n, d_c);
    ZK_LAUNCH_CHECK();
    return 0;
}

int contract_rows_dev(const uint64_t* d_v, const uint64_t* d_eq, uint64_t R, uint64_t K, uint64_t* d_out,
                      cudaStream_t s) {
    k_contract_rows<<<(unsigned)ceil_div(K, kThreads), kThreads, 0, s>>>(d_v, d_eq, R, K, d_out);
    ZK_LAUNCH_CHECK();
    return 0;
}

int eq_table_dev(const uint64_t* h_r, uint32_t d, uint64_t* d_out, cudaStream_t s) {
    return eq_table(h_r, d, d_out, s);
}

int contract_dev(const uint64_t* v, const uint64_t* eq, uint64_t X, uint64_t Y, uint64_t* out,
                 cudaStream_t s) {
    return contract(v, eq, X, Y, out, s);
}

// ---- allocation-free sumcheck ------------------------------------------------------
// The scratch of zkie2_sumcheck_prove_noalloc lives in this file-scope device
// array, sized for the largest accepted sumcheck: partial sums and folded
// vectors of a 2^kNoAllocMaxVars-element f and h, then the round polynomials
// and the two final values.  Every GPU that loads the library holds it
// (about 2.4 MB) until the process exits.
constexpr uint32_t kNoAllocMaxVars = 24;
constexpr uint64_t kNoAllocScratchElems = sumcheck_scratch_elems_c(kNoAllocMaxVars) + 3ull * kNoAllocMaxVars + 4;
static __device__ __align__(256) uint64_t g_noalloc_scratch[kNoAllocScratchElems];

namespace {
std::mutex g_noalloc_mu;
uint64_t* g_noalloc_ptr[kMaxDevices];

// Device address of g_noalloc_scratch on the current device, looked up once
// per device.  In host code the array's name is only a host-side stand-in, so
// its device address must come from cudaGetSymbolAddress.
int noalloc_scratch(uint64_t** out) {
    const int d = current_device();
    if (d < 0 || d >= kMaxDevices) return (int)cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> g(g_noalloc_mu);
    if (!g_noalloc_ptr[d]) {
        void* p = nullptr;
        ZK_TRY(cudaGetSymbolAddress(&p, g_noalloc_scratch));
        g_noalloc_ptr[d] = static_cast<uint64_t*>(p);
    }
    *out = g_noalloc_ptr[d];
    return 0;
}
}  // namespace

}  // namespace zk

using namespace zk;

extern "C" {

uint32_t zkie2_sumcheck_noalloc_max_vars(void) { return kNoAllocMaxVars; }

int zkie2_sumcheck_prove_noalloc(const uint64_t* d_f, const uint64_t* d_h, uint32_t t, const uint64_t* h_ch,
                                 uint64_t* h_rounds, uint64_t* h_finals, cudaStream_t stream) {
    if (t > kNoAllocMaxVars) return (int)cudaErrorInvalidValue;  // larger than the static scratch
    if (!d_f || !d_h || !h_finals || (t && (!h_ch || !h_rounds))) return (int)cudaErrorInvalidValue;
    uint64_t* scratch = nullptr;
    int rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    // No part of the scratch needs to start at zero: every partial sum and
    // folded value is written by the launch that precedes its first read.
    uint64_t* d_rounds = scratch + sumcheck_scratch_elems_c(t);
    uint64_t* d_finals = d_rounds + 3ull * t;
    rc = sumcheck_dev(d_f, d_h, t, h_ch, d_rounds, d_finals, scratch, stream);
    if (rc) return rc;
    if (t) ZK_TRY(cudaMemcpyAsync(h_rounds, d_rounds, 24ull * t, cudaMemcpyDeviceToHost, stream));
    ZK_TRY(cudaMemcpyAsync(h_finals, d_finals, 16, cudaMemcpyDeviceToHost, stream));
    ZK_TRY(cudaStreamSynchronize(stream));
    return 0;
}

}  // extern "C"
