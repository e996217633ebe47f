// sumcheck.cu -- the matmul GKR reduction on the device: MLE eq-contractions
// (eval / partial_eval), the degree-2 sumcheck with all rounds run from
// challenges known up front, and the field matmul that produces the witness.
//
// Reference: crates/zkie-core/src/common/{mle.rs:8-64, sumcheck.rs:33-89,
// matmul.rs:17-46}.  Because the reference draws every challenge before it
// proves (sumcheck.rs:33-38, zkie-ops/src/compose.rs:1727-1735), no round needs
// a host round trip: one launch runs nine rounds, each warp folding its own
// 512-element chunk in registers, so a 2^t-element sumcheck reads f and h from
// HBM once per nine rounds (in practice once: the second level reads 1/512).
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

// The same table for d >= 8 with about one multiplication per element: x
// splits into hi = x >> 8 and lo = x & 255, eq(r, x) = eq(r_hi, hi) eq(r_lo, lo).
// A 256-thread block builds the 256 low factors (8 products each) and the
// high factors of its kEqHiPerBlock consecutive hi values (d - 8 each) in
// shared memory, then writes kEqHiPerBlock rows of 256 with one product per
// element (consecutive threads, consecutive addresses).
constexpr uint32_t kEqHiPerBlock = 32;
__global__ void __launch_bounds__(256) k_eq_table_split(Point p, uint32_t d, uint64_t* __restrict__ out) {
    __shared__ uint64_t lo[256], hi[kEqHiPerBlock];
    const uint32_t t = threadIdx.x;
    const uint64_t nhi = 1ull << (d - 8);
    const uint32_t per = nhi < kEqHiPerBlock ? (uint32_t)nhi : kEqHiPerBlock;
    const uint64_t h0 = (uint64_t)blockIdx.x * per;
    uint64_t a = 1;
#pragma unroll
    for (uint32_t j = 0; j < 8; j++) {
        const uint64_t rj = p.r[j];
        a = gl_mul(a, ((t >> j) & 1) ? rj : gl_sub(1, rj));
    }
    lo[t] = a;
    if (t < per) {
        const uint64_t h = h0 + t;
        uint64_t b = 1;
        for (uint32_t j = 8; j < d; j++) {
            const uint64_t rj = p.r[j];
            b = gl_mul(b, ((h >> (j - 8)) & 1) ? rj : gl_sub(1, rj));
        }
        hi[t] = b;
    }
    __syncthreads();
    for (uint32_t i = 0; i < per; i++) out[((h0 + i) << 8) + t] = gl_canon(gl_mul(hi[i], lo[t]));
}

__device__ __forceinline__ uint64_t warp_sum(uint64_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = gl_add(v, __shfl_down_sync(0xffffffffu, v, o));
    return v;
}

// Two consecutive elements p[2i], p[2i+1]: one 16-byte load when the caller
// guarantees 16-byte alignment of p, else two 8-byte loads.
template <bool kVec>
__device__ __forceinline__ ulonglong2 load_pair(const uint64_t* __restrict__ p, uint64_t i) {
    if (kVec) return __ldg(reinterpret_cast<const ulonglong2*>(p) + i);
    return make_ulonglong2(__ldg(p + 2 * i), __ldg(p + 2 * i + 1));
}

// out[y] = sum_{x < X} v[y*X + x] * eq[x] for X = 2^lg_x >= 2 (mle.rs:25-38
// as a contraction with the equality table).  A group of L = 2^lg_l lanes
// (L <= min(32, X/2)) owns one row; lane j streams the element pairs
// j, j + L, j + 2L, ... of the row and of eq, four pairs per iteration so
// eight 16-byte loads are in flight, and accumulates the exact products in
// an Acc160.  Each lane reduces once; a shuffle tree sums the group.
template <bool kVec>
__global__ void __launch_bounds__(kThreads)
    k_contract(const uint64_t* __restrict__ v, const uint64_t* __restrict__ eq, uint32_t lg_x, uint32_t lg_l,
               uint64_t Y, uint64_t* __restrict__ out) {
    const uint64_t gt = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t y = gt >> lg_l;
    const uint32_t L = 1u << lg_l;
    const uint32_t j = (uint32_t)gt & (L - 1);
    Acc160 acc = acc160_zero();
    if (y < Y) {
        const uint64_t* row = v + (y << lg_x);
        const uint32_t npairs = 1u << (lg_x - 1);
        uint32_t i = j;
        for (; i + 3 * L < npairs; i += 4 * L) {
            const ulonglong2 a0 = load_pair<kVec>(row, i), a1 = load_pair<kVec>(row, i + L);
            const ulonglong2 a2 = load_pair<kVec>(row, i + 2 * L), a3 = load_pair<kVec>(row, i + 3 * L);
            const ulonglong2 e0 = load_pair<kVec>(eq, i), e1 = load_pair<kVec>(eq, i + L);
            const ulonglong2 e2 = load_pair<kVec>(eq, i + 2 * L), e3 = load_pair<kVec>(eq, i + 3 * L);
            acc160_mac(acc, a0.x, e0.x);
            acc160_mac(acc, a0.y, e0.y);
            acc160_mac(acc, a1.x, e1.x);
            acc160_mac(acc, a1.y, e1.y);
            acc160_mac(acc, a2.x, e2.x);
            acc160_mac(acc, a2.y, e2.y);
            acc160_mac(acc, a3.x, e3.x);
            acc160_mac(acc, a3.y, e3.y);
        }
        for (; i < npairs; i += L) {
            const ulonglong2 a = load_pair<kVec>(row, i), e = load_pair<kVec>(eq, i);
            acc160_mac(acc, a.x, e.x);
            acc160_mac(acc, a.y, e.y);
        }
    }
    uint64_t s = acc160_reduce(acc);
    for (uint32_t o = L >> 1; o > 0; o >>= 1) s = gl_add(s, __shfl_xor_sync(0xffffffffu, s, o));
    if (y < Y && j == 0) out[y] = gl_canon(s);
}

// part[b][c] = sum over rows r of row block b of v[r*K + c] * eq[r]: the
// contraction over the rows of an R x K row-major matrix, i.e. partial_eval
// of its transpose without materialising the transpose (zkie-ops/src/
// compose.rs:52-60 + mle.rs:25-38).  Grid (column-pair groups, row blocks);
// each thread owns two adjacent columns and streams its block's rows four at
// a time.  With a single row block the result is final and canonical.
template <bool kVec>
__global__ void __launch_bounds__(kThreads)
    k_contract_rows(const uint64_t* __restrict__ v, const uint64_t* __restrict__ eq, uint64_t R, uint64_t K,
                    uint64_t rows_per_block, uint64_t* __restrict__ part) {
    const uint64_t c = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) * 2;
    if (c >= K) return;
    const uint64_t r0 = (uint64_t)blockIdx.y * rows_per_block;
    const uint64_t r1 = r0 + rows_per_block < R ? r0 + rows_per_block : R;
    const bool two = c + 1 < K;  // always true on the vector path (K even)
    Acc160 a0 = acc160_zero(), a1 = acc160_zero();
    auto pair_at = [&](uint64_t r) -> ulonglong2 {
        const uint64_t* p = v + r * K + c;
        if (kVec) return __ldg(reinterpret_cast<const ulonglong2*>(p));
        return make_ulonglong2(__ldg(p), two ? __ldg(p + 1) : 0ull);
    };
    uint64_t r = r0;
    for (; r + 4 <= r1; r += 4) {
        const ulonglong2 x0 = pair_at(r), x1 = pair_at(r + 1), x2 = pair_at(r + 2), x3 = pair_at(r + 3);
        const uint64_t e0 = __ldg(eq + r), e1 = __ldg(eq + r + 1), e2 = __ldg(eq + r + 2), e3 = __ldg(eq + r + 3);
        acc160_mac(a0, x0.x, e0);
        acc160_mac(a1, x0.y, e0);
        acc160_mac(a0, x1.x, e1);
        acc160_mac(a1, x1.y, e1);
        acc160_mac(a0, x2.x, e2);
        acc160_mac(a1, x2.y, e2);
        acc160_mac(a0, x3.x, e3);
        acc160_mac(a1, x3.y, e3);
    }
    for (; r < r1; r++) {
        const ulonglong2 x = pair_at(r);
        const uint64_t e = __ldg(eq + r);
        acc160_mac(a0, x.x, e);
        acc160_mac(a1, x.y, e);
    }
    uint64_t* o = part + (uint64_t)blockIdx.y * K + c;
    const bool fin = gridDim.y == 1;
    const uint64_t s0 = acc160_reduce(a0), s1 = acc160_reduce(a1);
    o[0] = fin ? gl_canon(s0) : s0;
    if (two) o[1] = fin ? gl_canon(s1) : s1;
}

// out[c] = sum_{b < nb} part[b*K + c], canonical.
__global__ void k_sum_rows(const uint64_t* __restrict__ part, uint64_t nb, uint64_t K, uint64_t* __restrict__ out) {
    const uint64_t c = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= K) return;
    uint64_t s = 0;
    for (uint64_t b = 0; b < nb; b++) s = gl_add(s, __ldg(part + b * K + c));
    out[c] = gl_canon(s);
}

// ---- sumcheck rounds -------------------------------------------------------------------
// sumcheck.rs:48-72: round i sums, over the pairs (f0, f1), (h0, h1) of
// adjacent elements, y0 = f0 h0, y1 = f1 h1 and y2 = (2f1 - f0)(2h1 - h0),
// emits c0 = y0, c1 = (4y1 - y2 - 3y0)/2, c2 = (y2 - 2y1 + y0)/2, then folds
// both vectors to a + r_i (b - a).  Here the third sum is s = (f0 + f1)(h0 + h1)
// instead: y2 = 6y1 + 3y0 - 2s, which turns the coefficients into
// c1 = s - y1 - 3y0 and c2 = 2(y0 + y1) - s -- the same field elements with
// two field additions per pair fewer and no halving.
//
// One warp owns a chunk of 2^9 consecutive elements of f and of h: each lane
// holds 16 consecutive elements and does rounds 0-3 in registers (the sums accumulate exactly in
// Acc160 and reduce once per round); rounds 4-8 run on the 32 folded values
// per chunk staged in shared memory, one pair per thread across the block.
// The 27 per-round sums are reduced across the warp by a butterfly
// reduce-scatter and across the block's 8 warps through shared memory, so each
// block writes one row of 27 partial sums.
constexpr int kWarpRounds = 9;
constexpr int kLaneElems = 16;
constexpr int kChunkWarps = kThreads / 32;
constexpr int kRoundVals = 3 * kWarpRounds;
struct Chal {
    uint64_t r[kWarpRounds];
};

// Butterfly reduce-scatter over a warp: afterwards lane l holds the sum over
// all 32 lanes of v[l].
__device__ __forceinline__ uint64_t warp_transpose_sum(uint64_t (&v)[32]) {
    const uint32_t lane = threadIdx.x & 31;
#pragma unroll
    for (int n = 16; n >= 1; n >>= 1) {
        const bool upper = (lane & n) != 0;
#pragma unroll
        for (int i = 0; i < n; i++) {
            const uint64_t send = upper ? v[i] : v[i + n];
            const uint64_t keep = upper ? v[i + n] : v[i];
            v[i] = gl_add(keep, __shfl_xor_sync(0xffffffffu, send, n));
        }
    }
    return v[0];
}

// Chunk c of the current vectors covers elements [c*512, c*512 + 512); only
// the first n_valid elements of f and h exist, the rest read as zero.  A batch
// of tables runs as gridDim.y tables at element stride in_stride; table y
// writes its folded values at y * out_stride and its block partials after
// those of tables < y, so one reduce over all rows sums the batch.  A tail
// chunk (q < 9 rounds, one chunk) is padded that way: zero pairs add nothing
// to the sums of rounds < q, and the folded value of the real data is taken
// from lane 0 after round q - 1.  Sums of rounds >= q are never read.
template <bool kVec>
__global__ void __launch_bounds__(kThreads)
    k_sumcheck_warp(const uint64_t* __restrict__ f, const uint64_t* __restrict__ h, uint64_t n_valid, uint64_t G,
                    uint32_t q, Chal ch, uint64_t* __restrict__ partials, uint64_t* __restrict__ f_out,
                    uint64_t* __restrict__ h_out, uint64_t in_stride, uint64_t out_stride) {
    __shared__ uint64_t red[kChunkWarps][32];
    // blockIdx.y selects the table of a batch (prove_sum_of_products)
    f += blockIdx.y * in_stride;
    h += blockIdx.y * in_stride;
    f_out += blockIdx.y * out_stride;
    h_out += blockIdx.y * out_stride;
    partials += (uint64_t)blockIdx.y * gridDim.x * kRoundVals;
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint64_t chunk = (uint64_t)blockIdx.x * kChunkWarps + warp;
    uint64_t fv[kLaneElems], hv[kLaneElems], vals[32];
#pragma unroll
    for (int i = 0; i < 32; i++) vals[i] = 0;
    const uint64_t base = (chunk << kWarpRounds) + (uint64_t)lane * kLaneElems;
    if (chunk < G && kVec && base + kLaneElems <= n_valid) {
        const ulonglong2* f2 = reinterpret_cast<const ulonglong2*>(f + base);
        const ulonglong2* h2 = reinterpret_cast<const ulonglong2*>(h + base);
#pragma unroll
        for (int i = 0; i < kLaneElems / 2; i++) {
            const ulonglong2 a = __ldg(f2 + i), b = __ldg(h2 + i);
            fv[2 * i] = a.x;
            fv[2 * i + 1] = a.y;
            hv[2 * i] = b.x;
            hv[2 * i + 1] = b.y;
        }
    } else {
#pragma unroll
        for (int i = 0; i < kLaneElems; i++) {
            const bool ok = chunk < G && base + i < n_valid;
            fv[i] = ok ? __ldg(f + base + i) : 0ull;
            hv[i] = ok ? __ldg(h + base + i) : 0ull;
        }
    }
    uint64_t fin_f = 0, fin_h = 0;
    // rounds 0-3: pairs inside the lane's registers
#pragma unroll
    for (int rd = 0; rd < 4; rd++) {
        const int pairs = (kLaneElems / 2) >> rd;
        const uint64_t r = ch.r[rd];
        Acc160 a0 = acc160_zero(), a1 = acc160_zero(), as = acc160_zero();
#pragma unroll
        for (int s = 0; s < pairs; s++) {
            const uint64_t f0 = fv[2 * s], f1 = fv[2 * s + 1], h0 = hv[2 * s], h1 = hv[2 * s + 1];
            acc160_mac(a0, f0, h0);
            acc160_mac(a1, f1, h1);
            acc160_mac(as, gl_add(f0, f1), gl_add(h0, h1));
            fv[s] = gl_add(f0, gl_mul(r, gl_sub(f1, f0)));
            hv[s] = gl_add(h0, gl_mul(r, gl_sub(h1, h0)));
        }
        vals[3 * rd] = acc160_reduce(a0);
        vals[3 * rd + 1] = acc160_reduce(a1);
        vals[3 * rd + 2] = acc160_reduce(as);
        if ((uint32_t)rd + 1 == q) {
            fin_f = fv[0];
            fin_h = hv[0];
        }
    }
    // rounds 4-8 on the 32 folded values of each of the block's 8 chunks,
    // staged in shared memory: round 4 + k has 16 >> k pairs per chunk and
    // takes one pair per thread (the first 8 (16 >> k) threads), so no lane
    // computes a pair that is not there (ping-pong buffers, one barrier per
    // round)
    __shared__ uint64_t sx[2][kChunkWarps][32], sz[2][kChunkWarps][32];
    sx[0][warp][lane] = fv[0];
    sz[0][warp][lane] = hv[0];
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 5; k++) {
        const int rd = 4 + k, lp = 4 - k;  // 2^lp pairs per chunk
        const uint32_t tid = threadIdx.x;
        if (tid < ((uint32_t)kChunkWarps << lp)) {
            const uint32_t w = tid >> lp, pr = tid & ((1u << lp) - 1);
            const uint64_t x0 = sx[k & 1][w][2 * pr], x1 = sx[k & 1][w][2 * pr + 1];
            const uint64_t z0 = sz[k & 1][w][2 * pr], z1 = sz[k & 1][w][2 * pr + 1];
            vals[3 * rd] = gl_mul(x0, z0);
            vals[3 * rd + 1] = gl_mul(x1, z1);
            vals[3 * rd + 2] = gl_mul(gl_add(x0, x1), gl_add(z0, z1));
            const uint64_t r = ch.r[rd];
            sx[(k + 1) & 1][w][pr] = gl_add(x0, gl_mul(r, gl_sub(x1, x0)));
            sz[(k + 1) & 1][w][pr] = gl_add(z0, gl_mul(r, gl_sub(z1, z0)));
        }
        __syncthreads();
    }
    // after round 4 + k the chunk's folded values sit in buffer (k + 1) & 1
    if (q > 4) {
        fin_f = sx[(q - 4) & 1][warp][0];
        fin_h = sz[(q - 4) & 1][warp][0];
    }
    red[warp][lane] = warp_transpose_sum(vals);
    __syncthreads();
    if (warp == 0 && lane < kRoundVals) {
        uint64_t s = red[0][lane];
#pragma unroll
        for (int w = 1; w < kChunkWarps; w++) s = gl_add(s, red[w][lane]);
        partials[(uint64_t)blockIdx.x * kRoundVals + lane] = s;
    }
    if (lane == 0 && chunk < G) {
        f_out[chunk] = gl_canon(fin_f);
        h_out[chunk] = gl_canon(fin_h);
    }
}

// One block per round: sum (y0, y1, s) over the nb block rows of partials and
// write the round polynomial c0 = y0, c1 = s - y1 - 3y0, c2 = 2(y0 + y1) - s.
__global__ void k_sumcheck_reduce(const uint64_t* __restrict__ partials, uint64_t nb,
                                  uint64_t* __restrict__ rounds) {
    __shared__ uint64_t red[3][kThreads / 32];
    const uint32_t rd = blockIdx.x;
    uint64_t y0 = 0, y1 = 0, s = 0;
    for (uint64_t b = threadIdx.x; b < nb; b += kThreads) {
        const uint64_t* p = partials + b * kRoundVals + 3 * rd;
        y0 = gl_add(y0, __ldg(p));
        y1 = gl_add(y1, __ldg(p + 1));
        s = gl_add(s, __ldg(p + 2));
    }
    y0 = warp_sum(y0);
    y1 = warp_sum(y1);
    s = warp_sum(s);
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
        red[0][w] = y0;
        red[1][w] = y1;
        red[2][w] = s;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int i = 1; i < kThreads / 32; i++) {
            y0 = gl_add(y0, red[0][i]);
            y1 = gl_add(y1, red[1][i]);
            s = gl_add(s, red[2][i]);
        }
        const uint64_t c1 = gl_sub(gl_sub(s, y1), gl_mul(3, y0));
        const uint64_t c2 = gl_sub(gl_add(gl_add(y0, y0), gl_add(y1, y1)), s);
        uint64_t* o = rounds + 3ull * rd;
        o[0] = gl_canon(y0);
        o[1] = gl_canon(c1);
        o[2] = gl_canon(c2);
    }
}

// Field matmul C = A (m x k) @ B (k x n), the forward witness of Op::MatMul
// (zkie-ops/src/compose.rs:1327-1331; par.rs:41-89 computes the same field
// value through i64 when it cannot overflow).
// Block (32 columns x 8 k-slices): lane x owns column j of row i, warp y the
// k-slice q = y, y + 8, ...; each thread sums its products exactly (Acc160)
// and the eight slices are added through shared memory.  A warp reads 32
// consecutive entries of a row of B per q (coalesced) and one broadcast
// entry of A.
constexpr int kMmSlices = 8;
__global__ void __launch_bounds__(32 * kMmSlices)
    k_matmul_field(const uint64_t* __restrict__ a, const uint64_t* __restrict__ b, uint64_t m, uint64_t k,
                   uint64_t n, uint64_t* __restrict__ c) {
    __shared__ uint64_t red[kMmSlices][32];
    const uint64_t j = (uint64_t)blockIdx.x * 32 + threadIdx.x;
    const uint64_t i = blockIdx.y;
    const uint32_t y = threadIdx.y;
    Acc160 acc = acc160_zero();
    if (j < n) {
        const uint64_t* ar = a + i * k;
        uint64_t q = y;
        for (; q + 3 * kMmSlices < k; q += 4 * kMmSlices) {
            const uint64_t a0 = __ldg(ar + q), a1 = __ldg(ar + q + kMmSlices);
            const uint64_t a2 = __ldg(ar + q + 2 * kMmSlices), a3 = __ldg(ar + q + 3 * kMmSlices);
            const uint64_t b0 = __ldg(b + q * n + j), b1 = __ldg(b + (q + kMmSlices) * n + j);
            const uint64_t b2 = __ldg(b + (q + 2 * kMmSlices) * n + j), b3 = __ldg(b + (q + 3 * kMmSlices) * n + j);
            acc160_mac(acc, a0, b0);
            acc160_mac(acc, a1, b1);
            acc160_mac(acc, a2, b2);
            acc160_mac(acc, a3, b3);
        }
        for (; q < k; q += kMmSlices) acc160_mac(acc, __ldg(ar + q), __ldg(b + q * n + j));
    }
    red[y][threadIdx.x] = acc160_reduce(acc);
    __syncthreads();
    if (y == 0 && j < n) {
        uint64_t s = red[0][threadIdx.x];
#pragma unroll
        for (int t = 1; t < kMmSlices; t++) s = gl_add(s, red[t][threadIdx.x]);
        c[i * n + j] = gl_canon(s);
    }
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
    if (d >= 8) {
        const uint64_t nhi = 1ull << (d - 8);
        const uint64_t blocks = nhi < kEqHiPerBlock ? 1 : nhi / kEqHiPerBlock;
        if (blocks > 0x7FFFFFFFull) return (int)cudaErrorInvalidValue;
        k_eq_table_split<<<(unsigned)blocks, 256, 0, s>>>(p, d, d_out);
    } else {
        k_eq_table<<<(unsigned)ceil_div(n, kThreads), kThreads, 0, s>>>(p, d, d_out);
    }
    ZK_LAUNCH_CHECK();
    return 0;
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// X must be a power of two (the eq table of log2(X) variables).
int contract(const uint64_t* v, const uint64_t* eq, uint64_t X, uint64_t Y, uint64_t* out, cudaStream_t s) {
    if (Y == 0) return 0;
    if (X == 0 || (X & (X - 1)) || X > (1ull << 31)) return (int)cudaErrorInvalidValue;
    if (X == 1) {
        // eq of zero variables is the single value 1
        k_canon_copy<<<(unsigned)ceil_div(Y, kThreads), kThreads, 0, s>>>(v, out, Y);
        ZK_LAUNCH_CHECK();
        return 0;
    }
    const uint32_t lg_x = log2_exact(X);
    const uint32_t lg_l = lg_x - 1 < 5 ? lg_x - 1 : 5;
    const uint64_t blocks = ceil_div(Y << lg_l, kThreads);
    if (blocks > 0x7FFFFFFFull) return (int)cudaErrorInvalidValue;
    if (aligned16(v) && aligned16(eq))
        k_contract<true><<<(unsigned)blocks, kThreads, 0, s>>>(v, eq, lg_x, lg_l, Y, out);
    else
        k_contract<false><<<(unsigned)blocks, kThreads, 0, s>>>(v, eq, lg_x, lg_l, Y, out);
    ZK_LAUNCH_CHECK();
    return 0;
}

// Row blocks of the row contraction: at most 64, of at least 8 rows.
uint64_t rows_blocks(uint64_t R) {
    const uint64_t nb = ceil_div(R, 8);
    return nb < 64 ? (nb ? nb : 1) : 64;
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

constexpr uint64_t sumcheck_chunks0(uint32_t t) {
    return t > (uint32_t)kWarpRounds ? (1ull << (t - kWarpRounds)) : 2;
}

constexpr uint64_t sumcheck_batch_scratch_elems_c(uint64_t n_tables, uint32_t t) {
    // per table: two ping-pong pairs of folded vectors (<= 2^(t-9) each) and
    // one row of partial sums per block of the first level
    return n_tables * (4 * sumcheck_chunks0(t) +
                       kRoundVals * ((sumcheck_chunks0(t) + kChunkWarps - 1) / kChunkWarps)) + 64;
}

constexpr uint64_t sumcheck_scratch_elems_c(uint32_t t) { return sumcheck_batch_scratch_elems_c(1, t); }

uint64_t sumcheck_scratch_elems(uint32_t t) { return sumcheck_scratch_elems_c(t); }

// All t rounds of the degree-2 sumcheck over a batch of n tables (table i of
// f and h at element i * 2^t), nine rounds per level: each level is one
// chunk launch over every table and one reduce launch over all their block
// partials, so the round messages are those of sum_i f_i h_i.  rounds (3t)
// go to d_rounds, the folded f_i and h_i (canonical) to d_ffin[i], d_hfin[i].
int sumcheck_batch_dev(const uint64_t* d_f, const uint64_t* d_h, uint32_t n, uint32_t t, const uint64_t* h_ch,
                       uint64_t* d_rounds, uint64_t* d_ffin, uint64_t* d_hfin, uint64_t* d_scratch, cudaStream_t s) {
    if (n == 0 || n > 65535) return (int)cudaErrorInvalidValue;
    if (t == 0) {
        k_canon_copy<<<(unsigned)ceil_div(n, kThreads), kThreads, 0, s>>>(d_f, d_ffin, n);
        k_canon_copy<<<(unsigned)ceil_div(n, kThreads), kThreads, 0, s>>>(d_h, d_hfin, n);
        ZK_LAUNCH_CHECK();
        return 0;
    }
    const uint64_t chunks0 = sumcheck_chunks0(t) * n;
    uint64_t* fa = d_scratch;
    uint64_t* ha = fa + chunks0;
    uint64_t* fb = ha + chunks0;
    uint64_t* hb = fb + chunks0;
    uint64_t* partials = hb + chunks0;
    const uint64_t* cf = d_f;
    const uint64_t* chh = d_h;
    uint32_t done = 0;
    bool first = true;
    while (done < t) {
        const uint32_t rem = t - done;
        const uint32_t q = rem < (uint32_t)kWarpRounds ? rem : (uint32_t)kWarpRounds;
        const uint64_t G = 1ull << (rem - q);
        const uint64_t nb = ceil_div(G, kChunkWarps);
        if (nb > 0x7FFFFFFFull) return (int)cudaErrorInvalidValue;
        Chal ch{};
        for (uint32_t i = 0; i < q; i++) ch.r[i] = h_ch[done + i];
        const bool last = rem == q;
        uint64_t* of = last ? d_ffin : (first ? fa : (cf == fa ? fb : fa));
        uint64_t* oh = last ? d_hfin : (first ? ha : (chh == ha ? hb : ha));
        const uint64_t n_valid = 1ull << rem;
        const dim3 grid((unsigned)nb, n);
        if (aligned16(cf) && aligned16(chh))
            k_sumcheck_warp<true><<<grid, kThreads, 0, s>>>(cf, chh, n_valid, G, q, ch, partials, of, oh, n_valid, G);
        else
            k_sumcheck_warp<false><<<grid, kThreads, 0, s>>>(cf, chh, n_valid, G, q, ch, partials, of, oh, n_valid, G);
        ZK_LAUNCH_CHECK();
        k_sumcheck_reduce<<<q, kThreads, 0, s>>>(partials, nb * n, d_rounds + 3ull * done);
        ZK_LAUNCH_CHECK();
        cf = of;
        chh = oh;
        done += q;
        first = false;
    }
    return 0;
}

// sumcheck::prove on one pair: rounds (3t) and finals (f, h) in device memory.
int sumcheck_dev(const uint64_t* d_f, const uint64_t* d_h, uint32_t t, const uint64_t* h_ch,
                 uint64_t* d_rounds, uint64_t* d_finals, uint64_t* d_scratch, cudaStream_t s) {
    return sumcheck_batch_dev(d_f, d_h, 1, t, h_ch, d_rounds, d_finals, d_finals + 1, d_scratch, s);
}

// out[0] = sum_i f[i] h[i], canonical (one block).
__global__ void k_dot_small(const uint64_t* __restrict__ f, const uint64_t* __restrict__ h, uint32_t n,
                            uint64_t* __restrict__ out) {
    __shared__ uint64_t red[kThreads / 32];
    Acc160 a = acc160_zero();
    for (uint32_t i = threadIdx.x; i < n; i += kThreads) acc160_mac(a, f[i], h[i]);
    uint64_t v = warp_sum(acc160_reduce(a));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kThreads / 32; w++) v = gl_add(v, red[w]);
        out[0] = gl_canon(v);
    }
}

uint64_t sum_of_products_scratch_elems(uint32_t n, uint32_t t) {
    return sumcheck_batch_scratch_elems_c(n, t) + 3ull * t + 2ull * n + 8;
}

// prove_sum_of_products: rounds (3t) then b_eval (1) at d_out.
int sum_of_products_dev(const uint64_t* d_w, const uint64_t* d_v, uint32_t n, uint32_t t, const uint64_t* h_ch,
                        uint64_t* d_out, uint64_t* d_scratch, cudaStream_t s) {
    uint64_t* fin = d_scratch + sumcheck_batch_scratch_elems_c(n, t);
    int rc = sumcheck_batch_dev(d_w, d_v, n, t, h_ch, d_out, fin, fin + n, d_scratch, s);
    if (rc) return rc;
    k_dot_small<<<1, kThreads, 0, s>>>(fin, fin + n, n, d_out + 3ull * t);
    ZK_LAUNCH_CHECK();
    return 0;
}

int matmul_field_dev(const uint64_t* d_a, const uint64_t* d_b, uint64_t m, uint64_t k, uint64_t n,
                     uint64_t* d_c, cudaStream_t s) {
    if (m == 0 || n == 0) return 0;
    if (ceil_div(n, 32) > 0x7FFFFFFFull) return (int)cudaErrorInvalidValue;
    // grid.y holds at most 65535 rows: taller products run as row blocks
    constexpr uint64_t kRowsPerLaunch = 65535;
    for (uint64_t r0 = 0; r0 < m; r0 += kRowsPerLaunch) {
        const uint64_t rows = m - r0 < kRowsPerLaunch ? m - r0 : kRowsPerLaunch;
        const dim3 grid((unsigned)ceil_div(n, 32), (unsigned)rows), block(32, kMmSlices);
        k_matmul_field<<<grid, block, 0, s>>>(d_a + r0 * k, d_b, rows, k, n, d_c + r0 * n);
        ZK_LAUNCH_CHECK();
    }
    return 0;
}

uint64_t contract_rows_scratch_elems(uint64_t R, uint64_t K) {
    const uint64_t nb = rows_blocks(R);
    return nb > 1 ? nb * K : 0;
}

// out[c] = sum_r v[r*K + c] eq[r] for an R x K row-major v; d_part holds
// contract_rows_scratch_elems(R, K) u64.
int contract_rows_dev(const uint64_t* d_v, const uint64_t* d_eq, uint64_t R, uint64_t K, uint64_t* d_out,
                      uint64_t* d_part, cudaStream_t s) {
    if (K == 0) return 0;
    const uint64_t nb = rows_blocks(R);
    const uint64_t rpb = ceil_div(R ? R : 1, nb);
    const dim3 grid((unsigned)ceil_div(ceil_div(K, 2), kThreads), (unsigned)nb);
    uint64_t* part = nb > 1 ? d_part : d_out;
    if (nb > 1 && !d_part) return (int)cudaErrorInvalidValue;
    if (aligned16(d_v) && (K % 2) == 0)
        k_contract_rows<true><<<grid, kThreads, 0, s>>>(d_v, d_eq, R, K, rpb, part);
    else
        k_contract_rows<false><<<grid, kThreads, 0, s>>>(d_v, d_eq, R, K, rpb, part);
    ZK_LAUNCH_CHECK();
    if (nb > 1) {
        k_sum_rows<<<(unsigned)ceil_div(K, kThreads), kThreads, 0, s>>>(part, nb, K, d_out);
        ZK_LAUNCH_CHECK();
    }
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
// (about 1.9 MB) until the process exits.
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
