// virtual.cu -- the virtual-polynomial sumcheck (prove_virtual) on the device.
//
// Reference: crates/zkie-core/src/common/sumcheck.rs:378-438.  The claim is
// sum_{x in {0,1}^t} g(x) with g(x) = sum_i coeff_i * prod_{j in term_i} f_j(x)
// over n_mles multilinear tables of 2^t values.  Each round sends the d + 1
// evaluations g_round(k), k = 0..d (d = the largest term size), where over the
// pairs (f_j[2s], f_j[2s+1]) of every table f_j(k) = k f1 - (k - 1) f0, and
// then folds every table to (1 - r) f0 + r f1.
//
// As in the degree-2 sumcheck all challenges are known before proving
// (callers draw them up front: compose.rs:392, projection.rs:83), so a launch
// runs q <= 8 rounds on independent chunks of 2^q consecutive positions: one
// 128-thread block stages its chunk of every table in shared memory, runs the
// q rounds there (ping-pong buffers, one barrier per round) and writes
// per-round partial sums plus one folded value per table.  A general term
// list is split into (term, pair) work items, so the late rounds with few
// pairs still spread over the block; the term shapes of the reference's
// callers (eq times a linear combination, the logUp layer) have dedicated
// pair-at-a-time evaluations with fewer products.  A second launch sums the
// partials of all chunks.  The folded vectors (1/2^q of the input) feed the next level.
// The input tables are read from HBM exactly once.
//
// f_j(k) for k = 0..d is formed incrementally (f0, f0 + (f1 - f0), ...), the
// same field elements as k f1 - (k - 1) f0, and the last factor of every
// term product is multiplied into an exact Acc160 sum (one reduction per
// round and evaluation point instead of one per product).
#include <cuda_pipeline.h>

#include <atomic>
#include <map>
#include <mutex>

#include "../../include/zkie2.h"
#include "common.cuh"
#include "gl64.cuh"

namespace zk {

namespace {

constexpr int kVThreads = 128;
constexpr int kVMaxMles = 16;
constexpr int kVMaxTerms = 32;
constexpr int kVMaxFactors = 64;
constexpr int kVMaxDeg = 8;
constexpr int kVMaxQ = 10;
constexpr int kVQCap = 8;  // rounds per launch: 2^8 positions per 128-thread block
constexpr uint32_t kVSmemBytes = 46 * 1024;  // dynamic part; the static reduction buffer rides on top

// Term shapes with a dedicated evaluation, classified on the host:
//  kShapeGeneric  any term list; (term, pair) work items.
//  kShapeEqLinear degree 2, every term is [e, j] or [e] for one common table
//                 e (Projection affine, projection.rs:74-83): g = f_e * I with
//                 I = sum_i c_i f_{j_i} linear in k, so I is summed at k = 0, 1
//                 only and g(2) = (2 e1 - e0)(2 I1 - I0).
//  kShapeFraction the five terms of a logUp layer (logup_gkr.rs:19-28) over
//                 [eq, nn, nd, nl, nh, dl, dh]: g = eq * I with
//                 I = nn + c nd - nl dh - nh dl - c dl dh quadratic in k, so
//                 I(3) = I(0) + 3 (I(2) - I(1)).
// Both special shapes evaluate one pair per work item with every table's
// pair read once; the values equal those of the term-by-term formula.
enum : uint32_t { kShapeGeneric = 0, kShapeEqLinear = 1, kShapeFraction = 2 };

struct VTerms {
    uint64_t coeff[kVMaxTerms];
    uint8_t off[kVMaxTerms + 1];
    uint8_t idx[kVMaxFactors];
    int8_t other[kVMaxTerms];  // kShapeEqLinear: the second table of term i, -1 for [e] alone
    uint32_t n_terms, n_mles, deg, shape, common;
    // kShapeFraction over a fraction-tree layer whose next-level tables were
    // computed from its halves (nn = nl dh + nh dl, nd = dl dh at every
    // boolean point): then I = 0 at every boolean point, so in the first
    // round g(0) = g(1) = 0, I(3) = 3 I(2), and only I(2) is evaluated.
    uint32_t tree_layer;
};
struct VIn {
    const uint64_t* p[kVMaxMles];
};
struct VChal {
    uint64_t r[kVMaxQ];
};

__device__ __forceinline__ uint64_t v_warp_sum(uint64_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = gl_add(v, __shfl_down_sync(0xffffffffu, v, o));
    return v;
}

// Warp sums of V values at once (V a power of two <= 32): log2 V butterfly
// steps each hand half of the remaining values to the partner lane, the
// remaining steps reduce one value.  Afterwards lane k * (32 / V) holds the
// total of value k.  V - 1 + 5 - log2 V shuffle-adds instead of 5 V.
template <int V>
__device__ __forceinline__ uint64_t warp_multi_sum(uint64_t (&v)[V]) {
    const uint32_t lane = threadIdx.x & 31;
#pragma unroll
    for (int st = 0; st < 5; st++) {
        const int n = 16 >> st, h = (V >> st) / 2;  // values held before this step: V >> st
        if (h >= 1) {
            const bool upper = (lane & n) != 0;
#pragma unroll
            for (int i = 0; i < h; i++) {
                const uint64_t send = upper ? v[i] : v[i + h];
                const uint64_t keep = upper ? v[i + h] : v[i];
                v[i] = gl_add(keep, __shfl_xor_sync(0xffffffffu, send, n));
            }
        } else {
            v[0] = gl_add(v[0], __shfl_xor_sync(0xffffffffu, v[0], n));
        }
    }
    return v[0];
}

__host__ __device__ constexpr int pow2_ceil(int x) { return x <= 1 ? 1 : 2 * pow2_ceil((x + 1) / 2); }

// I = nn + c nd - nl dh - nh dl - c dl dh (one exact sum per sign)
__device__ __forceinline__ uint64_t frac_inner(uint64_t c, uint64_t nn, uint64_t nd, uint64_t nl, uint64_t nh,
                                               uint64_t dl, uint64_t dh) {
    Acc160 pos = acc160_zero(), neg = acc160_zero();
    acc160_mac(pos, c, nd);
    acc160_add(pos, nn);
    acc160_mac(neg, nl, dh);
    acc160_mac(neg, nh, dl);
    acc160_mac(neg, gl_mul(c, dl), dh);
    return gl_sub(acc160_reduce(pos), acc160_reduce(neg));
}

// One block per chunk of 2^q positions.  Shared memory: every table's chunk
// (n_mles x 2^q) followed by a half-size buffer (n_mles x 2^(q-1)).
// partials[(chunk * q + round) * (d + 1) + k]; out[j * out_stride + chunk] is
// the chunk's folded value of table j (canonical).
// kF bounds the factors per term (and so the degree): the kernel is
// instantiated for 2, 4 and 8 so the per-factor loops unroll to what the
// terms need.  The term tables are copied to shared memory once per block,
// where the per-pair lookups by term and factor index are cheap.
template <int kF, uint32_t kShape>
__global__ void __launch_bounds__(kVThreads)
    k_virtual_chunk(VIn in, uint32_t q, uint64_t chunks, VTerms T, VChal ch, uint64_t* __restrict__ partials,
                    uint64_t* __restrict__ out, uint64_t out_stride) {
    constexpr int kV = pow2_ceil(kF + 1);
    extern __shared__ __align__(16) uint64_t sm[];
    __shared__ uint64_t red[2][kVThreads / 32][kF + 1];
    __shared__ uint64_t s_coeff[kVMaxTerms];
    __shared__ uint32_t s_off[kVMaxTerms + 1], s_idx[kVMaxFactors];
    __shared__ int32_t s_other[kVMaxTerms];
    __shared__ uint64_t s_ch[kVMaxQ];
    const uint32_t nm = T.n_mles, deg = T.deg, nt = T.n_terms, Q = 1u << q;
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid < kVMaxTerms) {
        s_coeff[tid] = T.coeff[tid];
        s_other[tid] = T.other[tid];
    }
    if (tid <= kVMaxTerms) s_off[tid] = T.off[tid];
    if (tid < kVMaxFactors) s_idx[tid] = T.idx[tid];
    if (tid < kVMaxQ) s_ch[tid] = ch.r[tid];
    // Shared memory: two chunk buffers (nm x Q each) and one half-size
    // buffer.  The block walks chunks blockIdx.x, + gridDim.x, ...; while it
    // runs the rounds of one chunk out of one buffer (and the half buffer),
    // cp.async fills the other with the next chunk.
    uint64_t* const buf0 = sm;
    uint64_t* const buf1 = sm + (size_t)nm * Q;
    uint64_t* const half_buf = sm + 2 * (size_t)nm * Q;
    const uint64_t n_chunks = chunks;
    auto prefetch = [&](uint64_t chunk, uint64_t* dst) {
        const uint64_t base = chunk << q;
#pragma unroll
        for (uint32_t j = 0; j < (uint32_t)kVMaxMles; j++) {
            if (j >= nm) break;
            const uint64_t* src = in.p[j] + base;
            uint64_t* d = dst + (size_t)j * Q;
            if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(d)) & 15) == 0) {
                for (uint32_t i = 2 * tid; i < Q; i += 2 * kVThreads) __pipeline_memcpy_async(d + i, src + i, 16);
            } else {
                for (uint32_t i = tid; i < Q; i += kVThreads) __pipeline_memcpy_async(d + i, src + i, 8);
            }
        }
        __pipeline_commit();
    };
    const uint32_t e = T.common;
    const uint64_t fc = T.coeff[3];  // the logUp layer's c
    uint32_t which = 0;
    if ((uint64_t)blockIdx.x < n_chunks) prefetch(blockIdx.x, buf0);
    for (uint64_t chunk = blockIdx.x; chunk < n_chunks; chunk += gridDim.x) {
    const uint64_t next = chunk + gridDim.x;
    if (next < n_chunks) {
        prefetch(next, which ? buf0 : buf1);
        __pipeline_wait_prior(1);
    } else {
        __pipeline_wait_prior(0);
    }
    __syncthreads();
    uint64_t* cur = which ? buf1 : buf0;
    uint64_t* nxt = half_buf;
    uint32_t sc = Q, sn = Q >> 1;
    for (uint32_t rd = 0; rd < q; rd++) {
        const uint32_t lg_pairs = q - 1 - rd, pairs = 1u << lg_pairs;
        const uint64_t r = s_ch[rd];
        Acc160 acc[kF + 1];
#pragma unroll
        for (int k = 0; k <= kF; k++) acc[k] = acc160_zero();
        auto pair_of = [&](uint32_t j, uint32_t s) { return reinterpret_cast<const ulonglong2*>(cur + j * sc)[s]; };
        uint32_t items;
        if (kShape == kShapeEqLinear) {
            items = pairs;
            for (uint32_t s = tid; s < pairs; s += kVThreads) {
                const ulonglong2 ep = pair_of(e, s);
                Acc160 i0 = acc160_zero(), i1 = acc160_zero();
                for (uint32_t ti = 0; ti < nt; ti++) {
                    const int32_t o = s_other[ti];
                    const uint64_t c = s_coeff[ti];
                    if (o < 0) {
                        acc160_add(i0, c);
                        acc160_add(i1, c);
                    } else {
                        const ulonglong2 fp = pair_of((uint32_t)o, s);
                        acc160_mac(i0, c, fp.x);
                        acc160_mac(i1, c, fp.y);
                    }
                }
                const uint64_t a0 = acc160_reduce(i0), a1 = acc160_reduce(i1);
                acc160_mac(acc[0], ep.x, a0);
                acc160_mac(acc[1], ep.y, a1);
                acc160_mac(acc[2], gl_sub(gl_add(ep.y, ep.y), ep.x), gl_sub(gl_add(a1, a1), a0));
            }
        } else if (kShape == kShapeFraction && T.tree_layer && rd == 0) {
            items = pairs;
            for (uint32_t s = tid; s < pairs; s += kVThreads) {
                const ulonglong2 eq = pair_of(0, s), nn = pair_of(1, s), nd = pair_of(2, s), nl = pair_of(3, s),
                                 nh = pair_of(4, s), dl = pair_of(5, s), dh = pair_of(6, s);
                auto f2 = [](ulonglong2 v) { return gl_add(v.y, gl_sub(v.y, v.x)); };
                const uint64_t i2 = frac_inner(fc, f2(nn), f2(nd), f2(nl), f2(nh), f2(dl), f2(dh));
                const uint64_t de = gl_sub(eq.y, eq.x);
                const uint64_t e2 = gl_add(eq.y, de);
                acc160_mac(acc[2], e2, i2);
                acc160_mac(acc[3], gl_add(e2, de), gl_add(gl_add(i2, i2), i2));
            }
        } else if (kShape == kShapeFraction) {
            items = pairs;
            for (uint32_t s = tid; s < pairs; s += kVThreads) {
                const ulonglong2 eq = pair_of(0, s), nn = pair_of(1, s), nd = pair_of(2, s), nl = pair_of(3, s),
                                 nh = pair_of(4, s), dl = pair_of(5, s), dh = pair_of(6, s);
                const uint64_t i0 = frac_inner(fc, nn.x, nd.x, nl.x, nh.x, dl.x, dh.x);
                const uint64_t i1 = frac_inner(fc, nn.y, nd.y, nl.y, nh.y, dl.y, dh.y);
                // f(2) = f1 + (f1 - f0)
                auto f2 = [](ulonglong2 v) { return gl_add(v.y, gl_sub(v.y, v.x)); };
                const uint64_t i2 = frac_inner(fc, f2(nn), f2(nd), f2(nl), f2(nh), f2(dl), f2(dh));
                const uint64_t d21 = gl_sub(i2, i1);
                const uint64_t i3 = gl_add(i0, gl_add(gl_add(d21, d21), d21));
                const uint64_t de = gl_sub(eq.y, eq.x);
                const uint64_t e2 = gl_add(eq.y, de);
                acc160_mac(acc[0], eq.x, i0);
                acc160_mac(acc[1], eq.y, i1);
                acc160_mac(acc[2], e2, i2);
                acc160_mac(acc[3], gl_add(e2, de), i3);
            }
        } else {
            // work items (term ti, pair s), term-major: neighbouring threads take
            // neighbouring pairs of one term, so their shared-memory reads are
            // consecutive 16-byte pairs
            items = nt << lg_pairs;
            for (uint32_t it = tid; it < items; it += kVThreads) {
                const uint32_t ti = it >> lg_pairs, s = it & (pairs - 1);
                const uint32_t o0 = s_off[ti], nf = s_off[ti + 1] - o0;
                const uint64_t c = s_coeff[ti];
                uint64_t fv[kF], dv[kF];
#pragma unroll
                for (int f = 0; f < kF; f++) {
                    fv[f] = 1;
                    dv[f] = 0;
                    if ((uint32_t)f < nf) {
                        const ulonglong2 pr = pair_of(s_idx[o0 + f], s);
                        fv[f] = pr.x;
                        dv[f] = gl_sub(pr.y, pr.x);
                    }
                }
#pragma unroll
                for (int k = 0; k <= kF; k++) {
                    if ((uint32_t)k <= deg) {
                        // c * prod_{f < nf} f_f(k): all but the last factor reduced,
                        // the last one multiplied into the exact sum
                        uint64_t p = c, last = 1;
#pragma unroll
                        for (int f = 0; f < kF; f++) {
                            if ((uint32_t)f + 1 < nf) p = gl_mul(p, fv[f]);
                            else if ((uint32_t)f + 1 == nf) last = fv[f];
                        }
                        acc160_mac(acc[k], p, last);
                        if ((uint32_t)k < deg) {
#pragma unroll
                            for (int f = 0; f < kF; f++)
                                if ((uint32_t)f < nf) fv[f] = gl_add(fv[f], dv[f]);
                        }
                    }
                }
            }
        }
        // fold items (table j, pair s)
        const uint32_t fitems = nm << lg_pairs;
        for (uint32_t it = tid; it < fitems; it += kVThreads) {
            const uint32_t j = it >> lg_pairs, s = it & (pairs - 1);
            const ulonglong2 pr = pair_of(j, s);
            nxt[j * sn + s] = gl_add(pr.x, gl_mul(r, gl_sub(pr.y, pr.x)));
        }
        if (warp * 32 < items) {  // warp-uniform: warps past the last item hold zeros
            uint64_t v[kV];
#pragma unroll
            for (int k = 0; k < kV; k++) v[k] = (k <= kF && (uint32_t)k <= deg) ? acc160_reduce(acc[k < kF + 1 ? k : 0]) : 0;
            const uint64_t tot = warp_multi_sum<kV>(v);
            const uint32_t k = lane / (32 / kV);
            if (lane % (32 / kV) == 0 && k <= deg) red[rd & 1][warp][k] = tot;
        }
        __syncthreads();
        if (tid <= deg) {
            const uint32_t nw = items >= (uint32_t)kVThreads ? kVThreads / 32 : (items + 31) / 32;
            uint64_t v = 0;  // no terms: every round sends zeros
            for (uint32_t w = 0; w < nw; w++) v = gl_add(v, red[rd & 1][w][tid]);
            partials[(chunk * q + rd) * (deg + 1) + tid] = v;
        }
        uint64_t* t = cur;
        cur = nxt;
        nxt = t;
        const uint32_t ts = sc;
        sc = sn;
        sn = ts;
    }
    if (tid < nm) out[tid * out_stride + chunk] = gl_canon(cur[(size_t)tid * sc]);
    __syncthreads();  // the buffers are reused by the next chunk
    which ^= 1;
    }
}

// rounds[rd * (d + 1) + k] = sum over the G chunks of their partial sums.
// One block per (round, k).
__global__ void k_virtual_reduce(const uint64_t* __restrict__ partials, uint64_t G, uint32_t q, uint32_t deg,
                                 uint64_t* __restrict__ rounds) {
    __shared__ uint64_t red[kVThreads / 32];
    const uint32_t rd = blockIdx.x / (deg + 1), k = blockIdx.x % (deg + 1);
    uint64_t v = 0;
    for (uint64_t g = threadIdx.x; g < G; g += kVThreads) v = gl_add(v, __ldg(partials + (g * q + rd) * (deg + 1) + k));
    v = v_warp_sum(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kVThreads / 32; w++) v = gl_add(v, red[w]);
        rounds[rd * (deg + 1) + k] = gl_canon(v);
    }
}

// First stage of the round sums for many chunks: block b sums a contiguous
// run of chunks for every (round, k) slot (S = q (d + 1) slots per chunk,
// consecutive threads reading consecutive slots) and writes one row of S
// sums in the partials layout, so k_virtual_reduce finishes over the blocks.
constexpr uint32_t kVRedBlocks = 296;
constexpr uint32_t kVRedThreads = 256;
constexpr uint64_t kVRedMinChunks = 2048;
__global__ void __launch_bounds__(kVRedThreads)
    k_virtual_reduce_blocks(const uint64_t* __restrict__ partials, uint64_t G, uint32_t S,
                            uint64_t* __restrict__ block_out) {
    __shared__ uint64_t red[kVRedThreads];
    const uint32_t t = threadIdx.x, groups = kVRedThreads / S, slot = t % S, grp = t / S;
    const uint64_t per = (G + gridDim.x - 1) / gridDim.x;
    const uint64_t c0 = (uint64_t)blockIdx.x * per, c1 = c0 + per < G ? c0 + per : G;
    uint64_t v = 0;
    if (grp < groups)
        for (uint64_t c = c0 + grp; c < c1; c += groups) v = gl_add(v, __ldg(partials + c * S + slot));
    red[t] = v;
    __syncthreads();
    if (t < S) {
        for (uint32_t g = 1; g < groups; g++) v = gl_add(v, red[t + g * S]);
        block_out[(uint64_t)blockIdx.x * S + t] = v;
    }
}

__global__ void k_virtual_t0(VIn in, uint32_t nm, uint64_t* __restrict__ out) {
    const uint32_t j = threadIdx.x;
    if (j < nm) out[j] = gl_canon(in.p[j][0]);
}

// The early rounds of a large set of tables, one launch per round: thread s
// evaluates pair s of every table straight from HBM (16-byte loads, pair s
// of table j at p_j[2s], p_j[2s + 1]), adds its share of the round message
// and writes the pair's folded value of every table; each block writes one
// partial per evaluation point.  Every thread has a pair, so these rounds
// stream at memory speed, where the chunk kernel's later in-chunk rounds
// leave most of a block idle.  The per-pair values are the chunk kernel's.
constexpr int kSThreads = 256;
constexpr uint32_t kStreamMinVars = 16;  // rounds over more than 2^16 positions stream
constexpr unsigned kSMaxBlocks = 148 * 8;

template <int kF, uint32_t kShape>
__global__ void __launch_bounds__(kSThreads)
    k_virtual_stream(VIn in, uint64_t pairs, VTerms T, uint64_t r, uint64_t* __restrict__ partials,
                     uint64_t* __restrict__ out) {
    constexpr int kV = pow2_ceil(kF + 1);
    __shared__ uint64_t red[kSThreads / 32][kF + 1];
    __shared__ const uint64_t* s_p[kVMaxMles];
    __shared__ uint64_t s_coeff[kVMaxTerms];
    __shared__ uint32_t s_off[kVMaxTerms + 1], s_idx[kVMaxFactors];
    __shared__ int32_t s_other[kVMaxTerms];
    const uint32_t nm = T.n_mles, deg = T.deg, nt = T.n_terms;
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid < kVMaxMles) s_p[tid] = in.p[tid];
    if (tid < kVMaxTerms) {
        s_coeff[tid] = T.coeff[tid];
        s_other[tid] = T.other[tid];
    }
    if (tid <= kVMaxTerms) s_off[tid] = T.off[tid];
    if (tid < kVMaxFactors) s_idx[tid] = T.idx[tid];
    __syncthreads();
    Acc160 acc[kF + 1];
#pragma unroll
    for (int k = 0; k <= kF; k++) acc[k] = acc160_zero();
    const uint64_t fc = T.coeff[3];
    const bool tree0 = kShape == kShapeFraction && T.tree_layer;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t s = (uint64_t)blockIdx.x * blockDim.x + tid; s < pairs; s += stride) {
        auto pr = [&](uint32_t j) { return __ldg(reinterpret_cast<const ulonglong2*>(s_p[j]) + s); };
        if (kShape == kShapeFraction) {
            const ulonglong2 eq = pr(0), nn = pr(1), nd = pr(2), nl = pr(3), nh = pr(4), dl = pr(5), dh = pr(6);
            auto f2 = [](ulonglong2 v) { return gl_add(v.y, gl_sub(v.y, v.x)); };
            const uint64_t i2 = frac_inner(fc, f2(nn), f2(nd), f2(nl), f2(nh), f2(dl), f2(dh));
            const uint64_t de = gl_sub(eq.y, eq.x);
            const uint64_t e2 = gl_add(eq.y, de);
            if (tree0) {
                acc160_mac(acc[2], e2, i2);
                acc160_mac(acc[3], gl_add(e2, de), gl_add(gl_add(i2, i2), i2));
            } else {
                const uint64_t i0 = frac_inner(fc, nn.x, nd.x, nl.x, nh.x, dl.x, dh.x);
                const uint64_t i1 = frac_inner(fc, nn.y, nd.y, nl.y, nh.y, dl.y, dh.y);
                const uint64_t d21 = gl_sub(i2, i1);
                const uint64_t i3 = gl_add(i0, gl_add(gl_add(d21, d21), d21));
                acc160_mac(acc[0], eq.x, i0);
                acc160_mac(acc[1], eq.y, i1);
                acc160_mac(acc[2], e2, i2);
                acc160_mac(acc[3], gl_add(e2, de), i3);
            }
        } else if (kShape == kShapeEqLinear) {
            const ulonglong2 ep = pr(T.common);
            Acc160 i0 = acc160_zero(), i1 = acc160_zero();
            for (uint32_t ti = 0; ti < nt; ti++) {
                const int32_t o = s_other[ti];
                const uint64_t c = s_coeff[ti];
                if (o < 0) {
                    acc160_add(i0, c);
                    acc160_add(i1, c);
                } else {
                    const ulonglong2 fp = pr((uint32_t)o);
                    acc160_mac(i0, c, fp.x);
                    acc160_mac(i1, c, fp.y);
                }
            }
            const uint64_t a0 = acc160_reduce(i0), a1 = acc160_reduce(i1);
            acc160_mac(acc[0], ep.x, a0);
            acc160_mac(acc[1], ep.y, a1);
            acc160_mac(acc[2], gl_sub(gl_add(ep.y, ep.y), ep.x), gl_sub(gl_add(a1, a1), a0));
        } else {
            for (uint32_t ti = 0; ti < nt; ti++) {
                const uint32_t o0 = s_off[ti], nf = s_off[ti + 1] - o0;
                const uint64_t c = s_coeff[ti];
                uint64_t fv[kF], dv[kF];
#pragma unroll
                for (int f = 0; f < kF; f++) {
                    fv[f] = 1;
                    dv[f] = 0;
                    if ((uint32_t)f < nf) {
                        const ulonglong2 pp = pr(s_idx[o0 + f]);
                        fv[f] = pp.x;
                        dv[f] = gl_sub(pp.y, pp.x);
                    }
                }
#pragma unroll
                for (int k = 0; k <= kF; k++) {
                    if ((uint32_t)k <= deg) {
                        uint64_t p = c, last = 1;
#pragma unroll
                        for (int f = 0; f < kF; f++) {
                            if ((uint32_t)f + 1 < nf) p = gl_mul(p, fv[f]);
                            else if ((uint32_t)f + 1 == nf) last = fv[f];
                        }
                        acc160_mac(acc[k], p, last);
                        if ((uint32_t)k < deg) {
#pragma unroll
                            for (int f = 0; f < kF; f++)
                                if ((uint32_t)f < nf) fv[f] = gl_add(fv[f], dv[f]);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (uint32_t j = 0; j < (uint32_t)kVMaxMles; j++) {
            if (j >= nm) break;
            const ulonglong2 pp = pr(j);
            out[(uint64_t)j * pairs + s] = gl_canon(gl_add(pp.x, gl_mul(r, gl_sub(pp.y, pp.x))));
        }
    }
    uint64_t v[kV];
#pragma unroll
    for (int k = 0; k < kV; k++) v[k] = (k <= kF && (uint32_t)k <= deg) ? acc160_reduce(acc[k < kF + 1 ? k : 0]) : 0;
    const uint64_t tot = warp_multi_sum<kV>(v);
    const uint32_t kk = lane / (32 / kV);
    if (lane % (32 / kV) == 0 && kk <= deg) red[warp][kk] = tot;
    __syncthreads();
    if (tid <= deg) {
        uint64_t a = 0;
        for (int w = 0; w < kSThreads / 32; w++) a = gl_add(a, red[w][tid]);
        partials[(uint64_t)blockIdx.x * (deg + 1) + tid] = a;
    }
}

// One wave of resident blocks of a streaming kernel (queried once per device).
template <int kF, uint32_t kShape>
unsigned s_wave() {
    static std::atomic<unsigned> wave[kMaxDevices];
    const int d = current_device();
    if (d < 0 || d >= kMaxDevices) return kSMaxBlocks;
    unsigned w = wave[d].load(std::memory_order_relaxed);
    if (!w) {
        int per_sm = 0, sms = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_virtual_stream<kF, kShape>, kSThreads, 0) !=
                cudaSuccess ||
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, d) != cudaSuccess)
            return kSMaxBlocks;
        w = (unsigned)((per_sm > 0 ? per_sm : 1) * (sms > 0 ? sms : 1));
        w = w < kSMaxBlocks ? w : kSMaxBlocks;
        wave[d].store(w, std::memory_order_relaxed);
    }
    return w;
}

template <int kF, uint32_t kShape>
int s_launch(uint64_t pairs, cudaStream_t s, const VIn& in, const VTerms& T, uint64_t r, uint64_t* partials,
             uint64_t* out, unsigned* grid_out) {
    const uint64_t want = (pairs + kSThreads - 1) / kSThreads;
    const unsigned wave = s_wave<kF, kShape>();
    const unsigned grid = (unsigned)(want < wave ? want : wave);
    k_virtual_stream<kF, kShape><<<grid, kSThreads, 0, s>>>(in, pairs, T, r, partials, out);
    *grid_out = grid;
    ZK_LAUNCH_CHECK();
    return 0;
}

// Rounds per launch for n_mles tables: two chunk buffers and a half-size
// ping-pong buffer (20 bytes per table per position) fit in 46 KB of dynamic
// shared memory (under the 48 KB default limit together with the static part).
uint32_t v_qmax(uint32_t nm) {
    uint32_t q = 1;
    while (q < (uint32_t)kVQCap && 20ull * nm * (2ull << q) <= kVSmemBytes) q++;
    return q;
}

struct VPlan {
    uint64_t g1;            // chunks of the first chunk level (= folded length it leaves)
    uint32_t q1;            // rounds of the first chunk level
    uint64_t stream_elems;  // the streaming rounds' two folded buffers and partials (0: none)
    uint64_t elems;         // scratch u64
};

// The scratch: the streaming region (when t > kStreamMinVars: folded
// buffers of nm x 2^(t-1) and nm x 2^(t-2), then kSMaxBlocks partials per
// evaluation point), then the chunk region, sized for t (it also serves the
// fallback without streaming).
VPlan v_plan(uint32_t nm, uint32_t t) {
    VPlan p{};
    const uint32_t qm = v_qmax(nm);
    p.q1 = t < qm ? t : qm;
    p.g1 = 1ull << (t - p.q1);
    if (t > kStreamMinVars)
        p.stream_elems = (uint64_t)nm * (3ull << (t - 2)) + (uint64_t)kSMaxBlocks * (kVMaxDeg + 1) + 8;
    // two folded buffers (nm x g1, 16-byte aligned) + the first level's partials
    // + the first reduce stage's block sums
    p.elems = p.stream_elems + 2 * ((nm * p.g1 + 1) & ~1ull) + p.g1 * (p.q1 ? p.q1 : 1) * (kVMaxDeg + 1) + 8 +
              (uint64_t)kVRedBlocks * kVMaxQ * (kVMaxDeg + 1);
    return p;
}

}  // namespace

// Launch of one chunk-kernel instantiation; the first launch on each device
// asks for the largest shared-memory carveout (more resident blocks: a block
// stages 12 bytes per table and position, e.g. 21 KB for seven tables).
// The grid is one wave of resident blocks (the occupancy of this shared
// memory size, queried once per device and size), each walking its chunks.
template <int kF, uint32_t kShape>
int v_launch(unsigned G, size_t smem, cudaStream_t s, const VIn& in, uint32_t q, const VTerms& T, const VChal& ch,
             uint64_t* partials, uint64_t* out, uint64_t out_stride) {
    static std::atomic<bool> carved[kMaxDevices];
    static std::mutex mu;
    static std::map<std::pair<int, size_t>, unsigned> waves;
    const int d = current_device();
    if (d >= 0 && d < kMaxDevices && !carved[d].load(std::memory_order_relaxed)) {
        ZK_TRY(cudaFuncSetAttribute(k_virtual_chunk<kF, kShape>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                    (int)cudaSharedmemCarveoutMaxShared));
        carved[d].store(true, std::memory_order_relaxed);
    }
    unsigned wave = 0;
    {
        std::lock_guard<std::mutex> g(mu);
        auto it = waves.find({d, smem});
        if (it == waves.end()) {
            int per_sm = 0, sms = 0;
            ZK_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_virtual_chunk<kF, kShape>, kVThreads,
                                                                 smem));
            ZK_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, d));
            wave = (unsigned)((per_sm > 0 ? per_sm : 1) * (sms > 0 ? sms : 1));
            waves[{d, smem}] = wave;
        } else {
            wave = it->second;
        }
    }
    const unsigned grid = G < wave ? G : wave;
    k_virtual_chunk<kF, kShape><<<grid, kVThreads, smem, s>>>(in, q, G, T, ch, partials, out, out_stride);
    ZK_LAUNCH_CHECK();
    return 0;
}

// Picks the term shape's evaluation (see kShapeGeneric ...).  T's
// coefficients are canonical.
void v_classify(VTerms& T) {
    T.shape = kShapeGeneric;
    T.common = 0;
    for (int i = 0; i < kVMaxTerms; i++) T.other[i] = -1;
    const uint32_t nt = T.n_terms;
    // logUp layer: [eq, nn, nd, nl, nh, dl, dh] with terms 1*[0,1], -1*[0,3,6],
    // -1*[0,4,5], c*[0,2], -c*[0,5,6]
    static const uint8_t kFracOff[6] = {0, 2, 5, 8, 10, 13};
    static const uint8_t kFracIdx[13] = {0, 1, 0, 3, 6, 0, 4, 5, 0, 2, 0, 5, 6};
    if (T.n_mles == 7 && nt == 5 && T.deg == 3) {
        bool same = true;
        for (int i = 0; i < 6; i++) same = same && T.off[i] == kFracOff[i];
        for (int i = 0; same && i < 13; i++) same = same && T.idx[i] == kFracIdx[i];
        const uint64_t c = T.coeff[3];
        if (same && T.coeff[0] == 1 && T.coeff[1] == GL_P - 1 && T.coeff[2] == GL_P - 1 &&
            T.coeff[4] == (c ? GL_P - c : 0)) {
            T.shape = kShapeFraction;
            return;
        }
    }
    // f_e times a linear combination: every term [e, j], [j, e] or [e]
    if (T.deg != 2 || nt == 0) return;
    const uint32_t o0 = T.off[0], n0 = T.off[1] - o0;
    for (uint32_t cand = 0; cand < n0; cand++) {
        const uint32_t e = T.idx[o0 + cand];
        bool ok = true;
        for (uint32_t i = 0; ok && i < nt; i++) {
            const uint32_t o = T.off[i], nf = T.off[i + 1] - o;
            if (nf == 1 && T.idx[o] == e)
                T.other[i] = -1;
            else if (nf == 2 && T.idx[o] == e)
                T.other[i] = (int8_t)T.idx[o + 1];
            else if (nf == 2 && T.idx[o + 1] == e)
                T.other[i] = (int8_t)T.idx[o];
            else
                ok = false;
        }
        if (ok) {
            T.shape = kShapeEqLinear;
            T.common = e;
            return;
        }
    }
    for (int i = 0; i < kVMaxTerms; i++) T.other[i] = -1;
}

// All t rounds on the device; rounds (t x (d+1)) and finals (n_mles) go to
// device memory.
int virtual_dev(const uint64_t* const* d_mles, uint32_t nm, uint32_t t, const VTerms& T, const uint64_t* h_ch,
                uint64_t* d_rounds, uint64_t* d_finals, uint64_t* d_scratch, cudaStream_t s) {
    VIn in{};
    for (uint32_t j = 0; j < nm; j++) in.p[j] = d_mles[j];
    if (t == 0) {
        k_virtual_t0<<<1, 32, 0, s>>>(in, nm, d_finals);
        ZK_LAUNCH_CHECK();
        return 0;
    }
    const VPlan plan = v_plan(nm, t);
    const uint32_t qm = v_qmax(nm);
    uint32_t done = 0;
    // the streaming rounds (16-byte aligned tables only)
    bool aligned = true;
    for (uint32_t j = 0; j < nm; j++) aligned = aligned && (reinterpret_cast<uintptr_t>(in.p[j]) & 15) == 0;
    if (plan.stream_elems && aligned) {
        uint64_t* sbuf[2] = {d_scratch, d_scratch + (uint64_t)nm * (1ull << (t - 1))};
        uint64_t* spart = d_scratch + (uint64_t)nm * (3ull << (t - 2));
        uint32_t sw = 0;
        while (t - done > kStreamMinVars) {
            const uint64_t pairs = 1ull << (t - done - 1);
            VTerms Tl = T;
            Tl.tree_layer = T.tree_layer && done == 0;
            uint64_t* out = sbuf[sw];
            const uint64_t r = h_ch[done];
            unsigned grid = 0;
            int rc;
            if (T.shape == kShapeEqLinear)
                rc = s_launch<2, kShapeEqLinear>(pairs, s, in, Tl, r, spart, out, &grid);
            else if (T.shape == kShapeFraction)
                rc = s_launch<3, kShapeFraction>(pairs, s, in, Tl, r, spart, out, &grid);
            else if (T.deg <= 2)
                rc = s_launch<2, kShapeGeneric>(pairs, s, in, Tl, r, spart, out, &grid);
            else if (T.deg <= 4)
                rc = s_launch<4, kShapeGeneric>(pairs, s, in, Tl, r, spart, out, &grid);
            else
                rc = s_launch<8, kShapeGeneric>(pairs, s, in, Tl, r, spart, out, &grid);
            if (rc) return rc;
            k_virtual_reduce<<<T.deg + 1, kVThreads, 0, s>>>(spart, grid, 1, T.deg,
                                                             d_rounds + (uint64_t)done * (T.deg + 1));
            ZK_LAUNCH_CHECK();
            for (uint32_t j = 0; j < nm; j++) in.p[j] = out + j * pairs;
            sw ^= 1;
            done++;
        }
    }
    uint64_t* const chunk_base = d_scratch + plan.stream_elems;
    const uint64_t bufsz = (nm * plan.g1 + 1) & ~1ull;
    uint64_t* buf[2] = {chunk_base, chunk_base + bufsz};
    uint64_t* partials = chunk_base + 2 * bufsz;
    uint64_t* block_sums = partials + plan.g1 * (plan.q1 ? plan.q1 : 1) * (kVMaxDeg + 1) + 8;
    uint32_t which = 0;
    while (done < t) {
        const uint32_t rem = t - done;
        const uint32_t q = rem < qm ? rem : qm;
        const uint64_t G = 1ull << (rem - q);
        if (G > 0x7FFFFFFFull) return (int)cudaErrorInvalidValue;
        VChal ch{};
        for (uint32_t i = 0; i < q; i++) ch.r[i] = h_ch[done + i];
        VTerms Tl = T;
        Tl.tree_layer = T.tree_layer && done == 0;
        const bool last = rem == q;
        uint64_t* out = last ? d_finals : buf[which];
        const uint64_t out_stride = last ? 1 : G;
        const size_t smem = ((size_t)20 * nm) << q;  // nm x (2 x 2^q + 2^(q-1)) u64
        int rc;
        if (T.shape == kShapeEqLinear)
            rc = v_launch<2, kShapeEqLinear>((unsigned)G, smem, s, in, q, Tl, ch, partials, out, out_stride);
        else if (T.shape == kShapeFraction)
            rc = v_launch<3, kShapeFraction>((unsigned)G, smem, s, in, q, Tl, ch, partials, out, out_stride);
        else if (T.deg <= 2)
            rc = v_launch<2, kShapeGeneric>((unsigned)G, smem, s, in, q, Tl, ch, partials, out, out_stride);
        else if (T.deg <= 4)
            rc = v_launch<4, kShapeGeneric>((unsigned)G, smem, s, in, q, Tl, ch, partials, out, out_stride);
        else
            rc = v_launch<8, kShapeGeneric>((unsigned)G, smem, s, in, q, Tl, ch, partials, out, out_stride);
        if (rc) return rc;
        ZK_LAUNCH_CHECK();
        uint64_t* rounds = d_rounds + (uint64_t)done * (T.deg + 1);
        if (G >= kVRedMinChunks) {
            k_virtual_reduce_blocks<<<kVRedBlocks, kVRedThreads, 0, s>>>(partials, G, q * (T.deg + 1), block_sums);
            ZK_LAUNCH_CHECK();
            k_virtual_reduce<<<q * (T.deg + 1), kVThreads, 0, s>>>(block_sums, kVRedBlocks, q, T.deg, rounds);
        } else {
            k_virtual_reduce<<<q * (T.deg + 1), kVThreads, 0, s>>>(partials, G, q, T.deg, rounds);
        }
        ZK_LAUNCH_CHECK();
        if (!last) {
            for (uint32_t j = 0; j < nm; j++) in.p[j] = out + j * G;
            which ^= 1;
        }
        done += q;
    }
    return 0;
}

uint64_t virtual_plan_elems(uint32_t n_mles, uint32_t t) {
    if (n_mles == 0 || n_mles > (uint32_t)kVMaxMles || t > 40) return 0;
    return v_plan(n_mles, t).elems;
}

// Term-list validation plus all launches, no synchronization: the round
// messages (t x (d + 1), d = the largest term) land in d_rounds and the
// finals (n_mles) in d_finals, both device memory outside d_scratch.
int virtual_enqueue(const uint64_t* const* d_mles, uint32_t n_mles, uint32_t t, const uint64_t* coeffs,
                    const uint32_t* idx_off, const uint32_t* idx, uint32_t n_terms, const uint64_t* h_ch,
                    uint64_t* d_rounds, uint64_t* d_finals, uint32_t* deg_out, uint64_t* d_scratch,
                    cudaStream_t stream, bool tree_layer) {
    if (!d_mles || !d_finals || !d_scratch || n_mles == 0 || n_mles > (uint32_t)kVMaxMles || t > 40 ||
        n_terms > (uint32_t)kVMaxTerms || (n_terms && (!coeffs || !idx_off)) || (t && (!h_ch || !d_rounds)))
        return (int)cudaErrorInvalidValue;
    VTerms T{};
    T.n_terms = n_terms;
    T.n_mles = n_mles;
    uint32_t deg = 0;
    if (n_terms) {
        if (idx_off[0] != 0 || idx_off[n_terms] > (uint32_t)kVMaxFactors || (idx_off[n_terms] && !idx))
            return (int)cudaErrorInvalidValue;
        for (uint32_t i = 0; i < n_terms; i++) {
            if (idx_off[i + 1] < idx_off[i]) return (int)cudaErrorInvalidValue;
            const uint32_t nf = idx_off[i + 1] - idx_off[i];
            if (nf > (uint32_t)kVMaxDeg) return (int)cudaErrorInvalidValue;
            deg = nf > deg ? nf : deg;
            T.coeff[i] = gl_canon(coeffs[i]);
            T.off[i] = (uint8_t)idx_off[i];
        }
        T.off[n_terms] = (uint8_t)idx_off[n_terms];
        for (uint32_t q = 0; q < idx_off[n_terms]; q++) {
            if (idx[q] >= n_mles) return (int)cudaErrorInvalidValue;
            T.idx[q] = (uint8_t)idx[q];
        }
    }
    T.deg = deg;
    v_classify(T);
    T.tree_layer = tree_layer && T.shape == kShapeFraction;
    for (uint32_t j = 0; j < n_mles; j++)
        if (!d_mles[j]) return (int)cudaErrorInvalidValue;
    if (deg_out) *deg_out = deg;
    return virtual_dev(d_mles, n_mles, t, T, h_ch, d_rounds, d_finals, d_scratch, stream);
}

}  // namespace zk

using namespace zk;

extern "C" {

// plan scratch, then the round messages (t x at most kVMaxDeg + 1) and the finals
uint64_t zkie2_virtual_scratch_elems(uint32_t n_mles, uint32_t t) {
    if (n_mles == 0 || n_mles > (uint32_t)kVMaxMles || t > 40) return 0;
    return v_plan(n_mles, t).elems + (uint64_t)t * (kVMaxDeg + 1) + kVMaxMles;
}

int zkie2_virtual_prove(const uint64_t* const* d_mles, uint32_t n_mles, uint32_t t, const uint64_t* coeffs,
                        const uint32_t* idx_off, const uint32_t* idx, uint32_t n_terms, const uint64_t* h_ch,
                        uint64_t* h_rounds, uint64_t* h_finals, uint64_t* d_scratch, cudaStream_t stream) {
    if (!h_finals || !d_scratch || n_mles == 0 || n_mles > (uint32_t)kVMaxMles || t > 40 || (t && !h_rounds))
        return (int)cudaErrorInvalidValue;
    // the round messages and the finals live behind the plan's scratch
    uint64_t* d_rounds = d_scratch + v_plan(n_mles, t).elems;
    uint64_t* d_finals = d_rounds + (uint64_t)t * (kVMaxDeg + 1);
    uint32_t deg = 0;
    int rc = virtual_enqueue(d_mles, n_mles, t, coeffs, idx_off, idx, n_terms, h_ch, d_rounds, d_finals, &deg,
                             d_scratch, stream, false);
    if (rc) return rc;
    if (t) ZK_TRY(cudaMemcpyAsync(h_rounds, d_rounds, 8ull * t * (deg + 1), cudaMemcpyDeviceToHost, stream));
    ZK_TRY(cudaMemcpyAsync(h_finals, d_finals, 8ull * n_mles, cudaMemcpyDeviceToHost, stream));
    ZK_TRY(cudaStreamSynchronize(stream));
    return 0;
}

// prove_virtual with device outputs and no synchronization: rounds (t x
// (d + 1), d the largest term) into d_rounds, the n_mles finals into d_finals.
int zkie2_virtual_prove_async(const uint64_t* const* d_mles, uint32_t n_mles, uint32_t t, const uint64_t* coeffs,
                              const uint32_t* idx_off, const uint32_t* idx, uint32_t n_terms, const uint64_t* h_ch,
                              uint64_t* d_rounds, uint64_t* d_finals, uint64_t* d_scratch, cudaStream_t stream) {
    return virtual_enqueue(d_mles, n_mles, t, coeffs, idx_off, idx, n_terms, h_ch, d_rounds, d_finals, nullptr,
                           d_scratch, stream, false);
}

}  // extern "C"
