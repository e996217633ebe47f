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
// per-round partial sums plus one folded value per table.  A round is split
// into (term, pair) work items rather than pairs, so the late rounds with few
// pairs still spread over the block.  A second launch sums the partials of
// all chunks.  The folded vectors (1/2^q of the input) feed the next level.
// The input tables are read from HBM exactly once.
//
// f_j(k) for k = 0..d is formed incrementally (f0, f0 + (f1 - f0), ...), the
// same field elements as k f1 - (k - 1) f0, and the last factor of every
// term product is multiplied into an exact Acc160 sum (one reduction per
// round and evaluation point instead of one per product).
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

struct VTerms {
    uint64_t coeff[kVMaxTerms];
    uint8_t off[kVMaxTerms + 1];
    uint8_t idx[kVMaxFactors];
    uint32_t n_terms, n_mles, deg;
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

// One block per chunk of 2^q positions.  Shared memory: every table's chunk
// (n_mles x 2^q) followed by a half-size buffer (n_mles x 2^(q-1)).
// partials[(chunk * q + round) * (d + 1) + k]; out[j * out_stride + chunk] is
// the chunk's folded value of table j (canonical).
// kF bounds the factors per term (and so the degree): the kernel is
// instantiated for 2, 4 and 8 so the per-factor loops unroll to what the
// terms need.  The term tables are copied to shared memory once per block,
// where the per-pair lookups by term and factor index are cheap.
template <int kF>
__global__ void __launch_bounds__(kVThreads)
    k_virtual_chunk(VIn in, uint32_t q, VTerms T, VChal ch, uint64_t* __restrict__ partials,
                    uint64_t* __restrict__ out, uint64_t out_stride) {
    extern __shared__ __align__(16) uint64_t sm[];
    __shared__ uint64_t red[2][kVThreads / 32][kF + 1];
    __shared__ uint64_t s_coeff[kVMaxTerms];
    __shared__ uint32_t s_off[kVMaxTerms + 1], s_idx[kVMaxFactors];
    __shared__ uint64_t s_ch[kVMaxQ];
    const uint32_t nm = T.n_mles, deg = T.deg, nt = T.n_terms, Q = 1u << q;
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid < kVMaxTerms) s_coeff[tid] = T.coeff[tid];
    if (tid <= kVMaxTerms) s_off[tid] = T.off[tid];
    if (tid < kVMaxFactors) s_idx[tid] = T.idx[tid];
    if (tid < kVMaxQ) s_ch[tid] = ch.r[tid];
    const uint64_t base = (uint64_t)blockIdx.x << q;
#pragma unroll
    for (int j = 0; j < kVMaxMles; j++) {
        if ((uint32_t)j < nm) {
            const uint64_t* src = in.p[j] + base;
            for (uint32_t i = tid; i < Q; i += kVThreads) sm[j * Q + i] = __ldg(src + i);
        }
    }
    __syncthreads();
    uint64_t* cur = sm;
    uint64_t* nxt = sm + (size_t)nm * Q;
    uint32_t sc = Q, sn = Q >> 1;
    for (uint32_t rd = 0; rd < q; rd++) {
        const uint32_t lg_pairs = q - 1 - rd, pairs = 1u << lg_pairs;
        const uint64_t r = s_ch[rd];
        Acc160 acc[kF + 1];
#pragma unroll
        for (int k = 0; k <= kF; k++) acc[k] = acc160_zero();
        // work items (term ti, pair s), term-major: neighbouring threads take
        // neighbouring pairs of one term, so their shared-memory reads are
        // consecutive 16-byte pairs
        const uint32_t items = nt << lg_pairs;
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
                    const ulonglong2 pr = reinterpret_cast<const ulonglong2*>(cur + s_idx[o0 + f] * sc)[s];
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
        // fold items (table j, pair s)
        const uint32_t fitems = nm << lg_pairs;
        for (uint32_t it = tid; it < fitems; it += kVThreads) {
            const uint32_t j = it >> lg_pairs, s = it & (pairs - 1);
            const ulonglong2 pr = reinterpret_cast<const ulonglong2*>(cur + j * sc)[s];
            nxt[j * sn + s] = gl_add(pr.x, gl_mul(r, gl_sub(pr.y, pr.x)));
        }
        if (warp * 32 < items) {  // warp-uniform: warps past the last item hold zeros
#pragma unroll
            for (int k = 0; k <= kF; k++) {
                if ((uint32_t)k <= deg) {
                    const uint64_t v = v_warp_sum(acc160_reduce(acc[k]));
                    if (lane == 0) red[rd & 1][warp][k] = v;
                }
            }
        }
        __syncthreads();
        if (tid <= deg) {
            const uint32_t nw = items >= (uint32_t)kVThreads ? kVThreads / 32 : (items + 31) / 32;
            uint64_t v = 0;  // no terms: every round sends zeros
            for (uint32_t w = 0; w < nw; w++) v = gl_add(v, red[rd & 1][w][tid]);
            partials[((uint64_t)blockIdx.x * q + rd) * (deg + 1) + tid] = v;
        }
        uint64_t* t = cur;
        cur = nxt;
        nxt = t;
        const uint32_t ts = sc;
        sc = sn;
        sn = ts;
    }
    if (tid < nm) out[tid * out_stride + blockIdx.x] = gl_canon(cur[(size_t)tid * sc]);
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

__global__ void k_virtual_t0(VIn in, uint32_t nm, uint64_t* __restrict__ out) {
    const uint32_t j = threadIdx.x;
    if (j < nm) out[j] = gl_canon(in.p[j][0]);
}

// Rounds per launch for n_mles tables: the chunk and its half-size ping-pong
// buffer (12 bytes per table per position) fit in 46 KB of dynamic shared
// memory (under the 48 KB default limit together with the static part).
uint32_t v_qmax(uint32_t nm) {
    uint32_t q = 1;
    while (q < (uint32_t)kVQCap && 12ull * nm * (2ull << q) <= kVSmemBytes) q++;
    return q;
}

struct VPlan {
    uint64_t g1;     // chunks of the first level (= folded length it leaves)
    uint32_t q1;     // rounds of the first level
    uint64_t elems;  // scratch u64
};

VPlan v_plan(uint32_t nm, uint32_t t) {
    VPlan p{};
    const uint32_t qm = v_qmax(nm);
    p.q1 = t < qm ? t : qm;
    p.g1 = 1ull << (t - p.q1);
    // two folded buffers (nm x g1, 16-byte aligned) + the first level's partials
    p.elems = 2 * ((nm * p.g1 + 1) & ~1ull) + p.g1 * (p.q1 ? p.q1 : 1) * (kVMaxDeg + 1) + 8;
    return p;
}

}  // namespace

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
    const uint64_t bufsz = (nm * plan.g1 + 1) & ~1ull;
    uint64_t* buf[2] = {d_scratch, d_scratch + bufsz};
    uint64_t* partials = d_scratch + 2 * bufsz;
    uint32_t done = 0, which = 0;
    while (done < t) {
        const uint32_t rem = t - done;
        const uint32_t q = rem < qm ? rem : qm;
        const uint64_t G = 1ull << (rem - q);
        if (G > 0x7FFFFFFFull) return (int)cudaErrorInvalidValue;
        VChal ch{};
        for (uint32_t i = 0; i < q; i++) ch.r[i] = h_ch[done + i];
        const bool last = rem == q;
        uint64_t* out = last ? d_finals : buf[which];
        const uint64_t out_stride = last ? 1 : G;
        const size_t smem = ((size_t)12 * nm) << q;  // nm x (2^q + 2^(q-1)) u64
        if (T.deg <= 2)
            k_virtual_chunk<2><<<(unsigned)G, kVThreads, smem, s>>>(in, q, T, ch, partials, out, out_stride);
        else if (T.deg <= 4)
            k_virtual_chunk<4><<<(unsigned)G, kVThreads, smem, s>>>(in, q, T, ch, partials, out, out_stride);
        else
            k_virtual_chunk<8><<<(unsigned)G, kVThreads, smem, s>>>(in, q, T, ch, partials, out, out_stride);
        ZK_LAUNCH_CHECK();
        k_virtual_reduce<<<q * (T.deg + 1), kVThreads, 0, s>>>(partials, G, q, T.deg, d_rounds + (uint64_t)done * (T.deg + 1));
        ZK_LAUNCH_CHECK();
        if (!last) {
            for (uint32_t j = 0; j < nm; j++) in.p[j] = out + j * G;
            which ^= 1;
        }
        done += q;
    }
    return 0;
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
    if (!d_mles || !h_finals || !d_scratch || n_mles == 0 || n_mles > (uint32_t)kVMaxMles || t > 40 ||
        n_terms > (uint32_t)kVMaxTerms || (n_terms && (!coeffs || !idx_off)) || (t && (!h_ch || !h_rounds)))
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
    for (uint32_t j = 0; j < n_mles; j++)
        if (!d_mles[j]) return (int)cudaErrorInvalidValue;
    // the round messages and the finals live behind the plan's scratch
    uint64_t* d_rounds = d_scratch + v_plan(n_mles, t).elems;
    uint64_t* d_finals = d_rounds + (uint64_t)t * (deg + 1);
    int rc = virtual_dev(d_mles, n_mles, t, T, h_ch, d_rounds, d_finals, d_scratch, stream);
    if (rc) return rc;
    if (t) ZK_TRY(cudaMemcpyAsync(h_rounds, d_rounds, 8ull * t * (deg + 1), cudaMemcpyDeviceToHost, stream));
    ZK_TRY(cudaMemcpyAsync(h_finals, d_finals, 8ull * n_mles, cudaMemcpyDeviceToHost, stream));
    ZK_TRY(cudaStreamSynchronize(stream));
    return 0;
}

}  // extern "C"
