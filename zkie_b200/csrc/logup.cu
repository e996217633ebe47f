// logup.cu -- the logUp GKR fraction tree on the device: prove_fractional and
// the lookup numerator / denominator columns it is run on.
//
// Reference: crates/zkie-core/src/common/logup_gkr.rs.
// prove_fractional_with_challenges (:29-69) proves sum_i num[i] / den[i] one
// layer at a time.  With the current layer split into halves (lo = [0, half),
// hi = [half, 2 half)) the next layer is
//     next_num = num_lo * den_hi + num_hi * den_lo,   next_den = den_lo * den_hi
// (:45-51), and layer l is a virtual sumcheck (prove_virtual,
// sumcheck.rs:378-438) over the seven tables
//     [eq(r), next_num, next_den, num_lo, num_hi, den_lo, den_hi]
// with r = full_r[0 .. lg n - l - 1] as both the eq point and the round
// challenges, and the five terms of build_terms (:19-28):
//     eq next_num - eq num_lo den_hi - eq num_hi den_lo + c eq next_den - c eq den_lo den_hi.
// Here every layer stays in HBM: the halves are pointer offsets into the
// current layer, the next layer comes from one fused kernel, the eq table
// from the MLE kernel, and the round messages of all layers go to the host
// in one copy at the end.
#include <map>
#include <memory>
#include <mutex>

#include "../../include/zkie2.h"
#include "common.cuh"
#include "gl64.cuh"
#include "hist.cuh"
#include "internal.h"

namespace zk {

namespace {

constexpr int kFracThreads = 256;
constexpr uint32_t kFracMles = 7, kFracTerms = 5, kFracDeg = 3;
constexpr uint32_t kMaxLg = 40;

// next_num[s] = num[s] den[s + half] + num[s + half] den[s] (one exact sum of
// two 128-bit products, reduced once), next_den[s] = den[s] den[s + half].
// Two consecutive s per thread when every pointer is 16-byte aligned.
__device__ __forceinline__ void frac_pair(uint64_t a, uint64_t b, uint64_t c, uint64_t d, uint64_t& nn,
                                          uint64_t& nd) {
    Acc160 acc = acc160_zero();
    acc160_mac(acc, a, d);
    acc160_mac(acc, b, c);
    nn = gl_canon(acc160_reduce(acc));
    nd = gl_canon(gl_mul(c, d));
}

template <bool kVec>
__global__ void __launch_bounds__(kFracThreads)
    k_fraction_layer(const uint64_t* __restrict__ num, const uint64_t* __restrict__ den, uint64_t half,
                     uint64_t* __restrict__ nnum, uint64_t* __restrict__ nden) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    if (kVec) {
        const ulonglong2* nl = reinterpret_cast<const ulonglong2*>(num);
        const ulonglong2* nh = reinterpret_cast<const ulonglong2*>(num + half);
        const ulonglong2* dl = reinterpret_cast<const ulonglong2*>(den);
        const ulonglong2* dh = reinterpret_cast<const ulonglong2*>(den + half);
        ulonglong2* on = reinterpret_cast<ulonglong2*>(nnum);
        ulonglong2* od = reinterpret_cast<ulonglong2*>(nden);
        for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < half / 2; i += stride) {
            const ulonglong2 a = __ldg(nl + i), b = __ldg(nh + i), c = __ldg(dl + i), d = __ldg(dh + i);
            uint64_t n0, d0, n1, d1;
            frac_pair(a.x, b.x, c.x, d.x, n0, d0);
            frac_pair(a.y, b.y, c.y, d.y, n1, d1);
            on[i] = make_ulonglong2(n0, n1);
            od[i] = make_ulonglong2(d0, d1);
        }
    } else {
        for (uint64_t s = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; s < half; s += stride)
            frac_pair(__ldg(num + s), __ldg(num + half + s), __ldg(den + s), __ldg(den + half + s), nnum[s], nden[s]);
    }
}

// The tail of the tree in one launch: layer l with t = lg - l - 1 <= kSmallVars
// variables is one block, which holds the layer's seven tables (eq from
// full_r, the next level's num / den, the halves of level l) in shared
// memory and runs all t rounds there: per round the four evaluations of
//     I(k) = eq (next_num - num_lo den_hi - num_hi den_lo + c (next_den - den_lo den_hi))
// at k = 0..3 (each table at f0 + k (f1 - f0)), summed over the pairs, then
// the fold f <- f0 + r_j (f1 - f0).  The same sums as prove_virtual's,
// without one eq-table launch and a few sumcheck launches per layer.
constexpr uint32_t kSmallVars = 10;
struct SmallTail {
    uint64_t r[kMaxLg];
    uint64_t c[kMaxLg];
    const uint64_t* num[kMaxLg + 1];
    const uint64_t* den[kMaxLg + 1];
    uint64_t roff[kMaxLg];
    uint32_t lg, l0;
};

__global__ void __launch_bounds__(kFracThreads) k_frac_small_layers(SmallTail T, uint64_t* __restrict__ rounds,
                                                                    uint64_t* __restrict__ finals) {
    extern __shared__ uint64_t sm[];
    __shared__ uint64_t red[kFracThreads / 32][4];
    const uint32_t l = T.l0 + blockIdx.x;
    const uint32_t t = T.lg - l - 1;
    const uint64_t half = 1ull << t;
    uint64_t* tab[kFracMles];
    for (uint32_t i = 0; i < kFracMles; i++) tab[i] = sm + i * half;
    const uint64_t* num = T.num[l];
    const uint64_t* den = T.den[l];
    const uint64_t* nnum = T.num[l + 1];
    const uint64_t* nden = T.den[l + 1];
    for (uint64_t x = threadIdx.x; x < half; x += blockDim.x) {
        uint64_t e = 1;
        for (uint32_t j = 0; j < t; j++) {
            const uint64_t rj = gl_canon(T.r[j]);
            e = gl_mul(e, ((x >> j) & 1) ? rj : gl_sub(1, rj));
        }
        tab[0][x] = gl_canon(e);
        tab[1][x] = gl_canon(nnum[x]);
        tab[2][x] = gl_canon(nden[x]);
        tab[3][x] = gl_canon(num[x]);
        tab[4][x] = gl_canon(num[x + half]);
        tab[5][x] = gl_canon(den[x]);
        tab[6][x] = gl_canon(den[x + half]);
    }
    __syncthreads();
    const uint64_t c = gl_canon(T.c[l]);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t len = half;
    for (uint32_t j = 0; j < t; j++) {
        const uint64_t pairs = len >> 1;
        uint64_t acc[4] = {0, 0, 0, 0};
        for (uint64_t q = threadIdx.x; q < pairs; q += blockDim.x) {
            uint64_t v[kFracMles][4];
            for (uint32_t i = 0; i < kFracMles; i++) {
                const uint64_t a0 = tab[i][2 * q], a1 = tab[i][2 * q + 1];
                const uint64_t d = gl_sub(a1, a0);
                v[i][0] = a0;
                v[i][1] = a1;
                v[i][2] = gl_add(a1, d);
                v[i][3] = gl_add(v[i][2], d);
            }
            // in the layer's first round I vanishes at k = 0, 1 (the next level
            // is the halves' fraction sum) and I(3) = 3 I(2)
            for (int k = (j == 0 ? 2 : 0); k < (j == 0 ? 3 : 4); k++) {
                const uint64_t dd = gl_mul(v[5][k], v[6][k]);
                uint64_t in = gl_sub(v[1][k], gl_mul(v[3][k], v[6][k]));
                in = gl_sub(in, gl_mul(v[4][k], v[5][k]));
                in = gl_add(in, gl_mul(c, gl_sub(v[2][k], dd)));
                acc[k] = gl_add(acc[k], gl_mul(v[0][k], in));
                if (j == 0) acc[3] = gl_add(acc[3], gl_mul(v[0][3], gl_add(gl_add(in, in), in)));
            }
        }
        for (int k = 0; k < 4; k++) {
            uint64_t a = acc[k];
            for (int o = 16; o; o >>= 1) a = gl_add(a, __shfl_xor_sync(0xFFFFFFFFu, a, o));
            if (lane == 0) red[warp][k] = a;
        }
        __syncthreads();
        if (threadIdx.x < 4) {
            uint64_t a = 0;
            for (int w = 0; w < kFracThreads / 32; w++) a = gl_add(a, red[w][threadIdx.x]);
            rounds[T.roff[l] + 4ull * j + threadIdx.x] = gl_canon(a);
        }
        // fold: new values into registers, then one barrier, then the writes
        const uint64_t rj = gl_canon(T.r[j]);
        uint64_t nv[2][kFracMles];
        for (int h = 0; h < 2; h++) {
            const uint64_t x = threadIdx.x + (uint64_t)h * blockDim.x;
            if (x < pairs)
                for (uint32_t i = 0; i < kFracMles; i++) {
                    const uint64_t a0 = tab[i][2 * x], a1 = tab[i][2 * x + 1];
                    nv[h][i] = gl_canon(gl_add(a0, gl_mul(rj, gl_sub(a1, a0))));
                }
        }
        __syncthreads();
        for (int h = 0; h < 2; h++) {
            const uint64_t x = threadIdx.x + (uint64_t)h * blockDim.x;
            if (x < pairs)
                for (uint32_t i = 0; i < kFracMles; i++) tab[i][x] = nv[h][i];
        }
        __syncthreads();
        len = pairs;
    }
    if (threadIdx.x < kFracMles) finals[(uint64_t)kFracMles * l + threadIdx.x] = gl_canon(tab[threadIdx.x][0]);
}

__global__ void k_fraction_final(const uint64_t* num, const uint64_t* den, uint64_t* out) {
    if (threadIdx.x == 0) {
        out[0] = gl_canon(num[0]);
        out[1] = gl_canon(den[0]);
    }
}

unsigned frac_grid(uint64_t work) {
    const uint64_t b = ceil_div(work, kFracThreads);
    return (unsigned)(b < 148ull * 16 ? (b ? b : 1) : 148ull * 16);
}

int launch_fraction_layer(const uint64_t* num, const uint64_t* den, uint64_t half, uint64_t* nnum, uint64_t* nden,
                          cudaStream_t s) {
    const bool vec = half % 2 == 0 &&
                     ((reinterpret_cast<uintptr_t>(num) | reinterpret_cast<uintptr_t>(den) |
                       reinterpret_cast<uintptr_t>(nnum) | reinterpret_cast<uintptr_t>(nden)) & 15) == 0;
    if (vec)
        k_fraction_layer<true><<<frac_grid(half / 2), kFracThreads, 0, s>>>(num, den, half, nnum, nden);
    else
        k_fraction_layer<false><<<frac_grid(half), kFracThreads, 0, s>>>(num, den, half, nnum, nden);
    ZK_LAUNCH_CHECK();
    return 0;
}

// Scratch layout of zkie2_fractional_prove for n = 2^lg (u64 offsets, every
// region a multiple of two elements so 16-byte alignment carries through):
// every level of the fraction tree (level l + 1 = the next fractions of level
// l, 2^(lg-l-1) values each of num and den), every layer's eq table and
// virtual-sumcheck scratch, then the round messages and final evaluations.
// All layers stay in HBM, so the layer sumchecks need not wait for each
// other (their challenges are all given up front).
struct FracScratch {
    uint64_t *num[kMaxLg + 1], *den[kMaxLg + 1];  // levels 1 .. lg (level 0 is the caller's input)
    uint64_t *eq[kMaxLg], *vscr[kMaxLg];
    uint64_t *rounds, *finals, *final_nd;
};

uint64_t even(uint64_t x) { return (x + 1) & ~1ull; }

uint64_t frac_layout(uint32_t lg, FracScratch* fs, uint64_t* base) {
    uint64_t off = 0;
    auto take = [&](uint64_t** p, uint64_t cnt) {
        if (base) *p = base + off;
        off += even(cnt);
    };
    FracScratch s{};
    for (uint32_t l = 1; l <= lg; l++) {
        take(&s.num[l], 1ull << (lg - l));
        take(&s.den[l], 1ull << (lg - l));
    }
    for (uint32_t l = 0; l < lg; l++) {
        take(&s.eq[l], 1ull << (lg - l - 1));
        take(&s.vscr[l], virtual_plan_elems(kFracMles, lg - l - 1));
    }
    take(&s.rounds, 2ull * lg * (lg ? lg - 1 : 0) + 2);
    take(&s.finals, (uint64_t)kFracMles * lg + 1);
    take(&s.final_nd, 2);
    if (fs) *fs = s;
    return off;
}

// Side streams of the layer sumchecks, one set per (device, caller stream):
// calls on different caller streams fan out on their own side streams and
// run concurrently; calls on one caller stream share a set, and its mutex
// covers an enqueue, so the shared events are never re-recorded under
// another call.
constexpr int kFracStreams = 4;
struct FracStreams {
    cudaStream_t s[kFracStreams] = {};
    cudaEvent_t start = nullptr, level[kMaxLg + 1] = {}, done[kFracStreams] = {};
    std::mutex call;
};
std::mutex g_frac_mu;
std::map<std::pair<int, cudaStream_t>, std::unique_ptr<FracStreams>> g_frac;

int frac_streams(cudaStream_t caller, FracStreams** out) {
    const int d = current_device();
    if (d < 0) return (int)cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> g(g_frac_mu);
    std::unique_ptr<FracStreams>& slot = g_frac[{d, caller}];
    if (!slot) {
        auto f = std::make_unique<FracStreams>();
        for (auto& st : f->s) ZK_TRY(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
        ZK_TRY(cudaEventCreateWithFlags(&f->start, cudaEventDisableTiming));
        for (auto& e : f->level) ZK_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        for (auto& e : f->done) ZK_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        slot = std::move(f);
    }
    *out = slot.get();
    return 0;
}

// Lookup column modes (logup_gkr.rs): the merged witness + table columns
// (build_lookup_num_den :210-240), the witness side alone
// (build_lookup_witness_num_den :261-277, prove_lookup_witness_batch :317-339),
// the witness side as committed columns (prove_lookup_witness_batch_columns
// :340-370: at least 32 rows, padding rows get den = alpha), and the table
// side with caller multiplicities (build_lookup_table_num_den :285-301).
enum : uint32_t { kLookupMerged = 0, kLookupWitness = 1, kLookupWitnessColumns = 2, kLookupTable = 3 };

// the tail kernel's dynamic shared memory above 48 KB, set once per device
std::mutex g_tail_mu;
bool g_tail_ready[kMaxDevices];

int small_tail_attr(size_t smem) {
    if (smem <= 48 * 1024) return 0;
    const int d = current_device();
    if (d < 0 || d >= kMaxDevices) return (int)cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> g(g_tail_mu);
    if (!g_tail_ready[d]) {
        ZK_TRY(cudaFuncSetAttribute(k_frac_small_layers, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)((size_t)kFracMles * (1ull << kSmallVars) * 8)));
        g_tail_ready[d] = true;
    }
    return 0;
}

uint64_t next_pow2(uint64_t x) {
    uint64_t p = 1;
    while (p < x) p <<= 1;
    return p;
}

uint64_t lookup_len(uint64_t n, uint64_t t, uint32_t mode) {
    switch (mode) {
        case kLookupMerged: return next_pow2(n + t);
        case kLookupWitness: return next_pow2(n);
        case kLookupWitnessColumns: {
            const uint64_t l = next_pow2(n);
            return l < 32 ? 32 : l;
        }
        case kLookupTable: return next_pow2(t);
        default: return 0;
    }
}

// m[x[i]] += 1 for i < n; an index at or above t raises *bad (hist.cuh)
__global__ void k_lookup_hist(const uint32_t* __restrict__ x, uint64_t n, uint64_t t, uint32_t* __restrict__ m,
                              uint32_t* __restrict__ bad) {
    hist_grid(x, n, t, m, bad, 1u);
}

// alpha + j + beta * v as a canonical field element
__device__ __forceinline__ uint64_t lookup_den(uint64_t alpha, uint64_t j, uint64_t beta, uint64_t v) {
    return gl_canon(gl_add(gl_add(alpha, j), gl_mul(beta, v)));
}

__global__ void k_lookup_fill(const uint32_t* __restrict__ x, const uint64_t* __restrict__ y, uint64_t n,
                              const uint64_t* __restrict__ table, uint64_t t, const uint32_t* __restrict__ m32,
                              const uint64_t* __restrict__ m64, uint32_t mode, uint64_t alpha, uint64_t beta,
                              uint64_t total, uint64_t* __restrict__ num, uint64_t* __restrict__ den) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        uint64_t nv, dv;
        if (mode == kLookupTable) {
            const bool in = i < t;
            nv = in ? gl_canon(__ldg(m64 + i)) : 0;
            dv = lookup_den(alpha, i, beta, in ? __ldg(table + i) : 0);
        } else if (i < n) {
            nv = 1;
            dv = lookup_den(alpha, __ldg(x + i), beta, __ldg(y + i));
        } else if (mode == kLookupMerged && i - n < t) {
            const uint64_t j = i - n;
            const uint32_t c = __ldg(m32 + j);
            nv = c ? GL_P - c : 0;  // from_i64(-m)
            dv = lookup_den(alpha, j, beta, __ldg(table + j));
        } else {
            nv = 0;
            dv = mode == kLookupWitnessColumns ? gl_canon(alpha) : 1;
        }
        num[i] = nv;
        den[i] = dv;
    }
}

}  // namespace

// prove_fractional_with_challenges enqueued on `stream` (the tree's levels)
// and the side streams (the layer sumchecks), joined back into `stream`
// before returning; nothing is synchronized or copied to the host.  The
// round messages (4 per round, layer after layer: *n_rounds values), the
// finals (7 per layer) and the last level's (num, den) stay in d_scratch at
// *d_rounds, *d_finals, *d_nd.
int fractional_enqueue(const uint64_t* d_num, const uint64_t* d_den, uint32_t lg_n, const uint64_t* h_full_r,
                       const uint64_t* h_cs, uint64_t* d_scratch, cudaStream_t stream, uint64_t** d_rounds,
                       uint64_t** d_finals, uint64_t** d_nd, uint64_t* n_rounds) {
    if (!d_num || !d_den || !d_scratch || lg_n > kMaxLg || (lg_n && (!h_full_r || !h_cs)))
        return (int)cudaErrorInvalidValue;
    FracStreams* fst = nullptr;
    int rc = frac_streams(stream, &fst);
    if (rc) return rc;
    std::lock_guard<std::mutex> call_lock(fst->call);
    FracScratch fs;
    frac_layout(lg_n, &fs, d_scratch);
    const uint64_t n = 1ull << lg_n;
    const uint32_t off[kFracTerms + 1] = {0, 2, 5, 8, 10, 13};
    const uint32_t idx[13] = {0, 1, 0, 3, 6, 0, 4, 5, 0, 2, 0, 5, 6};
    // Level l + 1 of the tree from level l, all on the caller's stream; an
    // event marks each level.  Layer l's sumcheck (over levels l and l + 1,
    // its own eq table and scratch) runs on a side stream as soon as level
    // l + 1 exists, concurrently with the other layers.
    const uint64_t* lnum[kMaxLg + 1];
    const uint64_t* lden[kMaxLg + 1];
    lnum[0] = d_num;
    lden[0] = d_den;
    for (uint32_t l = 1; l <= lg_n; l++) {
        lnum[l] = fs.num[l];
        lden[l] = fs.den[l];
    }
    ZK_TRY(cudaEventRecord(fst->start, stream));
    for (auto& ss : fst->s) ZK_TRY(cudaStreamWaitEvent(ss, fst->start, 0));
    for (uint32_t l = 0; l < lg_n && !rc; l++) {
        rc = launch_fraction_layer(lnum[l], lden[l], n >> (l + 1), fs.num[l + 1], fs.den[l + 1], stream);
        if (!rc) rc = (int)cudaEventRecord(fst->level[l + 1], stream);
    }
    // layers with more than kSmallVars variables: eq table and virtual
    // sumcheck on a side stream each; the rest: one launch after the levels
    const uint32_t l0 = lg_n > kSmallVars + 1 ? lg_n - kSmallVars - 1 : 0;
    uint64_t roff = 0;
    SmallTail tail{};
    for (uint32_t l = 0; l < lg_n && !rc; l++) {
        if (l >= l0) {
            tail.roff[l] = roff;
            roff += (uint64_t)(kFracDeg + 1) * (lg_n - l - 1);
            continue;
        }
        cudaStream_t ss = fst->s[l % kFracStreams];
        const uint64_t half = n >> (l + 1);
        const uint32_t t = lg_n - l - 1;
        rc = eq_table_dev(h_full_r, t, fs.eq[l], ss);  // independent of the tree
        if (!rc) rc = (int)cudaStreamWaitEvent(ss, fst->level[l + 1], 0);
        if (rc) break;
        const uint64_t c = gl_canon(h_cs[l]);
        const uint64_t coeffs[kFracTerms] = {1, GL_P - 1, GL_P - 1, c, gl_canon(GL_P - c)};
        const uint64_t* mles[kFracMles] = {fs.eq[l], lnum[l + 1], lden[l + 1], lnum[l], lnum[l] + half,
                                           lden[l], lden[l] + half};
        // the next level was computed from this one: the first round's g(0), g(1) vanish
        rc = virtual_enqueue(mles, kFracMles, t, coeffs, off, idx, kFracTerms, h_full_r, fs.rounds + roff,
                             fs.finals + (uint64_t)kFracMles * l, nullptr, fs.vscr[l], ss, true);
        roff += (uint64_t)(kFracDeg + 1) * t;
    }
    if (!rc && lg_n > l0) {
        tail.lg = lg_n;
        tail.l0 = l0;
        for (uint32_t j = 0; j < lg_n; j++) {
            tail.r[j] = h_full_r[j];
            tail.c[j] = h_cs[j];
        }
        for (uint32_t l = 0; l <= lg_n; l++) {
            tail.num[l] = lnum[l];
            tail.den[l] = lden[l];
        }
        const uint32_t tmax = lg_n - l0 - 1;
        const size_t smem = (size_t)kFracMles * (1ull << tmax) * 8;
        rc = small_tail_attr(smem);
        if (!rc) {
            k_frac_small_layers<<<lg_n - l0, kFracThreads, smem, stream>>>(tail, fs.rounds, fs.finals);
            rc = (int)cudaGetLastError();
        }
    }
    // join the side streams (also after an error part-way, so that the
    // caller's synchronization covers everything enqueued)
    for (int i = 0; i < kFracStreams; i++) {
        if (cudaEventRecord(fst->done[i], fst->s[i]) == cudaSuccess) cudaStreamWaitEvent(stream, fst->done[i], 0);
    }
    if (!rc) {
        k_fraction_final<<<1, 32, 0, stream>>>(lnum[lg_n], lden[lg_n], fs.final_nd);
        rc = (int)cudaGetLastError();
    }
    *d_rounds = fs.rounds;
    *d_finals = fs.finals;
    *d_nd = fs.final_nd;
    *n_rounds = roff;
    return rc;
}

}  // namespace zk

using namespace zk;

extern "C" {

uint64_t zkie2_fractional_scratch_elems(uint32_t lg_n) { return lg_n > kMaxLg ? 0 : frac_layout(lg_n, nullptr, nullptr); }

int zkie2_fractional_prove(const uint64_t* d_num, const uint64_t* d_den, uint32_t lg_n, const uint64_t* h_full_r,
                           const uint64_t* h_cs, uint64_t* h_rounds, uint64_t* h_finals, uint64_t* h_final_nd,
                           uint64_t* d_scratch, cudaStream_t stream) {
    if (!d_num || !d_den || !h_final_nd || !d_scratch || lg_n > kMaxLg ||
        (lg_n && (!h_full_r || !h_cs || !h_finals)) || (lg_n > 1 && !h_rounds))
        return (int)cudaErrorInvalidValue;
    uint64_t *d_rounds = nullptr, *d_finals = nullptr, *d_nd = nullptr, roff = 0;
    int rc = fractional_enqueue(d_num, d_den, lg_n, h_full_r, h_cs, d_scratch, stream, &d_rounds, &d_finals, &d_nd,
                                &roff);
    if (!rc && roff) rc = (int)cudaMemcpyAsync(h_rounds, d_rounds, 8 * roff, cudaMemcpyDeviceToHost, stream);
    if (!rc && lg_n)
        rc = (int)cudaMemcpyAsync(h_finals, d_finals, 8ull * kFracMles * lg_n, cudaMemcpyDeviceToHost, stream);
    if (!rc) rc = (int)cudaMemcpyAsync(h_final_nd, d_nd, 16, cudaMemcpyDeviceToHost, stream);
    const cudaError_t e = cudaStreamSynchronize(stream);
    if (!rc && e != cudaSuccess) rc = (int)e;
    return rc;
}

uint64_t zkie2_lookup_len(uint64_t n, uint64_t t, uint32_t mode) { return lookup_len(n, t, mode); }

uint64_t zkie2_lookup_scratch_elems(uint64_t t) { return t / 2 + 2; }

// Lookup columns enqueued without synchronization; an index at or past t
// (mode 0) sets bit 1 of *d_bad.
static int lookup_enqueue(const uint32_t* d_x, const uint64_t* d_y, uint64_t n, const uint64_t* d_table,
                          const uint64_t* d_m, uint64_t t, uint32_t mode, uint64_t alpha, uint64_t beta,
                          uint64_t* d_num, uint64_t* d_den, uint64_t* d_scratch, uint32_t* d_bad,
                          cudaStream_t stream) {
    if (mode > kLookupTable || !d_num || !d_den) return (int)cudaErrorInvalidValue;
    if (mode != kLookupTable && n && (!d_x || !d_y)) return (int)cudaErrorInvalidValue;
    if ((mode == kLookupMerged || mode == kLookupTable) && t && !d_table) return (int)cudaErrorInvalidValue;
    if (mode == kLookupTable && t && !d_m) return (int)cudaErrorInvalidValue;
    if (mode == kLookupMerged && (!d_scratch || !d_bad || n > 0xFFFFFFFFull)) return (int)cudaErrorInvalidValue;
    const uint64_t total = lookup_len(n, t, mode);
    uint32_t* m32 = nullptr;
    if (mode == kLookupMerged) {
        m32 = reinterpret_cast<uint32_t*>(d_scratch);
        ZK_TRY(cudaMemsetAsync(m32, 0, 4 * t, stream));
        if (n) {
            k_lookup_hist<<<frac_grid(n), kFracThreads, 0, stream>>>(d_x, n, t, m32, d_bad);
            ZK_LAUNCH_CHECK();
        }
    }
    k_lookup_fill<<<frac_grid(total), kFracThreads, 0, stream>>>(d_x, d_y, n, d_table, t, m32, d_m, mode,
                                                                   gl_canon(alpha), gl_canon(beta), total, d_num,
                                                                   d_den);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_lookup_num_den(const uint32_t* d_x, const uint64_t* d_y, uint64_t n, const uint64_t* d_table,
                         const uint64_t* d_m, uint64_t t, uint32_t mode, uint64_t alpha, uint64_t beta,
                         uint64_t* d_num, uint64_t* d_den, uint64_t* d_scratch, cudaStream_t stream) {
    uint32_t* bad = nullptr;
    if (mode == kLookupMerged) {
        if (!d_scratch) return (int)cudaErrorInvalidValue;
        bad = reinterpret_cast<uint32_t*>(d_scratch) + 2 * (t / 2 + 1);
        ZK_TRY(cudaMemsetAsync(bad, 0, 4, stream));
    }
    int rc = lookup_enqueue(d_x, d_y, n, d_table, d_m, t, mode, alpha, beta, d_num, d_den, d_scratch, bad, stream);
    if (rc) return rc;
    if (mode == kLookupMerged) {
        uint32_t h_bad = 0;
        ZK_TRY(cudaMemcpyAsync(&h_bad, bad, 4, cudaMemcpyDeviceToHost, stream));
        ZK_TRY(cudaStreamSynchronize(stream));
        if (h_bad) return (int)cudaErrorInvalidValue;
    }
    return 0;
}

int zkie2_lookup_num_den_async(const uint32_t* d_x, const uint64_t* d_y, uint64_t n, const uint64_t* d_table,
                               const uint64_t* d_m, uint64_t t, uint32_t mode, uint64_t alpha, uint64_t beta,
                               uint64_t* d_num, uint64_t* d_den, uint64_t* d_scratch, uint32_t* d_err,
                               cudaStream_t stream) {
    if (mode == kLookupMerged && !d_err) return (int)cudaErrorInvalidValue;
    return lookup_enqueue(d_x, d_y, n, d_table, d_m, t, mode, alpha, beta, d_num, d_den, d_scratch, d_err, stream);
}

uint64_t zkie2_fractional_proof_elems(uint32_t lg_n) {
    if (lg_n > kMaxLg) return 0;
    return 2ull * lg_n * (lg_n ? lg_n - 1 : 0) + 7ull * lg_n + 2;
}

int zkie2_fractional_prove_async(const uint64_t* d_num, const uint64_t* d_den, uint32_t lg_n,
                                 const uint64_t* h_full_r, const uint64_t* h_cs, uint64_t* d_proof,
                                 uint64_t* d_scratch, cudaStream_t stream) {
    if (!d_proof) return (int)cudaErrorInvalidValue;
    uint64_t *d_rounds = nullptr, *d_finals = nullptr, *d_nd = nullptr, roff = 0;
    int rc = fractional_enqueue(d_num, d_den, lg_n, h_full_r, h_cs, d_scratch, stream, &d_rounds, &d_finals, &d_nd,
                                &roff);
    if (rc) return rc;
    if (roff) ZK_TRY(cudaMemcpyAsync(d_proof, d_rounds, 8 * roff, cudaMemcpyDeviceToDevice, stream));
    if (lg_n) ZK_TRY(cudaMemcpyAsync(d_proof + roff, d_finals, 56ull * lg_n, cudaMemcpyDeviceToDevice, stream));
    ZK_TRY(cudaMemcpyAsync(d_proof + roff + 7ull * lg_n, d_nd, 16, cudaMemcpyDeviceToDevice, stream));
    return 0;
}

}  // extern "C"
