// projection.cu -- the forward witness of the projection block and the lookup
// index column its range check reads.
//
// Reference: crates/zkie-ops/src/projection.rs.  The block proves
//     out = round((x @ W) / 2^shift) + bias
// with h = x @ W kept as a GKR claim, the rounding as the affine constraint
//     rem_off = h - (out - bias) 2^shift + 2^(shift-1),   0 <= rem_off < 2^shift,
// and the range of rem_off as a logUp lookup into the table 0 .. 2^shift - 1
// whose indices are to_i32(rem_off) as u32 (prove_projection, :44-101).  The
// witness columns out and rem_off are what the reference's tests build on the
// host with div_round (:136-176): q = floor(a / 2^shift), plus one when the
// remainder is at least half.  Values are signed fixed point embedded in the
// field (fixed_point.rs: from_i64 / to_i64 / to_i32).
#include <cstring>
#include <mutex>

#include "../../include/zkie2.h"
#include "common.cuh"
#include "gl64.cuh"
#include "internal.h"

namespace zk {

namespace {

constexpr int kThreads = 256;
constexpr uint64_t kP = 0xFFFFFFFF00000001ull;

// to_i64 of a field element (fixed_point.rs): v if v <= i64::MAX, else -(p - v)
__device__ __forceinline__ int64_t to_i64(uint64_t v) {
    v = v >= kP ? v - kP : v;
    return v <= 0x7FFFFFFFFFFFFFFFull ? (int64_t)v : -(int64_t)(kP - v);
}

// from_i64: x if x >= 0, else p - |x|
__device__ __forceinline__ uint64_t from_i64(int64_t x) {
    return x >= 0 ? (uint64_t)x : kP - (uint64_t)(-(x + 1)) - 1;
}

// to_i32(v) as u32 (fixed_point.rs): v if v <= i32::MAX, else the negation of
// (p - v) truncated to i32, both reinterpreted as u32
__device__ __forceinline__ uint32_t to_i32_index(uint64_t v) {
    v = v >= kP ? v - kP : v;
    if (v <= 0x7FFFFFFFull) return (uint32_t)v;
    const uint32_t t = (uint32_t)(kP - v);  // the low 32 bits: `as i32`
    return 0u - t;
}

__global__ void k_projection_witness(const uint64_t* __restrict__ h, const uint64_t* __restrict__ bias, uint64_t n,
                                     uint32_t shift, uint64_t* __restrict__ out, uint64_t* __restrict__ rem_off,
                                     uint32_t* __restrict__ idx) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const int64_t half = (int64_t)1 << (shift - 1), mask = ((int64_t)1 << shift) - 1;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const int64_t a = to_i64(__ldg(h + i)), b = to_i64(__ldg(bias + i));
        const int64_t q = (a >> shift) + ((a & mask) >= half ? 1 : 0);  // div_round(a, 2^shift)
        const int64_t o = q + b;
        const uint64_t r = from_i64(a - (o - b) * ((int64_t)1 << shift) + half);
        out[i] = from_i64(o);
        rem_off[i] = r;
        if (idx) idx[i] = to_i32_index(r);
    }
}

__global__ void k_lookup_index_i32(const uint64_t* __restrict__ v, uint64_t n, uint32_t* __restrict__ idx) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        idx[i] = to_i32_index(__ldg(v + i));
}

__global__ void k_fill_const(uint64_t* __restrict__ out, uint64_t n, uint64_t v) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) out[i] = v;
}

__global__ void k_fill_iota(uint64_t* __restrict__ out, uint64_t n) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) out[i] = i;
}

unsigned grid_for(uint64_t n) {
    const uint64_t b = ceil_div(n, kThreads);
    return (unsigned)(b < 148ull * 16 ? b : 148ull * 16);
}

bool is_pow2(uint64_t x) { return x && !(x & (x - 1)); }

// Side streams of the projection block: the MatMul GKR and the affine
// sumcheck run on them while the caller's stream builds the lookup columns
// and proves the fraction tree (the three proofs share no data beyond the
// inputs, and every challenge is drawn on the host first).
struct ProjStreams {
    cudaStream_t gkr = nullptr, aff = nullptr;
    cudaEvent_t start = nullptr, gkr_done = nullptr, aff_done = nullptr;
    std::mutex call;
    bool ready = false;
};
std::mutex g_proj_mu;
ProjStreams g_proj[kMaxDevices];

int proj_streams(ProjStreams** out) {
    const int d = current_device();
    if (d < 0 || d >= kMaxDevices) return (int)cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> g(g_proj_mu);
    ProjStreams& p = g_proj[d];
    if (!p.ready) {
        ZK_TRY(cudaStreamCreateWithFlags(&p.gkr, cudaStreamNonBlocking));
        ZK_TRY(cudaStreamCreateWithFlags(&p.aff, cudaStreamNonBlocking));
        for (cudaEvent_t* e : {&p.start, &p.gkr_done, &p.aff_done})
            ZK_TRY(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
        p.ready = true;
    }
    *out = &p;
    return 0;
}

uint32_t lg_of(uint64_t x) {
    uint32_t r = 0;
    while ((1ull << r) < x) r++;
    return r;
}

// Scratch layout of zkie2_projection_prove (u64 elements, each region even-sized).
struct ProjLayout {
    uint64_t h, eq, ones, table, idx, num, den, fixed, op, virt, aff, look, frac, total;
};

ProjLayout proj_layout(uint64_t m, uint64_t k, uint64_t n, uint32_t shift) {
    ProjLayout L{};
    uint64_t off = 0;
    auto take = [&](uint64_t& at, uint64_t cnt) {
        at = off;
        off += (cnt + 1) & ~1ull;
    };
    const uint64_t mn = m * n, t = 1ull << shift;
    const uint64_t frac_n = zkie2_lookup_len(mn, t, 0);
    take(L.h, mn);
    take(L.eq, mn);
    take(L.ones, mn);
    take(L.table, t);
    take(L.idx, (mn + 1) / 2);
    take(L.num, frac_n);
    take(L.den, frac_n);
    take(L.fixed, zkie2_matmul_fixed_scratch_elems(m, k, n));
    take(L.op, zkie2_op_matmul_scratch_elems(m, k, n));
    take(L.virt, zkie2_virtual_scratch_elems(6, lg_of(mn)));
    take(L.aff, 3ull * lg_of(mn) + 6);
    take(L.look, zkie2_lookup_scratch_elems(t));
    take(L.frac, zkie2_fractional_scratch_elems(lg_of(frac_n)));
    L.total = off;
    return L;
}

}  // namespace

}  // namespace zk

using namespace zk;

extern "C" {

int zkie2_projection_witness(const uint64_t* d_h, const uint64_t* d_bias, uint64_t n, uint32_t shift,
                             uint64_t* d_out, uint64_t* d_rem_off, uint32_t* d_idx, cudaStream_t stream) {
    if (shift < 1 || shift > 30) return (int)cudaErrorInvalidValue;
    if (n == 0) return 0;
    if (!d_h || !d_bias || !d_out || !d_rem_off) return (int)cudaErrorInvalidValue;
    k_projection_witness<<<grid_for(n), kThreads, 0, stream>>>(d_h, d_bias, n, shift, d_out, d_rem_off, d_idx);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_lookup_index_i32(const uint64_t* d_v, uint64_t n, uint32_t* d_idx, cudaStream_t stream) {
    if (n == 0) return 0;
    if (!d_v || !d_idx) return (int)cudaErrorInvalidValue;
    k_lookup_index_i32<<<grid_for(n), kThreads, 0, stream>>>(d_v, n, d_idx);
    ZK_LAUNCH_CHECK();
    return 0;
}

uint32_t zkie2_projection_lookup_vars(uint64_t m, uint64_t n, uint32_t shift) {
    if (shift < 1 || shift > 30) return 0;
    return lg_of(zkie2_lookup_len(m * n, 1ull << shift, 0));
}

uint64_t zkie2_projection_scratch_elems(uint64_t m, uint64_t k, uint64_t n, uint32_t shift) {
    if (!is_pow2(m) || !is_pow2(k) || !is_pow2(n) || shift < 1 || shift > 30) return 0;
    return proj_layout(m, k, n, shift).total;
}

// prove_projection (crates/zkie-ops/src/projection.rs:44-101) in one call:
//   h = x W (mm_par_fixed, unless the caller passes h), the MatMul GKR with u,
//   v, ch drawn from src (matmul::prove(x^T, W, h, u, v, ch): the Op::MatMul
//   kernels), prove_virtual over [eq(v||u), rem_off, h, out, bias, ones] with
//   the five affine terms, alpha and beta from src, the merged lookup columns
//   of (to_i32(rem_off) as u32, rem_off) into the table 0 .. 2^shift - 1 and
//   their fraction tree (full_r then cs from src).  The challenger advances
//   exactly as the reference's does.  Synchronous.
int zkie2_projection_prove(const uint64_t* d_x, const uint64_t* d_w, const uint64_t* d_bias, const uint64_t* d_out,
                           const uint64_t* d_rem_off, const uint64_t* d_h, uint64_t m, uint64_t k, uint64_t n,
                           uint32_t shift, zkie2_challenger* src, uint64_t* h_claimed, uint64_t* h_mm_rounds,
                           uint64_t* h_mm_finals, uint64_t* h_u, uint64_t* h_v, uint64_t* h_ch,
                           uint64_t* h_aff_rounds, uint64_t* h_aff_finals, uint64_t* h_alpha_beta,
                           uint64_t* h_full_r, uint64_t* h_cs, uint64_t* h_frac_rounds, uint64_t* h_frac_finals,
                           uint64_t* h_frac_nd, uint64_t* d_scratch, cudaStream_t stream) {
    if (!d_x || !d_w || !d_bias || !d_out || !d_rem_off || !src || !d_scratch || !h_claimed || !h_mm_finals ||
        !h_aff_finals || !h_alpha_beta || !h_frac_nd)
        return (int)cudaErrorInvalidValue;
    if (!is_pow2(m) || !is_pow2(k) || !is_pow2(n) || shift < 1 || shift > 30) return (int)cudaErrorInvalidValue;
    const uint64_t mn = m * n, t = 1ull << shift;
    const uint32_t lm = lg_of(m), lk = lg_of(k), ln = lg_of(n), tv = lm + ln;
    const uint64_t frac_n = zkie2_lookup_len(mn, t, 0);
    const uint32_t lg = lg_of(frac_n);
    if (lm > 32 || lk > 32 || ln > 32) return (int)cudaErrorInvalidValue;
    if ((lk && (!h_mm_rounds || !h_ch)) || (lm && !h_u) || (ln && !h_v) || (tv && !h_aff_rounds) ||
        (lg && (!h_full_r || !h_cs || !h_frac_finals)) || (lg > 1 && !h_frac_rounds))
        return (int)cudaErrorInvalidValue;
    const ProjLayout L = proj_layout(m, k, n, shift);
    ProjStreams* ps = nullptr;
    int rc = proj_streams(&ps);
    if (rc) return rc;
    std::lock_guard<std::mutex> call_lock(ps->call);
    uint64_t* S = d_scratch;
    const uint64_t* h = d_h;
    if (!h) {
        rc = zkie2_matmul_fixed(d_x, d_w, m, k, n, S + L.h, 0, nullptr, S + L.fixed, stream);
        if (rc) return rc;
        h = S + L.h;
    }
    // every challenge in the reference's order: u, v, ch (the MatMul arm),
    // alpha, beta, then full_r and cs of the fraction tree
    uint64_t u[32], v[32], ch[32], pt[64];
    for (uint32_t i = 0; i < lm; i++) u[i] = zkie2_challenger_field(src);
    for (uint32_t i = 0; i < ln; i++) v[i] = zkie2_challenger_field(src);
    for (uint32_t i = 0; i < lk; i++) ch[i] = zkie2_challenger_field(src);
    h_alpha_beta[0] = zkie2_challenger_field(src);
    h_alpha_beta[1] = zkie2_challenger_field(src);
    for (uint32_t i = 0; i < lg; i++) h_full_r[i] = zkie2_challenger_field(src);
    for (uint32_t i = 0; i < lg; i++) h_cs[i] = zkie2_challenger_field(src);
    if (lm) std::memcpy(h_u, u, 8ull * lm);
    if (ln) std::memcpy(h_v, v, 8ull * ln);
    if (lk) std::memcpy(h_ch, ch, 8ull * lk);
    for (uint32_t i = 0; i < ln; i++) pt[i] = v[i];
    for (uint32_t i = 0; i < lm; i++) pt[ln + i] = u[i];
    ZK_TRY(cudaEventRecord(ps->start, stream));  // h and the caller's inputs are ready
    ZK_TRY(cudaStreamWaitEvent(ps->gkr, ps->start, 0));
    ZK_TRY(cudaStreamWaitEvent(ps->aff, ps->start, 0));
    // the MatMul GKR (matmul::prove(x^T, W, h, u, v, ch)) on its side stream
    uint64_t* d_mm = nullptr;
    rc = op_matmul_enqueue(d_x, d_w, h, m, k, n, u, v, ch, S + L.op, &d_mm, ps->gkr);
    // the affine constraint at pt = v || u on the other
    const uint64_t neg = kP - 1, two = 1ull << shift, half = 1ull << (shift - 1);
    const uint64_t coeffs[5] = {1, neg, two, gl_mul_host(neg, two), gl_mul_host(neg, half)};
    const uint32_t idx_off[6] = {0, 2, 4, 6, 8, 10};
    const uint32_t idx[10] = {0, 1, 0, 2, 0, 3, 0, 4, 0, 5};
    const uint64_t* mles[6] = {S + L.eq, d_rem_off, h, d_out, d_bias, S + L.ones};
    uint64_t* d_aff_rounds = S + L.aff;
    uint64_t* d_aff_finals = d_aff_rounds + 3ull * tv;
    if (!rc) rc = eq_table_dev(pt, tv, S + L.eq, ps->aff);
    if (!rc) {
        k_fill_const<<<grid_for(mn), kThreads, 0, ps->aff>>>(S + L.ones, mn, 1);
        rc = (int)cudaGetLastError();
    }
    if (!rc)
        rc = virtual_enqueue(mles, 6, tv, coeffs, idx_off, idx, 5, pt, d_aff_rounds, d_aff_finals, nullptr,
                             S + L.virt, ps->aff);
    // the range check on the caller's stream: the lookup columns (this step
    // reads one flag back, which synchronizes only the caller's stream), then
    // the fraction tree with its own side streams
    uint64_t *d_fr = nullptr, *d_ff = nullptr, *d_nd = nullptr, roff = 0;
    uint32_t* d_idx = reinterpret_cast<uint32_t*>(S + L.idx);
    if (!rc) {
        k_fill_iota<<<grid_for(t), kThreads, 0, stream>>>(S + L.table, t);
        rc = (int)cudaGetLastError();
    }
    if (!rc) rc = zkie2_lookup_index_i32(d_rem_off, mn, d_idx, stream);
    if (!rc)
        rc = zkie2_lookup_num_den(d_idx, d_rem_off, mn, S + L.table, nullptr, t, 0, h_alpha_beta[0], h_alpha_beta[1],
                                  S + L.num, S + L.den, S + L.look, stream);
    if (!rc)
        rc = fractional_enqueue(S + L.num, S + L.den, lg, h_full_r, h_cs, S + L.frac, stream, &d_fr, &d_ff, &d_nd,
                                &roff);
    // join the side streams, then one round of copies to the host
    if (cudaEventRecord(ps->gkr_done, ps->gkr) == cudaSuccess) cudaStreamWaitEvent(stream, ps->gkr_done, 0);
    if (cudaEventRecord(ps->aff_done, ps->aff) == cudaSuccess) cudaStreamWaitEvent(stream, ps->aff_done, 0);
    auto d2h = [&](void* dst, const void* src, uint64_t bytes) {
        if (!rc && bytes) rc = (int)cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, stream);
    };
    if (!rc) {
        d2h(h_claimed, d_mm, 8);
        d2h(h_mm_rounds, d_mm + 1, 24ull * lk);
        d2h(h_mm_finals, d_mm + 1 + 3ull * lk, 16);
        d2h(h_aff_rounds, d_aff_rounds, 24ull * tv);
        d2h(h_aff_finals, d_aff_finals, 48);
        d2h(h_frac_rounds, d_fr, 8 * roff);
        d2h(h_frac_finals, d_ff, 56ull * lg);
        d2h(h_frac_nd, d_nd, 16);
    }
    const cudaError_t e = cudaStreamSynchronize(stream);
    if (!rc && e != cudaSuccess) rc = (int)e;
    return rc;
}

}  // extern "C"
