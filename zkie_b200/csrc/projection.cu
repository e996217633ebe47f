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
#include <map>
#include <memory>
#include <mutex>
#include <vector>

#include "../../include/zkie2.h"
#include "common.cuh"
#include "fixed.cuh"
#include "gl64.cuh"
#include "internal.h"

namespace zk {

namespace {

constexpr int kThreads = 256;
constexpr uint64_t kP = 0xFFFFFFFF00000001ull;

__global__ void k_projection_witness(const uint64_t* __restrict__ h, const uint64_t* __restrict__ bias, uint64_t n,
                                     uint32_t shift, uint64_t* __restrict__ out, uint64_t* __restrict__ rem_off,
                                     uint32_t* __restrict__ idx) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const int64_t half = (int64_t)1 << (shift - 1);
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const int64_t a = fx_to_i64(__ldg(h + i)), b = fx_to_i64(__ldg(bias + i));
        const uint64_t o = fx_from_i64(fx_wadd(fx_round_div_pow2(a, shift), b));  // div_round(a, 2^shift) + b
        const uint64_t r =
            fx_from_i64(fx_wadd(fx_wsub(a, fx_wmul(fx_wsub(fx_to_i64(o), b), (int64_t)1 << shift)), half));
        out[i] = o;
        rem_off[i] = r;
        if (idx) idx[i] = fx_to_i32_index(r);
    }
}

__global__ void k_lookup_index_i32(const uint64_t* __restrict__ v, uint64_t n, uint32_t* __restrict__ idx) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        idx[i] = fx_to_i32_index(__ldg(v + i));
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
// inputs, and every challenge is drawn on the host first).  One set per
// (device, caller stream), so calls on different caller streams overlap.
struct ProjStreams {
    cudaStream_t gkr = nullptr, aff = nullptr;
    cudaEvent_t start = nullptr, gkr_done = nullptr, aff_done = nullptr;
    std::mutex call;
};
std::mutex g_proj_mu;
std::map<std::pair<int, cudaStream_t>, std::unique_ptr<ProjStreams>> g_proj;

int proj_streams(cudaStream_t caller, ProjStreams** out) {
    const int d = current_device();
    if (d < 0) return (int)cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> g(g_proj_mu);
    std::unique_ptr<ProjStreams>& slot = g_proj[{d, caller}];
    if (!slot) {
        auto p = std::make_unique<ProjStreams>();
        ZK_TRY(cudaStreamCreateWithFlags(&p->gkr, cudaStreamNonBlocking));
        ZK_TRY(cudaStreamCreateWithFlags(&p->aff, cudaStreamNonBlocking));
        for (cudaEvent_t* e : {&p->start, &p->gkr_done, &p->aff_done})
            ZK_TRY(cudaEventCreateWithFlags(e, cudaEventDisableTiming));
        slot = std::move(p);
    }
    *out = slot.get();
    return 0;
}

uint32_t lg_of(uint64_t x) {
    uint32_t r = 0;
    while ((1ull << r) < x) r++;
    return r;
}

// Scratch layout of zkie2_projection_prove (u64 elements, each region even-sized).
struct ProjLayout {
    uint64_t h, eq, ones, table, idx, num, den, fixed, op, virt, aff, look, frac, err, proof, total;
};

// The proof fields in one device array: claimed (1) | mm_rounds (3 lk) |
// mm_finals (2) | aff_rounds (3 tv) | aff_finals (6) | frac_rounds
// (2 lg (lg - 1)) | frac_finals (7 lg) | frac_nd (2).
struct ProjProofLayout {
    uint64_t claimed, mm_rounds, mm_finals, aff_rounds, aff_finals, frac_rounds, frac_finals, frac_nd, total;
};

ProjProofLayout proj_proof_layout(uint32_t lk, uint32_t tv, uint32_t lg) {
    ProjProofLayout P{};
    P.claimed = 0;
    P.mm_rounds = 1;
    P.mm_finals = P.mm_rounds + 3ull * lk;
    P.aff_rounds = P.mm_finals + 2;
    P.aff_finals = P.aff_rounds + 3ull * tv;
    P.frac_rounds = P.aff_finals + 6;
    P.frac_finals = P.frac_rounds + 2ull * lg * (lg ? lg - 1 : 0);
    P.frac_nd = P.frac_finals + 7ull * lg;
    P.total = P.frac_nd + 2;
    return P;
}

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
    take(L.err, 2);
    take(L.proof, proj_proof_layout(lg_of(k), lg_of(mn), lg_of(frac_n)).total);
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

uint64_t zkie2_projection_proof_elems(uint64_t m, uint64_t k, uint64_t n, uint32_t shift) {
    if (!is_pow2(m) || !is_pow2(k) || !is_pow2(n) || shift < 1 || shift > 30) return 0;
    return proj_proof_layout(lg_of(k), lg_of(m * n), zkie2_projection_lookup_vars(m, n, shift)).total;
}

}  // extern "C"

namespace zk {
namespace {

// prove_projection with every challenge given (u, v, ch, alpha, beta, full_r,
// cs), enqueued without synchronization: the proof fields land in d_proof
// (ProjProofLayout), a bad lookup index sets *d_err.  The MatMul GKR and the
// affine sumcheck run on the side streams while the caller's stream builds
// the lookup columns and proves the fraction tree; both join back into the
// caller's stream before the proof is assembled.
int projection_enqueue(const uint64_t* d_x, const uint64_t* d_w, const uint64_t* d_bias, const uint64_t* d_out,
                       const uint64_t* d_rem_off, const uint64_t* d_h, uint64_t m, uint64_t k, uint64_t n,
                       uint32_t shift, const uint64_t* u, const uint64_t* v, const uint64_t* ch, uint64_t alpha,
                       uint64_t beta, const uint64_t* full_r, const uint64_t* cs, uint64_t* d_proof, uint32_t* d_err,
                       uint64_t* d_scratch, cudaStream_t stream) {
    const uint64_t mn = m * n, t = 1ull << shift;
    const uint32_t lm = lg_of(m), lk = lg_of(k), ln = lg_of(n), tv = lm + ln;
    const uint32_t lg = lg_of(zkie2_lookup_len(mn, t, 0));
    const ProjLayout L = proj_layout(m, k, n, shift);
    const ProjProofLayout PL = proj_proof_layout(lk, tv, lg);
    ProjStreams* ps = nullptr;
    int rc = proj_streams(stream, &ps);
    if (rc) return rc;
    std::lock_guard<std::mutex> call_lock(ps->call);
    uint64_t* S = d_scratch;
    const uint64_t* h = d_h;
    if (!h) {
        rc = zkie2_matmul_fixed(d_x, d_w, m, k, n, S + L.h, 0, nullptr, S + L.fixed, stream);
        if (rc) return rc;
        h = S + L.h;
    }
    uint64_t pt[64];
    for (uint32_t i = 0; i < ln; i++) pt[i] = v[i];
    for (uint32_t i = 0; i < lm; i++) pt[ln + i] = u[i];
    ZK_TRY(cudaEventRecord(ps->start, stream));  // h and the caller's inputs are ready
    ZK_TRY(cudaStreamWaitEvent(ps->gkr, ps->start, 0));
    ZK_TRY(cudaStreamWaitEvent(ps->aff, ps->start, 0));
    // the MatMul GKR (matmul::prove(x^T, W, h, u, v, ch)) on its side stream
    uint64_t* d_mm = nullptr;
    rc = op_matmul_enqueue(d_x, d_w, h, m, k, n, u, v, ch, S + L.op, &d_mm, ps->gkr);
    if (!rc)
        rc = (int)cudaMemcpyAsync(d_proof + PL.claimed, d_mm, 8ull * (3 + 3ull * lk), cudaMemcpyDeviceToDevice,
                                  ps->gkr);
    // the affine constraint at pt = v || u on the other
    const uint64_t neg = kP - 1, two = 1ull << shift, half = 1ull << (shift - 1);
    const uint64_t coeffs[5] = {1, neg, two, gl_mul_host(neg, two), gl_mul_host(neg, half)};
    const uint32_t idx_off[6] = {0, 2, 4, 6, 8, 10};
    const uint32_t idx[10] = {0, 1, 0, 2, 0, 3, 0, 4, 0, 5};
    const uint64_t* mles[6] = {S + L.eq, d_rem_off, h, d_out, d_bias, S + L.ones};
    if (!rc) rc = eq_table_dev(pt, tv, S + L.eq, ps->aff);
    if (!rc) {
        k_fill_const<<<grid_for(mn), kThreads, 0, ps->aff>>>(S + L.ones, mn, 1);
        rc = (int)cudaGetLastError();
    }
    if (!rc)
        rc = virtual_enqueue(mles, 6, tv, coeffs, idx_off, idx, 5, pt, d_proof + PL.aff_rounds,
                             d_proof + PL.aff_finals, nullptr, S + L.virt, ps->aff);
    // the range check on the caller's stream: the lookup columns, then the
    // fraction tree with its own side streams
    uint64_t *d_fr = nullptr, *d_ff = nullptr, *d_nd = nullptr, roff = 0;
    uint32_t* d_idx = reinterpret_cast<uint32_t*>(S + L.idx);
    if (!rc) {
        k_fill_iota<<<grid_for(t), kThreads, 0, stream>>>(S + L.table, t);
        rc = (int)cudaGetLastError();
    }
    if (!rc) rc = zkie2_lookup_index_i32(d_rem_off, mn, d_idx, stream);
    if (!rc)
        rc = zkie2_lookup_num_den_async(d_idx, d_rem_off, mn, S + L.table, nullptr, t, 0, alpha, beta, S + L.num,
                                        S + L.den, S + L.look, d_err, stream);
    if (!rc)
        rc = fractional_enqueue(S + L.num, S + L.den, lg, full_r, cs, S + L.frac, stream, &d_fr, &d_ff, &d_nd, &roff);
    // join the side streams, then assemble the proof on the caller's stream
    if (cudaEventRecord(ps->gkr_done, ps->gkr) == cudaSuccess) cudaStreamWaitEvent(stream, ps->gkr_done, 0);
    if (cudaEventRecord(ps->aff_done, ps->aff) == cudaSuccess) cudaStreamWaitEvent(stream, ps->aff_done, 0);
    auto d2d = [&](uint64_t at, const void* src, uint64_t bytes) {
        if (!rc && bytes) rc = (int)cudaMemcpyAsync(d_proof + at, src, bytes, cudaMemcpyDeviceToDevice, stream);
    };
    d2d(PL.frac_rounds, d_fr, 8 * roff);
    d2d(PL.frac_finals, d_ff, 56ull * lg);
    d2d(PL.frac_nd, d_nd, 16);
    return rc;
}

bool proj_args_ok(const uint64_t* d_x, const uint64_t* d_w, const uint64_t* d_bias, const uint64_t* d_out,
                  const uint64_t* d_rem_off, const uint64_t* d_scratch, uint64_t m, uint64_t k, uint64_t n,
                  uint32_t shift) {
    if (!d_x || !d_w || !d_bias || !d_out || !d_rem_off || !d_scratch) return false;
    if (!is_pow2(m) || !is_pow2(k) || !is_pow2(n) || shift < 1 || shift > 30) return false;
    return lg_of(m) <= 32 && lg_of(k) <= 32 && lg_of(n) <= 32;
}

}  // namespace
}  // namespace zk

extern "C" {

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
    if (!proj_args_ok(d_x, d_w, d_bias, d_out, d_rem_off, d_scratch, m, k, n, shift) || !src || !h_claimed ||
        !h_mm_finals || !h_aff_finals || !h_alpha_beta || !h_frac_nd)
        return (int)cudaErrorInvalidValue;
    const uint64_t mn = m * n, t = 1ull << shift;
    const uint32_t lm = lg_of(m), lk = lg_of(k), ln = lg_of(n), tv = lm + ln;
    const uint32_t lg = lg_of(zkie2_lookup_len(mn, t, 0));
    if ((lk && (!h_mm_rounds || !h_ch)) || (lm && !h_u) || (ln && !h_v) || (tv && !h_aff_rounds) ||
        (lg && (!h_full_r || !h_cs || !h_frac_finals)) || (lg > 1 && !h_frac_rounds))
        return (int)cudaErrorInvalidValue;
    const ProjLayout L = proj_layout(m, k, n, shift);
    const ProjProofLayout PL = proj_proof_layout(lk, tv, lg);
    // every challenge in the reference's order: u, v, ch (the MatMul arm),
    // alpha, beta, then full_r and cs of the fraction tree
    uint64_t u[32], v[32], ch[32];
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
    uint64_t* d_proof = d_scratch + L.proof;
    uint32_t* d_err = reinterpret_cast<uint32_t*>(d_scratch + L.err);
    ZK_TRY(cudaMemsetAsync(d_err, 0, 4, stream));
    int rc = projection_enqueue(d_x, d_w, d_bias, d_out, d_rem_off, d_h, m, k, n, shift, u, v, ch, h_alpha_beta[0],
                                h_alpha_beta[1], h_full_r, h_cs, d_proof, d_err, d_scratch, stream);
    std::vector<uint64_t> hp(PL.total);
    uint32_t h_err = 0;
    if (!rc) rc = (int)cudaMemcpyAsync(hp.data(), d_proof, 8 * PL.total, cudaMemcpyDeviceToHost, stream);
    if (!rc) rc = (int)cudaMemcpyAsync(&h_err, d_err, 4, cudaMemcpyDeviceToHost, stream);
    const cudaError_t e = cudaStreamSynchronize(stream);
    if (!rc && e != cudaSuccess) rc = (int)e;
    if (!rc && h_err) rc = (int)cudaErrorInvalidValue;
    if (rc) return rc;
    *h_claimed = hp[PL.claimed];
    if (lk) std::memcpy(h_mm_rounds, hp.data() + PL.mm_rounds, 24ull * lk);
    std::memcpy(h_mm_finals, hp.data() + PL.mm_finals, 16);
    if (tv) std::memcpy(h_aff_rounds, hp.data() + PL.aff_rounds, 24ull * tv);
    std::memcpy(h_aff_finals, hp.data() + PL.aff_finals, 48);
    if (lg > 1) std::memcpy(h_frac_rounds, hp.data() + PL.frac_rounds, 16ull * lg * (lg - 1));
    if (lg) std::memcpy(h_frac_finals, hp.data() + PL.frac_finals, 56ull * lg);
    std::memcpy(h_frac_nd, hp.data() + PL.frac_nd, 16);
    return 0;
}

// The same with every challenge given by the caller and the proof fields
// (zkie2_projection_proof_elems, the order above) left in d_proof on the
// device; a lookup index outside the table sets bit 1 of *d_err.  No
// synchronization.
int zkie2_projection_prove_async(const uint64_t* d_x, const uint64_t* d_w, const uint64_t* d_bias,
                                 const uint64_t* d_out, const uint64_t* d_rem_off, const uint64_t* d_h, uint64_t m,
                                 uint64_t k, uint64_t n, uint32_t shift, const uint64_t* h_u, const uint64_t* h_v,
                                 const uint64_t* h_ch, uint64_t alpha, uint64_t beta, const uint64_t* h_full_r,
                                 const uint64_t* h_cs, uint64_t* d_proof, uint32_t* d_err, uint64_t* d_scratch,
                                 cudaStream_t stream) {
    if (!proj_args_ok(d_x, d_w, d_bias, d_out, d_rem_off, d_scratch, m, k, n, shift) || !d_proof || !d_err)
        return (int)cudaErrorInvalidValue;
    const uint32_t lm = lg_of(m), lk = lg_of(k), ln = lg_of(n);
    const uint32_t lg = zkie2_projection_lookup_vars(m, n, shift);
    if ((lm && !h_u) || (ln && !h_v) || (lk && !h_ch) || (lg && (!h_full_r || !h_cs)))
        return (int)cudaErrorInvalidValue;
    return projection_enqueue(d_x, d_w, d_bias, d_out, d_rem_off, d_h, m, k, n, shift, h_u, h_v, h_ch, alpha, beta,
                              h_full_r, h_cs, d_proof, d_err, d_scratch, stream);
}

}  // extern "C"
