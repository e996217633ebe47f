// prove.cu -- exported entry points of the matmul GKR path: MLE evaluation,
// the degree-2 sumcheck, matmul::prove, the Op::MatMul arm and the
// single-shard MatMul prove of the BASELINE configuration 1.
#include <cstring>
#include <vector>

#include "../../include/zkie2.h"
#include "common.cuh"
#include "internal.h"

namespace zk {
int partial_eval_dev(const uint64_t* d_values, uint32_t t, const uint64_t* h_fix, uint32_t f,
                     uint64_t* d_out, uint64_t* d_scratch, cudaStream_t s);
int eval_dev(const uint64_t* d_values, uint32_t t, const uint64_t* h_point, uint64_t* d_out,
             uint64_t* d_scratch, cudaStream_t s);
uint64_t eval_scratch_elems(uint32_t t);
uint64_t sumcheck_scratch_elems(uint32_t t);
int sumcheck_dev(const uint64_t* d_f, const uint64_t* d_h, uint32_t t, const uint64_t* h_ch,
                 uint64_t* d_rounds, uint64_t* d_finals, uint64_t* d_scratch, cudaStream_t s);
int matmul_field_dev(const uint64_t* d_a, const uint64_t* d_b, uint64_t m, uint64_t k, uint64_t n,
                     uint64_t* d_c, cudaStream_t s);
int contract_rows_dev(const uint64_t* d_v, const uint64_t* d_eq, uint64_t R, uint64_t K, uint64_t* d_out,
                      uint64_t* d_part, cudaStream_t s);
uint64_t contract_rows_scratch_elems(uint64_t R, uint64_t K);
int eq_table_dev(const uint64_t* h_r, uint32_t d, uint64_t* d_out, cudaStream_t s);
int contract_dev(const uint64_t* v, const uint64_t* eq, uint64_t X, uint64_t Y, uint64_t* out,
                 cudaStream_t s);
int commit_device(const uint64_t* d_in, uint32_t lg_l, uint32_t lg_blowup, uint64_t w, uint64_t* d_lde,
                  uint64_t* d_layers, uint64_t* d_scratch, cudaStream_t s);
uint64_t sum_of_products_scratch_elems(uint32_t n, uint32_t t);
int sum_of_products_dev(const uint64_t* d_w, const uint64_t* d_v, uint32_t n, uint32_t t, const uint64_t* h_ch,
                        uint64_t* d_out, uint64_t* d_scratch, cudaStream_t s);

namespace {

bool pow2(uint64_t x) { return x && !(x & (x - 1)); }

// Device layout of a matmul proof: claimed | rounds (3 lk) | finals (2).
struct MatmulScratch {
    uint64_t *eq_u, *eq_v, *ar, *br, *eval_scr, *sc_scr, *rows_part, *out;
};

uint64_t matmul_scratch(uint64_t m, uint64_t k, uint64_t n, MatmulScratch* ms, uint64_t* base) {
    const uint32_t lm = log2_exact(m), lk = log2_exact(k), ln = log2_exact(n);
    uint64_t off = 0;
    auto take = [&](uint64_t** p, uint64_t cnt) {
        cnt = (cnt + 1) & ~1ull;  // keep 16-byte alignment
        if (base) *p = base + off;
        off += cnt;
    };
    MatmulScratch s{};
    take(&s.eq_u, m);
    take(&s.eq_v, n);
    take(&s.ar, k);
    take(&s.br, k);
    take(&s.eval_scr, eval_scratch_elems(ln + lm) + m);
    take(&s.sc_scr, sumcheck_scratch_elems(lk));
    take(&s.rows_part, contract_rows_scratch_elems(m, k));
    take(&s.out, 1 + 3 * lk + 2 + 8);
    if (ms) *ms = s;
    return off;
}

// matmul::prove body once a_r (k) is in ms.ar.  Leaves claimed|rounds|finals
// in ms.out on the device.
int matmul_core(const uint64_t* d_b, const uint64_t* d_c, uint64_t m, uint64_t k, uint64_t n,
                const uint64_t* u, const uint64_t* v, const uint64_t* ch, const MatmulScratch& ms,
                cudaStream_t s) {
    const uint32_t lm = log2_exact(m), lk = log2_exact(k), ln = log2_exact(n);
    // b_r = partial_eval(B, v): contract each row of B (n wide) with eq(v).
    int rc = partial_eval_dev(d_b, lk + ln, v, ln, ms.br, ms.eq_v, s);
    if (rc) return rc;
    // claimed = eval(C, v || u)
    std::vector<uint64_t> cp(ln + lm);
    for (uint32_t i = 0; i < ln; i++) cp[i] = v[i];
    for (uint32_t i = 0; i < lm; i++) cp[ln + i] = u[i];
    rc = eval_dev(d_c, ln + lm, cp.data(), ms.out, ms.eval_scr, s);
    if (rc) return rc;
    return sumcheck_dev(ms.ar, ms.br, lk, ch, ms.out + 1, ms.out + 1 + 3 * lk, ms.sc_scr, s);
}

int download_proof(const MatmulScratch& ms, uint32_t lk, uint64_t* claimed, uint64_t* rounds,
                   uint64_t* finals, cudaStream_t s) {
    std::vector<uint64_t> h(1 + 3 * lk + 2);
    ZK_TRY(cudaMemcpyAsync(h.data(), ms.out, 8 * h.size(), cudaMemcpyDeviceToHost, s));
    ZK_TRY(cudaStreamSynchronize(s));
    if (claimed) *claimed = h[0];
    if (rounds) std::memcpy(rounds, h.data() + 1, 8 * 3 * lk);
    if (finals) std::memcpy(finals, h.data() + 1 + 3 * lk, 16);
    return 0;
}

}  // namespace

uint64_t op_matmul_scratch_elems(uint64_t m, uint64_t k, uint64_t n) {
    return matmul_scratch(m, k, n, nullptr, nullptr);
}

// The Op::MatMul proof with host-drawn challenges u, v, ch, enqueued on s with
// no synchronization: claimed | rounds (3 lk) | finals (2) land at *d_out
// (a pointer into d_scratch).  Dimensions must be powers of two.
int op_matmul_enqueue(const uint64_t* d_a, const uint64_t* d_b, const uint64_t* d_c, uint64_t m, uint64_t k,
                      uint64_t n, const uint64_t* u, const uint64_t* v, const uint64_t* ch, uint64_t* d_scratch,
                      uint64_t** d_out, cudaStream_t s) {
    if (!pow2(m) || !pow2(k) || !pow2(n)) return (int)cudaErrorInvalidValue;
    const uint32_t lm = log2_exact(m);
    MatmulScratch ms;
    matmul_scratch(m, k, n, &ms, d_scratch);
    int rc = eq_table_dev(u, lm, ms.eq_u, s);
    if (rc) return rc;
    rc = contract_rows_dev(d_a, ms.eq_u, m, k, ms.ar, ms.rows_part, s);
    if (rc) return rc;
    rc = matmul_core(d_b, d_c, m, k, n, u, v, ch, ms, s);
    if (rc) return rc;
    *d_out = ms.out;
    return 0;
}

}  // namespace zk

using namespace zk;

extern "C" {

int zkie2_eq_evals(const uint64_t* h_r, uint32_t d, uint64_t* d_out, cudaStream_t stream) {
    if (!d_out || (d && !h_r)) return (int)cudaErrorInvalidValue;
    return eq_table_dev(h_r, d, d_out, stream);
}

uint64_t zkie2_mle_scratch_elems(uint32_t t) { return eval_scratch_elems(t) + (1ull << (t < 20 ? t : 20)); }

int zkie2_mle_partial_eval(const uint64_t* d_values, uint32_t t, const uint64_t* h_fix, uint32_t f,
                           uint64_t* d_out, uint64_t* d_scratch, cudaStream_t stream) {
    if (!d_values || !d_out || (f && (!h_fix || !d_scratch)) || f > t) return (int)cudaErrorInvalidValue;
    if (f > 20) {
        // Fix the first 20 variables at a time.
        uint64_t* tmp = d_scratch + (1ull << 20);
        int rc = partial_eval_dev(d_values, t, h_fix, 20, tmp, d_scratch, stream);
        if (rc) return rc;
        return zkie2_mle_partial_eval(tmp, t - 20, h_fix + 20, f - 20, d_out, d_scratch + (1ull << 20) + (1ull << (t - 20)), stream);
    }
    return partial_eval_dev(d_values, t, h_fix, f, d_out, d_scratch, stream);
}

int zkie2_mle_eval(const uint64_t* d_values, uint32_t t, const uint64_t* h_point, uint64_t* h_out,
                   uint64_t* d_scratch, cudaStream_t stream) {
    if (!d_values || !h_out || !d_scratch || (t && !h_point)) return (int)cudaErrorInvalidValue;
    uint64_t* d_out = d_scratch + eval_scratch_elems(t);
    int rc = eval_dev(d_values, t, h_point, d_out, d_scratch, stream);
    if (rc) return rc;
    ZK_TRY(cudaMemcpyAsync(h_out, d_out, 8, cudaMemcpyDeviceToHost, stream));
    ZK_TRY(cudaStreamSynchronize(stream));
    return 0;
}

int zkie2_mle_eval_async(const uint64_t* d_values, uint32_t t, const uint64_t* h_point, uint64_t* d_out,
                         uint64_t* d_scratch, cudaStream_t stream) {
    if (!d_values || !d_out || !d_scratch || (t && !h_point)) return (int)cudaErrorInvalidValue;
    return eval_dev(d_values, t, h_point, d_out, d_scratch, stream);
}

uint64_t zkie2_mle_eval_many_scratch_elems(uint32_t max_t) { return eval_scratch_elems(max_t); }

// eval of count tables at their points, one after another on the stream
// (the scratch is reused: the launches are ordered), values into d_out.
int zkie2_mle_eval_many(const uint64_t* const* d_values, const uint32_t* ts, const uint64_t* h_points,
                        uint32_t count, uint64_t* d_out, uint64_t* d_scratch, cudaStream_t stream) {
    if (count && (!d_values || !ts || !d_out || !d_scratch)) return (int)cudaErrorInvalidValue;
    uint64_t off = 0;
    for (uint32_t i = 0; i < count; i++) {
        if (!d_values[i] || ts[i] > 40 || (ts[i] && !h_points)) return (int)cudaErrorInvalidValue;
        int rc = eval_dev(d_values[i], ts[i], h_points + off, d_out + i, d_scratch, stream);
        if (rc) return rc;
        off += ts[i];
    }
    return 0;
}

uint64_t zkie2_sumcheck_scratch_elems(uint32_t t) { return sumcheck_scratch_elems(t) + 3ull * t + 4; }

int zkie2_sumcheck_prove(const uint64_t* d_f, const uint64_t* d_h, uint32_t t, const uint64_t* h_ch,
                         uint64_t* h_rounds, uint64_t* h_finals, uint64_t* d_scratch, cudaStream_t stream) {
    if (!d_f || !d_h || !h_finals || !d_scratch || (t && (!h_ch || !h_rounds)) || t > 40)
        return (int)cudaErrorInvalidValue;
    uint64_t* d_rounds = d_scratch + sumcheck_scratch_elems(t);
    uint64_t* d_finals = d_rounds + 3ull * t;
    int rc = sumcheck_dev(d_f, d_h, t, h_ch, d_rounds, d_finals, d_scratch, stream);
    if (rc) return rc;
    if (t) ZK_TRY(cudaMemcpyAsync(h_rounds, d_rounds, 24ull * t, cudaMemcpyDeviceToHost, stream));
    ZK_TRY(cudaMemcpyAsync(h_finals, d_finals, 16, cudaMemcpyDeviceToHost, stream));
    ZK_TRY(cudaStreamSynchronize(stream));
    return 0;
}

uint64_t zkie2_matmul_scratch_elems(uint64_t m, uint64_t k, uint64_t n) {
    if (!pow2(m) || !pow2(k) || !pow2(n)) return 0;
    return matmul_scratch(m, k, n, nullptr, nullptr);
}

// matmul::prove (crates/zkie-core/src/common/matmul.rs:17-46) with device
// tensors: at = A^T (k x m), b (k x n), c (m x n); u, v, ch on the host.
int zkie2_matmul_prove(const uint64_t* d_at, const uint64_t* d_b, const uint64_t* d_c, uint64_t m, uint64_t k,
                       uint64_t n, const uint64_t* h_u, const uint64_t* h_v, const uint64_t* h_ch,
                       uint64_t* h_claimed, uint64_t* h_rounds, uint64_t* h_finals, uint64_t* d_scratch,
                       cudaStream_t stream) {
    if (!pow2(m) || !pow2(k) || !pow2(n)) return (int)cudaErrorInvalidValue;
    if (!d_at || !d_b || !d_c || !d_scratch || !h_claimed || !h_finals) return (int)cudaErrorInvalidValue;
    MatmulScratch ms;
    matmul_scratch(m, k, n, &ms, d_scratch);
    const uint32_t lm = log2_exact(m), lk = log2_exact(k);
    // a_r = partial_eval(A^T, u)
    int rc = partial_eval_dev(d_at, lk + lm, h_u, lm, ms.ar, ms.eq_u, stream);
    if (rc) return rc;
    rc = matmul_core(d_b, d_c, m, k, n, h_u, h_v, h_ch, ms, stream);
    if (rc) return rc;
    return download_proof(ms, lk, h_claimed, h_rounds, h_finals, stream);
}

uint64_t zkie2_op_matmul_scratch_elems(uint64_t m, uint64_t k, uint64_t n) {
    return zkie2_matmul_scratch_elems(m, k, n);
}

// Op::MatMul arm of prove_shard_precomputed (zkie-ops/src/compose.rs:
// 1724-1747): draws u (log m), v (log n), ch (log k) from `src`, proves
// C = A @ B, and returns the three claims eval(A, ch||u), eval(B, v||ch),
// eval(C, v||u).  A is used directly (m x k); the transpose the reference
// materialises is folded into the contraction.  The claims on A and B equal
// the sumcheck's final f and h evaluations, and the claim on C equals the
// claimed sum, so no tensor is streamed a second time.
int zkie2_op_matmul_prove(const uint64_t* d_a, const uint64_t* d_b, const uint64_t* d_c, uint64_t m,
                          uint64_t k, uint64_t n, zkie2_challenger* src, uint64_t* out_u, uint64_t* out_v,
                          uint64_t* out_ch, uint64_t* out_claimed, uint64_t* out_rounds, uint64_t* out_finals,
                          uint64_t* out_claims, uint64_t* d_scratch, cudaStream_t stream) {
    if (!pow2(m) || !pow2(k) || !pow2(n)) return (int)cudaErrorInvalidValue;
    if (!d_a || !d_b || !d_c || !src || !d_scratch || !out_claimed || !out_finals || !out_claims)
        return (int)cudaErrorInvalidValue;
    const uint32_t lm = log2_exact(m), lk = log2_exact(k), ln = log2_exact(n);
    std::vector<uint64_t> u(lm), v(ln), ch(lk);
    for (auto& x : u) x = zkie2_challenger_field(src);
    for (auto& x : v) x = zkie2_challenger_field(src);
    for (auto& x : ch) x = zkie2_challenger_field(src);
    MatmulScratch ms;
    matmul_scratch(m, k, n, &ms, d_scratch);
    int rc = eq_table_dev(u.data(), lm, ms.eq_u, stream);
    if (rc) return rc;
    rc = contract_rows_dev(d_a, ms.eq_u, m, k, ms.ar, ms.rows_part, stream);
    if (rc) return rc;
    rc = matmul_core(d_b, d_c, m, k, n, u.data(), v.data(), ch.data(), ms, stream);
    if (rc) return rc;
    rc = download_proof(ms, lk, out_claimed, out_rounds, out_finals, stream);
    if (rc) return rc;
    if (out_u && lm) std::memcpy(out_u, u.data(), 8 * lm);
    if (out_v && ln) std::memcpy(out_v, v.data(), 8 * ln);
    if (out_ch && lk) std::memcpy(out_ch, ch.data(), 8 * lk);
    out_claims[0] = out_finals[0];
    out_claims[1] = out_finals[1];
    out_claims[2] = *out_claimed;
    return 0;
}

int zkie2_matmul_field(const uint64_t* d_a, const uint64_t* d_b, uint64_t m, uint64_t k, uint64_t n,
                       uint64_t* d_c, cudaStream_t stream) {
    if (!d_a || !d_b || !d_c) return (int)cudaErrorInvalidValue;
    return matmul_field_dev(d_a, d_b, m, k, n, d_c, stream);
}

// scratch of the batch sumcheck, then rounds (3t) and b_eval
uint64_t zkie2_sum_of_products_scratch_elems(uint32_t n_tables, uint32_t t) {
    if (n_tables == 0 || n_tables > 65535 || t > 40) return 0;
    return sum_of_products_scratch_elems(n_tables, t) + 3ull * t + 2;
}

// prove_sum_of_products (crates/zkie-core/src/common/sumcheck.rs:243-286).
int zkie2_sum_of_products_prove(const uint64_t* d_weights, const uint64_t* d_values, uint32_t n_tables, uint32_t t,
                                const uint64_t* h_ch, uint64_t* h_rounds, uint64_t* h_b_eval, uint64_t* d_scratch,
                                cudaStream_t stream) {
    if (!d_weights || !d_values || !h_b_eval || !d_scratch || n_tables == 0 || n_tables > 65535 || t > 40 ||
        (t && (!h_ch || !h_rounds)))
        return (int)cudaErrorInvalidValue;
    uint64_t* d_out = d_scratch + sum_of_products_scratch_elems(n_tables, t);
    int rc = sum_of_products_dev(d_weights, d_values, n_tables, t, h_ch, d_out, d_scratch, stream);
    if (rc) return rc;
    if (t) ZK_TRY(cudaMemcpyAsync(h_rounds, d_out, 24ull * t, cudaMemcpyDeviceToHost, stream));
    ZK_TRY(cudaMemcpyAsync(h_b_eval, d_out + 3ull * t, 8, cudaMemcpyDeviceToHost, stream));
    ZK_TRY(cudaStreamSynchronize(stream));
    return 0;
}

// The Op::MatMul proof with the caller's u, v, ch, no synchronization:
// claimed | rounds (3 log2 k) | finals (2) into d_proof on the device.
int zkie2_op_matmul_prove_async(const uint64_t* d_a, const uint64_t* d_b, const uint64_t* d_c, uint64_t m,
                                uint64_t k, uint64_t n, const uint64_t* h_u, const uint64_t* h_v,
                                const uint64_t* h_ch, uint64_t* d_proof, uint64_t* d_scratch, cudaStream_t stream) {
    if (!d_a || !d_b || !d_c || !d_proof || !d_scratch || !pow2(m) || !pow2(k) || !pow2(n))
        return (int)cudaErrorInvalidValue;
    const uint32_t lm = log2_exact(m), lk = log2_exact(k), ln = log2_exact(n);
    if ((lm && !h_u) || (ln && !h_v) || (lk && !h_ch)) return (int)cudaErrorInvalidValue;
    uint64_t* d_mm = nullptr;
    int rc = op_matmul_enqueue(d_a, d_b, d_c, m, k, n, h_u, h_v, h_ch, d_scratch, &d_mm, stream);
    if (rc) return rc;
    ZK_TRY(cudaMemcpyAsync(d_proof, d_mm, 8ull * (3 + 3ull * lk), cudaMemcpyDeviceToDevice, stream));
    return 0;
}

}  // extern "C"
