// ops.cu -- the op layer of zkie-ops on the device: the forward witness of
// the arms a GPT-2 model uses (crates/zkie-ops/src/compose.rs forward_ops,
// :1174-1583) and the columns their proofs read (the arms of
// prove_shard_precomputed, :1602-2091; layer_norm_centered.rs,
// layernorm_chain.rs, softmax_scaled.rs, topk.rs, common/same_poly.rs).
//
// Every tensor is a flat row-major array of field elements (u64, canonical on
// output) or of u32 lookup indices, as in the reference's Store.  Rows are
// independent in every row-wise arm (softmax, layer norms, row maxima), so
// those kernels run one block per row; the elementwise arms are grid-stride
// loops.  Fixed-point arithmetic follows fixed.cuh (wrapping i64, the
// reference's release-build semantics).  Data-dependent failures where the
// reference panics (an index outside a table, a zero softmax row sum) set a
// bit in the caller's device error word instead of faulting; the host reads
// it once after the forward pass.
#include <cstring>
#include <vector>

#include "../../include/zkie2.h"
#include "common.cuh"
#include "fixed.cuh"
#include "gl64.cuh"
#include "hist.cuh"
#include "internal.h"

namespace zk {

namespace {

constexpr int kOpThreads = 256;
constexpr int kRowThreads = 256;
constexpr int kRowWarps = kRowThreads / 32;

// error bits of the device error word
constexpr uint32_t kErrIndex = 1u;     // a lookup index at or past the end of its table
constexpr uint32_t kErrDivide = 2u;    // round_div by zero (or i64::MIN / -1)

unsigned ew_grid(uint64_t n) {
    const uint64_t b = ceil_div(n, kOpThreads);
    return (unsigned)(b < 148ull * 16 ? (b ? b : 1) : 148ull * 16);
}

unsigned row_grid(uint64_t m) { return (unsigned)(m < 65535ull * 16 ? m : 65535ull * 16); }

// ---- block reductions (one block of kRowThreads per row) ------------------------------
template <typename T, typename Op>
__device__ __forceinline__ T block_reduce(T v, Op op, T* sh) {
    for (int o = 16; o; o >>= 1) v = op(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();  // sh may still be read by a previous reduction
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    v = sh[0];
    for (int w = 1; w < kRowWarps; w++) v = op(v, sh[w]);
    return v;
}

struct FieldAdd {
    __device__ uint64_t operator()(uint64_t a, uint64_t b) const { return gl_add(a, b); }
};
struct WrapAdd {
    __device__ uint64_t operator()(uint64_t a, uint64_t b) const { return a + b; }
};
struct MaxI64 {
    __device__ int64_t operator()(int64_t a, int64_t b) const { return b > a ? b : a; }
};

// rsqrt_index (compose.rs:884-896): the piecewise index of a 2^32-scale variance
__device__ __forceinline__ uint32_t rsqrt_index(int64_t var) {
    constexpr int64_t kFine = 1ll << 20, kCoarse = 1ll << 22;
    constexpr int64_t kCoarseEnd = kFine + kCoarse * (1ll << 8);
    const int64_t raw = fx_round_div_pow2(var, 18);
    if (raw < kFine) return (uint32_t)(raw > 0 ? raw : 0);
    if (raw < kCoarseEnd) return (uint32_t)(kFine + ((raw - kFine) >> 8));
    return (uint32_t)fx_wadd(kFine + kCoarse, (raw - kCoarseEnd) >> 16);
}

// ---- elementwise arms -----------------------------------------------------------------
__global__ void k_field_add(const uint64_t* __restrict__ a, const uint64_t* __restrict__ b, uint64_t n,
                            uint64_t* __restrict__ out) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = gl_canon(gl_add(__ldg(a + i), __ldg(b + i)));
}

// Op::Scale: from_i64(round_div(to_i64(v) * factor, 2^shift))
__global__ void k_fixed_scale(const uint64_t* __restrict__ x, uint64_t n, int64_t factor, uint32_t shift,
                              uint64_t* __restrict__ out) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = fx_from_i64(fx_round_div_pow2(fx_wmul(fx_to_i64(__ldg(x + i)), factor), shift));
}

// Op::SoftmaxIndex: (max(to_i64(s), 0) as u64) % table_len
__global__ void k_softmax_index(const uint64_t* __restrict__ x, uint64_t n, uint64_t len,
                                uint32_t* __restrict__ idx) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const int64_t v = fx_to_i64(__ldg(x + i));
        idx[i] = (uint32_t)((uint64_t)(v > 0 ? v : 0) % len);
    }
}

__device__ __forceinline__ uint32_t clamp_index(int64_t v, uint64_t len) {
    const int64_t hi = (int64_t)len - 1;
    return (uint32_t)(v < 0 ? 0 : (v > hi ? hi : v));
}

// Op::GeluIndex: clamp(to_i64(v) + offset, 0, table_len - 1)
__global__ void k_gelu_index(const uint64_t* __restrict__ x, uint64_t n, int64_t offset, uint64_t len,
                             uint32_t* __restrict__ idx) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        idx[i] = clamp_index(fx_wadd(fx_to_i64(__ldg(x + i)), offset), len);
}

// Op::Lookup: out = table[idx]
__global__ void k_lookup_gather(const uint32_t* __restrict__ idx, uint64_t n, const uint64_t* __restrict__ table,
                                uint64_t t, uint64_t* __restrict__ out, uint32_t* __restrict__ err) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const uint32_t j = __ldg(idx + i);
        if (j < t) {
            out[i] = __ldg(table + j);
        } else {
            out[i] = 0;
            atomicOr(err, kErrIndex);
        }
    }
}

// x (m x k) -> out (k x m), 32 x 32 tiles through shared memory
__global__ void k_transpose(const uint64_t* __restrict__ x, uint64_t m, uint64_t k, uint64_t* __restrict__ out) {
    __shared__ uint64_t tile[32][33];
    const uint64_t c0 = (uint64_t)blockIdx.x * 32, r0 = (uint64_t)blockIdx.y * 32;
    for (int dy = threadIdx.y; dy < 32; dy += blockDim.y) {
        const uint64_t r = r0 + dy, c = c0 + threadIdx.x;
        if (r < m && c < k) tile[dy][threadIdx.x] = __ldg(x + r * k + c);
    }
    __syncthreads();
    for (int dy = threadIdx.y; dy < 32; dy += blockDim.y) {
        const uint64_t c = c0 + dy, r = r0 + threadIdx.x;
        if (r < m && c < k) out[c * m + r] = tile[threadIdx.x][dy];
    }
}

__global__ void k_fill(uint64_t* __restrict__ out, uint64_t n, uint64_t v) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) out[i] = v;
}

// ---- row-wise arms (one block per row) ------------------------------------------------------
// out[r * n + j] = v[r]
__global__ void k_row_broadcast(const uint64_t* __restrict__ v, uint64_t m, uint64_t n, uint64_t* __restrict__ out) {
    for (uint64_t r = blockIdx.x; r < m; r += gridDim.x) {
        const uint64_t x = gl_canon(__ldg(v + r));
        for (uint64_t j = threadIdx.x; j < n; j += blockDim.x) out[r * n + j] = x;
    }
}

// out[r] = sum_{j < ncols} x[r * d + j] over the field
__global__ void __launch_bounds__(kRowThreads) k_row_sums(const uint64_t* __restrict__ x, uint64_t m, uint64_t d,
                                                          uint64_t ncols, uint64_t* __restrict__ out) {
    __shared__ uint64_t sh[kRowWarps];
    for (uint64_t r = blockIdx.x; r < m; r += gridDim.x) {
        uint64_t s = 0;
        for (uint64_t j = threadIdx.x; j < ncols; j += blockDim.x) s = gl_add(s, __ldg(x + r * d + j));
        s = block_reduce(s, FieldAdd{}, sh);
        if (threadIdx.x == 0) out[r] = gl_canon(s);
    }
}

// Op::StableSoftmaxIndex: masked = x + mask, row max by to_i64, index =
// clamp(to_i64(masked) - to_i64(row max) + offset, 0, table_len - 1)
__global__ void __launch_bounds__(kRowThreads) k_stable_softmax_index(const uint64_t* __restrict__ x,
                                                                      const uint64_t* __restrict__ mask, uint64_t m,
                                                                      uint64_t n, int64_t offset, uint64_t len,
                                                                      uint32_t* __restrict__ idx) {
    __shared__ int64_t sh[kRowWarps];
    for (uint64_t r = blockIdx.x; r < m; r += gridDim.x) {
        const uint64_t* xr = x + r * n;
        const uint64_t* mr = mask + r * n;
        int64_t mx = INT64_MIN;
        for (uint64_t j = threadIdx.x; j < n; j += blockDim.x) {
            const int64_t v = fx_to_i64(gl_canon(gl_add(__ldg(xr + j), __ldg(mr + j))));
            mx = v > mx ? v : mx;
        }
        mx = block_reduce(mx, MaxI64{}, sh);
        for (uint64_t j = threadIdx.x; j < n; j += blockDim.x) {
            const int64_t v = fx_to_i64(gl_canon(gl_add(__ldg(xr + j), __ldg(mr + j))));
            idx[r * n + j] = clamp_index(fx_wadd(fx_wsub(v, mx), offset), len);
        }
    }
}

// Op::Softmax: e = table[idx], sum = the row's field sum, out =
// from_i64(round_div(to_i64(e) * 2^16, to_i64(sum)))
__global__ void __launch_bounds__(kRowThreads) k_softmax_fwd(const uint32_t* __restrict__ idx,
                                                             const uint64_t* __restrict__ table, uint64_t t,
                                                             uint64_t m, uint64_t n, uint64_t* __restrict__ e,
                                                             uint64_t* __restrict__ out, uint64_t* __restrict__ sum,
                                                             uint32_t* __restrict__ err) {
    __shared__ uint64_t sh[kRowWarps];
    for (uint64_t r = blockIdx.x; r < m; r += gridDim.x) {
        uint64_t s = 0;
        for (uint64_t j = threadIdx.x; j < n; j += blockDim.x) {
            const uint32_t k = __ldg(idx + r * n + j);
            uint64_t v = 0;
            if (k < t)
                v = __ldg(table + k);
            else
                atomicOr(err, kErrIndex);
            e[r * n + j] = v;
            s = gl_add(s, v);
        }
        s = gl_canon(block_reduce(s, FieldAdd{}, sh));
        if (sum && threadIdx.x == 0) sum[r] = s;
        const int64_t si = fx_to_i64(s);
        for (uint64_t j = threadIdx.x; j < n; j += blockDim.x) {
            int64_t q = 0;
            if (!fx_round_div(fx_wmul(fx_to_i64(e[r * n + j]), 1ll << 16), si, &q)) atomicOr(err, kErrDivide);
            out[r * n + j] = fx_from_i64(q);
        }
    }
}

// sum_b = the row sum broadcast, rem = from_i64(to_i64(e) 2^16 - to_i64(out) to_i64(sum_b))
// (prove_softmax_rounded, softmax_scaled.rs:69-80)
__global__ void k_softmax_rem(const uint64_t* __restrict__ e, const uint64_t* __restrict__ out,
                              const uint64_t* __restrict__ sum, uint64_t m, uint64_t n, uint64_t* __restrict__ sum_b,
                              uint64_t* __restrict__ rem) {
    for (uint64_t r = blockIdx.x; r < m; r += gridDim.x) {
        const uint64_t s = gl_canon(__ldg(sum + r));
        const int64_t si = fx_to_i64(s);
        for (uint64_t j = threadIdx.x; j < n; j += blockDim.x) {
            const uint64_t i = r * n + j;
            sum_b[i] = s;
            rem[i] = fx_from_i64(fx_wsub(fx_wmul(fx_to_i64(__ldg(e + i)), 1ll << 16),
                                         fx_wmul(fx_to_i64(__ldg(out + i)), si)));
        }
    }
}

// The outputs of layer_norm_forward (layer_norm_centered.rs:42-120), one
// block per row of d values of which the first n_real are real.
struct LncOut {
    uint64_t *mean, *centered, *var, *rstd, *raw, *out, *rem_out, *sum_mean, *rem_mean, *sum_var, *rem_var;
    uint32_t* s_index;
};

__global__ void __launch_bounds__(kRowThreads) k_ln_centered_fwd(const uint64_t* __restrict__ x,
                                                                 const uint64_t* __restrict__ w,
                                                                 const uint64_t* __restrict__ b,
                                                                 const uint64_t* __restrict__ table, uint64_t t,
                                                                 uint64_t m, uint64_t d, uint64_t n_real, LncOut o,
                                                                 uint32_t* __restrict__ err) {
    __shared__ uint64_t sh[kRowWarps];
    const int64_t nr = (int64_t)n_real;
    for (uint64_t r = blockIdx.x; r < m; r += gridDim.x) {
        const uint64_t* xr = x + r * d;
        // mean = round_div(sum of to_i64(x), n_real); sum_mean = the field sum
        uint64_t si = 0, sf = 0;
        for (uint64_t j = threadIdx.x; j < n_real; j += blockDim.x) {
            const uint64_t v = __ldg(xr + j);
            si += (uint64_t)fx_to_i64(v);
            sf = gl_add(sf, v);
        }
        si = block_reduce(si, WrapAdd{}, sh);
        sf = gl_canon(block_reduce(sf, FieldAdd{}, sh));
        int64_t mq = 0;
        fx_round_div((int64_t)si, nr, &mq);
        const uint64_t mean = fx_from_i64(mq);
        // centered = x - mean (every column); var from the first n_real
        uint64_t qi = 0, qf = 0;
        for (uint64_t j = threadIdx.x; j < d; j += blockDim.x) {
            const uint64_t c = gl_canon(gl_sub(__ldg(xr + j), mean));
            o.centered[r * d + j] = c;
            if (j < n_real) {
                const int64_t ci = fx_to_i64(c);
                qi += (uint64_t)fx_wmul(ci, ci);
                qf = gl_add(qf, gl_mul(c, c));
            }
        }
        qi = block_reduce(qi, WrapAdd{}, sh);
        qf = gl_canon(block_reduce(qf, FieldAdd{}, sh));
        int64_t vq = 0;
        fx_round_div((int64_t)qi, nr, &vq);
        const uint64_t var = fx_from_i64(vq);
        const uint32_t sidx = rsqrt_index(fx_to_i64(var));
        uint64_t rstd = 0;
        if (sidx < t)
            rstd = __ldg(table + sidx);
        else if (threadIdx.x == 0)
            atomicOr(err, kErrIndex);
        if (threadIdx.x == 0) {
            const int64_t half = nr / 2;
            o.mean[r] = mean;
            o.var[r] = var;
            o.s_index[r] = sidx;
            o.rstd[r] = rstd;
            o.sum_mean[r] = sf;
            o.rem_mean[r] = fx_from_i64(fx_wadd(fx_wsub(fx_to_i64(sf), fx_wmul(fx_to_i64(mean), nr)), half));
            o.sum_var[r] = qf;
            o.rem_var[r] = fx_from_i64(fx_wadd(fx_wsub(fx_to_i64(qf), fx_wmul(fx_to_i64(var), nr)), half));
        }
        // raw = centered rstd w; out = round_div(to_i64(raw), 2^32) + to_i64(b);
        // rem_out = to_i64(raw) - (to_i64(out) - to_i64(b)) 2^32 + 2^31
        for (uint64_t j = threadIdx.x; j < d; j += blockDim.x) {
            const uint64_t i = r * d + j;
            const uint64_t c = gl_canon(gl_sub(__ldg(xr + j), mean));
            const uint64_t raw = gl_canon(gl_mul(gl_mul(c, rstd), __ldg(w + i)));
            const int64_t ri = fx_to_i64(raw), bi = fx_to_i64(__ldg(b + i));
            const uint64_t out = fx_from_i64(fx_wadd(fx_round_div_pow2(ri, 32), bi));
            o.raw[i] = raw;
            o.out[i] = out;
            o.rem_out[i] =
                fx_from_i64(fx_wadd(fx_wsub(ri, fx_wmul(fx_wsub(fx_to_i64(out), bi), 1ll << 32)), 1ll << 31));
        }
    }
}

// The RmsNorm arm (rms_norm.rs:37-95), one block per row: ms =
// round_div(sum of to_i64(x)^2 over n_real, n_real) in wrapping i64, rstd =
// table[rsqrt_index(ms)], raw = x rstd w (field), out = round_div(to_i64(raw),
// 2^32), rem_out = to_i64(raw) - to_i64(out) 2^32 + 2^31 split into rem_lo =
// rem_out & 0xFFFF and rem_hi = rem_out >> 16 (arithmetic); sum_sq = the
// field sum of x^2 over n_real, rem_s = sum_sq - ms n_real + n_real / 2.
struct RmsOut {
    uint64_t *ms, *rstd, *raw, *out, *rem_out, *rem_lo, *rem_hi, *sum_sq, *rem_s;
    uint32_t* s_index;
};

__global__ void __launch_bounds__(kRowThreads) k_rms_norm_fwd(const uint64_t* __restrict__ x,
                                                              const uint64_t* __restrict__ w,
                                                              const uint64_t* __restrict__ table, uint64_t t,
                                                              uint64_t m, uint64_t d, uint64_t n_real, RmsOut o,
                                                              uint32_t* __restrict__ err) {
    __shared__ uint64_t sh[kRowWarps];
    const int64_t nr = (int64_t)n_real;
    for (uint64_t r = blockIdx.x; r < m; r += gridDim.x) {
        const uint64_t* xr = x + r * d;
        uint64_t qi = 0, qf = 0;
        for (uint64_t j = threadIdx.x; j < n_real; j += blockDim.x) {
            const uint64_t v = gl_canon(__ldg(xr + j));
            const int64_t vi = fx_to_i64(v);
            qi += (uint64_t)fx_wmul(vi, vi);
            qf = gl_add(qf, gl_mul(v, v));
        }
        qi = block_reduce(qi, WrapAdd{}, sh);
        qf = gl_canon(block_reduce(qf, FieldAdd{}, sh));
        int64_t q = 0;
        fx_round_div((int64_t)qi, nr, &q);
        const uint64_t ms = fx_from_i64(q);
        const uint32_t sidx = rsqrt_index(fx_to_i64(ms));
        uint64_t rstd = 0;
        if (sidx < t)
            rstd = __ldg(table + sidx);
        else if (threadIdx.x == 0)
            atomicOr(err, kErrIndex);
        if (threadIdx.x == 0) {
            o.ms[r] = ms;
            o.s_index[r] = sidx;
            o.rstd[r] = rstd;
            o.sum_sq[r] = qf;
            o.rem_s[r] = fx_from_i64(fx_wadd(fx_wsub(fx_to_i64(qf), fx_wmul(fx_to_i64(ms), nr)), nr / 2));
        }
        for (uint64_t j = threadIdx.x; j < d; j += blockDim.x) {
            const uint64_t i = r * d + j;
            const uint64_t raw = gl_canon(gl_mul(gl_mul(__ldg(xr + j), rstd), __ldg(w + i)));
            const int64_t ri = fx_to_i64(raw);
            const int64_t oi = fx_round_div_pow2(ri, 32);
            const int64_t rem = fx_wadd(fx_wsub(ri, fx_wmul(oi, 1ll << 32)), 1ll << 31);
            o.raw[i] = raw;
            o.out[i] = fx_from_i64(oi);
            o.rem_out[i] = fx_from_i64(rem);
            o.rem_lo[i] = fx_from_i64(rem & 0xFFFF);
            o.rem_hi[i] = fx_from_i64(rem >> 16);
        }
    }
}

// The Layernorm arm (compose.rs:1467-1496, layernorm_chain.rs:34-44):
// mean_sq = sum_j x^2, idx = max(to_i64(mean_sq), 0) % len, rsqrt =
// table[idx], scale = rsqrt w, out = x scale + b
__global__ void __launch_bounds__(kRowThreads) k_layernorm_fwd(const uint64_t* __restrict__ x,
                                                               const uint64_t* __restrict__ w,
                                                               const uint64_t* __restrict__ b,
                                                               const uint64_t* __restrict__ table, uint64_t t,
                                                               uint64_t m, uint64_t d, uint64_t* __restrict__ mean_sq,
                                                               uint32_t* __restrict__ ridx,
                                                               uint64_t* __restrict__ rsqrt,
                                                               uint64_t* __restrict__ scale,
                                                               uint64_t* __restrict__ out) {
    __shared__ uint64_t sh[kRowWarps];
    for (uint64_t r = blockIdx.x; r < m; r += gridDim.x) {
        uint64_t s = 0;
        for (uint64_t j = threadIdx.x; j < d; j += blockDim.x) {
            const uint64_t v = __ldg(x + r * d + j);
            s = gl_add(s, gl_mul(v, v));
        }
        s = gl_canon(block_reduce(s, FieldAdd{}, sh));
        const int64_t si = fx_to_i64(s);
        const uint32_t k = (uint32_t)((uint64_t)(si > 0 ? si : 0) % t);
        const uint64_t rs = __ldg(table + k);
        if (threadIdx.x == 0) {
            mean_sq[r] = s;
            ridx[r] = k;
            rsqrt[r] = rs;
        }
        for (uint64_t j = threadIdx.x; j < d; j += blockDim.x) {
            const uint64_t i = r * d + j;
            const uint64_t sc = gl_canon(gl_mul(rs, __ldg(w + i)));
            scale[i] = sc;
            out[i] = gl_canon(gl_add(gl_mul(__ldg(x + i), sc), __ldg(b + i)));
        }
    }
}

// ---- same_poly (common/same_poly.rs:13-45) ------------------------------------------------
// E(x) = sum_i c_i eq(r_i, x): the claims' eq tables combined with their
// batching coefficients.  Since every term of the reference's virtual
// polynomial is c_i f eq_i, its round messages equal those of f E.  Each eq
// splits into a low table over tl bits and a high table over th bits (the
// high one scaled by c_i), so an output costs two loads and one product per
// claim.
// Points and coefficients of up to kEqChunk claims, passed by value so the
// launch needs no host-to-device copy (and can be recorded in a CUDA graph).
constexpr int kEqChunk = 8;
constexpr int kEqMaxVars = 40;
struct EqChunk {
    uint64_t r[kEqChunk][kEqMaxVars];
    uint64_t coeff[kEqChunk];
};

__global__ void k_eq_split_tables(EqChunk ck, uint32_t c, uint32_t t, uint32_t tl, uint64_t* __restrict__ tabs) {
    const uint32_t th = t - tl;
    const uint64_t nl = 1ull << tl, nh = 1ull << th, per = nl + nh;
    const uint64_t total = per * c;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t g = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += stride) {
        const uint64_t ci = g / per, e = g % per;
        uint64_t v;
        uint32_t bits, base;
        uint64_t x;
        if (e < nl) {
            v = 1;
            bits = tl;
            base = 0;
            x = e;
        } else {
            v = gl_canon(ck.coeff[ci]);
            bits = th;
            base = tl;
            x = e - nl;
        }
        for (uint32_t j = 0; j < bits; j++) {
            const uint64_t rj = gl_canon(ck.r[ci][base + j]);
            v = gl_mul(v, ((x >> j) & 1) ? rj : gl_sub(1, rj));
        }
        tabs[g] = gl_canon(v);
    }
}

__global__ void k_eq_combine(const uint64_t* __restrict__ tabs, uint32_t c, uint32_t tl, uint32_t th,
                             uint64_t n, uint64_t* __restrict__ out) {
    const uint64_t nl = 1ull << tl, per = nl + (1ull << th), lmask = nl - 1;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t x = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; x < n; x += stride) {
        uint64_t s = 0;
        const uint64_t lo = x & lmask, hi = x >> tl;
        for (uint32_t i = 0; i < c; i++) {
            const uint64_t* tb = tabs + (uint64_t)i * per;
            s = gl_add(s, gl_mul(__ldg(tb + lo), __ldg(tb + nl + hi)));
        }
        out[x] = gl_canon(s);
    }
}

// ---- lookup multiplicities (common/logup_gkr.rs:251-260) ----------------------------------
__global__ void k_multiplicity(const uint32_t* __restrict__ x, uint64_t n, uint64_t t,
                               unsigned long long* __restrict__ m, uint32_t* __restrict__ err) {
    hist_grid(x, n, t, m, err, kErrIndex);
}

// ---- top-k selection and argmax (topk.rs:41-80, 272-297) -----------------------------------
constexpr uint64_t kTopkMaxCols = 4096;  // a row held in shared memory when k > 1

// topk_forward's order within a row: the larger value (to_i64) first, the
// smaller position first among equal values
__device__ __forceinline__ bool ranks_before(int64_t va, uint64_t ja, int64_t vb, uint64_t jb) {
    return va > vb || (va == vb && ja < jb);
}

// Op::TopKSelect / Op::Argmax forward, one block per row: thr = the k-th
// entry in that order, sel = 1 on the first k entries, gate = x sel, d1 =
// sel (x - thr), d2 = (1 - sel) (thr - x) in wrapping i64; out[r] (given for
// k = 1) = the row's first position of its maximum.  k = 1 is a block
// reduction over any row length; k > 1 ranks every entry of a row of at most
// kTopkMaxCols held in shared memory (writing sel in that pass).
__global__ void __launch_bounds__(kRowThreads) k_topk_rows(const uint64_t* __restrict__ x, uint64_t m, uint64_t n,
                                                           uint64_t k, uint64_t* __restrict__ thr,
                                                           uint64_t* __restrict__ sel, uint64_t* __restrict__ gate,
                                                           uint64_t* __restrict__ d1, uint64_t* __restrict__ d2,
                                                           uint32_t* __restrict__ out) {
    extern __shared__ int64_t row[];
    __shared__ int64_t sv[kRowWarps];
    __shared__ uint64_t sj[kRowWarps];
    __shared__ uint64_t s_kth;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (uint64_t r = blockIdx.x; r < m; r += gridDim.x) {
        const uint64_t* xr = x + r * n;
        uint64_t tj;
        __syncthreads();  // the previous row's shared values are no longer read
        if (k == 1) {
            int64_t bv = INT64_MIN;
            uint64_t bj = UINT64_MAX;  // ranks after every entry
            for (uint64_t j = threadIdx.x; j < n; j += blockDim.x) {
                const int64_t v = fx_to_i64(gl_canon(__ldg(xr + j)));
                if (ranks_before(v, j, bv, bj)) {
                    bv = v;
                    bj = j;
                }
            }
            for (int o = 16; o; o >>= 1) {
                const int64_t ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
                const uint64_t oj = __shfl_xor_sync(0xFFFFFFFFu, bj, o);
                if (ranks_before(ov, oj, bv, bj)) {
                    bv = ov;
                    bj = oj;
                }
            }
            if (lane == 0) {
                sv[warp] = bv;
                sj[warp] = bj;
            }
            __syncthreads();
            bv = sv[0];
            bj = sj[0];
            for (int w = 1; w < kRowWarps; w++) {
                if (ranks_before(sv[w], sj[w], bv, bj)) {
                    bv = sv[w];
                    bj = sj[w];
                }
            }
            tj = bj;
        } else {
            for (uint64_t j = threadIdx.x; j < n; j += blockDim.x) row[j] = fx_to_i64(gl_canon(__ldg(xr + j)));
            __syncthreads();
            for (uint64_t j = threadIdx.x; j < n; j += blockDim.x) {
                const int64_t v = row[j];
                uint64_t rank = 0;
                for (uint64_t i = 0; i < n; i++) rank += ranks_before(row[i], i, v, j) ? 1 : 0;
                sel[r * n + j] = rank < k ? 1 : 0;
                if (rank == k - 1) s_kth = j;
            }
            __syncthreads();
            tj = s_kth;
        }
        const uint64_t tval = gl_canon(__ldg(xr + tj));
        const int64_t ti = fx_to_i64(tval);
        if (threadIdx.x == 0) {
            thr[r] = tval;
            if (out) out[r] = (uint32_t)tj;
        }
        for (uint64_t j = threadIdx.x; j < n; j += blockDim.x) {
            const uint64_t o = r * n + j;
            const uint64_t xv = gl_canon(__ldg(xr + j));
            const int64_t xi = fx_to_i64(xv);
            const bool s = k == 1 ? j == tj : sel[o] != 0;  // k > 1: this thread's own write above
            if (k == 1) sel[o] = s ? 1 : 0;
            gate[o] = s ? xv : 0;
            d1[o] = s ? fx_from_i64(fx_wsub(xi, ti)) : 0;
            d2[o] = s ? 0 : fx_from_i64(fx_wsub(ti, xi));
        }
    }
}

// The lookup columns of prove_topk (topk.rs:141-154) and prove_range_decomp
// (:395-419): to_i32(v) as u32 of sel and d1, and the three 16-bit limbs of
// to_i64(d2) as u64 (values and indices, limb c at offset c n)
__global__ void k_topk_limbs(const uint64_t* __restrict__ sel, const uint64_t* __restrict__ d1,
                             const uint64_t* __restrict__ d2, uint64_t n, uint32_t* __restrict__ sel_idx,
                             uint32_t* __restrict__ d1_idx, uint64_t* __restrict__ limbs,
                             uint32_t* __restrict__ limb_idx) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        sel_idx[i] = fx_to_i32_index(__ldg(sel + i));
        d1_idx[i] = fx_to_i32_index(__ldg(d1 + i));
        const uint64_t v = (uint64_t)fx_to_i64(gl_canon(__ldg(d2 + i)));
        for (int c = 0; c < 3; c++) {
            const uint64_t l = (v >> (16 * c)) & 0xFFFFull;
            limbs[c * n + i] = l;
            limb_idx[c * n + i] = (uint32_t)l;
        }
    }
}

__global__ void k_iota(uint64_t* __restrict__ out, uint64_t n) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) out[i] = i;
}

}  // namespace

}  // namespace zk

using namespace zk;

extern "C" {

int zkie2_op_add(const uint64_t* d_a, const uint64_t* d_b, uint64_t n, uint64_t* d_out, cudaStream_t stream) {
    if (n == 0) return 0;
    if (!d_a || !d_b || !d_out) return (int)cudaErrorInvalidValue;
    k_field_add<<<ew_grid(n), kOpThreads, 0, stream>>>(d_a, d_b, n, d_out);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_scale(const uint64_t* d_x, uint64_t n, int64_t factor, uint32_t shift, uint64_t* d_out,
                   cudaStream_t stream) {
    if (shift > 62) return (int)cudaErrorInvalidValue;
    if (n == 0) return 0;
    if (!d_x || !d_out) return (int)cudaErrorInvalidValue;
    k_fixed_scale<<<ew_grid(n), kOpThreads, 0, stream>>>(d_x, n, factor, shift, d_out);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_transpose(const uint64_t* d_x, uint64_t m, uint64_t k, uint64_t* d_out, cudaStream_t stream) {
    if (m == 0 || k == 0) return 0;
    if (!d_x || !d_out || ceil_div(k, 32) > 0x7FFFFFFFull || ceil_div(m, 32) > 65535) return (int)cudaErrorInvalidValue;
    k_transpose<<<dim3((unsigned)ceil_div(k, 32), (unsigned)ceil_div(m, 32)), dim3(32, 8), 0, stream>>>(d_x, m, k,
                                                                                                         d_out);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_softmax_index(const uint64_t* d_x, uint64_t n, uint64_t table_len, uint32_t* d_idx,
                           cudaStream_t stream) {
    if (table_len == 0) return (int)cudaErrorInvalidValue;
    if (n == 0) return 0;
    if (!d_x || !d_idx) return (int)cudaErrorInvalidValue;
    k_softmax_index<<<ew_grid(n), kOpThreads, 0, stream>>>(d_x, n, table_len, d_idx);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_gelu_index(const uint64_t* d_x, uint64_t n, int64_t offset, uint64_t table_len, uint32_t* d_idx,
                        cudaStream_t stream) {
    if (table_len == 0 || table_len > 0xFFFFFFFFull) return (int)cudaErrorInvalidValue;
    if (n == 0) return 0;
    if (!d_x || !d_idx) return (int)cudaErrorInvalidValue;
    k_gelu_index<<<ew_grid(n), kOpThreads, 0, stream>>>(d_x, n, offset, table_len, d_idx);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_stable_softmax_index(const uint64_t* d_x, const uint64_t* d_mask, uint64_t m, uint64_t n,
                                  int64_t offset, uint64_t table_len, uint32_t* d_idx, cudaStream_t stream) {
    if (table_len == 0 || table_len > 0xFFFFFFFFull) return (int)cudaErrorInvalidValue;
    if (m == 0 || n == 0) return 0;
    if (!d_x || !d_mask || !d_idx) return (int)cudaErrorInvalidValue;
    k_stable_softmax_index<<<row_grid(m), kRowThreads, 0, stream>>>(d_x, d_mask, m, n, offset, table_len, d_idx);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_lookup(const uint32_t* d_idx, uint64_t n, const uint64_t* d_table, uint64_t t, uint64_t* d_out,
                    uint32_t* d_err, cudaStream_t stream) {
    if (n == 0) return 0;
    if (!d_idx || !d_table || !d_out || !d_err) return (int)cudaErrorInvalidValue;
    k_lookup_gather<<<ew_grid(n), kOpThreads, 0, stream>>>(d_idx, n, d_table, t, d_out, d_err);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_softmax(const uint32_t* d_idx, const uint64_t* d_table, uint64_t t, uint64_t m, uint64_t n,
                     uint64_t* d_e, uint64_t* d_out, uint64_t* d_sum, uint32_t* d_err, cudaStream_t stream) {
    if (m == 0 || n == 0) return 0;
    if (!d_idx || !d_table || !d_e || !d_out || !d_err) return (int)cudaErrorInvalidValue;
    k_softmax_fwd<<<row_grid(m), kRowThreads, 0, stream>>>(d_idx, d_table, t, m, n, d_e, d_out, d_sum, d_err);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_softmax_rem(const uint64_t* d_e, const uint64_t* d_out, const uint64_t* d_sum, uint64_t m, uint64_t n,
                         uint64_t* d_sum_b, uint64_t* d_rem, cudaStream_t stream) {
    if (m == 0 || n == 0) return 0;
    if (!d_e || !d_out || !d_sum || !d_sum_b || !d_rem) return (int)cudaErrorInvalidValue;
    k_softmax_rem<<<row_grid(m), kRowThreads, 0, stream>>>(d_e, d_out, d_sum, m, n, d_sum_b, d_rem);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_layer_norm_centered(const uint64_t* d_x, const uint64_t* d_w, const uint64_t* d_b,
                                 const uint64_t* d_table, uint64_t t, uint64_t m, uint64_t d, uint64_t n_real,
                                 uint64_t* const* d_outs, uint32_t* d_s_index, uint32_t* d_err, cudaStream_t stream) {
    if (m == 0 || d == 0) return 0;
    if (n_real == 0 || n_real > d || !d_x || !d_w || !d_b || !d_table || !d_outs || !d_s_index || !d_err)
        return (int)cudaErrorInvalidValue;
    for (int i = 0; i < 11; i++)
        if (!d_outs[i]) return (int)cudaErrorInvalidValue;
    LncOut o{d_outs[0], d_outs[1], d_outs[2], d_outs[3], d_outs[4],  d_outs[5],
             d_outs[6], d_outs[7], d_outs[8], d_outs[9], d_outs[10], d_s_index};
    k_ln_centered_fwd<<<row_grid(m), kRowThreads, 0, stream>>>(d_x, d_w, d_b, d_table, t, m, d, n_real, o, d_err);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_layernorm(const uint64_t* d_x, const uint64_t* d_w, const uint64_t* d_b, const uint64_t* d_table,
                       uint64_t t, uint64_t m, uint64_t d, uint64_t* d_mean_sq, uint32_t* d_idx, uint64_t* d_rsqrt,
                       uint64_t* d_scale, uint64_t* d_out, cudaStream_t stream) {
    if (m == 0 || d == 0) return 0;
    if (t == 0 || !d_x || !d_w || !d_b || !d_table || !d_mean_sq || !d_idx || !d_rsqrt || !d_scale || !d_out)
        return (int)cudaErrorInvalidValue;
    k_layernorm_fwd<<<row_grid(m), kRowThreads, 0, stream>>>(d_x, d_w, d_b, d_table, t, m, d, d_mean_sq, d_idx,
                                                             d_rsqrt, d_scale, d_out);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_row_broadcast(const uint64_t* d_v, uint64_t m, uint64_t n, uint64_t* d_out, cudaStream_t stream) {
    if (m == 0 || n == 0) return 0;
    if (!d_v || !d_out) return (int)cudaErrorInvalidValue;
    k_row_broadcast<<<row_grid(m), kRowThreads, 0, stream>>>(d_v, m, n, d_out);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_row_sums(const uint64_t* d_x, uint64_t m, uint64_t d, uint64_t ncols, uint64_t* d_out,
                      cudaStream_t stream) {
    if (m == 0) return 0;
    if (ncols > d || !d_x || !d_out) return (int)cudaErrorInvalidValue;
    k_row_sums<<<row_grid(m), kRowThreads, 0, stream>>>(d_x, m, d, ncols, d_out);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_rms_norm(const uint64_t* d_x, const uint64_t* d_w, const uint64_t* d_table, uint64_t t, uint64_t m,
                      uint64_t d, uint64_t n_real, uint64_t* const* d_outs, uint32_t* d_s_index, uint32_t* d_err,
                      cudaStream_t stream) {
    if (n_real == 0 || n_real > d) return (int)cudaErrorInvalidValue;
    if (m == 0 || d == 0) return 0;
    if (!d_x || !d_w || !d_table || !d_outs || !d_s_index || !d_err) return (int)cudaErrorInvalidValue;
    for (int i = 0; i < 9; i++)
        if (!d_outs[i]) return (int)cudaErrorInvalidValue;
    RmsOut o{d_outs[0], d_outs[1], d_outs[2], d_outs[3], d_outs[4], d_outs[5], d_outs[6], d_outs[7], d_outs[8],
             d_s_index};
    k_rms_norm_fwd<<<row_grid(m), kRowThreads, 0, stream>>>(d_x, d_w, d_table, t, m, d, n_real, o, d_err);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_topk(const uint64_t* d_x, uint64_t m, uint64_t n, uint64_t k, uint64_t* d_thr, uint64_t* d_sel,
                  uint64_t* d_gate, uint64_t* d_d1, uint64_t* d_d2, uint32_t* d_out, cudaStream_t stream) {
    if (k == 0 || k > n || (k > 1 && (n > kTopkMaxCols || d_out)) || n > 0xFFFFFFFFull)
        return (int)cudaErrorInvalidValue;
    if (m == 0) return 0;
    if (!d_x || !d_thr || !d_sel || !d_gate || !d_d1 || !d_d2) return (int)cudaErrorInvalidValue;
    const size_t shared = k > 1 ? 8 * n : 0;
    k_topk_rows<<<row_grid(m), kRowThreads, shared, stream>>>(d_x, m, n, k, d_thr, d_sel, d_gate, d_d1, d_d2, d_out);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_topk_limbs(const uint64_t* d_sel, const uint64_t* d_d1, const uint64_t* d_d2, uint64_t n,
                        uint32_t* d_sel_idx, uint32_t* d_d1_idx, uint64_t* d_limbs, uint32_t* d_limb_idx,
                        cudaStream_t stream) {
    if (n == 0) return 0;
    if (!d_sel || !d_d1 || !d_d2 || !d_sel_idx || !d_d1_idx || !d_limbs || !d_limb_idx)
        return (int)cudaErrorInvalidValue;
    k_topk_limbs<<<ew_grid(n), kOpThreads, 0, stream>>>(d_sel, d_d1, d_d2, n, d_sel_idx, d_d1_idx, d_limbs,
                                                          d_limb_idx);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_iota(uint64_t* d_out, uint64_t n, cudaStream_t stream) {
    if (n == 0) return 0;
    if (!d_out) return (int)cudaErrorInvalidValue;
    k_iota<<<ew_grid(n), kOpThreads, 0, stream>>>(d_out, n);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_fill(uint64_t* d_out, uint64_t n, uint64_t value, cudaStream_t stream) {
    if (n == 0) return 0;
    if (!d_out) return (int)cudaErrorInvalidValue;
    k_fill<<<ew_grid(n), kOpThreads, 0, stream>>>(d_out, n, value);
    ZK_LAUNCH_CHECK();
    return 0;
}

uint64_t zkie2_eq_combine_scratch_elems(uint32_t c, uint32_t t) {
    if (c == 0 || t > kEqMaxVars) return 0;
    const uint32_t tl = t / 2, th = t - tl;
    return (uint64_t)c * ((1ull << tl) + (1ull << th)) + 2;
}

int zkie2_eq_combine(const uint64_t* h_points, const uint64_t* h_coeffs, uint32_t c, uint32_t t, uint64_t* d_out,
                     uint64_t* d_scratch, cudaStream_t stream) {
    if (c == 0 || t > kEqMaxVars || !h_coeffs || !d_out || !d_scratch || (t && !h_points))
        return (int)cudaErrorInvalidValue;
    const uint32_t tl = t / 2, th = t - tl;
    const uint64_t per = (1ull << tl) + (1ull << th);
    for (uint32_t c0 = 0; c0 < c; c0 += kEqChunk) {
        const uint32_t cn = c - c0 < (uint32_t)kEqChunk ? c - c0 : (uint32_t)kEqChunk;
        EqChunk ck{};
        for (uint32_t i = 0; i < cn; i++) {
            for (uint32_t j = 0; j < t; j++) ck.r[i][j] = h_points[(uint64_t)(c0 + i) * t + j];
            ck.coeff[i] = h_coeffs[c0 + i];
        }
        k_eq_split_tables<<<ew_grid(per * cn), kOpThreads, 0, stream>>>(ck, cn, t, tl, d_scratch + per * c0);
        ZK_LAUNCH_CHECK();
    }
    const uint64_t n = 1ull << t;
    k_eq_combine<<<ew_grid(n), kOpThreads, 0, stream>>>(d_scratch, c, tl, th, n, d_out);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_lookup_multiplicity(const uint32_t* d_x, uint64_t n, uint64_t t, uint64_t* d_m, int accumulate,
                              uint32_t* d_err, cudaStream_t stream) {
    if (!d_m || !d_err || (n && !d_x)) return (int)cudaErrorInvalidValue;
    if (!accumulate && t) ZK_TRY(cudaMemsetAsync(d_m, 0, 8 * t, stream));
    if (n == 0) return 0;
    k_multiplicity<<<ew_grid(n), kOpThreads, 0, stream>>>(d_x, n, t, reinterpret_cast<unsigned long long*>(d_m),
                                                          d_err);
    ZK_LAUNCH_CHECK();
    return 0;
}

}  // extern "C"
