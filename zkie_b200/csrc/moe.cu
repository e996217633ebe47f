// moe.cu -- the arms of an MLA attention / mixture-of-experts layer
// (DeepSeek-V2-style graphs) on the device: the forward witness of ScaleVec,
// BroadcastScale, IdxBroadcast, CombineIdx, PadIdx, RoPE, Scatter, Gather and
// GatherMatMul (crates/zkie-ops/src/compose.rs:1193-1293, rope.rs, scatter.rs,
// gather.rs, zkie-core common/batched_matmul.rs) and the columns their proofs
// read (prove_rope, prove_scatter / prove_permutation, prove_scatter_add,
// prove_gather_matmul).
//
// Tensors are flat row-major arrays of field elements (u64, canonical on
// output) or u32 indices, as in the reference's Store.  The expert-major
// routing tensors are short (6 m positions), so their builders run one block
// per expert or per token with block-wide compactions; everything else is a
// grid-stride elementwise loop.  An index the reference would use out of
// bounds sets bit 1 of the caller's device error word.
#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/zkie2.h"
#include "common.cuh"
#include "fixed.cuh"
#include "gl64.cuh"
#include "internal.h"

namespace zk {

namespace {

constexpr int kMoeThreads = 256;
constexpr int kMoeWarps = kMoeThreads / 32;
constexpr uint32_t kErrIndex = 1u;

unsigned moe_grid(uint64_t n) {
    const uint64_t b = ceil_div(n, kMoeThreads);
    return (unsigned)(b < 148ull * 16 ? (b ? b : 1) : 148ull * 16);
}

unsigned block_grid(uint64_t m) { return (unsigned)(m < 65535ull * 16 ? (m ? m : 1) : 65535ull * 16); }

__device__ __forceinline__ uint64_t field_block_sum(uint64_t v, uint64_t* sh) {
    for (int o = 16; o; o >>= 1) v = gl_add(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    v = sh[0];
    for (int w = 1; w < kMoeWarps; w++) v = gl_add(v, sh[w]);
    return gl_canon(v);
}

// ---- the arms without a proof of their own ----------------------------------------------
// ScaleVec: out[i] = from_i64(round_div(to_i64(x[i]) to_i64(scale[i % len]), 2^shift))
__global__ void k_scale_vec(const uint64_t* __restrict__ x, uint64_t n, const uint64_t* __restrict__ sc, uint64_t len,
                            uint32_t shift, uint64_t* __restrict__ out) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const int64_t v = fx_wmul(fx_to_i64(gl_canon(__ldg(x + i))), fx_to_i64(gl_canon(__ldg(sc + i % len))));
        out[i] = fx_from_i64(fx_round_div_pow2(v, shift));
    }
}

// BroadcastScale: out[i] = x[i] scale[i / h] (field)
__global__ void k_broadcast_scale(const uint64_t* __restrict__ x, uint64_t n, const uint64_t* __restrict__ sc,
                                  uint64_t h, uint64_t* __restrict__ out) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = gl_canon(gl_mul(__ldg(x + i), __ldg(sc + i / h)));
}

// IdxBroadcast: out[i b + j] = base[i] b + j (u32, wrapping)
__global__ void k_idx_broadcast(const uint32_t* __restrict__ base, uint64_t nb, uint32_t b,
                                uint32_t* __restrict__ out) {
    const uint64_t n = nb * b, stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = __ldg(base + i / b) * b + (uint32_t)(i % b);
}

// CombineIdx: out[i] = a[i] scale + b[i] (u32, wrapping)
__global__ void k_combine_idx(const uint32_t* __restrict__ a, const uint32_t* __restrict__ b, uint64_t n,
                              uint32_t scale, uint32_t* __restrict__ out) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride)
        out[i] = __ldg(a + i) * scale + __ldg(b + i);
}

// ScaleGate (compose.rs:1294-1318): out[i] = from_i64(round_div(to_i64(x[i])
// to_i64(gate[(i / h) n + col]), 2^shift))
__global__ void k_scale_gate(const uint64_t* __restrict__ x, uint64_t len, const uint64_t* __restrict__ gate,
                             uint64_t col, uint64_t n, uint64_t h, uint32_t shift, uint64_t* __restrict__ out) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < len; i += stride) {
        const int64_t g = fx_to_i64(gl_canon(__ldg(gate + (i / h) * n + col)));
        out[i] = fx_from_i64(fx_round_div_pow2(fx_wmul(fx_to_i64(gl_canon(__ldg(x + i))), g), shift));
    }
}

// Relu (compose.rs:1319-1326): x where to_i64(x) > 0, else 0
__global__ void k_relu(const uint64_t* __restrict__ x, uint64_t n, uint64_t* __restrict__ out) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const uint64_t v = gl_canon(__ldg(x + i));
        out[i] = fx_to_i64(v) > 0 ? v : 0;
    }
}

// BatchedMatMul forward (batched_matmul.rs:112-134): g[pos n + j] = sum_d
// a[pos k + d] w[pos k n + d n + j] (field); one thread per output, the
// reads of w along j coalesced, every element of w read once
__global__ void k_batched_matmul(const uint64_t* __restrict__ a, const uint64_t* __restrict__ w, uint64_t s,
                                 uint64_t k, uint64_t n, uint64_t* __restrict__ g) {
    const uint64_t total = s * n, stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t o = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; o < total; o += stride) {
        const uint64_t pos = o / n, j = o % n;
        const uint64_t* ap = a + pos * k;
        const uint64_t* wp = w + pos * k * n + j;
        uint64_t acc = 0;
        for (uint64_t d = 0; d < k; d++) acc = gl_add(acc, gl_mul(__ldg(ap + d), __ldg(wp + d * n)));
        g[o] = gl_canon(acc);
    }
}

// ---- RoPE (rope.rs:87-124 forward, :126-196 the prover's columns) ------------------------
struct RopeCols {
    uint64_t *x_f, *x_s, *o_f, *o_s, *cos_b, *sin_b, *rem_f, *rem_s;
};

// k over m heads d/2 rotated pairs: (p, h, i) -> x[p h d + h d + i] and
// [.. + d/2 + i] with cos / sin[p d/2 + i]; raw_f = xf c - xs s, raw_s = xs c
// + xf s (wrapping i64), each rounded by 2^shift.  out given: the forward;
// cols given: the halves of x and out (out read, not written), cos and sin
// broadcast over the heads, and the remainders raw - o 2^shift + 2^(shift-1).
__global__ void k_rope(const uint64_t* __restrict__ x, const uint64_t* __restrict__ cs,
                       const uint64_t* __restrict__ sn, uint64_t m, uint64_t heads, uint64_t d, uint32_t shift,
                       uint64_t* __restrict__ out, const uint64_t* __restrict__ out_in, RopeCols c) {
    const uint64_t half = d / 2, total = m * heads * half;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const int64_t two = 1ll << shift, hs = 1ll << (shift - 1);
    for (uint64_t k = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; k < total; k += stride) {
        const uint64_t p = k / (heads * half), i = k % half;
        const uint64_t base = (k / half) * d;  // (p heads + h) d
        const uint64_t xf = gl_canon(__ldg(x + base + i)), xs = gl_canon(__ldg(x + base + half + i));
        const uint64_t cv = gl_canon(__ldg(cs + p * half + i)), sv = gl_canon(__ldg(sn + p * half + i));
        const int64_t xfi = fx_to_i64(xf), xsi = fx_to_i64(xs), ci = fx_to_i64(cv), si = fx_to_i64(sv);
        const int64_t raw_f = fx_wsub(fx_wmul(xfi, ci), fx_wmul(xsi, si));
        const int64_t raw_s = fx_wadd(fx_wmul(xsi, ci), fx_wmul(xfi, si));
        const int64_t of = fx_round_div_pow2(raw_f, shift), os = fx_round_div_pow2(raw_s, shift);
        if (out) {
            out[base + i] = fx_from_i64(of);
            out[base + half + i] = fx_from_i64(os);
        }
        if (c.rem_f) {
            c.x_f[k] = xf;
            c.x_s[k] = xs;
            c.cos_b[k] = cv;
            c.sin_b[k] = sv;
            c.o_f[k] = gl_canon(__ldg(out_in + base + i));
            c.o_s[k] = gl_canon(__ldg(out_in + base + half + i));
            c.rem_f[k] = fx_from_i64(fx_wadd(fx_wsub(raw_f, fx_wmul(of, two)), hs));
            c.rem_s[k] = fx_from_i64(fx_wadd(fx_wsub(raw_s, fx_wmul(os, two)), hs));
        }
    }
}

// ---- Scatter (scatter.rs:12-55) -----------------------------------------------------------
// Block-wide ordered compaction: each thread's flag, the block's running base
// (in *base, thread 0 advances it) -> the flagged threads' output slots.
__device__ __forceinline__ uint64_t compact_slot(bool f, uint32_t* warp_cnt, uint64_t* base) {
    const unsigned lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const unsigned ballot = __ballot_sync(0xFFFFFFFFu, f);
    if (lane == 0) warp_cnt[warp] = (uint32_t)__popc(ballot);
    __syncthreads();
    uint64_t before = 0, total = 0;
    for (unsigned w = 0; w < kMoeWarps; w++) {
        if (w < warp) before += warp_cnt[w];
        total += warp_cnt[w];
    }
    const uint64_t slot = *base + before + (uint64_t)__popc(ballot & ((1u << lane) - 1));
    __syncthreads();
    if (threadIdx.x == 0) *base += total;
    return slot;
}

// cnt[c] = #{r < len : sel[c lstride + r estride] == 1}, one block per line c
__global__ void k_sel_counts(const uint64_t* __restrict__ sel, uint64_t lines, uint64_t len, uint64_t lstride,
                             uint64_t estride, uint32_t* __restrict__ cnt) {
    __shared__ uint32_t sh[kMoeWarps];
    for (uint64_t c = blockIdx.x; c < lines; c += gridDim.x) {
        uint32_t k = 0;
        for (uint64_t r = threadIdx.x; r < len; r += blockDim.x) k += gl_canon(__ldg(sel + c * lstride + r * estride)) == 1;
        for (int o = 16; o; o >>= 1) k += __shfl_xor_sync(0xFFFFFFFFu, k, o);
        __syncthreads();
        if ((threadIdx.x & 31) == 0) sh[threadIdx.x >> 5] = k;
        __syncthreads();
        if (threadIdx.x == 0) {
            uint32_t s = 0;
            for (int w = 0; w < kMoeWarps; w++) s += sh[w];
            cnt[c] = s;
        }
    }
}

// Line c of the one-hot (an expert column for the expert-major scatter, a
// token row for the token-major source encodings): its ones in order, after
// the ones of the lines before it.  expert-major: token_id = r, expert_of =
// c; token-major: enc = c n + r (the source encodings t n + e).
__global__ void k_sel_compact(const uint64_t* __restrict__ sel, uint64_t lines, uint64_t len, uint64_t lstride,
                              uint64_t estride, const uint64_t* __restrict__ first, uint32_t* __restrict__ token_id,
                              uint32_t* __restrict__ expert_of, uint64_t* __restrict__ enc, uint64_t n) {
    __shared__ uint32_t warp_cnt[kMoeWarps];
    __shared__ uint64_t base;
    for (uint64_t c = blockIdx.x; c < lines; c += gridDim.x) {
        __syncthreads();
        if (threadIdx.x == 0) base = first[c];
        __syncthreads();
        for (uint64_t r0 = 0; r0 < len; r0 += blockDim.x) {
            const uint64_t r = r0 + threadIdx.x;
            const bool f = r < len && gl_canon(__ldg(sel + c * lstride + r * estride)) == 1;
            const uint64_t slot = compact_slot(f, warp_cnt, &base);
            if (f) {
                if (enc) {
                    enc[slot] = c * n + r;
                } else {
                    token_id[slot] = (uint32_t)r;
                    expert_of[slot] = (uint32_t)c;
                }
            }
            __syncthreads();
        }
    }
}

// first[c] = cnt[0] + .. + cnt[c - 1] (one thread: the lines are tokens or
// experts); with err given, *err |= 1 unless the total is s (the multisets
// of a permutation have one length)
__global__ void k_line_offsets(const uint32_t* __restrict__ cnt, uint64_t lines, uint64_t* __restrict__ first,
                               uint64_t s, uint32_t* __restrict__ err) {
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        uint64_t a = 0;
        for (uint64_t c = 0; c < lines; c++) {
            first[c] = a;
            a += cnt[c];
        }
        if (err && a != s) atomicOr(err, kErrIndex);
    }
}

// b[pos] = token_id[pos] n + expert_of[pos]
__global__ void k_scatter_targets(const uint32_t* __restrict__ tid, const uint32_t* __restrict__ eof, uint64_t s,
                                  uint64_t n, uint64_t* __restrict__ b) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < s; i += stride)
        b[i] = gl_canon((uint64_t)__ldg(tid + i) * n + __ldg(eof + i));
}

// build_perm_num_den (logup_gkr.rs:807-820): num 1 / den alpha - v for i <
// len, then 0 / alpha
__global__ void k_perm_cols(const uint64_t* __restrict__ v, uint64_t len, uint64_t total, uint64_t alpha,
                            uint64_t* __restrict__ num, uint64_t* __restrict__ den) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        const bool in = i < len;
        num[i] = in ? 1 : 0;
        den[i] = in ? gl_canon(gl_sub(alpha, __ldg(v + i))) : alpha;
    }
}

// ---- Gather / scatter-add (gather.rs:36-157) ------------------------------------------------
// positions per token: count, offsets (one block), lists
__global__ void k_token_count(const uint32_t* __restrict__ tid, uint64_t s, uint64_t m, uint32_t* __restrict__ cnt,
                              uint32_t* __restrict__ err) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < s; i += stride) {
        const uint32_t t = __ldg(tid + i);
        if (t < m)
            atomicAdd(cnt + t, 1u);
        else
            atomicOr(err, kErrIndex);
    }
}

__global__ void k_token_offsets(const uint32_t* __restrict__ cnt, uint64_t m, uint32_t* __restrict__ off) {
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        uint32_t a = 0;
        for (uint64_t t = 0; t < m; t++) {
            off[t] = a;
            a += cnt[t];
        }
        off[m] = a;
    }
}

__global__ void k_token_fill(const uint32_t* __restrict__ tid, uint64_t s, uint64_t m,
                             const uint32_t* __restrict__ off, uint32_t* __restrict__ cursor,
                             uint32_t* __restrict__ list) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < s; i += stride) {
        const uint32_t t = __ldg(tid + i);
        if (t < m) list[off[t] + atomicAdd(cursor + t, 1u)] = (uint32_t)i;
    }
}

// out[t h + d] = sum over the token's positions of weighted[pos h + d]
// gate[pos] (field sums: the list order does not matter).  Block (t, y)
// covers columns y 256 .. + 255 of token t, one column per thread; the
// token's positions and gates are staged in shared memory 256 at a time, so
// a long list (the padding positions all route to token 0) costs one
// coalesced load per position and column, four in flight per thread.
__global__ void __launch_bounds__(kMoeThreads) k_gather_rows(const uint64_t* __restrict__ weighted,
                                                             const uint64_t* __restrict__ gate, uint64_t h,
                                                             const uint32_t* __restrict__ off,
                                                             const uint32_t* __restrict__ list, uint64_t m,
                                                             uint64_t* __restrict__ out) {
    __shared__ uint32_t s_pos[kMoeThreads];
    __shared__ uint64_t s_gate[kMoeThreads];
    const uint64_t d = (uint64_t)blockIdx.y * kMoeThreads + threadIdx.x;
    for (uint64_t t = blockIdx.x; t < m; t += gridDim.x) {
        const uint32_t q0 = off[t], q1 = off[t + 1];
        uint64_t acc = 0;
        for (uint32_t c0 = q0; c0 < q1; c0 += kMoeThreads) {
            const uint32_t cn = q1 - c0 < (uint32_t)kMoeThreads ? q1 - c0 : (uint32_t)kMoeThreads;
            __syncthreads();  // the previous chunk is no longer read
            if (threadIdx.x < cn) {
                const uint32_t pos = list[c0 + threadIdx.x];
                s_pos[threadIdx.x] = pos;
                s_gate[threadIdx.x] = __ldg(gate + pos);
            }
            __syncthreads();
            if (d < h) {
                uint32_t q = 0;
                for (; q + 4 <= cn; q += 4) {
                    const uint64_t w0 = __ldg(weighted + (uint64_t)s_pos[q] * h + d);
                    const uint64_t w1 = __ldg(weighted + (uint64_t)s_pos[q + 1] * h + d);
                    const uint64_t w2 = __ldg(weighted + (uint64_t)s_pos[q + 2] * h + d);
                    const uint64_t w3 = __ldg(weighted + (uint64_t)s_pos[q + 3] * h + d);
                    acc = gl_add(acc, gl_mul(w0, s_gate[q]));
                    acc = gl_add(acc, gl_mul(w1, s_gate[q + 1]));
                    acc = gl_add(acc, gl_mul(w2, s_gate[q + 2]));
                    acc = gl_add(acc, gl_mul(w3, s_gate[q + 3]));
                }
                for (; q < cn; q++) acc = gl_add(acc, gl_mul(__ldg(weighted + (uint64_t)s_pos[q] * h + d), s_gate[q]));
            }
        }
        if (d < h) out[t * h + d] = gl_canon(acc);
    }
}

// The scatter-add proof's columns.  source (tid given): i < s h: num =
// gamma[d] weighted[i] gate[pos], den = alpha - tid[pos], gamma_b =
// gamma[d], gate_b = gate[pos], w_pad = weighted[i]; target: i < m h: num =
// gamma[d] out[i], den = alpha - t, gamma_b = gamma[d], w_pad = out[i];
// past the end 0 / alpha / 0 / 0 / 0.
__global__ void k_scatter_add_cols(const uint64_t* __restrict__ vals, const uint64_t* __restrict__ gate,
                                   const uint32_t* __restrict__ tid, const uint64_t* __restrict__ gamma, uint64_t rows,
                                   uint64_t h, uint64_t total, uint64_t alpha, uint64_t* __restrict__ num,
                                   uint64_t* __restrict__ den, uint64_t* __restrict__ gamma_b,
                                   uint64_t* __restrict__ gate_b, uint64_t* __restrict__ v_pad) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
        if (i < rows * h) {
            const uint64_t pos = i / h, g = __ldg(gamma + i % h), v = gl_canon(__ldg(vals + i));
            const uint64_t gt = gate ? gl_canon(__ldg(gate + pos)) : 1;
            const uint64_t key = tid ? (uint64_t)__ldg(tid + pos) : pos;
            num[i] = gl_canon(gl_mul(gl_mul(g, v), gt));
            den[i] = gl_canon(gl_sub(alpha, key));
            gamma_b[i] = g;
            if (gate_b) gate_b[i] = gt;
            v_pad[i] = v;
        } else {
            num[i] = 0;
            den[i] = alpha;
            gamma_b[i] = 0;
            if (gate_b) gate_b[i] = 0;
            v_pad[i] = 0;
        }
    }
}

// ---- GatherMatMul (batched_matmul.rs:219-290, 359-494) -------------------------------------
// out[pos k + d] = wv[expert_of[pos] k + d]
__global__ void k_expert_rows(const uint64_t* __restrict__ wv, const uint32_t* __restrict__ eof, uint64_t s,
                              uint64_t k, uint64_t n_experts, uint64_t* __restrict__ out,
                              uint32_t* __restrict__ err) {
    const uint64_t n = s * k, stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
        const uint32_t e = __ldg(eof + i / k);
        if (e < n_experts) {
            out[i] = __ldg(wv + (uint64_t)e * k + i % k);
        } else {
            out[i] = 0;
            atomicOr(err, kErrIndex);
        }
    }
}

// counts[e] = sum_{pos : expert_of[pos] = e} eq_pos[pos]; table[e] = sum_d
// eq_d[d] wv[e k + d]; one block per expert
__global__ void k_expert_open(const uint32_t* __restrict__ eof, uint64_t s, const uint64_t* __restrict__ eq_pos,
                              const uint64_t* __restrict__ wv, uint64_t k, const uint64_t* __restrict__ eq_d,
                              uint64_t n_experts, uint64_t* __restrict__ counts, uint64_t* __restrict__ table) {
    __shared__ uint64_t sh[kMoeWarps];
    for (uint64_t e = blockIdx.x; e < n_experts; e += gridDim.x) {
        uint64_t c = 0, t = 0;
        for (uint64_t pos = threadIdx.x; pos < s; pos += blockDim.x)
            if (__ldg(eof + pos) == e) c = gl_add(c, __ldg(eq_pos + pos));
        for (uint64_t d = threadIdx.x; d < k; d += blockDim.x) t = gl_add(t, gl_mul(__ldg(eq_d + d), __ldg(wv + e * k + d)));
        c = field_block_sum(c, sh);
        t = field_block_sum(t, sh);
        if (threadIdx.x == 0) {
            counts[e] = c;
            table[e] = t;
        }
    }
}

}  // namespace

}  // namespace zk

using namespace zk;

extern "C" {

int zkie2_op_scale_vec(const uint64_t* d_x, uint64_t n, const uint64_t* d_scale, uint64_t len, uint32_t shift,
                       uint64_t* d_out, cudaStream_t stream) {
    if (shift > 62 || (n && len == 0)) return (int)cudaErrorInvalidValue;
    if (n == 0) return 0;
    if (!d_x || !d_scale || !d_out) return (int)cudaErrorInvalidValue;
    k_scale_vec<<<moe_grid(n), kMoeThreads, 0, stream>>>(d_x, n, d_scale, len, shift, d_out);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_scale_gate(const uint64_t* d_x, uint64_t len, const uint64_t* d_gate, uint64_t gate_len, uint64_t col,
                        uint64_t n, uint64_t h, uint32_t shift, uint64_t* d_out, cudaStream_t stream) {
    if (shift > 62 || h == 0 || col >= n || (len && ((len - 1) / h) * n + col >= gate_len))
        return (int)cudaErrorInvalidValue;
    if (len == 0) return 0;
    if (!d_x || !d_gate || !d_out) return (int)cudaErrorInvalidValue;
    k_scale_gate<<<moe_grid(len), kMoeThreads, 0, stream>>>(d_x, len, d_gate, col, n, h, shift, d_out);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_relu(const uint64_t* d_x, uint64_t n, uint64_t* d_out, cudaStream_t stream) {
    if (n == 0) return 0;
    if (!d_x || !d_out) return (int)cudaErrorInvalidValue;
    k_relu<<<moe_grid(n), kMoeThreads, 0, stream>>>(d_x, n, d_out);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_batched_matmul(const uint64_t* d_a, const uint64_t* d_w, uint64_t s, uint64_t k, uint64_t n,
                            uint64_t* d_c, cudaStream_t stream) {
    if (s == 0 || n == 0) return 0;
    if (!d_c || (k && (!d_a || !d_w))) return (int)cudaErrorInvalidValue;
    k_batched_matmul<<<moe_grid(s * n), kMoeThreads, 0, stream>>>(d_a, d_w, s, k, n, d_c);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_broadcast_scale(const uint64_t* d_x, uint64_t n, const uint64_t* d_scale, uint64_t len, uint64_t h,
                             uint64_t* d_out, cudaStream_t stream) {
    if (h == 0 || (n && (n - 1) / h >= len)) return (int)cudaErrorInvalidValue;
    if (n == 0) return 0;
    if (!d_x || !d_scale || !d_out) return (int)cudaErrorInvalidValue;
    k_broadcast_scale<<<moe_grid(n), kMoeThreads, 0, stream>>>(d_x, n, d_scale, h, d_out);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_idx_broadcast(const uint32_t* d_base, uint64_t nb, uint32_t b, uint32_t* d_out, cudaStream_t stream) {
    if (nb == 0 || b == 0) return 0;
    if (!d_base || !d_out) return (int)cudaErrorInvalidValue;
    k_idx_broadcast<<<moe_grid(nb * b), kMoeThreads, 0, stream>>>(d_base, nb, b, d_out);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_combine_idx(const uint32_t* d_a, const uint32_t* d_b, uint64_t n, uint32_t scale, uint32_t* d_out,
                         cudaStream_t stream) {
    if (n == 0) return 0;
    if (!d_a || !d_b || !d_out) return (int)cudaErrorInvalidValue;
    k_combine_idx<<<moe_grid(n), kMoeThreads, 0, stream>>>(d_a, d_b, n, scale, d_out);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_pad_idx(const uint32_t* d_base, uint64_t nb, uint64_t len, uint32_t* d_out, cudaStream_t stream) {
    if (len == 0) return 0;
    if (!d_out || (nb && !d_base)) return (int)cudaErrorInvalidValue;
    const uint64_t keep = nb < len ? nb : len;
    if (keep < len) ZK_TRY(cudaMemsetAsync(d_out + keep, 0, 4 * (len - keep), stream));
    if (keep) ZK_TRY(cudaMemcpyAsync(d_out, d_base, 4 * keep, cudaMemcpyDeviceToDevice, stream));
    return 0;
}

int zkie2_op_rope(const uint64_t* d_x, uint64_t n, const uint64_t* d_cos, const uint64_t* d_sin, uint64_t m,
                  uint64_t d, uint32_t shift, uint64_t* d_out, cudaStream_t stream) {
    if (shift == 0 || shift > 62 || d == 0 || d % 2 || m == 0 || n % (m * d)) return (int)cudaErrorInvalidValue;
    if (n == 0) return 0;
    if (!d_x || !d_cos || !d_sin || !d_out) return (int)cudaErrorInvalidValue;
    k_rope<<<moe_grid(n / 2), kMoeThreads, 0, stream>>>(d_x, d_cos, d_sin, m, n / (m * d), d, shift, d_out, nullptr,
                                                         RopeCols{});
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_rope_columns(const uint64_t* d_x, const uint64_t* d_out, uint64_t n, const uint64_t* d_cos,
                          const uint64_t* d_sin, uint64_t m, uint64_t d, uint32_t shift, uint64_t* const* d_cols,
                          cudaStream_t stream) {
    if (shift == 0 || shift > 62 || d == 0 || d % 2 || m == 0 || n % (m * d)) return (int)cudaErrorInvalidValue;
    if (n == 0) return 0;
    if (!d_x || !d_out || !d_cos || !d_sin || !d_cols) return (int)cudaErrorInvalidValue;
    for (int i = 0; i < 8; i++)
        if (!d_cols[i]) return (int)cudaErrorInvalidValue;
    RopeCols c{d_cols[0], d_cols[1], d_cols[2], d_cols[3], d_cols[4], d_cols[5], d_cols[6], d_cols[7]};
    k_rope<<<moe_grid(n / 2), kMoeThreads, 0, stream>>>(d_x, d_cos, d_sin, m, n / (m * d), d, shift, nullptr, d_out,
                                                         c);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_sel_counts(const uint64_t* d_sel, uint64_t m, uint64_t n, uint32_t by_token, uint32_t* d_cnt,
                        cudaStream_t stream) {
    // token and expert ids and the per-line counts are u32
    if (m >= (1ull << 32) || n >= (1ull << 32)) return (int)cudaErrorInvalidValue;
    if (m == 0 || n == 0) return 0;
    if (!d_sel || !d_cnt) return (int)cudaErrorInvalidValue;
    if (by_token)
        k_sel_counts<<<block_grid(m), kMoeThreads, 0, stream>>>(d_sel, m, n, n, 1, d_cnt);
    else
        k_sel_counts<<<block_grid(n), kMoeThreads, 0, stream>>>(d_sel, n, m, 1, n, d_cnt);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_scatter(const uint64_t* d_sel, uint64_t m, uint64_t n, const uint32_t* d_expert_cnt,
                     uint32_t* d_token_id, uint32_t* d_expert_of, uint64_t* d_scratch, cudaStream_t stream) {
    // token and expert ids and the per-line counts are u32
    if (m >= (1ull << 32) || n >= (1ull << 32)) return (int)cudaErrorInvalidValue;
    if (m == 0 || n == 0) return 0;
    if (!d_sel || !d_expert_cnt || !d_token_id || !d_expert_of || !d_scratch) return (int)cudaErrorInvalidValue;
    k_line_offsets<<<1, 32, 0, stream>>>(d_expert_cnt, n, d_scratch, 0, nullptr);
    ZK_LAUNCH_CHECK();
    k_sel_compact<<<block_grid(n), kMoeThreads, 0, stream>>>(d_sel, n, m, 1, n, d_scratch, d_token_id, d_expert_of,
                                                              nullptr, n);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_op_scatter_encodings(const uint64_t* d_sel, uint64_t m, uint64_t n, const uint32_t* d_token_cnt,
                               const uint32_t* d_token_id, const uint32_t* d_expert_of, uint64_t s, uint64_t* d_a,
                               uint64_t* d_b, uint64_t* d_scratch, uint32_t* d_err, cudaStream_t stream) {
    // token and expert ids and the per-line counts are u32
    if (m >= (1ull << 32) || n >= (1ull << 32)) return (int)cudaErrorInvalidValue;
    if (m == 0 || n == 0) return 0;
    if (!d_sel || !d_token_cnt || !d_a || !d_b || !d_scratch || !d_err || (s && (!d_token_id || !d_expert_of)))
        return (int)cudaErrorInvalidValue;
    k_line_offsets<<<1, 32, 0, stream>>>(d_token_cnt, m, d_scratch, s, d_err);
    ZK_LAUNCH_CHECK();
    k_sel_compact<<<block_grid(m), kMoeThreads, 0, stream>>>(d_sel, m, n, n, 1, d_scratch, nullptr, nullptr, d_a,
                                                              n);
    ZK_LAUNCH_CHECK();
    if (s) {
        k_scatter_targets<<<moe_grid(s), kMoeThreads, 0, stream>>>(d_token_id, d_expert_of, s, n, d_b);
        ZK_LAUNCH_CHECK();
    }
    return 0;
}

int zkie2_perm_num_den(const uint64_t* d_v, uint64_t len, uint64_t total, uint64_t alpha, uint64_t* d_num,
                       uint64_t* d_den, cudaStream_t stream) {
    if (total < len) return (int)cudaErrorInvalidValue;
    if (total == 0) return 0;
    if (!d_num || !d_den || (len && !d_v)) return (int)cudaErrorInvalidValue;
    k_perm_cols<<<moe_grid(total), kMoeThreads, 0, stream>>>(d_v, len, total, gl_canon(alpha), d_num, d_den);
    ZK_LAUNCH_CHECK();
    return 0;
}

uint64_t zkie2_op_gather_scratch_u32(uint64_t s, uint64_t m) { return 3 * m + 1 + s; }

int zkie2_op_gather(const uint64_t* d_weighted, const uint32_t* d_token_id, const uint64_t* d_gate, uint64_t s,
                    uint64_t m, uint64_t h, uint64_t* d_out, uint32_t* d_scratch_u32, uint32_t* d_err,
                    cudaStream_t stream) {
    // the per-token offsets and the position lists are u32: s and m below 2^32
    if (s >= (1ull << 32) || m >= (1ull << 32) - 1) return (int)cudaErrorInvalidValue;
    if (m == 0 || h == 0) return 0;
    if (!d_out || !d_scratch_u32 || !d_err || (s && (!d_weighted || !d_token_id || !d_gate)))
        return (int)cudaErrorInvalidValue;
    uint32_t* cnt = d_scratch_u32;
    uint32_t* cursor = cnt + m;
    uint32_t* off = cursor + m;
    uint32_t* list = off + m + 1;
    ZK_TRY(cudaMemsetAsync(cnt, 0, 8 * m, stream));  // cnt and cursor
    if (s) {
        k_token_count<<<moe_grid(s), kMoeThreads, 0, stream>>>(d_token_id, s, m, cnt, d_err);
        ZK_LAUNCH_CHECK();
    }
    k_token_offsets<<<1, 32, 0, stream>>>(cnt, m, off);
    ZK_LAUNCH_CHECK();
    if (s) {
        k_token_fill<<<moe_grid(s), kMoeThreads, 0, stream>>>(d_token_id, s, m, off, cursor, list);
        ZK_LAUNCH_CHECK();
    }
    const uint64_t dblocks = ceil_div(h, kMoeThreads);
    if (dblocks > 65535) return (int)cudaErrorInvalidValue;
    const dim3 grid(m < 65535ull * 16 ? (unsigned)m : 65535u * 16, (unsigned)dblocks);
    k_gather_rows<<<grid, kMoeThreads, 0, stream>>>(d_weighted, d_gate, h, off, list, m, d_out);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_scatter_add_columns(const uint64_t* d_vals, const uint64_t* d_gate, const uint32_t* d_token_id,
                              const uint64_t* d_gamma, uint64_t rows, uint64_t h, uint64_t total, uint64_t alpha,
                              uint64_t* const* d_cols, cudaStream_t stream) {
    if (total < rows * h || h == 0) return (int)cudaErrorInvalidValue;
    if (total == 0) return 0;
    if (!d_cols || !d_cols[0] || !d_cols[1] || !d_cols[2] || !d_cols[4] || (rows && (!d_vals || !d_gamma)) ||
        (d_gate && !d_cols[3]) || (d_token_id && !d_gate))
        return (int)cudaErrorInvalidValue;
    k_scatter_add_cols<<<moe_grid(total), kMoeThreads, 0, stream>>>(d_vals, d_gate, d_token_id, d_gamma, rows, h,
                                                                     total, gl_canon(alpha), d_cols[0],
                                                                     d_cols[1], d_cols[2], d_cols[3], d_cols[4]);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_expert_rows(const uint64_t* d_wv, const uint32_t* d_expert_of, uint64_t s, uint64_t k, uint64_t n_experts,
                      uint64_t* d_out, uint32_t* d_err, cudaStream_t stream) {
    if (s == 0 || k == 0) return 0;
    if (!d_wv || !d_expert_of || !d_out || !d_err) return (int)cudaErrorInvalidValue;
    k_expert_rows<<<moe_grid(s * k), kMoeThreads, 0, stream>>>(d_wv, d_expert_of, s, k, n_experts, d_out, d_err);
    ZK_LAUNCH_CHECK();
    return 0;
}

int zkie2_expert_open(const uint32_t* d_expert_of, uint64_t s, const uint64_t* d_eq_pos, const uint64_t* d_wv,
                      uint64_t k, const uint64_t* d_eq_d, uint64_t n_experts, uint64_t* d_counts, uint64_t* d_table,
                      cudaStream_t stream) {
    if (n_experts == 0) return 0;
    if (!d_counts || !d_table || (s && (!d_expert_of || !d_eq_pos)) || (k && (!d_wv || !d_eq_d)))
        return (int)cudaErrorInvalidValue;
    k_expert_open<<<block_grid(n_experts), kMoeThreads, 0, stream>>>(d_expert_of, s, d_eq_pos, d_wv, k, d_eq_d,
                                                                      n_experts, d_counts, d_table);
    ZK_LAUNCH_CHECK();
    return 0;
}

}  // extern "C"
