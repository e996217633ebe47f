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
#include "../../include/zkie2.h"
#include "common.cuh"
#include "gl64.cuh"

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

unsigned grid_for(uint64_t n) {
    const uint64_t b = ceil_div(n, kThreads);
    return (unsigned)(b < 148ull * 16 ? b : 148ull * 16);
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

}  // extern "C"
