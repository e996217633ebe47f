// fixed_matmul_tc.cu -- the forward witness of a fixed-point matmul on the
// tensor cores: par::mm_par_fixed (crates/zkie-ops/src/par.rs:41-89).
//
// The reference maps every field element to i64 (to_i64: values above p/2
// are negative), takes exact i64 dot products and maps them back (from_i64);
// the result equals the field matmul, and it falls back to the field matmul
// when the i64 sums could overflow.  Here, when every input lies in
// [-2^23, 2^23) (fixed point up to 24 bits: the inference witness range,
// 16-bit weights against Q16 activations), the products run on the
// 5th-generation tensor cores as u8 x u8 -> s32 GEMMs.  Each operand takes
// P = 2 or 3 byte planes (2 when all its values lie in [-2^15, 2^15)):
//   a' = a + 2^(8 P_a - 1) in [0, 2^(8 P_a)), a' = sum_q 2^(8q) a_q, so
//   sum_k a'b' = sum_s 2^(8s) sum_{q_a + q_b = s} A_{q_a} B_{q_b},
// each plane-sum s as ONE GEMM over the pairs' planes concatenated along K
// (three GEMMs for 2 x 2 planes, five for 3 x 3), and the offsets come off
// exactly:  sum_k a b = sum_k a'b' - o_b rowsum_i(A') - o_a colsum_j(B')
// + K o_a o_b, in wrapping u64 arithmetic (|sum_k a b| <= K 2^(8 (P_a + P_b) - 2)
// < 2^63: K < 2^17 for three planes on both sides, the field kernel past it).
// Every s32 sum stays below 3 * 8192 * 255^2 < 2^31 by splitting K into
// chunks of at most 8192.  Inputs outside 24 bits, or a K or N that TMA
// cannot address (K % 16, N % 4), take the exact field kernel instead, so
// the output always equals the field matmul.
//
// The GEMMs are CUTLASS sm100 collectives (tcgen05.mma kind::i8 issued by one
// thread, operands staged by TMA, accumulators in TMEM), 128 x 128 x 128
// tiles on one SM each, static 1 x 1 x 1 clusters: no TMA multicast.
#include <mutex>

#include "cutlass/cutlass.h"
#include "cute/tensor.hpp"
#include "cutlass/epilogue/collective/collective_builder.hpp"
#include "cutlass/gemm/collective/collective_builder.hpp"
#include "cutlass/gemm/device/gemm_universal_adapter.h"
#include "cutlass/gemm/dispatch_policy.hpp"
#include "cutlass/gemm/kernel/gemm_universal.hpp"

#include "../../include/zkie2.h"
#include "common.cuh"
#include "gl64.cuh"
#include "internal.h"

namespace zk {

namespace {

using namespace cute;

using TcTile = Shape<_128, _128, _128>;
using TcCluster = Shape<_1, _1, _1>;
using TcEpilogue = typename cutlass::epilogue::collective::CollectiveBuilder<
    cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, TcTile, TcCluster,
    cutlass::epilogue::collective::EpilogueTileAuto, int32_t, int32_t, void, cutlass::layout::RowMajor, 4, int32_t,
    cutlass::layout::RowMajor, 4, cutlass::epilogue::TmaWarpSpecialized1Sm>::CollectiveOp;
using TcMainloop = typename cutlass::gemm::collective::CollectiveBuilder<
    cutlass::arch::Sm100, cutlass::arch::OpClassTensorOp, uint8_t, cutlass::layout::RowMajor, 16, uint8_t,
    cutlass::layout::ColumnMajor, 16, int32_t, TcTile, TcCluster,
    cutlass::gemm::collective::StageCountAutoCarveout<static_cast<int>(sizeof(typename TcEpilogue::SharedStorage))>,
    cutlass::gemm::KernelTmaWarpSpecialized1SmSm100>::CollectiveOp;
using TcKernel = cutlass::gemm::kernel::GemmUniversal<Shape<int, int, int, int>, TcMainloop, TcEpilogue>;
using TcGemm = cutlass::gemm::device::GemmUniversalAdapter<TcKernel>;

constexpr uint64_t kKChunk = 8192;  // 3 * kKChunk * 255^2 < 2^31
constexpr int kThr = 256;
constexpr uint32_t kMaxPlanes = 3;

// The byte planes of an operand whose values all lie in [-2^(8P-1), 2^(8P-1)):
// v' = to_i64(v) + 2^(8P-1) in [0, 2^(8P)), plane q = byte q of v'.  Products
// group by s = q_a + q_b: G_s = sum over the pairs (q_a, s - q_a) of the
// plane products, one GEMM per s over the pairs' planes concatenated along K
// (per K chunk), and sum_k a'b' = sum_s 2^(8s) G_s.

// pair p of plane-sum s (p-th q_a from max(0, s - PB + 1)); count of pairs
__host__ __device__ __forceinline__ uint32_t pair_lo(uint32_t s, uint32_t pb) { return s + 1 > pb ? s + 1 - pb : 0; }
__host__ __device__ __forceinline__ uint32_t pair_count(uint32_t s, uint32_t pa, uint32_t pb) {
    const uint32_t lo = pair_lo(s, pb), hi = s < pa - 1 ? s : pa - 1;
    return hi + 1 - lo;
}
// byte offset of region s in a packed operand of `rows` rows (regions in s order)
__host__ __device__ __forceinline__ uint64_t region_off(uint32_t s, uint32_t pa, uint32_t pb, uint64_t rows,
                                                        uint64_t K) {
    uint64_t off = 0;
    for (uint32_t q = 0; q < s; q++) off += pair_count(q, pa, pb) * rows * K;
    return off;
}

// column of element k (chunk c0, width kc) for pair p of a region with `cnt`
// pairs: per chunk the pairs' planes side by side
__device__ __forceinline__ uint64_t cat_col(uint64_t k, uint64_t K, uint32_t cnt, uint32_t p) {
    const uint64_t c0 = k / kKChunk * kKChunk;
    const uint64_t kc = K - c0 < kKChunk ? K - c0 : kKChunk;
    return cnt * c0 + p * kc + (k - c0);
}

// bit 0: outside [-2^15, 2^15); bit 1: outside [-2^23, 2^23)
__device__ __forceinline__ uint32_t width_flags(uint64_t x) {
    x = gl_canon(x);
    const bool neg = x > GL_P / 2;
    const uint64_t mag = neg ? GL_P - x : x;
    return ((neg ? mag > (1ull << 15) : mag >= (1ull << 15)) ? 1u : 0u) |
           ((neg ? mag > (1ull << 23) : mag >= (1ull << 23)) ? 2u : 0u);
}

// bit 0: a value outside [-2^15, 2^15); bit 1: outside [-2^23, 2^23)
__global__ void k_tc_range(const uint64_t* __restrict__ v, uint64_t n, uint32_t* __restrict__ flags) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    uint32_t f = 0;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) f |= width_flags(__ldg(v + i));
    f = __reduce_or_sync(0xffffffffu, f);
    if ((threadIdx.x & 31) == 0 && f) atomicOr(flags, f);
}

__device__ __forceinline__ uint32_t shifted(uint64_t x, uint64_t off) {
    x = gl_canon(x);
    return (uint32_t)(x < off ? x + off : x - (GL_P - off));
}

// A (M x K field, row-major) -> its PA planes placed in every region pair
// they take part in (row stride cnt_s K in region s), rowsum[i] = sum_k a'.
// One thread per 16 consecutive elements of a row (K % 16 == 0, chunk widths
// multiples of 16): 16-byte loads and 16-byte stores of each plane.
__global__ void __launch_bounds__(kThr)
    k_pack_a(const uint64_t* __restrict__ a, uint64_t M, uint64_t K, uint32_t pa, uint32_t pb,
             uint8_t* __restrict__ acat, unsigned long long* __restrict__ rowsum, uint32_t* __restrict__ flags) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t groups = M * K / 16, span = (groups + 31) & ~31ull;  // warp-uniform trip count
    const uint64_t off = 1ull << (8 * pa - 1);
    uint32_t wf = 0;
    for (uint64_t gi = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; gi < span; gi += stride) {
        const bool in = gi < groups;
        const uint64_t idx = in ? gi * 16 : 0, i = idx / K, k = idx - i * K;
        unsigned long long sum = 0;
        if (in) {
            const ulonglong2* src = reinterpret_cast<const ulonglong2*>(a + idx);
            uint32_t w[kMaxPlanes][4] = {};
#pragma unroll
            for (int q = 0; q < 8; q++) {
                const ulonglong2 pr = __ldg(src + q);
                wf |= width_flags(pr.x) | width_flags(pr.y);
                const uint32_t v0 = shifted(pr.x, off), v1 = shifted(pr.y, off);
                sum += v0 + v1;
                const int e = 2 * q, wi = e >> 2, sh = (e & 3) * 8;
#pragma unroll
                for (uint32_t pl = 0; pl < kMaxPlanes; pl++)
                    w[pl][wi] |= (((v0 >> (8 * pl)) & 255u) << sh) | (((v1 >> (8 * pl)) & 255u) << (sh + 8));
            }
            const uint4 pl0 = make_uint4(w[0][0], w[0][1], w[0][2], w[0][3]);
            const uint4 pl1 = make_uint4(w[1][0], w[1][1], w[1][2], w[1][3]);
            const uint4 pl2 = make_uint4(w[2][0], w[2][1], w[2][2], w[2][3]);
            for (uint32_t s = 0; s + 1 < pa + pb; s++) {
                const uint32_t lo = pair_lo(s, pb), cnt = pair_count(s, pa, pb);
                uint8_t* reg = acat + region_off(s, pa, pb, M, K) + i * cnt * K;
                for (uint32_t p = 0; p < cnt; p++) {
                    const uint32_t qa = lo + p;  // selects, not an indexed (local-memory) array
                    *reinterpret_cast<uint4*>(reg + cat_col(k, K, cnt, p)) = qa == 0 ? pl0 : qa == 1 ? pl1 : pl2;
                }
            }
        }
        // one atomic per warp when its 32 groups share a row
        const uint64_t i0 = __shfl_sync(0xffffffffu, i, 0);
        if (__all_sync(0xffffffffu, !in || i == i0)) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) sum += __shfl_down_sync(0xffffffffu, sum, o);
            if ((threadIdx.x & 31) == 0 && sum) atomicAdd(rowsum + i0, sum);
        } else if (in) {
            atomicAdd(rowsum + i, sum);
        }
    }
    wf = __reduce_or_sync(0xffffffffu, wf);  // every lane runs the same trip count
    if ((threadIdx.x & 31) == 0 && wf) atomicOr(flags, wf);
}

// B (K x N field, row-major) -> its PB planes transposed (N x K bytes) into
// every region pair they take part in (pair p of region s uses plane s -
// q_a); colsum[j] = sum_k b'.  32 x 32 tiles through shared memory so the
// field reads run along rows of B and the byte writes (four bytes per
// store) along rows of the transposes; one atomic per column per tile.
__global__ void __launch_bounds__(kThr)
    k_pack_b(const uint64_t* __restrict__ b, uint64_t K, uint64_t N, uint32_t pa, uint32_t pb,
             uint8_t* __restrict__ bcat, unsigned long long* __restrict__ colsum, uint32_t* __restrict__ flags) {
    __shared__ uint32_t tile[32][33];
    const uint64_t k0 = (uint64_t)blockIdx.y * 32, n0 = (uint64_t)blockIdx.x * 32;
    const uint32_t tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
    const uint64_t off = 1ull << (8 * pb - 1);
    uint32_t wf = 0;
    for (uint32_t r = ty; r < 32; r += 8) {
        const uint64_t k = k0 + r, n = n0 + tx;
        uint32_t v = 0;
        if (k < K && n < N) {
            const uint64_t x = __ldg(b + k * N + n);
            wf |= width_flags(x);
            v = shifted(x, off);
        }
        tile[r][tx] = v;
    }
    wf = __reduce_or_sync(0xffffffffu, wf);
    if (tx == 0 && wf) atomicOr(flags, wf);
    __syncthreads();
    if (ty == 0 && n0 + tx < N) {
        unsigned long long sum = 0;
#pragma unroll 8
        for (int r = 0; r < 32; r++) sum += tile[r][tx];
        if (sum) atomicAdd(colsum + n0 + tx, sum);
    }
    // thread t writes bytes k0 + 4 (t % 8) .. + 3 of row n0 + t / 8
    const uint32_t nr = threadIdx.x >> 3, kq = (threadIdx.x & 7) * 4;
    const uint64_t n = n0 + nr, k = k0 + kq;
    if (n < N && k < K) {  // K % 16 == 0: the four bytes are all inside
        uint32_t w[kMaxPlanes] = {};
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const uint32_t v = tile[kq + e][nr];
#pragma unroll
            for (uint32_t pl = 0; pl < kMaxPlanes; pl++) w[pl] |= ((v >> (8 * pl)) & 255u) << (8 * e);
        }
        for (uint32_t s = 0; s + 1 < pa + pb; s++) {
            const uint32_t lo = pair_lo(s, pb), cnt = pair_count(s, pa, pb);
            uint8_t* reg = bcat + region_off(s, pa, pb, N, K) + n * cnt * K;
            for (uint32_t p = 0; p < cnt; p++) {
                const uint32_t qb = s - (lo + p);
                *reinterpret_cast<uint32_t*>(reg + cat_col(k, K, cnt, p)) = qb == 0 ? w[0] : qb == 1 ? w[1] : w[2];
            }
        }
    }
}

// A planned product whose operands need more planes than planned (or more
// than 24 bits) sets bit 3 (value 4) of *err: its result is not the product.
__global__ void k_tc_plan_check(const uint32_t* __restrict__ flags, uint32_t pa, uint32_t pb,
                                uint32_t* __restrict__ err) {
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        const uint32_t fa = flags[0], fb = flags[1];
        if (((fa | fb) & 2u) || (pa == 2 && (fa & 1u)) || (pb == 2 && (fb & 1u))) atomicOr(err, 4u);
    }
}

// The plane-sum GEMMs' s32 outputs (one per s, at most five)
constexpr uint32_t kMaxSums = 2 * kMaxPlanes - 1;
struct PlaneSums {
    const int32_t* g[kMaxSums];
    uint32_t count;
};

__device__ __forceinline__ uint64_t plane_sum(const PlaneSums& ps, uint64_t i) {
    uint64_t v = 0;
#pragma unroll
    for (uint32_t q = 0; q < kMaxSums; q++)
        if (q < ps.count) v += (uint64_t)(int64_t)ps.g[q][i] << (8 * q);
    return v;
}

// acc (+)= sum_s 2^(8s) G_s (u64, wrapping): one K chunk of a long K
__global__ void k_tc_accumulate(PlaneSums ps, uint64_t mn, uint64_t* __restrict__ acc, int first) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < mn; i += stride) {
        const uint64_t v = plane_sum(ps, i);
        acc[i] = first ? v : acc[i] + v;
    }
}

// c = from_i64(sum a'b' - oB rowsum_i - oA colsum_j + K oA oB), in wrapping
// u64 arithmetic (the true value sum a b has |.| < 2^63: the caller's K
// bound), with sum a'b' the accumulator or, for one K chunk, the plane sums.
__global__ void k_tc_finish(PlaneSums ps, const uint64_t* __restrict__ acc,
                            const unsigned long long* __restrict__ rowsum,
                            const unsigned long long* __restrict__ colsum, uint64_t M, uint64_t N, uint64_t K,
                            uint64_t oa, uint64_t ob, uint64_t* __restrict__ c) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < M * N; idx += stride) {
        const uint64_t i = idx / N, j = idx - i * N;
        const uint64_t sum = acc ? acc[idx] : plane_sum(ps, idx);
        const int64_t v = (int64_t)(sum - ob * rowsum[i] - oa * colsum[j] + K * oa * ob);
        c[idx] = v >= 0 ? (uint64_t)v : GL_P - (uint64_t)(-v);  // from_i64
    }
}

unsigned tc_grid(uint64_t work) {
    const uint64_t b = ceil_div(work, kThr);
    return (unsigned)(b < 148ull * 16 ? (b ? b : 1) : 148ull * 16);
}

// Scratch layout in bytes (regions 256-byte aligned), sized for three planes
// on each side (nine plane pairs).
struct TcScratch {
    uint8_t *acat, *bcat;
    int32_t* g[kMaxSums];
    uint64_t* acc;
    unsigned long long *rowsum, *colsum;
    uint32_t* flags;
    void* ws;
    uint64_t ws_bytes;
};

uint64_t tc_layout(uint64_t M, uint64_t K, uint64_t N, uint64_t ws_bytes, TcScratch* t, uint8_t* base) {
    uint64_t off = 0;
    auto take = [&](auto** p, uint64_t bytes) {
        if (base) *p = reinterpret_cast<std::remove_pointer_t<decltype(p)>>(base + off);
        off += (bytes + 255) & ~255ull;
    };
    TcScratch s{};
    const uint64_t pairs = (uint64_t)kMaxPlanes * kMaxPlanes;
    take(&s.acat, pairs * M * K);
    take(&s.bcat, pairs * N * K);
    for (uint32_t q = 0; q < kMaxSums; q++) take(&s.g[q], 4 * M * N);
    take(&s.acc, K > kKChunk ? 8 * M * N : 0);
    take(&s.rowsum, 8 * M);
    take(&s.colsum, 8 * N);
    take(&s.flags, 8);
    take(&s.ws, ws_bytes);
    s.ws_bytes = ws_bytes;
    if (t) *t = s;
    return off;
}

typename TcGemm::Arguments tc_args(const uint8_t* a, uint64_t lda, const uint8_t* b, uint64_t ldb, int32_t* d, int m,
                                   int n, int k, int sm_count, int dev) {
    using SA = typename TcKernel::StrideA;
    using SB = typename TcKernel::StrideB;
    using SD = typename TcKernel::StrideD;
    SA sa = cute::make_stride((int64_t)lda, cute::Int<1>{}, (int64_t)0);
    SB sb = cute::make_stride((int64_t)ldb, cute::Int<1>{}, (int64_t)0);
    SD sd = cute::make_stride((int64_t)n, cute::Int<1>{}, (int64_t)0);
    cutlass::KernelHardwareInfo hw;
    hw.device_id = dev;
    hw.sm_count = sm_count;
    return typename TcGemm::Arguments{cutlass::gemm::GemmUniversalMode::kGemm, {m, n, k, 1}, {a, sa, b, sb},
                                      {{1, 0}, nullptr, sd, d, sd}, hw};
}

// workspace of the largest of the GEMM shapes (one to three plane pairs)
uint64_t tc_ws_bytes(uint64_t M, uint64_t K, uint64_t N) {
    const int kc = (int)(K < kKChunk ? K : kKChunk);
    uint64_t w = 0;
    for (int kk : {kc, 2 * kc, 3 * kc}) {
        auto args = tc_args(nullptr, K, nullptr, K, nullptr, (int)M, (int)N, kk, 148, 0);
        const uint64_t b = TcGemm::get_workspace_size(args);
        w = b > w ? b : w;
    }
    return w;
}

int run_gemm(const uint8_t* a, uint64_t lda, const uint8_t* b, uint64_t ldb, int32_t* d, uint64_t M, uint64_t N,
             uint64_t k, const TcScratch& s, int sm_count, int dev, cudaStream_t st) {
    auto args = tc_args(a, lda, b, ldb, d, (int)M, (int)N, (int)k, sm_count, dev);
    TcGemm g;
    if (g.can_implement(args) != cutlass::Status::kSuccess) return (int)cudaErrorInvalidValue;
    if (TcGemm::get_workspace_size(args) > s.ws_bytes) return (int)cudaErrorInvalidValue;
    if (g.initialize(args, s.ws, st) != cutlass::Status::kSuccess) return (int)cudaErrorUnknown;
    if (g.run(st) != cutlass::Status::kSuccess) return (int)cudaErrorLaunchFailure;
    ZK_LAUNCH_CHECK();
    return 0;
}

std::mutex g_sm_mu;
int g_sm_count[kMaxDevices];

int sm_count_of(int dev) {
    std::lock_guard<std::mutex> g(g_sm_mu);
    if (!g_sm_count[dev]) ZK_TRY(cudaDeviceGetAttribute(&g_sm_count[dev], cudaDevAttrMultiProcessorCount, dev));
    return 0;
}

bool tc_shape_ok(uint64_t M, uint64_t K, uint64_t N) {
    // TMA row strides of 16 bytes (u8 K, i32 N), int tile coordinates; the
    // plane kernel of B puts K / 32 in grid.y (at most 65535)
    return M && K && N && K % 16 == 0 && N % 4 == 0 && M < (1ull << 30) && N < (1ull << 30) &&
           3 * K < (1ull << 30) && ceil_div(K, 32) <= 65535;
}

// Zero the row / column sums and the width flags, then pack both operands
// for pa x pb planes (the flags record the operands' widths on the way).
int tc_pack(const uint64_t* d_a, const uint64_t* d_b, uint64_t m, uint64_t k, uint64_t n, uint32_t pa, uint32_t pb,
            const TcScratch& s, cudaStream_t stream) {
    ZK_TRY(cudaMemsetAsync(s.rowsum, 0, 8 * m, stream));
    ZK_TRY(cudaMemsetAsync(s.colsum, 0, 8 * n, stream));
    ZK_TRY(cudaMemsetAsync(s.flags, 0, 8, stream));
    k_pack_a<<<tc_grid(m * k / 16), kThr, 0, stream>>>(d_a, m, k, pa, pb, s.acat, s.rowsum, s.flags);
    ZK_LAUNCH_CHECK();
    const dim3 gb((unsigned)ceil_div(n, 32), (unsigned)ceil_div(k, 32));
    k_pack_b<<<gb, kThr, 0, stream>>>(d_b, k, n, pa, pb, s.bcat, s.colsum, s.flags + 1);
    ZK_LAUNCH_CHECK();
    return 0;
}

// The tensor path once the plane counts are known: the K bound, the packing
// (unless already done for these plane counts), one GEMM per plane-sum and K
// chunk, the recombination.
int tc_product(const uint64_t* d_a, const uint64_t* d_b, uint64_t m, uint64_t k, uint64_t n, uint64_t* d_c,
               uint32_t pa, uint32_t pb, const TcScratch& s, int dev, uint32_t* h_path, cudaStream_t stream,
               bool packed = false) {
    int rc = 0;
    // |sum_k a b| <= K 2^(8 (pa + pb) - 2) must stay below 2^63 for the
    // wrapping recombination: K < 2^(65 - 8 (pa + pb)) (2^17 for 3 x 3 planes)
    if (k >= (1ull << (65 - 8 * (pa + pb)))) {
        if (h_path) *h_path = 1;
        return matmul_field_dev(d_a, d_b, m, k, n, d_c, stream);
    }
    if (!packed) {
        rc = tc_pack(d_a, d_b, m, k, n, pa, pb, s, stream);
        if (rc) return rc;
    }
    const int sms = g_sm_count[dev];
    const uint64_t chunks = ceil_div(k, kKChunk);
    PlaneSums ps{};
    ps.count = pa + pb - 1;
    for (uint32_t q = 0; q < ps.count; q++) ps.g[q] = s.g[q];
    for (uint64_t c = 0; c < chunks; c++) {
        const uint64_t c0 = c * kKChunk, kc = k - c0 < kKChunk ? k - c0 : kKChunk;
        for (uint32_t sp = 0; sp + 1 < pa + pb; sp++) {
            const uint64_t cnt = pair_count(sp, pa, pb);
            const uint8_t* ar = s.acat + region_off(sp, pa, pb, m, k) + cnt * c0;
            const uint8_t* br = s.bcat + region_off(sp, pa, pb, n, k) + cnt * c0;
            rc = run_gemm(ar, cnt * k, br, cnt * k, s.g[sp], m, n, cnt * kc, s, sms, dev, stream);
            if (rc) return rc;
        }
        if (chunks > 1) {
            k_tc_accumulate<<<tc_grid(m * n), kThr, 0, stream>>>(ps, m * n, s.acc, c == 0 ? 1 : 0);
            ZK_LAUNCH_CHECK();
        }
    }
    k_tc_finish<<<tc_grid(m * n), kThr, 0, stream>>>(ps, chunks > 1 ? s.acc : nullptr, s.rowsum, s.colsum, m, n, k,
                                                     1ull << (8 * pa - 1), 1ull << (8 * pb - 1), d_c);
    ZK_LAUNCH_CHECK();
    if (h_path) *h_path = 0;
    return 0;
}

}  // namespace

}  // namespace zk

using namespace zk;

extern "C" {

uint64_t zkie2_matmul_fixed_scratch_elems(uint64_t m, uint64_t k, uint64_t n) {
    if (!tc_shape_ok(m, k, n)) return 1;
    return (tc_layout(m, k, n, tc_ws_bytes(m, k, n), nullptr, nullptr) + 7) / 8;
}

int zkie2_matmul_fixed(const uint64_t* d_a, const uint64_t* d_b, uint64_t m, uint64_t k, uint64_t n, uint64_t* d_c,
                       uint32_t policy, uint32_t* h_path, uint64_t* d_scratch, cudaStream_t stream) {
    uint32_t plan[3] = {1, 0, 0};
    const int rc = zkie2_matmul_fixed_ex(d_a, d_b, m, k, n, d_c, policy, plan, d_scratch, stream);
    if (!rc && h_path) *h_path = plan[0];
    return rc;
}

int zkie2_matmul_fixed_ex(const uint64_t* d_a, const uint64_t* d_b, uint64_t m, uint64_t k, uint64_t n,
                          uint64_t* d_c, uint32_t policy, uint32_t* h_plan, uint64_t* d_scratch,
                          cudaStream_t stream) {
    if (!h_plan) return (int)cudaErrorInvalidValue;
    h_plan[0] = 1;
    h_plan[1] = h_plan[2] = 0;
    uint32_t* h_path = h_plan;
    if (!d_a || !d_b || !d_c || !m || !k || !n || policy > 1) return (int)cudaErrorInvalidValue;
    // below ~2^27 multiply-adds the field kernel beats the tensor path's fixed
    // cost (range check read-back, plane packing, three GEMM launches)
    const bool small = (double)m * (double)k * (double)n < (double)(1ull << 27);
    const bool aligned = (reinterpret_cast<uintptr_t>(d_a) & 15) == 0;  // 16-byte loads of A
    if (!tc_shape_ok(m, k, n) || !aligned || (policy == 0 && small)) {
        if (h_path) *h_path = 1;
        return matmul_field_dev(d_a, d_b, m, k, n, d_c, stream);
    }
    if (!d_scratch) return (int)cudaErrorInvalidValue;
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) return (int)cudaErrorInvalidDevice;
    int rc = sm_count_of(dev);
    if (rc) return rc;
    TcScratch s;
    tc_layout(m, k, n, tc_ws_bytes(m, k, n), &s, reinterpret_cast<uint8_t*>(d_scratch));
    // pack for 16-bit operands (two planes) while recording their widths;
    // repack for three planes where a width needs it
    rc = tc_pack(d_a, d_b, m, k, n, 2, 2, s, stream);
    if (rc) return rc;
    uint32_t flags[2] = {0, 0};
    ZK_TRY(cudaMemcpyAsync(flags, s.flags, 8, cudaMemcpyDeviceToHost, stream));
    ZK_TRY(cudaStreamSynchronize(stream));
    if ((flags[0] | flags[1]) & 2u) {  // a value outside 24-bit fixed point: the exact field kernel
        if (h_path) *h_path = 1;
        return matmul_field_dev(d_a, d_b, m, k, n, d_c, stream);
    }
    const uint32_t pa = flags[0] ? 3 : 2, pb = flags[1] ? 3 : 2;
    const bool packed = pa == 2 && pb == 2;
    rc = tc_product(d_a, d_b, m, k, n, d_c, pa, pb, s, dev, h_path, stream, packed);
    if (!rc && h_plan[0] == 0) {
        h_plan[1] = pa;
        h_plan[2] = pb;
    }
    return rc;
}

int zkie2_matmul_fixed_planned(const uint64_t* d_a, const uint64_t* d_b, uint64_t m, uint64_t k, uint64_t n,
                               uint64_t* d_c, const uint32_t* h_plan, uint64_t* d_scratch, uint32_t* d_err,
                               cudaStream_t stream) {
    if (!d_a || !d_b || !d_c || !m || !k || !n || !h_plan) return (int)cudaErrorInvalidValue;
    if (h_plan[0] != 0) return matmul_field_dev(d_a, d_b, m, k, n, d_c, stream);
    const uint32_t pa = h_plan[1], pb = h_plan[2];
    if (pa < 2 || pa > 3 || pb < 2 || pb > 3 || !d_scratch || !d_err || !tc_shape_ok(m, k, n) ||
        (reinterpret_cast<uintptr_t>(d_a) & 15) != 0)
        return (int)cudaErrorInvalidValue;
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) return (int)cudaErrorInvalidDevice;
    int rc = sm_count_of(dev);
    if (rc) return rc;
    TcScratch s;
    tc_layout(m, k, n, tc_ws_bytes(m, k, n), &s, reinterpret_cast<uint8_t*>(d_scratch));
    rc = tc_pack(d_a, d_b, m, k, n, pa, pb, s, stream);
    if (rc) return rc;
    k_tc_plan_check<<<1, 32, 0, stream>>>(s.flags, pa, pb, d_err);
    ZK_LAUNCH_CHECK();
    uint32_t path = 0;
    return tc_product(d_a, d_b, m, k, n, d_c, pa, pb, s, dev, &path, stream, true);
}

uint64_t zkie2_matmul_fixed_runs_scratch_elems(uint64_t rows, uint64_t k, uint64_t n) {
    return zkie2_matmul_fixed_scratch_elems(rows, k, n);
}

int zkie2_matmul_fixed_runs(const uint64_t* d_a, const uint64_t* d_w, uint64_t n_experts, uint64_t k, uint64_t n,
                            const uint64_t* h_runs, uint64_t n_runs, uint64_t* d_c, uint64_t* d_scratch,
                            cudaStream_t stream) {
    if (!d_a || !d_w || !d_c || !h_runs || !k || !n) return (int)cudaErrorInvalidValue;
    uint64_t rows = 0, max_rows = 0;
    for (uint64_t r = 0; r < n_runs; r++) {
        const uint64_t e = h_runs[3 * r], r0 = h_runs[3 * r + 1], nr = h_runs[3 * r + 2];
        if (e >= n_experts || r0 != rows || nr == 0) return (int)cudaErrorInvalidValue;  // consecutive runs
        rows += nr;
        max_rows = nr > max_rows ? nr : max_rows;
    }
    if (rows == 0) return 0;
    // every run's rows start 16-byte aligned when d_a is (k % 16 == 0)
    const bool tc_ok = tc_shape_ok(max_rows, k, n) && (reinterpret_cast<uintptr_t>(d_a) & 15) == 0 && d_scratch;
    uint32_t pa = 0, pb = 0;
    TcScratch s{};
    const int dev = current_device();
    if (tc_ok) {
        if (dev < 0 || dev >= kMaxDevices) return (int)cudaErrorInvalidDevice;
        int rc = sm_count_of(dev);
        if (rc) return rc;
        tc_layout(max_rows, k, n, tc_ws_bytes(max_rows, k, n), &s, reinterpret_cast<uint8_t*>(d_scratch));
        // one range pass over every row and every expert block, one read-back
        ZK_TRY(cudaMemsetAsync(s.flags, 0, 8, stream));
        k_tc_range<<<tc_grid(rows * k), kThr, 0, stream>>>(d_a, rows * k, s.flags);
        ZK_LAUNCH_CHECK();
        k_tc_range<<<tc_grid(n_experts * k * n), kThr, 0, stream>>>(d_w, n_experts * k * n, s.flags + 1);
        ZK_LAUNCH_CHECK();
        uint32_t flags[2] = {0, 0};
        ZK_TRY(cudaMemcpyAsync(flags, s.flags, 8, cudaMemcpyDeviceToHost, stream));
        ZK_TRY(cudaStreamSynchronize(stream));
        if (!((flags[0] | flags[1]) & 2u)) {
            pa = flags[0] ? 3 : 2;
            pb = flags[1] ? 3 : 2;
            if (k >= (1ull << (65 - 8 * (pa + pb)))) pa = pb = 0;
        }
    }
    for (uint64_t r = 0; r < n_runs; r++) {
        const uint64_t e = h_runs[3 * r], r0 = h_runs[3 * r + 1], nr = h_runs[3 * r + 2];
        const uint64_t* a = d_a + r0 * k;
        const uint64_t* w = d_w + e * k * n;
        uint64_t* c = d_c + r0 * n;
        const bool small = (double)nr * (double)k * (double)n < (double)(1ull << 27);
        int rc;
        if (pa && !small) {
            uint32_t path = 0;
            rc = tc_product(a, w, nr, k, n, c, pa, pb, s, dev, &path, stream);
        } else {
            rc = matmul_field_dev(a, w, nr, k, n, c, stream);
        }
        if (rc) return rc;
    }
    return 0;
}

}  // extern "C"
