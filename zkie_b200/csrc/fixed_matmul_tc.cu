// fixed_matmul_tc.cu -- the forward witness of a fixed-point matmul on the
// tensor cores: par::mm_par_fixed (crates/zkie-ops/src/par.rs:41-89).
//
// The reference maps every field element to i64 (to_i64: values above p/2
// are negative), takes exact i64 dot products and maps them back (from_i64);
// the result equals the field matmul, and it falls back to the field matmul
// when the i64 sums could overflow.  Here, when every input lies in
// [-2^15, 2^15) (16-bit fixed point, the inference witness range), the
// products run on the 5th-generation tensor cores as u8 x u8 -> s32 GEMMs:
//   a' = a + 2^15 in [0, 2^16) splits into bytes a' = 256 a_h + a_l, so
//   sum_k a'b' = 2^16 (A_h B_h) + 2^8 (A_h B_l + A_l B_h) + A_l B_l,
// the middle term as ONE GEMM over a doubled K ([A_h | A_l] times [B_l ; B_h]),
// and the offset comes off exactly:
//   sum_k a b = sum_k a'b' - 2^15 (rowsum_i(A') + colsum_j(B')) + K 2^30.
// Every s32 sum stays below 2 * 8192 * 255^2 < 2^31 by splitting K into
// chunks of at most 8192 (partial results add up in i64).  Inputs outside
// 16 bits, or a K or N that TMA cannot address (K % 16, N % 4), take the
// exact field kernel instead, so the output always equals the field matmul.
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

constexpr uint64_t kKChunk = 8192;  // 2 * kKChunk * 255^2 < 2^31
constexpr uint64_t kOffset = 1ull << 15;
constexpr int kThr = 256;

// to_i64(x) + 2^15 when to_i64(x) is in [-2^15, 2^15), else sets *bad
__device__ __forceinline__ uint32_t shifted16(uint64_t x, uint32_t* bad) {
    x = gl_canon(x);
    if (x < kOffset) return (uint32_t)(x + kOffset);
    if (x >= GL_P - kOffset) return (uint32_t)(x - (GL_P - kOffset));
    atomicOr(bad, 1u);
    return 0;
}

// Column of chunk layout: element k of a row lands at 2 * kc0 + (k - kc0) for
// the high (or first) plane and at 2 * kc0 + kc + (k - kc0) for the other,
// kc0 = the chunk start, kc = the chunk width.
__device__ __forceinline__ void cat_cols(uint64_t k, uint64_t K, uint64_t& first, uint64_t& second) {
    const uint64_t c0 = k / kKChunk * kKChunk;
    const uint64_t kc = K - c0 < kKChunk ? K - c0 : kKChunk;
    first = 2 * c0 + (k - c0);
    second = first + kc;
}

// A (M x K field, row-major) -> AH, AL (M x K bytes), ACAT (M x 2K: per chunk
// [a_h | a_l]), rowsum[i] = sum_k a'.  One thread per 16 consecutive elements
// of a row (K % 16 == 0, and chunk widths are multiples of 16): 16-byte loads
// and 16-byte stores of each plane.
__global__ void __launch_bounds__(kThr)
    k_planes_a(const uint64_t* __restrict__ a, uint64_t M, uint64_t K, uint8_t* __restrict__ ah,
               uint8_t* __restrict__ al, uint8_t* __restrict__ acat, unsigned long long* __restrict__ rowsum,
               uint32_t* __restrict__ bad) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t groups = M * K / 16, span = (groups + 31) & ~31ull;  // warp-uniform trip count
    for (uint64_t gi = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; gi < span; gi += stride) {
        const bool in = gi < groups;
        const uint64_t idx = in ? gi * 16 : 0, i = idx / K, k = idx - i * K;
        unsigned long long sum = 0;
        if (in) {
        const ulonglong2* src = reinterpret_cast<const ulonglong2*>(a + idx);
        uint32_t hw[4] = {0, 0, 0, 0}, lw[4] = {0, 0, 0, 0};
#pragma unroll
        for (int q = 0; q < 8; q++) {
            const ulonglong2 pr = __ldg(src + q);
            const uint32_t v0 = shifted16(pr.x, bad), v1 = shifted16(pr.y, bad);
            sum += v0 + v1;
            const int e = 2 * q, w = e >> 2, sh = (e & 3) * 8;
            hw[w] |= ((v0 >> 8) << sh) | ((v1 >> 8) << (sh + 8));
            lw[w] |= ((v0 & 255u) << sh) | ((v1 & 255u) << (sh + 8));
        }
        const uint4 h = make_uint4(hw[0], hw[1], hw[2], hw[3]), l = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        *reinterpret_cast<uint4*>(ah + idx) = h;
        *reinterpret_cast<uint4*>(al + idx) = l;
        uint64_t c1, c2;
        cat_cols(k, K, c1, c2);
        *reinterpret_cast<uint4*>(acat + i * 2 * K + c1) = h;
        *reinterpret_cast<uint4*>(acat + i * 2 * K + c2) = l;
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
}

// B (K x N field, row-major) -> transposed planes BH, BL (N x K bytes) and
// BCAT (N x 2K: per chunk [b_l | b_h]), colsum[j] = sum_k b'; 32 x 32 tiles
// through shared memory so the field reads run along rows of B and the byte
// writes (four bytes per store) along rows of the transposes.  One atomic per
// column per tile.
__global__ void __launch_bounds__(kThr)
    k_planes_b(const uint64_t* __restrict__ b, uint64_t K, uint64_t N, uint8_t* __restrict__ bh,
               uint8_t* __restrict__ bl, uint8_t* __restrict__ bcat, unsigned long long* __restrict__ colsum,
               uint32_t* __restrict__ bad) {
    __shared__ uint32_t tile[32][33];
    const uint64_t k0 = (uint64_t)blockIdx.y * 32, n0 = (uint64_t)blockIdx.x * 32;
    const uint32_t tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8
    for (uint32_t r = ty; r < 32; r += 8) {
        const uint64_t k = k0 + r, n = n0 + tx;
        tile[r][tx] = (k < K && n < N) ? shifted16(__ldg(b + k * N + n), bad) : 0;
    }
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
        uint32_t h = 0, l = 0;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const uint32_t v = tile[kq + e][nr];
            h |= (v >> 8) << (8 * e);
            l |= (v & 255u) << (8 * e);
        }
        *reinterpret_cast<uint32_t*>(bh + n * K + k) = h;
        *reinterpret_cast<uint32_t*>(bl + n * K + k) = l;
        uint64_t c1, c2;
        cat_cols(k, K, c1, c2);
        *reinterpret_cast<uint32_t*>(bcat + n * 2 * K + c1) = l;
        *reinterpret_cast<uint32_t*>(bcat + n * 2 * K + c2) = h;
    }
}

// acc (+)= 2^16 hh + 2^8 x + ll
__global__ void k_tc_accumulate(const int32_t* __restrict__ hh, const int32_t* __restrict__ x,
                                const int32_t* __restrict__ ll, uint64_t mn, int64_t* __restrict__ acc, int first) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < mn; i += stride) {
        const int64_t v = ((int64_t)hh[i] << 16) + ((int64_t)x[i] << 8) + (int64_t)ll[i];
        acc[i] = first ? v : acc[i] + v;
    }
}

// c = from_i64(sum - 2^15 (rowsum_i + colsum_j) + K 2^30), with sum either the
// i64 accumulator or, for one chunk, 2^16 hh + 2^8 x + ll directly.
__global__ void k_tc_finish(const int32_t* __restrict__ hh, const int32_t* __restrict__ x,
                            const int32_t* __restrict__ ll, const int64_t* __restrict__ acc,
                            const unsigned long long* __restrict__ rowsum,
                            const unsigned long long* __restrict__ colsum, uint64_t M, uint64_t N, uint64_t K,
                            uint64_t* __restrict__ c) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < M * N; idx += stride) {
        const uint64_t i = idx / N, j = idx - i * N;
        const int64_t s = acc ? acc[idx] : ((int64_t)hh[idx] << 16) + ((int64_t)x[idx] << 8) + (int64_t)ll[idx];
        const int64_t v = s - (int64_t)((rowsum[i] + colsum[j]) << 15) + (int64_t)(K << 30);
        c[idx] = v >= 0 ? (uint64_t)v : GL_P - (uint64_t)(-v);  // from_i64; |v| < 2^62
    }
}

unsigned tc_grid(uint64_t work) {
    const uint64_t b = ceil_div(work, kThr);
    return (unsigned)(b < 148ull * 16 ? (b ? b : 1) : 148ull * 16);
}

// Scratch layout in bytes (regions 256-byte aligned).
struct TcScratch {
    uint8_t *ah, *al, *acat, *bh, *bl, *bcat;
    int32_t *hh, *x, *ll;
    int64_t* acc;
    unsigned long long *rowsum, *colsum;
    uint32_t* bad;
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
    take(&s.ah, M * K);
    take(&s.al, M * K);
    take(&s.acat, 2 * M * K);
    take(&s.bh, N * K);
    take(&s.bl, N * K);
    take(&s.bcat, 2 * N * K);
    take(&s.hh, 4 * M * N);
    take(&s.x, 4 * M * N);
    take(&s.ll, 4 * M * N);
    take(&s.acc, K > kKChunk ? 8 * M * N : 0);
    take(&s.rowsum, 8 * M);
    take(&s.colsum, 8 * N);
    take(&s.bad, 8);
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

// workspace of the largest of the three GEMM shapes
uint64_t tc_ws_bytes(uint64_t M, uint64_t K, uint64_t N) {
    const int kc = (int)(K < kKChunk ? K : kKChunk);
    uint64_t w = 0;
    for (int kk : {kc, 2 * kc}) {
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
           2 * K < (1ull << 30) && ceil_div(K, 32) <= 65535;
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
    ZK_TRY(cudaMemsetAsync(s.rowsum, 0, 8 * m, stream));
    ZK_TRY(cudaMemsetAsync(s.colsum, 0, 8 * n, stream));
    ZK_TRY(cudaMemsetAsync(s.bad, 0, 4, stream));
    k_planes_a<<<tc_grid(m * k / 16), kThr, 0, stream>>>(d_a, m, k, s.ah, s.al, s.acat, s.rowsum, s.bad);
    ZK_LAUNCH_CHECK();
    const dim3 gb((unsigned)ceil_div(n, 32), (unsigned)ceil_div(k, 32));
    if (gb.y > 65535) return (int)cudaErrorInvalidValue;
    k_planes_b<<<gb, kThr, 0, stream>>>(d_b, k, n, s.bh, s.bl, s.bcat, s.colsum, s.bad);
    ZK_LAUNCH_CHECK();
    uint32_t bad = 0;
    ZK_TRY(cudaMemcpyAsync(&bad, s.bad, 4, cudaMemcpyDeviceToHost, stream));
    ZK_TRY(cudaStreamSynchronize(stream));
    if (bad) {  // a value outside 16-bit fixed point: the exact field kernel
        if (h_path) *h_path = 1;
        return matmul_field_dev(d_a, d_b, m, k, n, d_c, stream);
    }
    const int sms = g_sm_count[dev];
    const uint64_t chunks = ceil_div(k, kKChunk);
    for (uint64_t c = 0; c < chunks; c++) {
        const uint64_t c0 = c * kKChunk, kc = k - c0 < kKChunk ? k - c0 : kKChunk;
        rc = run_gemm(s.ah + c0, k, s.bh + c0, k, s.hh, m, n, kc, s, sms, dev, stream);
        if (!rc) rc = run_gemm(s.acat + 2 * c0, 2 * k, s.bcat + 2 * c0, 2 * k, s.x, m, n, 2 * kc, s, sms, dev, stream);
        if (!rc) rc = run_gemm(s.al + c0, k, s.bl + c0, k, s.ll, m, n, kc, s, sms, dev, stream);
        if (rc) return rc;
        if (chunks > 1) {
            k_tc_accumulate<<<tc_grid(m * n), kThr, 0, stream>>>(s.hh, s.x, s.ll, m * n, s.acc, c == 0);
            ZK_LAUNCH_CHECK();
        }
    }
    k_tc_finish<<<tc_grid(m * n), kThr, 0, stream>>>(s.hh, s.x, s.ll, chunks > 1 ? s.acc : nullptr, s.rowsum, s.colsum,
                                                     m, n, k, d_c);
    ZK_LAUNCH_CHECK();
    if (h_path) *h_path = 0;
    return 0;
}

}  // extern "C"
