// hist.cuh -- lookup multiplicities: m[x[i]] += 1 for i < n over a table of
// t entries, an index at or past t flagged in *bad (the reference would index
// out of bounds and panic; common/logup_gkr.rs:251-260).
//
// Lookup columns are often concentrated on a few entries (one-hot
// selections, zero distances, the high limbs of similar values), where one
// global atomic per element serialises on a handful of addresses.  Each warp
// therefore merges equal indices first (__match_any_sync: one atomic per
// distinct index per warp), and indices below kHistShared are counted in a
// per-block shared-memory histogram that goes to the global one once per
// non-empty bin at the end.
#pragma once

#include <cstdint>

namespace zk {

constexpr uint32_t kHistShared = 4096;  // shared-memory bins per block (16 KB)

__device__ __forceinline__ void hist_global_add(uint32_t* m, uint32_t j, uint32_t c) { atomicAdd(m + j, c); }
__device__ __forceinline__ void hist_global_add(unsigned long long* m, uint32_t j, uint32_t c) {
    atomicAdd(m + j, (unsigned long long)c);
}

// The whole grid walks x in warp-sized strides (every lane of a warp takes
// the same trip count, as __match_any_sync needs); blockDim is a multiple of
// 32.
template <typename Count>
__device__ __forceinline__ void hist_grid(const uint32_t* __restrict__ x, uint64_t n, uint64_t t,
                                          Count* __restrict__ m, uint32_t* __restrict__ bad, uint32_t bad_bit) {
    __shared__ uint32_t bins[kHistShared];
    const uint32_t nb = t < kHistShared ? (uint32_t)t : kHistShared;
    for (uint32_t j = threadIdx.x; j < nb; j += blockDim.x) bins[j] = 0;
    __syncthreads();
    const unsigned lane = threadIdx.x & 31;
    const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x >> 5);
    const uint64_t w = (uint64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    for (uint64_t base = w * 32; base < n; base += warps * 32) {
        const uint64_t i = base + lane;
        const uint32_t xi = i < n ? __ldg(x + i) : 0;
        const bool in = i < n && xi < t;
        if (i < n && !in) atomicOr(bad, bad_bit);
        const unsigned long long key = in ? (unsigned long long)xi : (1ull << 32);
        const unsigned peers = __match_any_sync(0xFFFFFFFFu, key);
        if (in && lane == (unsigned)(__ffs(peers) - 1)) {
            const uint32_t c = (uint32_t)__popc(peers);
            if (xi < nb)
                atomicAdd(bins + xi, c);
            else
                hist_global_add(m, xi, c);
        }
    }
    __syncthreads();
    for (uint32_t j = threadIdx.x; j < nb; j += blockDim.x) {
        const uint32_t c = bins[j];
        if (c) hist_global_add(m, j, c);
    }
}

}  // namespace zk
