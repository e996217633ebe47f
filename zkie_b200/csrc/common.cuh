// common.cuh -- shared host/device helpers of libzkie_b200.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>

namespace zk {

// Return the first CUDA error as an int, the convention of every exported
// entry point (0 = success), as in crates/zkie-core/src/pcs/cuda_ffi.rs:2-46.
#define ZK_TRY(expr)                                   \
    do {                                               \
        cudaError_t _e = (expr);                       \
        if (_e != cudaSuccess) return (int)_e;         \
    } while (0)

#define ZK_LAUNCH_CHECK() ZK_TRY(cudaGetLastError())

constexpr int kMaxDevices = 64;

inline int current_device() {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess) return -1;
    return d;
}

inline uint64_t ceil_div(uint64_t a, uint64_t b) { return (a + b - 1) / b; }

inline uint32_t log2_exact(uint64_t x) {
    uint32_t r = 0;
    while ((1ull << r) < x) r++;
    return r;
}

}  // namespace zk
