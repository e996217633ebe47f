// Stand-in for sppark 0.1.15's <util/gpu_t.cuh> as the reference's
// poseidon2_merkle.cu uses it: ngpus(), the number of visible CUDA devices
// (0 when the runtime reports none).  Test infrastructure
// (oracle/build_ref.py only).
#pragma once
#include <cuda_runtime.h>

#include <cstddef>

inline size_t ngpus() {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return (size_t)n;
}
