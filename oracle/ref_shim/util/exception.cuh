// Stand-in for sppark 0.1.15's <util/exception.cuh> as the reference's
// goldilocks_ntt.cu uses it: CUDA_OK(expr) throws cuda_error when expr is not
// cudaSuccess, and cuda_error::code() returns that error.  Test
// infrastructure (oracle/build_ref.py only).
#pragma once
#include <cuda_runtime.h>

class cuda_error {
    cudaError_t c;

public:
    explicit cuda_error(cudaError_t e) : c(e) {}
    cudaError_t code() const { return c; }
};

#define CUDA_OK(expr)                                   \
    do {                                                \
        cudaError_t _zk_ref_e = (expr);                 \
        if (_zk_ref_e != cudaSuccess) throw cuda_error(_zk_ref_e); \
    } while (0)
