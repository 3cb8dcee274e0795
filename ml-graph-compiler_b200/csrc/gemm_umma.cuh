// tcgen05 (UMMA) GEMM for sm_100a: placeholder that declines every problem until the tensor-core
// kernel lands; run_gemm then uses the exact-fp32 SIMT kernel.
#pragma once

#include "common.cuh"
#include "gemm_simt.cuh"

namespace mgc {

inline int try_gemm_umma(const GemmParams &p, cudaStream_t stream, int *taken) {
    (void)p;
    (void)stream;
    *taken = 0;
    return MGC_CUDA_OK;
}

}  // namespace mgc
