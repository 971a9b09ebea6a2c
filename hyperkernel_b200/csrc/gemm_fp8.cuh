// Internal interfaces of the FP8 block-scaled GEMM kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace hk {

int quant_fp8_launch(const uint16_t* x, int64_t rows, int32_t k, uint8_t* xq, float* sx,
                     cudaStream_t stream);

int gemm_fp8_portable(const uint8_t* xq, const float* sx, const uint8_t* wq, const float* sw,
                      int64_t m, int32_t n, int32_t k, uint16_t* y, cudaStream_t stream);

bool gemm_fp8_sm100_supported(int64_t m, int32_t n, int32_t k);

int gemm_fp8_sm100(const uint8_t* xq, const float* sx, const uint8_t* wq, const float* sw,
                   int64_t m, int32_t n, int32_t k, uint16_t* y, cudaStream_t stream);

// Fewer than 128 token rows: the swap-AB tensor-core kernel (weights on the MMA's M side).
bool gemm_fp8_swapab_supported(int64_t m, int32_t n, int32_t k);

int gemm_fp8_swapab(const uint8_t* xq, const float* sx, const uint8_t* wq, const float* sw,
                    int64_t m, int32_t n, int32_t k, uint16_t* y, cudaStream_t stream);

}  // namespace hk
