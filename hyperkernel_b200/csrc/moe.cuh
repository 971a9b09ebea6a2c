// Internal interface of the grouped MoE FFN launcher (moe.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace hk {

// hk_moe_grouped's launcher with the device error word passed in (nullptr: bad rows are
// skipped without being recorded).
int moe_grouped_run(const uint8_t* xq, const float* sx, int32_t tokens, const int32_t* offsets,
                    const int32_t* perm_token, int64_t rows, int32_t num_experts, int32_t hidden,
                    int32_t inter, const uint8_t* w13, const float* s13, const uint8_t* w2,
                    const float* s2, uint16_t* y, void* workspace, size_t workspace_bytes,
                    unsigned long long* err, cudaStream_t s);

}  // namespace hk
