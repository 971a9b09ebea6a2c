// Internal interfaces shared by the attention translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace hk {

int lse_merge_launch(const float* o_parts, const float* lse_parts, int32_t n_parts, int64_t rows,
                     int32_t dv, void* out, bool bf16_out, float* lse_out, cudaStream_t stream);

size_t mla_portable_workspace(int32_t num_tokens, int32_t heads, int32_t max_kv_len);

int mla_portable(const uint16_t* q, const uint16_t* kv_bf16, const uint8_t* kv_fp8,
                 const float* kv_scale, const int32_t* bt, int32_t bt_stride, const int32_t* cu,
                 const int32_t* positions, int32_t num_lanes, int32_t num_tokens, int32_t heads,
                 int32_t page_size, int64_t num_slots, int32_t max_kv_len, float scale,
                 uint16_t* out, float* lse, void* workspace, size_t workspace_bytes,
                 cudaStream_t stream);

int mla_portable_partial(const uint16_t* q, const uint8_t* kv_fp8, const float* kv_scale,
                         const int32_t* bt, int32_t bt_stride, const int32_t* cu,
                         const int32_t* positions, const int32_t* kv_begin, const int32_t* kv_end,
                         int32_t num_lanes, int32_t num_tokens, int32_t heads, int32_t page_size,
                         int64_t num_slots, int32_t max_kv_len, float scale, float* o_part,
                         float* lse_part, void* workspace, size_t workspace_bytes,
                         cudaStream_t stream);

}  // namespace hk
