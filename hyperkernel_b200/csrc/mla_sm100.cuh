// Interface of the tcgen05 2-SM MLA decode kernel (mla_sm100.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace hk {

bool mla_sm100_supported(int32_t heads, int32_t page_size, int32_t num_tokens, int32_t num_lanes);

size_t mla_sm100_workspace(int32_t num_lanes, int32_t num_tokens, int32_t heads,
                           int32_t max_kv_len);

// kv_begin / kv_end (device, per lane; both null for whole causal prefixes) restrict each
// lane to KV rows [kv_begin, kv_end); out_f32, when not null, takes the output in fp32
// instead of `out` (bf16).  Rows with nothing to attend get o = 0, lse = -inf.
int mla_sm100(const uint16_t* q, const uint16_t* kv_cache, const int32_t* block_table,
              int32_t bt_stride, const int32_t* cu_seqlens, const int32_t* positions,
              const int32_t* kv_begin, const int32_t* kv_end, int32_t num_lanes,
              int32_t num_tokens, int32_t heads, int32_t page_size, int64_t num_slots,
              int32_t max_kv_len, float scale, uint16_t* out, float* out_f32, float* lse,
              void* workspace, size_t workspace_bytes, cudaStream_t stream);

}  // namespace hk
