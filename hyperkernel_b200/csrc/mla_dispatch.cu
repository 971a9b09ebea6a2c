// hk_mla_decode: chooses between the tcgen05 2-SM kernel (128 heads, bf16 cache) and the
// portable CUDA-core kernel, and sizes the scratch both need.
#include "attn.cuh"
#include "common.cuh"
#include "mla_sm100.cuh"

extern "C" {

size_t hk_mla_workspace_size(int32_t num_lanes, int32_t num_tokens, int32_t heads,
                             int32_t max_kv_len) {
  size_t a = hk::mla_portable_workspace(num_tokens, heads, max_kv_len);
  size_t b = hk::mla_sm100_workspace(num_lanes, num_tokens, heads, max_kv_len);
  return a > b ? a : b;
}

int hk_mla_decode(const uint16_t* q, const uint16_t* kv_cache, const int32_t* block_table,
                  int32_t bt_stride, const int32_t* cu_seqlens, const int32_t* positions,
                  int32_t num_lanes, int32_t num_tokens, int32_t heads, int32_t page_size,
                  int64_t num_slots, int32_t max_kv_len, float scale, uint16_t* out, float* lse,
                  void* workspace, size_t workspace_bytes, int32_t impl, void* stream) {
  HK_TRY(hk::ensure_device());
  HK_REQUIRE(num_tokens == 0 || (q && kv_cache && block_table && cu_seqlens && positions && out && lse),
             "hk_mla_decode: null pointer");
  HK_REQUIRE(heads > 0 && heads % 16 == 0, "hk_mla_decode: heads %d not a multiple of 16", heads);
  HK_REQUIRE(num_lanes > 0 && num_tokens >= 0 && page_size > 0 && bt_stride > 0 && max_kv_len >= 0,
             "hk_mla_decode: bad sizes");
  HK_REQUIRE(impl >= 0 && impl <= 2, "hk_mla_decode: impl %d not in 0..2", impl);
  HK_REQUIRE(((uintptr_t)q | (uintptr_t)kv_cache | (uintptr_t)out) % 16 == 0,
             "hk_mla_decode: q, cache and out must be 16-byte aligned");
  if (num_tokens == 0) return HK_OK;
  const bool sm100_ok = hk::mla_sm100_supported(heads, page_size, num_tokens, num_lanes);
  if (impl == 2 && !sm100_ok)
    return hk::fail(HK_EINVAL, "hk_mla_decode: the tcgen05 kernel needs 128 heads, pages of 64 "
                               "rows and one query row per lane");
  if (impl == 2 || (impl == 0 && sm100_ok))
    return hk::mla_sm100(q, kv_cache, block_table, bt_stride, cu_seqlens, positions, nullptr,
                         nullptr, num_lanes, num_tokens, heads, page_size, num_slots, max_kv_len,
                         scale, out, nullptr, lse, workspace, workspace_bytes, (cudaStream_t)stream);
  return hk::mla_portable(q, kv_cache, nullptr, nullptr, block_table, bt_stride, cu_seqlens,
                          positions, num_lanes, num_tokens, heads, page_size, num_slots,
                          max_kv_len, scale, out, lse, workspace, workspace_bytes,
                          (cudaStream_t)stream);
}

int hk_mla_partial(const uint16_t* q, const uint16_t* kv_cache, const int32_t* block_table,
                   int32_t bt_stride, const int32_t* cu_seqlens, const int32_t* positions,
                   const int32_t* kv_begin, const int32_t* kv_end, int32_t num_lanes,
                   int32_t num_tokens, int32_t heads, int32_t page_size, int64_t num_slots,
                   int32_t max_kv_len, float scale, float* o_part, float* lse_part,
                   void* workspace, size_t workspace_bytes, void* stream) {
  HK_TRY(hk::ensure_device());
  HK_REQUIRE(num_tokens == 0 || (q && kv_cache && block_table && cu_seqlens && positions && kv_begin &&
                                  kv_end && o_part && lse_part),
             "hk_mla_partial: null pointer");
  HK_REQUIRE(num_lanes > 0 && num_tokens >= 0 && page_size > 0 && bt_stride > 0 && max_kv_len >= 0,
             "hk_mla_partial: bad sizes");
  HK_REQUIRE(((uintptr_t)q | (uintptr_t)kv_cache | (uintptr_t)o_part) % 16 == 0,
             "hk_mla_partial: q, cache and o_part must be 16-byte aligned");
  if (num_tokens == 0) return HK_OK;
  if (!hk::mla_sm100_supported(heads, page_size, num_tokens, num_lanes))
    return hk::fail(HK_EINVAL, "hk_mla_partial: the tcgen05 kernel needs 128 heads and pages of 64 "
                               "rows (hk_mla_partial_fp8 takes other shapes)");
  return hk::mla_sm100(q, kv_cache, block_table, bt_stride, cu_seqlens, positions, kv_begin, kv_end,
                       num_lanes, num_tokens, heads, page_size, num_slots, max_kv_len, scale, nullptr,
                       o_part, lse_part, workspace, workspace_bytes, (cudaStream_t)stream);
}

}  // extern "C"
