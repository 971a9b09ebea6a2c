// a7 pack and a8 KV append.
//
// pack: one CTA of 1024 threads scans the lanes (warp shuffles + one smem hop per CTA
// round), then every warp expands its lanes' rows.  The step's index arrays are a few KB,
// so this kernel is latency-bound by design; it replaces the packing the reference's
// closed megakernel does from the `drafting` ring message (src/gpu/feed.rs:40-103 fills
// it; block-table rows come from Cache::pages, src/engine/cache.rs:195-226).
//
// append: one warp per new row, 16-byte loads and stores, the row scattered to
// cache[slot].  Rows are 1152 B (576 bf16) for the MLA latent cache, so a warp moves a
// row in 3 coalesced sweeps.
#include "common.cuh"

namespace {

constexpr int kPackThreads = 1024;

// Block-wide exclusive scan of one int per thread; returns the exclusive prefix and sets
// *total to the block sum.  Uses the caller's 32-int smem scratch.
__device__ __forceinline__ int block_excl_scan(int v, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = (lane < (int)(blockDim.x >> 5)) ? warp_sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    warp_sums[lane] = w;  // inclusive prefix over warps
  }
  __syncthreads();
  int before = (warp > 0 ? warp_sums[warp - 1] : 0) + x - v;
  *total = warp_sums[(blockDim.x >> 5) - 1];
  __syncthreads();
  return before;
}

__global__ void __launch_bounds__(kPackThreads) pack_kernel(
    const int32_t* __restrict__ lane_tokens, const int32_t* __restrict__ lane_pos,
    const int32_t* __restrict__ block_table, int32_t bt_stride, int32_t num_lanes,
    int32_t page_size, int32_t num_pages, int32_t max_tokens, int32_t* __restrict__ cu_seqlens,
    int32_t* __restrict__ seq_lens, int32_t* __restrict__ positions,
    int32_t* __restrict__ slot_mapping, int32_t* __restrict__ token_lane,
    int32_t* __restrict__ active, unsigned long long* err) {
  __shared__ int warp_sums[32];
  int carry = 0, active_carry = 0;
  for (int base = 0; base < num_lanes; base += kPackThreads) {
    const int i = base + (int)threadIdx.x;
    int n = (i < num_lanes) ? lane_tokens[i] : 0;
    n = n > 0 ? n : 0;
    int total, active_total;
    int excl = block_excl_scan(n, warp_sums, &total);
    // Active lanes compacted in ascending order: ballot inside the warp, scan across warps.
    int is_active = n > 0;
    int a_excl = block_excl_scan(is_active, warp_sums, &active_total);
    if (i < num_lanes) {
      cu_seqlens[i] = carry + excl;
      seq_lens[i] = n > 0 ? lane_pos[i] + n : 0;
      if (is_active) active[1 + active_carry + a_excl] = i;
    }
    carry += total;
    active_carry += active_total;
  }
  if (threadIdx.x == 0) {
    cu_seqlens[num_lanes] = carry;
    active[0] = active_carry;
    if (carry > max_tokens) hk_flag(err, hk::kErrPackOverflow, (unsigned)carry);
  }
  __syncthreads();  // cu_seqlens written by this block are visible to it after the barrier
  const int lane_id = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int b = warp; b < num_lanes; b += kPackThreads / 32) {
    const int n = lane_tokens[b];
    if (n <= 0) continue;
    const int start = cu_seqlens[b];
    const int pos0 = lane_pos[b];
    for (int j = lane_id; j < n; j += 32) {
      const int t = start + j;
      if (t >= max_tokens) continue;  // flagged above
      const int pos = pos0 + j;
      const int blk = pos / page_size;
      const int page = (pos >= 0 && blk < bt_stride) ? block_table[(int64_t)b * bt_stride + blk] : -1;
      int slot;
      if (page <= 0 || page >= num_pages) {
        hk_flag(err, hk::kErrPackPage, (unsigned)b);
        slot = -1;
      } else {
        slot = page * page_size + pos % page_size;
      }
      positions[t] = pos;
      slot_mapping[t] = slot;
      token_lane[t] = b;
    }
  }
}

__global__ void append_vec_kernel(const uint4* __restrict__ src, const int32_t* __restrict__ slot,
                                  int32_t num_tokens, int32_t row_vec, uint4* __restrict__ cache,
                                  int64_t num_slots, unsigned long long* err) {
  const int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= num_tokens) return;
  const int s = slot[t];
  if (s < 0 || s >= num_slots) {
    if (lane == 0) hk_flag(err, hk::kErrAppendSlot, (unsigned)t);
    return;
  }
  const uint4* in = src + t * row_vec;
  uint4* out = cache + (int64_t)s * row_vec;
  for (int v = lane; v < row_vec; v += 32) out[v] = in[v];
}

// Page-blocked latent rows: 16-byte vector v of a row (8 elements) goes to block v / 8 of
// the row's page, at row (slot % page_rows), column (v % 8) * 8.
__global__ void append_blocked_kernel(const uint4* __restrict__ src,
                                      const int32_t* __restrict__ slot, int32_t num_tokens,
                                      int32_t row_vec, int32_t page_rows,
                                      uint4* __restrict__ cache, int64_t num_slots,
                                      unsigned long long* err) {
  const int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= num_tokens) return;
  const int s = slot[t];
  if (s < 0 || s >= num_slots) {
    if (lane == 0) hk_flag(err, hk::kErrAppendSlot, (unsigned)t);
    return;
  }
  const uint4* in = src + t * row_vec;
  uint4* page = cache + (int64_t)(s / page_rows) * page_rows * row_vec;
  const int r = s % page_rows;
  for (int v = lane; v < row_vec; v += 32)
    page[(int64_t)(v >> 3) * page_rows * 8 + r * 8 + (v & 7)] = in[v];
}

// Two-buffer variant for GQA K and V rows.
__global__ void append_kv_kernel(const uint4* __restrict__ k_src, const uint4* __restrict__ v_src,
                                 const int32_t* __restrict__ slot, int32_t num_tokens,
                                 int32_t row_vec, uint4* __restrict__ k_cache,
                                 uint4* __restrict__ v_cache, int64_t num_slots,
                                 unsigned long long* err) {
  const int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= num_tokens) return;
  const int s = slot[t];
  if (s < 0 || s >= num_slots) {
    if (lane == 0) hk_flag(err, hk::kErrAppendSlot, (unsigned)t);
    return;
  }
  for (int v = lane; v < row_vec; v += 32) {
    k_cache[(int64_t)s * row_vec + v] = k_src[t * row_vec + v];
    v_cache[(int64_t)s * row_vec + v] = v_src[t * row_vec + v];
  }
}

// e4m3 row quantisation: scale = max(amax, 1e-12) / 448, q = e4m3_rn_satfinite(x / scale).
// FP8 rows -> the page-blocked bf16 layout: one warp per cache row, bf16(e4m3 * scale).
__global__ void dequant_fp8_blocked_kernel(const uint2* __restrict__ src, const float* __restrict__ scales,
                                           int64_t num_slots, int32_t row_vec, int32_t page_rows,
                                           const int32_t* __restrict__ pages, int64_t num_pages,
                                           const int32_t* __restrict__ slots, int64_t rows,
                                           uint4* __restrict__ dst, unsigned long long* err) {
  const int64_t i = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (i >= rows) return;
  // cache row: i itself; with a page list, row i % page_rows of listed page i / page_rows;
  // with a slot list, slots[i]
  int64_t s = i;
  if (slots != nullptr) {
    const int32_t sl = slots[i];
    if (sl < 0 || sl >= num_slots) {
      if (lane == 0) hk_flag(err, hk::kErrAttnPage, (unsigned)i);
      return;
    }
    s = sl;
  } else if (pages != nullptr) {
    const int32_t pg = pages[i / page_rows];
    if (pg < 0 || (int64_t)pg * page_rows >= num_slots || pg >= num_pages) {
      if (lane == 0) hk_flag(err, hk::kErrAttnPage, (unsigned)(i / page_rows));
      return;
    }
    s = (int64_t)pg * page_rows + i % page_rows;
  }
  const float sc = scales[s];
  const uint2* in = src + s * row_vec;
  uint4* page = dst + (s / page_rows) * page_rows * row_vec;
  const int64_t r = s % page_rows;
  for (int v = lane; v < row_vec; v += 32) {
    const uint2 u = in[v];
    const uint32_t b[2] = {u.x, u.y};
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t word = b[i >> 1] >> (16 * (i & 1));
      const float lo = e4m3_to_f32((uint8_t)(word & 0xff)) * sc;
      const float hi = e4m3_to_f32((uint8_t)((word >> 8) & 0xff)) * sc;
      w[i] = (uint32_t)f32_to_bf16_bits(lo) | ((uint32_t)f32_to_bf16_bits(hi) << 16);
    }
    page[(int64_t)(v >> 3) * page_rows * 8 + r * 8 + (v & 7)] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

__global__ void append_fp8_kernel(const uint4* __restrict__ src, const int32_t* __restrict__ slot,
                                  int32_t num_tokens, int32_t row_vec, uint2* __restrict__ cache,
                                  float* __restrict__ scales, int64_t num_slots,
                                  unsigned long long* err) {
  const int64_t t = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (t >= num_tokens) return;
  const int s = slot[t];
  if (s < 0 || s >= num_slots) {
    if (lane == 0) hk_flag(err, hk::kErrAppendSlot, (unsigned)t);
    return;
  }
  const uint4* in = src + t * row_vec;
  float amax = 0.f;
  for (int v = lane; v < row_vec; v += 32) {
    uint4 u = in[v];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      amax = fmaxf(amax, fabsf(__uint_as_float(w[i] << 16)));
      amax = fmaxf(amax, fabsf(__uint_as_float(w[i] & 0xffff0000u)));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float scale = __fdiv_rn(fmaxf(amax, 1e-12f), 448.0f);
  for (int v = lane; v < row_vec; v += 32) {
    uint4 u = in[v];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    uint32_t q[2] = {0, 0};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t lo = f32_to_e4m3(__fdiv_rn(__uint_as_float(w[i] << 16), scale));
      uint32_t hi = f32_to_e4m3(__fdiv_rn(__uint_as_float(w[i] & 0xffff0000u), scale));
      q[i >> 1] |= (lo | (hi << 8)) << ((i & 1) * 16);
    }
    cache[(int64_t)s * row_vec + v] = make_uint2(q[0], q[1]);
  }
  if (lane == 0) scales[s] = scale;
}

}  // namespace

extern "C" {

int hk_pack(const int32_t* lane_tokens, const int32_t* lane_pos, const int32_t* block_table,
            int32_t bt_stride, int32_t num_lanes, int32_t page_size, int32_t num_pages,
            int32_t max_tokens, int32_t* cu_seqlens, int32_t* seq_lens, int32_t* positions,
            int32_t* slot_mapping, int32_t* token_lane, int32_t* active, void* stream) {
  HK_TRY(hk::ensure_device());
  HK_REQUIRE(lane_tokens && lane_pos && block_table && cu_seqlens && seq_lens && positions &&
                 slot_mapping && token_lane && active,
             "hk_pack: null pointer");
  HK_REQUIRE(num_lanes >= 0 && bt_stride > 0 && page_size > 0 && num_pages > 0 && max_tokens >= 0,
             "hk_pack: bad sizes (lanes %d, stride %d, page %d, pages %d, max_tokens %d)",
             num_lanes, bt_stride, page_size, num_pages, max_tokens);
  pack_kernel<<<1, kPackThreads, 0, (cudaStream_t)stream>>>(
      lane_tokens, lane_pos, block_table, bt_stride, num_lanes, page_size, num_pages, max_tokens,
      cu_seqlens, seq_lens, positions, slot_mapping, token_lane, active, hk::err_word());
  HK_TRY_LAUNCH("pack_kernel");
  return HK_OK;
}

int hk_kv_append_bf16(const uint16_t* kv_new, const int32_t* slot_mapping, int32_t num_tokens,
                      int32_t row_elems, int32_t page_rows, uint16_t* kv_cache, int64_t num_slots,
                      void* stream) {
  HK_TRY(hk::ensure_device());
  HK_REQUIRE(num_tokens == 0 || (kv_new && slot_mapping && kv_cache), "hk_kv_append_bf16: null pointer");
  HK_REQUIRE(num_tokens >= 0 && row_elems > 0 && row_elems % 8 == 0 && num_slots > 0,
             "hk_kv_append_bf16: row_elems %d must be a positive multiple of 8", row_elems);
  HK_REQUIRE(page_rows >= 0 && (page_rows == 0 || (row_elems % 64 == 0 && num_slots % page_rows == 0)),
             "hk_kv_append_bf16: page_rows %d needs row_elems %% 64 == 0 and whole pages",
             page_rows);
  HK_REQUIRE(((uintptr_t)kv_new | (uintptr_t)kv_cache) % 16 == 0,
             "hk_kv_append_bf16: buffers must be 16-byte aligned");
  if (num_tokens == 0) return HK_OK;
  const int64_t threads = (int64_t)num_tokens * 32;
  if (page_rows == 0) {
    append_vec_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        (const uint4*)kv_new, slot_mapping, num_tokens, row_elems / 8, (uint4*)kv_cache,
        num_slots, hk::err_word());
    HK_TRY_LAUNCH("append_vec_kernel");
  } else {
    append_blocked_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
        (const uint4*)kv_new, slot_mapping, num_tokens, row_elems / 8, page_rows,
        (uint4*)kv_cache, num_slots, hk::err_word());
    HK_TRY_LAUNCH("append_blocked_kernel");
  }
  return HK_OK;
}

int hk_kv_dequant_fp8(const uint8_t* kv_fp8, const float* kv_scale, int64_t num_slots, int32_t row_elems,
                      int32_t page_rows, const int32_t* pages, int64_t n_pages, uint16_t* kv_bf16,
                      void* stream) {
  HK_TRY(hk::ensure_device());
  HK_REQUIRE((pages ? n_pages == 0 : num_slots == 0) || (kv_fp8 && kv_scale && kv_bf16),
             "hk_kv_dequant_fp8: null pointer");
  HK_REQUIRE(num_slots >= 0 && page_rows > 0 && num_slots % page_rows == 0 && row_elems > 0 && row_elems % 64 == 0,
             "hk_kv_dequant_fp8: num_slots %lld (a multiple of page_rows %d), row_elems %d (a multiple of 64)",
             (long long)num_slots, page_rows, row_elems);
  HK_REQUIRE(((uintptr_t)kv_fp8 % 8 == 0) && ((uintptr_t)kv_bf16 % 16 == 0), "hk_kv_dequant_fp8: misaligned buffers");
  HK_REQUIRE(pages == nullptr || n_pages >= 0, "hk_kv_dequant_fp8: negative page count");
  const int64_t rows = pages == nullptr ? num_slots : n_pages * page_rows;
  if (rows == 0) return HK_OK;
  const int64_t threads = rows * 32;
  dequant_fp8_blocked_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      (const uint2*)kv_fp8, kv_scale, num_slots, row_elems / 8, page_rows, pages, num_slots / page_rows, nullptr,
      rows, (uint4*)kv_bf16, hk::err_word());
  HK_TRY_LAUNCH("dequant_fp8_blocked_kernel");
  return HK_OK;
}

int hk_kv_dequant_fp8_rows(const uint8_t* kv_fp8, const float* kv_scale, int64_t num_slots, int32_t row_elems,
                           int32_t page_rows, const int32_t* slots, int64_t n_rows, uint16_t* kv_bf16,
                           void* stream) {
  HK_TRY(hk::ensure_device());
  HK_REQUIRE(n_rows == 0 || (kv_fp8 && kv_scale && kv_bf16 && slots), "hk_kv_dequant_fp8_rows: null pointer");
  HK_REQUIRE(num_slots >= 0 && page_rows > 0 && num_slots % page_rows == 0 && row_elems > 0 && row_elems % 64 == 0,
             "hk_kv_dequant_fp8_rows: num_slots %lld (a multiple of page_rows %d), row_elems %d (a multiple of 64)",
             (long long)num_slots, page_rows, row_elems);
  HK_REQUIRE(((uintptr_t)kv_fp8 % 8 == 0) && ((uintptr_t)kv_bf16 % 16 == 0),
             "hk_kv_dequant_fp8_rows: misaligned buffers");
  HK_REQUIRE(n_rows >= 0, "hk_kv_dequant_fp8_rows: negative row count");
  if (n_rows == 0) return HK_OK;
  const int64_t threads = n_rows * 32;
  dequant_fp8_blocked_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      (const uint2*)kv_fp8, kv_scale, num_slots, row_elems / 8, page_rows, nullptr, num_slots / page_rows, slots,
      n_rows, (uint4*)kv_bf16, hk::err_word());
  HK_TRY_LAUNCH("dequant_fp8_blocked_kernel");
  return HK_OK;
}

int hk_kv_append_fp8(const uint16_t* kv_new, const int32_t* slot_mapping, int32_t num_tokens,
                     int32_t row_elems, uint8_t* kv_cache, float* kv_scale, int64_t num_slots,
                     void* stream) {
  HK_TRY(hk::ensure_device());
  HK_REQUIRE(num_tokens == 0 || (kv_new && slot_mapping && kv_cache && kv_scale), "hk_kv_append_fp8: null pointer");
  HK_REQUIRE(num_tokens >= 0 && row_elems > 0 && row_elems % 8 == 0 && num_slots > 0,
             "hk_kv_append_fp8: row_elems %d must be a positive multiple of 8", row_elems);
  HK_REQUIRE(((uintptr_t)kv_new % 16 == 0) && ((uintptr_t)kv_cache % 8 == 0),
             "hk_kv_append_fp8: misaligned buffers");
  if (num_tokens == 0) return HK_OK;
  const int64_t threads = (int64_t)num_tokens * 32;
  append_fp8_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      (const uint4*)kv_new, slot_mapping, num_tokens, row_elems / 8, (uint2*)kv_cache, kv_scale,
      num_slots, hk::err_word());
  HK_TRY_LAUNCH("append_fp8_kernel");
  return HK_OK;
}

int hk_kv_append_f32(const float* k_new, const float* v_new, const int32_t* slot_mapping,
                     int32_t num_tokens, int32_t row_elems, float* k_cache, float* v_cache,
                     int64_t num_slots, void* stream) {
  HK_TRY(hk::ensure_device());
  HK_REQUIRE(num_tokens == 0 || (k_new && v_new && slot_mapping && k_cache && v_cache),
             "hk_kv_append_f32: null pointer");
  HK_REQUIRE(num_tokens >= 0 && row_elems > 0 && row_elems % 4 == 0 && num_slots > 0,
             "hk_kv_append_f32: row_elems %d must be a positive multiple of 4", row_elems);
  HK_REQUIRE(((uintptr_t)k_new | (uintptr_t)v_new | (uintptr_t)k_cache | (uintptr_t)v_cache) % 16 == 0,
             "hk_kv_append_f32: buffers must be 16-byte aligned");
  if (num_tokens == 0) return HK_OK;
  const int64_t threads = (int64_t)num_tokens * 32;
  append_kv_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      (const uint4*)k_new, (const uint4*)v_new, slot_mapping, num_tokens, row_elems / 4,
      (uint4*)k_cache, (uint4*)v_cache, num_slots, hk::err_word());
  HK_TRY_LAUNCH("append_kv_kernel");
  return HK_OK;
}

}  // extern "C"
