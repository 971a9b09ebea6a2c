// Row gather / scatter: the data movement around the expert-parallel all-to-all.
//
// Dispatch sends each rank the routed rows of its experts in permuted order
// (dst[i] = src[idx[i]]); combine puts the expert outputs that arrive back in sender order
// (dst[idx[i]] = src[i]).  One CTA per row, 16-byte vectors when the row allows them, else
// 4-byte words; an index outside the source (gather) or destination (scatter) is skipped and
// recorded in the device error word.
#include "common.cuh"

namespace {

template <typename V>
__global__ void gather_rows_bytes_kernel(const V* __restrict__ src, int64_t src_rows,
                                         const int32_t* __restrict__ idx, int64_t rows, int32_t vecs,
                                         V* __restrict__ dst, unsigned long long* err) {
  const int64_t r = blockIdx.x;
  if (r >= rows) return;
  const int32_t s = idx[r];
  if (s < 0 || s >= src_rows) {
    if (threadIdx.x == 0) hk_flag(err, hk::kErrMoeRow, (unsigned)r);
    return;
  }
  for (int i = threadIdx.x; i < vecs; i += blockDim.x) dst[r * vecs + i] = src[(int64_t)s * vecs + i];
}

template <typename V>
__global__ void scatter_rows_bytes_kernel(const V* __restrict__ src, int64_t rows,
                                          const int32_t* __restrict__ idx, int64_t dst_rows, int32_t vecs,
                                          V* __restrict__ dst, unsigned long long* err) {
  const int64_t r = blockIdx.x;
  if (r >= rows) return;
  const int32_t d = idx[r];
  if (d < 0 || d >= dst_rows) {
    if (threadIdx.x == 0) hk_flag(err, hk::kErrMoeRow, (unsigned)r);
    return;
  }
  for (int i = threadIdx.x; i < vecs; i += blockDim.x) dst[(int64_t)d * vecs + i] = src[r * vecs + i];
}

int check_rows(const void* src, const int32_t* idx, const void* dst, int64_t rows, int32_t row_bytes) {
  HK_REQUIRE(rows == 0 || (src && idx && dst), "null pointer");
  HK_REQUIRE(rows >= 0 && rows < (1ll << 31), "rows %lld", (long long)rows);
  HK_REQUIRE(row_bytes > 0 && row_bytes % 4 == 0, "row_bytes %d must be a positive multiple of 4", row_bytes);
  HK_REQUIRE(((uintptr_t)src | (uintptr_t)dst) % 4 == 0, "rows must be 4-byte aligned");
  return HK_OK;
}

}  // namespace

extern "C" {

int hk_gather_rows(const void* src, int64_t src_rows, const int32_t* idx, int64_t rows, int32_t row_bytes,
                   void* dst, void* stream) {
  HK_TRY(hk::ensure_device());
  HK_TRY(check_rows(src, idx, dst, rows, row_bytes));
  if (rows == 0) return HK_OK;
  if (row_bytes % 16 == 0 && ((uintptr_t)src | (uintptr_t)dst) % 16 == 0)
    gather_rows_bytes_kernel<uint4><<<(unsigned)rows, 128, 0, (cudaStream_t)stream>>>(
        (const uint4*)src, src_rows, idx, rows, row_bytes / 16, (uint4*)dst, hk::err_word());
  else
    gather_rows_bytes_kernel<uint32_t><<<(unsigned)rows, 128, 0, (cudaStream_t)stream>>>(
        (const uint32_t*)src, src_rows, idx, rows, row_bytes / 4, (uint32_t*)dst, hk::err_word());
  HK_TRY_LAUNCH("gather_rows_bytes_kernel");
  return HK_OK;
}

int hk_scatter_rows(const void* src, int64_t rows, const int32_t* idx, int64_t dst_rows, int32_t row_bytes,
                    void* dst, void* stream) {
  HK_TRY(hk::ensure_device());
  HK_TRY(check_rows(src, idx, dst, rows, row_bytes));
  if (rows == 0) return HK_OK;
  if (row_bytes % 16 == 0 && ((uintptr_t)src | (uintptr_t)dst) % 16 == 0)
    scatter_rows_bytes_kernel<uint4><<<(unsigned)rows, 128, 0, (cudaStream_t)stream>>>(
        (const uint4*)src, rows, idx, dst_rows, row_bytes / 16, (uint4*)dst, hk::err_word());
  else
    scatter_rows_bytes_kernel<uint32_t><<<(unsigned)rows, 128, 0, (cudaStream_t)stream>>>(
        (const uint32_t*)src, rows, idx, dst_rows, row_bytes / 4, (uint32_t*)dst, hk::err_word());
  HK_TRY_LAUNCH("scatter_rows_bytes_kernel");
  return HK_OK;
}

}  // extern "C"
