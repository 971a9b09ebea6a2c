// hk_moe_grouped_noalloc: the grouped expert FFN with its scratch in a fixed device array.
//
// Some callers cannot allocate device memory: an engine that reaches this library only
// through the C ABI from another language, with no CUDA allocator of its own; a host whose
// device memory is owned by a pool allocator that forbids raw cudaMalloc; a step loop that
// must not take cudaMalloc's implicit device-wide synchronisation.  For them this entry point
// takes no workspace argument and allocates nothing: the scratch that hk_moe_grouped asks its
// caller for (the requantised intermediate h, its scales and the tile list) lives in the
// file-scope array below, which the driver reserves on every GPU that loads this library and
// keeps until the process exits.
//
// Limits: at most kMaxRows permuted rows and an intermediate size of at most kMaxInter
// (kScratchBytes = 2,167,040 bytes, about 2.1 MB).  Larger problems are refused with
// HK_EINVAL; use hk_moe_grouped with a caller workspace for them.
//
// Every call uses the same array and the array keeps the last call's contents.  Nothing in
// it has to start at zero: each call writes the tile list, h and its scales before reading
// them.  Calls whose executions overlap on the GPU (two streams, or two host threads) race on
// the array and corrupt each other's results; serialise them.  Rows whose indices are out of
// range are skipped as in hk_moe_grouped but are not recorded in the device error word
// (recording would need the error word that the library allocates on first use); offsets that
// are not a valid scan give an empty tile list, so y is left unwritten, also unreported.
//
// The first call on a device looks the array's device address up with cudaGetSymbolAddress
// (host code cannot use the symbol itself: in host code it names a host-side shadow, not
// device memory).  That first call should therefore come before any stream capture.
#include <mutex>

#include "common.cuh"
#include "moe.cuh"

namespace {

constexpr int64_t kMaxRows = 1024;
constexpr int32_t kMaxInter = 2048;
constexpr int kMaxExperts = 512;  // hk_moe_grouped's expert limit (tile list capacity)
constexpr size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }
// The same arithmetic as hk::moe_portable_workspace(kMaxRows, kMaxInter): the scratch of the
// CUDA-core expert kernels, which this entry point runs.
constexpr size_t kScratchBytes =
    al256((size_t)kMaxRows * kMaxInter) + al256((size_t)kMaxRows * (kMaxInter / 128) * 4) +
    al256((size_t)(kMaxRows / 64 + kMaxExperts + 1) * 2 * 4 + 4);
static_assert(kScratchBytes == 2167040, "scratch size stated in the header comment");

static __device__ __align__(256) uint8_t g_moe_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_mu;

// Device address of this device's copy of g_moe_scratch (looked up once per device).
int scratch_of_device(void** out) {
  int dev = -1;
  HK_TRY_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return hk::fail(HK_ENODEV, "device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_moe_scratch);
    if (e != cudaSuccess) return hk::cuda_fail(e, "cudaGetSymbolAddress(g_moe_scratch)");
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return HK_OK;
}

}  // namespace

extern "C" int hk_moe_grouped_noalloc(const uint8_t* xq, const float* sx, int32_t tokens,
                                      const int32_t* offsets, const int32_t* perm_token,
                                      int64_t rows, int32_t num_experts, int32_t hidden,
                                      int32_t inter, const uint8_t* w13, const float* s13,
                                      const uint8_t* w2, const float* s2, uint16_t* y,
                                      void* stream) {
  HK_TRY(hk::ensure_device());
  HK_REQUIRE(rows >= 0 && rows <= kMaxRows,
             "hk_moe_grouped_noalloc: %lld rows, at most %lld (use hk_moe_grouped)",
             (long long)rows, (long long)kMaxRows);
  HK_REQUIRE(inter > 0 && inter <= kMaxInter,
             "hk_moe_grouped_noalloc: inter %d, at most %d (use hk_moe_grouped)", inter, kMaxInter);
  HK_REQUIRE(hk::moe_portable_workspace(rows, inter) <= kScratchBytes,
             "hk_moe_grouped_noalloc: scratch of %zu bytes too small", kScratchBytes);
  void* scratch = nullptr;
  HK_TRY(scratch_of_device(&scratch));
  return hk::moe_grouped_run(xq, sx, tokens, offsets, perm_token, rows, num_experts, hidden, inter,
                             w13, s13, w2, s2, y, scratch, kScratchBytes, true, nullptr,
                             (cudaStream_t)stream);
}
