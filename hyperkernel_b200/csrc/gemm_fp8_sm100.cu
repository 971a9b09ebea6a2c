// tcgen05 FP8 block-scaled GEMM: placeholder until the kernel lands; reports itself
// unsupported so hk_gemm_fp8 takes the portable kernel.
#include "common.cuh"
#include "gemm_fp8.cuh"

namespace hk {

bool gemm_fp8_sm100_supported(int64_t, int32_t, int32_t) { return false; }

int gemm_fp8_sm100(const uint8_t*, const float*, const uint8_t*, const float*, int64_t, int32_t,
                   int32_t, uint16_t*, cudaStream_t) {
  return fail(HK_EINVAL, "gemm_fp8_sm100: not built");
}

}  // namespace hk
