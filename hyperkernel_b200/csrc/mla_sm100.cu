// tcgen05 2-SM MLA decode kernel: placeholder until the kernel lands; reports itself
// unsupported so hk_mla_decode(impl=0) takes the portable kernel.
#include "common.cuh"
#include "mla_sm100.cuh"

namespace hk {

bool mla_sm100_supported(int32_t, int32_t, int32_t, int32_t) { return false; }

size_t mla_sm100_workspace(int32_t, int32_t, int32_t, int32_t) { return 0; }

int mla_sm100(const uint16_t*, const uint16_t*, const int32_t*, int32_t, const int32_t*,
              const int32_t*, int32_t, int32_t, int32_t, int32_t, int64_t, int32_t, float,
              uint16_t*, float*, void*, size_t, cudaStream_t) {
  return fail(HK_EINVAL, "mla_sm100: not built");
}

}  // namespace hk
