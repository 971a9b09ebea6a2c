// Shared helpers for the sm_100a kernels behind include/hk.h: error plumbing, the device
// error word, bf16 / e4m3 conversions and the deterministic sigmoid used by the router.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/hk.h"

namespace hk {

// Host side (common.cu).
int fail(int code, const char* fmt, ...);
int cuda_fail(cudaError_t e, const char* what);
void clear_error();
// HK_OK when the current device is usable (sm_100 family), else HK_ENODEV / HK_ECUDA.
int ensure_device();
// Device pointer to the current device's error word (allocated once per device).
unsigned long long* err_word();
int sm_count();
// Counts kernel launches made by this library (HK_TRY_LAUNCH calls it after each launch).
void note_launch();

// Sites recorded in the device error word (upper 32 bits), with a detail value below.
enum ErrSite : unsigned {
  kErrPackOverflow = 1,   // more rows than max_tokens
  kErrPackPage = 2,       // a row whose page is the scratch page or past the pool
  kErrAppendSlot = 3,     // a slot outside the cache
  kErrAttnPage = 4,       // an attention read through a page id outside the pool
  kErrWaitTimeout = 5,    // a bounded mbarrier wait ran out
  kErrMoeRow = 6,         // a permuted row or token index out of range
  kErrRouteInput = 7,     // non-finite router logits
  kErrToken = 8,          // a token id outside the vocabulary (the model's embedding lookup)
};

}  // namespace hk

#define HK_TRY_CUDA(call)                                          \
  do {                                                             \
    cudaError_t hk_e_ = (call);                                    \
    if (hk_e_ != cudaSuccess) return hk::cuda_fail(hk_e_, #call);  \
  } while (0)

#define HK_TRY_LAUNCH(name)                                        \
  do {                                                             \
    cudaError_t hk_e_ = cudaGetLastError();                        \
    if (hk_e_ != cudaSuccess) return hk::cuda_fail(hk_e_, name);   \
    hk::note_launch();                                             \
  } while (0)

#define HK_REQUIRE(cond, ...)                                      \
  do {                                                             \
    if (!(cond)) return hk::fail(HK_EINVAL, __VA_ARGS__);          \
  } while (0)

#define HK_TRY(expr)                 \
  do {                               \
    int hk_r_ = (expr);              \
    if (hk_r_ != HK_OK) return hk_r_; \
  } while (0)

// Records the first error on the device: bit 63 set, site in bits 32..62, detail below.
__device__ __forceinline__ void hk_flag(unsigned long long* word, unsigned site, unsigned detail) {
  if (word != nullptr) {
    unsigned long long v = (1ull << 63) | ((unsigned long long)site << 32) | detail;
    atomicCAS(word, 0ull, v);
  }
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
  return __uint_as_float(((uint32_t)b) << 16);
}

__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  __nv_bfloat16 h = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&h);
}

// e4m3 byte -> float (exact).
__device__ __forceinline__ float e4m3_to_f32(uint8_t v) {
  __nv_fp8_e4m3 t;
  t.__x = v;
  return float(t);
}

// float -> e4m3 byte, round to nearest even, saturating to +-448 (cvt.rn.satfinite).
__device__ __forceinline__ uint8_t f32_to_e4m3(float f) {
  return (uint8_t)__nv_cvt_float_to_fp8(f, __NV_SATFINITE, __NV_E4M3);
}

// Deterministic sigmoid: 1 / (1 + e^-x) with e^y computed by this file's own routine
// (Cody-Waite split of y*log2(e) into n + r, then a degree-7 Taylor polynomial for
// 2^r = e^(r ln 2) evaluated by Horner's rule with fmaf), so the CPU oracle reproduces
// it bit for bit with the same fmaf sequence.  Relative error ~1e-7 over the router's range.
#ifdef __CUDA_ARCH__
#define HK_MUL_RN(a, b) __fmul_rn((a), (b))
#define HK_SUB_RN(a, b) __fsub_rn((a), (b))
#define HK_ADD_RN(a, b) __fadd_rn((a), (b))
#define HK_DIV_RN(a, b) __fdiv_rn((a), (b))
#else
#define HK_MUL_RN(a, b) ((a) * (b))
#define HK_SUB_RN(a, b) ((a) - (b))
#define HK_ADD_RN(a, b) ((a) + (b))
#define HK_DIV_RN(a, b) ((a) / (b))
#endif

__device__ __host__ __forceinline__ float hk_exp_det(float y) {
  if (y > 88.0f) y = 88.0f;
  if (y < -87.0f) y = -87.0f;
  const float kLog2e = 1.44269504088896341f;
  float t = HK_MUL_RN(y, kLog2e);  // explicit rounding: never contracted into an fma
  float n = rintf(t);
  float r = HK_SUB_RN(t, n);  // |r| <= 0.5, exact for |t| < 2^23
  // 2^r = e^(r*ln2): Taylor coefficients (ln2)^i / i!.
  const float c1 = 0.693147180559945309f, c2 = 0.240226506959100712f,
              c3 = 0.0555041086648215800f, c4 = 0.00961812910762847717f,
              c5 = 0.00133335581464284434f, c6 = 0.000154035303933816099f,
              c7 = 0.0000152527338040598403f;
  float p = c7;
  p = fmaf(p, r, c6);
  p = fmaf(p, r, c5);
  p = fmaf(p, r, c4);
  p = fmaf(p, r, c3);
  p = fmaf(p, r, c2);
  p = fmaf(p, r, c1);
  p = fmaf(p, r, 1.0f);
  return ldexpf(p, (int)n);
}

__device__ __host__ __forceinline__ float hk_sigmoid_det(float x) {
  return HK_DIV_RN(1.0f, HK_ADD_RN(1.0f, hk_exp_det(-x)));
}
