// a11: FP8 block-scaled linear.
//
//  * hk_quant_fp8: bf16 activations -> e4m3 in 1x128 blocks (a half-warp per block,
//    16-byte loads, amax by shuffle).
//  * hk_gemm_fp8: y = sum_kb (xq . wq)_kb * sx * sw.  The portable kernel here runs on CUDA
//    cores with an smem e4m3->fp32 table; the tcgen05 kernel (gemm_fp8_sm100.cu) takes over
//    the shapes it supports.
#include "common.cuh"
#include "gemm_fp8.cuh"

namespace {

constexpr int kBM = 64, kBN = 64, kBK = 128;

__global__ void quant_fp8_kernel(const uint4* __restrict__ x, int64_t rows, int32_t k,
                                 uint2* __restrict__ xq, float* __restrict__ sx) {
  // One half-warp per (row, 128-block): each lane converts 8 consecutive values (16-byte load,
  // 8-byte store); the block amax is reduced over the 16 lanes.
  const int64_t blocks_per_row = k / 128;
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t w = t >> 4;
  const int lane = threadIdx.x & 15;
  const bool on = w < rows * blocks_per_row;  // whole half-warps are on or off together
  const int64_t r = on ? w / blocks_per_row : 0, kb = on ? w % blocks_per_row : 0;
  uint4 u = make_uint4(0, 0, 0, 0);
  if (on) u = x[(r * k + kb * 128) / 8 + lane];
  const uint32_t wd[4] = {u.x, u.y, u.z, u.w};
  float v[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(wd[i] << 16);
    v[2 * i + 1] = __uint_as_float(wd[i] & 0xffff0000u);
  }
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (!on) return;
  const float s = __fdiv_rn(fmaxf(amax, 1e-12f), 448.0f);
  uint32_t lo = 0, hi = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) lo |= (uint32_t)f32_to_e4m3(__fdiv_rn(v[i], s)) << (8 * i);
#pragma unroll
  for (int i = 0; i < 4; ++i) hi |= (uint32_t)f32_to_e4m3(__fdiv_rn(v[4 + i], s)) << (8 * i);
  xq[(r * k + kb * 128) / 8 + lane] = make_uint2(lo, hi);
  if (lane == 0) sx[r * blocks_per_row + kb] = s;
}

// Portable tile: 64x64 outputs per CTA, 256 threads with 4x4 each, K stepped by the
// 128-wide scale blocks.  Optional row gather (MoE) through `rows_idx`.
__global__ void __launch_bounds__(256) gemm_fp8_portable_kernel(
    const uint8_t* __restrict__ xq, const float* __restrict__ sx, const uint8_t* __restrict__ wq,
    const float* __restrict__ sw, int64_t m, int32_t n, int32_t k, uint16_t* __restrict__ y) {
  __shared__ float lut[256];
  __shared__ uint8_t xs[kBM][kBK + 4];
  __shared__ uint8_t ws[kBN][kBK + 4];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int64_t m0 = (int64_t)blockIdx.x * kBM;
  const int n0 = blockIdx.y * kBN;
  lut[tid] = e4m3_to_f32((uint8_t)tid);
  const int kblocks = k / kBK;
  float acc[4][4] = {};
  for (int kb = 0; kb < kblocks; ++kb) {
    __syncthreads();
    for (int i = tid; i < kBM * (kBK / 16); i += 256) {
      const int r = i / (kBK / 16), c = i % (kBK / 16);
      uint4 vx = make_uint4(0, 0, 0, 0), vw = make_uint4(0, 0, 0, 0);
      if (m0 + r < m) vx = *reinterpret_cast<const uint4*>(xq + (m0 + r) * k + kb * kBK + c * 16);
      if (n0 + r < n) vw = *reinterpret_cast<const uint4*>(wq + (int64_t)(n0 + r) * k + kb * kBK + c * 16);
      uint32_t* dx = reinterpret_cast<uint32_t*>(&xs[r][c * 16]);
      uint32_t* dw = reinterpret_cast<uint32_t*>(&ws[r][c * 16]);
      dx[0] = vx.x; dx[1] = vx.y; dx[2] = vx.z; dx[3] = vx.w;
      dw[0] = vw.x; dw[1] = vw.y; dw[2] = vw.z; dw[3] = vw.w;
    }
    __syncthreads();
    float part[4][4] = {};
    for (int kk = 0; kk < kBK; ++kk) {
      float a[4], bv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = lut[xs[ty * 4 + i][kk]];
#pragma unroll
      for (int j = 0; j < 4; ++j) bv[j] = lut[ws[tx * 4 + j][kk]];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) part[i][j] = fmaf(a[i], bv[j], part[i][j]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t r = m0 + ty * 4 + i;
      const float a_s = r < m ? sx[r * kblocks + kb] : 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = n0 + tx * 4 + j;
        const float b_s = c < n ? sw[(int64_t)(c / 128) * kblocks + kb] : 0.f;
        acc[i][j] = fmaf(part[i][j], a_s * b_s, acc[i][j]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = m0 + ty * 4 + i;
    if (r >= m) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = n0 + tx * 4 + j;
      if (c < n) y[r * n + c] = f32_to_bf16_bits(acc[i][j]);
    }
  }
}

}  // namespace

namespace hk {

int gemm_fp8_portable(const uint8_t* xq, const float* sx, const uint8_t* wq, const float* sw,
                      int64_t m, int32_t n, int32_t k, uint16_t* y, cudaStream_t stream) {
  dim3 grid((unsigned)((m + kBM - 1) / kBM), (unsigned)((n + kBN - 1) / kBN));
  gemm_fp8_portable_kernel<<<grid, 256, 0, stream>>>(xq, sx, wq, sw, m, n, k, y);
  HK_TRY_LAUNCH("gemm_fp8_portable_kernel");
  return HK_OK;
}

int quant_fp8_launch(const uint16_t* x, int64_t rows, int32_t k, uint8_t* xq, float* sx,
                     cudaStream_t stream) {
  const int64_t threads = rows * (k / 128) * 16;
  if (threads == 0) return HK_OK;
  quant_fp8_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, stream>>>(
      (const uint4*)x, rows, k, (uint2*)xq, sx);
  HK_TRY_LAUNCH("quant_fp8_kernel");
  return HK_OK;
}

}  // namespace hk

extern "C" {

int hk_quant_fp8(const uint16_t* x, int64_t rows, int32_t k, uint8_t* xq, float* sx,
                 void* stream) {
  HK_TRY(hk::ensure_device());
  HK_REQUIRE(rows == 0 || (x && xq && sx), "hk_quant_fp8: null pointer");
  HK_REQUIRE(rows >= 0 && k > 0 && k % 128 == 0, "hk_quant_fp8: k %d must be a multiple of 128", k);
  HK_REQUIRE(((uintptr_t)x % 16 == 0) && ((uintptr_t)xq % 8 == 0), "hk_quant_fp8: misaligned buffers");
  return hk::quant_fp8_launch(x, rows, k, xq, sx, (cudaStream_t)stream);
}

int hk_gemm_fp8(const uint8_t* xq, const float* sx, const uint8_t* wq, const float* sw,
                int64_t m, int32_t n, int32_t k, uint16_t* y, void* stream) {
  HK_TRY(hk::ensure_device());
  HK_REQUIRE(m == 0 || (xq && sx && wq && sw && y), "hk_gemm_fp8: null pointer");
  HK_REQUIRE(m >= 0 && n > 0 && n % 16 == 0 && k > 0 && k % 128 == 0,
             "hk_gemm_fp8: m %lld n %d k %d (n a multiple of 16, k of 128)", (long long)m, n, k);
  HK_REQUIRE(((uintptr_t)xq | (uintptr_t)wq) % 16 == 0, "hk_gemm_fp8: operands must be 16-byte aligned");
  if (m == 0) return HK_OK;
  if (hk::gemm_fp8_sm100_supported(m, n, k))
    return hk::gemm_fp8_sm100(xq, sx, wq, sw, m, n, k, y, (cudaStream_t)stream);
  if (hk::gemm_fp8_swapab_supported(m, n, k))
    return hk::gemm_fp8_swapab(xq, sx, wq, sw, m, n, k, y, (cudaStream_t)stream);
  return hk::gemm_fp8_portable(xq, sx, wq, sw, m, n, k, y, (cudaStream_t)stream);
}

}  // extern "C"
