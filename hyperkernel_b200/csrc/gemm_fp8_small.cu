// a11 for decode-sized batches: the FP8 block-scaled GEMM with fewer than 128 token rows, on the
// tensor cores in swap-AB form.
//
// A decode step's projections multiply a handful of token rows (one per live lane, or 1 + drafts)
// by a large weight matrix, so the weights are the operand that matters and the GEMM is
// HBM-bound on them (2 m flops per weight byte, far below the FP8 ridge).  The weights take the
// MMA's M side (128 weight rows = one 128x128 scale block row) and a tile of up to 64 token rows
// the N side: D[128 weight rows][64 tokens] = W[rows][kb] . X[tokens][kb]^T per 128-wide K block
// (tcgen05 kind::f8f6f4, M 128, N 64, four K-32 instructions), into one of four TMEM buffers.
// Promotion warps add D * sw[row block][kb] * sx[token][kb] in fp32 registers, the DeepSeek-style
// scale rule the one- and two-SM kernels apply, and write y[token][weight row] as bf16 at the end.
//
// Work unit = (128-row weight block, 64-row token tile), so each weight byte is read once per
// token tile (once in all for m <= 64).  Roles per CTA (10 warps): warp 0 TMA producer, warp 1
// TMEM owner and MMA issuer, warps 2..9 promotion (two per TMEM lane quarter, 32 token columns
// each; thread = weight row).  Persistent over the units; every wait is bounded (1 s) and
// records the error word; copies and MMAs in flight are drained before exit.
#include <cuda.h>

#include "common.cuh"
#include "gemm_fp8.cuh"
#include "sm100.cuh"

namespace {

using namespace hk::sm100;

constexpr int kTok = 64;     // token rows per unit: the MMA's N
constexpr int kWRows = 128;  // weight rows per unit: the MMA's M
constexpr int kBK = 128;
constexpr int kThreads = 320;
constexpr int kCols = 32;    // token columns per promotion warp
constexpr int kWBytes = kWRows * kBK;  // 16 KB
constexpr int kXBytes = kTok * kBK;    // 8 KB
constexpr int kStageBytes = kWBytes + kXBytes;
constexpr int kStages = 8;
constexpr int kTBufs = 4;
constexpr uint32_t kTmemCols = kTBufs * kTok;  // 256
constexpr uint32_t kIdesc = idesc_e4m3(kWRows, kTok);
constexpr unsigned long long kDrainNs = 1000000000ull;

constexpr int kOffCtl = kStages * kStageBytes;
constexpr int kBarFull = 0;     // [kStages]
constexpr int kBarEmpty = 64;   // [kStages]
constexpr int kBarTFull = 128;  // [kTBufs]
constexpr int kBarTEmpty = 160; // [kTBufs]
constexpr int kTmemSlot = 192;
constexpr int kAbort = 196;
constexpr int kCtlBytes = 256;
constexpr int kSmem = kOffCtl + kCtlBytes;
static_assert(kSmem <= 232448, "shared memory budget");
static_assert(kStageBytes % 1024 == 0 && kWBytes % 1024 == 0, "128-byte swizzle atoms stay aligned");

struct Params {
  const float* sx;  // [m][kblocks]
  const float* sw;  // [ceil(n/128)][kblocks]
  uint16_t* y;      // [m][n]
  int64_t m;
  int32_t n, kblocks, wblocks, tiles;
  unsigned long long* err;
};

__global__ void __launch_bounds__(kThreads, 1)
    gemm_fp8_swapab_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                           Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* ctl = smem + kOffCtl;
  const uint32_t ctl_u = smem_u32(ctl);
  volatile int* abort = reinterpret_cast<volatile int*>(ctl + kAbort);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if ((smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0) hk_flag(p.err, hk::kErrWaitTimeout, 950);
    return;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(ctl_u + kBarFull + 8 * s, 1);
      mbar_init(ctl_u + kBarEmpty + 8 * s, 1);
    }
    for (int b = 0; b < kTBufs; ++b) {
      mbar_init(ctl_u + kBarTFull + 8 * b, 1);
      mbar_init(ctl_u + kBarTEmpty + 8 * b, 8);
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(ctl_u + kTmemSlot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(ctl + kTmemSlot);
  const int units = p.wblocks * p.tiles;

  if (warp == 0) {
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
        const int wb = u % p.wblocks, tile = u / p.wblocks;
        for (int kb = 0; kb < p.kblocks; ++kb) {
          const int s = g % kStages, fill = g / kStages;
          if (fill > 0 && !mbar_wait(ctl_u + kBarEmpty + 8 * s, (fill - 1) & 1, abort, p.err, 951)) {
            ok = false;
            break;
          }
          const uint32_t dst = smem_u32(smem + s * kStageBytes);
          const uint32_t full = ctl_u + kBarFull + 8 * s;
          mbar_expect_tx(full, kStageBytes);
          tma_load_2d(dst, &wmap, full, kb * kBK, wb * kWRows);
          tma_load_2d(dst + kWBytes, &xmap, full, kb * kBK, tile * kTok);
          ++g;
        }
      }
      // drain: the copies still in flight complete before the CTA exits
      for (int i = g > kStages ? g - kStages : 0; i < g; ++i) {
        const int s = i % kStages, fill = i / kStages;
        const unsigned long long t0 = globaltimer();
        while (!mbar_try_wait(ctl_u + kBarFull + 8 * s, fill & 1) && globaltimer() - t0 < kDrainNs) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
        for (int kb = 0; kb < p.kblocks; ++kb) {
          const int s = g % kStages, fill = g / kStages, buf = g % kTBufs, use = g / kTBufs;
          if (!mbar_wait(ctl_u + kBarFull + 8 * s, fill & 1, abort, p.err, 952) ||
              (use > 0 && !mbar_wait(ctl_u + kBarTEmpty + 8 * buf, (use - 1) & 1, abort, p.err, 953))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(smem + s * kStageBytes);
          const uint32_t x = a + kWBytes;
          const uint32_t d = tmem + (uint32_t)(buf * kTok);
#pragma unroll
          for (int kk = 0; kk < kBK / 32; ++kk)
            umma_f8(d, sdesc_sw128(a + 32 * kk, 16, 1024), sdesc_sw128(x + 32 * kk, 16, 1024), kIdesc,
                    kk > 0 ? 1u : 0u);
          umma_commit(ctl_u + kBarEmpty + 8 * s);
          umma_commit(ctl_u + kBarTFull + 8 * buf);
          ++g;
        }
      }
      if (g > 0) {  // the last MMAs complete before the CTA exits
        const int last = g - 1;
        const unsigned long long t0 = globaltimer();
        while (!mbar_try_wait(ctl_u + kBarTFull + 8 * (last % kTBufs), (last / kTBufs) & 1) &&
               globaltimer() - t0 < kDrainNs) {
        }
      }
    }
  } else {
    const int q = warp & 3;            // TMEM lane quarter
    const int half = (warp - 2) >> 2;  // token columns [half * 32, half * 32 + 32)
    const int r = q * 32 + lane;       // weight row inside the unit's 128-row block
    int g = 0;
    bool live = true;
    for (int u = blockIdx.x; live && u < units; u += gridDim.x) {
      const int wb = u % p.wblocks, tile = u / p.wblocks;
      const int64_t t0 = (int64_t)tile * kTok + half * kCols;  // this warp's first token row
      float acc[kCols];
#pragma unroll
      for (int i = 0; i < kCols; ++i) acc[i] = 0.f;
      const float* swr = p.sw + (int64_t)wb * p.kblocks;
      for (int kb = 0; kb < p.kblocks; ++kb, ++g) {
        if (!live) continue;
        const int buf = g % kTBufs, use = g / kTBufs;
        bool ok = true;
        if (lane == 0) ok = mbar_wait(ctl_u + kBarTFull + 8 * buf, use & 1, abort, p.err, 954);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) {
          live = false;
          continue;
        }
        tc_fence_after();
        float v[kCols];
        tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * kTok + half * kCols), v);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(ctl_u + kBarTEmpty + 8 * buf);
        const float s_w = __ldg(swr + kb);
#pragma unroll
        for (int i = 0; i < kCols; ++i) {
          const int64_t t = t0 + i;
          const float s_x = t < p.m ? __ldg(p.sx + t * p.kblocks + kb) : 0.f;
          acc[i] = fmaf(v[i], s_x * s_w, acc[i]);
        }
      }
      const int64_t col = (int64_t)wb * kWRows + r;
      if (live && col < p.n) {
#pragma unroll
        for (int i = 0; i < kCols; ++i) {
          const int64_t t = t0 + i;
          if (t < p.m) p.y[t * p.n + col] = f32_to_bf16_bits(acc[i]);
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

namespace hk {

bool gemm_fp8_swapab_supported(int64_t m, int32_t n, int32_t k) {
  return m >= 1 && m < 128 && n >= kWRows && k >= kBK && k % kBK == 0 && (int64_t)n * k < (1ll << 40);
}

int gemm_fp8_swapab(const uint8_t* xq, const float* sx, const uint8_t* wq, const float* sw, int64_t m, int32_t n,
                    int32_t k, uint16_t* y, cudaStream_t stream) {
  HK_REQUIRE(gemm_fp8_swapab_supported(m, n, k), "gemm_fp8_swapab: m %lld n %d k %d", (long long)m, n, k);
  static bool attr = false;
  if (!attr) {
    HK_TRY_CUDA(cudaFuncSetAttribute(gemm_fp8_swapab_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    attr = true;
  }
  CUtensorMap wmap, xmap;
  HK_TRY(sm100::make_map_u8(&wmap, wq, (uint64_t)n, (uint64_t)k, kWRows));
  HK_TRY(sm100::make_map_u8(&xmap, xq, (uint64_t)m, (uint64_t)k, kTok));
  Params p{};
  p.sx = sx;
  p.sw = sw;
  p.y = y;
  p.m = m;
  p.n = n;
  p.kblocks = k / kBK;
  p.wblocks = (n + kWRows - 1) / kWRows;
  p.tiles = (int32_t)((m + kTok - 1) / kTok);
  p.err = err_word();
  const int units = p.wblocks * p.tiles;
  const int grid = units < sm_count() ? units : sm_count();
  gemm_fp8_swapab_kernel<<<grid, kThreads, kSmem, stream>>>(wmap, xmap, p);
  HK_TRY_LAUNCH("gemm_fp8_swapab_kernel");
  return HK_OK;
}

}  // namespace hk
