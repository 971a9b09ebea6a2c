// a11 for decode-sized batches: the FP8 block-scaled GEMM with fewer than 128 token rows, on the
// tensor cores in swap-AB form.
//
// A decode step's projections multiply a handful of token rows (one per live lane, or 1 + drafts)
// by a large weight matrix, so the weights are the operand that matters and the GEMM is
// HBM-bound on them (2 m flops per weight byte, far below the FP8 ridge).  The weights take the
// MMA's M side and a tile of up to 64 token rows the N side: per 128-wide K block,
// D[128 weight rows][64 tokens] = W[rows][kb] . X[tokens][kb]^T (tcgen05 kind::f8f6f4, M 128,
// N 64, four K-32 instructions) for two 128-row weight blocks side by side in one of four TMEM
// buffers.  Promotion warps add D * sw[row block][kb] * sx[token][kb] in fp32 registers, the
// DeepSeek-style scale rule of the one- and two-SM kernels, and write y[token][weight row] as
// bf16 at the end of the unit.
//
// Work unit = (64-row token tile, 256 weight rows = two scale-block rows), so each weight byte
// is read once per token tile (once in all for m <= 64), and the token tile (8 KB) is re-read once
// per 32 KB of weights.  Small-n, long-K shapes (the o projection: 7168 x 65536 has 28 units)
// would leave most SMs idle, so their K range is split into up to 4 parts: each work item writes
// its fp32 partial to a stream-ordered scratch (from a memory pool of this library's own, on the
// call's stream), and a second kernel adds the parts in a fixed order and writes y
// (deterministic).
//
// Roles per CTA (10 warps): warp 0 TMA producer, warp 1 TMEM owner and MMA issuer, warps 2..9
// promotion (two per TMEM lane quarter, 32 token columns each; thread = one row of each weight
// block).  The activation scales of the tile are staged in shared memory 64 K blocks at a time
// by the promotion warps.  Persistent over the units; every wait is bounded (1 s) and records
// the error word; copies and MMAs in flight are drained before exit.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "gemm_fp8.cuh"
#include "sm100.cuh"

namespace {

using namespace hk::sm100;

constexpr int kTok = 64;     // token rows per unit: the MMA's N
constexpr int kWRows = 128;  // rows of one weight block: the MMA's M
constexpr int kBK = 128;
constexpr int kThreads = 320;
constexpr int kPromo = 256;  // promotion threads (warps 2..9)
constexpr int kCols = 32;    // token columns per promotion warp
constexpr int kWBytes = kWRows * kBK;  // 16 KB
constexpr int kXBytes = kTok * kBK;    // 8 KB
constexpr int kStageBytes = 2 * kWBytes + kXBytes;  // 40 KB
constexpr int kStages = 5;
constexpr int kTBufs = 4;
constexpr uint32_t kTmemCols = kTBufs * 2 * kTok;  // 512
constexpr uint32_t kIdesc = idesc_e4m3(kWRows, kTok);
constexpr unsigned long long kDrainNs = 1000000000ull;
constexpr int kChunk = 64;  // K blocks of activation scales staged at a time

constexpr int kOffScales = kStages * kStageBytes;  // [kTok][kChunk] floats
constexpr int kOffCtl = kOffScales + kTok * kChunk * 4;
constexpr int kBarFull = 0;      // [kStages]
constexpr int kBarEmpty = 64;    // [kStages]
constexpr int kBarTFull = 128;   // [kTBufs]
constexpr int kBarTEmpty = 160;  // [kTBufs]
constexpr int kTmemSlot = 208;
constexpr int kAbort = 212;
constexpr int kCtlBytes = 256;
constexpr int kSmem = kOffCtl + kCtlBytes;
static_assert(kSmem <= 232448, "shared memory budget");
static_assert(kStageBytes % 1024 == 0 && kWBytes % 1024 == 0 && kOffScales % 1024 == 0, "swizzle atoms aligned");

struct Params {
  const float* sx;  // [m][kblocks]
  const float* sw;  // [ceil(n/128)][kblocks]
  uint16_t* y;      // [m][n] (split == 1)
  float* part;      // [split][m][n] fp32 partials (split > 1)
  int64_t m;
  int32_t n, kblocks, wblocks, pairs, tiles, split;
  unsigned long long* err;
};

// Named barrier over the promotion threads that also ANDs a predicate across them.
__device__ __forceinline__ bool promo_and(bool v) {
  int out;
  asm volatile(
      "{\n.reg .pred p, q;\nsetp.ne.b32 p, %1, 0;\nbar.red.and.pred q, 1, 256, p;\nselp.s32 %0, 1, 0, q;\n}"
      : "=r"(out)
      : "r"((int)v)
      : "memory");
  return out != 0;
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_fp8_swapab_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                           Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* ctl = smem + kOffCtl;
  float* scales = reinterpret_cast<float*>(smem + kOffScales);  // [kTok][kChunk]
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
  // work item w = (unit w / split, K part w % split); unit = (pair of weight blocks, token tile)
  const int items = p.pairs * p.tiles * p.split;

  if (warp == 0) {
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int w = blockIdx.x; ok && w < items; w += gridDim.x) {
        const int u = w / p.split, ks = w % p.split;
        const int pr = u % p.pairs, tile = u / p.pairs;
        const int kb0 = (int)((int64_t)p.kblocks * ks / p.split), kb1 = (int)((int64_t)p.kblocks * (ks + 1) / p.split);
        for (int kb = kb0; kb < kb1; ++kb) {
          const int s = g % kStages, fill = g / kStages;
          if (fill > 0 && !mbar_wait(ctl_u + kBarEmpty + 8 * s, (fill - 1) & 1, abort, p.err, 951)) {
            ok = false;
            break;
          }
          const uint32_t dst = smem_u32(smem + s * kStageBytes);
          const uint32_t full = ctl_u + kBarFull + 8 * s;
          mbar_expect_tx(full, kStageBytes);
          tma_load_2d(dst, &wmap, full, kb * kBK, pr * 2 * kWRows);
          tma_load_2d(dst + kWBytes, &wmap, full, kb * kBK, pr * 2 * kWRows + kWRows);
          tma_load_2d(dst + 2 * kWBytes, &xmap, full, kb * kBK, tile * kTok);
          ++g;
        }
      }
      for (int i = g > kStages ? g - kStages : 0; i < g; ++i) {  // copies in flight complete first
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
      for (int w = blockIdx.x; ok && w < items; w += gridDim.x) {
        const int ks = w % p.split;
        const int kb0 = (int)((int64_t)p.kblocks * ks / p.split), kb1 = (int)((int64_t)p.kblocks * (ks + 1) / p.split);
        for (int kb = kb0; kb < kb1; ++kb) {
          const int s = g % kStages, fill = g / kStages, buf = g % kTBufs, use = g / kTBufs;
          if (!mbar_wait(ctl_u + kBarFull + 8 * s, fill & 1, abort, p.err, 952) ||
              (use > 0 && !mbar_wait(ctl_u + kBarTEmpty + 8 * buf, (use - 1) & 1, abort, p.err, 953))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(smem + s * kStageBytes);
          const uint32_t x = a + 2 * kWBytes;
          const uint32_t d = tmem + (uint32_t)(buf * 2 * kTok);
#pragma unroll
          for (int kk = 0; kk < kBK / 32; ++kk) {
            const uint64_t bdesc = sdesc_sw128(x + 32 * kk, 16, 1024);
            umma_f8(d, sdesc_sw128(a + 32 * kk, 16, 1024), bdesc, kIdesc, kk > 0 ? 1u : 0u);
            umma_f8(d + kTok, sdesc_sw128(a + kWBytes + 32 * kk, 16, 1024), bdesc, kIdesc, kk > 0 ? 1u : 0u);
          }
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
    const int r = q * 32 + lane;       // row inside each of the unit's two 128-row weight blocks
    const int et = threadIdx.x - 64;   // 0..255 among the promotion threads
    int g = 0;
    bool live = true;
    for (int w = blockIdx.x; live && w < items; w += gridDim.x) {
      const int u = w / p.split, ks = w % p.split;
      const int pr = u % p.pairs, tile = u / p.pairs;
      const int kb0 = (int)((int64_t)p.kblocks * ks / p.split), kb1 = (int)((int64_t)p.kblocks * (ks + 1) / p.split);
      const int64_t tok0 = (int64_t)tile * kTok;
      const bool second = 2 * pr + 1 < p.wblocks;
      const float* swa = p.sw + (int64_t)(2 * pr) * p.kblocks;
      const float* swb = second ? swa + p.kblocks : swa;
      float acc_a[kCols], acc_b[kCols];
#pragma unroll
      for (int i = 0; i < kCols; ++i) acc_a[i] = acc_b[i] = 0.f;
      for (int kb = kb0; kb < kb1; ++kb, ++g) {
        const int kl = (kb - kb0) % kChunk;
        if (kl == 0) {  // stage the next chunk of the tile's activation scales, [token][kb]
          if (!promo_and(live)) live = false;  // every promotion thread is past the previous chunk
          for (int i = et; i < kTok * kChunk; i += kPromo) {
            const int t = i / kChunk, c = i % kChunk;
            const int64_t tt = tok0 + t;
            const int kk = kb + c;
            scales[t * kChunk + c] = (tt < p.m && kk < kb1) ? __ldg(p.sx + tt * p.kblocks + kk) : 0.f;
          }
          asm volatile("bar.sync 1, 256;" ::: "memory");
        }
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
        const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * 2 * kTok + half * kCols);
        float va[kCols], vb[kCols];
        tmem_ld32x2(base, base + kTok, va, vb);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(ctl_u + kBarTEmpty + 8 * buf);
        const float sa = __ldg(swa + kb), sb = __ldg(swb + kb);
        const float* sc = scales + (half * kCols) * kChunk + kl;
#pragma unroll
        for (int i = 0; i < kCols; ++i) {
          const float sv = sc[i * kChunk];
          acc_a[i] = fmaf(va[i], sv * sa, acc_a[i]);
          acc_b[i] = fmaf(vb[i], sv * sb, acc_b[i]);
        }
      }
      if (!promo_and(live)) {  // the promotion threads leave together
        live = false;
        break;
      }
      const int64_t col_a = (int64_t)(2 * pr) * kWRows + r;
      const int64_t col_b = col_a + kWRows;
#pragma unroll
      for (int i = 0; i < kCols; ++i) {
        const int64_t t = tok0 + half * kCols + i;
        if (t >= p.m) continue;
        if (p.split == 1) {
          if (col_a < p.n) p.y[t * p.n + col_a] = f32_to_bf16_bits(acc_a[i]);
          if (second && col_b < p.n) p.y[t * p.n + col_b] = f32_to_bf16_bits(acc_b[i]);
        } else {
          float* pt = p.part + ((int64_t)ks * p.m + t) * p.n;
          if (col_a < p.n) pt[col_a] = acc_a[i];
          if (second && col_b < p.n) pt[col_b] = acc_b[i];
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

// y = bf16(sum over the split parts, in part order) of the fp32 partials.
__global__ void reduce_parts_kernel(const float* __restrict__ part, int32_t split, int64_t count,
                                    uint16_t* __restrict__ y) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x) {
    float v = 0.f;
    for (int s = 0; s < split; ++s) v += part[s * count + i];
    y[i] = f32_to_bf16_bits(v);
  }
}

// A memory pool of this library's own per device for the split-K scratch: stream-ordered
// allocations that stay mapped between calls (the default pool hands memory back at every
// synchronisation, which made each call re-map its scratch).
constexpr int kMaxDevices = 64;
cudaMemPool_t g_pool[kMaxDevices] = {};
std::mutex g_pool_mu;

int scratch_pool(cudaMemPool_t* out) {
  int dev = -1;
  HK_TRY_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return hk::fail(HK_ENODEV, "device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_pool_mu);
  if (g_pool[dev] == nullptr) {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t pool = nullptr;
    HK_TRY_CUDA(cudaMemPoolCreate(&pool, &props));
    uint64_t keep = UINT64_MAX;
    HK_TRY_CUDA(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep));
    g_pool[dev] = pool;
  }
  *out = g_pool[dev];
  return HK_OK;
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
  p.pairs = (p.wblocks + 1) / 2;
  p.tiles = (int32_t)((m + kTok - 1) / kTok);
  p.err = err_word();
  const int units = p.pairs * p.tiles, sms = sm_count();
  // split K when the units fill less than half the SMs and every part keeps >= 8 K blocks
  p.split = 1;
  while (p.split < 4 && units * p.split * 2 <= sms && p.kblocks >= 16 * p.split) p.split *= 2;
  const int items = units * p.split;
  const int grid = items < sms ? items : sms;
  if (p.split > 1) {
    const size_t bytes = sizeof(float) * (size_t)p.split * (size_t)m * (size_t)n;
    cudaMemPool_t pool = nullptr;
    HK_TRY(scratch_pool(&pool));
    HK_TRY_CUDA(cudaMallocFromPoolAsync(reinterpret_cast<void**>(&p.part), bytes, pool, stream));
    gemm_fp8_swapab_kernel<<<grid, kThreads, kSmem, stream>>>(wmap, xmap, p);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) {
      note_launch();
      const int64_t count = m * (int64_t)n;
      reduce_parts_kernel<<<(unsigned)std::min<int64_t>((count + 255) / 256, 4 * sms), 256, 0, stream>>>(
          p.part, p.split, count, y);
      e = cudaGetLastError();
      if (e == cudaSuccess) note_launch();
    }
    const cudaError_t f = cudaFreeAsync(p.part, stream);
    if (e != cudaSuccess) return cuda_fail(e, "gemm_fp8_swapab (split K)");
    if (f != cudaSuccess) return cuda_fail(f, "cudaFreeAsync");
    return HK_OK;
  }
  gemm_fp8_swapab_kernel<<<grid, kThreads, kSmem, stream>>>(wmap, xmap, p);
  HK_TRY_LAUNCH("gemm_fp8_swapab_kernel");
  return HK_OK;
}

}  // namespace hk
