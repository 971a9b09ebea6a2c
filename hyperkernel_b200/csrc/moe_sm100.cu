// a14 on the tensor cores: the grouped FP8 expert FFN in swap-AB form.
//
// Decode-sized MoE gives each expert a handful of rows (config 4: ~16 of 4096 permuted rows
// per expert), so the expert weights are the large operand and the kernel is HBM-bound on
// them.  Weights therefore take the MMA's M side (128 weight rows, one 128x128 scale block)
// and the expert's rows the N side (a row tile), and each work unit streams one 128-row block
// of one expert's weights exactly once per row tile.
//
// Four row-tile widths (N 16, 32, 64, 96), one per call: the device-built tile list cuts every
// expert's rows in the widest width whose threshold the experts' average rows reach (below 8
// rows: 16; 8-23: 32; 24-55: 64; 56 and up: 96), so most experts stream their weights once and
// the tile is no wider than they need.  A narrower tile leaves room for more weights in flight:
// six 34 or 36 KB stages (16 and 32 rows), five 40 KB stages (64), four 44 KB stages (96).
// The host launches every width the call's rows per expert can reach; a launched width that the
// list did not choose returns at once (a decode batch launches only the 16-row kernel).  The
// 96-row form's promotion threads hold 48 token columns each (gate and up: 96 fp32 sums, what
// the 168 registers of a 320-thread CTA's threads hold beside the rest).
//
//  gather   xp[p] = xq[perm_token[p]], sxp[p] = sx[perm_token[p]]: the routed rows laid out
//           contiguously in permuted order, so TMA can load a row tile (out-of-range
//           indices are recorded and give a zero row).
//  up       unit = (row tile, 128-column block nb of h): D_g = Wg[nb] . X^T and
//           D_u = Wu[nb] . X^T per 128-wide K block (tcgen05 kind::f8f6f4, M 128, N = tile width)
//           into multi-buffered TMEM; promotion warps add partial * sw * sx[row] in registers;
//           at the end h = silu(g) * u is requantised to e4m3 with one scale per (row, nb)
//           (amax over the block's 128 columns across the four warps).
//  down     unit = (row tile, 256-column block of y as two 128-row blocks of W2):
//           D = W2[block] . hq^T over inter, promoted with sw * hs[row], stored as bf16.
// Roles per CTA (10 warps): warp 0 TMA, warp 1 MMA and TMEM owner, warps 2..9 promotion (two
// per TMEM lane quarter, each with half of the tile's token columns; thread = weight row), so
// a K block costs each promotion warp one TMEM round trip.  Every output element is one
// weight row's dot product with one token row in the same K-block order whichever tile holds
// the row, so a row's result does not depend on the tile width.  Persistent over the units of
// the tile list; every wait bounded (1 s) with the error word, in-flight copies and MMAs
// drained before exit.
#include <cuda.h>
#include <math.h>

#include "common.cuh"
#include "moe.cuh"
#include "sm100.cuh"

namespace {

using namespace hk::sm100;

constexpr int kWRows = 128;     // weight rows per unit: the MMA's M
constexpr int kBK = 128;
constexpr int kThreads = 320;       // TMA, MMA, 8 promotion warps
constexpr int kWBytes = kWRows * kBK;      // 16 KB
constexpr unsigned long long kDrainNs = 1000000000ull;
// TMEM accumulator buffers of the forms up to 64 rows: the MMA runs this many K blocks ahead of
// the promotion warps, which covers their per-unit work (scale table at the start,
// requantisation or stores at the end).
#ifndef HK_MOE_TBUFS
#define HK_MOE_TBUFS 4
#endif
static_assert(HK_MOE_TBUFS == 2 || HK_MOE_TBUFS == 4, "TMEM buffers");


// Control block offsets (after the ring and the scale table).
constexpr int kBarFull = 0;      // [8]
constexpr int kBarEmpty = 64;    // [8]
constexpr int kBarTFull = 128;   // [kTBufs]
constexpr int kBarTEmpty = 160;  // [kTBufs]
constexpr int kTmemSlot = 192;
constexpr int kAbort = 196;
constexpr int kRed = 256;        // [4][kRows] floats: per-warp column amax (up epilogue)

// kRows: token rows per unit, the MMA's N (16, 32, 64 or 96).
template <bool kUp, int kRows>
struct Cfg {
  static_assert(kRows == 16 || kRows == 32 || kRows == 64 || kRows == 96, "row tile");
  static constexpr int kXBytes = kRows * kBK;                // 2 to 12 KB
  static constexpr int kStageBytes = 2 * kWBytes + kXBytes;  // two weight blocks, one row tile
  static constexpr int kMaxKb = kUp ? 64 : 32;  // scale-table capacity in K blocks
  static constexpr int kStages = kRows <= 32 ? 6 : kRows == 64 ? 5 : 4;
  static constexpr int kTBufs = kRows <= 64 ? HK_MOE_TBUFS : 2;  // 2 * kRows columns each
  static constexpr int kCols = kRows / 2;       // token columns per promotion warp
  static constexpr int kChunk = kRows == 64 ? 32 : kRows == 16 ? 8 : 16;  // columns per TMEM load
  static constexpr int kOffScales = kStages * kStageBytes;
  static constexpr int kOffCtl = kOffScales + kMaxKb * kRows * 4;
  static constexpr int kCtlBytes = kRed + 4 * kRows * 4;
  static constexpr int kSmem = kOffCtl + kCtlBytes;
  static constexpr uint32_t kTmemCols = 512;  // allocated (a power of two); kTBufs * 2 * kRows used
  static constexpr uint32_t kIdesc = idesc_e4m3(kWRows, kRows);
  static_assert(kTBufs * 2 * kRows <= 512 && kCols % kChunk == 0 && kRows % 16 == 0, "TMEM columns");
  static_assert(kStageBytes % 1024 == 0, "stage alignment (128-byte swizzle atoms)");
  static_assert(kSmem <= 232448, "shared memory budget");
};

struct Params {
  const int32_t* offsets;
  const int32_t* tile_expert;
  const int32_t* tile_row;
  const int32_t* num_tiles;
  int32_t hidden, inter, num_experts;
  int64_t rows;
  const float* act_scale;  // up: sxp [rows][hidden/128]; down: hs [rows][inter/128]
  const float* w_scale;    // up: s13; down: s2
  uint8_t* hq;             // up output
  float* hs;               // up output
  uint16_t* y;             // down output
  unsigned long long* err;
};

__global__ void gather_rows_kernel(const uint8_t* __restrict__ xq, const float* __restrict__ sx,
                                   const int32_t* __restrict__ perm_token, int64_t rows, int32_t tokens,
                                   int32_t hidden, uint8_t* __restrict__ xp, float* __restrict__ sxp,
                                   unsigned long long* err) {
  const int64_t p = blockIdx.x;
  if (p >= rows) return;
  const int32_t src = perm_token[p];
  const bool ok = src >= 0 && src < tokens;
  if (!ok && threadIdx.x == 0) hk_flag(err, hk::kErrMoeRow, (unsigned)p);
  const int vecs = hidden / 16;
  const uint4* s = reinterpret_cast<const uint4*>(xq + (int64_t)(ok ? src : 0) * hidden);
  uint4* d = reinterpret_cast<uint4*>(xp + p * hidden);
  for (int i = threadIdx.x; i < vecs; i += blockDim.x) d[i] = ok ? s[i] : make_uint4(0, 0, 0, 0);
  const int kb = hidden / 128;
  for (int i = threadIdx.x; i < kb; i += blockDim.x) sxp[p * kb + i] = ok ? sx[(int64_t)src * kb + i] : 0.f;
}

// Named barrier `id` over `count` threads that also ANDs a predicate across them.
__device__ __forceinline__ bool bar_and(int id, int count, bool v) {
  int out;
  asm volatile(
      "{\n.reg .pred p, q;\nsetp.ne.b32 p, %1, 0;\nbar.red.and.pred q, %2, %3, p;\nselp.s32 %0, 1, 0, q;\n}"
      : "=r"(out)
      : "r"((int)v), "r"(id), "r"(count)
      : "memory");
  return out != 0;
}

template <bool kUp, int kRows>
__global__ void __launch_bounds__(kThreads, 1)
    moe_sm100_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap, Params p) {
  using C = Cfg<kUp, kRows>;
  constexpr int kTBufs = C::kTBufs, kCols = C::kCols, kChunk = C::kChunk;
  // not the width the tile list chose (or no tiles): leave before any set-up
  if (p.num_tiles[0] == 0 || p.num_tiles[1] != kRows) return;
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* ctl = smem + C::kOffCtl;
  float* scales = reinterpret_cast<float*>(smem + C::kOffScales);  // [kb][64]
  const uint32_t ctl_u = smem_u32(ctl);
  volatile int* abort = reinterpret_cast<volatile int*>(ctl + kAbort);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if ((smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0) hk_flag(p.err, hk::kErrWaitTimeout, 960);
    return;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
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
  if (warp == 1) tmem_alloc(ctl_u + kTmemSlot, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(ctl + kTmemSlot);

  // up: K = hidden, units per tile = inter / 128; down: K = inter, units per tile = hidden / 128
  const int kblocks = (kUp ? p.hidden : p.inter) / kBK;
  // up: one unit per 128-column block of h (its gate and up row blocks); down: one unit per
  // pair of 128-row blocks of W2 (256 output columns; the second is empty past hidden).
  const int nblocks = kUp ? p.inter / 128 : (p.hidden / 128 + 1) / 2;
  const int units = p.num_tiles[0] * nblocks;

  if (warp == 0) {
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
        const int tile = u / nblocks, nb = u % nblocks;
        const int e = p.tile_expert[tile], r0 = p.tile_row[tile];
        // weight rows of this unit (gate block, and up block inter rows later)
        const int wrow = kUp ? e * 2 * p.inter + nb * 128 : e * p.hidden + nb * 256;
        for (int kb = 0; kb < kblocks; ++kb) {
          const int s = g % C::kStages, fill = g / C::kStages;
          if (fill > 0 && !mbar_wait(ctl_u + kBarEmpty + 8 * s, (fill - 1) & 1, abort, p.err, 961)) {
            ok = false;
            break;
          }
          const uint32_t dst = smem_u32(smem + s * C::kStageBytes);
          const uint32_t full = ctl_u + kBarFull + 8 * s;
          mbar_expect_tx(full, C::kStageBytes);
          tma_load_2d(dst, &wmap, full, kb * kBK, wrow);
          tma_load_2d(dst + kWBytes, &wmap, full, kb * kBK, wrow + (kUp ? p.inter : 128));
          tma_load_2d(dst + 2 * kWBytes, &xmap, full, kb * kBK, r0);
          ++g;
        }
      }
      for (int i = g > C::kStages ? g - C::kStages : 0; i < g; ++i) {
        const int s = i % C::kStages, fill = i / C::kStages;
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
        for (int kb = 0; kb < kblocks; ++kb) {
          const int s = g % C::kStages, fill = g / C::kStages, buf = g % kTBufs, use = g / kTBufs;
          if (!mbar_wait(ctl_u + kBarFull + 8 * s, fill & 1, abort, p.err, 962) ||
              (use > 0 && !mbar_wait(ctl_u + kBarTEmpty + 8 * buf, (use - 1) & 1, abort, p.err, 963))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(smem + s * C::kStageBytes);
          const uint32_t x = a + 2 * kWBytes;
          const uint32_t d = tmem + (uint32_t)(buf * 2 * kRows);
#pragma unroll
          for (int kk = 0; kk < kBK / 32; ++kk) {
            const uint64_t bdesc = sdesc_sw128(x + 32 * kk, 16, 1024);
            umma_f8(d, sdesc_sw128(a + 32 * kk, 16, 1024), bdesc, C::kIdesc, kk > 0 ? 1u : 0u);
            umma_f8(d + kRows, sdesc_sw128(a + kWBytes + 32 * kk, 16, 1024), bdesc, C::kIdesc, kk > 0 ? 1u : 0u);
          }
          umma_commit(ctl_u + kBarEmpty + 8 * s);
          umma_commit(ctl_u + kBarTFull + 8 * buf);
          ++g;
        }
      }
      if (g > 0) {
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
    const int m = q * 32 + lane;       // weight row inside the unit's 128-row block
    const int et = threadIdx.x - 64;   // 0..255 among the promotion threads
    float* red = reinterpret_cast<float*>(ctl + kRed);
    int g = 0;
    bool live = true;
    for (int u = blockIdx.x; live && u < units; u += gridDim.x) {
      const int tile = u / nblocks, nb = u % nblocks;
      const int e = p.tile_expert[tile], r0 = p.tile_row[tile];
      const int count = min(kRows, p.offsets[e + 1] - r0);
      // Per-row activation scales of the tile for every K block: scales[kb][n].
      asm volatile("bar.sync 1, 256;" ::: "memory");  // the previous unit is done reading them
      for (int i = et; i < kblocks * kRows; i += 256) {
        const int n = i % kRows, kb = i / kRows;
        scales[kb * kRows + n] = n < count ? p.act_scale[(int64_t)(r0 + n) * kblocks + kb] : 0.f;
      }
      asm volatile("bar.sync 1, 256;" ::: "memory");
      // Weight scales of the unit's two row blocks (g: gate or first block, u: up or second).
      const int hb = p.hidden / 128;
      const bool second = kUp || 2 * nb + 1 < hb;
      const float* wsc = kUp ? p.w_scale + ((int64_t)e * (2 * p.inter / 128) + nb) * kblocks
                             : p.w_scale + ((int64_t)e * hb + 2 * nb) * kblocks;
      const float* wsu = kUp ? wsc + (int64_t)(p.inter / 128) * kblocks : (second ? wsc + kblocks : wsc);
      float acc_g[kCols], acc_u[kCols];
#pragma unroll
      for (int i = 0; i < kCols; ++i) acc_g[i] = 0.f;
#pragma unroll
      for (int i = 0; i < kCols; ++i) acc_u[i] = 0.f;
      // A warp whose wait fails stops waiting but stays in step, so the promotion warps always
      // meet at the named barriers and leave the unit loop together.
      for (int kb = 0; kb < kblocks; ++kb, ++g) {
        if (!live) continue;
        const int buf = g % kTBufs, use = g / kTBufs;
        const float sg = wsc[kb];
        const float su = wsu[kb];
        bool ok = true;
        if (lane == 0) ok = mbar_wait(ctl_u + kBarTFull + 8 * buf, use & 1, abort, p.err, 964);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) {
          live = false;
          continue;
        }
        tc_fence_after();
        const uint32_t base =
            tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * 2 * kRows + half * kCols);
#pragma unroll
        for (int c = 0; c < kCols / kChunk; ++c) {
          float vg[kChunk], vu[kChunk];
          // both blocks' columns of this chunk, one wait
          if constexpr (kChunk == 32) {
            tmem_ld32x2(base + c * kChunk, base + kRows + c * kChunk, vg, vu);
          } else if constexpr (kChunk == 8) {
            tmem_ld8x2(base + c * kChunk, base + kRows + c * kChunk, vg, vu);
          } else {
            tmem_ld16x2(base + c * kChunk, base + kRows + c * kChunk, vg, vu);
          }
          const float4* sc4 = reinterpret_cast<const float4*>(scales + kb * kRows + half * kCols + c * kChunk);
#pragma unroll
          for (int j = 0; j < kChunk / 4; ++j) {
            const float4 s4 = sc4[j];
            const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int col = c * kChunk + 4 * j + i;
              acc_g[col] = fmaf(vg[4 * j + i], sv[i] * sg, acc_g[col]);
              acc_u[col] = fmaf(vu[4 * j + i], sv[i] * su, acc_u[col]);
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(ctl_u + kBarTEmpty + 8 * buf);
      }
      if (!bar_and(1, 256, live)) break;
      if constexpr (kUp) {
        // h = silu(g) * u, then one e4m3 scale per (row, nb) from the amax over this block's
        // 128 columns: the four warps of this column half, one per lane quarter.
#pragma unroll
        for (int i = 0; i < kCols; ++i) {
          const float gv = acc_g[i];
          acc_g[i] = gv / (1.f + expf(-gv)) * acc_u[i];
          float a = fabsf(acc_g[i]);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
          if (lane == 0) red[q * kRows + half * kCols + i] = a;
        }
        asm volatile("bar.sync 1, 256;" ::: "memory");
        const int inter_blocks = p.inter / 128;
#pragma unroll
        for (int i = 0; i < kCols; ++i) {
          const int n = half * kCols + i;
          if (n < count) {
            const float amax = fmaxf(fmaxf(red[n], red[kRows + n]), fmaxf(red[2 * kRows + n], red[3 * kRows + n]));
            const float s = __fdiv_rn(fmaxf(amax, 1e-12f), 448.0f);
            const int64_t row = r0 + n;
            p.hq[row * p.inter + nb * 128 + m] = f32_to_e4m3(__fdiv_rn(acc_g[i], s));
            if (m == 0) p.hs[row * inter_blocks + nb] = s;
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < kCols; ++i) {
          const int n = half * kCols + i;
          if (n < count) {
            uint16_t* yr = p.y + (int64_t)(r0 + n) * p.hidden + nb * 256 + m;
            yr[0] = f32_to_bf16_bits(acc_g[i]);
            if (second) yr[128] = f32_to_bf16_bits(acc_u[i]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

template <bool kUp, int kRows>
int launch(const CUtensorMap& wmap, const CUtensorMap& xmap, const Params& p, int grid, cudaStream_t s) {
  using C = Cfg<kUp, kRows>;
  static bool attr = false;
  if (!attr) {
    HK_TRY_CUDA(cudaFuncSetAttribute(moe_sm100_kernel<kUp, kRows>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     C::kSmem));
    attr = true;
  }
  moe_sm100_kernel<kUp, kRows><<<grid, kThreads, C::kSmem, s>>>(wmap, xmap, p);
  HK_TRY_LAUNCH(kUp ? "moe_sm100_kernel<up>" : "moe_sm100_kernel<down>");
  return HK_OK;
}

}  // namespace

namespace hk {

bool moe_sm100_supported(int32_t num_experts, int32_t hidden, int32_t inter) {
  return hidden % 128 == 0 && inter % 128 == 0 && hidden / 128 <= Cfg<true, 64>::kMaxKb &&
         inter / 128 <= Cfg<false, 64>::kMaxKb && (int64_t)num_experts * 2 * inter < (1ll << 31) &&
         (int64_t)num_experts * hidden < (1ll << 31);
}

int moe_sm100_run(const uint8_t* xq, const float* sx, int32_t tokens, const int32_t* offsets,
                  const int32_t* perm_token, int64_t rows, int32_t num_experts, int32_t hidden, int32_t inter,
                  const uint8_t* w13, const float* s13, const uint8_t* w2, const float* s2, uint16_t* y,
                  const MoeScratch& ws, int widths, unsigned long long* err, cudaStream_t s) {
  HK_REQUIRE(moe_sm100_supported(num_experts, hidden, inter), "moe_sm100: hidden %d inter %d", hidden, inter);
  HK_REQUIRE(rows < (1ll << 31), "moe_sm100: %lld rows", (long long)rows);
  gather_rows_kernel<<<(unsigned)rows, 128, 0, s>>>(xq, sx, perm_token, rows, tokens, hidden, ws.xp, ws.sxp, err);
  HK_TRY_LAUNCH("gather_rows_kernel");
  CUtensorMap w13map, w2map, xmap[4], hmap[4];
  HK_TRY(sm100::make_map_u8(&w13map, w13, (uint64_t)num_experts * 2 * inter, (uint64_t)hidden, kWRows));
  HK_TRY(sm100::make_map_u8(&w2map, w2, (uint64_t)num_experts * hidden, (uint64_t)inter, kWRows));
  for (int i = 0; i < 4; ++i) {
    if (!((widths >> i) & 1)) continue;
    HK_TRY(sm100::make_map_u8(&xmap[i], ws.xp, (uint64_t)rows, (uint64_t)hidden, moe_tile_width(i)));
    HK_TRY(sm100::make_map_u8(&hmap[i], ws.hq, (uint64_t)rows, (uint64_t)inter, moe_tile_width(i)));
  }
  Params p{};
  p.offsets = offsets;
  p.tile_expert = ws.tc_expert;
  p.tile_row = ws.tc_row;
  p.num_tiles = ws.tc_num;
  p.hidden = hidden;
  p.inter = inter;
  p.num_experts = num_experts;
  p.rows = rows;
  p.err = err;
  const int grid = sm_count();
  p.act_scale = ws.sxp;
  p.w_scale = s13;
  p.hq = ws.hq;
  p.hs = ws.hs;
  if (widths & 1) HK_TRY((launch<true, 16>(w13map, xmap[0], p, grid, s)));
  if (widths & 2) HK_TRY((launch<true, 32>(w13map, xmap[1], p, grid, s)));
  if (widths & 4) HK_TRY((launch<true, 64>(w13map, xmap[2], p, grid, s)));
  if (widths & 8) HK_TRY((launch<true, 96>(w13map, xmap[3], p, grid, s)));
  p.act_scale = ws.hs;
  p.w_scale = s2;
  p.y = y;
  if (widths & 1) HK_TRY((launch<false, 16>(w2map, hmap[0], p, grid, s)));
  if (widths & 2) HK_TRY((launch<false, 32>(w2map, hmap[1], p, grid, s)));
  if (widths & 4) HK_TRY((launch<false, 64>(w2map, hmap[2], p, grid, s)));
  if (widths & 8) HK_TRY((launch<false, 96>(w2map, hmap[3], p, grid, s)));
  return HK_OK;
}

}  // namespace hk
