// a11 on the tensor cores: y[m][n] bf16 = sum_kb (xq . wq^T)_kb * sx[m][kb] * sw[n/128][kb],
// e4m3 operands, fp32 block scales (activations 1x128, weights 128x128), fp32 accumulation.
//
// m >= 256 runs the pair form further down (two SMs, tcgen05 cta_group::2, 256 x 256 tiles).
// 128 <= m < 256: persistent kernel, one CTA per SM, tile 128 tokens x 256 weight rows:
//   warp 0      TMA producer: per 128-wide K block, the X tile (128 x 128 B) and the W tile
//               (256 x 128 B), 128-byte swizzled, into a 4-stage ring (48 KB a stage);
//   warp 1      MMA issuer: four tcgen05.mma kind::f8f6f4 (K = 32 each) per K block into a
//               fresh fp32 accumulator in TMEM, double-buffered (2 x 256 columns);
//   warps 2..9  scale promotion: each thread owns one row and 128 columns, which lie in one
//               128-row weight scale block, so a K block's partial sums take one scalar
//               sx[row][kb] * sw[group][kb]; acc += partial * scale in registers, then the
//               TMEM buffer goes back to the MMA warp.  After the last K block, bf16 stores.
// Registers: 10 warps put 3 warps on some SM sub-partitions, so a thread has at most 168; the
// promotion loop reads TMEM 16 columns at a time to keep its 128 accumulators in registers.
// Every wait is bounded (1 s); on a timeout the kernel records the error word, lets the
// copies and MMAs in flight finish, frees TMEM and returns.
#include <cuda.h>

#include "common.cuh"
#include "gemm_fp8.cuh"
#include "sm100.cuh"

namespace hk {
namespace sm100 {

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

int make_map_u8(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  EncodeTiledFn f = encode_tiled();
  if (f == nullptr) return fail(HK_ECUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols};
  cuuint32_t box[2] = {128, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = f(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(HK_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return HK_OK;
}

// 2-D bf16 map of y [rows][cols] for TMA stores: boxes of 32 rows x 64 columns (128 bytes),
// 128-byte swizzle; elements outside the tensor are not written.
static int make_map_y(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols) {
  EncodeTiledFn f = encode_tiled();
  if (f == nullptr) return fail(HK_ECUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(cols * 2)};
  cuuint32_t box[2] = {64, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = f(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(HK_ECUDA, "cuTensorMapEncodeTiled (y) failed (%d)", (int)r);
  return HK_OK;
}

}  // namespace sm100
}  // namespace hk

namespace {

using namespace hk::sm100;

// Tile width (weight rows) and the TMEM columns read per wait in the promotion loop.
#ifndef HK_GEMM_BN
#define HK_GEMM_BN 256
#endif
#ifndef HK_GEMM_LDC
#define HK_GEMM_LDC 16
#endif
constexpr int kBM = 128, kBN = HK_GEMM_BN, kBK = 128;
constexpr int kLdCols = HK_GEMM_LDC;
constexpr int kEpiWarps = 4 * (kBN / 128);          // one warp per lane quarter and 128 columns
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr int kABytes = kBM * kBK;                  // 16 KB
constexpr int kBBytes = kBN * kBK;                  // 16 or 32 KB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kStages = 196608 / kStageBytes < 8 ? 196608 / kStageBytes : 8;
constexpr int kOffCtl = kStages * kStageBytes;
constexpr int kSmemBytes = kOffCtl + 1024;
constexpr int kTBufs = 512 / kBN;                    // TMEM accumulators (all 512 columns)
constexpr uint32_t kTmemCols = kTBufs * kBN;
static_assert(kBN == 128 || kBN == 256, "tile width");
static_assert(kLdCols == 16 || kLdCols == 32 || kLdCols == 64, "TMEM load width");
static_assert(kSmemBytes <= 232448, "shared memory budget");

constexpr int kBarFull = 0;     // [kStages] TMA bytes of a stage landed
constexpr int kBarEmpty = 64;   // [kStages] the stage's MMAs completed
constexpr int kBarTFull = 128;  // [kTBufs] a TMEM accumulator holds a finished K block
constexpr int kBarTEmpty = 160; // [kTBufs] every promotion warp has read it
constexpr int kTmemSlot = 192;
constexpr int kAbort = 196;
constexpr uint32_t kIdesc = idesc_e4m3(kBM, kBN);
constexpr unsigned long long kDrainNs = 1000000000ull;

struct Params {
  int64_t m;
  int32_t n, k;
  int32_t tiles_m, tiles_n;
  const float* sx;
  const float* sw;
  uint16_t* y;
  unsigned long long* err;
};

__global__ void __launch_bounds__(kThreads, 1)
    gemm_fp8_sm100_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
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
      mbar_init(ctl_u + kBarTEmpty + 8 * b, kEpiWarps);
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(ctl_u + kTmemSlot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(ctl + kTmemSlot);
  const int kblocks = p.k / kBK;
  const int tiles = p.tiles_m * p.tiles_n;

  if (warp == 0) {
    if (lane == 0) {
      int g = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
        const int tm = t % p.tiles_m, tn = t / p.tiles_m;
        for (int kb = 0; kb < kblocks; ++kb) {
          const int s = g % kStages, fill = g / kStages;
          if (fill > 0 && !mbar_wait(ctl_u + kBarEmpty + 8 * s, (fill - 1) & 1, abort, p.err, 951)) {
            ok = false;
            break;
          }
          const uint32_t dst = smem_u32(smem + s * kStageBytes);
          mbar_expect_tx(ctl_u + kBarFull + 8 * s, kStageBytes);
          tma_load_2d(dst, &xmap, ctl_u + kBarFull + 8 * s, kb * kBK, tm * kBM);
          tma_load_2d(dst + kABytes, &wmap, ctl_u + kBarFull + 8 * s, kb * kBK, tn * kBN);
          ++g;
        }
      }
      // Let the last fill of every stage land before the CTA can exit.
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
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
        for (int kb = 0; kb < kblocks; ++kb) {
          const int s = g % kStages, fill = g / kStages, buf = g % kTBufs, use = g / kTBufs;
          if (!mbar_wait(ctl_u + kBarFull + 8 * s, fill & 1, abort, p.err, 952) ||
              (use > 0 && !mbar_wait(ctl_u + kBarTEmpty + 8 * buf, (use - 1) & 1, abort, p.err, 953))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(smem + s * kStageBytes), b = a + kABytes;
          const uint32_t d = tmem + (uint32_t)(buf * kBN);
#pragma unroll
          for (int kk = 0; kk < kBK / 32; ++kk)
            umma_f8(d, sdesc_sw128(a + 32 * kk, 16, 1024), sdesc_sw128(b + 32 * kk, 16, 1024), kIdesc,
                    kk > 0 ? 1u : 0u);
          umma_commit(ctl_u + kBarEmpty + 8 * s);
          umma_commit(ctl_u + kBarTFull + 8 * buf);
          ++g;
        }
      }
      // MMAs complete in order: the last commit landing means none is in flight.
      if (g > 0) {
        const int last = g - 1;
        const unsigned long long t0 = globaltimer();
        while (!mbar_try_wait(ctl_u + kBarTFull + 8 * (last % kTBufs), (last / kTBufs) & 1) &&
               globaltimer() - t0 < kDrainNs) {
        }
      }
    }
  } else {
    const int q = warp & 3;              // the TMEM lane quarter this warp may read
    const int half = (warp - 2) >> 2;    // columns 0..127 or 128..255 of the tile
    const int row = q * 32 + lane;
    const int groups = (p.n + 127) / 128;
    int g = 0;
    bool live = true;
    for (int t = blockIdx.x; live && t < tiles; t += gridDim.x) {
      const int tm = t % p.tiles_m, tn = t / p.tiles_m;
      const int64_t r = (int64_t)tm * kBM + row;
      const int grp = tn * (kBN / 128) + half;
      const bool use = r < p.m && grp < groups;
      const float* sxr = p.sx + (use ? r * kblocks : 0);
      const float* swr = p.sw + (use ? (int64_t)grp * kblocks : 0);
      float acc[128];
#pragma unroll
      for (int i = 0; i < 128; ++i) acc[i] = 0.f;
      float sc_next = use ? sxr[0] * swr[0] : 0.f;
      for (int kb = 0; kb < kblocks; ++kb) {
        const int buf = g % kTBufs, u = g / kTBufs;
        const float sc = sc_next;
        if (use && kb + 1 < kblocks) sc_next = sxr[kb + 1] * swr[kb + 1];
        bool ok = true;
        if (lane == 0) ok = mbar_wait(ctl_u + kBarTFull + 8 * buf, u & 1, abort, p.err, 954);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) {
          live = false;
          break;
        }
        tc_fence_after();
        const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * kBN + half * 128);
#pragma unroll
        for (int c = 0; c < 128 / kLdCols; ++c) {
          float v[kLdCols];
          if constexpr (kLdCols == 16) tmem_ld16(base + 16 * c, v);
          if constexpr (kLdCols == 32) tmem_ld32(base + 32 * c, v);
          if constexpr (kLdCols == 64) tmem_ld64(base + 64 * c, v);
#pragma unroll
          for (int i = 0; i < kLdCols; ++i) acc[kLdCols * c + i] = fmaf(v[i], sc, acc[kLdCols * c + i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(ctl_u + kBarTEmpty + 8 * buf);
        ++g;
      }
      if (!live) break;
      if (r < p.m) {
        const int col0 = tn * kBN + half * 128;
        uint16_t* yr = p.y + r * p.n;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const int col = col0 + 8 * c;
          if (col + 8 <= p.n) {
            uint32_t w[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
              w[i] = (uint32_t)f32_to_bf16_bits(acc[8 * c + 2 * i]) |
                     ((uint32_t)f32_to_bf16_bits(acc[8 * c + 2 * i + 1]) << 16);
            *reinterpret_cast<uint4*>(yr + col) = make_uint4(w[0], w[1], w[2], w[3]);
          }
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

// ---------------------------------------------------------------------------------------
// Pair form (m >= 256): a cluster of two SMs, tcgen05 cta_group::2, tile 256 tokens x 256
// weight rows.  Each SM brings its 128 token rows of X and its 128 weight rows of W per K
// block (32 KB) — against 48 KB for the 128 x 256 tile of one SM with the same MMA work per
// SM — because the pair's MMA reads the partner's half of W from the partner's shared memory
// instead of through L2.  The kernel is bound by the rate TMA fills shared memory from L2, so
// a third less fill per MAC is a third less time.
//   warp 0 (both SMs)  TMA producer: its X and W boxes to its own stage, completing on the
//                      leader's full barrier (the leader alone expects the pair's bytes);
//   warp 1 (leader)    MMA issuer: four M=256 N=256 K=32 MMAs per K block into one of two
//                      TMEM accumulators; commits arrive on both SMs' barriers;
//   warps 2..9         scale promotion of the SM's 128 rows, as in the one-SM kernel; the
//                      accumulator is released by arrives on the leader's barrier.
// ---------------------------------------------------------------------------------------
constexpr int kPM = 256, kPN = 256;                  // pair tile; 128 x 128 boxes per SM
constexpr int kPHalfBytes = 128 * kBK;               // 16 KB
constexpr int kPStageBytes = 2 * kPHalfBytes;        // X box + W box
constexpr int kPStages = 5;
#ifndef HK_GEMM_PAIR_WARPS
#define HK_GEMM_PAIR_WARPS 8
#endif
constexpr int kPEpiWarps = HK_GEMM_PAIR_WARPS;       // promotion warps: 4 per TMEM lane quarter
constexpr int kPCols = 4 * kPN / kPEpiWarps;         // columns of the tile per promotion warp
constexpr int kPThreads = 64 + 32 * kPEpiWarps;
constexpr int kPEpiBytes = 32 * kPCols * 2;          // a warp's 32 rows x kPCols bf16 columns
static_assert(kPEpiWarps == 8 || kPEpiWarps == 16, "promotion warps");
constexpr int kPOffEpi = kPStages * kPStageBytes;
constexpr int kPOffCtl = kPOffEpi + kPEpiWarps * kPEpiBytes;
constexpr int kPSmemBytes = kPOffCtl + 1024;
constexpr uint32_t kPIdesc = idesc_e4m3(kPM, kPN);
constexpr unsigned long long kPTeardownNs = 2000000ull;
static_assert(kPSmemBytes <= 232448, "shared memory budget");
static_assert(kPStages <= 8, "barrier slots");

__device__ __forceinline__ uint32_t pair_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t pair_mapa(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void pair_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on the leader's barrier at the same offset (CTA-scope release; the tcgen05 fences
// the callers issue order the tensor-memory reads it publishes).
__device__ __forceinline__ void pair_arrive_leader(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(pair_mapa(bar, 0)) : "memory");
}
__device__ __forceinline__ void pair_tma_load(uint32_t dst, const CUtensorMap* map, uint32_t bar_leader, int x,
                                              int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"((uint64_t)map), "r"(bar_leader), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void pair_umma_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// Arrives once on `bar` (same offset) in both SMs when the leader's prior MMAs complete.
__device__ __forceinline__ void pair_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(bar),
      "h"((uint16_t)3)
      : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"((uint64_t)map),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__global__ void __launch_bounds__(kPThreads, 1)
    gemm_fp8_pair_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap,
                         const __grid_constant__ CUtensorMap ymap, Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint8_t* ctl = smem + kPOffCtl;
  const uint32_t ctl_u = smem_u32(ctl);
  volatile int* abort = reinterpret_cast<volatile int*>(ctl + kAbort);
  const uint32_t rank = pair_rank();
  const int pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Both SMs of a pair see the same alignment (same kernel, same layout): they leave together.
  if ((smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0) hk_flag(p.err, hk::kErrWaitTimeout, 960);
    return;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPStages; ++s) {
      mbar_init(ctl_u + kBarFull + 8 * s, 1);
      mbar_init(ctl_u + kBarEmpty + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(ctl_u + kBarTFull + 8 * b, 1);
      mbar_init(ctl_u + kBarTEmpty + 8 * b, 2 * kPEpiWarps);
    }
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(ctl_u + kTmemSlot),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  pair_sync();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(ctl + kTmemSlot);
  const int kblocks = p.k / kBK;
  const int tiles = p.tiles_m * p.tiles_n;

  if (warp == 0) {
    if (lane == 0) {
      int g = 0;
      for (int t = pair; t < tiles; t += pairs) {
        const int tm = t % p.tiles_m, tn = t / p.tiles_m;
        bool ok = true;
        for (int kb = 0; kb < kblocks; ++kb) {
          const int s = g % kPStages, fill = g / kPStages;
          if (fill > 0 && !mbar_wait(ctl_u + kBarEmpty + 8 * s, (fill - 1) & 1, abort, p.err, 961)) {
            ok = false;
            break;
          }
          const uint32_t full = ctl_u + kBarFull + 8 * s;
          if (rank == 0) mbar_expect_tx(full, 2 * kPStageBytes);
          const uint32_t dst = smem_u32(smem + s * kPStageBytes);
          const uint32_t lead = pair_mapa(full, 0);
          pair_tma_load(dst, &xmap, lead, kb * kBK, tm * kPM + 128 * (int)rank);
          pair_tma_load(dst + kPHalfBytes, &wmap, lead, kb * kBK, tn * kPN + 128 * (int)rank);
          ++g;
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (rank == 0 && lane == 0) {
      int g = 0;
      bool ok = true;
      for (int t = pair; ok && t < tiles; t += pairs) {
        for (int kb = 0; kb < kblocks; ++kb) {
          const int s = g % kPStages, fill = g / kPStages, buf = g & 1, use = g >> 1;
          if (!mbar_wait(ctl_u + kBarFull + 8 * s, fill & 1, abort, p.err, 962) ||
              (use > 0 && !mbar_wait(ctl_u + kBarTEmpty + 8 * buf, (use - 1) & 1, abort, p.err, 963))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(smem + s * kPStageBytes), b = a + kPHalfBytes;
          const uint32_t d = tmem + (uint32_t)(buf * kPN);
#pragma unroll
          for (int kk = 0; kk < kBK / 32; ++kk)
            pair_umma_f8(d, sdesc_sw128(a + 32 * kk, 16, 1024), sdesc_sw128(b + 32 * kk, 16, 1024), kPIdesc,
                         kk > 0 ? 1u : 0u);
          pair_commit(ctl_u + kBarEmpty + 8 * s);
          pair_commit(ctl_u + kBarTFull + 8 * buf);
          ++g;
        }
      }
    }
  } else {
    const int q = warp & 3;              // the TMEM lane quarter this warp may read
    const int part = (warp - 2) >> 2;    // columns part * kPCols .. + kPCols of the tile
    const int row = (int)rank * 128 + q * 32 + lane;
    const int groups = (p.n + 127) / 128;
    int g = 0;
    bool live = true;
    for (int t = pair; live && t < tiles; t += pairs) {
      const int tm = t % p.tiles_m, tn = t / p.tiles_m;
      const int64_t r = (int64_t)tm * kPM + row;
      const int grp = (tn * kPN + part * kPCols) / 128;
      const bool use = r < p.m && grp < groups;
      const float* sxr = p.sx + (use ? r * kblocks : 0);
      const float* swr = p.sw + (use ? (int64_t)grp * kblocks : 0);
      float acc[kPCols];
#pragma unroll
      for (int i = 0; i < kPCols; ++i) acc[i] = 0.f;
      float sc_next = use ? sxr[0] * swr[0] : 0.f;
      for (int kb = 0; kb < kblocks; ++kb) {
        const int buf = g & 1, u = g >> 1;
        const float sc = sc_next;
        if (use && kb + 1 < kblocks) sc_next = sxr[kb + 1] * swr[kb + 1];
        bool ok = true;
        if (lane == 0) ok = mbar_wait(ctl_u + kBarTFull + 8 * buf, u & 1, abort, p.err, 964);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) {
          live = false;
          break;
        }
        tc_fence_after();
        const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * kPN + part * kPCols);
#pragma unroll
        for (int c = 0; c < kPCols / 16; ++c) {
          float v[16];
          tmem_ld16(base + 16 * c, v);
#pragma unroll
          for (int i = 0; i < 16; ++i) acc[16 * c + i] = fmaf(v[i], sc, acc[16 * c + i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) pair_arrive_leader(ctl_u + kBarTEmpty + 8 * buf);
        ++g;
      }
      if (!live) break;
      // The warp's 32 rows x kPCols columns go through its own shared memory (32 x 64 boxes,
      // 128-byte swizzle: a row's 16-byte chunk c sits at c ^ (row & 7), so the stores of 8
      // consecutive rows cover all banks) and out with TMA stores, which the warp does not wait
      // for; the buffer is reused once those stores have read it, a tile later.
      {
        const uint32_t eb = smem_u32(smem + kPOffEpi + (warp - 2) * kPEpiBytes);
        if (lane == 0) bulk_wait_read();
        __syncwarp();
#pragma unroll
        for (int c = 0; c < kPCols / 8; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            w[i] = (uint32_t)f32_to_bf16_bits(acc[8 * c + 2 * i]) |
                   ((uint32_t)f32_to_bf16_bits(acc[8 * c + 2 * i + 1]) << 16);
          const uint32_t addr = eb + (uint32_t)((c >> 3) * 4096 + lane * 128 + (((c & 7) ^ (lane & 7)) << 4));
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(w[0]), "r"(w[1]), "r"(w[2]),
                       "r"(w[3])
                       : "memory");
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          const int64_t row0 = (int64_t)tm * kPM + (int)rank * 128 + q * 32;
          const int col0 = tn * kPN + part * kPCols;
          if (row0 < p.m)
            for (int bx = 0; bx < kPCols / 64; ++bx)
              if (col0 + 64 * bx < p.n) tma_store_2d(&ymap, eb + 4096 * bx, col0 + 64 * bx, (int)row0);
          bulk_commit();
        }
      }
    }
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }
  // Teardown: on a timed-out pair, give copies and MMAs in flight time to land before shared
  // and tensor memory go away (on success every copy was consumed and every MMA observed).
  __syncwarp();
  if (*abort) {
    const unsigned long long t0 = globaltimer();
    while (globaltimer() - t0 < kPTeardownNs) {
    }
  }
  tc_fence_before();
  pair_sync();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512) : "memory");
  }
}

}  // namespace

namespace hk {

bool gemm_fp8_sm100_supported(int64_t m, int32_t n, int32_t k) {
  return m >= kBM && m < (1ll << 31) && n >= kBN && n % 16 == 0 && k % kBK == 0 && k >= kBK;
}

// m >= 256: the pair kernel, one cluster of two CTAs per two SMs.
static int gemm_fp8_pair(const uint8_t* xq, const float* sx, const uint8_t* wq, const float* sw, int64_t m,
                         int32_t n, int32_t k, uint16_t* y, cudaStream_t stream) {
  CUtensorMap xmap, wmap;
  HK_TRY(sm100::make_map_u8(&xmap, xq, (uint64_t)m, (uint64_t)k, 128));
  HK_TRY(sm100::make_map_u8(&wmap, wq, (uint64_t)n, (uint64_t)k, 128));
  CUtensorMap ymap;
  HK_TRY(sm100::make_map_y(&ymap, y, (uint64_t)m, (uint64_t)n));
  static bool attr = false;
  if (!attr) {
    HK_TRY_CUDA(cudaFuncSetAttribute(gemm_fp8_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kPSmemBytes));
    attr = true;
  }
  Params p;
  p.m = m;
  p.n = n;
  p.k = k;
  p.tiles_m = (int32_t)((m + kPM - 1) / kPM);
  p.tiles_n = (n + kPN - 1) / kPN;
  p.sx = sx;
  p.sw = sw;
  p.y = y;
  p.err = err_word();
  const int64_t tiles = (int64_t)p.tiles_m * p.tiles_n;
  HK_REQUIRE(tiles < (1ll << 30), "gemm_fp8_sm100: too many tiles");
  const int pairs = (int)std::min<int64_t>(tiles, sm_count() / 2);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * pairs));
  cfg.blockDim = dim3(kPThreads);
  cfg.dynamicSmemBytes = kPSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr2[1];
  attr2[0].id = cudaLaunchAttributeClusterDimension;
  attr2[0].val.clusterDim.x = 2;
  attr2[0].val.clusterDim.y = 1;
  attr2[0].val.clusterDim.z = 1;
  cfg.attrs = attr2;
  cfg.numAttrs = 1;
  HK_TRY_CUDA(cudaLaunchKernelEx(&cfg, gemm_fp8_pair_kernel, xmap, wmap, ymap, p));
  note_launch();
  return HK_OK;
}

int gemm_fp8_sm100(const uint8_t* xq, const float* sx, const uint8_t* wq, const float* sw, int64_t m,
                   int32_t n, int32_t k, uint16_t* y, cudaStream_t stream) {
  HK_REQUIRE(gemm_fp8_sm100_supported(m, n, k), "gemm_fp8_sm100: shape m %lld n %d k %d", (long long)m, n, k);
  HK_REQUIRE((uintptr_t)y % 16 == 0, "gemm_fp8_sm100: y must be 16-byte aligned");
  if (m >= kPM && sm_count() >= 2) return gemm_fp8_pair(xq, sx, wq, sw, m, n, k, y, stream);
  CUtensorMap xmap, wmap;
  HK_TRY(sm100::make_map_u8(&xmap, xq, (uint64_t)m, (uint64_t)k, kBM));
  HK_TRY(sm100::make_map_u8(&wmap, wq, (uint64_t)n, (uint64_t)k, kBN));
  static bool attr = false;
  if (!attr) {
    HK_TRY_CUDA(cudaFuncSetAttribute(gemm_fp8_sm100_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     kSmemBytes));
    attr = true;
  }
  Params p;
  p.m = m;
  p.n = n;
  p.k = k;
  p.tiles_m = (int32_t)((m + kBM - 1) / kBM);
  p.tiles_n = (n + kBN - 1) / kBN;
  p.sx = sx;
  p.sw = sw;
  p.y = y;
  p.err = err_word();
  const int64_t tiles = (int64_t)p.tiles_m * p.tiles_n;
  HK_REQUIRE(tiles < (1ll << 31), "gemm_fp8_sm100: too many tiles");
  const int grid = (int)std::min<int64_t>(tiles, sm_count());
  gemm_fp8_sm100_kernel<<<grid, kThreads, kSmemBytes, stream>>>(xmap, wmap, p);
  HK_TRY_LAUNCH("gemm_fp8_sm100_kernel");
  return HK_OK;
}

}  // namespace hk
