// tcgen05 2-SM ragged paged MLA decode (128 heads, latent 512 + rope 64, bf16, pages of 64).
//
// Why two SMs: the output of one query row is 128 heads x 512 dims of fp32 = 256 KB, the
// whole tensor memory of one SM.  A CTA pair (cluster of 2, tcgen05 cta_group::2) splits the
// heads 64/64: each SM keeps its 64 heads x 512 dims of O (256 TMEM columns) plus two
// 256-token score buffers (2 x 128 columns), and the pair issues M=128 MMAs whose B operand
// (the KV tile) is split between the two SMs' shared memories.
//
// Per KV tile of 256 tokens (4 pages; CTA r holds pages 2r and 2r+1 for the scores):
//   S  = Q K^T   : 9 chunks x 4 MMAs M=128 N=256 K=16 (A = Q chunk, K-major; B = 128 KV rows)
//   P  = exp2(S*scale*log2e - m)  in 4 softmax warps per SM (lazy rescale of O when the
//                                  running max grows by more than 8 in log2 units)
//   O += P V     : 2 N-blocks x 4 pages x 4 MMAs M=128 N=256 K=16 (A = P, K-major; B = V,
//                  MN-major; CTA r supplies dims 256j + 128r .. +127 of every token)
// The cache is page-blocked (each page stores its rows' dims in nine 64-dim blocks), so each
// TMA box is one contiguous 8 KB block.  K chunks ([128 rows][64 dims]) and V chunks
// ([64 tokens][128 dims]) stream through one
// ring of five 16 KB entries in the exact order the MMA warp consumes them, so a chunk is
// refilled as soon as its four MMAs retire.  Shared memory per SM: Q 72 KB + P 32 KB + ring
// 7 x 16 KB = 216 KB.  HBM bytes are the KV rows once; the V half each SM needs from its
// partner's rows is read a second time through L2.
//
// Work split: the 256-token tiles of all query rows are laid end to end and cut into one
// contiguous range per cluster (plan kernel).  A row that spans several clusters is written
// as fp32 partials (normalised O and LSE) and merged by LSE afterwards (merge kernel).
//
// Roles (192 threads per CTA): warp 0 TMA producer, warp 1 TMEM allocator + MMA issuer
// (leader CTA only issues), warps 2-5 softmax / O rescale / epilogue.  Every mbarrier wait
// is bounded (1 s of globaltimer); a timeout sets the device error word and an abort flag,
// and all roles wind down to the common teardown.
#include <cuda.h>

#include <math.h>

#include "attn.cuh"
#include "common.cuh"
#include "mla_sm100.cuh"

namespace {

constexpr int kHeads = 128;
constexpr int kDK = 576, kDV = 512;
constexpr int kPage = 64;
constexpr int kTileTok = 256;            // tokens per tile = 4 pages
constexpr int kClusterCTAs = 2;
constexpr int kThreads = 192;

constexpr int kBox = 64 * 128;           // one TMA box: [64 rows][64 dims] bf16, 128B-swizzled
constexpr int kEntry = 2 * kBox;         // ring entry: two boxes
constexpr int kRing = 7;
constexpr int kPAtom = kBox;             // [64 heads][64 tokens]
constexpr int kPBuf = 4 * kPAtom;        // 256 tokens

constexpr int kOffQ = 0;                 // 9 boxes
constexpr int kOffP = kOffQ + 9 * kBox;
constexpr int kOffRing = kOffP + kPBuf;       // one P buffer: softmax(g) writes it after PV(g-1)
constexpr int kOffCtl = kOffRing + kRing * kEntry;
constexpr int kCtlBytes = 2048;
constexpr int kSmemBytes = kOffCtl + kCtlBytes;
static_assert(kSmemBytes <= 232448, "shared memory budget");

// Control block layout (byte offsets inside the control block).
constexpr int kBarFull = 0;      // [kRing] leader: both SMs' TMA bytes of a ring entry
constexpr int kBarEmpty = 64;    // [kRing] each SM: entry consumed (MMA commit, multicast)
constexpr int kBarQFull = 128;   // leader: both SMs' Q bytes
constexpr int kBarQEmpty = 136;  // each SM: Q no longer read (MMA commit)
constexpr int kBarSFull = 144;   // [2] each SM: S ready (MMA commit)
constexpr int kBarSFree = 160;   // [2] leader: S read by all 8 softmax warps
constexpr int kBarPFull = 176;   // [2] leader: P written by all 8 softmax warps
constexpr int kBarODone = 192;   // each SM: PV of a tile complete (MMA commit)
constexpr int kBarOFree = 200;   // leader: epilogue of a segment done reading O
constexpr int kTmemSlot = 208;
constexpr int kAbort = 212;
constexpr int kXchMax = 256;     // [2][128] floats (kXchL ends at 1792 < kCtlBytes)
constexpr int kXchL = kXchMax + 1024;  // [128] floats

constexpr int kTmemO = 0;        // 256 columns
constexpr int kTmemS = 256;      // 2 x 128 columns
constexpr unsigned long long kTimeoutNs = 1000000000ull;

// ---------------------------------------------------------------------------------------
// PTX helpers
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t mapa_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
               "r"(bytes)
               : "memory");
}
// Arrive on the barrier at the same offset in CTA 0 of the pair (local when rank 0).  The
// arrive keeps the default CTA-scope release: a cluster-scope release measured ≈1,300-1,900
// cycles per arrive here (it drains far more than the few shared-memory stores it orders),
// against ≈30-100 for this form.  What it orders for the MMA is covered by the proxy and
// tcgen05 fences the callers issue before it.
__device__ __forceinline__ void mbar_arrive_leader(uint32_t bar, uint32_t rank) {
  const uint32_t remote = mapa_rank(bar, 0);
  (void)rank;
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(remote) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\n"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: true when the phase of `parity` completed; false on abort / timeout.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort,
                                          unsigned long long* err, unsigned site) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (globaltimer() - t0 > kTimeoutNs) {
      *abort = 1;
      hk_flag(err, hk::kErrWaitTimeout, site);
      return false;
    }
  }
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map,
                                                 uint32_t bar_leader, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"((uint64_t)map), "r"(bar_leader), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void umma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// Arrives once on `bar` (same offset) in both SMs of the pair when all prior MMAs complete.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(bar),
      "h"((uint16_t)3)
      : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t addr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(addr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
// Two back-to-back 32-column loads with one wait (columns addr .. addr+63).
__device__ __forceinline__ void tmem_ld64(uint32_t addr, float* v) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,"
      "%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,"
      "%58,%59,%60,%61,%62,%63}, [%64];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]),
        "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]),
        "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]),
        "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]),
        "=r"(r[62]), "=r"(r[63])
      : "r"(addr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ void tmem_st32(uint32_t addr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
      "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(
          addr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

// UMMA shared-memory descriptor (sm_100 format): start >> 4, leading / stride byte offsets
// >> 4, version 1, 128-byte swizzle.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor, kind::f16: D fp32, A and B bf16, M=128 (pair), N, majors.
constexpr uint32_t idesc_bf16(int n, int b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)b_mn_major << 16) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}
constexpr uint32_t kIdescQK = idesc_bf16(256, 0);
constexpr uint32_t kIdescPV = idesc_bf16(256, 1);

__device__ __forceinline__ int lane_of_row(const int32_t* __restrict__ cu, int num_lanes, int t) {
  int lo = 0, hi = num_lanes;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (cu[mid] <= t) lo = mid; else hi = mid;
  }
  return lo;
}

struct Plan {
  int32_t* row_tile_start;  // [T+1] prefix of 256-token tiles per row
  int32_t* first_cluster;   // [T]
  int32_t* n_split;         // [T]
  int32_t* split_base;      // [T], -1 when the row is not split
  int32_t* meta;            // [0] total tiles, [1] tiles per cluster
};

struct Params {
  const int32_t* bt;
  int32_t bt_stride;
  const int32_t* cu;
  const int32_t* positions;
  const int32_t* kv_begin;  // optional KV range per lane (context-parallel partials)
  const int32_t* kv_end;
  int32_t num_lanes, num_tokens;
  int32_t num_pages;
  float scale_log2;
  uint16_t* out;            // bf16 output, or
  float* out_f32;           // fp32 output (partials), when not null
  float* lse;
  float* part_o;
  float* part_lse;
  Plan plan;
  unsigned long long* err;
};

// KV rows [lo, hi) that row t of lane b attends: its causal prefix [0, pos], cut to the
// lane's [kv_begin, kv_end) when a range is given.  hi <= lo: the row attends nothing.
__device__ __forceinline__ void row_span(const int32_t* __restrict__ positions,
                                         const int32_t* __restrict__ kv_begin,
                                         const int32_t* __restrict__ kv_end, int t, int b,
                                         int& lo, int& hi) {
  lo = 0;
  hi = positions[t] + 1;
  if (kv_begin != nullptr) {
    lo = max(0, kv_begin[b]);
    hi = min(hi, kv_end[b]);
  }
}

// ---------------------------------------------------------------------------------------
// plan: tiles per row, their prefix, the cluster cut, and which rows need partials.
// A row's tiles start at the page holding its first KV row.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ int block_scan_excl(int v, int* sums, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nw ? sums[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    sums[lane] = w;
  }
  __syncthreads();
  const int before = (warp > 0 ? sums[warp - 1] : 0) + x - v;
  *total = sums[nw - 1];
  __syncthreads();
  return before;
}

__global__ void __launch_bounds__(1024) mla_plan_kernel(const int32_t* __restrict__ positions,
                                                        const int32_t* __restrict__ cu,
                                                        int32_t num_lanes,
                                                        const int32_t* __restrict__ kv_begin,
                                                        const int32_t* __restrict__ kv_end,
                                                        int32_t T, int32_t clusters, Plan plan,
                                                        unsigned long long* err) {
  __shared__ int sums[32];
  __shared__ int s_tpc;
  int carry = 0;
  for (int base = 0; base < T; base += blockDim.x) {
    const int t = base + threadIdx.x;
    int tiles = 0;
    if (t < T) {
      const int pos = positions[t];
      if (pos < 0) hk_flag(err, hk::kErrAttnPage, (unsigned)t);
      int lo, hi;
      row_span(positions, kv_begin, kv_end, t, lane_of_row(cu, num_lanes, t), lo, hi);
      const int base = lo - lo % kPage;
      tiles = (pos >= 0 && hi > lo) ? (hi - base + kTileTok - 1) / kTileTok : 0;
    }
    int total;
    const int ex = block_scan_excl(tiles, sums, &total);
    if (t < T) plan.row_tile_start[t] = carry + ex;
    carry += total;
  }
  if (threadIdx.x == 0) {
    plan.row_tile_start[T] = carry;
    const int tpc = carry > 0 ? (carry + clusters - 1) / clusters : 1;
    plan.meta[0] = carry;
    plan.meta[1] = tpc;
    s_tpc = tpc;
  }
  __syncthreads();
  const int tpc = s_tpc;
  int split_carry = 0;
  for (int base = 0; base < T; base += blockDim.x) {
    const int t = base + threadIdx.x;
    int n = 0, first = 0;
    if (t < T) {
      const int a = plan.row_tile_start[t], b = plan.row_tile_start[t + 1];
      if (b > a) {
        first = a / tpc;
        n = (b - 1) / tpc - first + 1;
      }
    }
    const int parts = n > 1 ? n : 0;
    int total;
    const int ex = block_scan_excl(parts, sums, &total);
    if (t < T) {
      plan.first_cluster[t] = first;
      plan.n_split[t] = n;
      plan.split_base[t] = n > 1 ? split_carry + ex : -1;
    }
    split_carry += total;
  }
}

// Page id of page `pg` of row-lane `b`, or the scratch page past the row's pages (those rows
// are masked) or when the table entry is out of range (flagged).
__device__ __forceinline__ int page_of(const Params& prm, int b, int pg, int row_pages) {
  if (pg >= row_pages) return 0;
  int page = pg < prm.bt_stride ? prm.bt[(int64_t)b * prm.bt_stride + pg] : -1;
  if (page <= 0 || page >= prm.num_pages) {
    hk_flag(prm.err, hk::kErrAttnPage, (unsigned)b);
    page = 0;
  }
  return page;
}

// ---------------------------------------------------------------------------------------
// main kernel
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads, 1)
    mla_decode_sm100_kernel(const __grid_constant__ CUtensorMap q_map,
                            const __grid_constant__ CUtensorMap kv_map,
                            const __grid_constant__ CUtensorMap kv_map2, Params prm) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const uint32_t rank = cluster_rank();
  const int cid = blockIdx.x / kClusterCTAs;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* ctl = smem + kOffCtl;
  volatile int* abort = reinterpret_cast<volatile int*>(ctl + kAbort);
  const uint32_t ctl_u32 = smem_u32(ctl);
  auto bar = [&](int off) { return ctl_u32 + (uint32_t)off; };

  // Cluster tile range (identical in both SMs).
  const int total_tiles = prm.plan.meta[0];
  const int tpc = prm.plan.meta[1];
  const int c0 = cid * tpc;
  const int c1 = min(total_tiles, c0 + tpc);
  if (c0 >= c1) return;  // no work: both SMs of the pair leave together
  if ((smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0) hk_flag(prm.err, hk::kErrWaitTimeout, 900);
    return;
  }

  if (threadIdx.x == 0) {
    for (int i = 0; i < kRing; ++i) {
      mbar_init(bar(kBarFull + 8 * i), 1);
      mbar_init(bar(kBarEmpty + 8 * i), 1);
    }
    mbar_init(bar(kBarQFull), 1);
    mbar_init(bar(kBarQEmpty), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar(kBarSFull + 8 * i), 1);
      mbar_init(bar(kBarSFree + 8 * i), 8);
      mbar_init(bar(kBarPFull + 8 * i), 8);
    }
    mbar_init(bar(kBarODone), 1);
    mbar_init(bar(kBarOFree), 8);
    *abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     bar(kTmemSlot)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(ctl + kTmemSlot);

  const int32_t* rts = prm.plan.row_tile_start;
  int t_first;
  {
    int lo = 0, hi = prm.num_tokens;  // largest t with row_tile_start[t] <= c0
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (rts[mid] <= c0) lo = mid; else hi = mid;
    }
    t_first = lo;
  }

  if (warp == 0) {
    // ----------------------------------------------------------------- TMA producer
    // Entry order (must match the MMA warp): per segment, for each tile i: its 9 K chunks,
    // then (i > 0) the 8 V chunks of tile i-1; after the last tile, its 8 V chunks.
    if (lane == 0) {
      const uint32_t q_s = smem_u32(smem + kOffQ);
      const uint32_t ring = smem_u32(smem + kOffRing);
      int e = 0, seg = 0;
      bool ok = true;
      auto next_entry = [&](uint32_t& dst, uint32_t& fbar) -> bool {
        const int slot = e % kRing;
        if (e >= kRing &&
            !mbar_wait(bar(kBarEmpty + 8 * slot), ((e / kRing) - 1) & 1, abort, prm.err, 2))
          return false;
        if (rank == 0) mbar_expect_tx(bar(kBarFull + 8 * slot), 2 * kEntry);
        fbar = mapa_rank(bar(kBarFull + 8 * slot), 0);
        dst = ring + slot * kEntry;
        ++e;
        return true;
      };
      auto load_v = [&](const int* pages) -> bool {
        for (int j = 0; j < 2; ++j)
          for (int p = 0; p < 4; ++p) {
            uint32_t dst, fbar;
            if (!next_entry(dst, fbar)) return false;
            // this SM's two V chunks of the page are adjacent blocks: one 16 KB box
            tma_load_2d_pair(dst, &kv_map2, fbar, 0, (pages[p] * 9 + 4 * j + 2 * (int)rank) * kPage);
          }
        return true;
      };
      for (int t = t_first; ok && t < prm.num_tokens && rts[t] < c1 && !*abort; ++t) {
        const int a = max(c0, rts[t]) - rts[t], z = min(c1, rts[t + 1]) - rts[t];
        if (a >= z) continue;
        const int b = lane_of_row(prm.cu, prm.num_lanes, t);
        int lo, hi;
        row_span(prm.positions, prm.kv_begin, prm.kv_end, t, b, lo, hi);
        const int pg0 = lo / kPage;                        // page of the row's first KV row
        const int row_pages = (hi + kPage - 1) / kPage;    // pages up to its last
        if (seg > 0 && !mbar_wait(bar(kBarQEmpty), (seg - 1) & 1, abort, prm.err, 1)) break;
        if (rank == 0) mbar_expect_tx(bar(kBarQFull), 2 * 9 * kBox);
        const uint32_t qbar = mapa_rank(bar(kBarQFull), 0);
        for (int d = 0; d < 9; ++d)
          tma_load_2d_pair(q_s + d * kBox, &q_map, qbar, 64 * d, t * kHeads + 64 * (int)rank);
        int prev[4] = {0, 0, 0, 0};
        for (int i = a; ok && i < z; ++i) {
          int cur[4];
          for (int p = 0; p < 4; ++p) cur[p] = page_of(prm, b, pg0 + 4 * i + p, row_pages);
          for (int d = 0; d < 9 && ok; ++d) {
            uint32_t dst, fbar;
            if (!next_entry(dst, fbar)) { ok = false; break; }
            for (int hh = 0; hh < 2; ++hh)
              tma_load_2d_pair(dst + hh * kBox, &kv_map, fbar, 0,
                               (cur[2 * (int)rank + hh] * 9 + d) * kPage);
          }
          if (ok && i > a) ok = load_v(prev);
          for (int p = 0; p < 4; ++p) prev[p] = cur[p];
        }
        if (ok) ok = load_v(prev);
        ++seg;
      }
    }
  } else if (warp == 1) {
    // ----------------------------------------------------------------- MMA issuer
    if (rank == 0 && lane == 0) {
      // Operand descriptors are built once; per MMA only the start-address field (bits 0-13,
      // address / 16) moves, and every shared address here stays below 2^18 bytes, so adding
      // the offset / 16 to the whole descriptor never carries out of the field.
      const uint64_t q_desc = sdesc_sw128(smem_u32(smem + kOffQ), 16, 1024);
      const uint64_t p_desc = sdesc_sw128(smem_u32(smem + kOffP), 16, 1024);
      const uint64_t k_desc = sdesc_sw128(smem_u32(smem + kOffRing), 16, 1024);
      const uint64_t v_desc = sdesc_sw128(smem_u32(smem + kOffRing), kBox, 1024);
      const uint32_t full0 = bar(kBarFull), empty0 = bar(kBarEmpty);
      uint32_t slot = 0, phase = 0;  // ring position and parity of the next entry
      int g = 0, seg = 0;
      bool ok = true;
      auto take_entry = [&](uint32_t& src) -> bool {
        if (!mbar_wait(full0 + 8 * slot, phase, abort, prm.err, 6)) return false;
        tc_fence_after();
        src = slot * (kEntry >> 4);
        return true;
      };
      auto release_entry = [&]() {
        umma_commit_pair(empty0 + 8 * slot);
        if (++slot == kRing) {
          slot = 0;
          phase ^= 1;
        }
      };
      auto issue_pv = [&](int gg, bool first, int seg_of) -> bool {
        const int s = gg & 1;
        if (!mbar_wait(bar(kBarPFull + 8 * s), (gg >> 1) & 1, abort, prm.err, 3)) return false;
        if (first && seg_of > 0 && !mbar_wait(bar(kBarOFree), (seg_of - 1) & 1, abort, prm.err, 4))
          return false;
        tc_fence_after();
#pragma unroll
        for (int j = 0; j < 2; ++j) {
#pragma unroll
          for (int p = 0; p < 4; ++p) {
            uint32_t src;
            if (!take_entry(src)) return false;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_pair(tmem + kTmemO + 128 * j, p_desc + ((p * kPAtom + 32 * kk) >> 4),
                        v_desc + src + ((kk * 2048) >> 4), kIdescPV,
                        (first && p == 0 && kk == 0) ? 0u : 1u);
            release_entry();
          }
        }
        umma_commit_pair(bar(kBarODone));
        return true;
      };
      for (int t = t_first; ok && t < prm.num_tokens && rts[t] < c1 && !*abort; ++t) {
        const int a = max(c0, rts[t]) - rts[t], z = min(c1, rts[t + 1]) - rts[t];
        if (a >= z) continue;
        if (!mbar_wait(bar(kBarQFull), seg & 1, abort, prm.err, 5)) break;
        const int g_first = g;
        for (int i = a; i < z; ++i, ++g) {
          const int s = g & 1;
          if (g >= 2 && !mbar_wait(bar(kBarSFree + 8 * s), ((g >> 1) - 1) & 1, abort, prm.err, 7)) {
            ok = false;
            break;
          }
          for (int d = 0; d < 9; ++d) {
            uint32_t src;
            if (!take_entry(src)) { ok = false; break; }
#pragma unroll
            for (int k = 0; k < 4; ++k)
              umma_pair(tmem + kTmemS + 128 * s, q_desc + ((d * kBox + 32 * k) >> 4),
                        k_desc + src + ((32 * k) >> 4), kIdescQK, (d | k) ? 1u : 0u);
            release_entry();
          }
          if (!ok) break;
          umma_commit_pair(bar(kBarSFull + 8 * s));
          if (i == z - 1) umma_commit_pair(bar(kBarQEmpty));
          if (g > g_first && !issue_pv(g - 1, g - 1 == g_first, seg)) { ok = false; break; }
        }
        if (!ok) break;
        if (!issue_pv(g - 1, g - 1 == g_first, seg)) break;
        ++seg;
      }
    }
  } else {
    // ----------------------------------------------------------------- softmax / epilogue
    // The four softmax warps meet at named barrier 1 at the same points whatever happens:
    // a failed (timed-out or aborted) wait only clears `live`, which is kept warp-uniform,
    // and a dead warp skips its tensor-memory and barrier traffic but not the bar.syncs.
    const int sub = warp & 3;                 // TMEM lane quarter of this warp
    const int L = sub * 32 + lane;            // TMEM lane = row of this thread
    const int hd = L & 63;                    // head within this SM's 64
    const int th = L >> 6;                    // token half of the tile / O column half
    const uint32_t lane_addr = (uint32_t)(sub * 32) << 16;
    float* xmax = reinterpret_cast<float*>(ctl + kXchMax);
    float* xl = reinterpret_cast<float*>(ctl + kXchL);
    uint8_t* p_base = smem + kOffP;
    int g = 0;
    bool live = true;
    for (int t = t_first; t < prm.num_tokens && rts[t] < c1; ++t) {
      const int a = max(c0, rts[t]) - rts[t], z = min(c1, rts[t + 1]) - rts[t];
      if (a >= z) continue;
      int kv_lo, kv_len;
      row_span(prm.positions, prm.kv_begin, prm.kv_end, t, lane_of_row(prm.cu, prm.num_lanes, t),
               kv_lo, kv_len);
      kv_len -= kv_lo - kv_lo % kPage;  // tile coordinates start at the first page
      kv_lo %= kPage;                   // rows of the first page before the range
      float m_run = -INFINITY, l_part = 0.f;
      const int g_first = g;
      for (int i = a; i < z; ++i, ++g) {
        const int s = g & 1;
        live = live && mbar_wait(bar(kBarSFull + 8 * s), (g >> 1) & 1, abort, prm.err, 8);
        live = __all_sync(0xffffffffu, live);
        float v[128];
        float mt = -INFINITY;
        if (live) {
          tc_fence_after();
          tmem_ld64(tmem + lane_addr + kTmemS + 128 * s, v);
          tmem_ld64(tmem + lane_addr + kTmemS + 128 * s + 64, v + 64);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_leader(bar(kBarSFree + 8 * s), rank);
          const int tok0 = i * kTileTok + th * 128;
          const int valid = kv_len - tok0;  // tokens of this thread's 128 that exist
          const int skip = tok0 == 0 ? kv_lo : 0;  // leading rows outside the range
          if (skip == 0) {
#pragma unroll
            for (int k = 0; k < 128; ++k) {
              v[k] = (k < valid) ? v[k] * prm.scale_log2 : -INFINITY;
              mt = fmaxf(mt, v[k]);
            }
          } else {
#pragma unroll
            for (int k = 0; k < 128; ++k) {
              v[k] = (k >= skip && k < valid) ? v[k] * prm.scale_log2 : -INFINITY;
              mt = fmaxf(mt, v[k]);
            }
          }
        }
        float* xm = xmax + (g & 1) * 128;
        xm[L] = mt;
        asm volatile("bar.sync 1, 128;" ::: "memory");
        mt = fmaxf(mt, xm[L ^ 64]);
        if (!live) continue;
        const bool first = (g == g_first);
        const float m_new = fmaxf(m_run, mt);
        const bool rescale = !first && (m_new > m_run + 8.0f);
        const float m_use = (first || rescale) ? m_new : m_run;
        const float corr = rescale ? ex2_approx(m_run - m_new) : 1.f;
        const float m_sub = (m_use == -INFINITY) ? 0.f : m_use;
        // The single P buffer and (on a rescale) O are rewritten only once PV(g-1) is done.
        // PV(g-2) is known complete (S(g) was ready), so this parity wait is unambiguous.
        if (g >= 1) {
          live = mbar_wait(bar(kBarODone), (g - 1) & 1, abort, prm.err, 9);
          live = __all_sync(0xffffffffu, live);
          if (!live) continue;
        }
        if (__any_sync(0xffffffffu, rescale)) {
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < 8; ++c) {
            float o[32];
            tmem_ld32(tmem + lane_addr + kTmemO + 32 * c, o);
#pragma unroll
            for (int k = 0; k < 32; ++k) o[k] *= corr;
            tmem_st32(tmem + lane_addr + kTmemO + 32 * c, o);
          }
          asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
        }
        // P row hd, tokens th*128 .. th*128+127: 16 chunks of 8 tokens in atoms of 64.
        float psum = 0.f;
        uint8_t* prow = p_base + hd * 128;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const float x0 = ex2_approx(v[8 * c + 2 * k] - m_sub);
            const float x1 = ex2_approx(v[8 * c + 2 * k + 1] - m_sub);
            psum += x0 + x1;
            __nv_bfloat162 pr = __floats2bfloat162_rn(x0, x1);
            w[k] = *reinterpret_cast<uint32_t*>(&pr);
          }
          const int atom = th * 2 + (c >> 3), kc = c & 7;
          *reinterpret_cast<uint4*>(prow + atom * kPAtom + ((kc ^ (hd & 7)) << 4)) =
              make_uint4(w[0], w[1], w[2], w[3]);
        }
        l_part = first ? psum : l_part * corr + psum;
        m_run = m_use;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_leader(bar(kBarPFull + 8 * s), rank);
      }
      // Epilogue: wait for the segment's last PV, normalise, store.  A parity wait only
      // tells completion k apart from k-2, and here only PV(g_last-2) is known complete
      // (S(g_last) was ready), so PV(g_last-1) is waited for first.
      const int g_last = g - 1;
      if (g_last >= 1)
        live = live && mbar_wait(bar(kBarODone), (g_last - 1) & 1, abort, prm.err, 11);
      live = live && mbar_wait(bar(kBarODone), g_last & 1, abort, prm.err, 10);
      live = __all_sync(0xffffffffu, live);
      xl[L] = l_part;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      const float l_tot = l_part + xl[L ^ 64];
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (!live) continue;
      tc_fence_after();
      const float inv = l_tot > 0.f ? 1.f / l_tot : 0.f;
      const float lse_v =
          l_tot > 0.f ? (m_run + log2f(l_tot)) * 0.69314718055994530942f : -INFINITY;
      const int head = 64 * (int)rank + hd;
      const bool split = prm.plan.n_split[t] > 1;
      const int64_t orow =
          split ? (int64_t)(prm.plan.split_base[t] + (cid - prm.plan.first_cluster[t])) * kHeads + head
                : (int64_t)t * kHeads + head;
#pragma unroll 1
      for (int c = 0; c < 8; ++c) {
        float o[32];
        tmem_ld32(tmem + lane_addr + kTmemO + 32 * c, o);
        const int dim0 = 256 * (c >> 2) + 128 * th + 32 * (c & 3);
        if (split || prm.out_f32 != nullptr) {
          float4* dst = reinterpret_cast<float4*>((split ? prm.part_o : prm.out_f32) + orow * kDV + dim0);
#pragma unroll
          for (int k = 0; k < 8; ++k)
            dst[k] = make_float4(o[4 * k] * inv, o[4 * k + 1] * inv, o[4 * k + 2] * inv,
                                 o[4 * k + 3] * inv);
        } else {
          uint4* dst = reinterpret_cast<uint4*>(prm.out + orow * kDV + dim0);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            uint32_t w[4];
#pragma unroll
            for (int m = 0; m < 4; ++m) {
              __nv_bfloat162 pr =
                  __floats2bfloat162_rn(o[8 * k + 2 * m] * inv, o[8 * k + 2 * m + 1] * inv);
              w[m] = *reinterpret_cast<uint32_t*>(&pr);
            }
            dst[k] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
      if (th == 0) {
        if (split) prm.part_lse[orow] = lse_v;
        else prm.lse[orow] = lse_v;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_leader(bar(kBarOFree), rank);
    }
  }

  // Teardown: a timed-out pair gives in-flight copies time to land before smem goes away.
  __syncwarp();
  if (*abort) {
    const unsigned long long t0 = globaltimer();
    while (globaltimer() - t0 < 2000000ull) {
    }
  }
  tc_fence_before();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512)
                 : "memory");
  }
}

// Merge of split rows: one CTA of 128 threads (4 dims each) per (row, head).
// A row with no tile (its range is empty) gets o = 0 and lse = -inf here.
__global__ void mla_merge_kernel(const float* __restrict__ part_o, const float* __restrict__ part_lse,
                                 Plan plan, int32_t T, uint16_t* __restrict__ out,
                                 float* __restrict__ out_f32, float* __restrict__ lse) {
  const int t = blockIdx.x / kHeads, h = blockIdx.x % kHeads;
  const int n = plan.n_split[t];
  if (n == 1) return;
  const int base = plan.split_base[t];
  float m = -INFINITY;
  for (int i = 0; i < n; ++i) m = fmaxf(m, part_lse[(int64_t)(base + i) * kHeads + h]);
  float sum = 0.f;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int i = 0; i < n; ++i) {
    const float li = part_lse[(int64_t)(base + i) * kHeads + h];
    const float w = li == -INFINITY ? 0.f : expf(li - m);
    sum += w;
    const float4 o = reinterpret_cast<const float4*>(part_o + ((int64_t)(base + i) * kHeads + h) * kDV)[threadIdx.x];
    acc.x = fmaf(w, o.x, acc.x);
    acc.y = fmaf(w, o.y, acc.y);
    acc.z = fmaf(w, o.z, acc.z);
    acc.w = fmaf(w, o.w, acc.w);
  }
  const float inv = sum > 0.f ? 1.f / sum : 0.f;
  const int64_t row = (int64_t)t * kHeads + h;
  if (out_f32 != nullptr) {
    reinterpret_cast<float4*>(out_f32 + row * kDV)[threadIdx.x] =
        make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
  } else {
    uint2 pk;
    __nv_bfloat162 a = __floats2bfloat162_rn(acc.x * inv, acc.y * inv);
    __nv_bfloat162 b = __floats2bfloat162_rn(acc.z * inv, acc.w * inv);
    pk.x = *reinterpret_cast<uint32_t*>(&a);
    pk.y = *reinterpret_cast<uint32_t*>(&b);
    reinterpret_cast<uint2*>(out + row * kDV)[threadIdx.x] = pk;
  }
  if (threadIdx.x == 0) lse[row] = sum > 0.f ? m + logf(sum) : -INFINITY;
}

// ---------------------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
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

// 2-D bf16 map of `rows` rows of `cols` elements, boxes of box_rows x 64, 128B swizzle.
int make_map_bf16(CUtensorMap* m, const void* base, uint64_t rows, uint32_t cols,
                  uint32_t box_rows) {
  EncodeTiledFn f = encode_fn();
  if (f == nullptr) return hk::fail(HK_ECUDA, "cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = f(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                 estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return hk::fail(HK_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return HK_OK;
}

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

constexpr int kMaxClusters = 128;

}  // namespace

namespace hk {

bool mla_sm100_supported(int32_t heads, int32_t page_size, int32_t num_tokens, int32_t) {
  return heads == kHeads && page_size == kPage && num_tokens > 0;
}

size_t mla_sm100_workspace(int32_t, int32_t num_tokens, int32_t heads, int32_t) {
  if (heads != kHeads) return 0;
  const size_t T = (size_t)num_tokens;
  const size_t plan = align256(sizeof(int32_t) * (4 * T + 1 + 8));
  const size_t parts = T + kMaxClusters;
  return plan + align256(parts * kHeads * kDV * sizeof(float)) +
         align256(parts * kHeads * sizeof(float));
}

int mla_sm100(const uint16_t* q, const uint16_t* kv_cache, const int32_t* block_table,
              int32_t bt_stride, const int32_t* cu_seqlens, const int32_t* positions,
              const int32_t* kv_begin, const int32_t* kv_end, int32_t num_lanes,
              int32_t num_tokens, int32_t heads, int32_t page_size, int64_t num_slots,
              int32_t max_kv_len, float scale, uint16_t* out, float* out_f32, float* lse,
              void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  (void)max_kv_len;
  const size_t need = mla_sm100_workspace(num_lanes, num_tokens, heads, max_kv_len);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(HK_ESPACE, "mla_sm100: workspace of %zu bytes, %zu needed", workspace_bytes, need);
  if (num_slots % kPage != 0)
    return fail(HK_EINVAL, "mla_sm100: cache rows %lld not a whole number of pages",
                (long long)num_slots);
  const size_t T = (size_t)num_tokens;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  Plan plan;
  plan.row_tile_start = reinterpret_cast<int32_t*>(ws);
  plan.first_cluster = plan.row_tile_start + T + 1;
  plan.n_split = plan.first_cluster + T;
  plan.split_base = plan.n_split + T;
  plan.meta = plan.split_base + T;
  float* part_o = reinterpret_cast<float*>(ws + align256(sizeof(int32_t) * (4 * T + 1 + 8)));
  float* part_lse = part_o + (T + kMaxClusters) * kHeads * kDV;

  int sms = sm_count();
  int clusters = sms / kClusterCTAs;
  if (clusters > kMaxClusters) clusters = kMaxClusters;

  CUtensorMap q_map, kv_map, kv_map2;
  // q: rows of 576 dims.  The page-blocked cache: every page is 9 blocks of 64 rows x 64 dims,
  // so as a 2-D array it is (num_slots * 9) rows of 64 dims; block d of page p starts at row
  // (p * 9 + d) * 64 and one box is a contiguous 8 KB (kv_map2: two adjacent blocks, 16 KB).
  HK_TRY(make_map_bf16(&q_map, q, (uint64_t)num_tokens * kHeads, kDK, 64));
  HK_TRY(make_map_bf16(&kv_map, kv_cache, (uint64_t)num_slots * 9, 64, 64));
  HK_TRY(make_map_bf16(&kv_map2, kv_cache, (uint64_t)num_slots * 9, 64, 128));

  mla_plan_kernel<<<1, 1024, 0, stream>>>(positions, cu_seqlens, num_lanes, kv_begin, kv_end,
                                          num_tokens, clusters, plan, err_word());
  HK_TRY_LAUNCH("mla_plan_kernel");

  Params prm;
  prm.bt = block_table;
  prm.bt_stride = bt_stride;
  prm.cu = cu_seqlens;
  prm.positions = positions;
  prm.kv_begin = kv_begin;
  prm.kv_end = kv_end;
  prm.num_lanes = num_lanes;
  prm.num_tokens = num_tokens;
  prm.num_pages = (int32_t)(num_slots / kPage);
  prm.scale_log2 = scale * 1.4426950408889634f;
  prm.out = out;
  prm.out_f32 = out_f32;
  prm.lse = lse;
  prm.part_o = part_o;
  prm.part_lse = part_lse;
  prm.plan = plan;
  prm.err = err_word();

  HK_TRY_CUDA(cudaFuncSetAttribute(mla_decode_sm100_kernel,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(clusters * kClusterCTAs);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kClusterCTAs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  HK_TRY_CUDA(cudaLaunchKernelEx(&cfg, mla_decode_sm100_kernel, q_map, kv_map, kv_map2, prm));
  note_launch();

  mla_merge_kernel<<<(unsigned)(T * kHeads), kDV / 4, 0, stream>>>(part_o, part_lse, plan,
                                                                   num_tokens, out, out_f32, lse);
  HK_TRY_LAUNCH("mla_merge_kernel");
  return HK_OK;
}

}  // namespace hk
