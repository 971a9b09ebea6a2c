// a12-a15: MoE router, permutation, grouped FP8 expert FFN and weighted combine.
//
//  * route: one warp per token; each lane holds ceil(E/32) scores, top_k rounds of a warp
//    arg-max (ties -> lower expert id).  The sigmoid is hk_sigmoid_det so the CPU oracle
//    reproduces selection bit for bit.
//  * permute: one CTA.  Histogram by smem atomics (order-free), exclusive scan, then a
//    stable rank of every (token, k) pair inside its expert: pairs go in rounds of 1024
//    in (token, k) order, __match_any_sync ranks them inside the warp and a per-expert
//    scan over the warps orders the warps.  No result depends on atomic order.
//  * grouped FFN (portable): a device-built list of 64-row tiles per expert drives two
//    tiled FP8 GEMM kernels (gate/up fused with silu*mul and the 1x128 requantisation of
//    h; then down).  Rows are gathered through perm_token.
//  * combine: one CTA per token, k-ordered fp32 sums of 8-wide bf16 vectors.
#include <math.h>

#include "common.cuh"
#include "gemm_fp8.cuh"
#include "moe.cuh"

namespace {

constexpr int kMaxExperts = 512;
constexpr int kPermThreads = 1024;
constexpr int kTileRows = 64;

__global__ void route_kernel(const float* __restrict__ logits, const float* __restrict__ bias,
                             int32_t tokens, int32_t E, int32_t top_k, float route_scale,
                             int32_t* __restrict__ ids, float* __restrict__ weights,
                             unsigned long long* err) {
  const int t = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= tokens) return;
  constexpr int kPer = 256 / 32;
  float s[kPer], sel[kPer];
  bool bad = false;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int e = lane + 32 * i;
    if (e < E) {
      const float x = logits[(int64_t)t * E + e];
      bad |= !isfinite(x);
      s[i] = hk_sigmoid_det(x);
      sel[i] = __fadd_rn(s[i], bias != nullptr ? bias[e] : 0.f);
    } else {
      s[i] = 0.f;
      sel[i] = -INFINITY;
    }
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0) hk_flag(err, hk::kErrRouteInput, (unsigned)t);
  float chosen_s = 0.f;
  int chosen_e = -1;
  float sum = 0.f;
  for (int k = 0; k < top_k; ++k) {
    float best = -INFINITY;
    int best_e = 0x7fffffff, best_i = -1;
#pragma unroll
    for (int i = 0; i < kPer; ++i) {
      const int e = lane + 32 * i;
      if (sel[i] > best || (sel[i] == best && e < best_e && sel[i] != -INFINITY)) {
        best = sel[i];
        best_e = e;
        best_i = i;
      }
    }
    // Warp arg-max with the lower expert id winning ties.
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oe = __shfl_xor_sync(0xffffffffu, best_e, o);
      if (ob > best || (ob == best && oe < best_e)) {
        best = ob;
        best_e = oe;
      }
    }
    float win_s = 0.f;
#pragma unroll
    for (int i = 0; i < kPer; ++i)
      if (lane + 32 * i == best_e) {
        win_s = s[i];
        sel[i] = -INFINITY;
      }
    (void)best_i;
    win_s = __shfl_sync(0xffffffffu, win_s, best_e & 31);
    sum = __fadd_rn(sum, win_s);
    if (lane == k) {
      chosen_s = win_s;
      chosen_e = best_e;
    }
  }
  if (lane < top_k) {
    ids[(int64_t)t * top_k + lane] = chosen_e;
    weights[(int64_t)t * top_k + lane] = __fmul_rn(__fdiv_rn(chosen_s, sum), route_scale);
  }
}

__global__ void __launch_bounds__(kPermThreads) permute_kernel(
    const int32_t* __restrict__ ids, const float* __restrict__ weights, int32_t tokens,
    int32_t top_k, int32_t E, int32_t* __restrict__ offsets, int32_t* __restrict__ perm_token,
    float* __restrict__ perm_weight, int32_t* __restrict__ inv, unsigned long long* err) {
  extern __shared__ int sm[];
  int* count = sm;                    // [E]
  int* base = count + E;              // [E]  running rank base per expert
  int* wcnt = base + E;               // [32][E] per-warp counts, then exclusive prefixes
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int P = tokens * top_k;
  for (int e = tid; e < E; e += kPermThreads) count[e] = 0;
  __syncthreads();
  for (int p = tid; p < P; p += kPermThreads) {
    const int e = ids[p];
    if (e >= 0 && e < E) atomicAdd(&count[e], 1);
    else hk_flag(err, hk::kErrMoeRow, (unsigned)p);
  }
  __syncthreads();
  if (tid == 0) {
    int run = 0;
    for (int e = 0; e < E; ++e) {
      offsets[e] = run;
      base[e] = run;
      run += count[e];
    }
    offsets[E] = run;
  }
  __syncthreads();
  int* round_total = count;  // the histogram is spent once offsets are written
  for (int r0 = 0; r0 < P; r0 += kPermThreads) {
    for (int i = tid; i < 32 * E; i += kPermThreads) wcnt[i] = 0;
    __syncthreads();
    const int p = r0 + tid;
    int e = -1;
    if (p < P) {
      e = ids[p];
      if (e < 0 || e >= E) e = -1;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank_in_warp = __popc(peers & ((1u << lane) - 1));
    if (e >= 0 && rank_in_warp == 0) wcnt[warp * E + e] = __popc(peers);
    __syncthreads();
    for (int x = tid; x < E; x += kPermThreads) {
      int run = 0;
      for (int w = 0; w < 32; ++w) {
        const int c = wcnt[w * E + x];
        wcnt[w * E + x] = run;
        run += c;
      }
      round_total[x] = run;
    }
    __syncthreads();
    if (e >= 0) {
      const int dst = base[e] + wcnt[warp * E + e] + rank_in_warp;
      perm_token[dst] = p / top_k;
      perm_weight[dst] = weights[p];
      inv[p] = dst;
    } else if (p < P) {
      inv[p] = -1;
    }
    __syncthreads();
    for (int x = tid; x < E; x += kPermThreads) base[x] += round_total[x];
    __syncthreads();
  }
}

// Builds the list of (expert, first row) tiles of kTileRows rows.  One warp: lanes take
// experts in rounds of 32, a warp scan of their tile counts places each expert's tiles.
__global__ void tile_list_kernel(const int32_t* __restrict__ offsets, int32_t E, int64_t rows,
                                 int32_t max_tiles, int32_t* __restrict__ tile_expert,
                                 int32_t* __restrict__ tile_row, int32_t* __restrict__ num_tiles,
                                 unsigned long long* err) {
  const int lane = threadIdx.x;
  if (lane >= 32) return;
  // Offsets must be non-decreasing and end within the caller's row buffers.
  bool bad = false;
  for (int e = lane; e < E; e += 32) bad |= offsets[e] > offsets[e + 1];
  bad = __any_sync(0xffffffffu, bad) || offsets[0] != 0 || offsets[E] > rows;
  if (bad) {
    if (lane == 0) {
      hk_flag(err, hk::kErrMoeRow, (unsigned)offsets[E]);
      *num_tiles = 0;
    }
    return;
  }
  int base = 0;
  for (int e0 = 0; e0 < E; e0 += 32) {
    const int e = e0 + lane;
    const int lo = e < E ? offsets[e] : 0, hi = e < E ? offsets[e + 1] : 0;
    const int n = (hi - lo + kTileRows - 1) / kTileRows;
    int incl = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const int first = base + incl - n;
    for (int i = 0; i < n; ++i) {
      if (first + i < max_tiles) {
        tile_expert[first + i] = e;
        tile_row[first + i] = lo + i * kTileRows;
      }
    }
    base += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) *num_tiles = base < max_tiles ? base : max_tiles;
}

// The tcgen05 kernels' tile list: every expert's rows cut into tiles of one width, the widest
// of those allowed (bit i of `widths` for moe_tile_width(i)) whose threshold the experts' rows
// per expert on average reach — a decode batch's ~2 rows an expert take 16-row tiles, config
// 4's ~18 take 32, a prompt pass's ~145 take 96 — so most experts stream their weights once,
// in the narrowest tile that holds them.  The choice reads the actual row total on the
// device, so a caller that passes a row capacity (expert parallelism) gets the right width;
// num[1] tells the launched kernels which of them has the tiles.  One warp, experts in rounds
// of 32, a warp scan.
__global__ void tc_list_kernel(const int32_t* __restrict__ offsets, int32_t E, int64_t rows, int32_t widths,
                               int32_t max_tiles, int32_t* __restrict__ tile_expert,
                               int32_t* __restrict__ tile_row, int32_t* __restrict__ num,
                               unsigned long long* err) {
  const int lane = threadIdx.x;
  if (lane >= 32) return;
  bool bad = false;
  for (int e = lane; e < E; e += 32) bad |= offsets[e] > offsets[e + 1];
  bad = __any_sync(0xffffffffu, bad) || offsets[0] != 0 || offsets[E] > rows;
  if (bad) {
    if (lane == 0) {
      hk_flag(err, hk::kErrMoeRow, (unsigned)offsets[E]);
      num[0] = 0;
      num[1] = 0;
    }
    return;
  }
  int step = hk::moe_tile_width(0);
#pragma unroll
  for (int i = 3; i > 0; --i)
    if ((widths >> i) & 1 && (int64_t)offsets[E] >= (int64_t)hk::moe_tile_min_avg(i) * E) {
      step = hk::moe_tile_width(i);
      break;
    }
  int base = 0;
  for (int e0 = 0; e0 < E; e0 += 32) {
    const int e = e0 + lane;
    const int lo = e < E ? offsets[e] : 0, hi = e < E ? offsets[e + 1] : 0;
    const int n = (hi - lo + step - 1) / step;
    int incl = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    const int first = base + incl - n;
    for (int i = 0; i < n; ++i) {
      if (first + i < max_tiles) {
        tile_expert[first + i] = e;
        tile_row[first + i] = lo + step * i;
      }
    }
    base += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) {
    num[0] = base < max_tiles ? base : max_tiles;
    num[1] = step;
  }
}

// Gate/up GEMM for one (row tile, 128-column block of h): g and u accumulate in fp32,
// h = silu(g) * u, then h is requantised to e4m3 with one scale per (row, 128 block).
__global__ void __launch_bounds__(256) moe_up_kernel(
    const uint8_t* __restrict__ xq, const float* __restrict__ sx, const int32_t* __restrict__ offsets,
    const int32_t* __restrict__ perm_token, const int32_t* __restrict__ tile_expert,
    const int32_t* __restrict__ tile_row, const int32_t* __restrict__ num_tiles, int32_t hidden,
    int32_t inter, int32_t tokens_limit, const uint8_t* __restrict__ w13,
    const float* __restrict__ s13, uint8_t* __restrict__ hq, float* __restrict__ hs,
    unsigned long long* err) {
  const int tile = blockIdx.x;
  if (tile >= *num_tiles) return;
  __shared__ float lut[256];
  __shared__ uint8_t xs[kTileRows][128 + 4];
  __shared__ uint8_t gs[128][128 + 4];  // gate rows of this column block
  __shared__ uint8_t us[128][128 + 4];  // up rows
  __shared__ int src_s[kTileRows];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int e = tile_expert[tile], r0 = tile_row[tile], r_end = offsets[e + 1];
  const int nb = blockIdx.y;  // 128-wide column block of h
  const int kblocks = hidden / 128;
  lut[tid] = e4m3_to_f32((uint8_t)tid);
  if (tid < kTileRows) {
    const int p = r0 + tid;
    int src = -1;
    if (p < r_end) {
      src = perm_token[p];
      if (src < 0 || src >= tokens_limit) {
        hk_flag(err, hk::kErrMoeRow, (unsigned)p);
        src = -1;
      }
    }
    src_s[tid] = src;
  }
  const uint8_t* wg = w13 + (int64_t)e * 2 * inter * hidden;
  const uint8_t* wu = wg + (int64_t)inter * hidden;
  const float* sg = s13 + (int64_t)e * (2 * inter / 128) * kblocks;
  const float* su = sg + (int64_t)(inter / 128) * kblocks;
  float g[4][8] = {}, u[4][8] = {};
  for (int kb = 0; kb < kblocks; ++kb) {
    __syncthreads();
    for (int i = tid; i < kTileRows * 8; i += 256) {
      const int r = i / 8, c = i % 8;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (src_s[r] >= 0) v = *reinterpret_cast<const uint4*>(xq + (int64_t)src_s[r] * hidden + kb * 128 + c * 16);
      uint32_t* d = reinterpret_cast<uint32_t*>(&xs[r][c * 16]);
      d[0] = v.x; d[1] = v.y; d[2] = v.z; d[3] = v.w;
    }
    for (int i = tid; i < 128 * 8; i += 256) {
      const int r = i / 8, c = i % 8;
      const int64_t wrow = (int64_t)(nb * 128 + r) * hidden + kb * 128 + c * 16;
      const uint4 vg = *reinterpret_cast<const uint4*>(wg + wrow);
      const uint4 vu = *reinterpret_cast<const uint4*>(wu + wrow);
      uint32_t* dg = reinterpret_cast<uint32_t*>(&gs[r][c * 16]);
      uint32_t* du = reinterpret_cast<uint32_t*>(&us[r][c * 16]);
      dg[0] = vg.x; dg[1] = vg.y; dg[2] = vg.z; dg[3] = vg.w;
      du[0] = vu.x; du[1] = vu.y; du[2] = vu.z; du[3] = vu.w;
    }
    __syncthreads();
    float pg[4][8] = {}, pu[4][8] = {};
    for (int kk = 0; kk < 128; ++kk) {
      float a[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = lut[xs[ty * 4 + i][kk]];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float bg = lut[gs[tx * 8 + j][kk]], bu = lut[us[tx * 8 + j][kk]];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          pg[i][j] = fmaf(a[i], bg, pg[i][j]);
          pu[i][j] = fmaf(a[i], bu, pu[i][j]);
        }
      }
    }
    const float wsg = sg[(int64_t)nb * kblocks + kb], wsu = su[(int64_t)nb * kblocks + kb];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int src = src_s[ty * 4 + i];
      const float xsc = src >= 0 ? sx[(int64_t)src * kblocks + kb] : 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        g[i][j] = fmaf(pg[i][j], xsc * wsg, g[i][j]);
        u[i][j] = fmaf(pu[i][j], xsc * wsu, u[i][j]);
      }
    }
  }
  // h = silu(g) * u; row amax over the 128 columns held by the 16 threads of this row group.
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float h[8], amax = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float gv = g[i][j];
      h[j] = gv / (1.f + expf(-gv)) * u[i][j];
      amax = fmaxf(amax, fabsf(h[j]));
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float s = __fdiv_rn(fmaxf(amax, 1e-12f), 448.0f);
    const int p = r0 + ty * 4 + i;
    if (p < r_end) {
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) lo |= (uint32_t)f32_to_e4m3(__fdiv_rn(h[j], s)) << (8 * j);
#pragma unroll
      for (int j = 0; j < 4; ++j) hi |= (uint32_t)f32_to_e4m3(__fdiv_rn(h[4 + j], s)) << (8 * j);
      *reinterpret_cast<uint2*>(hq + (int64_t)p * inter + nb * 128 + tx * 8) = make_uint2(lo, hi);
      if (tx == 0) hs[(int64_t)p * (inter / 128) + nb] = s;
    }
  }
}

// Down GEMM for one (row tile, 64 output columns): y[p] = sum_kb (hq . w2q) * hs * s2.
__global__ void __launch_bounds__(256) moe_down_kernel(
    const uint8_t* __restrict__ hq, const float* __restrict__ hs,
    const int32_t* __restrict__ offsets, const int32_t* __restrict__ tile_expert,
    const int32_t* __restrict__ tile_row, const int32_t* __restrict__ num_tiles, int32_t hidden,
    int32_t inter, const uint8_t* __restrict__ w2, const float* __restrict__ s2,
    uint16_t* __restrict__ y) {
  const int tile = blockIdx.x;
  if (tile >= *num_tiles) return;
  __shared__ float lut[256];
  __shared__ uint8_t xs[kTileRows][128 + 4];
  __shared__ uint8_t ws[64][128 + 4];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int e = tile_expert[tile], r0 = tile_row[tile], r_end = offsets[e + 1];
  const int n0 = blockIdx.y * 64;
  const int kblocks = inter / 128;
  lut[tid] = e4m3_to_f32((uint8_t)tid);
  const uint8_t* we = w2 + (int64_t)e * hidden * inter;
  const float* se = s2 + (int64_t)e * (hidden / 128) * kblocks;
  float acc[4][4] = {};
  for (int kb = 0; kb < kblocks; ++kb) {
    __syncthreads();
    for (int i = tid; i < kTileRows * 8; i += 256) {
      const int r = i / 8, c = i % 8;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (r0 + r < r_end) v = *reinterpret_cast<const uint4*>(hq + (int64_t)(r0 + r) * inter + kb * 128 + c * 16);
      uint32_t* d = reinterpret_cast<uint32_t*>(&xs[r][c * 16]);
      d[0] = v.x; d[1] = v.y; d[2] = v.z; d[3] = v.w;
      const uint4 w = *reinterpret_cast<const uint4*>(we + (int64_t)(n0 + r) * inter + kb * 128 + c * 16);
      uint32_t* dw = reinterpret_cast<uint32_t*>(&ws[r][c * 16]);
      dw[0] = w.x; dw[1] = w.y; dw[2] = w.z; dw[3] = w.w;
    }
    __syncthreads();
    float part[4][4] = {};
    for (int kk = 0; kk < 128; ++kk) {
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
      const int p = r0 + ty * 4 + i;
      const float a_s = p < r_end ? hs[(int64_t)p * kblocks + kb] : 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float b_s = se[(int64_t)((n0 + tx * 4 + j) / 128) * kblocks + kb];
        acc[i][j] = fmaf(part[i][j], a_s * b_s, acc[i][j]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int p = r0 + ty * 4 + i;
    if (p >= r_end) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) y[(int64_t)p * hidden + n0 + tx * 4 + j] = f32_to_bf16_bits(acc[i][j]);
  }
}

__global__ void combine_kernel(const uint4* __restrict__ y, int64_t y_rows,
                               const float* __restrict__ perm_weight,
                               const int32_t* __restrict__ inv, const uint4* __restrict__ shared,
                               int32_t top_k, int32_t hidden_vec, uint4* __restrict__ out,
                               unsigned long long* err) {
  const int t = blockIdx.x;
  __shared__ int rows[16];
  __shared__ float ws[16];
  if (threadIdx.x < top_k) {
    int r = inv[(int64_t)t * top_k + threadIdx.x];
    if (r >= y_rows) {
      hk_flag(err, hk::kErrMoeRow, (unsigned)t);
      r = -1;
    }
    rows[threadIdx.x] = r;
    ws[threadIdx.x] = r >= 0 ? perm_weight[r] : 0.f;
  }
  __syncthreads();
  for (int v = threadIdx.x; v < hidden_vec; v += blockDim.x) {
    float acc[8] = {};
    for (int k = 0; k < top_k; ++k) {
      if (rows[k] < 0) continue;
      const uint4 u = y[(int64_t)rows[k] * hidden_vec + v];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
      const float wk = ws[k];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[2 * i] = fmaf(wk, __uint_as_float(w[i] << 16), acc[2 * i]);
        acc[2 * i + 1] = fmaf(wk, __uint_as_float(w[i] & 0xffff0000u), acc[2 * i + 1]);
      }
    }
    if (shared != nullptr) {
      const uint4 u = shared[(int64_t)t * hidden_vec + v];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        acc[2 * i] += __uint_as_float(w[i] << 16);
        acc[2 * i + 1] += __uint_as_float(w[i] & 0xffff0000u);
      }
    }
    uint4 o;
    uint32_t* op = &o.x;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      op[i] = (uint32_t)f32_to_bf16_bits(acc[2 * i]) | ((uint32_t)f32_to_bf16_bits(acc[2 * i + 1]) << 16);
    out[(int64_t)t * hidden_vec + v] = o;
  }
}

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

}  // namespace

namespace hk {

size_t moe_portable_workspace(int64_t rows, int32_t inter) {
  const int64_t max_tiles = rows / kTileRows + kMaxExperts + 1;
  return align256((size_t)rows * inter) + align256((size_t)rows * (inter / 128) * sizeof(float)) +
         align256((size_t)max_tiles * 2 * sizeof(int32_t) + sizeof(int32_t));
}

// The tcgen05 path's tile list: expert / row pairs (room for 16-row tiles), count and width.
size_t tc_list_bytes(int64_t rows) {
  return align256((size_t)(rows / hk::moe_tile_width(0) + kMaxExperts + 1) * 2 * sizeof(int32_t) +
                  2 * sizeof(int32_t));
}

size_t moe_full_workspace(int64_t rows, int32_t hidden, int32_t inter) {
  return moe_portable_workspace(rows, inter) + align256((size_t)rows * hidden) +
         align256((size_t)rows * (hidden / 128) * sizeof(float)) + tc_list_bytes(rows);
}

// The grouped FFN launcher behind hk_moe_grouped: `err` is the device error word the kernels
// record bad rows in (nullptr: skipped without a record).
int moe_grouped_run(const uint8_t* xq, const float* sx, int32_t tokens, const int32_t* offsets,
                    const int32_t* perm_token, int64_t rows, int32_t num_experts, int32_t hidden,
                    int32_t inter, const uint8_t* w13, const float* s13, const uint8_t* w2,
                    const float* s2, uint16_t* y, void* workspace, size_t workspace_bytes,
                    bool portable_only, unsigned long long* err, cudaStream_t s) {
  HK_TRY(hk::ensure_device());
  HK_REQUIRE(rows == 0 || (xq && sx && offsets && perm_token && w13 && s13 && w2 && s2 && y),
             "hk_moe_grouped: null pointer");
  HK_REQUIRE(num_experts > 0 && num_experts <= kMaxExperts, "hk_moe_grouped: %d experts", num_experts);
  HK_REQUIRE(hidden > 0 && hidden % 128 == 0 && inter > 0 && inter % 128 == 0,
             "hk_moe_grouped: hidden %d and inter %d must be multiples of 128", hidden, inter);
  HK_REQUIRE(((uintptr_t)xq | (uintptr_t)w13 | (uintptr_t)w2) % 16 == 0,
             "hk_moe_grouped: operands must be 16-byte aligned");
  HK_REQUIRE(tokens >= 0 && rows >= 0, "hk_moe_grouped: negative sizes");
  if (rows == 0) return HK_OK;
  const bool tc = !portable_only && moe_sm100_supported(num_experts, hidden, inter) && rows < (1ll << 31);
  const size_t need = tc ? moe_full_workspace(rows, hidden, inter) : moe_portable_workspace(rows, inter);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(HK_ESPACE, "hk_moe_grouped: workspace of %zu bytes, %zu needed", workspace_bytes, need);
  HK_REQUIRE((uintptr_t)workspace % 256 == 0, "hk_moe_grouped: workspace must be 256-byte aligned");
  uint8_t* base = reinterpret_cast<uint8_t*>(workspace);
  MoeScratch ws{};
  ws.hq = base;
  ws.hs = reinterpret_cast<float*>(base + align256((size_t)rows * inter));
  int32_t* tiles = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(ws.hs) +
                                              align256((size_t)rows * (inter / 128) * sizeof(float)));
  ws.max_tiles = (int32_t)(rows / kTileRows + kMaxExperts + 1);
  ws.tile_expert = tiles;
  ws.tile_row = tiles + ws.max_tiles;
  ws.num_tiles = tiles + 2 * ws.max_tiles;
  ws.xp = base + moe_portable_workspace(rows, inter);
  ws.sxp = reinterpret_cast<float*>(ws.xp + align256((size_t)rows * hidden));
  if (tc) {
    int32_t* list = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(ws.sxp) +
                                               align256((size_t)rows * (hidden / 128) * sizeof(float)));
    ws.max_tc = (int32_t)(rows / hk::moe_tile_width(0) + kMaxExperts + 1);
    ws.tc_expert = list;
    ws.tc_row = list + ws.max_tc;
    ws.tc_num = list + 2 * ws.max_tc;
    // The widths the device may choose: a width whose threshold the call's rows per expert
    // cannot reach (rows / num_experts bounds the average) is not launched; 96-row tiles also
    // need more than 64 tokens (hk_permute gives an expert each token once).  A decode batch
    // launches the 16-row kernel alone.
    int widths = 1;
    for (int i = 1; i < 4; ++i)
      if (rows >= (int64_t)hk::moe_tile_min_avg(i) * num_experts && (i < 3 || tokens > 64)) widths |= 1 << i;
    tc_list_kernel<<<1, 32, 0, s>>>(offsets, num_experts, rows, widths, ws.max_tc, ws.tc_expert, ws.tc_row,
                                    ws.tc_num, err);
    HK_TRY_LAUNCH("tc_list_kernel");
    return moe_sm100_run(xq, sx, tokens, offsets, perm_token, rows, num_experts, hidden, inter, w13, s13, w2,
                         s2, y, ws, widths, err, s);
  }
  tile_list_kernel<<<1, 32, 0, s>>>(offsets, num_experts, rows, ws.max_tiles, ws.tile_expert, ws.tile_row,
                                    ws.num_tiles, err);
  HK_TRY_LAUNCH("tile_list_kernel");
  moe_up_kernel<<<dim3(ws.max_tiles, inter / 128), 256, 0, s>>>(
      xq, sx, offsets, perm_token, ws.tile_expert, ws.tile_row, ws.num_tiles, hidden, inter, tokens, w13, s13,
      ws.hq, ws.hs, err);
  HK_TRY_LAUNCH("moe_up_kernel");
  moe_down_kernel<<<dim3(ws.max_tiles, hidden / 64), 256, 0, s>>>(
      ws.hq, ws.hs, offsets, ws.tile_expert, ws.tile_row, ws.num_tiles, hidden, inter, w2, s2, y);
  HK_TRY_LAUNCH("moe_down_kernel");
  return HK_OK;
}

}  // namespace hk

extern "C" {

int hk_route(const float* logits, const float* bias, int32_t tokens, int32_t num_experts,
             int32_t top_k, float route_scale, int32_t* ids, float* weights, void* stream) {
  HK_TRY(hk::ensure_device());
  HK_REQUIRE(tokens == 0 || (logits && ids && weights), "hk_route: null pointer");
  HK_REQUIRE(num_experts > 0 && num_experts <= 256 && top_k > 0 && top_k <= 16 && top_k <= num_experts,
             "hk_route: %d experts, top %d (at most 256 experts, top 16)", num_experts, top_k);
  HK_REQUIRE(tokens >= 0, "hk_route: negative token count");
  if (tokens == 0) return HK_OK;
  const int64_t threads = (int64_t)tokens * 32;
  route_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, (cudaStream_t)stream>>>(
      logits, bias, tokens, num_experts, top_k, route_scale, ids, weights, hk::err_word());
  HK_TRY_LAUNCH("route_kernel");
  return HK_OK;
}

int hk_permute(const int32_t* ids, const float* weights, int32_t tokens, int32_t top_k,
               int32_t num_experts, int32_t* offsets, int32_t* perm_token, float* perm_weight,
               int32_t* inv, void* stream) {
  HK_TRY(hk::ensure_device());
  HK_REQUIRE(offsets && (tokens == 0 || (ids && weights && perm_token && perm_weight && inv)),
             "hk_permute: null pointer");
  HK_REQUIRE(num_experts > 0 && num_experts <= kMaxExperts && top_k > 0 && tokens >= 0,
             "hk_permute: %d experts (at most %d), top %d", num_experts, kMaxExperts, top_k);
  const size_t smem = sizeof(int) * (size_t)num_experts * 34;
  HK_TRY_CUDA(cudaFuncSetAttribute(permute_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  permute_kernel<<<1, kPermThreads, smem, (cudaStream_t)stream>>>(
      ids, weights, tokens, top_k, num_experts, offsets, perm_token, perm_weight, inv, hk::err_word());
  HK_TRY_LAUNCH("permute_kernel");
  return HK_OK;
}

size_t hk_moe_workspace_size(int64_t rows, int32_t hidden, int32_t inter) {
  if (rows <= 0 || hidden <= 0 || inter <= 0) return 0;
  return hk::moe_full_workspace(rows, hidden, inter);
}

int hk_moe_grouped(const uint8_t* xq, const float* sx, int32_t tokens, const int32_t* offsets,
                   const int32_t* perm_token, int64_t rows, int32_t num_experts, int32_t hidden,
                   int32_t inter, const uint8_t* w13, const float* s13, const uint8_t* w2,
                   const float* s2, uint16_t* y, void* workspace, size_t workspace_bytes,
                   void* stream) {
  return hk::moe_grouped_run(xq, sx, tokens, offsets, perm_token, rows, num_experts, hidden, inter,
                             w13, s13, w2, s2, y, workspace, workspace_bytes, false, hk::err_word(),
                             (cudaStream_t)stream);
}

int hk_combine(const uint16_t* y, int64_t rows, const float* perm_weight, const int32_t* inv,
               const uint16_t* shared, int32_t tokens, int32_t top_k, int32_t hidden,
               uint16_t* out, void* stream) {
  HK_TRY(hk::ensure_device());
  HK_REQUIRE(tokens == 0 || (y && perm_weight && inv && out), "hk_combine: null pointer");
  HK_REQUIRE(top_k > 0 && top_k <= 16 && hidden > 0 && hidden % 8 == 0 && tokens >= 0,
             "hk_combine: top %d, hidden %d", top_k, hidden);
  HK_REQUIRE(((uintptr_t)y | (uintptr_t)out | (uintptr_t)shared) % 16 == 0,
             "hk_combine: buffers must be 16-byte aligned");
  if (tokens == 0) return HK_OK;
  combine_kernel<<<tokens, 256, 0, (cudaStream_t)stream>>>(
      (const uint4*)y, rows, perm_weight, inv, (const uint4*)shared, top_k, hidden / 8,
      (uint4*)out, hk::err_word());
  HK_TRY_LAUNCH("combine_kernel");
  return HK_OK;
}

}  // extern "C"
