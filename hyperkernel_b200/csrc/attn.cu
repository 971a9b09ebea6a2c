// a9 / a10: ragged paged decode attention on CUDA cores (the portable kernels) and the
// log-sum-exp merge of split-KV partials.
//
//  * GQA fp32 (config 1): one CTA per (query row, KV head), one warp per query head of
//    the group; lanes split head_dim, online softmax in fp32.
//  * MLA (configs 2 and 5, any head count that is a multiple of 16): one CTA per
//    (query row, KV split, block of 16 heads).  A tile of 32 latent rows is staged in
//    shared memory as fp32 (a page-blocked bf16 cache, or a row-major e4m3 cache times its
//    per-row scale), scores use all 576 dims, values the first 512.  Partials of every split go to fp32 scratch and hk_lse_merge-style
//    merging produces the output.  The tcgen05 kernel (attn_mla_sm100.cu) replaces this
//    one for 128-head decode; this one stays for other head counts, the fp8 cache and
//    the context-parallel shard partials.
#include <math.h>

#include "attn.cuh"
#include "common.cuh"

namespace {

constexpr int kMlaDim = 576;   // 512 latent + 64 rope
constexpr int kMlaDv = 512;    // value dims
constexpr int kHeadBlock = 16; // heads per CTA
constexpr int kTile = 32;      // KV rows per smem tile
constexpr int kRowPad = 580;   // fp32 row stride in smem (4-word bank offset per row)
constexpr int kMlaThreads = 256;

__device__ __forceinline__ int lane_of_token(const int32_t* __restrict__ cu, int num_lanes, int t) {
  int lo = 0, hi = num_lanes;  // largest b with cu[b] <= t
  while (hi - lo > 1) {
    int mid = (lo + hi) >> 1;
    if (cu[mid] <= t) lo = mid; else hi = mid;
  }
  return lo;
}

// ---------------------------------------------------------------------------------------
// GQA fp32
// ---------------------------------------------------------------------------------------
template <int kPerLane>
__global__ void gqa_decode_kernel(const float* __restrict__ q, const float* __restrict__ kc,
                                  const float* __restrict__ vc, const int32_t* __restrict__ bt,
                                  int32_t bt_stride, const int32_t* __restrict__ cu,
                                  const int32_t* __restrict__ positions, int32_t num_lanes,
                                  int32_t q_heads, int32_t kv_heads, int32_t page_size,
                                  int64_t num_slots, float scale, float* __restrict__ out,
                                  float* __restrict__ lse, unsigned long long* err) {
  const int t = blockIdx.x, g = blockIdx.y;
  const int group = q_heads / kv_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp >= group) return;
  const int D = kPerLane * 32;
  const int h = g * group + warp;
  const int b = lane_of_token(cu, num_lanes, t);
  const int pos = positions[t];
  float qv[kPerLane], acc[kPerLane];
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) {
    qv[i] = q[((int64_t)t * q_heads + h) * D + lane + 32 * i];
    acc[i] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  for (int p = 0; p <= pos; ++p) {
    const int blk = p / page_size;
    const int page = blk < bt_stride ? bt[(int64_t)b * bt_stride + blk] : -1;
    const int64_t slot = (int64_t)page * page_size + p % page_size;
    if (page <= 0 || slot >= num_slots) {
      if (lane == 0) hk_flag(err, hk::kErrAttnPage, (unsigned)b);
      continue;
    }
    const float* krow = kc + (slot * kv_heads + g) * D;
    const float* vrow = vc + (slot * kv_heads + g) * D;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) s = fmaf(qv[i], krow[lane + 32 * i], s);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    s *= scale;
    const float m_new = fmaxf(m, s);
    const float corr = expf(m - m_new);
    const float w = expf(s - m_new);
    l = l * corr + w;
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) acc[i] = fmaf(w, vrow[lane + 32 * i], acc[i] * corr);
    m = m_new;
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
  for (int i = 0; i < kPerLane; ++i) out[((int64_t)t * q_heads + h) * D + lane + 32 * i] = acc[i] * inv;
  if (lane == 0) lse[(int64_t)t * q_heads + h] = l > 0.f ? m + logf(l) : -INFINITY;
}

// ---------------------------------------------------------------------------------------
// MLA portable
// ---------------------------------------------------------------------------------------
struct MlaArgs {
  const uint16_t* q;        // [T][heads][576] bf16
  const uint16_t* kv_bf16;  // [slots][576] bf16, or
  const uint8_t* kv_fp8;    // [slots][576] e4m3 with kv_scale[slots]
  const float* kv_scale;
  const int32_t* bt;
  int32_t bt_stride;
  const int32_t* cu;
  const int32_t* positions;
  const int32_t* kv_begin;  // optional shard range per lane (CP partials)
  const int32_t* kv_end;
  int32_t num_lanes, num_tokens, heads, page_size;
  int64_t num_slots;
  float scale;
  int32_t split_len, n_splits;
  uint16_t* out;   // final bf16 output when n_splits == 1 and out != null
  float* lse;      // final lse (with out)
  float* part_o;   // [n_splits][T*heads][512] fp32 partials (normalised)
  float* part_lse; // [n_splits][T*heads]
  unsigned long long* err;
};

template <bool kFp8>
__global__ void __launch_bounds__(kMlaThreads) mla_portable_kernel(MlaArgs a) {
  extern __shared__ float smem[];
  float* q_s = smem;                                // [16][576]
  float* k_s = q_s + kHeadBlock * kMlaDim;          // [32][580]
  float* p_s = k_s + kTile * kRowPad;               // [16][32]
  float* c_s = p_s + kHeadBlock * kTile;            // [16] rescale factors
  __shared__ int page_s[kTile];

  const int t = blockIdx.x, split = blockIdx.y, h0 = blockIdx.z * kHeadBlock;
  const int tid = threadIdx.x;
  const int b = lane_of_token(a.cu, a.num_lanes, t);
  const int pos = a.positions[t];
  int range_lo = 0, range_hi = pos + 1;
  if (a.kv_begin != nullptr) {
    range_lo = max(0, a.kv_begin[b]);
    range_hi = min(range_hi, a.kv_end[b]);
  }
  const int lo = range_lo + split * a.split_len;
  const int hi = min(lo + a.split_len, range_hi);
  const int64_t row0 = (int64_t)t * a.heads + h0;

  for (int i = tid; i < kHeadBlock * kMlaDim; i += kMlaThreads) {
    const int h = i / kMlaDim, d = i % kMlaDim;
    q_s[i] = bf16_bits_to_f32(a.q[(row0 + h) * kMlaDim + d]);
  }

  // Score role: head sh, tokens sj and sj + 16.  Value role: dims 2*tid, 2*tid+1.
  const int sh = tid >> 4, sj = tid & 15;
  float m = -INFINITY, l = 0.f;  // running stats of head sh (replicated in its 16 threads)
  float acc[kHeadBlock][2];
#pragma unroll
  for (int h = 0; h < kHeadBlock; ++h) acc[h][0] = acc[h][1] = 0.f;

  for (int base = lo; base < hi; base += kTile) {
    const int n = min(kTile, hi - base);
    __syncthreads();  // previous tile fully consumed (and q_s written on the first pass)
    if (tid < kTile) {
      int page = -1;
      if (tid < n) {
        const int p = base + tid, blk = p / a.page_size;
        page = blk < a.bt_stride ? a.bt[(int64_t)b * a.bt_stride + blk] : -1;
        const int64_t slot = (int64_t)page * a.page_size + p % a.page_size;
        if (page <= 0 || slot >= a.num_slots) {  // page 0 is the scratch page: never read
          hk_flag(a.err, hk::kErrAttnPage, (unsigned)b);
          page = -1;
        }
      }
      page_s[tid] = page;
    }
    __syncthreads();
    // Stage rows: 72 16-byte vectors per bf16 row, 36 per e4m3 row.
    if (!kFp8) {
      for (int i = tid; i < kTile * 72; i += kMlaThreads) {
        const int j = i / 72, v = i % 72;
        float* dst = k_s + j * kRowPad + v * 8;
        const int page = page_s[j];
        if (j < n && page >= 0) {
          // page-blocked layout: block v / 8 of the page, row (pos % page_size), column v % 8
          const int64_t r = (base + j) % a.page_size;
          const uint4 u = reinterpret_cast<const uint4*>(
              a.kv_bf16 + (int64_t)page * a.page_size * kMlaDim)[(v >> 3) * a.page_size * 8 + r * 8 + (v & 7)];
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            dst[2 * e] = __uint_as_float(w[e] << 16);
            dst[2 * e + 1] = __uint_as_float(w[e] & 0xffff0000u);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) dst[e] = 0.f;
        }
      }
    } else {
      for (int i = tid; i < kTile * 36; i += kMlaThreads) {
        const int j = i / 36, v = i % 36;
        float* dst = k_s + j * kRowPad + v * 16;
        const int page = page_s[j];
        if (j < n && page >= 0) {
          const int64_t slot = (int64_t)page * a.page_size + (base + j) % a.page_size;
          const float sc = a.kv_scale[slot];
          const uint4 u = reinterpret_cast<const uint4*>(a.kv_fp8 + slot * kMlaDim)[v];
          const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
          for (int e = 0; e < 16; ++e) dst[e] = e4m3_to_f32((uint8_t)(w[e >> 2] >> (8 * (e & 3)))) * sc;
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) dst[e] = 0.f;
        }
      }
    }
    __syncthreads();
    // Scores.
    float s0 = 0.f, s1 = 0.f;
    {
      const float4* qr = reinterpret_cast<const float4*>(q_s + sh * kMlaDim);
      const float4* k0 = reinterpret_cast<const float4*>(k_s + sj * kRowPad);
      const float4* k1 = reinterpret_cast<const float4*>(k_s + (sj + 16) * kRowPad);
#pragma unroll 4
      for (int d = 0; d < kMlaDim / 4; ++d) {
        const float4 x = qr[d], y0 = k0[d], y1 = k1[d];
        s0 = fmaf(x.x, y0.x, s0); s0 = fmaf(x.y, y0.y, s0); s0 = fmaf(x.z, y0.z, s0); s0 = fmaf(x.w, y0.w, s0);
        s1 = fmaf(x.x, y1.x, s1); s1 = fmaf(x.y, y1.y, s1); s1 = fmaf(x.z, y1.z, s1); s1 = fmaf(x.w, y1.w, s1);
      }
    }
    s0 = (sj < n && page_s[sj] >= 0) ? s0 * a.scale : -INFINITY;
    s1 = (sj + 16 < n && page_s[sj + 16] >= 0) ? s1 * a.scale : -INFINITY;
    float tmax = fmaxf(s0, s1);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
    const float m_new = fmaxf(m, tmax);
    const float corr = (m_new == -INFINITY) ? 1.f : expf(m - m_new);
    const float p0 = (s0 == -INFINITY) ? 0.f : expf(s0 - m_new);
    const float p1 = (s1 == -INFINITY) ? 0.f : expf(s1 - m_new);
    float psum = p0 + p1;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
    l = l * corr + psum;
    m = m_new;
    p_s[sh * kTile + sj] = p0;
    p_s[sh * kTile + sj + 16] = p1;
    if (sj == 0) c_s[sh] = corr;
    __syncthreads();
    // Values.
#pragma unroll
    for (int h = 0; h < kHeadBlock; ++h) {
      const float c = c_s[h];
      acc[h][0] *= c;
      acc[h][1] *= c;
    }
    for (int j = 0; j < n; ++j) {
      const float2 v = *reinterpret_cast<const float2*>(k_s + j * kRowPad + 2 * tid);
#pragma unroll
      for (int h = 0; h < kHeadBlock; ++h) {
        const float p = p_s[h * kTile + j];
        acc[h][0] = fmaf(p, v.x, acc[h][0]);
        acc[h][1] = fmaf(p, v.y, acc[h][1]);
      }
    }
  }
  // Publish the per-head l, m so every thread can normalise its dims.
  __syncthreads();
  if (sj == 0) {
    p_s[sh] = l;
    p_s[kHeadBlock + sh] = m;
  }
  __syncthreads();
  const bool final_out = a.out != nullptr;
#pragma unroll
  for (int h = 0; h < kHeadBlock; ++h) {
    const float lh = p_s[h], mh = p_s[kHeadBlock + h];
    const float inv = lh > 0.f ? 1.f / lh : 0.f;
    const int64_t row = row0 + h;
    if (final_out) {
      const uint32_t packed = (uint32_t)f32_to_bf16_bits(acc[h][0] * inv) |
                              ((uint32_t)f32_to_bf16_bits(acc[h][1] * inv) << 16);
      reinterpret_cast<uint32_t*>(a.out + row * kMlaDv)[tid] = packed;
      if (tid == 0) a.lse[row] = lh > 0.f ? mh + logf(lh) : -INFINITY;
    } else {
      const int64_t rows = (int64_t)a.num_tokens * a.heads;
      float* o = a.part_o + ((int64_t)split * rows + row) * kMlaDv;
      reinterpret_cast<float2*>(o)[tid] = make_float2(acc[h][0] * inv, acc[h][1] * inv);
      if (tid == 0) a.part_lse[(int64_t)split * rows + row] = lh > 0.f ? mh + logf(lh) : -INFINITY;
    }
  }
}

// ---------------------------------------------------------------------------------------
// LSE merge: one CTA of dv/4 threads per row, float4 per thread.
// ---------------------------------------------------------------------------------------
template <bool kBf16Out>
__global__ void lse_merge_kernel(const float* __restrict__ o_parts, const float* __restrict__ lse_parts,
                                 int32_t n_parts, int64_t rows, int32_t dv, void* __restrict__ out,
                                 float* __restrict__ lse_out) {
  const int64_t r = blockIdx.x;
  __shared__ float w_s[256];
  __shared__ float stat[2];
  if (threadIdx.x == 0) {
    float m = -INFINITY;
    for (int p = 0; p < n_parts; ++p) m = fmaxf(m, lse_parts[(int64_t)p * rows + r]);
    float sum = 0.f;
    for (int p = 0; p < n_parts; ++p) {
      const float lp = lse_parts[(int64_t)p * rows + r];
      const float w = (lp == -INFINITY) ? 0.f : expf(lp - m);
      w_s[p] = w;
      sum += w;
    }
    stat[0] = sum;
    stat[1] = m;
  }
  __syncthreads();
  const float sum = stat[0], inv = sum > 0.f ? 1.f / sum : 0.f;
  for (int d4 = threadIdx.x; d4 < dv / 4; d4 += blockDim.x) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p = 0; p < n_parts; ++p) {
      const float w = w_s[p];
      if (w == 0.f) continue;
      const float4 o = reinterpret_cast<const float4*>(o_parts + ((int64_t)p * rows + r) * dv)[d4];
      acc.x = fmaf(w, o.x, acc.x);
      acc.y = fmaf(w, o.y, acc.y);
      acc.z = fmaf(w, o.z, acc.z);
      acc.w = fmaf(w, o.w, acc.w);
    }
    acc.x *= inv; acc.y *= inv; acc.z *= inv; acc.w *= inv;
    if (kBf16Out) {
      uint2 pk;
      pk.x = (uint32_t)f32_to_bf16_bits(acc.x) | ((uint32_t)f32_to_bf16_bits(acc.y) << 16);
      pk.y = (uint32_t)f32_to_bf16_bits(acc.z) | ((uint32_t)f32_to_bf16_bits(acc.w) << 16);
      reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(out) + r * dv)[d4] = pk;
    } else {
      reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + r * dv)[d4] = acc;
    }
  }
  if (threadIdx.x == 0 && lse_out != nullptr) lse_out[r] = sum > 0.f ? stat[1] + logf(sum) : -INFINITY;
}

constexpr int kPortableSplit = 4096;
constexpr int kMaxSplits = 64;

int portable_splits(int32_t max_kv_len, int32_t* split_len) {
  int n = (max_kv_len + kPortableSplit - 1) / kPortableSplit;
  if (n < 1) n = 1;
  int len = kPortableSplit;
  if (n > kMaxSplits) {
    len = ((max_kv_len + kMaxSplits - 1) / kMaxSplits + kTile - 1) / kTile * kTile;
    n = (max_kv_len + len - 1) / len;
  }
  *split_len = len;
  return n;
}

size_t mla_smem_bytes() {
  return sizeof(float) * (kHeadBlock * kMlaDim + kTile * kRowPad + kHeadBlock * kTile + kHeadBlock);
}

int launch_mla_portable(MlaArgs a, bool fp8, cudaStream_t stream) {
  const size_t smem = mla_smem_bytes();
  dim3 grid(a.num_tokens, a.n_splits, a.heads / kHeadBlock);
  if (fp8) {
    HK_TRY_CUDA(cudaFuncSetAttribute(mla_portable_kernel<true>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    mla_portable_kernel<true><<<grid, kMlaThreads, smem, stream>>>(a);
  } else {
    HK_TRY_CUDA(cudaFuncSetAttribute(mla_portable_kernel<false>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    mla_portable_kernel<false><<<grid, kMlaThreads, smem, stream>>>(a);
  }
  HK_TRY_LAUNCH("mla_portable_kernel");
  return HK_OK;
}

}  // namespace

namespace hk {

int lse_merge_launch(const float* o_parts, const float* lse_parts, int32_t n_parts, int64_t rows,
                     int32_t dv, void* out, bool bf16_out, float* lse_out, cudaStream_t stream) {
  if (rows == 0) return HK_OK;
  const int threads = dv / 4 < 128 ? dv / 4 : 128;
  if (bf16_out)
    lse_merge_kernel<true><<<(unsigned)rows, threads, 0, stream>>>(o_parts, lse_parts, n_parts, rows, dv, out, lse_out);
  else
    lse_merge_kernel<false><<<(unsigned)rows, threads, 0, stream>>>(o_parts, lse_parts, n_parts, rows, dv, out, lse_out);
  HK_TRY_LAUNCH("lse_merge_kernel");
  return HK_OK;
}

size_t mla_portable_workspace(int32_t num_tokens, int32_t heads, int32_t max_kv_len) {
  int32_t len;
  const int n = portable_splits(max_kv_len, &len);
  if (n <= 1) return 0;
  return (size_t)n * num_tokens * heads * (kMlaDv + 1) * sizeof(float) + 256;
}

int mla_portable(const uint16_t* q, const uint16_t* kv_bf16, const uint8_t* kv_fp8,
                 const float* kv_scale, const int32_t* bt, int32_t bt_stride, const int32_t* cu,
                 const int32_t* positions, int32_t num_lanes, int32_t num_tokens, int32_t heads,
                 int32_t page_size, int64_t num_slots, int32_t max_kv_len, float scale,
                 uint16_t* out, float* lse, void* workspace, size_t workspace_bytes,
                 cudaStream_t stream) {
  MlaArgs a = {};
  a.q = q; a.kv_bf16 = kv_bf16; a.kv_fp8 = kv_fp8; a.kv_scale = kv_scale;
  a.bt = bt; a.bt_stride = bt_stride; a.cu = cu; a.positions = positions;
  a.num_lanes = num_lanes; a.num_tokens = num_tokens; a.heads = heads; a.page_size = page_size;
  a.num_slots = num_slots; a.scale = scale; a.err = err_word();
  a.n_splits = portable_splits(max_kv_len, &a.split_len);
  const int64_t rows = (int64_t)num_tokens * heads;
  if (a.n_splits == 1) {
    a.out = out;
    a.lse = lse;
    return launch_mla_portable(a, kv_fp8 != nullptr, stream);
  }
  const size_t need = mla_portable_workspace(num_tokens, heads, max_kv_len);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(HK_ESPACE, "mla: workspace of %zu bytes, %zu needed", workspace_bytes, need);
  a.part_o = reinterpret_cast<float*>(workspace);
  a.part_lse = a.part_o + (size_t)a.n_splits * rows * kMlaDv;
  HK_TRY(launch_mla_portable(a, kv_fp8 != nullptr, stream));
  return lse_merge_launch(a.part_o, a.part_lse, a.n_splits, rows, kMlaDv, out, true, lse, stream);
}

int mla_portable_partial(const uint16_t* q, const uint8_t* kv_fp8, const float* kv_scale,
                         const int32_t* bt, int32_t bt_stride, const int32_t* cu,
                         const int32_t* positions, const int32_t* kv_begin, const int32_t* kv_end,
                         int32_t num_lanes, int32_t num_tokens, int32_t heads, int32_t page_size,
                         int64_t num_slots, int32_t max_kv_len, float scale, float* o_part,
                         float* lse_part, void* workspace, size_t workspace_bytes,
                         cudaStream_t stream) {
  MlaArgs a = {};
  a.q = q; a.kv_fp8 = kv_fp8; a.kv_scale = kv_scale;
  a.bt = bt; a.bt_stride = bt_stride; a.cu = cu; a.positions = positions;
  a.kv_begin = kv_begin; a.kv_end = kv_end;
  a.num_lanes = num_lanes; a.num_tokens = num_tokens; a.heads = heads; a.page_size = page_size;
  a.num_slots = num_slots; a.scale = scale; a.err = err_word();
  a.n_splits = portable_splits(max_kv_len, &a.split_len);
  const int64_t rows = (int64_t)num_tokens * heads;
  if (a.n_splits == 1) {
    a.part_o = o_part;
    a.part_lse = lse_part;
    return launch_mla_portable(a, true, stream);
  }
  const size_t need = mla_portable_workspace(num_tokens, heads, max_kv_len);
  if (workspace == nullptr || workspace_bytes < need)
    return fail(HK_ESPACE, "mla partial: workspace of %zu bytes, %zu needed", workspace_bytes, need);
  a.part_o = reinterpret_cast<float*>(workspace);
  a.part_lse = a.part_o + (size_t)a.n_splits * rows * kMlaDv;
  HK_TRY(launch_mla_portable(a, true, stream));
  return lse_merge_launch(a.part_o, a.part_lse, a.n_splits, rows, kMlaDv, o_part, false, lse_part,
                          stream);
}

}  // namespace hk

extern "C" {

int hk_gqa_decode_f32(const float* q, const float* k_cache, const float* v_cache,
                      const int32_t* block_table, int32_t bt_stride, const int32_t* cu_seqlens,
                      const int32_t* positions, int32_t num_lanes, int32_t num_tokens,
                      int32_t q_heads, int32_t kv_heads, int32_t head_dim, int32_t page_size,
                      int64_t num_slots, float scale, float* out, float* lse, void* stream) {
  HK_TRY(hk::ensure_device());
  HK_REQUIRE(num_tokens == 0 ||
                 (q && k_cache && v_cache && block_table && cu_seqlens && positions && out && lse),
             "hk_gqa_decode_f32: null pointer");
  HK_REQUIRE(kv_heads > 0 && q_heads % kv_heads == 0 && q_heads / kv_heads <= 32,
             "hk_gqa_decode_f32: %d query heads over %d KV heads", q_heads, kv_heads);
  HK_REQUIRE(head_dim == 32 || head_dim == 64 || head_dim == 128 || head_dim == 256,
             "hk_gqa_decode_f32: head_dim %d not in {32, 64, 128, 256}", head_dim);
  HK_REQUIRE(num_lanes > 0 && num_tokens >= 0 && page_size > 0 && bt_stride > 0,
             "hk_gqa_decode_f32: bad sizes");
  HK_REQUIRE(num_slots > 0, "hk_gqa_decode_f32: empty cache");
  if (num_tokens == 0) return HK_OK;
  dim3 grid(num_tokens, kv_heads);
  const int threads = 32 * (q_heads / kv_heads);
  cudaStream_t s = (cudaStream_t)stream;
  unsigned long long* err = hk::err_word();
#define HK_GQA_CASE(P)                                                                       \
  gqa_decode_kernel<P><<<grid, threads, 0, s>>>(q, k_cache, v_cache, block_table, bt_stride,  \
                                                cu_seqlens, positions, num_lanes, q_heads,    \
                                                kv_heads, page_size, num_slots, scale, out,   \
                                                lse, err)
  switch (head_dim) {
    case 32: HK_GQA_CASE(1); break;
    case 64: HK_GQA_CASE(2); break;
    case 128: HK_GQA_CASE(4); break;
    default: HK_GQA_CASE(8); break;
  }
#undef HK_GQA_CASE
  HK_TRY_LAUNCH("gqa_decode_kernel");
  return HK_OK;
}

int hk_lse_merge(const float* o_parts, const float* lse_parts, int32_t n_parts, int64_t rows,
                 int32_t dv, uint16_t* out, float* lse_out, void* stream) {
  HK_TRY(hk::ensure_device());
  HK_REQUIRE(rows == 0 || (o_parts && lse_parts && out), "hk_lse_merge: null pointer");
  HK_REQUIRE(n_parts >= 1 && n_parts <= 256 && rows >= 0 && dv > 0 && dv % 4 == 0,
             "hk_lse_merge: %d parts of dv %d (1..256 parts, dv a multiple of 4)", n_parts, dv);
  HK_REQUIRE(((uintptr_t)o_parts % 16 == 0) && ((uintptr_t)out % 8 == 0),
             "hk_lse_merge: misaligned buffers");
  return hk::lse_merge_launch(o_parts, lse_parts, n_parts, rows, dv, out, true, lse_out,
                              (cudaStream_t)stream);
}

int hk_mla_decode_fp8(const uint16_t* q, const uint8_t* kv_cache, const float* kv_scale,
                      const int32_t* block_table, int32_t bt_stride, const int32_t* cu_seqlens,
                      const int32_t* positions, int32_t num_lanes, int32_t num_tokens,
                      int32_t heads, int32_t page_size, int64_t num_slots, int32_t max_kv_len,
                      float scale, uint16_t* out, float* lse, void* workspace,
                      size_t workspace_bytes, void* stream) {
  HK_TRY(hk::ensure_device());
  HK_REQUIRE(num_tokens == 0 ||
                 (q && kv_cache && kv_scale && block_table && cu_seqlens && positions && out && lse),
             "hk_mla_decode_fp8: null pointer");
  HK_REQUIRE(heads > 0 && heads % kHeadBlock == 0, "hk_mla_decode_fp8: heads %d not a multiple of 16", heads);
  HK_REQUIRE(num_lanes > 0 && num_tokens >= 0 && page_size > 0 && bt_stride > 0 && max_kv_len >= 0,
             "hk_mla_decode_fp8: bad sizes");
  HK_REQUIRE((uintptr_t)kv_cache % 16 == 0, "hk_mla_decode_fp8: cache must be 16-byte aligned");
  if (num_tokens == 0) return HK_OK;
  return hk::mla_portable(q, nullptr, kv_cache, kv_scale, block_table, bt_stride, cu_seqlens,
                          positions, num_lanes, num_tokens, heads, page_size, num_slots,
                          max_kv_len, scale, out, lse, workspace, workspace_bytes,
                          (cudaStream_t)stream);
}

int hk_mla_partial_fp8(const uint16_t* q, const uint8_t* kv_cache, const float* kv_scale,
                       const int32_t* block_table, int32_t bt_stride, const int32_t* cu_seqlens,
                       const int32_t* positions, const int32_t* kv_begin, const int32_t* kv_end,
                       int32_t num_lanes, int32_t num_tokens, int32_t heads, int32_t page_size,
                       int64_t num_slots, int32_t max_kv_len, float scale, float* o_part,
                       float* lse_part, void* workspace, size_t workspace_bytes, void* stream) {
  HK_TRY(hk::ensure_device());
  HK_REQUIRE(num_tokens == 0 || (q && kv_cache && kv_scale && block_table && cu_seqlens && positions &&
                                  kv_begin && kv_end && o_part && lse_part),
             "hk_mla_partial_fp8: null pointer");
  HK_REQUIRE(heads > 0 && heads % kHeadBlock == 0, "hk_mla_partial_fp8: heads %d not a multiple of 16", heads);
  HK_REQUIRE(num_lanes > 0 && num_tokens >= 0 && page_size > 0 && bt_stride > 0,
             "hk_mla_partial_fp8: bad sizes");
  if (num_tokens == 0) return HK_OK;
  return hk::mla_portable_partial(q, kv_cache, kv_scale, block_table, bt_stride, cu_seqlens,
                                  positions, kv_begin, kv_end, num_lanes, num_tokens, heads,
                                  page_size, num_slots, max_kv_len, scale, o_part, lse_part,
                                  workspace, workspace_bytes, (cudaStream_t)stream);
}

}  // extern "C"
