// HK_MODEL_MLA: a DeepSeek-shaped decoder behind the Kernel boundary (hk_open_mla), built from
// this library's kernels.  The layer math is stated in include/hk.h (hk_mla_model).
//
// One forward pass takes the rows of a packed batch (hk_pack over the lanes' block-table rows):
//   embed -> per layer [rmsnorm+quant -> q_a, kv_a GEMMs -> rmsnorm+quant -> q_b GEMM ->
//   RoPE + latent norm -> KV append -> tcgen05 MLA attention -> quant -> o GEMM ->
//   residual + rmsnorm + quant -> router GEMM -> route -> permute -> grouped expert FFN +
//   shared expert -> combine] -> residual + rmsnorm + quant of the sampled rows -> vocabulary
//   GEMM -> hk_sample_verify.
// The small fused kernels here are the glue between those entry points: the embedding gather,
// the residual add fused with the RMS norm and the 1x128 e4m3 quantisation of the next
// projection's input, RoPE fused with the latent norm, and the decode step's prepare (the
// lane's last token and its prompt-lookup drafts into the token stream and the token pool) and
// commit (the lane's last accepted token).
#include <math.h>
#include <string.h>

#include <algorithm>

#include "common.cuh"
#include "model.cuh"

namespace hk {

namespace {

constexpr int kHeads = 128, kLatent = 512, kRope = 64, kRow = kLatent + kRope;  // 576
constexpr int kPage = 64;
constexpr int kLookback = 4096;  // positions the prompt-lookup drafter searches
// Fault sites of the device kernel's error words (the handle's, read by hk_drain).
constexpr unsigned kFaultScratchWrite = 1, kFaultPagePastPool = 7;

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// A standard normal value for element i of a seeded tensor (Box-Muller over one 64-bit hash).
__device__ __forceinline__ float gauss(uint64_t seed, uint64_t i) {
  const uint64_t r = mix64(seed + (i + 1) * 0x9E3779B97F4A7C15ull);
  const float u1 = ((float)(uint32_t)(r >> 40) + 0.5f) * (1.0f / 16777216.0f);
  const float u2 = (float)(uint32_t)(r & 0xFFFFFFu) * (1.0f / 16777216.0f);
  return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

// e4m3 weights of N(0, sigma) values: q = e4m3(z * 112), scale = sigma / 112 (|z| = 4 maps to 448).
__global__ void gen_e4m3_kernel(uint8_t* w, int64_t n, uint64_t seed) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    w[i] = f32_to_e4m3(gauss(seed, (uint64_t)i) * 112.0f);
}

__global__ void gen_bf16_kernel(uint16_t* w, int64_t n, uint64_t seed) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    w[i] = f32_to_bf16_bits(gauss(seed, (uint64_t)i));
}

__global__ void fill_f32_kernel(float* p, int64_t n, float v) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    p[i] = v;
}

// The shared expert as expert E of the routed grouped call: its rows are every token in order,
// appended after the T*K permuted rows (perm_token[T*K + i] = i, offsets[E+1] = T*K + T), so
// its weights stream in the same launch as the routed experts' instead of a launch of its own
// that a decode batch's one row tile would spread over a tenth of the SMs.
__global__ void shared_rows_kernel(int32_t* __restrict__ offsets, int32_t* __restrict__ perm_token, int32_t E,
                                   int32_t T, int32_t K) {
  const int64_t base = (int64_t)T * K;
  for (int32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < T; i += gridDim.x * blockDim.x)
    perm_token[base + i] = i;
  if (blockIdx.x == 0 && threadIdx.x == 0) offsets[E + 1] = (int32_t)(base + T);
}

__device__ __forceinline__ void unpack8(const uint4 u, float* v) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    v[2 * k] = __uint_as_float(w[k] << 16);
    v[2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
  }
}

__device__ __forceinline__ uint4 pack8(const float* v) {
  uint32_t w[4];
#pragma unroll
  for (int k = 0; k < 4; ++k)
    w[k] = (uint32_t)f32_to_bf16_bits(v[2 * k]) | ((uint32_t)f32_to_bf16_bits(v[2 * k + 1]) << 16);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

// x[r] = embed[tokens[r]] (bf16 rows of H); a token outside the vocabulary gives a zero row and
// sets the device error word.
__global__ void embed_kernel(const int32_t* __restrict__ tokens, int32_t rows, const uint16_t* __restrict__ table,
                             int32_t H, int32_t V, uint16_t* __restrict__ x, unsigned long long* err) {
  const int r = blockIdx.x;
  if (r >= rows) return;
  const int32_t t = tokens[r];
  const bool ok = t >= 0 && t < V;
  if (!ok && threadIdx.x == 0) hk_flag(err, kErrToken, (unsigned)r);
  const uint4* src = reinterpret_cast<const uint4*>(table + (int64_t)(ok ? t : 0) * H);
  uint4* dst = reinterpret_cast<uint4*>(x + (int64_t)r * H);
  for (int c = threadIdx.x; c < H / 8; c += blockDim.x) dst[c] = ok ? src[c] : make_uint4(0, 0, 0, 0);
}

constexpr int kNormThreads = 128;

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
  __syncthreads();
  return t;
}

// One CTA per output row r, reading input row i = idx ? idx[r] : r:
//   v = x[i] (+ add[i]); when x_out is given, x_out[i] = bf16(v) and v takes that bf16 value
//   (the residual stream is kept in bf16); n = v / sqrt(mean(v^2) + 1e-6);
//   per 128-element block: s = max(amax(n), 1e-12) / 448, q = e4m3(n / s) (hk_quant_fp8's rule).
// H is a multiple of 128, so every 128-element block is one half-warp's 16 x 8 elements.
__global__ void __launch_bounds__(kNormThreads)
    rms_quant_kernel(const uint16_t* x, const uint16_t* __restrict__ add, uint16_t* x_out,
                     const int32_t* __restrict__ idx, int32_t rows, int32_t H, uint8_t* __restrict__ q,
                     float* __restrict__ s) {
  __shared__ float red[kNormThreads / 32];
  const int r = blockIdx.x;
  if (r >= rows) return;
  const int64_t i = idx ? (int64_t)idx[r] : (int64_t)r;
  const int chunks = H / 8;
  const uint4* xr = reinterpret_cast<const uint4*>(x + i * H);
  const uint4* ar = add ? reinterpret_cast<const uint4*>(add + i * H) : nullptr;
  uint4* xo = x_out ? reinterpret_cast<uint4*>(x_out + i * H) : nullptr;
  float ss = 0.f;
  for (int c = threadIdx.x; c < chunks; c += blockDim.x) {
    float v[8];
    unpack8(xr[c], v);
    if (ar) {
      float a[8];
      unpack8(ar[c], a);
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] += a[k];
    }
    if (xo) {
      const uint4 p = pack8(v);
      xo[c] = p;
      unpack8(p, v);
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) ss += v[k] * v[k];
  }
  const float total = block_sum(ss, red);
  const float inv = 1.0f / sqrtf(total / (float)H + 1e-6f);
  const uint4* src = xo ? reinterpret_cast<const uint4*>(xo) : xr;  // this thread's own chunks
  uint8_t* qr = q + (int64_t)r * H;
  float* sr = s + (int64_t)r * (H / 128);
  for (int base = 0; base < chunks; base += blockDim.x) {
    const int c = base + threadIdx.x;
    const bool on = c < chunks;
    float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (on) {
      unpack8(src[c], v);
      if (ar && !xo) {
        float a[8];
        unpack8(ar[c], a);
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] += a[k];
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) v[k] *= inv;
    }
    float amax = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fabsf(v[k]));
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float sc = fmaxf(amax, 1e-12f) / 448.0f;
    if (on) {
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        lo |= (uint32_t)f32_to_e4m3(v[k] / sc) << (8 * k);
        hi |= (uint32_t)f32_to_e4m3(v[k + 4] / sc) << (8 * k);
      }
      reinterpret_cast<uint2*>(qr)[c] = make_uint2(lo, hi);
      if ((threadIdx.x & 15) == 0) sr[c / 16] = sc;
    }
  }
}

// One CTA (128 threads) per row t at position p: every head's 64 rope dims of q and the row's
// kv rope dims rotated (dim i with dim i + 32 by p * theta^(-i/32), the angle in double), and the
// kv row's 512 latent dims RMS-normalised (eps 1e-6).
__global__ void __launch_bounds__(128)
    rope_norm_kernel(uint16_t* __restrict__ q, uint16_t* __restrict__ kv, const int32_t* __restrict__ positions,
                     int32_t rows, float theta) {
  __shared__ float cs[32], sn[32];
  __shared__ float red[4];
  const int t = blockIdx.x;
  if (t >= rows) return;
  if (threadIdx.x < 32) {
    const double f = pow((double)theta, -(double)threadIdx.x / 32.0);
    double sv, cv;
    sincos((double)positions[t] * f, &sv, &cv);
    cs[threadIdx.x] = (float)cv;
    sn[threadIdx.x] = (float)sv;
  }
  __syncthreads();
  uint16_t* qt = q + (int64_t)t * kHeads * kRow;
  for (int j = threadIdx.x; j < kHeads * 32; j += blockDim.x) {
    const int h = j >> 5, d = j & 31;
    uint16_t* p = qt + h * kRow + kLatent;
    const float a = bf16_bits_to_f32(p[d]), b = bf16_bits_to_f32(p[d + 32]);
    p[d] = f32_to_bf16_bits(a * cs[d] - b * sn[d]);
    p[d + 32] = f32_to_bf16_bits(a * sn[d] + b * cs[d]);
  }
  uint16_t* kt = kv + (int64_t)t * kRow;
  float v[4];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    v[k] = bf16_bits_to_f32(kt[threadIdx.x * 4 + k]);
    ss += v[k] * v[k];
  }
  const float total = block_sum(ss, red);
  const float inv = 1.0f / sqrtf(total / (float)kLatent + 1e-6f);
#pragma unroll
  for (int k = 0; k < 4; ++k) kt[threadIdx.x * 4 + k] = f32_to_bf16_bits(v[k] * inv);
  if (threadIdx.x < 32) {
    const int d = threadIdx.x;
    uint16_t* p = kt + kLatent;
    const float a = bf16_bits_to_f32(p[d]), b = bf16_bits_to_f32(p[d + 32]);
    p[d] = f32_to_bf16_bits(a * cs[d] - b * sn[d]);
    p[d + 32] = f32_to_bf16_bits(a * sn[d] + b * cs[d]);
  }
}

__global__ void f32_of_bf16_kernel(const uint16_t* __restrict__ in, float* __restrict__ out, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = bf16_bits_to_f32(in[i]);
}

// The token pool through a lane's block-table row: index of position p, or -1 when p is past the
// row or its page is the scratch page or past the pool.
struct PoolView {
  const int32_t* rows;
  int32_t* pool;
  int32_t bt_stride, entries, page_rows;
  int64_t pages;
};

__device__ __forceinline__ int64_t pool_at(const PoolView& v, int lane, int64_t p, unsigned* why) {
  const int64_t k = p / v.page_rows;
  if (p < 0 || k >= v.entries) {
    *why = kFaultPagePastPool;
    return -1;
  }
  const int32_t page = v.rows[(int64_t)lane * v.bt_stride + k];
  if (page <= 0 || page >= v.pages) {
    *why = page == 0 ? kFaultScratchWrite : kFaultPagePastPool;
    return -1;
  }
  return (int64_t)page * v.page_rows + p % v.page_rows;
}

__device__ void record_fault(unsigned long long* err, unsigned site, int lane, long long pos) {
  const unsigned long long w = (1ull << 63) | ((unsigned long long)site << 32);
  if (atomicCAS(err, 0ull, w) == 0ull) {
    err[1] = (unsigned long long)lane;
    err[2] = (unsigned long long)pos;
  }
}

// The decode step's inputs, a warp per lane with rows: the lane's last token goes to the token
// pool at its position; prompt lookup finds the latest earlier occurrence of that token in the
// lane's last kLookback positions and proposes the tokens that followed it (-1 past the
// current position or without a match); the rows' input tokens are the last token then the
// drafts (0 in place of -1: such a row can never be accepted), and they are written to the pool
// at their positions (rows that are not accepted are overwritten by later steps).
__global__ void prepare_kernel(PoolView v, const int32_t* __restrict__ lane_tokens,
                               const int32_t* __restrict__ lane_pos, const int32_t* __restrict__ cu,
                               const int32_t* __restrict__ tok, int32_t width, int32_t block,
                               int32_t* __restrict__ tokens_in, int32_t* __restrict__ drafts,
                               unsigned long long* dev_err) {
  const int l = (int)((blockIdx.x * (int64_t)blockDim.x + threadIdx.x) >> 5);
  const int ln = threadIdx.x & 31;
  if (l >= width) return;
  const int rows = lane_tokens[l];
  int32_t* dr = drafts + (int64_t)l * (block > 1 ? block - 1 : 1);
  if (rows <= 0) {
    for (int j = ln; j < block - 1; j += 32) dr[j] = -1;
    return;
  }
  const int64_t pos = lane_pos[l];
  const int32_t t0 = tok[l];
  if (ln == 0) {
    unsigned why = 0;
    const int64_t at = pool_at(v, l, pos, &why);
    if (at < 0) record_fault(dev_err, why, l, pos);
    else v.pool[at] = t0;
  }
  __syncwarp();
  int64_t found = -1;
  if (block > 1) {
    const int64_t lo = pos - kLookback > 0 ? pos - kLookback : 0;
    for (int64_t top = pos - 1; top >= lo; top -= 32) {
      const int64_t p = top - ln;
      bool hit = false;
      if (p >= lo) {
        unsigned why = 0;
        const int64_t at = pool_at(v, l, p, &why);
        hit = at >= 0 && v.pool[at] == t0;
      }
      const unsigned m = __ballot_sync(0xffffffffu, hit);
      if (m) {
        found = top - (__ffs(m) - 1);
        break;
      }
    }
  }
  for (int j = ln; j < block - 1; j += 32) {
    int32_t d = -1;
    const int64_t p = found + 1 + j;
    if (found >= 0 && p <= pos) {
      unsigned why = 0;
      const int64_t at = pool_at(v, l, p, &why);
      if (at >= 0) d = v.pool[at];
    }
    dr[j] = d;
  }
  __syncwarp();
  int32_t* ti = tokens_in + cu[l];
  for (int j = ln; j < rows; j += 32) {
    const int32_t in = j == 0 ? t0 : (dr[j - 1] >= 0 ? dr[j - 1] : 0);
    ti[j] = in;
    if (j > 0) {
      unsigned why = 0;
      const int64_t at = pool_at(v, l, pos + j, &why);
      if (at < 0) record_fault(dev_err, why, l, pos + j);
      else v.pool[at] = in;
    }
  }
}

// Prompt chunks: token t of the stream goes to the pool at positions[t] of lane token_lane[t].
__global__ void write_tokens_kernel(PoolView v, const int32_t* __restrict__ tokens,
                                    const int32_t* __restrict__ positions, const int32_t* __restrict__ lane_of,
                                    int32_t rows, unsigned long long* dev_err) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= rows) return;
  unsigned why = 0;
  const int64_t at = pool_at(v, lane_of[t], positions[t], &why);
  if (at < 0) record_fault(dev_err, why, lane_of[t], positions[t]);
  else v.pool[at] = tokens[t];
}

// The lane's last token after a step: the last accepted id of its row of `block` ids.
__global__ void commit_kernel(const int32_t* __restrict__ ids, int32_t width, int32_t block, int32_t* tok) {
  const int l = blockIdx.x * blockDim.x + threadIdx.x;
  if (l >= width) return;
  int32_t last = -1;
  for (int j = 0; j < block; ++j) {
    const int32_t id = ids[(int64_t)l * block + j];
    if (id == -2) break;
    if (id >= 0) last = id;
  }
  if (last >= 0) tok[l] = last;
}

int grid_for(int64_t n, int threads) {
  const int64_t g = (n + threads - 1) / threads;
  const int64_t cap = (int64_t)sm_count() * 8;
  return (int)(g < 1 ? 1 : g > cap ? cap : g);
}

int gen_e4m3(uint8_t* w, int64_t n, uint64_t seed, float* sw, int64_t ns, float sigma, cudaStream_t s) {
  gen_e4m3_kernel<<<grid_for(n, 256), 256, 0, s>>>(w, n, seed);
  HK_TRY_LAUNCH("gen_e4m3_kernel");
  fill_f32_kernel<<<grid_for(ns, 256), 256, 0, s>>>(sw, ns, sigma / 112.0f);
  HK_TRY_LAUNCH("fill_f32_kernel");
  return HK_OK;
}

size_t al256(size_t x) { return (x + 255) & ~(size_t)255; }

int dev_alloc(MlaModel* m, void** p, size_t bytes) {
  *p = nullptr;
  cudaError_t e = cudaMalloc(p, al256(bytes ? bytes : 1));
  if (e != cudaSuccess) return cuda_fail(e, "hk_open_mla: cudaMalloc");
  m->allocations.push_back(*p);
  return HK_OK;
}

template <class T>
int alloc(MlaModel* m, T** p, size_t count) {
  void* v = nullptr;
  HK_TRY(dev_alloc(m, &v, count * sizeof(T)));
  *p = static_cast<T*>(v);
  return HK_OK;
}

int gemm(const uint8_t* xq, const float* xs, const uint8_t* w, const float* sw, int64_t m, int32_t n, int32_t k,
         uint16_t* y, cudaStream_t s) {
  return hk_gemm_fp8(xq, xs, w, sw, m, n, k, y, s);
}

int rms_quant(const uint16_t* x, const uint16_t* add, uint16_t* x_out, const int32_t* idx, int32_t rows, int32_t H,
              uint8_t* q, float* sc, cudaStream_t s) {
  if (rows == 0) return HK_OK;
  rms_quant_kernel<<<rows, kNormThreads, 0, s>>>(x, add, x_out, idx, rows, H, q, sc);
  HK_TRY_LAUNCH("rms_quant_kernel");
  return HK_OK;
}

// The layers over the T packed rows (m->tokens_in, the pack outputs), then the final norm of
// the R sampled rows (gather[r] when `gather` is set, else row r) and the vocabulary GEMM into
// m->logits (fp32 [R][vocab]).
int forward(MlaModel* m, int32_t T, int32_t R, bool gather, const int32_t* rows_dev, int32_t max_kv,
            cudaStream_t s) {
  const hk_mla_model& d = m->dims;
  const int32_t H = (int32_t)d.hidden, QL = (int32_t)d.q_lora, E = (int32_t)d.experts, K = (int32_t)d.top_k,
                I = (int32_t)d.inter, V = (int32_t)d.vocab;
  const float theta = d.rope_theta > 0 ? d.rope_theta : 10000.0f;
  const float route_scale = d.route_scale > 0 ? d.route_scale : 1.0f;
  const int64_t slots = m->pages * kPage;
  embed_kernel<<<T, 128, 0, s>>>(m->tokens_in, T, m->embed, H, V, m->x, err_word());
  HK_TRY_LAUNCH("embed_kernel");
  const uint16_t* pending = nullptr;  // the previous layer's MoE output, added before the next norm
  for (size_t l = 0; l < m->layers.size(); ++l) {
    const MlaLayer& L = m->layers[l];
    HK_TRY(rms_quant(m->x, pending, pending ? m->x : nullptr, nullptr, T, H, m->xq, m->xs, s));
    HK_TRY(gemm(m->xq, m->xs, L.wqa, L.sqa, T, QL, H, m->qa, s));
    HK_TRY(gemm(m->xq, m->xs, L.wkva, L.skva, T, kRow, H, m->kvn, s));
    HK_TRY(rms_quant(m->qa, nullptr, nullptr, nullptr, T, QL, m->qaq, m->qas, s));
    HK_TRY(gemm(m->qaq, m->qas, L.wqb, L.sqb, T, kHeads * kRow, QL, m->q, s));
    rope_norm_kernel<<<T, 128, 0, s>>>(m->q, m->kvn, m->positions, T, theta);
    HK_TRY_LAUNCH("rope_norm_kernel");
    HK_TRY(hk_kv_append_bf16(m->kvn, m->slots, T, kRow, kPage, L.kv, slots, s));
    HK_TRY(hk_mla_decode(m->q, L.kv, rows_dev, m->bt_stride, m->cu_seqlens, m->positions, m->width, T, kHeads,
                         kPage, slots, max_kv, 1.0f / sqrtf((float)kRow), m->o, m->lse, m->attn_ws,
                         m->attn_ws_bytes, 0, s));
    HK_TRY(hk_quant_fp8(m->o, T, kHeads * kLatent, m->oq, m->os, s));
    HK_TRY(gemm(m->oq, m->os, L.wo, L.so, T, H, kHeads * kLatent, m->y, s));
    HK_TRY(rms_quant(m->x, m->y, m->x, nullptr, T, H, m->xq, m->xs, s));
    HK_TRY(gemm(m->xq, m->xs, L.wr, L.sr, T, E, H, m->rl, s));
    f32_of_bf16_kernel<<<grid_for((int64_t)T * E, 256), 256, 0, s>>>(m->rl, m->rlf, (int64_t)T * E);
    HK_TRY_LAUNCH("f32_of_bf16_kernel");
    HK_TRY(hk_route(m->rlf, nullptr, T, E, K, route_scale, m->ids_e, m->w_e, s));
    HK_TRY(hk_permute(m->ids_e, m->w_e, T, K, E, m->offsets, m->perm_token, m->perm_w, m->inv, s));
    shared_rows_kernel<<<grid_for(T, 256), 256, 0, s>>>(m->offsets, m->perm_token, E, T, K);
    HK_TRY_LAUNCH("shared_rows_kernel");
    // E + 1 experts (the shared one last, as the weights store it): rows [T*K, T*K + T) of ym
    // are the shared expert's output of every token
    HK_TRY(hk_moe_grouped(m->xq, m->xs, T, m->offsets, m->perm_token, (int64_t)T * (K + 1), E + 1, H, I, L.w13,
                          L.s13, L.w2, L.s2, m->ym, m->moe_ws, m->moe_ws_bytes, s));
    HK_TRY(hk_combine(m->ym, (int64_t)T * K, m->perm_w, m->inv, m->ym + (size_t)T * K * H, T, K, H, m->mo, s));
    pending = m->mo;
  }
  HK_TRY(rms_quant(m->x, pending, nullptr, gather ? m->gather : nullptr, R, H, m->xq, m->xs, s));
  HK_TRY(gemm(m->xq, m->xs, m->wvocab, m->svocab, R, V, H, m->logits_bf16, s));
  f32_of_bf16_kernel<<<grid_for((int64_t)R * V, 256), 256, 0, s>>>(m->logits_bf16, m->logits, (int64_t)R * V);
  HK_TRY_LAUNCH("f32_of_bf16_kernel");
  return HK_OK;
}

// Stage layout (int32 words): lane_tokens [width], lane_pos [width], cu_rows [width + 1],
// gather [r_cap], tokens_in [t_cap].
struct Stage {
  size_t lane_tokens, lane_pos, cu_rows, gather, tokens_in, words;
};

Stage stage_layout(int32_t width, int32_t r_cap, int32_t t_cap) {
  Stage st{};
  st.lane_tokens = 0;
  st.lane_pos = st.lane_tokens + width;
  st.cu_rows = st.lane_pos + width;
  st.gather = st.cu_rows + width + 1;
  st.tokens_in = st.gather + r_cap;
  st.words = st.tokens_in + t_cap;
  return st;
}

PoolView pool_view(const MlaModel* m, const int32_t* rows_dev, int32_t* pool) {
  PoolView v;
  v.rows = rows_dev;
  v.pool = pool;
  v.bt_stride = m->bt_stride;
  v.entries = m->entries;  // the row's page entries (its window entries follow them)
  v.page_rows = m->page_rows;
  v.pages = m->pages;
  return v;
}

}  // namespace

int mla_check(const hk_config& c, const hk_mla_model& d) {
  HK_REQUIRE(c.page_rows == kPage, "HK_MODEL_MLA: page_rows %u (the latent cache takes pages of 64 rows)",
             c.page_rows);
  HK_REQUIRE(c.transport == HK_TRANSPORT_LAUNCH, "HK_MODEL_MLA runs on HK_TRANSPORT_LAUNCH");
  HK_REQUIRE(c.block >= 1 && c.block <= 32, "HK_MODEL_MLA: block %u not in 1..32", c.block);
  HK_REQUIRE(d.hidden > 0 && d.hidden % 128 == 0 && d.hidden <= 16384, "hk_mla_model: hidden %u (a multiple of 128)",
             d.hidden);
  HK_REQUIRE(d.q_lora > 0 && d.q_lora % 128 == 0, "hk_mla_model: q_lora %u (a multiple of 128)", d.q_lora);
  HK_REQUIRE(d.vocab > 0 && d.vocab % 16 == 0 && d.vocab <= (1u << 22), "hk_mla_model: vocab %u", d.vocab);
  HK_REQUIRE(d.experts >= 16 && d.experts % 16 == 0 && d.experts <= 256, "hk_mla_model: experts %u (16..256, a "
             "multiple of 16)", d.experts);
  HK_REQUIRE(d.top_k >= 1 && d.top_k <= 16 && d.top_k <= d.experts, "hk_mla_model: top_k %u", d.top_k);
  HK_REQUIRE(d.inter > 0 && d.inter % 128 == 0, "hk_mla_model: inter %u (a multiple of 128)", d.inter);
  HK_REQUIRE(d.layers >= 1 && d.layers <= 128, "hk_mla_model: layers %u", d.layers);
  HK_REQUIRE(d.logprobs <= 64, "hk_mla_model: logprobs %u (at most 64)", d.logprobs);
  return HK_OK;
}

int mla_create(const hk_config& c, const hk_mla_model& d, MlaModel** out, cudaStream_t s) {
  *out = nullptr;
  HK_TRY(mla_check(c, d));
  auto* m = new MlaModel;
  auto fail = [&](int rc) {
    mla_destroy(m);
    return rc;
  };
  m->dims = d;
  m->width = (int32_t)c.width;
  m->block = (int32_t)c.block;
  m->page_rows = (int32_t)c.page_rows;
  m->context = (int32_t)c.context;
  m->chunk = (int32_t)c.chunk;
  m->entries = (int32_t)c.entries;
  m->bt_stride = (int32_t)(c.entries + c.window);
  m->pages = (int64_t)c.pages;
  // Rows of one forward pass: a decode step's rows, or a group of prompt chunks of distinct
  // lanes.  Every pass streams all the weights a few hundred rows already hit (the expert FFN
  // alone is ~11 GB at DeepSeek-V3's shape), so the prompt chunks of one share (an engine with
  // a prefill token budget sends several: the reference's tuned presets allow 8192 tokens a
  // step) go through in groups of up to 8192 rows (16 chunks of 512), not a pass a chunk.
  m->t_cap = std::max<int32_t>({m->width * m->block, m->chunk, std::min<int32_t>(16 * m->chunk, 8192)});
  m->r_cap = m->width * m->block;
  m->n_lp = (int32_t)d.logprobs;
  const int64_t H = d.hidden, QL = d.q_lora, E = d.experts, K = d.top_k, I = d.inter, V = d.vocab;
  const int64_t T = m->t_cap, R = m->r_cap;
  int rc = HK_OK;
#define HK_A(p, n) \
  if ((rc = alloc(m, &(p), (size_t)(n))) != HK_OK) return fail(rc)
  uint64_t seed = d.seed;
  auto next_seed = [&]() { return seed = seed * 6364136223846793005ull + 1442695040888963407ull; };
  auto weights = [&](uint8_t** w, float** sw, int64_t n, int64_t k, int64_t count) -> int {
    const int64_t ns = count * ((n + 127) / 128) * (k / 128);
    HK_TRY(alloc(m, w, (size_t)(count * n * k)));
    HK_TRY(alloc(m, sw, (size_t)ns));
    return gen_e4m3(*w, count * n * k, next_seed(), *sw, ns, 1.0f / sqrtf((float)k), s);
  };
  HK_A(m->embed, V * H);
  gen_bf16_kernel<<<grid_for(V * H, 256), 256, 0, s>>>(m->embed, V * H, next_seed());
  if ((rc = [&] { HK_TRY_LAUNCH("gen_bf16_kernel"); return HK_OK; }()) != HK_OK) return fail(rc);
  if ((rc = weights(&m->wvocab, &m->svocab, V, H, 1)) != HK_OK) return fail(rc);
  m->layers.resize(d.layers);
  for (uint32_t l = 0; l < d.layers; ++l) {
    MlaLayer& L = m->layers[l];
    if ((rc = weights(&L.wqa, &L.sqa, QL, H, 1)) != HK_OK) return fail(rc);
    if ((rc = weights(&L.wqb, &L.sqb, (int64_t)kHeads * kRow, QL, 1)) != HK_OK) return fail(rc);
    if ((rc = weights(&L.wkva, &L.skva, kRow, H, 1)) != HK_OK) return fail(rc);
    if ((rc = weights(&L.wo, &L.so, H, (int64_t)kHeads * kLatent, 1)) != HK_OK) return fail(rc);
    if ((rc = weights(&L.wr, &L.sr, E, H, 1)) != HK_OK) return fail(rc);
    if ((rc = weights(&L.w13, &L.s13, 2 * I, H, E + 1)) != HK_OK) return fail(rc);
    if ((rc = weights(&L.w2, &L.s2, H, I, E + 1)) != HK_OK) return fail(rc);
    HK_A(L.kv, m->pages * kPage * kRow);
    cudaError_t e = cudaMemsetAsync(L.kv, 0, (size_t)m->pages * kPage * kRow * 2, s);
    if (e != cudaSuccess) return fail(cuda_fail(e, "hk_open_mla: zeroing the latent cache"));
  }
  const int32_t W = m->width;
  HK_A(m->cu_seqlens, W + 1);
  HK_A(m->seq_lens, W);
  HK_A(m->positions, T);
  HK_A(m->slots, T);
  HK_A(m->token_lane, T);
  HK_A(m->active, W + 1);
  HK_A(m->drafts, (int64_t)W * std::max(1, m->block - 1));
  HK_A(m->x, T * H);
  HK_A(m->xq, T * H);
  HK_A(m->xs, T * (H / 128));
  HK_A(m->qa, T * QL);
  HK_A(m->qaq, T * QL);
  HK_A(m->qas, T * (QL / 128));
  HK_A(m->q, T * kHeads * kRow);
  HK_A(m->kvn, T * kRow);
  HK_A(m->o, T * kHeads * kLatent);
  HK_A(m->oq, T * kHeads * kLatent);
  HK_A(m->os, T * (kHeads * kLatent / 128));
  HK_A(m->lse, T * kHeads);
  HK_A(m->y, T * H);
  HK_A(m->rl, T * E);
  HK_A(m->rlf, T * E);
  HK_A(m->ids_e, T * K);
  HK_A(m->w_e, T * K);
  HK_A(m->offsets, E + 2);
  HK_A(m->perm_token, T * (K + 1));
  HK_A(m->perm_w, T * K);
  HK_A(m->inv, T * K);
  HK_A(m->ym, T * (K + 1) * H);
  HK_A(m->mo, T * H);
  HK_A(m->logits_bf16, R * V);
  HK_A(m->logits, R * V);
  HK_A(m->out_ids, (int64_t)W * m->block);
  HK_A(m->lp, (int64_t)W * m->block * (2 * m->n_lp + 1));
  HK_A(m->sampling, W);
  HK_A(m->state, W);
  HK_A(m->tok, W);
  m->attn_ws_bytes = hk_mla_workspace_size(W, (int32_t)T, kHeads, m->context);
  m->moe_ws_bytes = hk_moe_workspace_size(T * (K + 1), (int32_t)H, (int32_t)I);
  m->sample_ws_bytes = hk_sample_workspace_size((int32_t)R, (int32_t)V);
  if ((rc = dev_alloc(m, &m->attn_ws, m->attn_ws_bytes)) != HK_OK) return fail(rc);
  if ((rc = dev_alloc(m, &m->moe_ws, m->moe_ws_bytes)) != HK_OK) return fail(rc);
  if ((rc = dev_alloc(m, &m->sample_ws, m->sample_ws_bytes)) != HK_OK) return fail(rc);
  const Stage st = stage_layout(W, (int32_t)R, (int32_t)T);
  m->stage_words = st.words;
  HK_A(m->stage_d, st.words);
  {
    cudaError_t e = cudaMallocHost(&m->stage_h, st.words * 4);
    if (e != cudaSuccess) return fail(cuda_fail(e, "hk_open_mla: staging"));
  }
  m->lane_tokens = m->stage_d + st.lane_tokens;
  m->lane_pos = m->stage_d + st.lane_pos;
  m->cu_rows = m->stage_d + st.cu_rows;
  m->gather = m->stage_d + st.gather;
  m->tokens_in = m->stage_d + st.tokens_in;
  cudaError_t e = cudaMemsetAsync(m->sampling, 0, sizeof(hk_sampling) * W, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(m->state, 0, sizeof(uint64_t) * W, s);
  if (e == cudaSuccess) e = cudaMemsetAsync(m->tok, 0, sizeof(int32_t) * W, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return fail(cuda_fail(e, "hk_open_mla"));
#undef HK_A
  *out = m;
  return HK_OK;
}

void mla_destroy(MlaModel* m) {
  if (!m) return;
  for (void* p : m->allocations) cudaFree(p);
  if (m->stage_h) cudaFreeHost(m->stage_h);
  delete m;
}

int mla_tensor(MlaModel* m, int32_t* token_pool, size_t token_pool_bytes, uint32_t layer, const char* name,
               void** ptr, size_t* bytes) {
  HK_REQUIRE(m && name && ptr && bytes, "hk_model_tensor: null argument");
  const hk_mla_model& d = m->dims;
  const size_t H = d.hidden, QL = d.q_lora, E = d.experts, I = d.inter, V = d.vocab;
  auto sc = [](size_t n, size_t k) { return ((n + 127) / 128) * (k / 128) * sizeof(float); };
  const std::string n = name;
  if (n == "embed") { *ptr = m->embed; *bytes = V * H * 2; return HK_OK; }
  if (n == "vocab") { *ptr = m->wvocab; *bytes = V * H; return HK_OK; }
  if (n == "vocab.scale") { *ptr = m->svocab; *bytes = sc(V, H); return HK_OK; }
  if (n == "tokens") { *ptr = token_pool; *bytes = token_pool_bytes; return HK_OK; }
  HK_REQUIRE(layer < m->layers.size(), "hk_model_tensor: layer %u of %zu", layer, m->layers.size());
  const MlaLayer& L = m->layers[layer];
  struct Entry {
    const char* name;
    void* p;
    size_t bytes;
  };
  const size_t R = kRow, HL = (size_t)kHeads * kLatent, QH = (size_t)kHeads * kRow;
  const Entry table[] = {
      {"wqa", L.wqa, QL * H}, {"wqa.scale", L.sqa, sc(QL, H)},
      {"wqb", L.wqb, QH * QL}, {"wqb.scale", L.sqb, sc(QH, QL)},
      {"wkva", L.wkva, R * H}, {"wkva.scale", L.skva, sc(R, H)},
      {"wo", L.wo, H * HL}, {"wo.scale", L.so, sc(H, HL)},
      {"router", L.wr, E * H}, {"router.scale", L.sr, sc(E, H)},
      {"w13", L.w13, (E + 1) * 2 * I * H}, {"w13.scale", L.s13, (E + 1) * sc(2 * I, H)},
      {"w2", L.w2, (E + 1) * H * I}, {"w2.scale", L.s2, (E + 1) * sc(H, I)},
      {"kv", L.kv, (size_t)m->pages * kPage * kRow * 2},
  };
  for (const Entry& e : table)
    if (n == e.name) {
      *ptr = e.p;
      *bytes = e.bytes;
      return HK_OK;
    }
  return fail(HK_EINVAL, "hk_model_tensor: no tensor named %s", name);
}

int mla_decode_step(MlaModel* m, const std::vector<MlaLaneRows>& lanes, const int32_t* rows_dev, int32_t* pool,
                    unsigned long long* dev_err, cudaStream_t s) {
  int32_t* tok = m->tok;
  const Stage st = stage_layout(m->width, m->r_cap, m->t_cap);
  int32_t* h = m->stage_h;
  memset(h, 0, st.words * 4);
  int32_t T = 0, max_kv = 1;
  for (const MlaLaneRows& r : lanes) {
    h[st.lane_tokens + r.lane] = r.rows;
    h[st.lane_pos + r.lane] = r.pos;
    T += r.rows;
    max_kv = std::max(max_kv, r.pos + r.rows);
  }
  HK_REQUIRE(T <= m->r_cap, "MLA decode step: %d rows past %d", T, m->r_cap);
  HK_TRY_CUDA(cudaMemcpyAsync(m->stage_d, h, st.tokens_in * 4, cudaMemcpyHostToDevice, s));
  HK_TRY(hk_pack(m->lane_tokens, m->lane_pos, rows_dev, m->bt_stride, m->width, kPage, (int32_t)m->pages, m->t_cap,
                 m->cu_seqlens, m->seq_lens, m->positions, m->slots, m->token_lane, m->active, s));
  prepare_kernel<<<(m->width * 32 + 127) / 128, 128, 0, s>>>(pool_view(m, rows_dev, pool), m->lane_tokens,
                                                              m->lane_pos, m->cu_seqlens, tok, m->width, m->block,
                                                              m->tokens_in, m->drafts, dev_err);
  HK_TRY_LAUNCH("prepare_kernel");
  if (T > 0) HK_TRY(forward(m, T, T, false, rows_dev, max_kv, s));
  HK_TRY(hk_sample_verify(m->logits, (int32_t)m->dims.vocab, m->cu_seqlens, m->width, T, m->block, m->sampling,
                          m->state, m->block > 1 ? m->drafts : nullptr, m->n_lp, m->out_ids,
                          m->n_lp > 0 ? m->lp : nullptr, m->sample_ws, m->sample_ws_bytes, s));
  commit_kernel<<<(m->width + 127) / 128, 128, 0, s>>>(m->out_ids, m->width, m->block, tok);
  HK_TRY_LAUNCH("commit_kernel");
  return HK_OK;
}

int mla_prompt_step(MlaModel* m, const std::vector<MlaLaneRows>& lanes, const std::vector<int32_t>& tokens,
                    const int32_t* rows_dev, int32_t* pool, unsigned long long* dev_err, cudaStream_t s) {
  int32_t* tok = m->tok;
  const Stage st = stage_layout(m->width, m->r_cap, m->t_cap);
  int32_t* h = m->stage_h;
  memset(h, 0, st.words * 4);
  int32_t T = 0, max_kv = 1, n = 0;
  for (const MlaLaneRows& r : lanes) {
    h[st.lane_tokens + r.lane] = r.rows;
    h[st.lane_pos + r.lane] = r.pos;
    T += r.rows;
    h[st.gather + n++] = T - 1;  // the chunk's last row (lanes ascending: the pack keeps that order)
    max_kv = std::max(max_kv, r.pos + r.rows);
  }
  HK_REQUIRE(T <= m->t_cap && (size_t)T == tokens.size(), "MLA prompt step: %d rows (%zu tokens, cap %d)", T,
             tokens.size(), m->t_cap);
  HK_REQUIRE(max_kv <= m->context, "MLA prompt step: a chunk reaching position %d past the context %d", max_kv,
             m->context);
  int32_t acc = 0;
  for (int32_t l = 0; l < m->width; ++l) {  // one sampled row for each prompt lane
    h[st.cu_rows + l] = acc;
    for (const MlaLaneRows& r : lanes) acc += r.lane == l ? 1 : 0;
  }
  h[st.cu_rows + m->width] = acc;
  memcpy(h + st.tokens_in, tokens.data(), 4 * tokens.size());
  HK_TRY_CUDA(cudaMemcpyAsync(m->stage_d, h, (st.tokens_in + T) * 4, cudaMemcpyHostToDevice, s));
  HK_TRY(hk_pack(m->lane_tokens, m->lane_pos, rows_dev, m->bt_stride, m->width, kPage, (int32_t)m->pages, m->t_cap,
                 m->cu_seqlens, m->seq_lens, m->positions, m->slots, m->token_lane, m->active, s));
  write_tokens_kernel<<<(T + 127) / 128, 128, 0, s>>>(pool_view(m, rows_dev, pool), m->tokens_in, m->positions,
                                                       m->token_lane, T, dev_err);
  HK_TRY_LAUNCH("write_tokens_kernel");
  HK_TRY(forward(m, T, n, true, rows_dev, max_kv, s));
  HK_TRY(hk_sample_verify(m->logits, (int32_t)m->dims.vocab, m->cu_rows, m->width, n, 1, m->sampling, m->state,
                          nullptr, m->n_lp, m->out_ids, m->n_lp > 0 ? m->lp : nullptr, m->sample_ws,
                          m->sample_ws_bytes, s));
  commit_kernel<<<(m->width + 127) / 128, 128, 0, s>>>(m->out_ids, m->width, 1, tok);
  HK_TRY_LAUNCH("commit_kernel");
  return HK_OK;
}

}  // namespace hk
