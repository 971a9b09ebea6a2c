// Spec-decode verification with on-device sampling: the reply side of the decode step.
//
// Semantics (restated from the reference's source sampler, src/evo2/draw.rs:14-58, and its
// reply reader, src/gpu/feed.rs:163-208):
//   * a lane's rows are its 1 + drafts positions; row j is drawn with the lane's sampling and
//     generator state, and the chain goes on to row j + 1 only while the token drawn equals
//     draft j;
//   * greedy (temperature <= 0 or top_k == 1): the first index of the greatest logit, no draw;
//   * otherwise the row is sorted by value, descending in the IEEE total order, ties in index
//     order; the first top_k are kept (all when top_k == 0); p = softmax(value / temperature)
//     in f64; when 0 < top_p < 1 the tail whose inclusive sum from the bottom is <= 1 - top_p
//     is zeroed; u = splitmix(state) / 2^53 * kept picks the first index whose running sum
//     exceeds u, else the last index with a non-zero probability;
//   * a row with a non-finite logit gives id -1 and ends the lane;
//   * every accepted token gets a logprob row: n (id, logprob) pairs of log-softmax(row) at
//     temperature 1, best first, id -1 past the vocabulary, then the token's own logprob.
// Sums run in parallel here (the reference sums left to right): probabilities agree to the
// last few bits, so a draw differs only if u falls that close to a boundary.
//
// Kernels: one CTA per row sorts the row (stable LSD radix sort of total-order keys with the
// indices as payload, 4 passes of 8 bits, in global scratch) and prepares the row's running
// probabilities; then one thread per lane walks the chain.
#include "common.cuh"

namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxVocab = 1 << 22;

struct RowStat {
  double lse;      // log-sum-exp of the row (temperature 1)
  double kept;     // probability mass left after top-k / top-p (sampled rows)
  int32_t argmax;  // first index of the greatest logit
  int32_t m;       // entries kept by top-k
  int32_t flags;   // 1: a non-finite logit; 2: the row was sorted
  int32_t pad;
};

struct Scratch {
  uint32_t* keys;  // [rows][2][vocab]
  int32_t* idx;    // [rows][2][vocab]
  double* cum;     // [rows][vocab]
  RowStat* stats;  // [rows]
};

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

Scratch carve(void* ws, int32_t rows, int32_t vocab) {
  uint8_t* p = reinterpret_cast<uint8_t*>(ws);
  Scratch s;
  const size_t nv = (size_t)rows * vocab;
  s.keys = reinterpret_cast<uint32_t*>(p);
  p += align256(nv * 2 * sizeof(uint32_t));
  s.idx = reinterpret_cast<int32_t*>(p);
  p += align256(nv * 2 * sizeof(int32_t));
  s.cum = reinterpret_cast<double*>(p);
  p += align256(nv * sizeof(double));
  s.stats = reinterpret_cast<RowStat*>(p);
  return s;
}

size_t scratch_bytes(int32_t rows, int32_t vocab) {
  const size_t nv = (size_t)rows * vocab;
  return align256(nv * 8) + align256(nv * 8) + align256(nv * 8) + align256((size_t)rows * sizeof(RowStat));
}

// Descending IEEE total order as an ascending unsigned key, and back.
__device__ __forceinline__ uint32_t desc_key(float x) {
  const uint32_t b = __float_as_uint(x);
  const uint32_t asc = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ~asc;
}
__device__ __forceinline__ float key_value(uint32_t k) {
  const uint32_t asc = ~k;
  return __uint_as_float((asc & 0x80000000u) ? (asc & 0x7FFFFFFFu) : ~asc);
}

__device__ __forceinline__ bool greedy(const hk_sampling& s) {
  return !(s.temperature > 0.f) || s.top_k == 1;
}

__device__ __forceinline__ int lane_of(const int32_t* cu, int lanes, int r) {
  int lo = 0, hi = lanes;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (cu[mid] <= r) lo = mid; else hi = mid;
  }
  return lo;
}

// Block-wide sum of a double (every thread gets it); `red` holds kWarps doubles.
__device__ double block_sum(double v, double* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double t = 0.0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) t += red[w];
  return t;
}

// Block-wide exclusive prefix of a double in thread order (and the total).
__device__ double block_excl(double v, double* red, double* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  double x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31) red[warp] = x;
  __syncthreads();
  double before = 0.0, t = 0.0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    if (w < warp) before += red[w];
    t += red[w];
  }
  *total = t;
  return before + x - v;
}

__global__ void __launch_bounds__(kThreads) sample_rows_kernel(
    const float* __restrict__ logits, int32_t vocab, const int32_t* __restrict__ cu, int32_t lanes,
    int32_t rows, const hk_sampling* __restrict__ sampling, int32_t n_logprobs, Scratch s,
    unsigned long long* err) {
  __shared__ uint32_t hist[256], base[256], run[256];
  __shared__ uint32_t wcnt[kWarps][256];  // (tag << 16) | count of a digit in a warp's slice
  __shared__ double red[kWarps];
  __shared__ float smax[kWarps];
  __shared__ int sarg[kWarps], sbad[kWarps];
  const int r = blockIdx.x;
  if (r >= rows) return;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const hk_sampling smp = sampling[lane_of(cu, lanes, r)];
  const float* x = logits + (int64_t)r * vocab;
  RowStat* st = s.stats + r;

  // ---- the row's maximum (first index), finiteness and log-sum-exp
  float mx = -INFINITY;
  int arg = 0x7fffffff, bad = 0;
  for (int i = tid; i < vocab; i += kThreads) {
    const float v = x[i];
    if (!isfinite(v)) bad = 1;
    else if (v > mx || (v == mx && i < arg)) { mx = v; arg = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, mx, o);
    const int a2 = __shfl_xor_sync(0xffffffffu, arg, o);
    if (m2 > mx || (m2 == mx && a2 < arg)) { mx = m2; arg = a2; }
    bad |= __shfl_xor_sync(0xffffffffu, bad, o);
  }
  if (lane == 0) { smax[warp] = mx; sarg[warp] = arg; sbad[warp] = bad; }
  __syncthreads();
  mx = smax[0]; arg = sarg[0]; bad = sbad[0];
  for (int w = 1; w < kWarps; ++w) {
    if (smax[w] > mx || (smax[w] == mx && sarg[w] < arg)) { mx = smax[w]; arg = sarg[w]; }
    bad |= sbad[w];
  }
  if (bad) {
    if (tid == 0) { st->flags = 1; st->argmax = 0; st->m = 0; st->kept = 0.0; st->lse = 0.0; }
    return;
  }
  double e = 0.0;
  for (int i = tid; i < vocab; i += kThreads) e += exp((double)x[i] - (double)mx);
  const double lse = (double)mx + log(block_sum(e, red));
  const bool sampled = !greedy(smp);
  if (!sampled && n_logprobs == 0) {
    if (tid == 0) { st->flags = 0; st->argmax = arg; st->m = 0; st->kept = 0.0; st->lse = lse; }
    return;
  }

  // ---- stable LSD radix sort of (key, index), 4 passes of 8 bits, buffers 0 -> 1 -> 0 ...
  uint32_t* k0 = s.keys + (int64_t)r * 2 * vocab;
  uint32_t* k1 = k0 + vocab;
  int32_t* i0 = s.idx + (int64_t)r * 2 * vocab;
  int32_t* i1 = i0 + vocab;
  for (int i = tid; i < vocab; i += kThreads) { k0[i] = desc_key(x[i]); i0[i] = i; }
  for (int i = tid; i < kWarps * 256; i += kThreads) (&wcnt[0][0])[i] = 0u;
  const int tiles = (vocab + kThreads - 1) / kThreads;
  const uint32_t lt_mask = (1u << lane) - 1u;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 8 * pass;
    const uint32_t* ks = (pass & 1) ? k1 : k0;
    const int32_t* is = (pass & 1) ? i1 : i0;
    uint32_t* kd = (pass & 1) ? k0 : k1;
    int32_t* id = (pass & 1) ? i0 : i1;
    if (tid < 256) { hist[tid] = 0u; run[tid] = 0u; }
    __syncthreads();
    for (int i = tid; i < vocab; i += kThreads) atomicAdd(&hist[(ks[i] >> shift) & 255u], 1u);
    __syncthreads();
    if (warp == 0) {  // exclusive scan of the 256 digit counts, 8 per lane
      uint32_t loc[8], sum = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) { loc[j] = hist[lane * 8 + j]; sum += loc[j]; }
      uint32_t inc = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
      }
      uint32_t acc = inc - sum;
#pragma unroll
      for (int j = 0; j < 8; ++j) { base[lane * 8 + j] = acc; acc += loc[j]; }
    }
    __syncthreads();
    for (int t = 0; t < tiles; ++t) {
      const uint32_t tag = (uint32_t)(pass * tiles + t + 1);
      const int e_ = t * kThreads + tid;
      const bool valid = e_ < vocab;
      const uint32_t key = valid ? ks[e_] : 0u;
      const int32_t ix = valid ? is[e_] : 0;
      const uint32_t d = valid ? ((key >> shift) & 255u) : 256u;
      const uint32_t peers = __match_any_sync(0xffffffffu, d);
      const uint32_t wrank = __popc(peers & lt_mask);
      if (valid && lane == __ffs(peers) - 1) wcnt[warp][d] = (tag << 16) | (uint32_t)__popc(peers);
      __syncthreads();
      if (valid) {
        uint32_t before = 0;
        for (int w = 0; w < warp; ++w) {
          const uint32_t c = wcnt[w][d];
          if ((c >> 16) == tag) before += c & 0xFFFFu;
        }
        const uint32_t pos = base[d] + run[d] + before + wrank;
        kd[pos] = key;
        id[pos] = ix;
      }
      __syncthreads();
      if (tid < 256) {
        uint32_t tot = 0;
        for (int w = 0; w < kWarps; ++w) {
          const uint32_t c = wcnt[w][tid];
          if ((c >> 16) == tag) tot += c & 0xFFFFu;
        }
        run[tid] += tot;
      }
      __syncthreads();
    }
  }
  // sorted keys and indices are in k0 / i0

  int m = 0;
  double kept = 0.0;
  if (sampled) {
    m = smp.top_k > 0 ? (int)min((uint32_t)vocab, smp.top_k) : vocab;
    double* p = s.cum + (int64_t)r * vocab;
    const double temp = (double)smp.temperature;
    const double s0 = (double)key_value(k0[0]) / temp;
    const int chunk = (m + kThreads - 1) / kThreads;
    const int a = min(m, tid * chunk), z = min(m, a + chunk);
    double loc = 0.0;
    for (int i = a; i < z; ++i) {
      const double v = exp((double)key_value(k0[i]) / temp - s0);
      p[i] = v;
      loc += v;
    }
    const double total = block_sum(loc, red);
    for (int i = a; i < z; ++i) p[i] = p[i] / total;
    const double top_p = (double)smp.top_p;
    if (top_p > 0.0 && top_p < 1.0) {
      // zero the tail whose inclusive sum from the bottom is <= 1 - top_p
      loc = 0.0;
      for (int i = a; i < z; ++i) loc += p[i];
      double all;
      const double before = block_excl(loc, red, &all);
      double below = all - before - loc;  // mass of the chunks after this one
      for (int i = z - 1; i >= a; --i) {
        below += p[i];
        if (below <= 1.0 - top_p) p[i] = 0.0;
      }
      __syncthreads();
    }
    // running sums of what is left
    loc = 0.0;
    for (int i = a; i < z; ++i) loc += p[i];
    double all;
    double acc = block_excl(loc, red, &all);
    for (int i = a; i < z; ++i) {
      acc += p[i];
      p[i] = acc;
    }
    kept = all;
  }
  if (tid == 0) { st->flags = 2; st->argmax = arg; st->m = m; st->kept = kept; st->lse = lse; }
}

__device__ __forceinline__ uint64_t splitmix(uint64_t& state) {
  state += 0x9E3779B97F4A7C15ull;
  uint64_t z = state;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return (z ^ (z >> 31)) >> 11;
}

__global__ void sample_chain_kernel(const float* __restrict__ logits, int32_t vocab,
                                    const int32_t* __restrict__ cu, int32_t lanes, int32_t block,
                                    const hk_sampling* __restrict__ sampling, uint64_t* state,
                                    const int32_t* __restrict__ drafts, int32_t n_logprobs,
                                    int32_t* __restrict__ ids, float* __restrict__ lp, Scratch s,
                                    unsigned long long* err) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= lanes) return;
  const int width = 2 * n_logprobs + 1;
  for (int j = 0; j < block; ++j) {
    ids[(int64_t)b * block + j] = -2;
    if (n_logprobs > 0)
      for (int q = 0; q < width; ++q) lp[((int64_t)b * block + j) * width + q] = 0.f;
  }
  const int r0 = cu[b], rows = cu[b + 1] - r0;
  if (rows < 0 || rows > block) {
    hk_flag(err, hk::kErrMoeRow, (unsigned)b);
    return;
  }
  const hk_sampling smp = sampling[b];
  uint64_t st = state[b];
  for (int j = 0; j < rows; ++j) {
    const int r = r0 + j;
    const RowStat rs = s.stats[r];
    int32_t* out = ids + (int64_t)b * block + j;
    if (rs.flags & 1) {
      *out = -1;
      break;
    }
    const int32_t* sorted = s.idx + (int64_t)r * 2 * vocab;
    const uint32_t* keys = s.keys + (int64_t)r * 2 * vocab;
    int t;
    if (greedy(smp)) {
      t = rs.argmax;
    } else {
      const double* cum = s.cum + (int64_t)r * vocab;
      const double u = (double)splitmix(st) / 9007199254740992.0 * rs.kept;
      int lo = 0, hi = rs.m;  // first index whose running sum exceeds u
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (cum[mid] > u) hi = mid; else lo = mid + 1;
      }
      if (lo >= rs.m) {  // none: the last index with a non-zero probability
        const double last = cum[rs.m - 1];
        lo = 0;
        hi = rs.m - 1;
        while (lo < hi) {
          const int mid = (lo + hi) >> 1;
          if (cum[mid] >= last) hi = mid; else lo = mid + 1;
        }
      }
      t = sorted[lo];
    }
    *out = t;
    if (n_logprobs > 0) {
      float* row = lp + ((int64_t)b * block + j) * width;
      for (int q = 0; q < n_logprobs; ++q) {
        if (q < vocab) {
          row[2 * q] = (float)sorted[q];
          row[2 * q + 1] = (float)((double)key_value(keys[q]) - rs.lse);
        } else {
          row[2 * q] = -1.f;
        }
      }
      row[2 * n_logprobs] = (float)((double)logits[(int64_t)r * vocab + t] - rs.lse);
    }
    if (j + 1 < rows && t != drafts[(int64_t)b * (block - 1) + j]) break;
  }
  state[b] = st;
}

}  // namespace

extern "C" {

size_t hk_sample_workspace_size(int32_t rows, int32_t vocab) {
  if (rows <= 0 || vocab <= 0) return 256;
  return scratch_bytes(rows, vocab);
}

int hk_sample_verify(const float* logits, int32_t vocab, const int32_t* cu_rows, int32_t num_lanes,
                     int32_t num_rows, int32_t block, const hk_sampling* sampling, uint64_t* state,
                     const int32_t* drafts, int32_t n_logprobs, int32_t* ids, float* lp,
                     void* workspace, size_t workspace_bytes, void* stream) {
  HK_TRY(hk::ensure_device());
  HK_REQUIRE(logits && cu_rows && sampling && state && ids && workspace, "hk_sample_verify: null pointer");
  HK_REQUIRE(vocab > 0 && vocab <= kMaxVocab, "hk_sample_verify: vocab %d not in 1..%d", vocab, kMaxVocab);
  HK_REQUIRE(num_lanes > 0 && num_rows >= 0 && block >= 1 && n_logprobs >= 0 && n_logprobs <= 64,
             "hk_sample_verify: bad sizes");
  HK_REQUIRE(block == 1 || drafts != nullptr, "hk_sample_verify: drafts needed for block %d", block);
  HK_REQUIRE(n_logprobs == 0 || lp != nullptr, "hk_sample_verify: lp needed for %d logprobs", n_logprobs);
  HK_REQUIRE((uintptr_t)workspace % 256 == 0, "hk_sample_verify: workspace must be 256-byte aligned");
  const size_t need = hk_sample_workspace_size(num_rows, vocab);
  if (workspace_bytes < need)
    return hk::fail(HK_ESPACE, "hk_sample_verify: workspace of %zu bytes, %zu needed", workspace_bytes, need);
  Scratch s = carve(workspace, num_rows, vocab);
  cudaStream_t st = (cudaStream_t)stream;
  if (num_rows > 0) {
    sample_rows_kernel<<<num_rows, kThreads, 0, st>>>(logits, vocab, cu_rows, num_lanes, num_rows, sampling,
                                                      n_logprobs, s, hk::err_word());
    HK_TRY_LAUNCH("sample_rows_kernel");
  }
  sample_chain_kernel<<<(num_lanes + 63) / 64, 64, 0, st>>>(logits, vocab, cu_rows, num_lanes, block, sampling,
                                                            state, drafts, n_logprobs, ids, lp, s, hk::err_word());
  HK_TRY_LAUNCH("sample_chain_kernel");
  return HK_OK;
}

}  // extern "C"
