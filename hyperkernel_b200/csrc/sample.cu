// Spec-decode verification with on-device sampling: the reply side of the decode step.
//
// Semantics (restated from the reference's source sampler, src/evo2/draw.rs:14-58, and its
// reply reader, src/gpu/feed.rs:163-208):
//   * a lane's rows are its 1 + drafts positions; row j is drawn with the lane's sampling and
//     generator state, and the chain goes on to row j + 1 only while the token drawn equals
//     draft j;
//   * greedy (temperature <= 0 or top_k == 1): the first index of the greatest logit, no draw;
//   * otherwise the row is ordered by value, descending in the IEEE total order, ties in index
//     order; the first top_k are kept (all when top_k == 0); p = softmax(value / temperature)
//     in f64; when 0 < top_p < 1 the tail whose inclusive sum from the bottom is <= 1 - top_p
//     is zeroed; u = splitmix(state) / 2^53 * kept picks the first index whose running sum
//     exceeds u, else the last index with a non-zero probability;
//   * a row with a non-finite logit gives id -1 and ends the lane;
//   * every accepted token gets a logprob row: n (id, logprob) pairs of log-softmax(row) at
//     temperature 1, best first, id -1 past the vocabulary, then the token's own logprob.
//
// A row is drawn before it is known whether the chain reaches it: the state a row j draws
// with is the lane's state advanced j times (splitmix steps by a constant), so every row is
// independent and the chain kernel only compares tokens with drafts and counts the draws.
//
// Per row (one CTA) nothing is sorted in full.  The row's values go into 4096 buckets of
// equal width between its minimum and maximum (a monotone map, so the buckets are in value
// order); a bucket histogram of counts, or of probabilities, finds the bucket where a count
// or a running sum crosses its target, and only the elements up to (or of) that bucket are
// gathered into shared memory and sorted there (bitonic, by total-order key then index):
//   * top-n logprob pairs and the top-k set: the first n / k of the buckets up to the one
//     where the count reaches n / k; with top_k > 0 the whole reference computation then
//     runs on those k entries in shared memory, sums left to right as in the reference;
//   * top_k == 0: the top-p cut and the draw are running-sum crossings over the whole row:
//     bucket sums up to the crossing bucket (f64 exponentials, rounded to 2^-40 and summed
//     exactly as integers), then that bucket's entries in order with the reference's
//     arithmetic.  Those sums are not left to right, so a draw could differ from the
//     reference only where u lies within ~1e-12 of a boundary.
// A crossing bucket with more than kCap elements (near-constant rows) falls back to a full
// stable radix sort of the row in global scratch.
#include <cooperative_groups.h>

#include "common.cuh"

namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxVocab = 1 << 22;
constexpr int kBuckets = 4096;
constexpr int kCap = 8192;            // elements a gather may hold
constexpr int kMaxLogprobs = 64;
constexpr uint64_t kGamma = 0x9E3779B97F4A7C15ull;
constexpr int kDynSmem = kBuckets * (4 + 8) + kCap * 8 + kCap * 8;  // histograms, list, weights

struct RowStat {
  double lse;      // log-sum-exp of the row (temperature 1)
  int32_t argmax;  // first index of the greatest logit
  int32_t token;   // the drawn token (sampled rows)
  int32_t flags;   // 1: a non-finite logit
  int32_t ntop;    // pairs in the row's top list
};

struct Scratch {
  uint32_t* keys;  // [rows][2][vocab]  (full-sort fallback)
  int32_t* idx;    // [rows][2][vocab]
  int32_t* top;    // [rows][kMaxLogprobs] indices, best first
  float* topv;     // [rows][kMaxLogprobs] their logits
  RowStat* stats;  // [rows]
};

size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

size_t scratch_bytes(int32_t rows, int32_t vocab) {
  const size_t nv = (size_t)rows * vocab;
  return align256(nv * 8) + align256(nv * 8) + 2 * align256((size_t)rows * kMaxLogprobs * 4) +
         align256((size_t)rows * sizeof(RowStat));
}

Scratch carve(void* ws, int32_t rows, int32_t vocab) {
  uint8_t* p = reinterpret_cast<uint8_t*>(ws);
  const size_t nv = (size_t)rows * vocab;
  Scratch s;
  s.keys = reinterpret_cast<uint32_t*>(p);
  p += align256(nv * 8);
  s.idx = reinterpret_cast<int32_t*>(p);
  p += align256(nv * 8);
  s.top = reinterpret_cast<int32_t*>(p);
  p += align256((size_t)rows * kMaxLogprobs * 4);
  s.topv = reinterpret_cast<float*>(p);
  p += align256((size_t)rows * kMaxLogprobs * 4);
  s.stats = reinterpret_cast<RowStat*>(p);
  return s;
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

// The draw of the state advanced `steps` + 1 times (src/evo2/draw.rs:52-58).
__device__ __forceinline__ uint64_t splitmix_at(uint64_t state, uint64_t steps) {
  uint64_t z = state + (steps + 1) * kGamma;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return (z ^ (z >> 31)) >> 11;
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

// Block-wide exclusive prefix in thread order (and the total), for doubles and counts.
template <typename T>
__device__ T block_excl(T v, T* red, T* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  T x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const T y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  __syncthreads();
  if (lane == 31) red[warp] = x;
  __syncthreads();
  T before = 0, t = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    if (w < warp) before += red[w];
    t += red[w];
  }
  *total = t;
  return before + x - v;
}

// Sorts list[0..n) ascending (n <= kCap), padding to a power of two with ~0.
__device__ void bitonic(uint64_t* list, int n) {
  int N = 1;
  while (N < n) N <<= 1;
  for (int i = n + (int)threadIdx.x; i < N; i += kThreads) list[i] = ~0ull;
  __syncthreads();
  for (int k = 2; k <= N; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < N; i += kThreads) {
        const int l = i ^ j;
        if (l > i) {
          const uint64_t a = list[i], b = list[l];
          if ((a > b) == ((i & k) == 0)) {
            list[i] = b;
            list[l] = a;
          }
        }
      }
      __syncthreads();
    }
}

__device__ __forceinline__ uint64_t composite(float v, int i) {
  return ((uint64_t)desc_key(v) << 32) | (uint32_t)i;
}

// Calls f(i, x[i]) for this thread's share of the row: 16-byte loads, two in flight, when
// the row allows them.
template <typename F>
__device__ __forceinline__ void for_row(const float* __restrict__ x, int vocab, F f) {
  if ((vocab & 3) == 0 && ((uintptr_t)x & 15) == 0) {
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const int n4 = vocab >> 2;
#pragma unroll 2
    for (int i = threadIdx.x; i < n4; i += kThreads) {
      const float4 v = x4[i];
      f(4 * i, v.x);
      f(4 * i + 1, v.y);
      f(4 * i + 2, v.z);
      f(4 * i + 3, v.w);
    }
  } else {
    for (int i = threadIdx.x; i < vocab; i += kThreads) f(i, x[i]);
  }
}

struct Row {
  const float* x;
  int vocab;
  float xmax, inv_w;
  __device__ __forceinline__ int bucket(float v) const {
    const int b = (int)((xmax - v) * inv_w);
    return b < kBuckets - 1 ? b : kBuckets - 1;
  }
};

// The bucket where the inclusive count prefix reaches `target` (>= 1), and the count before it.
__device__ int count_cross(const uint32_t* hist_c, uint32_t target, uint32_t* before_out, uint32_t* red) {
  constexpr int kPer = kBuckets / kThreads;
  __shared__ int found;
  __shared__ uint32_t found_before;
  const int b0 = threadIdx.x * kPer;
  uint32_t loc = 0;
#pragma unroll
  for (int j = 0; j < kPer; ++j) loc += hist_c[b0 + j];
  uint32_t total;
  uint32_t acc = block_excl<uint32_t>(loc, red, &total);
  if (threadIdx.x == 0) { found = kBuckets - 1; found_before = 0; }
  __syncthreads();
  if (acc < target && acc + loc >= target) {
    for (int j = 0; j < kPer; ++j) {
      const uint32_t c = hist_c[b0 + j];
      if (acc + c >= target) { found = b0 + j; found_before = acc; break; }
      acc += c;
    }
  }
  __syncthreads();
  *before_out = found_before;
  return found;
}

// Bucket weights are fixed point: w * 2^40 rounded (w <= 1, so a row of 4M entries stays
// below 2^62), summed with integer atomics; prefix sums over buckets are then exact.
constexpr double kFix = 1099511627776.0;

// The first bucket whose inclusive weight prefix exceeds `target`, and the weight before it.
__device__ int weight_cross(const unsigned long long* hist_w, double target, double* before_out,
                            unsigned long long* red) {
  constexpr int kPer = kBuckets / kThreads;
  __shared__ int found;
  __shared__ unsigned long long found_before;
  const int b0 = threadIdx.x * kPer;
  unsigned long long loc = 0;
#pragma unroll
  for (int j = 0; j < kPer; ++j) loc += hist_w[b0 + j];
  unsigned long long total;
  unsigned long long acc = block_excl<unsigned long long>(loc, red, &total);
  const double tfix = target * kFix;
  if (threadIdx.x == 0) { found = -1; found_before = 0; }
  __syncthreads();
  if ((double)acc <= tfix && (double)(acc + loc) > tfix) {
    for (int j = 0; j < kPer; ++j) {
      const unsigned long long w = hist_w[b0 + j];
      if ((double)(acc + w) > tfix) { found = b0 + j; found_before = acc; break; }
      acc += w;
    }
  }
  __syncthreads();
  if (found < 0) {  // the target at the very end: the last non-empty bucket
    if (threadIdx.x == 0) {
      unsigned long long a = 0;
      for (int b = 0; b < kBuckets; ++b) {
        if (hist_w[b] > 0) { found = b; found_before = a; }
        a += hist_w[b];
      }
      if (found < 0) found = 0;
    }
    __syncthreads();
  }
  *before_out = (double)found_before / kFix;
  return found;
}

// Stable LSD radix sort of the row's (total-order key, index) pairs in global scratch, 4
// passes of 8 bits; the result is in k0 / i0.  The fallback for near-constant rows.
__device__ void full_sort(const float* x, int vocab, uint32_t* k0, uint32_t* k1, int32_t* i0, int32_t* i1,
                          uint32_t* hist, uint32_t* base, uint32_t* run, uint32_t (*wcnt)[256]) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
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
    if (warp == 0) {
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
      const int e = t * kThreads + tid;
      const bool valid = e < vocab;
      const uint32_t key = valid ? ks[e] : 0u;
      const int32_t ix = valid ? is[e] : 0;
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
}

// The reference draw over m sorted entries, run by one thread with every sum left to right
// (src/evo2/draw.rs:24-48): w(i) = exp(value_i / temperature - value_0 / temperature), id(i)
// the entry's index.
template <typename W, typename I>
__device__ int draw_sorted(int m, W w, I id, const hk_sampling& smp, uint64_t bits) {
  double total = 0.0;
  for (int i = 0; i < m; ++i) total += w(i);
  const double top_p = (double)smp.top_p;
  const bool cut = top_p > 0.0 && top_p < 1.0;
  // the zeroed tail is a suffix: find where it starts, summing from the bottom
  int keep = m;
  if (cut) {
    double below = 0.0;
    for (int i = m - 1; i >= 0; --i) {
      below += w(i) / total;
      if (below <= 1.0 - top_p) keep = i; else break;
    }
  }
  double kept = 0.0;
  for (int i = 0; i < keep; ++i) kept += w(i) / total;
  const double u = (double)bits / 9007199254740992.0 * kept;
  double seen = 0.0;
  for (int i = 0; i < keep; ++i) {
    seen += w(i) / total;
    if (u < seen) return id(i);
  }
  // the last index with a non-zero probability
  for (int i = keep - 1; i >= 0; --i)
    if (w(i) / total > 0.0) return id(i);
  return id(0);
}

// One cluster of CTAs per row: each CTA reads a contiguous slice of the row, the slices'
// histograms are merged over distributed shared memory, and the gathers land in the first
// CTA's list, which sorts and draws.  Every read of another CTA's shared memory is followed
// by a cluster barrier before that memory changes or its CTA leaves.
__global__ void __launch_bounds__(kThreads) sample_rows_kernel(
    const float* __restrict__ logits, int32_t vocab, const int32_t* __restrict__ cu, int32_t lanes,
    int32_t rows, const hk_sampling* __restrict__ sampling, const uint64_t* __restrict__ state,
    int32_t n_logprobs, Scratch s, unsigned long long* err) {
  namespace cg = cooperative_groups;
  extern __shared__ __align__(16) uint8_t dyn[];
  uint32_t* hist_c = reinterpret_cast<uint32_t*>(dyn);
  unsigned long long* hist_w = reinterpret_cast<unsigned long long*>(dyn + kBuckets * 4);
  uint64_t* list = reinterpret_cast<uint64_t*>(dyn + kBuckets * 12);
  double* wbuf = reinterpret_cast<double*>(dyn + kBuckets * 12 + kCap * 8);
  __shared__ uint32_t shist[256], sbase[256], srun[256];
  __shared__ uint32_t wcnt[kWarps][256];
  __shared__ double red[kWarps];
  __shared__ uint32_t redu[kWarps];
  __shared__ unsigned long long redl[kWarps];
  __shared__ float smax[kWarps], smin[kWarps];
  __shared__ int sarg[kWarps], sbad[kWarps];
  __shared__ int list_n, result;
  __shared__ float p_max, p_min;       // this CTA's slice: max, min, first argmax, non-finite
  __shared__ int p_arg, p_bad;
  __shared__ double p_e, res_incl;     // slice log-sum-exp partial; the leader's crossing sum
  cg::cluster_group cl = cg::this_cluster();
  const int C = (int)cl.num_blocks(), rank = (int)cl.block_rank();
  const int r = blockIdx.x / C;
  if (r >= rows) return;  // whole clusters only: rows * C blocks are launched
  const bool leader = rank == 0;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = lane_of(cu, lanes, r);
  const hk_sampling smp = sampling[b];
  const int j = r - cu[b];  // the row's position in its lane: draws before it
  const float* x = logits + (int64_t)r * vocab;
  RowStat* st = s.stats + r;
  // this CTA's slice, a multiple of 4 entries long
  const int seg = (((vocab + C - 1) / C) + 3) & ~3;
  const int lo = min(vocab, rank * seg), hi = min(vocab, lo + seg);
  auto for_slice = [&](auto f) { for_row(x + lo, hi - lo, [&](int i, float v) { f(lo + i, v); }); };

  // ---- maximum (first index), minimum, finiteness: slices, then merged in rank order
  float mx = -INFINITY, mn = INFINITY;
  int arg = 0x7fffffff, bad = 0;
  for_slice([&](int i, float v) {
    if (!isfinite(v)) { bad = 1; return; }
    if (v > mx || (v == mx && i < arg)) { mx = v; arg = i; }
    mn = fminf(mn, v);
  });
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, mx, o);
    const int a2 = __shfl_xor_sync(0xffffffffu, arg, o);
    if (m2 > mx || (m2 == mx && a2 < arg)) { mx = m2; arg = a2; }
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    bad |= __shfl_xor_sync(0xffffffffu, bad, o);
  }
  if (lane == 0) { smax[warp] = mx; smin[warp] = mn; sarg[warp] = arg; sbad[warp] = bad; }
  __syncthreads();
  if (tid == 0) {
    float m = smax[0], n_ = smin[0];
    int a = sarg[0], bd = sbad[0];
    for (int w = 1; w < kWarps; ++w) {
      if (smax[w] > m || (smax[w] == m && sarg[w] < a)) { m = smax[w]; a = sarg[w]; }
      n_ = fminf(n_, smin[w]);
      bd |= sbad[w];
    }
    p_max = m; p_min = n_; p_arg = a; p_bad = bd;
  }
  cl.sync();
  mx = -INFINITY; mn = INFINITY; arg = 0x7fffffff; bad = 0;
  for (int q = 0; q < C; ++q) {
    const float m2 = *cl.map_shared_rank(&p_max, q);
    const int a2 = *cl.map_shared_rank(&p_arg, q);
    if (m2 > mx || (m2 == mx && a2 < arg)) { mx = m2; arg = a2; }
    mn = fminf(mn, *cl.map_shared_rank(&p_min, q));
    bad |= *cl.map_shared_rank(&p_bad, q);
  }
  if (bad) {
    if (leader && tid == 0) { st->flags = 1; st->argmax = 0; st->token = -1; st->ntop = 0; st->lse = 0.0; }
    cl.sync();  // every CTA has read the others' partials before any leaves
    return;
  }
  // Replaces this CTA's histograms with the cluster's sums (bins tid, tid + kThreads, ...).
  auto merge_hist = [&](bool weights) {
    constexpr int kPer = kBuckets / kThreads;
    uint32_t mc[kPer];
    unsigned long long mw[kPer];
    for (int q = 0; q < kPer; ++q) { mc[q] = 0u; mw[q] = 0ull; }
    cl.sync();
    for (int o = 0; o < C; ++o) {
      const uint32_t* rc = cl.map_shared_rank(hist_c, o);
      const unsigned long long* rw = cl.map_shared_rank(hist_w, o);
      for (int q = 0; q < kPer; ++q) {
        mc[q] += rc[tid + q * kThreads];
        if (weights) mw[q] += rw[tid + q * kThreads];
      }
    }
    cl.sync();
    for (int q = 0; q < kPer; ++q) {
      hist_c[tid + q * kThreads] = mc[q];
      if (weights) hist_w[tid + q * kThreads] = mw[q];
    }
    __syncthreads();
  };
  double lse = 0.0;  // log-sum-exp for the logprob rows (computed with the top-n pass)
  const bool sampled = !greedy(smp);
  const Row row{x, vocab, mx, mx > mn ? (float)kBuckets / (mx - mn) : 0.f};
  const int n = min(n_logprobs, vocab);
  const int k = sampled && smp.top_k > 0 ? (int)min((uint32_t)vocab, smp.top_k) : 0;
  const uint64_t bits = sampled ? splitmix_at(state[b], (uint64_t)j) : 0ull;
  int token = arg;
  bool sorted_full = false;
  uint32_t* k0 = s.keys + (int64_t)r * 2 * vocab;
  int32_t* i0 = s.idx + (int64_t)r * 2 * vocab;
  uint64_t* list0 = cl.map_shared_rank(list, 0);
  int* list_n0 = cl.map_shared_rank(&list_n, 0);

  // ---- the top max(n, k) in order: buckets up to the count crossing, gathered and sorted
  const int c = max(n, k);
  if (c > 0) {
    for (int i = tid; i < kBuckets; i += kThreads) hist_c[i] = 0u;
    __syncthreads();
    // single-precision exponentials (one rounding each) summed in f64 for the log-sum-exp
    double e = 0.0;
    for_slice([&](int, float v) {
      atomicAdd(&hist_c[row.bucket(v)], 1u);
      if (n > 0) e += (double)expf(v - mx);
    });
    const double e_cta = block_sum(e, red);  // its barriers close the histogram
    if (tid == 0) p_e = e_cta;
    if (leader && tid == 0) list_n = 0;  // the gather below starts after the merge's barriers
    merge_hist(false);  // begins with a cluster barrier, so every p_e is in place
    double e_all = 0.0;
    for (int q = 0; q < C; ++q) e_all += *cl.map_shared_rank(&p_e, q);
    lse = (double)mx + log(e_all);
    uint32_t before;
    const int bc = count_cross(hist_c, (uint32_t)c, &before, redu);
    const uint32_t upto = before + hist_c[bc];  // elements in buckets 0..bc
    if (upto <= (uint32_t)kCap) {
      for_slice([&](int i, float v) {
        if (row.bucket(v) <= bc) list0[atomicAdd(list_n0, 1)] = composite(v, i);
      });
      cl.sync();
      if (leader) {
        bitonic(list, (int)upto);
        for (int q = tid; q < n; q += kThreads) {
          const uint64_t L = list[q];
          s.top[(int64_t)r * kMaxLogprobs + q] = (int32_t)(uint32_t)L;
          s.topv[(int64_t)r * kMaxLogprobs + q] = key_value((uint32_t)(L >> 32));
        }
        if (k > 0) {  // the exponentials in parallel, the sums by one thread in order
          const double temp = (double)smp.temperature;
          const double most = (double)key_value((uint32_t)(list[0] >> 32)) / temp;
          for (int q = tid; q < k; q += kThreads)
            wbuf[q] = exp((double)key_value((uint32_t)(list[q] >> 32)) / temp - most);
          __syncthreads();
          if (tid == 0)
            token = draw_sorted(
                k, [&](int i) { return wbuf[i]; }, [&](int i) { return (int)(uint32_t)list[i]; }, smp, bits);
        }
      }
    } else {
      sorted_full = true;
      if (leader) {
        full_sort(x, vocab, k0, k0 + vocab, i0, i0 + vocab, shist, sbase, srun, wcnt);
        for (int q = tid; q < n; q += kThreads) {
          s.top[(int64_t)r * kMaxLogprobs + q] = i0[q];
          s.topv[(int64_t)r * kMaxLogprobs + q] = key_value(k0[q]);
        }
        if (k > 0 && tid == 0)
          token = draw_sorted(
              k, [&](int i) { return exp((double)key_value(k0[i]) / (double)smp.temperature -
                                    (double)key_value(k0[0]) / (double)smp.temperature); },
              [&](int i) { return i0[i]; }, smp, bits);
      }
    }
  }

  // ---- top_k == 0: the top-p cut and the draw as running-sum crossings over the whole row
  if (sampled && k == 0) {
    const double temp = (double)smp.temperature;
    const double most = (double)mx / temp;
    if (sorted_full) {
      if (leader && tid == 0)
        token = draw_sorted(
            vocab, [&](int i) { return exp((double)key_value(k0[i]) / (double)smp.temperature -
                                  (double)key_value(k0[0]) / (double)smp.temperature); },
            [&](int i) { return i0[i]; }, smp, bits);
    } else {
      for (int i = tid; i < kBuckets; i += kThreads) { hist_c[i] = 0u; hist_w[i] = 0ull; }
      __syncthreads();
      // The sum of the buckets before the crossing one shifts every running sum inside it, so
      // a draw agrees with the reference only if that sum is accurate to far below the
      // probability of one entry: f64 exponentials (the fixed point adds ~1e-12).
      const double inv_t = 1.0 / temp;
      for_slice([&](int, float v) {
        const int bk = row.bucket(v);
        const unsigned long long w = __double2ull_rn(exp((double)v * inv_t - most) * kFix);
        atomicAdd(&hist_c[bk], 1u);
        atomicAdd(&hist_w[bk], w);
      });
      __syncthreads();
      if (leader && tid == 0) list_n = 0;  // the first crossing's gather follows the merge's barriers
      merge_hist(true);
      unsigned long long loc = 0;
      for (int q = tid; q < kBuckets; q += kThreads) loc += hist_w[q];
      unsigned long long tot_fix;
      block_excl<unsigned long long>(loc, redl, &tot_fix);
      const double total = (double)tot_fix / kFix;
      // Running-sum crossing of `target` (unnormalised): the element, and the sum through it.
      auto cross = [&](double target, double* incl) -> int {
        double before;
        const int bk = weight_cross(hist_w, target, &before, redl);
        const uint32_t cnt = hist_c[bk];
        __syncthreads();
        if (cnt > (uint32_t)kCap) return -1;
        // the leader's list count is 0 here: reset before a barrier that preceded this call
        for_slice([&](int i, float v) {
          if (row.bucket(v) == bk) list0[atomicAdd(list_n0, 1)] = composite(v, i);
        });
        cl.sync();
        if (leader) {
          bitonic(list, (int)cnt);
          for (uint32_t q = tid; q < cnt; q += kThreads)
            wbuf[q] = exp((double)key_value((uint32_t)(list[q] >> 32)) / temp - most);
          __syncthreads();
          if (tid == 0) {
            double acc = before;
            int pick = -1;
            for (uint32_t q = 0; q < cnt; ++q) {
              acc += wbuf[q];
              if (acc > target) { pick = (int)(uint32_t)list[q]; break; }
            }
            if (pick < 0 && cnt > 0) pick = (int)(uint32_t)list[cnt - 1];
            result = pick;
            res_incl = acc;
          }
        }
        cl.sync();
        *incl = *cl.map_shared_rank(&res_incl, 0);
        const int out = *cl.map_shared_rank(&result, 0);
        if (leader && tid == 0) list_n = 0;  // for the next crossing's gather, after the barrier below
        cl.sync();
        return out;
      };
      double kept = total;
      bool ok = true;
      const double top_p = (double)smp.top_p;
      if (top_p > 0.0 && top_p < 1.0) {
        double incl;
        ok = cross(top_p * total, &incl) >= 0;
        kept = incl;
      }
      if (ok) {
        double incl;
        const int t = cross((double)bits / 9007199254740992.0 * kept, &incl);
        ok = t >= 0;
        token = t;
      }
      if (!ok && leader) {  // a crossing bucket too full to gather: sort the row
        full_sort(x, vocab, k0, k0 + vocab, i0, i0 + vocab, shist, sbase, srun, wcnt);
        if (tid == 0)
          token = draw_sorted(
              vocab, [&](int i) { return exp((double)key_value(k0[i]) / (double)smp.temperature -
                                  (double)key_value(k0[0]) / (double)smp.temperature); },
              [&](int i) { return i0[i]; }, smp, bits);
      }
    }
  }
  if (leader && tid == 0) {
    st->flags = 0;
    st->argmax = arg;
    st->token = sampled ? token : arg;
    st->ntop = n;
    st->lse = lse;
  }
  cl.sync();  // no CTA leaves while another may still read its shared memory
}

// One warp per lane: lane 0 walks the chain, then the warp writes the ids and logprob rows.
// One warp per lane, one row per thread (block <= 32): every row's statistics and draft are
// loaded at once, the accepted prefix is a ballot (the chain stops at the first non-finite
// row, or at the first row whose token differs from the next row's draft), and the logprob
// rows are written by the whole warp, (row, pair) by (row, pair).
__global__ void sample_chain_kernel(const float* __restrict__ logits, int32_t vocab,
                                    const int32_t* __restrict__ cu, int32_t lanes, int32_t block,
                                    const hk_sampling* __restrict__ sampling, uint64_t* state,
                                    const int32_t* __restrict__ drafts, int32_t n_logprobs,
                                    int32_t* __restrict__ ids, float* __restrict__ lp, Scratch s,
                                    unsigned long long* err) {
  const int b = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  const int t32 = threadIdx.x & 31;
  if (b >= lanes) return;  // whole warps
  const int width = 2 * n_logprobs + 1;
  const int r0 = cu[b], rows = cu[b + 1] - r0;
  if (rows < 0 || rows > block) {
    if (t32 == 0) hk_flag(err, hk::kErrMoeRow, (unsigned)b);
    for (int j = t32; j < block; j += 32) ids[(int64_t)b * block + j] = -2;
    return;
  }
  RowStat rs{};
  int draft = 0;
  const bool in = t32 < rows;
  if (in) {
    rs = s.stats[r0 + t32];
    if (t32 + 1 < rows) draft = drafts[(int64_t)b * (block - 1) + t32];
  }
  const bool bad = in && (rs.flags & 1);
  const bool stop = bad || (in && t32 + 1 < rows && rs.token != draft);
  const unsigned stops = __ballot_sync(0xffffffffu, stop);
  const unsigned bads = __ballot_sync(0xffffffffu, bad);
  const int m = rows == 0 ? 0 : (stops ? __ffs(stops) : rows);   // accepted rows
  const int last_bad = m > 0 ? (int)((bads >> (m - 1)) & 1u) : 0;
  if (t32 == 0) state[b] += (greedy(sampling[b]) ? 0ull : (uint64_t)(m - last_bad)) * kGamma;
  if (t32 < block) {
    int32_t v = -2;
    if (t32 < m) v = (t32 == m - 1 && last_bad) ? -1 : rs.token;
    ids[(int64_t)b * block + t32] = v;
  }
  if (n_logprobs == 0) return;
  const int live_rows = m - last_bad;  // rows 0 .. live_rows-1 carry logprobs
  const int pairs = block * n_logprobs;
  for (int base = 0; base < pairs; base += 32) {  // warp-uniform trip count: the shuffles see all lanes
    const int idx = base + t32;
    const int j = idx < pairs ? idx / n_logprobs : 0, q = idx < pairs ? idx % n_logprobs : 0;
    const double lse_j = __shfl_sync(0xffffffffu, rs.lse, j);
    const int ntop_j = __shfl_sync(0xffffffffu, rs.ntop, j);
    if (idx >= pairs) continue;
    float* row = lp + ((int64_t)b * block + j) * width;
    const int r = r0 + j;
    if (j >= live_rows) {
      row[2 * q] = 0.f;
      row[2 * q + 1] = 0.f;
    } else if (q < ntop_j) {
      row[2 * q] = (float)s.top[(int64_t)r * kMaxLogprobs + q];
      row[2 * q + 1] = (float)((double)s.topv[(int64_t)r * kMaxLogprobs + q] - lse_j);
    } else {
      row[2 * q] = -1.f;
      row[2 * q + 1] = 0.f;
    }
  }
  if (t32 < block) {
    float* row = lp + ((int64_t)b * block + t32) * width;
    row[2 * n_logprobs] =
        t32 < live_rows ? (float)((double)logits[(int64_t)(r0 + t32) * vocab + rs.token] - rs.lse) : 0.f;
  }
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
  HK_REQUIRE((num_rows == 0 || (logits && workspace)) && cu_rows && sampling && state && ids,
             "hk_sample_verify: null pointer");
  HK_REQUIRE(vocab > 0 && vocab <= kMaxVocab, "hk_sample_verify: vocab %d not in 1..%d", vocab, kMaxVocab);
  HK_REQUIRE(num_lanes > 0 && num_rows >= 0 && block >= 1 && block <= 32 && n_logprobs >= 0 &&
                 n_logprobs <= kMaxLogprobs,
             "hk_sample_verify: bad sizes (block 1..32, at most %d logprobs)", kMaxLogprobs);
  HK_REQUIRE(block == 1 || num_rows == 0 || drafts != nullptr, "hk_sample_verify: drafts needed for block %d",
             block);
  HK_REQUIRE(n_logprobs == 0 || lp != nullptr, "hk_sample_verify: lp needed for %d logprobs", n_logprobs);
  HK_REQUIRE((uintptr_t)workspace % 256 == 0, "hk_sample_verify: workspace must be 256-byte aligned");
  const size_t need = hk_sample_workspace_size(num_rows, vocab);
  if (workspace_bytes < need)
    return hk::fail(HK_ESPACE, "hk_sample_verify: workspace of %zu bytes, %zu needed", workspace_bytes, need);
  Scratch s = carve(workspace, num_rows, vocab);
  cudaStream_t st = (cudaStream_t)stream;
  static bool attr = false;
  if (!attr) {
    HK_TRY_CUDA(cudaFuncSetAttribute(sample_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kDynSmem));
    attr = true;
  }
  if (num_rows > 0) {
    // a cluster of up to 8 CTAs per row, as many as the SMs allow in one wave
    int per_row = hk::sm_count() / num_rows;
    per_row = per_row < 1 ? 1 : per_row > 8 ? 8 : per_row;
    if (per_row > vocab / 4) per_row = vocab / 4 > 0 ? vocab / 4 : 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(num_rows * per_row));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kDynSmem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)per_row;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    HK_TRY_CUDA(cudaLaunchKernelEx(&cfg, sample_rows_kernel, logits, vocab, cu_rows, num_lanes, num_rows, sampling,
                                   (const uint64_t*)state, n_logprobs, s, hk::err_word()));
    hk::note_launch();
  }
  sample_chain_kernel<<<(num_lanes + 3) / 4, 128, 0, st>>>(logits, vocab, cu_rows, num_lanes, block, sampling,
                                                            state, drafts, n_logprobs, ids, lp, s, hk::err_word());
  HK_TRY_LAUNCH("sample_chain_kernel");
  return HK_OK;
}

}  // extern "C"
