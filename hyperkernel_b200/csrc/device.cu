// The device kernel behind the Kernel boundary: hk_open / hk_pools / hk_push / hk_drain,
// plus the request-ring encoder hk_encode_share and hk_kernel_ops_of.
//
// The reference's Feed (src/gpu/feed.rs:132-161) encodes each command into a mapped request
// ring that a persistent megakernel polls.  This build keeps the ring's encoding (wire.h,
// encoded by layout as ring::encode does, src/gpu/ring.rs:99-125) but not the polling: hk_push
// queues the share's commands with their step, and hk_drain applies the commands due at each
// step in one kernel over the encoded stream (one host->device copy per batch), then runs the
// granted decode steps.  State lives on the device: the block-table rows (pages ++ window
// pages per lane, as Command::Pages writes them), the lanes' positions / reserved rows /
// live flags, the paged token pool and the window page pool.
//
// The model is the reference's test model (tests/engine.rs:56-62 `next`): the next token of a
// sequence is an FNV-style fold of (token + 1000 * position), read back through the lane's
// block-table row from the pools.  Every read checks what the reference's test device asserts
// (tests/engine.rs:105-128, :153-160, :184): no write to the scratch page, no read of an
// unwritten position, window pages present and equal to the pages over the last page_rows
// positions, no decode at the idle position.  A violation is recorded in the handle's error
// words and fails hk_drain with the reference's wording.  The step/apply semantics (which
// commands wait for their step, when Idle is reported, how far the device may run) follow the
// test device's run loop, tests/engine.rs:130-211.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <deque>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"
#include "model.cuh"
#include "wire.h"

namespace {

using namespace hk::wire;

struct LaneState {
  int32_t upto, pos, live, tok;
};

struct LaneSampling {
  float temperature, top_p;
  uint32_t top_k, logprobs;
  uint32_t seed_lo, seed_hi;
  int32_t back[3];
  int32_t reserved;
};

enum ModelFault : unsigned {
  kFaultScratchWrite = 1,
  kFaultUnwritten = 2,
  kFaultWindowScratch = 3,
  kFaultWindowMismatch = 4,
  kFaultIdle = 5,
  kFaultChunkWindow = 6,
  kFaultPagePastPool = 7,
  kFaultMessage = 8,
};

struct Dev {
  int32_t* rows;       // [width][entries + window]
  int32_t* pool;       // [pages][page_rows], -1 = unwritten
  int32_t* windows;    // [window_pages][page_rows]
  LaneState* lanes;    // [width]
  LaneSampling* sampling;  // [width]
  unsigned long long* err;  // [0] flag word, [1] lane, [2] position
  int32_t width, entries, window, page_rows, context, chunk, block;
  int64_t pages, window_pages;
  hk_sampling* mla_sampling;  // HK_MODEL_MLA: the sampler's per-lane settings (Seat writes them)
  uint64_t* mla_state;        // HK_MODEL_MLA: per-lane generator state (Seat seeds it)
};

__device__ void fault(const Dev& d, unsigned site, int lane, long long pos) {
  const unsigned long long v = (1ull << 63) | ((unsigned long long)site << 32);
  if (atomicCAS(d.err, 0ull, v) == 0ull) {
    d.err[1] = (unsigned long long)lane;
    d.err[2] = (unsigned long long)pos;
  }
}

// The page of position p in the lane's row (entries first); -1 after recording a fault.
__device__ int64_t page_of(const Dev& d, int lane, long long p) {
  const long long k = p / d.page_rows;
  if (p < 0 || k >= d.entries) {
    fault(d, kFaultPagePastPool, lane, p);
    return -1;
  }
  const int32_t page = d.rows[(size_t)lane * (d.entries + d.window) + k];
  if (page < 0 || page >= d.pages) {
    fault(d, kFaultPagePastPool, lane, p);
    return -1;
  }
  return page;
}

__device__ int64_t window_of(const Dev& d, int lane, long long p) {
  const long long k = p / d.page_rows;
  if (p < 0 || k >= d.window) {
    fault(d, kFaultPagePastPool, lane, p);
    return -1;
  }
  const int32_t w = d.rows[(size_t)lane * (d.entries + d.window) + d.entries + k];
  if (w < 0 || w >= d.window_pages) {
    fault(d, kFaultPagePastPool, lane, p);
    return -1;
  }
  return w;
}

// Fake::write (tests/engine.rs:105-113): the page must not be the scratch page; the window
// page, when present, mirrors the token.
__device__ bool write_token(const Dev& d, int lane, long long p, int32_t t) {
  const int64_t page = page_of(d, lane, p);
  const int64_t w = window_of(d, lane, p);
  if (page < 0 || w < 0) return false;
  if (page == 0) {
    fault(d, kFaultScratchWrite, lane, p);
    return false;
  }
  d.pool[page * d.page_rows + p % d.page_rows] = t;
  if (w != 0) d.windows[w * d.page_rows + p % d.page_rows] = t;
  return true;
}

// The failure a read of position p through the lane's row would record (page_of, then the
// pool read), without recording it; the token in *v when it returns 0.
__device__ __forceinline__ unsigned token_at(const Dev& d, int64_t rowbase, long long p, int32_t* v) {
  const long long k = p / d.page_rows;
  if (k >= d.entries) return kFaultPagePastPool;
  const int32_t page = d.rows[rowbase + k];
  if (page < 0 || page >= d.pages) return kFaultPagePastPool;
  *v = d.pool[(int64_t)page * d.page_rows + p % d.page_rows];
  if (page == 0 || *v < 0) return kFaultUnwritten;
  return 0;
}

// The failure the window check of position q would record (window_of, the scratch window
// page, page_of, then the mirror comparison), without recording it.
__device__ __forceinline__ unsigned window_at(const Dev& d, int64_t rowbase, long long q) {
  const long long k = q / d.page_rows;
  if (k >= d.window) return kFaultPagePastPool;
  const int32_t w = d.rows[rowbase + d.entries + k];
  if (w < 0 || w >= d.window_pages) return kFaultPagePastPool;
  if (w == 0) return kFaultWindowScratch;
  if (k >= d.entries) return kFaultPagePastPool;
  const int32_t page = d.rows[rowbase + k];
  if (page < 0 || page >= d.pages) return kFaultPagePastPool;
  if (d.windows[(int64_t)w * d.page_rows + q % d.page_rows] != d.pool[(int64_t)page * d.page_rows + q % d.page_rows])
    return kFaultWindowMismatch;
  return 0;
}

constexpr int kPerThread = 4;  // positions each thread reads per chunk of model_token_warp

// Fake::token (tests/engine.rs:115-128) with `next` (:56-62), by one warp: reads positions
// 0..=last back through the row, checks the window over the last page_rows positions and
// folds (the fold state in *h_out; token_of maps it to the token).  Each chunk of 32 x kPerThread positions is read by the 32 threads at once; the
// first failing position of the chunk in position order records its fault (so the fault is
// the one the sequential read-back meets first), and the fold runs over the chunk's values
// in position order.  Every thread returns the same result.
__device__ bool fold_warp(const Dev& d, int lane, long long last, unsigned long long* h_out) {
  const int t = threadIdx.x & 31;
  const int64_t rowbase = (int64_t)lane * (d.entries + d.window);
  unsigned long long h = 1469598103ull;
  for (long long base = 0; base <= last; base += 32 * kPerThread) {
    int32_t v[kPerThread];
    unsigned code[kPerThread];
#pragma unroll
    for (int j = 0; j < kPerThread; ++j) {
      const long long p = base + 32 * j + t;
      v[j] = 0;
      code[j] = p <= last ? token_at(d, rowbase, p, &v[j]) : 0u;
    }
#pragma unroll
    for (int j = 0; j < kPerThread; ++j) {
      const unsigned bad = __ballot_sync(0xffffffffu, code[j] != 0);
      if (bad) {
        const int f = __ffs(bad) - 1;
        if (t == f) fault(d, code[j], lane, base + 32 * j + f);
        return false;
      }
    }
#pragma unroll
    for (int j = 0; j < kPerThread; ++j) {
      const long long p0 = base + 32 * j;
      const long long n = last - p0 + 1;  // positions of this row of the chunk (may be <= 0)
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int32_t vi = __shfl_sync(0xffffffffu, v[j], i);
        if (i < n) h = (h ^ ((unsigned long long)(uint32_t)vi + 1000ull * (unsigned long long)(p0 + i))) *
                       1099511628211ull;
      }
    }
  }
  const long long first = last + 1 > d.page_rows ? last + 1 - d.page_rows : 0;
  for (long long base = first; base <= last; base += 32) {
    const long long q = base + t;
    const unsigned code = q <= last ? window_at(d, rowbase, q) : 0u;
    const unsigned bad = __ballot_sync(0xffffffffu, code != 0);
    if (bad) {
      const int f = __ffs(bad) - 1;
      if (t == f) fault(d, code, lane, base + f);
      return false;
    }
  }
  *h_out = h;
  return true;
}

__device__ __forceinline__ int32_t token_of(unsigned long long h) { return (int32_t)(h % 400ull) + 10; }

__device__ bool model_token_warp(const Dev& d, int lane, long long last, int32_t* out) {
  unsigned long long h;
  if (!fold_warp(d, lane, last, &h)) return false;
  *out = token_of(h);
  return true;
}

// The read-back of a sequence one position longer than the last one checked in this step:
// positions before p passed the previous read-back and only this lane writes them, so
// reading position p, folding it and checking its window slot gives the same token and
// the same fault as reading the whole sequence again.  Every thread of the warp computes it.
__device__ bool fold_one(const Dev& d, int lane, long long p, unsigned long long* h) {
  const int64_t rowbase = (int64_t)lane * (d.entries + d.window);
  int32_t v = 0;
  unsigned code = token_at(d, rowbase, p, &v);
  if (code == 0) code = window_at(d, rowbase, p);
  if (code != 0) {
    if ((threadIdx.x & 31) == 0) fault(d, code, lane, p);
    return false;
  }
  *h = (*h ^ ((unsigned long long)(uint32_t)v + 1000ull * (unsigned long long)p)) * 1099511628211ull;
  return true;
}

__device__ __forceinline__ uint32_t rd32(const uint8_t* b, uint32_t at) {
  uint32_t v;
  memcpy(&v, b + at, 4);
  return v;
}
__device__ __forceinline__ uint64_t rd64(const uint8_t* b, uint32_t at) {
  uint64_t v;
  memcpy(&v, b + at, 8);
  return v;
}

// Applies n_msgs encoded commands in order (one CTA; commands of a batch can depend on each
// other, e.g. a Seat then the Prompt of the same lane).  Prompt replies go to replies[] in
// order.
// Applies n_msgs messages of an encoded stream (every thread of one CTA calls it).
__device__ void apply_messages(const Dev& d, const uint8_t* stream, uint64_t stream_bytes, int n_msgs,
                               int32_t* replies) {
  __shared__ int s_lane, s_pos, s_ok, s_reply;
  int n_replies = 0;
  for (int m = 0; m < n_msgs; ++m) {
    const uint8_t* slot = stream + (size_t)m * kSlot;
    const uint8_t* body = slot + kBodyAt;
    const uint32_t id = rd32(slot, 0);
    if (id == kIdPages) {
      const uint32_t lane = rd32(body, kPagesLane), from = rd32(body, kPagesFrom);
      const uint64_t addr = rd64(body, kPagesRow), n = rd64(body, kPagesRow + 8);
      const bool ok = lane < (uint32_t)d.width && from + n <= (uint64_t)(d.entries + d.window) &&
                      addr + 4 * n <= stream_bytes;
      if (!ok) {
        if (threadIdx.x == 0) fault(d, kFaultMessage, (int)lane, m);
      } else {
        const int32_t* src = reinterpret_cast<const int32_t*>(stream + addr);
        int32_t* dst = d.rows + (size_t)lane * (d.entries + d.window) + from;
        for (uint64_t i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
        if (threadIdx.x == 0) d.lanes[lane].upto = (int32_t)rd32(body, kPagesUpto);
      }
    } else if (id == kIdPrompt) {
      if (threadIdx.x == 0) {
        const uint32_t lane = rd32(body, kPromptLane), lens = rd32(body, kPromptLens);
        const uint64_t addr = rd64(body, kPromptTokens);
        s_ok = lane < (uint32_t)d.width && lens >= 1 && lens <= (uint32_t)d.chunk &&
               addr + 4ull * lens <= stream_bytes;
        if (!s_ok) fault(d, kFaultMessage, (int)lane, m);
        s_lane = (int)lane;
        s_pos = s_ok ? d.lanes[lane].pos : 0;
      }
      __syncthreads();
      if (s_ok) {
        const uint32_t lens = rd32(body, kPromptLens);
        const int32_t* toks = reinterpret_cast<const int32_t*>(stream + rd64(body, kPromptTokens));
        for (uint32_t j = threadIdx.x; j < lens; j += blockDim.x) {
          const long long p = (long long)s_pos + j;
          const int64_t w = window_of(d, s_lane, p);
          if (w == 0) fault(d, kFaultChunkWindow, s_lane, p);
          if (w > 0) write_token(d, s_lane, p, toks[j]);
        }
        __syncthreads();
        if (threadIdx.x < 32) {  // the first warp reads the chunk's sequence back
          const long long end = (long long)s_pos + lens;
          int32_t t = -1;
          model_token_warp(d, s_lane, end - 1, &t);
          if (threadIdx.x == 0) {
            d.lanes[s_lane].pos = (int32_t)end;
            d.lanes[s_lane].tok = t;
            s_reply = t;
          }
        }
        __syncthreads();
        if (threadIdx.x == 0) replies[n_replies] = s_reply;
      }
      ++n_replies;
    } else if (threadIdx.x == 0) {
      if (id == kIdEnd) {
        const uint32_t lane = rd32(body, kEndLane);
        if (lane < (uint32_t)d.width) {
          d.lanes[lane].live = 0;
          d.lanes[lane].upto = 0;
        } else {
          fault(d, kFaultMessage, (int)lane, m);
        }
      } else if (id == kIdSeat) {
        const uint32_t lane = rd32(body, kSeatLane);
        if (lane < (uint32_t)d.width) {
          d.lanes[lane].pos = (int32_t)rd32(body, kSeatPos);
          LaneSampling s;
          s.temperature = __uint_as_float(rd32(body, kSeatTemp));
          s.top_p = __uint_as_float(rd32(body, kSeatTopP));
          s.top_k = rd32(body, kSeatTopK);
          s.logprobs = rd32(body, kSeatLogprobs);
          s.seed_lo = rd32(body, kSeatSeedLo);
          s.seed_hi = rd32(body, kSeatSeedHi);
          for (int j = 0; j < 3; ++j) s.back[j] = (int32_t)rd32(body, kSeatBack + 4 * j);
          s.reserved = 0;
          d.sampling[lane] = s;
          if (d.mla_sampling) {
            hk_sampling hs;
            hs.temperature = s.temperature;
            hs.top_p = s.top_p;
            hs.top_k = s.top_k;
            hs.logprobs = s.logprobs;
            hs.seed = ((uint64_t)s.seed_hi << 32) | s.seed_lo;
            d.mla_sampling[lane] = hs;
            d.mla_state[lane] = hs.seed;
          }
        } else {
          fault(d, kFaultMessage, (int)lane, m);
        }
      } else if (id == kIdStart) {
        const uint32_t lane = rd32(body, kStartLane);
        if (lane < (uint32_t)d.width)
          d.lanes[lane].live = 1;
        else
          fault(d, kFaultMessage, (int)lane, m);
      } else {
        fault(d, kFaultMessage, -1, m);
      }
    }
    __syncthreads();
  }
}

__global__ void apply_kernel(Dev d, const uint8_t* stream, uint64_t stream_bytes, int n_msgs,
                             int32_t* replies) {
  apply_messages(d, stream, stream_bytes, n_msgs, replies);
}

// One decode step (the test device's step, tests/engine.rs:173-193): each live lane with
// reserved rows left emits 1 + ((step + lane) mod block) tokens, stopping early at its
// reserved rows or the context's last position.  out[lane][block], -2 past a lane's tokens.
// One decode step of lane l by one warp: the lane state and the writes by thread 0; the
// first token of the step reads the whole sequence back (fold_warp), each further token
// extends that read-back by its one new position (fold_one).
__device__ void step_lane(const Dev& d, uint32_t step, int l, int32_t* out) {
  const int t = threadIdx.x & 31;
  int32_t* o = out + (size_t)l * d.block;
  for (int k = t; k < d.block; k += 32) o[k] = -2;
  const LaneState st = d.lanes[l];
  if (!(st.live && st.pos < st.upto)) return;
  const int c = (int)(((unsigned long long)step + (unsigned long long)l) % (unsigned long long)d.block);
  long long pos = st.pos;
  int32_t tok = st.tok;
  unsigned long long h = 0;  // fold state of the sequence read back so far in this step
  for (int k = 0; k <= c; ++k) {
    if (k > 0 && (pos >= st.upto || pos >= d.context - 1)) break;
    if (pos >= d.context - 1) {
      if (t == 0) fault(d, kFaultIdle, l, pos);
      break;
    }
    int ok = 0;
    if (t == 0) ok = write_token(d, l, pos, tok) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    __syncwarp();  // thread 0's write, before the warp reads the sequence back
    if (!ok) break;
    if (!(k == 0 ? fold_warp(d, l, pos, &h) : fold_one(d, l, pos, &h))) break;
    const int32_t tk = token_of(h);
    if (t == 0) o[k] = tk;
    tok = tk;
    pos += 1;
  }
  if (t == 0) {
    d.lanes[l].pos = (int32_t)pos;
    d.lanes[l].tok = tok;
  }
}

// A warp per lane.
__global__ void step_kernel(Dev d, uint32_t step, int32_t* out) {
  const int l = (int)((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  if (l < d.width) step_lane(d, step, l, out);
}

// ---------------------------------------------------------------------------------------
// ring transport: a resident executor polls a mailbox in host-mapped memory
// ---------------------------------------------------------------------------------------

constexpr uint32_t kItemApply = 1, kItemStep = 2, kItemExit = 3;
constexpr int kExecThreads = 1024;  // 32 warps: a warp per lane per round

// The mailbox, in pinned host memory mapped into the device's address space.  The host
// fills the item fields, then publishes `posted`; the executor runs the item, copies the
// device error word into `err` and publishes `done`.  Pointers are the device's view.
struct RingCtl {
  unsigned long long posted;
  unsigned long long done;
  unsigned long long err[3];
  uint32_t kind, n_msgs;
  unsigned long long bytes;
  uint32_t step, out_base;
  unsigned long long src, dst, out;
};

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// One CTA.  Waits for items (polling with a short sleep) and exits when none arrives for
// idle_ns or on an exit item; the host relaunches it when it posts to an exited executor.
__global__ void __launch_bounds__(kExecThreads, 1)
    executor_kernel(Dev d, RingCtl* ctl, unsigned long long idle_ns) {
  __shared__ int s_go;
  __shared__ uint32_t s_kind, s_n, s_step, s_base;
  __shared__ unsigned long long s_bytes, s_src, s_dst, s_out;
  unsigned long long next = ld_acquire_sys(&ctl->done);
  for (;;) {
    if (threadIdx.x == 0) {
      const unsigned long long t0 = now_ns();
      int go = 0;
      for (;;) {
        if (ld_acquire_sys(&ctl->posted) > next) {
          go = 1;
          break;
        }
        if (now_ns() - t0 > idle_ns) break;
        __nanosleep(500);
      }
      if (go) {
        const volatile RingCtl* c = ctl;
        s_kind = c->kind;
        s_n = c->n_msgs;
        s_bytes = c->bytes;
        s_step = c->step;
        s_base = c->out_base;
        s_src = c->src;
        s_dst = c->dst;
        s_out = c->out;
      }
      s_go = go;
    }
    __syncthreads();
    if (!s_go) break;
    if (s_kind == kItemApply) {
      // the stream into device memory first: mapped host memory is read uncached, once
      const volatile uint32_t* src = reinterpret_cast<const volatile uint32_t*>(s_src);
      uint32_t* dst = reinterpret_cast<uint32_t*>(s_dst);
      for (unsigned long long i = threadIdx.x; i < s_bytes / 4; i += kExecThreads) dst[i] = src[i];
      __syncthreads();
      apply_messages(d, reinterpret_cast<const uint8_t*>(s_dst), s_bytes, (int)s_n,
                     reinterpret_cast<int32_t*>(s_out) + s_base);
    } else if (s_kind == kItemStep) {
      for (int l = (int)(threadIdx.x >> 5); l < d.width; l += kExecThreads / 32)
        step_lane(d, s_step, l, reinterpret_cast<int32_t*>(s_out));
    }
    __threadfence_system();  // this thread's replies, before `done`
    __syncthreads();
    if (threadIdx.x == 0) {
      volatile RingCtl* c = ctl;
      for (int k = 0; k < 3; ++k) c->err[k] = reinterpret_cast<volatile unsigned long long*>(d.err)[k];
      __threadfence_system();
      st_release_sys(&ctl->done, next + 1);
    }
    ++next;
    if (s_kind == kItemExit) break;
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------------------
// encoding (ring::encode restated over this build's message table)
// ---------------------------------------------------------------------------------------

enum class Kind { One, Array, Span };
enum class Dtype { I32, U32, F32, U64 };

struct Field {
  const char* name;
  uint32_t at;
  Kind kind;
  Dtype dtype;
  uint32_t n;
};

struct Message {
  const char* name;
  uint32_t id;
  uint32_t bytes;
  std::vector<Field> fields;
};

struct Value {
  enum { Int, Float, Ints, Span } tag;
  int64_t i = 0;
  float f = 0;
  std::vector<int64_t> ints;
  uint64_t addr = 0, elements = 0;
};

Value vint(int64_t x) { Value v{Value::Int}; v.i = x; return v; }
Value vfloat(float x) { Value v{Value::Float}; v.f = x; return v; }
Value vints(std::vector<int64_t> xs) { Value v{Value::Ints}; v.ints = std::move(xs); return v; }
Value vspan(uint64_t addr, uint64_t elements) { Value v{Value::Span}; v.addr = addr; v.elements = elements; return v; }

const std::vector<Message>& messages() {
  static const std::vector<Message> m = {
      {"end", kIdEnd, kEndBytes,
       {{"at", kEndAt, Kind::One, Dtype::U32, 0}, {"lane", kEndLane, Kind::One, Dtype::U32, 0}}},
      {"pages", kIdPages, kPagesBytes,
       {{"at", kPagesAt, Kind::One, Dtype::U32, 0},
        {"lane", kPagesLane, Kind::One, Dtype::U32, 0},
        {"from", kPagesFrom, Kind::One, Dtype::U32, 0},
        {"upto", kPagesUpto, Kind::One, Dtype::U32, 0},
        {"row", kPagesRow, Kind::Span, Dtype::I32, 0}}},
      {"seat", kIdSeat, kSeatBytes,
       {{"at", kSeatAt, Kind::One, Dtype::U32, 0},
        {"lane", kSeatLane, Kind::One, Dtype::U32, 0},
        {"pos", kSeatPos, Kind::One, Dtype::U32, 0},
        {"back", kSeatBack, Kind::Array, Dtype::I32, 3},
        {"slot", kSeatSlot, Kind::One, Dtype::U32, 0},
        {"temp", kSeatTemp, Kind::One, Dtype::F32, 0},
        {"seed_lo", kSeatSeedLo, Kind::One, Dtype::U32, 0},
        {"seed_hi", kSeatSeedHi, Kind::One, Dtype::U32, 0},
        {"top_p", kSeatTopP, Kind::One, Dtype::F32, 0},
        {"top_k", kSeatTopK, Kind::One, Dtype::U32, 0},
        {"logprobs", kSeatLogprobs, Kind::One, Dtype::U32, 0}}},
      {"prompt", kIdPrompt, kPromptBytes,
       {{"lane", kPromptLane, Kind::One, Dtype::U32, 0},
        {"lens", kPromptLens, Kind::One, Dtype::U32, 0},
        {"tokens", kPromptTokens, Kind::Span, Dtype::U32, 0},
        {"lps", kPromptLps, Kind::Span, Dtype::F32, 0}}},
      {"start", kIdStart, kStartBytes,
       {{"at", kStartAt, Kind::One, Dtype::U32, 0},
        {"lane", kStartLane, Kind::One, Dtype::U32, 0},
        {"noise", kStartNoise, Kind::One, Dtype::U32, 0},
        {"idle", kStartIdle, Kind::One, Dtype::U32, 0},
        {"scratch", kStartScratch, Kind::One, Dtype::U32, 0},
        {"lps", kStartLps, Kind::Span, Dtype::F32, 0},
        {"commits", kStartCommits, Kind::Span, Dtype::I32, 0}}},
  };
  return m;
}

const Message& message(uint32_t id) {
  for (const Message& m : messages())
    if (m.id == id) return m;
  return messages()[0];
}

uint32_t dtype_bytes(Dtype d) { return d == Dtype::U64 ? 8 : 4; }

void put_int(Dtype d, int64_t x, uint8_t* out) {
  if (d == Dtype::U64) {
    uint64_t v = (uint64_t)x;
    memcpy(out, &v, 8);
  } else {
    uint32_t v = (uint32_t)x;  // i32 and u32 both keep the low 32 bits (`x as i32` / `x as u32`)
    memcpy(out, &v, 4);
  }
}

// ring::encode: every named field written at its offset by its kind; a mismatch is an error.
bool encode(const Message& layout, const std::vector<std::pair<const char*, Value>>& fields, uint8_t* bytes,
            std::string* err) {
  memset(bytes, 0, layout.bytes);
  for (const auto& [name, v] : fields) {
    const Field* f = nullptr;
    for (const Field& x : layout.fields)
      if (strcmp(x.name, name) == 0) f = &x;
    if (!f) {
      *err = std::string(layout.name) + " has no field " + name;
      return false;
    }
    const uint32_t at = f->at, e = dtype_bytes(f->dtype);
    if (f->kind == Kind::One && v.tag == Value::Int && f->dtype != Dtype::F32) {
      put_int(f->dtype, v.i, bytes + at);
    } else if (f->kind == Kind::One && v.tag == Value::Float && f->dtype == Dtype::F32) {
      memcpy(bytes + at, &v.f, 4);
    } else if (f->kind == Kind::Array && v.tag == Value::Ints && v.ints.size() == f->n) {
      for (size_t i = 0; i < v.ints.size(); ++i) put_int(f->dtype, v.ints[i], bytes + at + i * e);
    } else if (f->kind == Kind::Span && v.tag == Value::Span) {
      const uint64_t elements = f->n > 0 ? f->n : v.elements;
      memcpy(bytes + at, &v.addr, 8);
      memcpy(bytes + at + 8, &elements, 8);
    } else {
      *err = std::string(layout.name) + "." + name + " written as the wrong kind";
      return false;
    }
  }
  return true;
}

struct Cmd {
  uint32_t at;
  hk_command c;
  std::vector<int32_t> data;
  int64_t start = -1;  // a Prompt's first position, set when the command is taken for its step
};

size_t round16(size_t x) { return (x + 15) / 16 * 16; }

// Bytes of the encoded stream of `cmds` (slots then side blocks).
size_t stream_bytes(const std::vector<Cmd>& cmds, uint32_t chunk) {
  size_t n = cmds.size() * kSlot;
  for (const Cmd& c : cmds) {
    if (c.c.kind == HK_CMD_PAGES) n += round16(4 * c.data.size());
    if (c.c.kind == HK_CMD_PROMPT) n += round16(4 * (size_t)chunk);
  }
  return n;
}

// Feed::command (src/gpu/feed.rs:40-103) for each command, into `out` (stream_bytes long).
bool encode_commands(const hk_config& cfg, const std::vector<Cmd>& cmds, uint8_t* out, std::string* err) {
  size_t side = cmds.size() * kSlot;
  const size_t total = stream_bytes(cmds, cfg.chunk);
  memset(out, 0, total);
  for (size_t i = 0; i < cmds.size(); ++i) {
    const Cmd& x = cmds[i];
    const hk_command& c = x.c;
    uint8_t* slot = out + i * kSlot;
    std::vector<std::pair<const char*, Value>> f;
    uint32_t id = 0;
    const auto at = std::make_pair("at", vint(x.at));
    const auto lane = std::make_pair("lane", vint(c.lane));
    switch (c.kind) {
      case HK_CMD_END:
        id = kIdEnd;
        f = {at, lane};
        break;
      case HK_CMD_PAGES: {
        id = kIdPages;
        memcpy(out + side, x.data.data(), 4 * x.data.size());
        f = {at, lane, {"from", vint(c.pos)}, {"upto", vint(c.upto)}, {"row", vspan(side, x.data.size())}};
        side += round16(4 * x.data.size());
        break;
      }
      case HK_CMD_SEAT:
        id = kIdSeat;
        f = {at,
             lane,
             {"pos", vint(c.pos)},
             {"back", vints({c.back[0], c.back[1], c.back[2]})},
             {"slot", vint((int64_t)c.lane + 1)},
             {"temp", vfloat(c.sampling.temperature)},
             {"seed_lo", vint((uint32_t)c.sampling.seed)},
             {"seed_hi", vint((uint32_t)(c.sampling.seed >> 32))},
             {"top_p", vfloat(c.sampling.top_p)},
             {"top_k", vint(c.sampling.top_k)},
             {"logprobs", vint(c.sampling.logprobs)}};
        break;
      case HK_CMD_PROMPT: {
        id = kIdPrompt;
        memcpy(out + side, x.data.data(), 4 * x.data.size());
        f = {lane, {"lens", vint((int64_t)x.data.size())}, {"tokens", vspan(side, cfg.chunk)}, {"lps", vspan(0, 0)}};
        side += round16(4 * (size_t)cfg.chunk);
        break;
      }
      case HK_CMD_START:
        id = kIdStart;
        f = {at, lane, {"noise", vint(0)}, {"idle", vint((int64_t)cfg.context - 1)}, {"scratch", vint(0)},
             {"lps", vspan(0, 0)}, {"commits", vspan(0, 0)}};
        break;
      default:
        *err = "a command of unknown kind " + std::to_string(c.kind);
        return false;
    }
    memcpy(slot, &id, 4);
    if (!encode(message(id), f, slot + kBodyAt, err)) return false;
  }
  return true;
}

// Checks a share against the configuration and copies its commands.
int take_share(const hk_config& cfg, const hk_share* s, std::vector<Cmd>* out) {
  HK_REQUIRE(s && (s->n_commands == 0 || s->commands) && (s->arena_words == 0 || s->arena),
             "hk_push: null share arrays");
  const size_t row = (size_t)cfg.entries + cfg.window;
  for (size_t i = 0; i < s->n_commands; ++i) {
    const hk_command& c = s->commands[i];
    HK_REQUIRE(c.kind <= HK_CMD_START, "command %zu: unknown kind %u", i, c.kind);
    HK_REQUIRE(c.lane < cfg.width, "command %zu: lane %u past the width %u", i, c.lane, cfg.width);
    Cmd x{s->at, c, {}, -1};
    if (c.kind == HK_CMD_PAGES || c.kind == HK_CMD_PROMPT) {
      HK_REQUIRE((size_t)c.arena + c.count <= s->arena_words, "command %zu: arena words %u..%u past %zu", i,
                 c.arena, c.arena + c.count, s->arena_words);
      x.data.assign(s->arena + c.arena, s->arena + c.arena + c.count);
    }
    if (c.kind == HK_CMD_PAGES)
      HK_REQUIRE((size_t)c.pos + c.count <= row, "command %zu: row entries %u..%u past %zu", i, c.pos,
                 c.pos + c.count, row);
    if (c.kind == HK_CMD_PROMPT)
      HK_REQUIRE(c.count >= 1 && c.count <= cfg.chunk, "command %zu: a prompt of %u tokens (chunk %u)", i,
                 c.count, cfg.chunk);
    out->push_back(std::move(x));
  }
  return HK_OK;
}

}  // namespace

struct hk_handle {
  hk_config cfg;
  cudaStream_t stream = nullptr;
  Dev dev{};
  int32_t* d_out = nullptr;  // [width * block] step ids, then prompt replies
  size_t out_cap = 0;        // words
  uint8_t* d_stream = nullptr;
  size_t d_stream_cap = 0;
  uint8_t* h_stream = nullptr;
  size_t h_stream_cap = 0;
  int32_t* h_out = nullptr;
  unsigned long long* h_err = nullptr;
  struct Mirror {
    uint32_t upto = 0, pos = 0;
    bool live = false;
  };
  std::vector<Mirror> lanes;
  std::deque<Cmd> queue;
  uint32_t s = 0;
  int64_t horizon = -1;
  bool applied = false;
  std::vector<hk_event> events;
  std::vector<int32_t> ids;
  std::string error;
  // ring transport (cfg.transport == HK_TRANSPORT_RING)
  bool ring = false;
  cudaStream_t exec_stream = nullptr;
  RingCtl* ctl = nullptr;      // host view of the mapped mailbox
  RingCtl* d_ctl = nullptr;    // device view
  uint8_t* d_h_stream = nullptr;  // device view of h_stream (mapped)
  int32_t* d_h_out = nullptr;     // device view of h_out (mapped)
  unsigned long long posted = 0;
  // Set when the executor gave no answer in time: it may still be running the abandoned item
  // (and publish `done` for it later), so the handle's device state is undefined and every
  // later hk_push / hk_drain fails with this message.
  std::string broken;
  // Logprob lists of the Sampled values of the pending events (one per id slot of a Step, one
  // per Prompted), and those of the events the last successful hk_drain returned.
  std::vector<uint32_t> pend_counts, last_counts;
  std::vector<hk_logprob> pend_pairs, last_pairs;
  // HK_MODEL_MLA
  hk::MlaModel* mla = nullptr;
  float* h_lp = nullptr;  // pinned: the step's logprob rows
};

namespace {

int handle_fail(hk_handle* h, int rc) {
  if (h && rc != HK_OK) h->error = hk_last_error();
  return rc;
}

int grow_device(uint8_t** p, size_t* cap, size_t need) {
  if (need <= *cap) return HK_OK;
  if (*p) cudaFree(*p);
  *p = nullptr;
  *cap = 0;
  size_t n = 1 << 16;
  while (n < need) n *= 2;
  HK_TRY_CUDA(cudaMalloc(p, n));
  *cap = n;
  return HK_OK;
}

// Pinned host memory, also mapped into the device's address space when `mapped_dev` is given.
int grow_host(uint8_t** p, size_t* cap, size_t need, uint8_t** mapped_dev = nullptr) {
  if (need <= *cap) return HK_OK;
  if (*p) cudaFreeHost(*p);
  *p = nullptr;
  *cap = 0;
  size_t n = 1 << 16;
  while (n < need) n *= 2;
  if (mapped_dev) {
    HK_TRY_CUDA(cudaHostAlloc(p, n, cudaHostAllocMapped));
    HK_TRY_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(mapped_dev), *p, 0));
  } else {
    HK_TRY_CUDA(cudaMallocHost(p, n));
  }
  *cap = n;
  return HK_OK;
}

// Copies `words` of d_out and the three error words back and synchronises; a recorded fault
// becomes HK_EDEVICE with the test device's wording.
int fault_status(const unsigned long long* err) {
  const unsigned long long w = err[0];
  if (!(w >> 63)) return HK_OK;
  const unsigned site = (unsigned)((w >> 32) & 0x7fffffff);
  const long long lane = (long long)err[1], pos = (long long)err[2];
  switch (site) {
    case kFaultScratchWrite:
      return hk::fail(HK_EDEVICE, "lane %lld writes position %lld to the scratch page", lane, pos);
    case kFaultUnwritten:
      return hk::fail(HK_EDEVICE, "lane %lld reads position %lld unwritten", lane, pos);
    case kFaultWindowScratch:
      return hk::fail(HK_EDEVICE, "lane %lld reads position %lld's window from the scratch window page", lane,
                      pos);
    case kFaultWindowMismatch:
      return hk::fail(HK_EDEVICE, "lane %lld's window at %lld", lane, pos);
    case kFaultIdle:
      return hk::fail(HK_EDEVICE, "lane %lld decodes at the idle position", lane);
    case kFaultChunkWindow:
      return hk::fail(HK_EDEVICE, "lane %lld's chunk writes position %lld's window to the scratch window page",
                      lane, pos);
    case kFaultPagePastPool:
      return hk::fail(HK_EDEVICE, "lane %lld: a page id past the pool or the row at position %lld", lane, pos);
    default:
      return hk::fail(HK_EDEVICE, "message %lld for lane %lld malformed", pos, lane);
  }
}

int readback(hk_handle* h, size_t words) {
  if (words) HK_TRY_CUDA(cudaMemcpyAsync(h->h_out, h->d_out, 4 * words, cudaMemcpyDeviceToHost, h->stream));
  HK_TRY_CUDA(cudaMemcpyAsync(h->h_err, h->dev.err, 3 * sizeof(unsigned long long), cudaMemcpyDeviceToHost,
                              h->stream));
  HK_TRY_CUDA(cudaStreamSynchronize(h->stream));
  return fault_status(h->h_err);
}

constexpr unsigned long long kExecIdleNs = 50000000ull;  // an executor exits after 50 ms idle
constexpr double kRingTimeoutS = 30.0;

int launch_executor(hk_handle* h) {
  executor_kernel<<<1, kExecThreads, 0, h->exec_stream>>>(h->dev, h->d_ctl, kExecIdleNs);
  HK_TRY_LAUNCH("executor_kernel");
  return HK_OK;
}

// Posts one item to the executor and waits for it (relaunching an executor that went idle).
int ring_run(hk_handle* h, uint32_t kind, uint32_t n_msgs, uint64_t bytes, uint32_t step, uint32_t out_base) {
  volatile RingCtl* c = h->ctl;
  c->kind = kind;
  c->n_msgs = n_msgs;
  c->bytes = bytes;
  c->step = step;
  c->out_base = out_base;
  c->src = (unsigned long long)(uintptr_t)h->d_h_stream;
  c->dst = (unsigned long long)(uintptr_t)h->d_stream;
  c->out = (unsigned long long)(uintptr_t)h->d_h_out;
  std::atomic_thread_fence(std::memory_order_seq_cst);
  c->posted = ++h->posted;
  std::atomic_thread_fence(std::memory_order_seq_cst);
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    if (c->done >= h->posted) break;
    const cudaError_t q = cudaStreamQuery(h->exec_stream);
    if (q == cudaSuccess) {
      if (c->done >= h->posted) break;
      HK_TRY(launch_executor(h));  // it had gone idle before the item was posted
    } else if (q != cudaErrorNotReady) {
      return hk::cuda_fail(q, "ring executor");
    }
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > kRingTimeoutS) {
      const int rc = hk::fail(HK_EDEVICE, "ring executor gave no answer in %.0f s", kRingTimeoutS);
      h->broken = hk_last_error();
      return rc;
    }
    std::this_thread::yield();
  }
  std::atomic_thread_fence(std::memory_order_seq_cst);
  unsigned long long err[3];
  for (int k = 0; k < 3; ++k) err[k] = c->err[k];
  return fault_status(err);
}

// Encodes and applies a batch; appends its Prompted replies to the events.
int apply_batch(hk_handle* h, const std::vector<Cmd>& batch) {
  const size_t bytes = stream_bytes(batch, h->cfg.chunk);
  HK_TRY(grow_host(&h->h_stream, &h->h_stream_cap, bytes, h->ring ? &h->d_h_stream : nullptr));
  HK_TRY(grow_device(&h->d_stream, &h->d_stream_cap, bytes));
  std::string err;
  if (!encode_commands(h->cfg, batch, h->h_stream, &err)) return hk::fail(HK_EINVAL, "%s", err.c_str());
  size_t prompts = 0;
  for (const Cmd& c : batch) prompts += c.c.kind == HK_CMD_PROMPT;
  const size_t base = (size_t)h->cfg.width * h->cfg.block;
  if (base + prompts > h->out_cap) {
    cudaFree(h->d_out);
    cudaFreeHost(h->h_out);
    h->d_out = nullptr;
    h->h_out = nullptr;
    h->out_cap = base + std::max<size_t>(prompts, 64);
    HK_TRY_CUDA(cudaMalloc(&h->d_out, 4 * h->out_cap));
    if (h->ring) {
      HK_TRY_CUDA(cudaHostAlloc(&h->h_out, 4 * h->out_cap, cudaHostAllocMapped));
      HK_TRY_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&h->d_h_out), h->h_out, 0));
    } else {
      HK_TRY_CUDA(cudaMallocHost(&h->h_out, 4 * h->out_cap));
    }
  }
  if (h->ring) {
    HK_TRY(ring_run(h, kItemApply, (uint32_t)batch.size(), bytes, 0, (uint32_t)base));
    size_t k = 0;
    for (const Cmd& c : batch) {
      if (c.c.kind != HK_CMD_PROMPT) continue;
      hk_event e{};
      e.kind = HK_EV_PROMPTED;
      e.lane = c.c.lane;
      e.token = h->h_out[base + k++];
      e.clipped = h->cfg.clip;
      h->events.push_back(e);
      h->pend_counts.push_back(0);  // the test model samples no logprobs
    }
    return HK_OK;
  }
  HK_TRY_CUDA(cudaMemcpyAsync(h->d_stream, h->h_stream, bytes, cudaMemcpyHostToDevice, h->stream));
  apply_kernel<<<1, 256, 0, h->stream>>>(h->dev, h->d_stream, bytes, (int)batch.size(), h->d_out + base);
  HK_TRY_LAUNCH("apply_kernel");
  // the stream buffer is reused by the next batch: the readback's synchronise orders them
  if (prompts) {
    HK_TRY_CUDA(cudaMemcpyAsync(h->h_out + base, h->d_out + base, 4 * prompts, cudaMemcpyDeviceToHost,
                                h->stream));
  }
  HK_TRY(readback(h, 0));
  size_t k = 0;
  for (const Cmd& c : batch) {
    if (c.c.kind != HK_CMD_PROMPT) continue;
    hk_event e{};
    e.kind = HK_EV_PROMPTED;
    e.lane = c.c.lane;
    e.token = h->h_out[base + k++];
    e.clipped = h->cfg.clip;
    h->events.push_back(e);
    h->pend_counts.push_back(0);
  }
  return HK_OK;
}

// ---------------------------------------------------------------------------------------
// HK_MODEL_MLA: prompt chunks prefilled through the model, decode steps verified by it
// ---------------------------------------------------------------------------------------

// One Sampled's logprob list from its row of 2n + 1 floats (the reply layout src/gpu/feed.rs:
// 202-208 reads): the top pairs while their id is >= 0, then the token's own logprob.
void push_logprob_list(hk_handle* h, int32_t id, const float* row, int32_t n) {
  if (id < 0 || row == nullptr) {
    h->pend_counts.push_back(0);
    return;
  }
  uint32_t count = 0;
  for (int32_t q = 0; q < n && row[2 * q] >= 0.0f; ++q, ++count)
    h->pend_pairs.push_back(hk_logprob{(uint32_t)row[2 * q], row[2 * q + 1]});
  h->pend_pairs.push_back(hk_logprob{(uint32_t)id, row[2 * n]});
  h->pend_counts.push_back(count + 1);
}

// Copies `words` sampled ids and `lp_floats` logprob floats back, synchronises, and reports the
// handle's error words and the library's device error word.
int mla_readback(hk_handle* h, size_t words, size_t lp_floats) {
  hk::MlaModel* m = h->mla;
  HK_TRY_CUDA(cudaMemcpyAsync(h->h_out, m->out_ids, 4 * words, cudaMemcpyDeviceToHost, h->stream));
  if (lp_floats)
    HK_TRY_CUDA(cudaMemcpyAsync(h->h_lp, m->lp, 4 * lp_floats, cudaMemcpyDeviceToHost, h->stream));
  HK_TRY_CUDA(cudaMemcpyAsync(h->h_err, h->dev.err, 3 * sizeof(unsigned long long), cudaMemcpyDeviceToHost,
                              h->stream));
  HK_TRY_CUDA(cudaStreamSynchronize(h->stream));
  HK_TRY(fault_status(h->h_err));
  return hk_check_errors();
}

// A group of prompt chunks of distinct lanes through one forward pass; Prompted events in the
// group's push order.
int mla_prompt_group(hk_handle* h, const std::vector<const Cmd*>& group) {
  hk::MlaModel* m = h->mla;
  std::vector<const Cmd*> by_lane = group;
  std::sort(by_lane.begin(), by_lane.end(), [](const Cmd* a, const Cmd* b) { return a->c.lane < b->c.lane; });
  std::vector<hk::MlaLaneRows> lanes;
  std::vector<int32_t> tokens;
  for (const Cmd* c : by_lane) {
    lanes.push_back(hk::MlaLaneRows{(int32_t)c->c.lane, (int32_t)c->start, (int32_t)c->data.size()});
    tokens.insert(tokens.end(), c->data.begin(), c->data.end());
  }
  HK_TRY(hk::mla_prompt_step(m, lanes, tokens, h->dev.rows, h->dev.pool, h->dev.err, h->stream));
  const size_t row = 2 * (size_t)m->n_lp + 1;
  HK_TRY(mla_readback(h, (size_t)h->cfg.width, m->n_lp > 0 ? (size_t)h->cfg.width * row : 0));
  for (const Cmd* c : group) {
    hk_event e{};
    e.kind = HK_EV_PROMPTED;
    e.lane = c->c.lane;
    e.token = h->h_out[c->c.lane];
    e.clipped = h->cfg.clip;
    h->events.push_back(e);
    push_logprob_list(h, e.token, m->n_lp > 0 ? h->h_lp + (size_t)c->c.lane * row : nullptr, m->n_lp);
  }
  return HK_OK;
}

// A batch's commands in order, with prompt chunks gathered into as few forward passes as
// possible: a pass takes prompt chunks of distinct lanes up to t_cap rows, and the non-prompt
// commands (pages, seats, starts, ends) met between them go to the apply kernel first when
// they concern none of the pass's lanes — they only touch their own lanes' block-table rows
// and state, which the pass does not read — and otherwise after the pass has run.  A lane's
// second chunk waits for the pass holding its first.  Prompted replies keep push order.
int apply_batch_mla(hk_handle* h, const std::vector<Cmd>& batch) {
  std::vector<const Cmd*> group;
  std::vector<uint32_t> lanes;
  std::vector<Cmd> run;  // non-prompt commands not yet applied
  size_t rows = 0;
  auto in_group = [&](uint32_t lane) { return std::find(lanes.begin(), lanes.end(), lane) != lanes.end(); };
  auto flush = [&]() -> int {
    if (!group.empty()) HK_TRY(mla_prompt_group(h, group));
    group.clear();
    lanes.clear();
    rows = 0;
    return HK_OK;
  };
  auto apply_run = [&]() -> int {
    if (run.empty()) return HK_OK;
    for (const Cmd& c : run)
      if (in_group(c.c.lane)) {
        HK_TRY(flush());
        break;
      }
    HK_TRY(apply_batch(h, run));
    run.clear();
    return HK_OK;
  };
  for (const Cmd& c : batch) {
    if (c.c.kind != HK_CMD_PROMPT) {
      run.push_back(c);
      continue;
    }
    HK_TRY(apply_run());
    if (in_group(c.c.lane) || (!group.empty() && rows + c.data.size() > (size_t)h->mla->t_cap)) HK_TRY(flush());
    group.push_back(&c);
    lanes.push_back(c.c.lane);
    rows += c.data.size();
  }
  HK_TRY(apply_run());
  return flush();
}

int run_step_mla(hk_handle* h) {
  hk::MlaModel* m = h->mla;
  const hk_config& c = h->cfg;
  std::vector<hk::MlaLaneRows> lanes;
  for (uint32_t l = 0; l < c.width; ++l) {
    const auto& st = h->lanes[l];
    if (!(st.live && st.pos < st.upto)) continue;
    if ((int64_t)st.pos >= (int64_t)c.context - 1)
      return hk::fail(HK_EDEVICE, "lane %u decodes at the idle position", l);
    const uint32_t rows = std::min<uint32_t>({c.block, st.upto - st.pos, c.context - 1 - st.pos});
    lanes.push_back(hk::MlaLaneRows{(int32_t)l, (int32_t)st.pos, (int32_t)rows});
  }
  HK_TRY(hk::mla_decode_step(m, lanes, h->dev.rows, h->dev.pool, h->dev.err, h->stream));
  const size_t words = (size_t)c.width * c.block, row = 2 * (size_t)m->n_lp + 1;
  HK_TRY(mla_readback(h, words, m->n_lp > 0 ? words * row : 0));
  hk_event e{};
  e.kind = HK_EV_STEP;
  e.step = h->s;
  e.ids = (uint32_t)h->ids.size();
  h->ids.insert(h->ids.end(), h->h_out, h->h_out + words);
  h->events.push_back(e);
  for (size_t k = 0; k < words; ++k)
    push_logprob_list(h, h->h_out[k], m->n_lp > 0 ? h->h_lp + k * row : nullptr, m->n_lp);
  for (uint32_t l = 0; l < c.width; ++l) {
    uint32_t n = 0;
    while (n < c.block && h->h_out[(size_t)l * c.block + n] != -2) ++n;
    h->lanes[l].pos += n;
  }
  h->s += 1;
  return HK_OK;
}

int run_step(hk_handle* h) {
  if (h->mla) return run_step_mla(h);
  const size_t words = (size_t)h->cfg.width * h->cfg.block;
  if (h->ring) {
    HK_TRY(ring_run(h, kItemStep, 0, 0, h->s, 0));
  } else {
    const int threads = 128;  // 4 lanes per block, a warp each
    const int blocks = (int)(((int64_t)h->cfg.width * 32 + threads - 1) / threads);
    step_kernel<<<blocks, threads, 0, h->stream>>>(h->dev, h->s, h->d_out);
    HK_TRY_LAUNCH("step_kernel");
    HK_TRY(readback(h, words));
  }
  hk_event e{};
  e.kind = HK_EV_STEP;
  e.step = h->s;
  e.ids = (uint32_t)h->ids.size();
  h->ids.insert(h->ids.end(), h->h_out, h->h_out + words);
  h->events.push_back(e);
  h->pend_counts.insert(h->pend_counts.end(), words, 0u);  // the test model samples no logprobs
  for (uint32_t l = 0; l < h->cfg.width; ++l) {
    uint32_t n = 0;
    while (n < h->cfg.block && h->h_out[(size_t)l * h->cfg.block + n] != -2) ++n;
    h->lanes[l].pos += n;
  }
  h->s += 1;
  return HK_OK;
}

// The test device's run loop (tests/engine.rs:130-211) over device kernels.
int run(hk_handle* h) {
  for (;;) {
    std::vector<Cmd> batch;
    while (!h->queue.empty()) {
      Cmd& c = h->queue.front();
      const bool delta = c.c.kind != HK_CMD_PROMPT;
      if (delta && c.at > h->s) break;
      h->applied |= delta;
      auto& m = h->lanes[c.c.lane];
      switch (c.c.kind) {
        case HK_CMD_END: m.live = false; m.upto = 0; break;
        case HK_CMD_PAGES: m.upto = c.c.upto; break;
        case HK_CMD_SEAT: m.pos = c.c.pos; break;
        case HK_CMD_START: m.live = true; break;
        default: c.start = m.pos; m.pos += (uint32_t)c.data.size(); break;
      }
      batch.push_back(std::move(h->queue.front()));
      h->queue.pop_front();
    }
    if (!batch.empty()) HK_TRY(h->mla ? apply_batch_mla(h, batch) : apply_batch(h, batch));
    bool runnable = false;
    for (auto& m : h->lanes) runnable |= m.live && m.pos < m.upto;
    if (runnable && (int64_t)h->s <= h->horizon) {
      HK_TRY(run_step(h));
      continue;
    }
    if (!runnable && h->applied) {
      hk_event e{};
      e.kind = HK_EV_IDLE;
      e.step = h->s;
      h->events.push_back(e);
      h->applied = false;
    }
    if (!h->queue.empty()) {
      const Cmd& c = h->queue.front();
      if (!runnable && c.c.kind != HK_CMD_PROMPT && c.at > h->s && (int64_t)c.at <= h->horizon + 1) {
        h->s = c.at;
        continue;
      }
    }
    return HK_OK;
  }
}

void release(hk_handle* h) {
  if (!h) return;
  if (h->ring && h->ctl && h->exec_stream) {
    if (cudaStreamQuery(h->exec_stream) == cudaErrorNotReady) {  // ask a running executor to exit
      volatile RingCtl* c = h->ctl;
      c->kind = kItemExit;
      std::atomic_thread_fence(std::memory_order_seq_cst);
      c->posted = ++h->posted;
    }
    cudaStreamSynchronize(h->exec_stream);
  }
  hk::mla_destroy(h->mla);
  if (h->h_lp) cudaFreeHost(h->h_lp);
  if (h->ctl) cudaFreeHost(h->ctl);
  if (h->exec_stream) cudaStreamDestroy(h->exec_stream);
  cudaFree(h->dev.rows);
  cudaFree(h->dev.pool);
  cudaFree(h->dev.windows);
  cudaFree(h->dev.lanes);
  cudaFree(h->dev.sampling);
  cudaFree(h->dev.err);
  cudaFree(h->d_out);
  cudaFree(h->d_stream);
  cudaFreeHost(h->h_stream);
  cudaFreeHost(h->h_out);
  cudaFreeHost(h->h_err);
  if (h->stream) cudaStreamDestroy(h->stream);
  delete h;
}

int c_pools(void* self, size_t* pages, size_t* window_pages) {
  return hk_pools(static_cast<hk_handle*>(self), pages, window_pages);
}
int c_push(void* self, const hk_share* share) { return hk_push(static_cast<hk_handle*>(self), share); }
int c_drain(void* self, hk_event* events, size_t cap, size_t* n, int32_t* ids, size_t ids_cap, size_t* ids_n) {
  return hk_drain(static_cast<hk_handle*>(self), events, cap, n, ids, ids_cap, ids_n);
}
const char* c_error(void* self) { return static_cast<hk_handle*>(self)->error.c_str(); }
int c_logprobs(void* self, uint32_t* counts, size_t counts_cap, size_t* n_counts, hk_logprob* pairs, size_t pairs_cap,
               size_t* n_pairs) {
  return hk_drain_logprobs(static_cast<hk_handle*>(self), counts, counts_cap, n_counts, pairs, pairs_cap, n_pairs);
}

int check_config(const hk_config* c) {
  HK_REQUIRE(c, "null config");
  HK_REQUIRE(c->model == HK_MODEL_FNV || c->model == HK_MODEL_MLA,
             "model %u: HK_MODEL_FNV (%d) or HK_MODEL_MLA (%d)", c->model, HK_MODEL_FNV, HK_MODEL_MLA);
  HK_REQUIRE(c->page_rows > 0 && c->entries > 0 && c->window > 0 && c->width > 0 && c->block > 0 &&
                 c->chunk > 0 && c->context >= 2,
             "page_rows, entries, window, width, block, chunk must be > 0 and context >= 2");
  HK_REQUIRE(c->pages >= 1 && c->window_pages >= 1 && c->pages < (1ull << 31) && c->window_pages < (1ull << 31),
             "pool sizes must be in 1..2^31");
  HK_REQUIRE((uint64_t)c->entries * c->page_rows < (1ull << 31), "a row covers at most 2^31 positions");
  HK_REQUIRE(c->transport == HK_TRANSPORT_LAUNCH || c->transport == HK_TRANSPORT_RING,
             "transport %u: HK_TRANSPORT_LAUNCH (0) or HK_TRANSPORT_RING (1)", c->transport);
  return HK_OK;
}

}  // namespace

extern "C" {

}  // extern "C"

namespace {

// The pools, block-table rows, lane state and transport of a handle (both models).
int open_handle(const hk_config* config, hk_handle** handle) {
  HK_REQUIRE(handle, "null handle pointer");
  *handle = nullptr;
  HK_TRY(check_config(config));
  HK_TRY_CUDA(cudaSetDevice(config->device));
  HK_TRY(hk::ensure_device());
  auto* h = new hk_handle;
  h->cfg = *config;
  h->lanes.resize(config->width);
  const hk_config& c = *config;
  Dev& d = h->dev;
  d.width = (int32_t)c.width;
  d.entries = (int32_t)c.entries;
  d.window = (int32_t)c.window;
  d.page_rows = (int32_t)c.page_rows;
  d.context = (int32_t)c.context;
  d.chunk = (int32_t)c.chunk;
  d.block = (int32_t)c.block;
  d.pages = (int64_t)c.pages;
  d.window_pages = (int64_t)c.window_pages;
  auto fail = [&](int rc) {
    release(h);
    return rc;
  };
  const size_t row_words = (size_t)c.width * (c.entries + c.window);
  cudaError_t e = cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&d.rows, 4 * row_words);
  if (e == cudaSuccess) e = cudaMalloc(&d.pool, 4 * (size_t)c.pages * c.page_rows);
  if (e == cudaSuccess) e = cudaMalloc(&d.windows, 4 * (size_t)c.window_pages * c.page_rows);
  if (e == cudaSuccess) e = cudaMalloc(&d.lanes, sizeof(LaneState) * c.width);
  if (e == cudaSuccess) e = cudaMalloc(&d.sampling, sizeof(LaneSampling) * c.width);
  if (e == cudaSuccess) e = cudaMalloc(&d.err, 4 * sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMallocHost(&h->h_err, 4 * sizeof(unsigned long long));
  if (e == cudaSuccess) {
    h->out_cap = (size_t)c.width * c.block + 64;
    e = cudaMalloc(&h->d_out, 4 * h->out_cap);
  }
  if (e == cudaSuccess) e = cudaMallocHost(&h->h_out, 4 * h->out_cap);
  if (e == cudaSuccess) e = cudaMemsetAsync(d.rows, 0, 4 * row_words, h->stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(d.pool, 0xff, 4 * (size_t)c.pages * c.page_rows, h->stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(d.windows, 0xff, 4 * (size_t)c.window_pages * c.page_rows, h->stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(d.lanes, 0, sizeof(LaneState) * c.width, h->stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(d.sampling, 0, sizeof(LaneSampling) * c.width, h->stream);
  if (e == cudaSuccess) e = cudaMemsetAsync(d.err, 0, 4 * sizeof(unsigned long long), h->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(h->stream);
  if (e != cudaSuccess) return fail(hk::cuda_fail(e, "hk_open"));
  if (c.transport == HK_TRANSPORT_RING) {
    h->ring = true;
    cudaFreeHost(h->h_out);
    h->h_out = nullptr;
    e = cudaStreamCreateWithFlags(&h->exec_stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaHostAlloc(&h->h_out, 4 * h->out_cap, cudaHostAllocMapped);
    if (e == cudaSuccess) e = cudaHostGetDevicePointer(reinterpret_cast<void**>(&h->d_h_out), h->h_out, 0);
    if (e == cudaSuccess) e = cudaHostAlloc(&h->ctl, sizeof(RingCtl), cudaHostAllocMapped);
    if (e == cudaSuccess) e = cudaHostGetDevicePointer(reinterpret_cast<void**>(&h->d_ctl), h->ctl, 0);
    if (e != cudaSuccess) return fail(hk::cuda_fail(e, "hk_open (ring)"));
    memset(h->ctl, 0, sizeof(RingCtl));
    const int rc = launch_executor(h);
    if (rc != HK_OK) return fail(rc);
  }
  *handle = h;
  return HK_OK;
}

}  // namespace

extern "C" {

int hk_open(const hk_config* config, hk_handle** handle) {
  HK_REQUIRE(handle, "null handle pointer");
  *handle = nullptr;
  HK_REQUIRE(config && config->model == HK_MODEL_FNV,
             "hk_open: model %u (HK_MODEL_FNV here; HK_MODEL_MLA opens with hk_open_mla)", config ? config->model : 0);
  return open_handle(config, handle);
}

int hk_open_mla(const hk_config* config, const hk_mla_model* model, hk_handle** handle) {
  HK_REQUIRE(handle && model, "hk_open_mla: null argument");
  *handle = nullptr;
  HK_REQUIRE(config && config->model == HK_MODEL_MLA, "hk_open_mla: config->model must be HK_MODEL_MLA (%d)",
             HK_MODEL_MLA);
  HK_TRY(check_config(config));
  HK_TRY(hk::mla_check(*config, *model));
  hk_handle* h = nullptr;
  HK_TRY(open_handle(config, &h));
  int rc = hk::mla_create(*config, *model, &h->mla, h->stream);
  if (rc == HK_OK) {
    const size_t floats = (size_t)config->width * config->block * (2 * (size_t)model->logprobs + 1);
    const cudaError_t e = cudaMallocHost(&h->h_lp, 4 * floats);
    if (e != cudaSuccess) rc = hk::cuda_fail(e, "hk_open_mla: logprob staging");
  }
  if (rc != HK_OK) {
    release(h);
    return rc;
  }
  h->dev.mla_sampling = h->mla->sampling;
  h->dev.mla_state = h->mla->state;
  *handle = h;
  return HK_OK;
}

int hk_model_tensor(hk_handle* h, uint32_t layer, const char* name, void** ptr, size_t* bytes) {
  HK_REQUIRE(h && h->mla, "hk_model_tensor: not an HK_MODEL_MLA handle");
  return hk::mla_tensor(h->mla, h->dev.pool, 4 * (size_t)h->cfg.pages * h->cfg.page_rows, layer, name, ptr, bytes);
}

void hk_close(hk_handle* handle) {
  if (handle) cudaSetDevice(handle->cfg.device);
  if (handle && handle->stream) cudaStreamSynchronize(handle->stream);
  release(handle);
}

int hk_pools(const hk_handle* h, size_t* pages, size_t* window_pages) {
  HK_REQUIRE(h && pages && window_pages, "hk_pools: null argument");
  *pages = (size_t)h->cfg.pages;
  *window_pages = (size_t)h->cfg.window_pages;
  return HK_OK;
}

int hk_push(hk_handle* h, const hk_share* share) {
  HK_REQUIRE(h && share, "hk_push: null argument");
  if (!h->broken.empty()) return handle_fail(h, hk::fail(HK_EDEVICE, "%s", h->broken.c_str()));
  if ((int64_t)share->at != h->horizon + 1)
    return handle_fail(h, hk::fail(HK_ESTATE, "a share at %u past a horizon of %lld", share->at,
                                   (long long)h->horizon));
  if (share->horizon < share->at)
    return handle_fail(h, hk::fail(HK_EINVAL, "a share's horizon %u before its step %u", share->horizon,
                                   share->at));
  std::vector<Cmd> cmds;
  int rc = take_share(h->cfg, share, &cmds);
  if (rc != HK_OK) return handle_fail(h, rc);
  for (Cmd& c : cmds) h->queue.push_back(std::move(c));
  h->horizon = share->horizon;
  return HK_OK;
}

int hk_drain(hk_handle* h, hk_event* events, size_t cap, size_t* n, int32_t* ids, size_t ids_cap,
             size_t* ids_n) {
  HK_REQUIRE(h && n && ids_n, "hk_drain: null argument");
  if (!h->broken.empty()) return handle_fail(h, hk::fail(HK_EDEVICE, "%s", h->broken.c_str()));
  HK_TRY_CUDA(cudaSetDevice(h->cfg.device));
  int rc = run(h);
  if (rc != HK_OK) return handle_fail(h, rc);
  *n = h->events.size();
  *ids_n = h->ids.size();
  if (h->events.size() > cap || h->ids.size() > ids_cap || (cap && !events && *n) || (ids_cap && !ids && *ids_n))
    return handle_fail(h, hk::fail(HK_ESPACE, "hk_drain: %zu events and %zu ids pending", *n, *ids_n));
  if (*n) memcpy(events, h->events.data(), sizeof(hk_event) * *n);
  if (*ids_n) memcpy(ids, h->ids.data(), 4 * *ids_n);
  h->last_counts = std::move(h->pend_counts);
  h->last_pairs = std::move(h->pend_pairs);
  h->pend_counts.clear();
  h->pend_pairs.clear();
  h->events.clear();
  h->ids.clear();
  return HK_OK;
}

int hk_drain_logprobs(hk_handle* h, uint32_t* counts, size_t counts_cap, size_t* n_counts, hk_logprob* pairs,
                      size_t pairs_cap, size_t* n_pairs) {
  HK_REQUIRE(h && n_counts && n_pairs, "hk_drain_logprobs: null argument");
  *n_counts = h->last_counts.size();
  *n_pairs = h->last_pairs.size();
  if (*n_counts > counts_cap || (*n_counts && !counts) || *n_pairs > pairs_cap || (*n_pairs && !pairs))
    return hk::fail(HK_ESPACE, "hk_drain_logprobs: %zu lists of %zu pairs", *n_counts, *n_pairs);
  if (*n_counts) memcpy(counts, h->last_counts.data(), 4 * *n_counts);
  if (*n_pairs) memcpy(pairs, h->last_pairs.data(), sizeof(hk_logprob) * *n_pairs);
  return HK_OK;
}

int hk_encode_share(const hk_config* config, const hk_share* share, uint8_t* out, size_t cap, size_t* bytes) {
  HK_REQUIRE(config && share && bytes, "hk_encode_share: null argument");
  HK_TRY(check_config(config));
  std::vector<Cmd> cmds;
  HK_TRY(take_share(*config, share, &cmds));
  *bytes = stream_bytes(cmds, config->chunk);
  if (*bytes == 0) return HK_OK;
  HK_REQUIRE(out && cap >= *bytes, "hk_encode_share: %zu bytes needed", *bytes);
  std::string err;
  if (!encode_commands(*config, cmds, out, &err)) return hk::fail(HK_EINVAL, "%s", err.c_str());
  return HK_OK;
}

int hk_kernel_ops_of(hk_handle* h, hk_kernel_ops* ops) {
  HK_REQUIRE(h && ops, "hk_kernel_ops_of: null argument");
  ops->self = h;
  ops->pools = c_pools;
  ops->push = c_push;
  ops->drain = c_drain;
  ops->error = c_error;
  ops->logprobs = c_logprobs;
  return HK_OK;
}

}  // extern "C"
