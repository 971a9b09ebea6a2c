// Expert-parallel dispatch and return over NVLink peer memory (no NCCL on the data path).
//
// Every rank holds the same set of symmetric buffers (one allocation per rank, each mapped into
// every rank's address space; `hk_ep_peers` carries the addresses).  Rank r owns experts
// [r El, (r+1) El), El = E / world.
//
//   hk_ep_counts    one CTA: writes this rank's per-expert row counts into row `rank` of every
//                   rank's count matrix [world][E], raises its epoch flag on every rank, waits
//                   until all ranks' flags carry the epoch, then derives from the full matrix
//                     send_base[e]  where this rank's rows of expert e start in the owner's
//                                   receive buffer (expert-major, sources in rank order),
//                     local_off[el] the receive buffer's expert offsets (for the grouped FFN),
//                     ret_base[s][el] where source s's rows of local expert el sit in s's
//                                   permuted order.
//   hk_ep_dispatch  a warp per routed row: copies xq[perm_token[p]] and its scales straight into
//                   the owner's receive buffers at send_base[e] + (p - offsets[e]); the last
//                   CTA to finish raises the dispatch flag on every rank.
//   hk_ep_return    a warp per received row: copies the expert output back into the source's
//                   return buffer at its permuted position; the last CTA raises the return flag.
//   hk_ep_wait      one thread: waits for a flag word from every rank to carry the epoch.
//
// Flags are epochs (a step counter the caller increments), so nothing is reset between steps.
// Every wait is bounded (timeout_us); on a timeout the kernel records the error word and
// returns, leaving the buffers undefined for that step.  A count exchange that timed out marks
// the step's plan invalid (send_base = -1, local_off[El] = -1): dispatch and return then move no
// row and raise no flag, so the other ranks' waits run out too and every rank reports the step.
#include "common.cuh"

namespace {

constexpr int kMaxWorld = 8;

struct Peers {
  void* p[kMaxWorld];
};

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void store_release_sys(uint32_t* addr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t load_acquire_sys(const uint32_t* addr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// Waits until flags[s] == epoch for every s < world (flags in this rank's memory).
__device__ bool wait_all(const uint32_t* flags, int world, uint32_t epoch, long long timeout_ns) {
  const unsigned long long t0 = now_ns();
  for (int s = 0; s < world; ++s) {
    while (load_acquire_sys(flags + s) != epoch) {
      if ((long long)(now_ns() - t0) > timeout_ns) return false;
    }
  }
  return true;
}

// flags layout in every rank's flag buffer: [3][kMaxWorld] words: counts, dispatch, return.
constexpr int kFlagCounts = 0, kFlagDispatch = kMaxWorld, kFlagReturn = 2 * kMaxWorld;

__global__ void ep_counts_kernel(const int32_t* __restrict__ offsets, int32_t E, int32_t world, int32_t rank,
                                 Peers counts, Peers flags, uint32_t epoch, long long timeout_ns,
                                 int32_t* __restrict__ send_base, int32_t* __restrict__ local_off,
                                 int32_t* __restrict__ ret_base, unsigned long long* err) {
  const int El = E / world;
  // 1. my counts into row `rank` of every rank's matrix
  for (int d = 0; d < world; ++d) {
    int32_t* m = reinterpret_cast<int32_t*>(counts.p[d]) + rank * E;
    for (int e = threadIdx.x; e < E; e += blockDim.x) m[e] = offsets[e + 1] - offsets[e];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int d = 0; d < world; ++d)
      store_release_sys(reinterpret_cast<uint32_t*>(flags.p[d]) + kFlagCounts + rank, epoch);
  }
  // 2. wait for every rank's row
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = wait_all(reinterpret_cast<const uint32_t*>(flags.p[rank]) + kFlagCounts, world, epoch, timeout_ns);
    if (!ok) hk_flag(err, hk::kErrWaitTimeout, 970);
  }
  __syncthreads();
  if (!ok) {
    // Mark this step's plan invalid, so hk_ep_dispatch and hk_ep_return skip (and flag) every
    // row instead of moving rows at stale offsets.
    for (int e = threadIdx.x; e < E; e += blockDim.x) send_base[e] = -1;
    for (int el = threadIdx.x; el <= El; el += blockDim.x) local_off[el] = el == El ? -1 : 0;
    return;
  }
  const int32_t* cnt = reinterpret_cast<const int32_t*>(counts.p[rank]);  // [world][E], all rows present
  // 3. send_base[e]: destination d = e / El, local el = e % El
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int d = e / El, el = e % El;
    int pos = 0;
    for (int e2 = d * El; e2 < d * El + el; ++e2)
      for (int s = 0; s < world; ++s) pos += cnt[s * E + e2];
    for (int s = 0; s < rank; ++s) pos += cnt[s * E + e];
    send_base[e] = pos;
  }
  // local offsets of my experts and the return bases
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int el = 0; el < El; ++el) {
      local_off[el] = acc;
      for (int s = 0; s < world; ++s) acc += cnt[s * E + rank * El + el];
    }
    local_off[El] = acc;
  }
  for (int i = threadIdx.x; i < world * El; i += blockDim.x) {
    const int s = i / El, el = i % El;
    int pos = 0;
    for (int e2 = 0; e2 < rank * El + el; ++e2) pos += cnt[s * E + e2];
    ret_base[i] = pos;
  }
}

// Copies `vecs` 16-byte words (and `svecs` 4-byte scale words) of one row with a warp.
__device__ __forceinline__ void copy_row(const uint4* src, uint4* dst, int vecs, const float* ssrc, float* sdst,
                                         int svecs, int lane) {
  for (int i = lane; i < vecs; i += 32) dst[i] = src[i];
  for (int i = lane; i < svecs; i += 32) sdst[i] = ssrc[i];
}

// Raises flag word `slot` (+ rank) on every rank once every CTA of the grid is done (when
// `raise` is false the counter is still reset but no flag goes up, so the other ranks' waits
// run out and report the failed step).
__device__ void last_cta_signals(uint32_t* done_ctr, Peers flags, int world, int rank, int slot, uint32_t epoch,
                                 bool raise = true) {
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(done_ctr, 1u);
    if (prev == gridDim.x - 1) {
      *done_ctr = 0;  // ready for the next step (every CTA of this launch has counted)
      __threadfence_system();
      if (raise)
        for (int d = 0; d < world; ++d)
          store_release_sys(reinterpret_cast<uint32_t*>(flags.p[d]) + slot + rank, epoch);
    }
  }
}

__global__ void ep_dispatch_kernel(const uint8_t* __restrict__ xq, const float* __restrict__ sx, int32_t tokens,
                                   const int32_t* __restrict__ perm_token, const int32_t* __restrict__ offsets,
                                   int32_t rows, int32_t E, int32_t world, int32_t rank, int32_t hidden,
                                   int32_t rows_cap, const int32_t* __restrict__ send_base, Peers recv_x,
                                   Peers recv_s, Peers flags, uint32_t* done_ctr, uint32_t epoch,
                                   unsigned long long* err) {
  const int El = E / world, kb = hidden / 128;
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  // send_base[0] < 0: this step's count exchange failed; move nothing and raise no flag.
  const bool valid = send_base[0] >= 0;
  if (!valid && blockIdx.x == 0 && threadIdx.x == 0) hk_flag(err, hk::kErrMoeRow, 0x7ffffffeu);
  if (!valid) rows = 0;
  for (int p = blockIdx.x * warps + (threadIdx.x >> 5); p < rows; p += gridDim.x * warps) {
    int lo = 0, hi = E;  // expert e with offsets[e] <= p < offsets[e+1]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (offsets[mid] <= p) lo = mid; else hi = mid;
    }
    const int e = lo, d = e / El;
    const int src = perm_token[p];
    const int dst = send_base[e] + (p - offsets[e]);
    if (src < 0 || src >= tokens || dst < 0 || dst >= rows_cap || d >= world) {
      if (lane == 0) hk_flag(err, hk::kErrMoeRow, (unsigned)p);
      continue;
    }
    copy_row(reinterpret_cast<const uint4*>(xq + (int64_t)src * hidden),
             reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(recv_x.p[d]) + (int64_t)dst * hidden), hidden / 16,
             sx + (int64_t)src * kb, reinterpret_cast<float*>(recv_s.p[d]) + (int64_t)dst * kb, kb, lane);
  }
  last_cta_signals(done_ctr, flags, world, rank, kFlagDispatch, epoch, valid);
}

__global__ void ep_return_kernel(const uint16_t* __restrict__ y, int32_t E, int32_t world, int32_t rank,
                                 int32_t hidden, const int32_t* __restrict__ local_off,
                                 const int32_t* __restrict__ counts, const int32_t* __restrict__ ret_base,
                                 int32_t back_cap, int32_t rows_bound, Peers back_y, Peers flags,
                                 uint32_t* done_ctr, uint32_t epoch, unsigned long long* err) {
  const int El = E / world;
  const int warps = blockDim.x >> 5, lane = threadIdx.x & 31;
  // local_off[El] comes from counts the peers wrote: never read y past its rows_bound rows,
  // and move nothing when this step's count exchange failed (local_off[El] < 0).
  const int total = local_off[El];
  const bool valid = total >= 0 && total <= rows_bound;
  if (!valid && blockIdx.x == 0 && threadIdx.x == 0) hk_flag(err, hk::kErrMoeRow, 0x7fffffffu);
  const int rows = valid ? total : 0;
  for (int j = blockIdx.x * warps + (threadIdx.x >> 5); j < rows; j += gridDim.x * warps) {
    int lo = 0, hi = El;  // local expert of row j
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (local_off[mid] <= j) lo = mid; else hi = mid;
    }
    const int el = lo, e = rank * El + el;
    int i = j - local_off[el], s = 0;  // source rank of the row: sources in rank order
    while (s < world - 1 && i >= counts[s * E + e]) i -= counts[s * E + e], ++s;
    const int pos = ret_base[s * El + el] + i;
    if (pos < 0 || pos >= back_cap) {
      if (lane == 0) hk_flag(err, hk::kErrMoeRow, (unsigned)j);
      continue;
    }
    copy_row(reinterpret_cast<const uint4*>(y + (int64_t)j * hidden),
             reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(back_y.p[s]) + (int64_t)pos * hidden),
             hidden * 2 / 16, nullptr, nullptr, 0, lane);
  }
  last_cta_signals(done_ctr, flags, world, rank, kFlagReturn, epoch, valid);
}

__global__ void ep_wait_kernel(const uint32_t* flags, int32_t slot, int32_t world, uint32_t epoch,
                               long long timeout_ns, unsigned long long* err) {
  if (threadIdx.x == 0 && !wait_all(flags + slot, world, epoch, timeout_ns))
    hk_flag(err, hk::kErrWaitTimeout, 971 + slot / kMaxWorld);
}

int peers_of(const uint64_t* addrs, int world, Peers* out) {
  HK_REQUIRE(addrs && world >= 1 && world <= kMaxWorld, "hk_ep: world %d (1..%d) and peer addresses", world,
             kMaxWorld);
  for (int i = 0; i < kMaxWorld; ++i) out->p[i] = i < world ? reinterpret_cast<void*>(addrs[i]) : nullptr;
  for (int i = 0; i < world; ++i) HK_REQUIRE(out->p[i] != nullptr, "hk_ep: null peer address of rank %d", i);
  return HK_OK;
}

}  // namespace

extern "C" {

int hk_ep_counts(const int32_t* offsets, int32_t num_experts, int32_t world, int32_t rank, const uint64_t* counts,
                 const uint64_t* flags, uint32_t epoch, int32_t timeout_us, int32_t* send_base, int32_t* local_off,
                 int32_t* ret_base, void* stream) {
  HK_TRY(hk::ensure_device());
  Peers c, f;
  HK_TRY(peers_of(counts, world, &c));
  HK_TRY(peers_of(flags, world, &f));
  HK_REQUIRE(offsets && send_base && local_off && ret_base, "hk_ep_counts: null pointer");
  HK_REQUIRE(rank >= 0 && rank < world && num_experts > 0 && num_experts % world == 0,
             "hk_ep_counts: rank %d of %d, %d experts (a multiple of the world)", rank, world, num_experts);
  HK_REQUIRE(epoch != 0 && timeout_us > 0, "hk_ep_counts: epoch must be nonzero, timeout positive");
  ep_counts_kernel<<<1, 256, 0, (cudaStream_t)stream>>>(offsets, num_experts, world, rank, c, f, epoch,
                                                        (long long)timeout_us * 1000, send_base, local_off,
                                                        ret_base, hk::err_word());
  HK_TRY_LAUNCH("ep_counts_kernel");
  return HK_OK;
}

int hk_ep_dispatch(const uint8_t* xq, const float* sx, int32_t tokens, const int32_t* perm_token,
                   const int32_t* offsets, int32_t rows, int32_t num_experts, int32_t world, int32_t rank,
                   int32_t hidden, int32_t rows_cap, const int32_t* send_base, const uint64_t* recv_x,
                   const uint64_t* recv_s, const uint64_t* flags, uint32_t* done_ctr, uint32_t epoch, void* stream) {
  HK_TRY(hk::ensure_device());
  Peers rx, rs, f;
  HK_TRY(peers_of(recv_x, world, &rx));
  HK_TRY(peers_of(recv_s, world, &rs));
  HK_TRY(peers_of(flags, world, &f));
  HK_REQUIRE(xq && sx && perm_token && offsets && send_base && done_ctr, "hk_ep_dispatch: null pointer");
  HK_REQUIRE(hidden > 0 && hidden % 128 == 0 && rows >= 0 && num_experts % world == 0 && rank >= 0 && rank < world,
             "hk_ep_dispatch: hidden %d rows %d experts %d world %d", hidden, rows, num_experts, world);
  HK_REQUIRE(((uintptr_t)xq % 16 == 0), "hk_ep_dispatch: xq must be 16-byte aligned");
  const int grid = std::max(1, std::min(hk::sm_count(), (rows + 7) / 8));
  ep_dispatch_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(xq, sx, tokens, perm_token, offsets, rows, num_experts,
                                                             world, rank, hidden, rows_cap, send_base, rx, rs, f,
                                                             done_ctr, epoch, hk::err_word());
  HK_TRY_LAUNCH("ep_dispatch_kernel");
  return HK_OK;
}

int hk_ep_return(const uint16_t* y, int32_t num_experts, int32_t world, int32_t rank, int32_t hidden,
                 const int32_t* local_off, const int32_t* counts, const int32_t* ret_base, int32_t back_cap,
                 int32_t rows_bound, const uint64_t* back_y, const uint64_t* flags, uint32_t* done_ctr,
                 uint32_t epoch, void* stream) {
  HK_TRY(hk::ensure_device());
  Peers b, f;
  HK_TRY(peers_of(back_y, world, &b));
  HK_TRY(peers_of(flags, world, &f));
  HK_REQUIRE(y && local_off && counts && ret_base && done_ctr, "hk_ep_return: null pointer");
  HK_REQUIRE(hidden > 0 && hidden % 8 == 0 && num_experts % world == 0 && rank >= 0 && rank < world,
             "hk_ep_return: hidden %d experts %d world %d", hidden, num_experts, world);
  const int grid = std::max(1, std::min(hk::sm_count(), (rows_bound + 7) / 8));
  ep_return_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(y, num_experts, world, rank, hidden, local_off, counts,
                                                           ret_base, back_cap, rows_bound, b, f, done_ctr,
                                                           epoch, hk::err_word());
  HK_TRY_LAUNCH("ep_return_kernel");
  return HK_OK;
}

int hk_ep_wait(const uint32_t* flags, int32_t which, int32_t world, uint32_t epoch, int32_t timeout_us,
               void* stream) {
  HK_TRY(hk::ensure_device());
  HK_REQUIRE(flags && which >= 0 && which < 3 && world >= 1 && world <= kMaxWorld && timeout_us > 0,
             "hk_ep_wait: flag set %d (0 counts, 1 dispatch, 2 return), world %d", which, world);
  ep_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(flags, which * kMaxWorld, world, epoch,
                                                     (long long)timeout_us * 1000, hk::err_word());
  HK_TRY_LAUNCH("ep_wait_kernel");
  return HK_OK;
}

}  // extern "C"
