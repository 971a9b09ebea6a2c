// Multi-GPU plumbing of the C ABI without PyTorch or NCCL on the data path.
//
//   hk_sym_alloc / hk_sym_import / hk_sym_close / hk_sym_free
//       a buffer one rank allocates (zeroed) and every other rank maps into its address space
//       from a 64-byte CUDA IPC handle the host passes around as bytes (any channel: the
//       reference's rank fabric, a socket, torch.distributed's object gather).  The expert-
//       parallel exchange (hk_ep_*) and the context-parallel merge below take the mapped
//       addresses of every rank's copy.
//   hk_cp_merge
//       the context-parallel exchange fused with its LSE merge: every rank's (o, lse) partial for
//       the same query rows sits in that rank's own symmetric buffer; a rank raises its epoch
//       flag on every rank, waits (bounded) for all flags, then reads every rank's partial over
//       NVLink with plain loads and merges them row by row (what an all-gather followed by
//       hk_lse_merge computes, without gathering the partials into local memory first).
#include <math.h>
#include <string.h>

#include "common.cuh"

namespace {

constexpr int kMaxWorld = 8;

struct Ptrs {
  const void* p[kMaxWorld];
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

constexpr int kMergeThreads = 256;

// Grid: rows are split over the CTAs, a warp per row.  Each CTA's thread 0 raises this rank's
// flag on every rank, then waits for all ranks' flags (bounded).
__global__ void __launch_bounds__(kMergeThreads)
    cp_merge_kernel(Ptrs o_parts, Ptrs lse_parts, Ptrs flags, int32_t world, int32_t rank, uint32_t epoch,
                    long long timeout_ns, int64_t rows, int32_t dv, uint16_t* __restrict__ out,
                    float* __restrict__ lse_out, unsigned long long* err) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    // every CTA raises the flag (the same value), so no CTA's wait depends on another being resident
    __threadfence_system();  // this rank's partial (written by earlier kernels) before its flag
    for (int d = 0; d < world; ++d)
      store_release_sys(const_cast<uint32_t*>(reinterpret_cast<const uint32_t*>(flags.p[d])) + rank, epoch);
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(flags.p[rank]);
    const unsigned long long t0 = now_ns();
    int good = 1;
    for (int s = 0; s < world && good; ++s)
      while (load_acquire_sys(mine + s) != epoch) {
        if ((long long)(now_ns() - t0) > timeout_ns) {
          good = 0;
          break;
        }
      }
    if (!good) hk_flag(err, hk::kErrWaitTimeout, 980);
    ok = good;
  }
  __syncthreads();
  if (!ok) return;
  const int warps = kMergeThreads / 32, lane = threadIdx.x & 31;
  for (int64_t r = (int64_t)blockIdx.x * warps + (threadIdx.x >> 5); r < rows; r += (int64_t)gridDim.x * warps) {
    float l[kMaxWorld];
    float m = -INFINITY;
    for (int s = 0; s < world; ++s) {
      l[s] = __ldcg(reinterpret_cast<const float*>(lse_parts.p[s]) + r);
      m = fmaxf(m, l[s]);
    }
    float w[kMaxWorld];
    float den = 0.f;
    for (int s = 0; s < world; ++s) {
      w[s] = (m == -INFINITY || l[s] == -INFINITY) ? 0.f : expf(l[s] - m);
      den += w[s];
    }
    const float inv = den > 0.f ? 1.0f / den : 0.f;
    for (int c = lane * 4; c < dv; c += 128) {
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int s = 0; s < world; ++s) {
        if (w[s] == 0.f) continue;
        const float4 v = __ldcg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(o_parts.p[s]) +
                                                                r * dv + c));
        acc.x += w[s] * v.x;
        acc.y += w[s] * v.y;
        acc.z += w[s] * v.z;
        acc.w += w[s] * v.w;
      }
      uint16_t* o = out + r * dv + c;
      o[0] = f32_to_bf16_bits(acc.x * inv);
      o[1] = f32_to_bf16_bits(acc.y * inv);
      o[2] = f32_to_bf16_bits(acc.z * inv);
      o[3] = f32_to_bf16_bits(acc.w * inv);
    }
    if (lane == 0 && lse_out) lse_out[r] = den > 0.f ? m + logf(den) : -INFINITY;
  }
}

int ptrs_of(const uint64_t* addrs, int world, Ptrs* out, const char* what) {
  HK_REQUIRE(addrs && world >= 1 && world <= kMaxWorld, "%s: world %d (1..%d) and peer addresses", what, world,
             kMaxWorld);
  for (int i = 0; i < kMaxWorld; ++i) out->p[i] = i < world ? reinterpret_cast<const void*>(addrs[i]) : nullptr;
  for (int i = 0; i < world; ++i) HK_REQUIRE(out->p[i] != nullptr, "%s: null address of rank %d", what, i);
  return HK_OK;
}

}  // namespace

extern "C" {

int hk_sym_alloc(size_t bytes, void** ptr, hk_ipc_handle* handle) {
  HK_TRY(hk::ensure_device());
  HK_REQUIRE(ptr && handle && bytes > 0, "hk_sym_alloc: null argument or zero bytes");
  *ptr = nullptr;
  void* p = nullptr;
  HK_TRY_CUDA(cudaMalloc(&p, bytes));
  cudaError_t e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(p);
    return hk::cuda_fail(e, "hk_sym_alloc");
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == sizeof(handle->bytes), "IPC handle size");
  memcpy(handle->bytes, &h, sizeof h);
  *ptr = p;
  return HK_OK;
}

int hk_sym_import(const hk_ipc_handle* handle, void** ptr) {
  HK_TRY(hk::ensure_device());
  HK_REQUIRE(handle && ptr, "hk_sym_import: null argument");
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle->bytes, sizeof h);
  HK_TRY_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return HK_OK;
}

int hk_sym_close(void* peer_ptr) {
  HK_REQUIRE(peer_ptr, "hk_sym_close: null address");
  HK_TRY_CUDA(cudaIpcCloseMemHandle(peer_ptr));
  return HK_OK;
}

int hk_sym_free(void* ptr) {
  HK_REQUIRE(ptr, "hk_sym_free: null address");
  HK_TRY_CUDA(cudaFree(ptr));
  return HK_OK;
}

int hk_cp_merge(const uint64_t* o_parts, const uint64_t* lse_parts, const uint64_t* flags, int32_t world,
                int32_t rank, uint32_t epoch, int32_t timeout_us, int64_t rows, int32_t dv, uint16_t* out,
                float* lse_out, void* stream) {
  HK_TRY(hk::ensure_device());
  Ptrs o, l, f;
  HK_TRY(ptrs_of(o_parts, world, &o, "hk_cp_merge o_parts"));
  HK_TRY(ptrs_of(lse_parts, world, &l, "hk_cp_merge lse_parts"));
  HK_TRY(ptrs_of(flags, world, &f, "hk_cp_merge flags"));
  HK_REQUIRE(rank >= 0 && rank < world && epoch != 0 && timeout_us > 0,
             "hk_cp_merge: rank %d of %d, nonzero epoch, positive timeout", rank, world);
  HK_REQUIRE(rows >= 0 && dv > 0 && dv % 4 == 0 && (rows == 0 || out), "hk_cp_merge: rows %lld dv %d",
             (long long)rows, dv);
  for (int i = 0; i < world; ++i)
    HK_REQUIRE(((uintptr_t)o.p[i] % 16) == 0, "hk_cp_merge: partial of rank %d not 16-byte aligned", i);
  const int64_t per = kMergeThreads / 32;
  int64_t grid = (rows + per - 1) / per;
  const int64_t cap = (int64_t)hk::sm_count();
  grid = grid < 1 ? 1 : grid > cap ? cap : grid;
  cp_merge_kernel<<<(unsigned)grid, kMergeThreads, 0, (cudaStream_t)stream>>>(
      o, l, f, world, rank, epoch, (long long)timeout_us * 1000, rows, dv, out, lse_out, hk::err_word());
  HK_TRY_LAUNCH("cp_merge_kernel");
  return HK_OK;
}

}  // extern "C"
