// Pool sizing for the page and window pools: hk_pages_within, hk_plan_pools.
//   pages_within        src/gpu/load.rs:903-908
//   plan (pool part)    src/gpu/load.rs:510-533, state_bytes :535-537
// Host arithmetic only; hk_plan_pools reads the device's free memory when asked to.
#include <cuda_runtime_api.h>

#include <string>

#include "hk.h"

namespace hk {
int fail(int code, const char* fmt, ...);  // common.cu: sets hk_last_error()
}

namespace {

// The summed per-unit bytes of the states of one kind; false if the sum overflows.
bool cost(const hk_pool_sizing* p, uint32_t unit, uint64_t* out) {
  uint64_t c = 0;
  for (size_t i = 0; i < p->n_states; ++i)
    if (p->states[i].unit == unit && __builtin_add_overflow(c, p->states[i].bytes, &c)) return false;
  *out = c;
  return true;
}

bool valid(const hk_pool_sizing* p) {
  if (p->n_states > 0 && !p->states) return false;
  for (size_t i = 0; i < p->n_states; ++i)
    if (p->states[i].unit != HK_UNIT_PAGE && p->states[i].unit != HK_UNIT_WINDOW) return false;
  return true;
}

// 1 = sized, 0 = the bytes hold no sequence, -1 = a cost overflows.
int within(const hk_pool_sizing* p, uint64_t bytes, uint64_t* pages) {
  uint64_t wcost, pcost, wbytes;
  if (!cost(p, HK_UNIT_WINDOW, &wcost) || !cost(p, HK_UNIT_PAGE, &pcost)) return -1;
  if (__builtin_mul_overflow(p->window_pages, wcost, &wbytes)) return -1;
  if (wbytes > bytes) return 0;
  uint64_t n = (bytes - wbytes) / (pcost > 0 ? pcost : 1);
  if (n > p->pages) n = p->pages;
  if (n <= p->entries) return 0;
  *pages = n;
  return 1;
}

}  // namespace

extern "C" {

int hk_pages_within(const hk_pool_sizing* pool, uint64_t bytes, size_t* pages, size_t* window_pages) {
  if (!pool || !pages || !window_pages || !valid(pool)) return hk::fail(HK_EINVAL, "hk_pages_within: bad argument");
  uint64_t n = 0;
  const int r = within(pool, bytes, &n);
  if (r < 0) return hk::fail(HK_EINVAL, "hk_pages_within: pool state costs overflow");
  if (r == 0) return hk::fail(HK_ESPACE, "%llu B of pools hold no sequence", (unsigned long long)bytes);
  *pages = (size_t)n;
  *window_pages = (size_t)pool->window_pages;
  return HK_OK;
}

int hk_plan_pools(const hk_pool_sizing* pool, const hk_pool_budget* budget, size_t* pages,
                  size_t* window_pages, size_t* slots, uint64_t* used) {
  if (!pool || !budget || !pages || !window_pages || !slots || !used || !valid(pool))
    return hk::fail(HK_EINVAL, "hk_plan_pools: bad argument");
  uint64_t free = budget->free;
  if (free == 0) {
    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    size_t f = 0, total = 0;
    cudaError_t e = cudaSetDevice(budget->device);
    if (e == cudaSuccess) e = cudaMemGetInfo(&f, &total);
    if (prev >= 0) cudaSetDevice(prev);
    if (e != cudaSuccess)
      return hk::fail(HK_ECUDA, "hk_plan_pools: free memory of device %d: %s", budget->device,
                      cudaGetErrorString(e));
    free = f;
  }
  uint64_t other = 0;
  if (__builtin_add_overflow(budget->other, budget->slack, &other) || other > free)
    return hk::fail(HK_ESPACE, "the kernel's %llu B and %llu B of slack past the GPU's %llu B free",
                    (unsigned long long)budget->other, (unsigned long long)budget->slack,
                    (unsigned long long)free);
  const uint64_t bytes = free - other;
  uint64_t n = 0;
  const int r = within(pool, bytes, &n);
  if (r < 0) return hk::fail(HK_EINVAL, "hk_plan_pools: pool state costs overflow");
  if (r == 0)
    return hk::fail(HK_ESPACE, "%llu B of pools hold no sequence of %u positions", (unsigned long long)bytes,
                    budget->context);
  const uint64_t need = (uint64_t)budget->lanes + 1;
  if (need > pool->slots)
    return hk::fail(HK_EINVAL, "%u lanes past the bundle's %llu slots", budget->lanes,
                    (unsigned long long)pool->slots);
  uint64_t sum = 0;
  for (size_t i = 0; i < pool->n_states; ++i) {
    const hk_pool_state& st = pool->states[i];
    sum += st.bytes * (st.unit == HK_UNIT_PAGE ? n : pool->window_pages);  // <= bytes: no overflow
  }
  *pages = (size_t)n;
  *window_pages = (size_t)pool->window_pages;
  *slots = (size_t)need;
  *used = sum;
  return HK_OK;
}

}  // extern "C"
