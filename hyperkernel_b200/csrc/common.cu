// Host-side plumbing shared by every entry point: the thread-local error message, device
// checks and the per-device error word that kernels use to report bad input without
// faulting.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "common.cuh"

namespace hk {

namespace {
thread_local char g_msg[512] = "";
constexpr int kMaxDevices = 64;
unsigned long long* g_err[kMaxDevices] = {};
int g_sms[kMaxDevices] = {};
int g_ok[kMaxDevices] = {};  // 0 unknown, 1 usable, -1 not usable
std::mutex g_mu;
std::atomic<unsigned long long> g_launches{0};
}  // namespace

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_msg, sizeof g_msg, fmt, ap);
  va_end(ap);
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  cudaGetLastError();  // clear a sticky launch error so the next call starts clean
  if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver)
    return fail(HK_ENODEV, "%s: %s", what, cudaGetErrorString(e));
  return fail(HK_ECUDA, "%s: %s", what, cudaGetErrorString(e));
}

void clear_error() { g_msg[0] = 0; }

static int current(int* dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (*dev < 0 || *dev >= kMaxDevices) return fail(HK_ENODEV, "device %d out of range", *dev);
  return HK_OK;
}

int ensure_device() {
  int dev;
  HK_TRY(current(&dev));
  if (g_ok[dev] == 1) return HK_OK;
  std::lock_guard<std::mutex> lock(g_mu);
  cudaDeviceProp p;
  cudaError_t e = cudaGetDeviceProperties(&p, dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
  if (p.major != 10) {
    g_ok[dev] = -1;
    return fail(HK_ENODEV, "device %d is sm_%d%d; this library is built for sm_100a only", dev,
                p.major, p.minor);
  }
  g_sms[dev] = p.multiProcessorCount;
  g_ok[dev] = 1;
  return HK_OK;
}

unsigned long long* err_word() {
  int dev;
  if (current(&dev) != HK_OK) return nullptr;
  if (g_err[dev] != nullptr) return g_err[dev];
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_err[dev] == nullptr) {
    unsigned long long* w = nullptr;
    if (cudaMalloc(&w, sizeof(unsigned long long)) != cudaSuccess) return nullptr;
    cudaMemset(w, 0, sizeof(unsigned long long));
    cudaDeviceSynchronize();
    g_err[dev] = w;
  }
  return g_err[dev];
}

int sm_count() {
  int dev;
  if (current(&dev) != HK_OK) return 148;
  if (g_sms[dev] == 0) ensure_device();
  return g_sms[dev] > 0 ? g_sms[dev] : 148;
}

}  // namespace hk

extern "C" {

const char* hk_version(void) { return "hyperkernel_b200 0.1.0 (sm_100a)"; }

const char* hk_last_error(void) { return hk::g_msg; }

uint64_t hk_kernel_launches(void) { return hk::g_launches.load(std::memory_order_relaxed); }

int hk_device_info(int* sm_count, int* cc_major, int* cc_minor) {
  HK_REQUIRE(sm_count && cc_major && cc_minor, "hk_device_info: null output");
  int dev;
  HK_TRY(hk::current(&dev));
  cudaDeviceProp p;
  HK_TRY_CUDA(cudaGetDeviceProperties(&p, dev));
  *sm_count = p.multiProcessorCount;
  *cc_major = p.major;
  *cc_minor = p.minor;
  return HK_OK;
}

int hk_check_errors(void) {
  HK_TRY(hk::ensure_device());
  unsigned long long* w = hk::err_word();
  if (w == nullptr) return hk::fail(HK_ECUDA, "no device error word");
  HK_TRY_CUDA(cudaDeviceSynchronize());
  unsigned long long v = 0;
  HK_TRY_CUDA(cudaMemcpy(&v, w, sizeof v, cudaMemcpyDeviceToHost));
  if (v == 0) return HK_OK;
  HK_TRY_CUDA(cudaMemset(w, 0, sizeof v));
  static const char* names[] = {"?",         "pack overflow",  "pack page", "append slot",
                                "attn page", "wait timeout",   "moe row",   "route input",
                                "token id"};
  unsigned site = (unsigned)((v >> 32) & 0x7fffffff);
  unsigned detail = (unsigned)(v & 0xffffffffu);
  return hk::fail(HK_EDEVICE, "device error: %s (site %u, detail %u)",
                  site < sizeof(names) / sizeof(names[0]) ? names[site] : "?", site, detail);
}

}  // extern "C"
