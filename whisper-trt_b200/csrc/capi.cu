// Status reporting and process-wide settings of the C ABI.
#include <atomic>
#include <cstdarg>
#include <cstdint>
#include <cstdio>

#include "common.cuh"

namespace wt {

namespace {
thread_local char g_last_error[512] = "";
std::atomic<int> g_launch_flags{0};
constexpr unsigned kDefaultWaitLimit = 1u << 22;
std::atomic<unsigned> g_wait_limit{kDefaultWaitLimit};
std::atomic<int> g_withhold_stage{0};
}  // namespace

int fail(int status, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int launch_flags() { return g_launch_flags.load(std::memory_order_relaxed); }
unsigned wait_limit() { return g_wait_limit.load(std::memory_order_relaxed); }
int test_withhold_stage() { return g_withhold_stage.load(std::memory_order_relaxed); }

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int current_device(int *dev, const char *what) {
  const cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return fail(WT_ERR_CUDA, "%s: cudaGetDevice: %s", what, cudaGetErrorString(e));
  if (*dev < 0 || *dev >= kMaxDevices)
    return fail(WT_ERR_CUDA, "%s: device %d is beyond the %d this library tracks", what, *dev, kMaxDevices);
  return WT_OK;
}

namespace {
std::atomic<int> g_sm_counts[kMaxDevices];
}  // namespace

int device_sm_count() {
  int dev = 0;
  if (current_device(&dev, "sm count") != WT_OK) return 0;
  int n = g_sm_counts[dev].load(std::memory_order_relaxed);
  if (n > 0) return n;
  const cudaError_t e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess || n <= 0) {
    fail(WT_ERR_CUDA, "sm count: cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
    return 0;
  }
  g_sm_counts[dev].store(n, std::memory_order_relaxed);
  return n;
}

}  // namespace wt

extern "C" {

int wt_abi_version(void) { return WT_ABI_VERSION; }

const char *wt_status_string(int status) {
  switch (status) {
    case WT_OK: return "ok";
    case WT_ERR_ARG: return "invalid argument";
    case WT_ERR_ALIGN: return "pointer not 16-byte aligned";
    case WT_ERR_DTYPE: return "unknown element type";
    case WT_ERR_UNSUPPORTED: return "unsupported shape";
    case WT_ERR_WORKSPACE: return "workspace missing or too small";
    case WT_ERR_CUDA: return "CUDA launch failed";
    default: return "unknown status";
  }
}

const char *wt_last_error(void) { return wt::g_last_error; }

int wt_set_launch_flags(int flags) { return wt::g_launch_flags.exchange(flags); }

unsigned wt_set_wait_limit(unsigned polls) {
  return wt::g_wait_limit.exchange(polls == 0 ? wt::kDefaultWaitLimit : polls);
}

int wt_set_test_withhold_stage(int on) { return wt::g_withhold_stage.exchange(on != 0 ? 1 : 0); }

}  // extern "C"
