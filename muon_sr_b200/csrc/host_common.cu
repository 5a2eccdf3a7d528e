// Error reporting, device queries and the device error record shared by all kernels.
#include "host_common.h"
#include "common.cuh"

#include <string.h>

#include <atomic>
#include <mutex>
#include <set>
#include <utility>

namespace msr {

static thread_local char t_last_error[512] = "";
static std::atomic<uint64_t> g_launches{0};
static std::atomic<int> g_sr_noise{MSR_SR_NOISE_REFERENCE};

int sr_noise_mode() { return g_sr_noise.load(std::memory_order_relaxed); }

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int check_launch(const char* what) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(MSR_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return MSR_OK;
}

int sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

int set_smem_attr(const void* func, size_t bytes, const char* name) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(MSR_ERR_CUDA, "%s: cudaGetDevice: %s", name, cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({func, dev})) return MSR_OK;
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (e != cudaSuccess) return fail(MSR_ERR_CUDA, "%s: cudaFuncSetAttribute: %s", name, cudaGetErrorString(e));
  done.insert({func, dev});
  return MSR_OK;
}

int require_sm100() {
  int dev = 0, major = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(MSR_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  if (major != 10) return fail(MSR_ERR_UNSUPPORTED, "device %d is sm_%d.x; this build runs on sm_100a only", dev, major);
  return MSR_OK;
}

}  // namespace msr

extern "C" {

int msr_abi_version(void) { return 2; }

int msr_set_sr_noise(int mode) {
  if (mode != MSR_SR_NOISE_REFERENCE && mode != MSR_SR_NOISE_FAST && mode != MSR_SR_NOISE_NONE)
    return msr::fail(MSR_ERR_INVALID, "msr_set_sr_noise: unknown mode %d", mode);
  msr::g_sr_noise.store(mode);
  return MSR_OK;
}

int msr_get_sr_noise(void) { return msr::sr_noise_mode(); }

const char* msr_status_string(int status) {
  switch (status) {
    case MSR_OK: return "ok";
    case MSR_ERR_INVALID: return "invalid argument";
    case MSR_ERR_CUDA: return "CUDA error";
    case MSR_ERR_UNSUPPORTED: return "unsupported";
    case MSR_ERR_WORKSPACE: return "workspace too small";
    case MSR_ERR_DEVICE_TIMEOUT: return "device wait timed out";
    default: return "unknown status";
  }
}

const char* msr_last_error(void) { return msr::t_last_error; }

uint64_t msr_launch_count(void) { return msr::g_launches.load(std::memory_order_relaxed); }

}  // extern "C"
