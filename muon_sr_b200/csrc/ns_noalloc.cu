// Newton-Schulz for callers that cannot allocate device memory.
//
// msr_newton_schulz_bf16 asks its caller for a workspace (msr_ns_workspace_bytes) for the
// Gram matrices and the ping-pong copy of X. Some callers cannot hand one over: a plugin
// that a host program loads and gives only input and output buffers, because the host owns
// every device allocation through its own memory pool (a raw cudaMalloc next to such a pool
// can fail or fragment it), or a C / FFI caller that has no device allocator of its own.
// For them, msr_newton_schulz_bf16_noalloc takes its scratch from a fixed area that lives in
// this library's device memory, so it allocates nothing.
//
// The area is a file-scope __device__ array of NS_NOALLOC_SCRATCH_BYTES (64 MiB). Every GPU
// on which the library's kernels are loaded holds it until the process exits. Its device
// address is looked up once per device (cudaGetSymbolAddress, with that device current) on
// the first call made on that device; host code never uses the array's name as a pointer.
// The looked-up address is cached for the life of the process; a device reset (which
// destroys the primary context the address belongs to) is not detected, so callers must not
// use this entry point again after resetting the device.
#include "common.cuh"
#include "host_common.h"

#include <mutex>

namespace {

constexpr size_t NS_NOALLOC_SCRATCH_BYTES = size_t(64) << 20;
constexpr int MAX_DEVICES = 64;

static __device__ __align__(256) unsigned char g_ns_noalloc_scratch[NS_NOALLOC_SCRATCH_BYTES];

std::mutex g_scratch_mutex;
void* g_scratch_addr[MAX_DEVICES] = {};

// Device address of the scratch array on the current device (looked up on first use).
int scratch_address(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return msr::fail(MSR_ERR_CUDA, "msr_newton_schulz_bf16_noalloc: cudaGetDevice: %s",
                                         cudaGetErrorString(e));
  if (dev < 0 || dev >= MAX_DEVICES)
    return msr::fail(MSR_ERR_UNSUPPORTED, "msr_newton_schulz_bf16_noalloc: device index %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_ns_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return msr::fail(MSR_ERR_CUDA, "msr_newton_schulz_bf16_noalloc: cudaGetSymbolAddress on device %d: %s", dev,
                       cudaGetErrorString(e));
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return MSR_OK;
}

}  // namespace

extern "C" int msr_newton_schulz_bf16_noalloc(const void* x, void* out, int64_t batch, int64_t rows, int64_t cols,
                                              int steps, int mode, const float* norm_sq, msr_stream_t stream) {
  if (!x || !out || batch <= 0 || rows <= 0 || cols <= 0 || steps < 0)
    return msr::fail(MSR_ERR_INVALID, "msr_newton_schulz_bf16_noalloc: null pointer or bad size");
  const size_t need = msr_ns_workspace_bytes(batch, rows, cols);
  if (need > NS_NOALLOC_SCRATCH_BYTES)
    return msr::fail(MSR_ERR_WORKSPACE,
                     "msr_newton_schulz_bf16_noalloc: %lld x %lld x %lld needs %zu bytes of scratch, more than the "
                     "fixed %zu-byte area; call msr_newton_schulz_bf16 with a workspace instead",
                     (long long)batch, (long long)rows, (long long)cols, need, NS_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  if (int st = scratch_address(&scratch)) return st;
  // Same chain as msr_newton_schulz_bf16 with the fixed area as its workspace. Every scratch
  // word the chain reads it has written earlier in the same call (norm partials, Gram
  // matrices, ping-pong buffers, zero padding), so the previous call's leftovers need no
  // clearing.
  return msr_newton_schulz_bf16(x, out, batch, rows, cols, steps, mode, norm_sq, scratch, NS_NOALLOC_SCRATCH_BYTES,
                                stream);
}
