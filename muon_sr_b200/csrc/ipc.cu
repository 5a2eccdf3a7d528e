// Peer mappings of device allocations for the sharded step's weight sharing: each rank
// maps the allocations that hold the parameters other ranks own and pulls the updated
// weights with copy-engine peer copies over NVLink, which leaves every SM to the
// Newton-Schulz GEMMs. Plain CUDA IPC (cudaIpcGetMemHandle / cudaIpcOpenMemHandle) on
// cudaMalloc'd allocations; no multicast objects are involved.
#include "common.cuh"
#include "host_common.h"

#include <cuda.h>

#include <mutex>

namespace {

using GetRangeFn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);

GetRangeFn get_range_fn() {
  static GetRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<GetRangeFn>(p);
  });
  return fn;
}

}  // namespace

extern "C" {

int msr_ipc_export(const void* ptr, void* handle_out, uint64_t* offset_out) {
  if (!ptr || !handle_out || !offset_out) return msr::fail(MSR_ERR_INVALID, "msr_ipc_export: null argument");
  GetRangeFn range = get_range_fn();
  if (!range) return msr::fail(MSR_ERR_CUDA, "msr_ipc_export: cuMemGetAddressRange is not available");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return msr::fail(MSR_ERR_CUDA, "msr_ipc_export: pointer %p is not device memory", ptr);
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess)
    return msr::fail(MSR_ERR_UNSUPPORTED, "msr_ipc_export: cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<uint64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return MSR_OK;
}

int msr_ipc_import(const void* handle, void** base_out) {
  if (!handle || !base_out) return msr::fail(MSR_ERR_INVALID, "msr_ipc_import: null argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess)
    return msr::fail(MSR_ERR_UNSUPPORTED, "msr_ipc_import: cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  return MSR_OK;
}

int msr_ipc_close(void* base) {
  if (!base) return MSR_OK;
  cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) return msr::fail(MSR_ERR_CUDA, "msr_ipc_close: %s", cudaGetErrorString(e));
  return MSR_OK;
}

int msr_ipc_event_create(void** event_out, void* handle_out) {
  if (!event_out || !handle_out) return msr::fail(MSR_ERR_INVALID, "msr_ipc_event_create: null argument");
  cudaEvent_t ev;
  cudaError_t e = cudaEventCreateWithFlags(&ev, cudaEventInterprocess | cudaEventDisableTiming);
  if (e != cudaSuccess) return msr::fail(MSR_ERR_CUDA, "msr_ipc_event_create: %s", cudaGetErrorString(e));
  cudaIpcEventHandle_t h;
  e = cudaIpcGetEventHandle(&h, ev);
  if (e != cudaSuccess) {
    cudaEventDestroy(ev);
    return msr::fail(MSR_ERR_CUDA, "msr_ipc_event_create: cudaIpcGetEventHandle: %s", cudaGetErrorString(e));
  }
  memcpy(handle_out, &h, sizeof(h));
  *event_out = ev;
  return MSR_OK;
}

int msr_ipc_event_open(const void* handle, void** event_out) {
  if (!handle || !event_out) return msr::fail(MSR_ERR_INVALID, "msr_ipc_event_open: null argument");
  cudaIpcEventHandle_t h;
  memcpy(&h, handle, sizeof(h));
  cudaEvent_t ev;
  cudaError_t e = cudaIpcOpenEventHandle(&ev, h);
  if (e != cudaSuccess) return msr::fail(MSR_ERR_CUDA, "msr_ipc_event_open: %s", cudaGetErrorString(e));
  *event_out = ev;
  return MSR_OK;
}

int msr_event_record(void* event, msr_stream_t stream) {
  cudaError_t e = cudaEventRecord(static_cast<cudaEvent_t>(event), msr::to_stream(stream));
  if (e != cudaSuccess) return msr::fail(MSR_ERR_CUDA, "msr_event_record: %s", cudaGetErrorString(e));
  return MSR_OK;
}

int msr_stream_wait_event(msr_stream_t stream, void* event) {
  cudaError_t e = cudaStreamWaitEvent(msr::to_stream(stream), static_cast<cudaEvent_t>(event), 0);
  if (e != cudaSuccess) return msr::fail(MSR_ERR_CUDA, "msr_stream_wait_event: %s", cudaGetErrorString(e));
  return MSR_OK;
}

int msr_event_destroy(void* event) {
  if (!event) return MSR_OK;
  cudaError_t e = cudaEventDestroy(static_cast<cudaEvent_t>(event));
  if (e != cudaSuccess) return msr::fail(MSR_ERR_CUDA, "msr_event_destroy: %s", cudaGetErrorString(e));
  return MSR_OK;
}

int msr_copy_async(void* dst, const void* src, size_t bytes, msr_stream_t stream) {
  if (bytes == 0) return MSR_OK;
  if (!dst || !src) return msr::fail(MSR_ERR_INVALID, "msr_copy_async: null pointer");
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, msr::to_stream(stream));
  if (e != cudaSuccess) return msr::fail(MSR_ERR_CUDA, "msr_copy_async: %s", cudaGetErrorString(e));
  return MSR_OK;
}

}  // extern "C"
