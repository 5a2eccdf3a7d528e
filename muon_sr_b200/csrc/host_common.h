// Host-side helpers shared by the C entry points: error reporting and launch sizing.
#pragma once

#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>

#include "../../include/muon_sr_b200.h"

namespace msr {

// Records a formatted detail message for msr_last_error() and returns `status`.
int fail(int status, const char* fmt, ...);

// Checks the launch of the kernel just enqueued (or any earlier sticky error).
int check_launch(const char* what);

// Number of SMs of the current device (cached per device).
int sm_count();

// Returns MSR_ERR_UNSUPPORTED unless the current device is compute capability 10.x.
int require_sm100();

inline cudaStream_t to_stream(msr_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

// Sets cudaFuncAttributeMaxDynamicSharedMemorySize of kernel function `func` to `bytes`,
// once per (function, device); returns an MSR status.
int set_smem_attr(const void* func, size_t bytes, const char* name);

// Stochastic-rounding noise stream selected with msr_set_sr_noise (an msr_sr_noise value).
int sr_noise_mode();

// The kernel instance for the selected noise stream.
template <class F>
F pick_noise(F reference, F fast, F none) {
  switch (sr_noise_mode()) {
    case MSR_SR_NOISE_FAST: return fast;
    case MSR_SR_NOISE_NONE: return none;
    default: return reference;
  }
}

}  // namespace msr
