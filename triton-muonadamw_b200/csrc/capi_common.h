// Host-side helpers shared by the C-ABI entry points: a per-thread error
// message, status-returning failure helpers and cached device properties.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>

#include "muon_adamw_b200.h"  // include/ of the repository (-I)

namespace mad {

// Defined in capi.cu.
char* error_buffer();
constexpr int kErrorBufferSize = 512;

inline void clear_error() { error_buffer()[0] = '\0'; }

inline int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(error_buffer(), kErrorBufferSize, fmt, ap);
  va_end(ap);
  return code;
}

inline int fail_cuda(const char* what) {
  const cudaError_t e = cudaGetLastError();
  return fail(MAD_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

inline int check_launch(const char* kernel) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(MAD_ERR_CUDA, "launch of %s failed: %s", kernel, cudaGetErrorString(e));
  return MAD_OK;
}

// Number of SMs of the current device (queried per call: cheap, and correct
// when the caller switches devices).
inline int num_sms() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

}  // namespace mad
