// Host-side helpers shared by the C-ABI entry points: a per-thread error
// message, status-returning failure helpers and cached device properties.
#pragma once

#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "elem_io.cuh"
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

// Device form of a mad_grad_reduce (null: no reduction, the local gradient).
inline int grad_reduce_from(const mad_grad_reduce* in, GradReduce* out, const char* who) {
  static_assert(MAD_MAX_RANKS == MAX_RANKS, "rank limit of the C ABI and the kernels");
  std::memset(out, 0, sizeof(*out));
  if (!in) return MAD_OK;
  if (in->n_ranks < 1 || in->n_ranks > MAX_RANKS)
    return fail(MAD_ERR_INVALID, "%s: n_ranks %d outside 1..%d", who, in->n_ranks, MAX_RANKS);
  if (!std::isfinite(in->scale)) return fail(MAD_ERR_INVALID, "%s: non-finite gradient scale", who);
  // The kernels read every rank's copy with 16-byte vector loads at g + delta[k];
  // a delta off that grid would make those loads misaligned on the device.
  for (int k = 0; k < in->n_ranks; ++k)
    if (in->delta[k] % 16 != 0)
      return fail(MAD_ERR_ALIGN, "%s: delta[%d] = %lld is not a multiple of 16 bytes", who, k,
                  static_cast<long long>(in->delta[k]));
  out->n = in->n_ranks;
  out->scale = in->scale;
  for (int k = 0; k < in->n_ranks; ++k) out->delta[k] = in->delta[k];
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
