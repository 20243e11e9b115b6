// Peer buffers: device memory the other processes of this node map with CUDA
// IPC, so a kernel on one GPU can read another rank's gradients over NVLink
// with plain loads (no multicast, no TMA from peer memory), and the copy
// engines can write updated parameters straight into the other ranks'
// replicas.  mad_ipc_alloc is the only entry point of the library that
// allocates.
#include <cuda_runtime.h>

#include <cstring>

#include "capi_common.h"

using namespace mad;

namespace {
int cuda_fail(cudaError_t e, const char* what) {
  cudaGetLastError();  // clear the non-sticky error state
  return fail(MAD_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}
}  // namespace

extern "C" int mad_ipc_alloc(int64_t bytes, void** dev_ptr, void* handle) {
  clear_error();
  static_assert(sizeof(cudaIpcMemHandle_t) == MAD_IPC_HANDLE_BYTES, "IPC handle size");
  if (bytes <= 0 || !dev_ptr || !handle) return fail(MAD_ERR_INVALID, "mad_ipc_alloc: bad arguments");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, static_cast<size_t>(bytes));
  if (e != cudaSuccess) return cuda_fail(e, "mad_ipc_alloc: cudaMalloc");
  cudaIpcMemHandle_t h;
  if ((e = cudaMemset(p, 0, static_cast<size_t>(bytes))) != cudaSuccess ||
      (e = cudaDeviceSynchronize()) != cudaSuccess || (e = cudaIpcGetMemHandle(&h, p)) != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "mad_ipc_alloc");
  }
  std::memcpy(handle, &h, sizeof(h));
  *dev_ptr = p;
  return MAD_OK;
}

extern "C" int mad_ipc_free(void* dev_ptr) {
  clear_error();
  if (!dev_ptr) return MAD_OK;
  const cudaError_t e = cudaFree(dev_ptr);
  return e == cudaSuccess ? MAD_OK : cuda_fail(e, "mad_ipc_free");
}

extern "C" int mad_ipc_open(const void* handle, void** peer_ptr) {
  clear_error();
  if (!handle || !peer_ptr) return fail(MAD_ERR_INVALID, "mad_ipc_open: bad arguments");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "mad_ipc_open");
  *peer_ptr = p;
  return MAD_OK;
}

extern "C" int mad_ipc_close(void* peer_ptr) {
  clear_error();
  if (!peer_ptr) return MAD_OK;
  const cudaError_t e = cudaIpcCloseMemHandle(peer_ptr);
  return e == cudaSuccess ? MAD_OK : cuda_fail(e, "mad_ipc_close");
}

extern "C" int mad_copy_async(void* dst, const void* src, int64_t bytes, void* stream) {
  clear_error();
  if (bytes < 0 || (bytes > 0 && (!dst || !src))) return fail(MAD_ERR_INVALID, "mad_copy_async: bad arguments");
  if (bytes == 0) return MAD_OK;
  const cudaError_t e =
      cudaMemcpyAsync(dst, src, static_cast<size_t>(bytes), cudaMemcpyDefault, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MAD_OK : cuda_fail(e, "mad_copy_async");
}
