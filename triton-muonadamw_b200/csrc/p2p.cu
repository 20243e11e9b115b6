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

namespace {

constexpr int PUSH_THREADS = 128;
constexpr int PUSH_UNROLL = 4;

struct PeerSet {
  int32_t n;
  int64_t delta[MAX_RANKS];
};

// Each thread loads PUSH_UNROLL 16-byte vectors of the source once and stores
// them to every peer's copy (rank-rotated start per CTA, so the ranks' CTAs
// spread over the switch).  128 threads, <= 64 registers, no shared memory:
// one CTA fits on an SM beside the persistent Newton-Schulz GEMM CTA (which
// leaves 11,776 registers and 1 KB of shared memory free), so the broadcast
// overlaps the GEMMs instead of waiting for them.
__global__ void __launch_bounds__(PUSH_THREADS, 1) peer_push_kernel(const uint4* __restrict__ src, int64_t n_vec,
                                                                    PeerSet ps) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * PUSH_THREADS;
  for (int64_t base = static_cast<int64_t>(blockIdx.x) * PUSH_THREADS + threadIdx.x; base < n_vec;
       base += stride * PUSH_UNROLL) {
    uint4 v[PUSH_UNROLL];
#pragma unroll
    for (int u = 0; u < PUSH_UNROLL; ++u) {
      const int64_t i = base + u * stride;
      if (i < n_vec) v[u] = __ldcs(src + i);
    }
    for (int j = 0; j < ps.n; ++j) {
      const int k = (j + blockIdx.x) % ps.n;
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<char*>(const_cast<uint4*>(src)) + ps.delta[k]);
#pragma unroll
      for (int u = 0; u < PUSH_UNROLL; ++u) {
        const int64_t i = base + u * stride;
        if (i < n_vec) dst[i] = v[u];
      }
    }
  }
  __threadfence_system();
}

}  // namespace

extern "C" int mad_peer_push(const void* src, int64_t bytes, const mad_peer_set* peers, void* stream) {
  clear_error();
  if (bytes < 0 || !peers || (bytes > 0 && !src)) return fail(MAD_ERR_INVALID, "mad_peer_push: bad arguments");
  if (peers->n_peers < 0 || peers->n_peers > MAX_RANKS)
    return fail(MAD_ERR_INVALID, "mad_peer_push: n_peers %d outside 0..%d", peers->n_peers, MAX_RANKS);
  if ((reinterpret_cast<uintptr_t>(src) & 15u) != 0 || (bytes & 15) != 0)
    return fail(MAD_ERR_ALIGN, "mad_peer_push: source and size must be multiples of 16 bytes");
  for (int k = 0; k < peers->n_peers; ++k)
    if ((peers->delta[k] & 15) != 0) return fail(MAD_ERR_ALIGN, "mad_peer_push: peer %d is not 16-byte aligned", k);
  if (bytes == 0 || peers->n_peers == 0) return MAD_OK;
  PeerSet ps;
  std::memset(&ps, 0, sizeof(ps));
  ps.n = peers->n_peers;
  for (int k = 0; k < ps.n; ++k) ps.delta[k] = peers->delta[k];
  const int64_t n_vec = bytes / 16;
  const int64_t want = (n_vec + PUSH_THREADS * PUSH_UNROLL - 1) / (PUSH_THREADS * PUSH_UNROLL);
  const int grid = static_cast<int>(want < num_sms() ? want : num_sms());
  peer_push_kernel<<<grid, PUSH_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const uint4*>(src),
                                                                                n_vec, ps);
  return check_launch("peer_push_kernel");
}
