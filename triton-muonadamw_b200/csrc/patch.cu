// Gradient pointers of an existing plan, rewritten in place.
//
// The AdamW table and the Muon plan hold each tensor's gradient address
// (AdamEntry::g, MatDesc::g) and nothing derived from it: no tensor map, tile
// or workspace depends on the gradient.  When a training loop drops its
// gradients (``zero_grad(set_to_none=True)``) and the next backward pass
// allocates new ones, only those addresses change, so instead of re-planning
// (tensor-map encodes, a table upload and a stream synchronisation) the new
// addresses are written by a small kernel that receives them as launch
// arguments: stream-ordered after the previous step's kernels, no host
// buffer to keep alive and no synchronisation.
//
// The planned vector width depends on the alignment of every pointer of an
// entry; a new gradient address must therefore be 16-byte aligned (then every
// vector access the entry was planned with stays legal).  Anything else is
// refused with MAD_ERR_ALIGN and the caller re-plans.
#include <cuda_runtime.h>

#include <cstddef>

#include "capi_common.h"
#include "plan.cuh"

namespace mad {
namespace {

constexpr int PATCH_CHUNK = 256;  // pointers per launch: 2 KB of kernel arguments

struct PtrChunk {
  const void* p[PATCH_CHUNK];
};

static_assert(offsetof(AdamEntry, g) == 8, "AdamEntry::g offset");
static_assert(offsetof(MatDesc, g) == 8, "MatDesc::g offset");

__global__ void patch_grad_pointers_kernel(uint8_t* base, int64_t stride, int32_t first, int32_t count,
                                           const __grid_constant__ PtrChunk chunk) {
  const int i = threadIdx.x;
  if (i < count) *reinterpret_cast<const void**>(base + (first + i) * stride + 8) = chunk.p[i];
}

int patch(uint8_t* base, int64_t stride, const void* const* grads, int32_t n, cudaStream_t stream, const char* who) {
  for (int32_t i = 0; i < n; ++i) {
    if (!grads[i]) return fail(MAD_ERR_INVALID, "%s: gradient %d is null", who, i);
    if (reinterpret_cast<uintptr_t>(grads[i]) & 15u)
      return fail(MAD_ERR_ALIGN, "%s: gradient %d is not 16-byte aligned (re-plan instead)", who, i);
  }
  for (int32_t first = 0; first < n; first += PATCH_CHUNK) {
    const int32_t count = n - first < PATCH_CHUNK ? n - first : PATCH_CHUNK;
    PtrChunk c;
    for (int32_t k = 0; k < PATCH_CHUNK; ++k) c.p[k] = k < count ? grads[first + k] : nullptr;
    patch_grad_pointers_kernel<<<1, PATCH_CHUNK, 0, stream>>>(base, stride, first, count, c);
    if (int rc = check_launch("patch_grad_pointers_kernel")) return rc;
  }
  return MAD_OK;
}

}  // namespace
}  // namespace mad

using namespace mad;

extern "C" int mad_adamw_set_grads(void* dev_table, int64_t n_tiles, const void* const* grads, int32_t n_tensors,
                                   void* stream) {
  clear_error();
  if (n_tensors < 0 || n_tiles < 0 || (n_tensors > 0 && (!grads || !dev_table)))
    return fail(MAD_ERR_INVALID, "mad_adamw_set_grads: bad arguments");
  if (n_tensors == 0) return MAD_OK;
  // The entries follow the int32 tile map, 256-byte aligned (adamw.cu's table layout).
  const int64_t off = (n_tiles * 4 + 255) / 256 * 256;
  return patch(static_cast<uint8_t*>(dev_table) + off, sizeof(AdamEntry), grads, n_tensors,
               static_cast<cudaStream_t>(stream), "mad_adamw_set_grads");
}

extern "C" int mad_muon_set_grads(const mad_muon_plan_info* info, void* dev_table, const void* const* grads,
                                  void* stream) {
  clear_error();
  if (!info || (info->n_mats > 0 && (!grads || !dev_table)))
    return fail(MAD_ERR_INVALID, "mad_muon_set_grads: bad arguments");
  if (info->n_mats == 0) return MAD_OK;
  return patch(static_cast<uint8_t*>(dev_table) + info->off_mats, sizeof(MatDesc), grads, info->n_mats,
               static_cast<cudaStream_t>(stream), "mad_muon_set_grads");
}
