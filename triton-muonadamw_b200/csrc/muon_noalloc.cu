// mad_muon_step_noalloc: the Muon step of one matrix without any allocation.
//
// Some callers cannot allocate device memory at the point where they step the
// optimizer: code running under a custom or pre-sized allocator, code that must
// not grow its memory footprint after start-up, or a foreign-language host that
// has no allocator binding for this library.  This entry point needs nothing
// from them but the parameter, gradient and momentum: the plan table and the
// bf16 Newton-Schulz workspaces live in one file-scope device array below,
// NOALLOC_SCRATCH_BYTES large, which every GPU that loads the library holds
// until the process exits.  The plan is staged in a file-scope host buffer, so
// no host allocation happens either.
//
// Limits: rows * cols <= NOALLOC_MAX_ELEMS and min(rows, cols) <= NOALLOC_MAX_MIN_DIM;
// larger matrices are rejected with MAD_ERR_INVALID.
//
// The array is shared by every call and keeps the last call's contents; each
// call rewrites the whole plan (counters and status start at zero).  Calls
// that overlap on the GPU (different streams, or different host threads
// without ordering) race on it.  The first call on a device resolves the
// array's device address for that device (cudaGetSymbolAddress).  Each call
// uploads its plan with a synchronous copy, which also waits for the stream's
// earlier work, and after its kernels reads their status word back (waiting
// for them to finish): a kernel that gave up waiting on a barrier makes the
// call return MAD_ERR_DEVICE.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "capi_common.h"
#include "plan.cuh"

namespace mad {
namespace {

constexpr int64_t NOALLOC_MAX_ELEMS = int64_t(1) << 20;
constexpr int64_t NOALLOC_MAX_MIN_DIM = 1024;
constexpr size_t NOALLOC_TABLE_BYTES = 256 << 10;          // plan table (tile lists, tensor maps, ...)
constexpr size_t NOALLOC_WORK_BYTES = 9 << 20;             // X ping-pong, A, B for the largest allowed matrix
constexpr size_t NOALLOC_SCRATCH_BYTES = NOALLOC_TABLE_BYTES + NOALLOC_WORK_BYTES + 1024;  // + 1 KB to align work

static __device__ __align__(256) uint8_t g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mutex;                       // one call at a time per process: the host staging buffer is shared
void* g_scratch_dev[kMaxDevices] = {nullptr};
alignas(128) uint8_t g_host_image[NOALLOC_TABLE_BYTES];

inline int64_t round_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// Same tensor-map formats the planner uses: 64-column boxes with the 128-byte
// swizzle for operand loads, 32x32 boxes with the 64-byte swizzle for stores.
bool encode(CUtensorMap* out, void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows, int box_cols) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  return fn(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            box_cols == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Device address of the scratch array on the current device, resolved once per device.
int scratch_for_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail_cuda("mad_muon_step_noalloc: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) return fail(MAD_ERR_INVALID, "mad_muon_step_noalloc: device %d out of range", dev);
  if (!g_scratch_dev[dev]) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr)
      return fail_cuda("mad_muon_step_noalloc: cudaGetSymbolAddress of the static scratch");
    g_scratch_dev[dev] = ptr;
  }
  *out = g_scratch_dev[dev];
  return MAD_OK;
}

}  // namespace
}  // namespace mad

using namespace mad;

extern "C" int mad_muon_step_noalloc(float* param, const float* grad, float* momentum, int64_t rows, int64_t cols,
                                     double lr_scale, double beta, int32_t nesterov, float a, float b, float c,
                                     int32_t ns_steps, float eps, double lr, double weight_decay, void* stream) {
  clear_error();
  if (!param || !grad || !momentum) return fail(MAD_ERR_INVALID, "mad_muon_step_noalloc: null pointer");
  if (rows <= 0 || cols <= 0) return fail(MAD_ERR_INVALID, "mad_muon_step_noalloc: bad shape");
  const int64_t m = rows < cols ? rows : cols, n = rows < cols ? cols : rows;
  if (rows * cols > NOALLOC_MAX_ELEMS || m > NOALLOC_MAX_MIN_DIM)
    return fail(MAD_ERR_INVALID,
                "mad_muon_step_noalloc: a %lldx%lld matrix exceeds the static scratch (at most %lld elements and "
                "min(rows, cols) <= %lld); use mad_muon_plan with caller-provided buffers",
                static_cast<long long>(rows), static_cast<long long>(cols),
                static_cast<long long>(NOALLOC_MAX_ELEMS), static_cast<long long>(NOALLOC_MAX_MIN_DIM));
  if (ns_steps < 1) return fail(MAD_ERR_INVALID, "mad_muon_step_noalloc: ns_steps must be >= 1");

  mad_muon_matrix mat;
  mat.param = param;
  mat.grad = grad;
  mat.momentum = momentum;
  mat.rows = rows;
  mat.cols = cols;
  mat.lr_scale = lr_scale;
  mat.dtype = MAD_DTYPE_F32;
  mat.pad = 0;
  mat.shadow = nullptr;
  mad_muon_plan_info info;
  if (int rc = mad_muon_plan_size(&mat, 1, &info)) return rc;
  if (info.table_bytes > static_cast<int64_t>(NOALLOC_TABLE_BYTES) ||
      info.work_bytes > static_cast<int64_t>(NOALLOC_WORK_BYTES))
    return fail(MAD_ERR_INVALID, "mad_muon_step_noalloc: plan needs %lld + %lld bytes, scratch holds %zu + %zu",
                static_cast<long long>(info.table_bytes), static_cast<long long>(info.work_bytes),
                NOALLOC_TABLE_BYTES, NOALLOC_WORK_BYTES);

  std::lock_guard<std::mutex> lock(g_mutex);
  void* scratch = nullptr;
  if (int rc = scratch_for_current_device(&scratch)) return rc;
  uint8_t* table = static_cast<uint8_t*>(scratch);
  uint8_t* work = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(table + NOALLOC_TABLE_BYTES) + 1023) & ~static_cast<uintptr_t>(1023));

  // Plan image for one matrix, in the layout mad_muon_plan_size reported.
  std::memset(g_host_image, 0, static_cast<size_t>(info.table_bytes));
  PlanHeader* hdr = reinterpret_cast<PlanHeader*>(g_host_image);
  hdr->n_mats = 1;
  MatDesc& d = *reinterpret_cast<MatDesc*>(g_host_image + info.off_mats);
  const int64_t ld_x = round_up(n, 64), ld_mm = round_up(m, 64);
  const int64_t xb = round_up(m * ld_x * 2, 1024), mmb = round_up(m * ld_mm * 2, 1024);
  d.p = param;
  d.g = grad;
  d.mom = momentum;
  d.x[0] = reinterpret_cast<__nv_bfloat16*>(work);
  d.x[1] = reinterpret_cast<__nv_bfloat16*>(work + xb);
  d.gram = reinterpret_cast<__nv_bfloat16*>(work + 2 * xb);
  d.poly = reinterpret_cast<__nv_bfloat16*>(work + 2 * xb + mmb);
  d.lr_scale = lr_scale;
  d.rows = static_cast<int32_t>(rows);
  d.cols = static_cast<int32_t>(cols);
  d.m = static_cast<int32_t>(m);
  d.n = static_cast<int32_t>(n);
  d.ld_x = static_cast<int32_t>(ld_x);
  d.ld_mm = static_cast<int32_t>(ld_mm);
  d.transposed = rows > cols ? 1 : 0;
  d.inv_norm = 1.0f;
  d.prep_begin = 0;
  d.prep_tiles_c = static_cast<int32_t>((cols + PREP_TILE - 1) / PREP_TILE);
  d.prep_count = static_cast<int32_t>(info.prep_tiles);
  d.done = 0;
  d.tmap_base = 0;
  d.vec = ((reinterpret_cast<uintptr_t>(param) | reinterpret_cast<uintptr_t>(grad) |
            reinterpret_cast<uintptr_t>(momentum)) & 15u) == 0 && cols % 4 == 0;
  CUtensorMap* t = reinterpret_cast<CUtensorMap*>(g_host_image + info.off_tmaps);
  const bool ok = encode(t + TM_XK0, d.x[0], m, n, ld_x, 128, 64) && encode(t + TM_XK1, d.x[1], m, n, ld_x, 128, 64) &&
                  encode(t + TM_XMN0, d.x[0], m, n, ld_x, 64, 64) && encode(t + TM_XMN1, d.x[1], m, n, ld_x, 64, 64) &&
                  encode(t + TM_GRAM, d.gram, m, m, ld_mm, 128, 64) && encode(t + TM_POLY, d.poly, m, m, ld_mm, 128, 64) &&
                  encode(t + TM_GRAM_ST, d.gram, m, m, ld_mm, 32, 32) &&
                  encode(t + TM_POLY_ST, d.poly, m, m, ld_mm, 32, 32) &&
                  encode(t + TM_X0_ST, d.x[0], m, n, ld_x, 32, 32) && encode(t + TM_X1_ST, d.x[1], m, n, ld_x, 32, 32);
  if (!ok) return fail(MAD_ERR_CUDA, "mad_muon_step_noalloc: cuTensorMapEncodeTiled failed");
  // Tile lists in the planner's order: 256x256 tiles, column-block-major; Gram and
  // polynomial only on or above the diagonal.
  const int64_t tms = (m + 255) / 256, tns_x = (n + 255) / 256;
  auto emit = [&](int64_t off, bool triangle, int64_t k_extent) {
    TileRef* out = reinterpret_cast<TileRef*>(g_host_image + off);
    int64_t k = 0;
    for (int64_t tn = 0; tn < (triangle ? tms : tns_x); ++tn)
      for (int64_t tm = 0; tm < (triangle ? (tn + 1 < tms ? tn + 1 : tms) : tms); ++tm) {
        out[k].mat = 0;
        out[k].tm = static_cast<int32_t>(tm);
        out[k].tn = static_cast<int32_t>(tn);
        out[k].nkb = static_cast<int32_t>((k_extent + 63) / 64);
        ++k;
      }
    return k;
  };
  if (emit(info.off_gram_tiles, true, n) != info.gram_tiles || emit(info.off_poly_tiles, true, m) != info.poly_tiles ||
      emit(info.off_update_tiles, false, m) != info.update_tiles)
    return fail(MAD_ERR_INVALID, "mad_muon_step_noalloc: internal tile count mismatch");
  // prep tile -> matrix map is all zeros (one matrix); partial sums are written before they are read.

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(table, g_host_image, static_cast<size_t>(info.table_bytes), cudaMemcpyHostToDevice, s) !=
          cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return fail_cuda("mad_muon_step_noalloc: plan upload");
  if (int rc = mad_muon_step_multi(&info, table, beta, nesterov, a, b, c, ns_steps, eps, lr, weight_decay, stream))
    return rc;
  // The caller holds no plan to read the kernels' status word from, and the
  // next call rewrites it: read it here, after this call's kernels finish.
  uint32_t status = 0;
  if (int rc = mad_muon_read_status(&info, table, &status, 1, stream)) return rc;
  if (status != 0)
    return fail(MAD_ERR_DEVICE,
                "mad_muon_step_noalloc: a Newton-Schulz kernel gave up waiting on a barrier (status 0x%x); the "
                "parameter and momentum written by this call are invalid",
                status);
  return MAD_OK;
}
