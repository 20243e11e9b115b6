// Host side of the Muon branch: plan layout, TMA tensor maps, tile lists and
// the C-ABI entry points that launch the prep and Newton-Schulz kernels.
//
// The plan replaces the reference's per-step Python allocations
// (triton_muon.py:319-321, 358-359, 422) with buffers laid out once: for each
// matrix two bf16 iterates X (m x n), the Gram matrix A and the polynomial B
// (m x m), each row padded to a multiple of 64 elements so every TMA row
// stride is a multiple of 128 bytes.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <numeric>
#include <vector>

#include "capi_common.h"
#include "plan.cuh"
#include "ptx_sm100.cuh"

namespace mad {

int launch_muon_prep(MatDesc* mats, int32_t n_mats, const int32_t* prep_map, float* partials, int64_t n_tiles,
                     double beta, int nesterov, float eps, const GradReduce& red, cudaStream_t stream);
int launch_ns_gemm(int mode, const MatDesc* mats, const CUtensorMap* tmaps, const TileRef* tiles, int64_t n_tiles,
                   int iter, int last, float a, float b, float c, double lr, float lr_wd, unsigned int* status,
                   cudaStream_t stream);

namespace {

// Output tiles are computed by CTA pairs: 256 x 256 (each CTA 128 rows).
constexpr int GEMM_BM = 256, GEMM_BN = 256, GEMM_BK = 64;

inline int64_t round_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }
inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool aligned8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; }

// 4-element vector access (16 B float32, 8 B bf16) to every row of p, g, mom (and the shadow).
inline bool vec_ok(const mad_muon_matrix& mt) {
  bool al;
  if (mt.dtype == MAD_DTYPE_BF16)
    al = aligned8(mt.param) && aligned8(mt.grad) && aligned8(mt.momentum);
  else if (mt.dtype == MAD_DTYPE_F32_MASTER)
    al = aligned16(mt.param) && aligned8(mt.grad) && aligned16(mt.momentum) && aligned8(mt.shadow);
  else
    al = aligned16(mt.param) && aligned16(mt.grad) && aligned16(mt.momentum);
  return al && mt.cols % 4 == 0;
}

struct Shape {
  int64_t m, n, ld_x, ld_mm;
  bool transposed;
};

Shape wide_shape(const mad_muon_matrix& mt) {
  Shape s;
  s.transposed = mt.rows > mt.cols;
  s.m = std::min(mt.rows, mt.cols);
  s.n = std::max(mt.rows, mt.cols);
  s.ld_x = round_up(s.n, 64);
  s.ld_mm = round_up(s.m, 64);
  return s;
}

int64_t work_bytes_of(const Shape& s) {
  const int64_t x = round_up(s.m * s.ld_x * 2, 1024);
  const int64_t mm = round_up(s.m * s.ld_mm * 2, 1024);
  return 2 * x + 2 * mm;
}

int64_t gram_tiles_of(const Shape& s) {
  // 256 x 256 tiles (tm, tn) of the m x m output on or above the diagonal: tn >= tm.
  const int64_t t = (s.m + GEMM_BM - 1) / GEMM_BM;
  return t * (t + 1) / 2;
}

int64_t update_tiles_of(const Shape& s) {
  return ((s.m + GEMM_BM - 1) / GEMM_BM) * ((s.n + GEMM_BN - 1) / GEMM_BN);
}

int64_t prep_tiles_of(const mad_muon_matrix& mt) {
  return ((mt.rows + PREP_TILE - 1) / PREP_TILE) * ((mt.cols + PREP_TILE - 1) / PREP_TILE);
}

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

// bf16 matrix rows x cols (leading dimension ld elements), boxes of
// box_cols x box_rows; box_cols = 64 uses the 128-byte swizzle (operand
// loads), box_cols = 32 the 64-byte swizzle (epilogue stores).
int encode_bf16(CUtensorMap* out, void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows,
                int box_cols = 64) {
  auto fn = encode_fn();
  if (!fn) return fail(MAD_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  const CUtensorMapSwizzle sw = box_cols == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  const CUresult r = fn(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(MAD_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) for %lldx%lld ld %lld box %d", static_cast<int>(r),
                static_cast<long long>(rows), static_cast<long long>(cols), static_cast<long long>(ld), box_rows);
  return MAD_OK;
}

// A parameter (rows x cols, float32 or bf16) in 32x32 boxes for the last
// update's TMA loads and stores: 128-byte rows of float32 take the 128-byte
// swizzle, 64-byte rows of bf16 the 64-byte one.  Returns false (and leaves
// the map unused) when TMA cannot address the tensor: a base that is not
// 16-byte aligned or a row pitch that is not a multiple of 16 bytes.
bool encode_param(CUtensorMap* out, void* base, int64_t rows, int64_t cols, bool f32) {
  const int64_t pitch = cols * (f32 ? 4 : 2);
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || (pitch & 15) || rows > (int64_t(1) << 31) ||
      cols > (int64_t(1) << 31))
    return false;
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(pitch)};
  cuuint32_t box[2] = {32u, 32u};
  cuuint32_t estr[2] = {1u, 1u};
  return fn(out, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int validate(const mad_muon_matrix* mats, int32_t n) {
  if (n < 0 || (n > 0 && !mats)) return fail(MAD_ERR_INVALID, "muon plan: bad matrix list");
  for (int32_t i = 0; i < n; ++i) {
    const mad_muon_matrix& mt = mats[i];
    if (mt.rows <= 0 || mt.cols <= 0) return fail(MAD_ERR_INVALID, "muon plan: matrix %d has shape %lldx%lld", i,
                                                  static_cast<long long>(mt.rows), static_cast<long long>(mt.cols));
    if (!(mt.lr_scale >= 0.0)) return fail(MAD_ERR_INVALID, "muon plan: matrix %d has a negative lr_scale", i);
    if (mt.rows > (1 << 24) || mt.cols > (1 << 24) || mt.rows * mt.cols > (int64_t(1) << 34))
      return fail(MAD_ERR_INVALID, "muon plan: matrix %d is too large", i);
    if (!mt.param || !mt.grad || !mt.momentum) return fail(MAD_ERR_INVALID, "muon plan: matrix %d has a null pointer", i);
    if (mt.dtype != MAD_DTYPE_F32 && mt.dtype != MAD_DTYPE_BF16 && mt.dtype != MAD_DTYPE_F32_MASTER)
      return fail(MAD_ERR_INVALID, "muon plan: matrix %d has unknown dtype %d", i, mt.dtype);
    if (mt.dtype == MAD_DTYPE_F32_MASTER && !mt.shadow)
      return fail(MAD_ERR_INVALID, "muon plan: matrix %d (float32 master) has no bf16 shadow", i);
  }
  return MAD_OK;
}

inline uint8_t* at(void* base, int64_t off) { return static_cast<uint8_t*>(base) + off; }

}  // namespace
}  // namespace mad

using namespace mad;

extern "C" int mad_muon_plan_size(const mad_muon_matrix* mats, int32_t n_mats, mad_muon_plan_info* info) {
  clear_error();
  if (!info) return fail(MAD_ERR_INVALID, "mad_muon_plan_size: null info");
  if (int rc = validate(mats, n_mats)) return rc;
  mad_muon_plan_info pi;
  std::memset(&pi, 0, sizeof(pi));
  pi.n_mats = n_mats;
  pi.num_sms = num_sms();
  int64_t work = 0;
  for (int32_t i = 0; i < n_mats; ++i) {
    const Shape s = wide_shape(mats[i]);
    work += work_bytes_of(s);
    pi.prep_tiles += prep_tiles_of(mats[i]);
    pi.gram_tiles += gram_tiles_of(s);
    pi.update_tiles += update_tiles_of(s);
  }
  pi.poly_tiles = pi.gram_tiles;
  if (pi.prep_tiles > INT32_MAX || pi.update_tiles > INT32_MAX)
    return fail(MAD_ERR_INVALID, "mad_muon_plan_size: too many tiles");
  int64_t off = sizeof(PlanHeader);
  pi.off_mats = off;
  off = round_up(off + n_mats * static_cast<int64_t>(sizeof(MatDesc)), 128);
  pi.off_tmaps = off;
  off += static_cast<int64_t>(n_mats) * TMAPS_PER_MAT * static_cast<int64_t>(sizeof(CUtensorMap));
  pi.off_gram_tiles = off;
  off = round_up(off + pi.gram_tiles * static_cast<int64_t>(sizeof(TileRef)), 256);
  pi.off_poly_tiles = off;
  off = round_up(off + pi.poly_tiles * static_cast<int64_t>(sizeof(TileRef)), 256);
  pi.off_update_tiles = off;
  off = round_up(off + pi.update_tiles * static_cast<int64_t>(sizeof(TileRef)), 256);
  pi.off_prep_map = off;
  off = round_up(off + pi.prep_tiles * 4, 256);
  pi.off_partials = off;
  off = round_up(off + pi.prep_tiles * 4 * PREP_PARTIALS_PER_TILE, 256);
  pi.table_bytes = off;
  pi.work_bytes = work;
  *info = pi;
  return MAD_OK;
}

extern "C" int mad_muon_plan(const mad_muon_matrix* mats, int32_t n_mats, void* dev_table, void* dev_work,
                             const mad_muon_plan_info* info, mad_muon_buffers* buffers, void* stream) {
  clear_error();
  if (!info || !dev_table) return fail(MAD_ERR_INVALID, "mad_muon_plan: null info or table");
  mad_muon_plan_info chk;
  if (int rc = mad_muon_plan_size(mats, n_mats, &chk)) return rc;
  if (chk.table_bytes != info->table_bytes || chk.work_bytes != info->work_bytes || chk.n_mats != info->n_mats)
    return fail(MAD_ERR_INVALID, "mad_muon_plan: info does not describe these matrices");
  if (chk.work_bytes > 0 && !dev_work) return fail(MAD_ERR_INVALID, "mad_muon_plan: null work buffer");
  if ((reinterpret_cast<uintptr_t>(dev_table) & 127u) || (reinterpret_cast<uintptr_t>(dev_work) & 1023u))
    return fail(MAD_ERR_ALIGN, "mad_muon_plan: table must be 128-byte and work 1024-byte aligned");

  std::vector<uint8_t> host(static_cast<size_t>(chk.table_bytes), 0);
  PlanHeader* hdr = reinterpret_cast<PlanHeader*>(host.data());
  hdr->status = 0;
  hdr->n_mats = n_mats;
  MatDesc* md = reinterpret_cast<MatDesc*>(host.data() + chk.off_mats);
  CUtensorMap* tm = reinterpret_cast<CUtensorMap*>(host.data() + chk.off_tmaps);

  // Workspaces and descriptors.
  int64_t woff = 0, prep_begin = 0;
  std::vector<Shape> shapes(n_mats);
  for (int32_t i = 0; i < n_mats; ++i) {
    const mad_muon_matrix& mt = mats[i];
    const Shape s = shapes[i] = wide_shape(mt);
    const int64_t xb = round_up(s.m * s.ld_x * 2, 1024), mmb = round_up(s.m * s.ld_mm * 2, 1024);
    MatDesc& d = md[i];
    d.p = mt.param;
    d.g = mt.grad;
    d.mom = mt.momentum;
    d.x[0] = reinterpret_cast<__nv_bfloat16*>(at(dev_work, woff));
    d.x[1] = reinterpret_cast<__nv_bfloat16*>(at(dev_work, woff + xb));
    d.gram = reinterpret_cast<__nv_bfloat16*>(at(dev_work, woff + 2 * xb));
    d.poly = reinterpret_cast<__nv_bfloat16*>(at(dev_work, woff + 2 * xb + mmb));
    woff += 2 * xb + 2 * mmb;
    d.rows = static_cast<int32_t>(mt.rows);
    d.cols = static_cast<int32_t>(mt.cols);
    d.m = static_cast<int32_t>(s.m);
    d.n = static_cast<int32_t>(s.n);
    d.ld_x = static_cast<int32_t>(s.ld_x);
    d.ld_mm = static_cast<int32_t>(s.ld_mm);
    d.transposed = s.transposed ? 1 : 0;
    d.lr_scale = mt.lr_scale;
    d.inv_norm = 1.0f;
    d.prep_begin = static_cast<int32_t>(prep_begin);
    d.prep_tiles_c = static_cast<int32_t>((mt.cols + PREP_TILE - 1) / PREP_TILE);
    d.prep_count = static_cast<int32_t>(prep_tiles_of(mt));
    d.done = 0;
    d.tmap_base = i * TMAPS_PER_MAT;
    d.vec = vec_ok(mt) ? 1 : 0;
    d.dtype = mt.dtype;
    d.shadow = mt.dtype == MAD_DTYPE_F32_MASTER ? mt.shadow : nullptr;
    prep_begin += d.prep_count;
    CUtensorMap* t = tm + d.tmap_base;
    if (int rc = encode_bf16(t + TM_XK0, d.x[0], s.m, s.n, s.ld_x, 128)) return rc;
    if (int rc = encode_bf16(t + TM_XK1, d.x[1], s.m, s.n, s.ld_x, 128)) return rc;
    if (int rc = encode_bf16(t + TM_XMN0, d.x[0], s.m, s.n, s.ld_x, 64)) return rc;
    if (int rc = encode_bf16(t + TM_XMN1, d.x[1], s.m, s.n, s.ld_x, 64)) return rc;
    if (int rc = encode_bf16(t + TM_GRAM, d.gram, s.m, s.m, s.ld_mm, 128)) return rc;
    if (int rc = encode_bf16(t + TM_POLY, d.poly, s.m, s.m, s.ld_mm, 128)) return rc;
    if (int rc = encode_bf16(t + TM_GRAM_ST, d.gram, s.m, s.m, s.ld_mm, 32, 32)) return rc;
    if (int rc = encode_bf16(t + TM_POLY_ST, d.poly, s.m, s.m, s.ld_mm, 32, 32)) return rc;
    if (int rc = encode_bf16(t + TM_X0_ST, d.x[0], s.m, s.n, s.ld_x, 32, 32)) return rc;
    if (int rc = encode_bf16(t + TM_X1_ST, d.x[1], s.m, s.n, s.ld_x, 32, 32)) return rc;
    // The parameter as stored (rows x cols), for the last update's writes.
    d.p_tma = encode_param(t + TM_P, mt.param, mt.rows, mt.cols, mt.dtype != MAD_DTYPE_BF16) ? 1 : 0;
    if (d.p_tma && mt.dtype == MAD_DTYPE_F32_MASTER)
      d.p_tma = encode_param(t + TM_SH, mt.shadow, mt.rows, mt.cols, false) ? 1 : 0;
    if (buffers) {
      mad_muon_buffers& b = buffers[i];
      b.x[0] = d.x[0];
      b.x[1] = d.x[1];
      b.gram = d.gram;
      b.poly = d.poly;
      b.m = s.m;
      b.n = s.n;
      b.ld_x = s.ld_x;
      b.ld_mm = s.ld_mm;
      b.transposed = d.transposed;
    }
  }

  // Tile lists: longest K first so the long tiles start early; within a
  // matrix, column-block-major so CTAs running together share operand panels.
  std::vector<int32_t> order(n_mats);
  std::iota(order.begin(), order.end(), 0);
  auto emit = [&](TileRef* out, bool gram_k, bool triangle) {
    std::vector<int32_t> ord = order;
    std::stable_sort(ord.begin(), ord.end(), [&](int32_t a, int32_t b) {
      const int64_t ka = gram_k ? shapes[a].n : shapes[a].m, kb = gram_k ? shapes[b].n : shapes[b].m;
      return ka > kb;
    });
    int64_t k = 0;
    for (int32_t i : ord) {
      const Shape& s = shapes[i];
      const int64_t tms = (s.m + GEMM_BM - 1) / GEMM_BM;
      const int64_t tns = ((triangle ? s.m : s.n) + GEMM_BN - 1) / GEMM_BN;
      for (int64_t tn = 0; tn < tns; ++tn) {
        const int64_t tm_end = triangle ? std::min<int64_t>(tms, tn + 1) : tms;
        for (int64_t tmi = 0; tmi < tm_end; ++tmi) {
          out[k].mat = i;
          out[k].tm = static_cast<int32_t>(tmi);
          out[k].tn = static_cast<int32_t>(tn);
          out[k].nkb = static_cast<int32_t>(((gram_k ? s.n : s.m) + GEMM_BK - 1) / GEMM_BK);
          ++k;
        }
      }
    }
    return k;
  };
  const int64_t ng = emit(reinterpret_cast<TileRef*>(host.data() + chk.off_gram_tiles), true, true);
  const int64_t np = emit(reinterpret_cast<TileRef*>(host.data() + chk.off_poly_tiles), false, true);
  const int64_t nu = emit(reinterpret_cast<TileRef*>(host.data() + chk.off_update_tiles), false, false);
  if (ng != chk.gram_tiles || np != chk.poly_tiles || nu != chk.update_tiles)
    return fail(MAD_ERR_INVALID, "mad_muon_plan: internal tile count mismatch");
  int32_t* pmap = reinterpret_cast<int32_t*>(host.data() + chk.off_prep_map);
  for (int32_t i = 0; i < n_mats; ++i)
    for (int32_t k = 0; k < md[i].prep_count; ++k) pmap[md[i].prep_begin + k] = i;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(dev_table, host.data(), host.size(), cudaMemcpyHostToDevice, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return fail_cuda("mad_muon_plan: table upload");
  return MAD_OK;
}

namespace {

struct Views {
  MatDesc* mats;
  const CUtensorMap* tmaps;
  const TileRef* gram;
  const TileRef* poly;
  const TileRef* update;
  const int32_t* prep_map;
  float* partials;
  unsigned int* status;
};

Views views(const mad_muon_plan_info* info, void* table) {
  Views v;
  v.mats = reinterpret_cast<MatDesc*>(at(table, info->off_mats));
  v.tmaps = reinterpret_cast<const CUtensorMap*>(at(table, info->off_tmaps));
  v.gram = reinterpret_cast<const TileRef*>(at(table, info->off_gram_tiles));
  v.poly = reinterpret_cast<const TileRef*>(at(table, info->off_poly_tiles));
  v.update = reinterpret_cast<const TileRef*>(at(table, info->off_update_tiles));
  v.prep_map = reinterpret_cast<const int32_t*>(at(table, info->off_prep_map));
  v.partials = reinterpret_cast<float*>(at(table, info->off_partials));
  v.status = reinterpret_cast<unsigned int*>(table);
  return v;
}

int check_args(const mad_muon_plan_info* info, void* table, const char* who) {
  if (!info) return fail(MAD_ERR_INVALID, "%s: null plan info", who);
  if (info->n_mats > 0 && !table) return fail(MAD_ERR_INVALID, "%s: null table", who);
  return MAD_OK;
}

}  // namespace

static int muon_prep(const mad_muon_plan_info* info, void* dev_table, double beta, int32_t nesterov, float eps,
                     const mad_grad_reduce* reduce, void* stream, const char* who) {
  clear_error();
  if (int rc = check_args(info, dev_table, who)) return rc;
  GradReduce red;
  if (int rc = grad_reduce_from(reduce, &red, who)) return rc;
  if (info->n_mats == 0) return MAD_OK;
  const Views v = views(info, dev_table);
  return launch_muon_prep(v.mats, info->n_mats, v.prep_map, v.partials, info->prep_tiles, beta, nesterov, eps, red,
                          static_cast<cudaStream_t>(stream));
}

extern "C" int mad_muon_prep(const mad_muon_plan_info* info, void* dev_table, double beta, int32_t nesterov,
                             float eps, void* stream) {
  return muon_prep(info, dev_table, beta, nesterov, eps, nullptr, stream, "mad_muon_prep");
}

extern "C" int mad_muon_prep_reduce(const mad_muon_plan_info* info, void* dev_table, double beta, int32_t nesterov,
                                    float eps, const mad_grad_reduce* reduce, void* stream) {
  if (!reduce) {
    clear_error();
    return fail(MAD_ERR_INVALID, "mad_muon_prep_reduce: null reduce descriptor");
  }
  return muon_prep(info, dev_table, beta, nesterov, eps, reduce, stream, "mad_muon_prep_reduce");
}

extern "C" int mad_ns_gram(const mad_muon_plan_info* info, void* dev_table, int32_t iter, void* stream) {
  clear_error();
  if (int rc = check_args(info, dev_table, "mad_ns_gram")) return rc;
  if (iter < 0) return fail(MAD_ERR_INVALID, "mad_ns_gram: negative iteration");
  if (info->n_mats == 0) return MAD_OK;
  const Views v = views(info, dev_table);
  return launch_ns_gemm(0, v.mats, v.tmaps, v.gram, info->gram_tiles, iter, 0, 0.f, 0.f, 0.f, 0.0, 0.f, v.status,
                        static_cast<cudaStream_t>(stream));
}

extern "C" int mad_ns_poly(const mad_muon_plan_info* info, void* dev_table, int32_t iter, float b, float c,
                           void* stream) {
  clear_error();
  if (int rc = check_args(info, dev_table, "mad_ns_poly")) return rc;
  if (iter < 0) return fail(MAD_ERR_INVALID, "mad_ns_poly: negative iteration");
  if (info->n_mats == 0) return MAD_OK;
  const Views v = views(info, dev_table);
  return launch_ns_gemm(1, v.mats, v.tmaps, v.poly, info->poly_tiles, iter, 0, 0.f, b, c, 0.0, 0.f, v.status,
                        static_cast<cudaStream_t>(stream));
}

extern "C" int mad_ns_update(const mad_muon_plan_info* info, void* dev_table, int32_t iter, int32_t last, float a,
                             double lr, double weight_decay, void* stream) {
  clear_error();
  if (int rc = check_args(info, dev_table, "mad_ns_update")) return rc;
  if (iter < 0) return fail(MAD_ERR_INVALID, "mad_ns_update: negative iteration");
  if (info->n_mats == 0) return MAD_OK;
  const Views v = views(info, dev_table);
  // lr*weight_decay is formed in double and rounded once, as the reference's
  // host-side product is (triton_muon.py:370).
  const float lr_wd = static_cast<float>(lr * weight_decay);
  return launch_ns_gemm(2, v.mats, v.tmaps, v.update, info->update_tiles, iter, last ? 1 : 0, a, 0.f, 0.f, lr, lr_wd,
                        v.status, static_cast<cudaStream_t>(stream));
}

static int muon_step_multi(const mad_muon_plan_info* info, void* dev_table, double beta, int32_t nesterov, float a,
                           float b, float c, int32_t ns_steps, float eps, double lr, double weight_decay,
                           const mad_grad_reduce* reduce, void* stream, const char* who) {
  clear_error();
  if (int rc = check_args(info, dev_table, who)) return rc;
  if (ns_steps < 1) return fail(MAD_ERR_INVALID, "%s: ns_steps must be >= 1", who);
  if (info->n_mats == 0) return MAD_OK;
  if (int rc = muon_prep(info, dev_table, beta, nesterov, eps, reduce, stream, who)) return rc;
  for (int32_t it = 0; it < ns_steps; ++it) {
    if (int rc = mad_ns_gram(info, dev_table, it, stream)) return rc;
    if (int rc = mad_ns_poly(info, dev_table, it, b, c, stream)) return rc;
    if (int rc = mad_ns_update(info, dev_table, it, it == ns_steps - 1, a, lr, weight_decay, stream)) return rc;
  }
  return MAD_OK;
}

extern "C" int mad_muon_step_multi(const mad_muon_plan_info* info, void* dev_table, double beta, int32_t nesterov,
                                   float a, float b, float c, int32_t ns_steps, float eps, double lr,
                                   double weight_decay, void* stream) {
  return muon_step_multi(info, dev_table, beta, nesterov, a, b, c, ns_steps, eps, lr, weight_decay, nullptr, stream,
                         "mad_muon_step_multi");
}

extern "C" int mad_muon_step_multi_reduce(const mad_muon_plan_info* info, void* dev_table, double beta,
                                          int32_t nesterov, float a, float b, float c, int32_t ns_steps, float eps,
                                          double lr, double weight_decay, const mad_grad_reduce* reduce,
                                          void* stream) {
  if (!reduce) {
    clear_error();
    return fail(MAD_ERR_INVALID, "mad_muon_step_multi_reduce: null reduce descriptor");
  }
  return muon_step_multi(info, dev_table, beta, nesterov, a, b, c, ns_steps, eps, lr, weight_decay, reduce, stream,
                         "mad_muon_step_multi_reduce");
}

extern "C" int mad_muon_read_status(const mad_muon_plan_info* info, void* dev_table, uint32_t* status, int32_t clear,
                                    void* stream) {
  clear_error();
  if (int rc = check_args(info, dev_table, "mad_muon_read_status")) return rc;
  if (!status) return fail(MAD_ERR_INVALID, "mad_muon_read_status: null status");
  *status = 0;
  if (info->n_mats == 0) return MAD_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(status, dev_table, sizeof(uint32_t), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return fail_cuda("mad_muon_read_status");
  if (clear && *status) {
    if (cudaMemsetAsync(dev_table, 0, sizeof(uint32_t), s) != cudaSuccess) return fail_cuda("mad_muon_read_status");
  }
  return MAD_OK;
}
