// AdamW branch: one elementwise fp32 update of param, exp_avg, exp_avg_sq.
// Parameters and gradients may be float32 or bf16 (moments always float32);
// bf16 values are widened on load and rounded once, to nearest even, on store.
// A float32 master parameter with a bf16 gradient also stores its bf16 copy.
//
// Follows the reference kernel's formula (triton_adam.py:53-63):
//   m = b1 m + (1-b1) g ; v = b2 v + (1-b2) g²
//   p = (1 - lr wd) p - lr (m/bias1) / (sqrt(v/bias2) + eps)
// with every product and sum rounded separately (no FMA contraction) so it
// agrees with the float32 CPU oracle to the last few ulps.
//
// Layout: a multi-tensor launch covers a table of tensors cut into 512-element
// tiles, one tile per 128-thread CTA; a tile -> tensor index map (int32 per
// tile) sits in front of the AdamEntry array, so each CTA finds its tensor
// with one load.  Each thread moves one float4 of each of p, g, m, v.  The
// grid is the tile count: the hardware keeps up to sixteen such CTAs per SM
// resident, and that occupancy -- not a deep per-thread pipeline -- is what
// keeps the 28 bytes per element streaming at the power-capped SM clock of
// the optimizer step.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "capi_common.h"
#include "elem_io.cuh"
#include "plan.cuh"

namespace mad {

struct AdamScalars {
  float lr, beta1, beta2, one_m_beta1, one_m_beta2, eps, decay, bias1, bias2;
  float rbias1, rbias2;  // RN(1/bias1), RN(1/bias2): correctly rounded reciprocals, formed on the host
  GradReduce red;  // red.n > 0: the gradient is the mean of every rank's copy (peer memory)
};

// a / b for a divisor b fixed for the whole launch, with rb = RN(1/b):
// Markstein's correction step (Markstein 1990; Muller et al., Handbook of
// Floating-Point Arithmetic, on FMA-based division) -- q = RN(a rb), the exact
// residual r = a - q b by FMA, RN(q + r rb) -- is the correctly rounded
// quotient whenever neither it nor the residual leaves the normal range, which
// the operand window below guarantees for divisors 1 >= b >= 2^-40 (rb == 0
// marks a divisor outside that range).  Other operands (zero, subnormal, huge,
// inf, NaN) take the IEEE division.  Three instructions instead of a full
// division on the AdamW path, which at the power-capped SM clock of the
// optimizer step is close to issue-bound.
__device__ __forceinline__ float div_uniform(float a, float b, float rb) {
  const float aa = fabsf(a);
  if (__builtin_expect(rb != 0.f && aa >= 0x1p-80f && aa <= 0x1p80f, 1)) {
    const float q = __fmul_rn(a, rb);
    const float r = __fmaf_rn(-q, b, a);
    return __fmaf_rn(r, rb, q);
  }
  return __fdiv_rn(a, b);
}

__device__ __forceinline__ void adam_elem(float& p, float g, float& m, float& v, const AdamScalars& s) {
  const float mt = __fadd_rn(__fmul_rn(s.beta1, m), __fmul_rn(s.one_m_beta1, g));
  const float vt = __fadd_rn(__fmul_rn(s.beta2, v), __fmul_rn(s.one_m_beta2, __fmul_rn(g, g)));
  const float mc = div_uniform(mt, s.bias1, s.rbias1);
  const float vc = div_uniform(vt, s.bias2, s.rbias2);
  const float step = __fdiv_rn(mc, __fadd_rn(__fsqrt_rn(vc), s.eps));
  p = __fsub_rn(__fmul_rn(s.decay, p), __fmul_rn(s.lr, step));
  m = mt;
  v = vt;
}

__device__ __forceinline__ void adam_vec(float4& p, const float4& g, float4& m, float4& v, const AdamScalars& s) {
  adam_elem(p.x, g.x, m.x, v.x, s);
  adam_elem(p.y, g.y, m.y, v.y, s);
  adam_elem(p.z, g.z, m.z, v.z, s);
  adam_elem(p.w, g.w, m.w, v.w, s);
}

// Stores of an updated parameter vector: the parameter itself and, for a
// float32 master (SHADOW), its bf16 copy rounded to nearest even.
template <typename TP, bool SHADOW>
__device__ __forceinline__ void put4(TP* p, __nv_bfloat16* sh, int64_t i, const float4& a) {
  st4(p, i, a);
  if (SHADOW) st4(sh, i, a);
}
template <typename TP, bool SHADOW>
__device__ __forceinline__ void put1(TP* p, __nv_bfloat16* sh, int64_t i, float a) {
  st1(p, i, a);
  if (SHADOW) st1(sh, i, a);
}

// The tile with the gradient summed over ranks.  Full tiles: each thread's
// vectors of every rank's copy, two ranks' in flight at a time, then p, m, v;
// the remote reads cross NVLink, which bounds this path.
template <typename TP, typename TG, bool SHADOW>
__device__ __forceinline__ void adam_tile_reduce(const AdamEntry& e, int64_t off, int len, const AdamScalars& s) {
  TP* __restrict__ p = static_cast<TP*>(e.p) + off;
  const TG* g = static_cast<const TG*>(e.g) + off;
  __nv_bfloat16* __restrict__ sh = SHADOW ? static_cast<__nv_bfloat16*>(e.shadow) + off : nullptr;
  float* __restrict__ m = e.m + off;
  float* __restrict__ v = e.v + off;
  const int t = threadIdx.x;
  if (e.vec && len == ADAM_TILE) {
    int64_t offs[ADAM_VECS];
    float4 gv[ADAM_VECS];
#pragma unroll
    for (int j = 0; j < ADAM_VECS; ++j) offs[j] = 4 * static_cast<int64_t>(j * ADAM_THREADS + t);
    ld4_ranks_rows<TG, ADAM_VECS>(g, offs, gv, s.red);
#pragma unroll
    for (int j = 0; j < ADAM_VECS; ++j) {
      const int idx = j * ADAM_THREADS + t;
      float4 a = ld4(p, idx);
      float4 c = __ldcs(reinterpret_cast<const float4*>(m) + idx);
      float4 d = __ldcs(reinterpret_cast<const float4*>(v) + idx);
      adam_vec(a, gv[j], c, d, s);
      put4<TP, SHADOW>(p, sh, idx, a);
      __stcs(reinterpret_cast<float4*>(m) + idx, c);
      __stcs(reinterpret_cast<float4*>(v) + idx, d);
    }
    return;
  }
  const int nvec = e.vec ? (len >> 2) : 0;
  for (int i = t; i < nvec; i += ADAM_THREADS) {
    const float4 b = ld4_ranks(g, i, s.red);
    float4 a = ld4(p, i);
    float4 c = __ldcs(reinterpret_cast<const float4*>(m) + i);
    float4 d = __ldcs(reinterpret_cast<const float4*>(v) + i);
    adam_vec(a, b, c, d, s);
    put4<TP, SHADOW>(p, sh, i, a);
    __stcs(reinterpret_cast<float4*>(m) + i, c);
    __stcs(reinterpret_cast<float4*>(v) + i, d);
  }
  for (int i = nvec * 4 + t; i < len; i += ADAM_THREADS) {
    float a = ld1(p, i), c = m[i], d = v[i];
    adam_elem(a, ld1_ranks(g, i, s.red), c, d, s);
    put1<TP, SHADOW>(p, sh, i, a);
    m[i] = c;
    v[i] = d;
  }
}

// One tile [off, off+len) of one tensor: parameter type TP, gradient type TG,
// float32 moments.  Full aligned tiles issue all their loads before any math;
// ragged or misaligned pieces take a generic loop.
template <typename TP, typename TG, bool SHADOW>
__device__ __forceinline__ void adam_tile(const AdamEntry& e, int64_t off, int len, const AdamScalars& s) {
  TP* __restrict__ p = static_cast<TP*>(e.p) + off;
  const TG* __restrict__ g = static_cast<const TG*>(e.g) + off;
  __nv_bfloat16* __restrict__ sh = SHADOW ? static_cast<__nv_bfloat16*>(e.shadow) + off : nullptr;
  float* __restrict__ m = e.m + off;
  float* __restrict__ v = e.v + off;
  const int t = threadIdx.x;
  if (e.vec && len == ADAM_TILE) {
    float4 rp[ADAM_VECS], rg[ADAM_VECS], rm[ADAM_VECS], rv[ADAM_VECS];
#pragma unroll
    for (int i = 0; i < ADAM_VECS; ++i) {
      const int idx = i * ADAM_THREADS + t;
      rp[i] = ld4(p, idx);
      rg[i] = ld4(g, idx);
      rm[i] = __ldcs(reinterpret_cast<const float4*>(m) + idx);
      rv[i] = __ldcs(reinterpret_cast<const float4*>(v) + idx);
    }
#pragma unroll
    for (int i = 0; i < ADAM_VECS; ++i) {
      adam_vec(rp[i], rg[i], rm[i], rv[i], s);
      const int idx = i * ADAM_THREADS + t;
      put4<TP, SHADOW>(p, sh, idx, rp[i]);
      __stcs(reinterpret_cast<float4*>(m) + idx, rm[i]);
      __stcs(reinterpret_cast<float4*>(v) + idx, rv[i]);
    }
    return;
  }
  const int nvec = e.vec ? (len >> 2) : 0;
  for (int i = t; i < nvec; i += ADAM_THREADS) {
    float4 a = ld4(p, i);
    float4 b = ld4(g, i);
    float4 c = __ldcs(reinterpret_cast<const float4*>(m) + i);
    float4 d = __ldcs(reinterpret_cast<const float4*>(v) + i);
    adam_vec(a, b, c, d, s);
    put4<TP, SHADOW>(p, sh, i, a);
    __stcs(reinterpret_cast<float4*>(m) + i, c);
    __stcs(reinterpret_cast<float4*>(v) + i, d);
  }
  for (int i = nvec * 4 + t; i < len; i += ADAM_THREADS) {
    float a = ld1(p, i), c = m[i], d = v[i];
    adam_elem(a, ld1(g, i), c, d, s);
    put1<TP, SHADOW>(p, sh, i, a);
    m[i] = c;
    v[i] = d;
  }
}

template <bool REDUCE, typename TP, typename TG, bool SHADOW>
__device__ __forceinline__ void adam_tile_typed(const AdamEntry& e, int64_t off, int len, const AdamScalars& s) {
  if (REDUCE)
    adam_tile_reduce<TP, TG, SHADOW>(e, off, len, s);
  else
    adam_tile<TP, TG, SHADOW>(e, off, len, s);
}

template <bool REDUCE>
__device__ __forceinline__ void adam_tile_any(const AdamEntry& e, int64_t off, int len, const AdamScalars& s) {
  if (e.dtype == MAD_DTYPE_BF16)
    adam_tile_typed<REDUCE, __nv_bfloat16, __nv_bfloat16, false>(e, off, len, s);
  else if (e.dtype == MAD_DTYPE_F32_MASTER)
    adam_tile_typed<REDUCE, float, __nv_bfloat16, true>(e, off, len, s);
  else
    adam_tile_typed<REDUCE, float, float, false>(e, off, len, s);
}

// REDUCE: the gradient summed over ranks (a separate instantiation, so the
// local path keeps its register budget and occupancy).
// One tile per CTA (the grid covers every tile).  REDUCE: the gradient summed
// over ranks (a separate instantiation with its own register budget).
template <bool REDUCE>
__global__ void __launch_bounds__(ADAM_THREADS, REDUCE ? 4 : 8) adamw_multi_kernel(
    const AdamEntry* __restrict__ entries, const int32_t* __restrict__ tile_map, int64_t n_tiles, AdamScalars s) {
  const int64_t tile = blockIdx.x;
  if (tile >= n_tiles) return;
  const AdamEntry& e = entries[tile_map[tile]];
  const int64_t off = (tile - e.tile_begin) * ADAM_TILE;
  const int64_t rem = e.numel - off;
  const int len = static_cast<int>(rem < ADAM_TILE ? rem : ADAM_TILE);
  adam_tile_any<REDUCE>(e, off, len, s);
}

__global__ void __launch_bounds__(ADAM_THREADS, 12) adamw_single_kernel(AdamEntry e, int64_t n_tiles, AdamScalars s) {
  for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
    const int64_t off = tile * ADAM_TILE;
    const int64_t rem = e.numel - off;
    const int len = static_cast<int>(rem < ADAM_TILE ? rem : ADAM_TILE);
    adam_tile_any<false>(e, off, len, s);
  }
}

// RN(1/b) for a divisor 1 >= b >= 2^-40 (else 0: div_uniform then divides):
// the float nearest 1/b, chosen among the double quotient's float rounding and
// its two neighbours by the exact residual |1 - b y| (b y is exact in double:
// 24 x 24 significant bits).
static float reciprocal_rn(float b) {
  if (!(b >= 0x1p-40f && b <= 1.0f)) return 0.0f;
  const float y0 = static_cast<float>(1.0 / static_cast<double>(b));
  float best = y0;
  double best_err = std::fabs(1.0 - static_cast<double>(b) * static_cast<double>(y0));
  for (float y : {std::nextafter(y0, 0.f), std::nextafter(y0, INFINITY)}) {
    const double err = std::fabs(1.0 - static_cast<double>(b) * static_cast<double>(y));
    if (err < best_err) {
      best = y;
      best_err = err;
    }
  }
  return best;
}

// The reference kernel receives its scalars as float32 and forms 1-beta1,
// 1-beta2 and 1-lr*wd in float32 (triton_adam.py:53-58); so do we.
static AdamScalars make_scalars(float lr, float beta1, float beta2, float eps, float wd, float bias1, float bias2) {
  AdamScalars s;
  std::memset(&s, 0, sizeof(s));
  volatile float lr_wd = lr * wd;  // one float32 rounding, never contracted into the subtraction
  s.lr = lr;
  s.beta1 = beta1;
  s.beta2 = beta2;
  s.one_m_beta1 = 1.0f - beta1;
  s.one_m_beta2 = 1.0f - beta2;
  s.eps = eps;
  s.decay = 1.0f - lr_wd;
  s.bias1 = bias1;
  s.bias2 = bias2;
  s.rbias1 = reciprocal_rn(bias1);
  s.rbias2 = reciprocal_rn(bias2);
  return s;
}

static int adam_grid(int64_t n_tiles) {
  // One CTA per tile.  A plan never has more than 2^31 - 1 tiles (mad_adamw_plan
  // refuses more); the single-tensor kernel strides over any beyond the cap.
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(n_tiles, INT32_MAX)));
}

static inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
static inline bool aligned8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; }

// 4-element vectors are legal when p, g (4 elements: 16 B float32, 8 B bf16)
// and the float32 moments (16 B) are aligned for them.
static inline int32_t vec_ok(const void* p, const void* g, const float* m, const float* v, const void* shadow,
                             int32_t dtype) {
  if (dtype == MAD_DTYPE_BF16) return aligned8(p) && aligned8(g) && aligned16(m) && aligned16(v);
  if (dtype == MAD_DTYPE_F32_MASTER)
    return aligned16(p) && aligned8(g) && aligned8(shadow) && aligned16(m) && aligned16(v);
  return aligned16(p) && aligned16(g) && aligned16(m) && aligned16(v);
}

// Table layout: int32 tile map [n_tiles] at offset 0, then the AdamEntry array
// at the next 256-byte boundary.  Both offsets follow from n_tiles alone, so a
// step call needs only the table pointer and the tile count.
static int64_t entries_offset(int64_t n_tiles) {
  return (n_tiles * static_cast<int64_t>(sizeof(int32_t)) + 255) / 256 * 256;
}

static int64_t table_layout(int32_t n, int64_t n_tiles) {
  return entries_offset(n_tiles) + static_cast<int64_t>(n) * static_cast<int64_t>(sizeof(AdamEntry));
}

}  // namespace mad

using namespace mad;

extern "C" int mad_adamw_step(float* param, const float* grad, float* exp_avg, float* exp_avg_sq, int64_t numel,
                              float lr, float bias1, float bias2, float beta1, float beta2, float weight_decay,
                              float eps, void* stream) {
  clear_error();
  if (numel < 0) return fail(MAD_ERR_INVALID, "mad_adamw_step: negative numel");
  if (numel == 0) return MAD_OK;
  if (!param || !grad || !exp_avg || !exp_avg_sq) return fail(MAD_ERR_INVALID, "mad_adamw_step: null pointer");
  if (!(bias1 > 0.f) || !(bias2 > 0.f)) return fail(MAD_ERR_INVALID, "mad_adamw_step: bias corrections must be > 0");
  AdamEntry e{};
  e.p = param;
  e.g = grad;
  e.m = exp_avg;
  e.v = exp_avg_sq;
  e.numel = numel;
  e.tile_begin = 0;
  e.dtype = MAD_DTYPE_F32;
  e.vec = vec_ok(param, grad, exp_avg, exp_avg_sq, nullptr, MAD_DTYPE_F32);
  const int64_t n_tiles = (numel + ADAM_TILE - 1) / ADAM_TILE;
  adamw_single_kernel<<<adam_grid(n_tiles), ADAM_THREADS, 0, static_cast<cudaStream_t>(stream)>>>(
      e, n_tiles, make_scalars(lr, beta1, beta2, eps, weight_decay, bias1, bias2));
  return check_launch("adamw_single_kernel");
}

extern "C" int mad_adamw_table_bytes(const mad_adamw_tensor* tensors, int32_t n_tensors, int64_t* table_bytes) {
  clear_error();
  if (n_tensors < 0 || (n_tensors > 0 && !tensors) || !table_bytes)
    return fail(MAD_ERR_INVALID, "mad_adamw_table_bytes: bad arguments");
  int64_t tiles = 0;
  for (int32_t i = 0; i < n_tensors; ++i) {
    if (tensors[i].numel < 0) return fail(MAD_ERR_INVALID, "mad_adamw_table_bytes: negative numel");
    tiles += (tensors[i].numel + ADAM_TILE - 1) / ADAM_TILE;
  }
  *table_bytes = table_layout(n_tensors, tiles);
  return MAD_OK;
}

extern "C" int mad_adamw_plan(const mad_adamw_tensor* tensors, int32_t n_tensors, void* dev_table,
                              int64_t table_bytes, int64_t* n_tiles_out, void* stream) {
  clear_error();
  if (n_tensors < 0 || (n_tensors > 0 && !tensors) || !n_tiles_out || (n_tensors > 0 && !dev_table))
    return fail(MAD_ERR_INVALID, "mad_adamw_plan: bad arguments");
  std::vector<AdamEntry> entries(n_tensors);
  int64_t tiles = 0;
  for (int32_t i = 0; i < n_tensors; ++i) {
    const mad_adamw_tensor& t = tensors[i];
    if (t.numel < 0) return fail(MAD_ERR_INVALID, "mad_adamw_plan: negative numel");
    if (t.numel > 0 && (!t.param || !t.grad || !t.exp_avg || !t.exp_avg_sq))
      return fail(MAD_ERR_INVALID, "mad_adamw_plan: null pointer in tensor %d", i);
    if (t.dtype != MAD_DTYPE_F32 && t.dtype != MAD_DTYPE_BF16 && t.dtype != MAD_DTYPE_F32_MASTER)
      return fail(MAD_ERR_INVALID, "mad_adamw_plan: tensor %d has unknown dtype %d", i, t.dtype);
    if (t.dtype == MAD_DTYPE_F32_MASTER && t.numel > 0 && !t.shadow)
      return fail(MAD_ERR_INVALID, "mad_adamw_plan: tensor %d (float32 master) has no bf16 shadow", i);
    AdamEntry& e = entries[i];
    std::memset(&e, 0, sizeof(e));
    e.p = t.param;
    e.g = t.grad;
    e.m = t.exp_avg;
    e.v = t.exp_avg_sq;
    e.numel = t.numel;
    e.tile_begin = tiles;
    e.dtype = t.dtype;
    e.shadow = t.dtype == MAD_DTYPE_F32_MASTER ? t.shadow : nullptr;
    e.vec = vec_ok(t.param, t.grad, t.exp_avg, t.exp_avg_sq, t.shadow, t.dtype);
    tiles += (t.numel + ADAM_TILE - 1) / ADAM_TILE;
  }
  if (tiles > INT32_MAX) return fail(MAD_ERR_INVALID, "mad_adamw_plan: too many tiles");
  const int64_t need = table_layout(n_tensors, tiles);
  if (table_bytes < need) return fail(MAD_ERR_WORKSPACE, "mad_adamw_plan: table needs %lld bytes, got %lld",
                                      static_cast<long long>(need), static_cast<long long>(table_bytes));
  *n_tiles_out = tiles;
  if (need == 0) return MAD_OK;
  std::vector<uint8_t> host(need, 0);
  std::memcpy(host.data() + entries_offset(tiles), entries.data(), entries.size() * sizeof(AdamEntry));
  int32_t* map = reinterpret_cast<int32_t*>(host.data());
  for (int32_t i = 0; i < n_tensors; ++i) {
    const int64_t nt = (entries[i].numel + ADAM_TILE - 1) / ADAM_TILE;
    for (int64_t k = 0; k < nt; ++k) map[entries[i].tile_begin + k] = i;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemcpyAsync(dev_table, host.data(), need, cudaMemcpyHostToDevice, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return fail_cuda("mad_adamw_plan: table upload");
  return MAD_OK;
}

static int adamw_step_multi(const void* dev_table, int64_t n_tiles, float lr, float beta1, float beta2, float eps,
                            float weight_decay, float bias1, float bias2, const mad_grad_reduce* reduce,
                            void* stream, const char* who) {
  clear_error();
  if (n_tiles < 0) return fail(MAD_ERR_INVALID, "%s: negative tile count", who);
  if (n_tiles == 0) return MAD_OK;
  if (!dev_table) return fail(MAD_ERR_INVALID, "%s: null table", who);
  if (!(bias1 > 0.f) || !(bias2 > 0.f)) return fail(MAD_ERR_INVALID, "%s: bias corrections must be > 0", who);
  AdamScalars sc = make_scalars(lr, beta1, beta2, eps, weight_decay, bias1, bias2);
  if (int rc = grad_reduce_from(reduce, &sc.red, who)) return rc;
  const uint8_t* base = static_cast<const uint8_t*>(dev_table);
  const int32_t* tile_map = reinterpret_cast<const int32_t*>(base);
  const AdamEntry* entries = reinterpret_cast<const AdamEntry*>(base + entries_offset(n_tiles));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (sc.red.n > 0)
    adamw_multi_kernel<true><<<adam_grid(n_tiles), ADAM_THREADS, 0, st>>>(entries, tile_map, n_tiles, sc);
  else
    adamw_multi_kernel<false><<<adam_grid(n_tiles), ADAM_THREADS, 0, st>>>(entries, tile_map, n_tiles, sc);
  return check_launch("adamw_multi_kernel");
}

extern "C" int mad_adamw_step_multi(const void* dev_table, int64_t n_tiles, float lr, float beta1, float beta2,
                                    float eps, float weight_decay, float bias1, float bias2, void* stream) {
  return adamw_step_multi(dev_table, n_tiles, lr, beta1, beta2, eps, weight_decay, bias1, bias2, nullptr, stream,
                          "mad_adamw_step_multi");
}

extern "C" int mad_adamw_step_multi_reduce(const void* dev_table, int64_t n_tiles, float lr, float beta1,
                                           float beta2, float eps, float weight_decay, float bias1, float bias2,
                                           const mad_grad_reduce* reduce, void* stream) {
  if (!reduce) {
    clear_error();
    return fail(MAD_ERR_INVALID, "mad_adamw_step_multi_reduce: null reduce descriptor");
  }
  return adamw_step_multi(dev_table, n_tiles, lr, beta1, beta2, eps, weight_decay, bias1, bias2, reduce, stream,
                          "mad_adamw_step_multi_reduce");
}
