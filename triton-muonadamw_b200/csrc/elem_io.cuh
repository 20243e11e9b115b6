// Element access shared by the elementwise kernels: parameters, gradients and
// Muon momentum are float32 or bf16 in memory and float32 in registers.
// bf16 loads widen exactly; bf16 stores round to nearest even.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>

namespace mad {

// 4-element vectors (float32: 16 B, bf16: 8 B), indexed in units of 4 elements.
__device__ __forceinline__ float4 ld4(const float* p, int64_t i) { return __ldcs(reinterpret_cast<const float4*>(p) + i); }
__device__ __forceinline__ float4 ld4(const __nv_bfloat16* p, int64_t i) {
  const uint2 u = __ldcs(reinterpret_cast<const uint2*>(p) + i);
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u), __uint_as_float(u.y << 16),
                     __uint_as_float(u.y & 0xFFFF0000u));
}
__device__ __forceinline__ void st4(float* p, int64_t i, const float4& v) { __stcs(reinterpret_cast<float4*>(p) + i, v); }
__device__ __forceinline__ void st4(__nv_bfloat16* p, int64_t i, const float4& v) {
  const __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
  uint2 u;
  u.x = *reinterpret_cast<const uint32_t*>(&lo);
  u.y = *reinterpret_cast<const uint32_t*>(&hi);
  __stcs(reinterpret_cast<uint2*>(p) + i, u);
}
__device__ __forceinline__ float ld1(const float* p, int64_t i) { return p[i]; }
__device__ __forceinline__ float ld1(const __nv_bfloat16* p, int64_t i) { return __bfloat162float(p[i]); }
__device__ __forceinline__ void st1(float* p, int64_t i, float v) { p[i] = v; }
__device__ __forceinline__ void st1(__nv_bfloat16* p, int64_t i, float v) { p[i] = __float2bfloat16_rn(v); }

// ------------------------------------------------------------ gradients summed over ranks
// A data-parallel gradient read as the sum of every rank's copy: rank k's copy
// of the element at address g lives at g + delta[k] bytes (peer memory mapped
// into this process, delta 0 for this rank's own copy).  Summed in rank order
// in float32, multiplied by `scale` (1/n for a mean), rounded to the gradient's
// element type.  n == 0: the local gradient alone, unchanged.
constexpr int MAX_RANKS = 8;

struct GradReduce {
  int32_t n;
  float scale;
  int64_t delta[MAX_RANKS];
};

// Loads of another rank's memory bypass L1 (ld.global.cg): the copy a peer
// wrote is never served from a line this SM cached earlier.
__device__ __forceinline__ float4 ld4_peer(const float* p, int64_t i) {
  return __ldcg(reinterpret_cast<const float4*>(p) + i);
}
__device__ __forceinline__ float4 ld4_peer(const __nv_bfloat16* p, int64_t i) {
  const uint2 u = __ldcg(reinterpret_cast<const uint2*>(p) + i);
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u), __uint_as_float(u.y << 16),
                     __uint_as_float(u.y & 0xFFFF0000u));
}
__device__ __forceinline__ float ld1_peer(const float* p, int64_t i) { return __ldcg(p + i); }
__device__ __forceinline__ float ld1_peer(const __nv_bfloat16* p, int64_t i) {
  return __uint_as_float(static_cast<uint32_t>(__ldcg(reinterpret_cast<const unsigned short*>(p) + i)) << 16);
}

template <typename T>
__device__ __forceinline__ const T* rank_copy(const T* g, int64_t delta) {
  return reinterpret_cast<const T*>(reinterpret_cast<const char*>(g) + delta);
}

__device__ __forceinline__ float round_as(const float*, float x) { return x; }
__device__ __forceinline__ float round_as(const __nv_bfloat16*, float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// All ranks' loads are issued before the first add (up to MAX_RANKS vectors in flight).
template <typename T>
__device__ __forceinline__ float4 ld4_ranks(const T* g, int64_t i, const GradReduce& r) {
  float4 v[MAX_RANKS];
#pragma unroll
  for (int k = 0; k < MAX_RANKS; ++k)
    if (k < r.n) v[k] = ld4_peer(rank_copy(g, r.delta[k]), i);
  float4 a = v[0];
#pragma unroll
  for (int k = 1; k < MAX_RANKS; ++k)
    if (k < r.n) {
      a.x = __fadd_rn(a.x, v[k].x);
      a.y = __fadd_rn(a.y, v[k].y);
      a.z = __fadd_rn(a.z, v[k].z);
      a.w = __fadd_rn(a.w, v[k].w);
    }
  return make_float4(round_as(g, __fmul_rn(a.x, r.scale)), round_as(g, __fmul_rn(a.y, r.scale)),
                     round_as(g, __fmul_rn(a.z, r.scale)), round_as(g, __fmul_rn(a.w, r.scale)));
}

__device__ __forceinline__ float4 add4(const float4& a, const float4& b) {
  return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}

// R vectors (at element offsets off[j] from g) summed over ranks, two ranks'
// loads (2R vectors) in flight at a time: remote reads are latency-bound, so
// the bytes in flight per thread set the NVLink throughput.  The sum starts
// from -0.0, which leaves rank 0's value unchanged (-0 + x == x for every x),
// so the result equals the plain rank-order sum.
template <typename T, int R>
__device__ __forceinline__ void ld4_ranks_rows(const T* g, const int64_t (&off)[R], float4 (&out)[R],
                                               const GradReduce& r) {
  float4 acc[R];
#pragma unroll
  for (int j = 0; j < R; ++j) acc[j] = make_float4(-0.f, -0.f, -0.f, -0.f);
  int k = 0;
  for (; k + 2 <= r.n; k += 2) {
    const T* ga = rank_copy(g, r.delta[k]);
    const T* gb = rank_copy(g, r.delta[k + 1]);
    float4 a[R], b[R];
#pragma unroll
    for (int j = 0; j < R; ++j) {
      a[j] = ld4_peer(ga + off[j], 0);
      b[j] = ld4_peer(gb + off[j], 0);
    }
#pragma unroll
    for (int j = 0; j < R; ++j) acc[j] = add4(add4(acc[j], a[j]), b[j]);
  }
  if (k < r.n) {
    const T* ga = rank_copy(g, r.delta[k]);
    float4 a[R];
#pragma unroll
    for (int j = 0; j < R; ++j) a[j] = ld4_peer(ga + off[j], 0);
#pragma unroll
    for (int j = 0; j < R; ++j) acc[j] = add4(acc[j], a[j]);
  }
#pragma unroll
  for (int j = 0; j < R; ++j)
    out[j] = make_float4(round_as(g, __fmul_rn(acc[j].x, r.scale)), round_as(g, __fmul_rn(acc[j].y, r.scale)),
                         round_as(g, __fmul_rn(acc[j].z, r.scale)), round_as(g, __fmul_rn(acc[j].w, r.scale)));
}

template <typename T>
__device__ __forceinline__ float ld1_ranks(const T* g, int64_t i, const GradReduce& r) {
  float v[MAX_RANKS];
#pragma unroll
  for (int k = 0; k < MAX_RANKS; ++k)
    if (k < r.n) v[k] = ld1_peer(rank_copy(g, r.delta[k]), i);
  float a = v[0];
#pragma unroll
  for (int k = 1; k < MAX_RANKS; ++k)
    if (k < r.n) a = __fadd_rn(a, v[k]);
  return round_as(g, __fmul_rn(a, r.scale));
}

}  // namespace mad
