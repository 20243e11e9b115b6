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

}  // namespace mad
