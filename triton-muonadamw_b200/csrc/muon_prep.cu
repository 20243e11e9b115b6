// Muon prologue, one pass over every planned matrix (triton_muon.py:346-356):
//   mom = beta*mom + (1-beta)*g              (buffer updated in place, fp32 or bf16)
//   u   = g + beta*(mom - g)  if nesterov    (the buffer itself is untouched)
//   X   = bf16(u), transposed when rows > cols, so X is m x n with m <= n
//   s   = 1 / max(bf16(||X||_F), bf16(eps))  (the reference's bf16 norm)
// X is written unnormalised; s is folded into the first Gram and update
// epilogues.
//
// The pass is HBM-bound: 14 B per element with float32 buffers (read g, mom;
// write mom, X), 8 B with bf16 buffers.  To keep bytes in flight at the
// power-capped SM clock the loop never stalls a CTA on bookkeeping:
//  * each warp writes the sum of squares of its part of a 64x64 tile to its
//    own slot (no block-wide reduction, no atomics, no fences in the loop);
//    a second launch, one CTA per matrix, adds a matrix's slots in a fixed
//    order in double precision -- the norm is deterministic;
//  * the gradient and momentum of a CTA's next two tiles are copied into a
//    shared-memory ring (cp.async) while the current tile is computed and
//    stored: two tiles of loads in flight per CTA, four per SM, held in
//    shared memory rather than registers;
//  * tall matrices are transposed through a bf16 shared-memory tile (the
//    only block barriers of the loop).
// With a gradient reduction the other ranks' gradient copies are read over
// NVLink instead (a separate kernel that reads directly: its summed loads
// keep two ranks' vectors in flight per thread).
#include <cuda_runtime.h>

#include "capi_common.h"
#include "elem_io.cuh"
#include "plan.cuh"
#include "ptx_sm100.cuh"

namespace mad {

constexpr int PREP_THREADS = 256;
constexpr int PREP_WARPS = PREP_THREADS / 32;  // partial sums per tile (one per warp)
static_assert(PREP_WARPS == PREP_PARTIALS_PER_TILE, "plan layout of the partial sums");
constexpr int FINALIZE_THREADS = 512;

struct PrepScalars {
  float beta, one_m_beta, eps_bf16;
  int nesterov;
  GradReduce red;  // red.n > 0: the gradient is the mean of every rank's copy (peer memory)
};

// mom.mul_(beta).add_(grad, alpha=1-beta) (triton_muon.py:346): one rounded
// product, then torch's fused `self + alpha*other` (a single FMA rounding).
// With bf16 buffers each eager op's float32 result is rounded to bf16 on its
// store, and so is each step of the Nesterov expression (triton_muon.py:348).
template <bool BF16>
__device__ __forceinline__ float prep_update(float g, float& mom, const PrepScalars& s) {
  if (BF16) {
    mom = bf16_round(__fmaf_rn(s.one_m_beta, g, bf16_round(__fmul_rn(mom, s.beta))));
    if (!s.nesterov) return mom;
    return bf16_round(__fadd_rn(g, bf16_round(__fmul_rn(s.beta, bf16_round(__fsub_rn(mom, g))))));
  }
  mom = __fmaf_rn(s.one_m_beta, g, __fmul_rn(mom, s.beta));
  return s.nesterov ? __fadd_rn(g, __fmul_rn(s.beta, __fsub_rn(mom, g))) : mom;
}

// One tile's position and the vectors a thread loads from it: rows
// r0 + 16 i + (t >> 4), i = 0..3, columns c0 + 4 (t & 15) .. + 3.
struct TileRef2 {
  MatDesc* md;
  int r0, c0;
  bool full;  // whole 64x64 tile inside the matrix and 4-element vectors legal
};

struct TileRegs {
  float4 g[4], m[4];
};

__device__ __forceinline__ TileRef2 locate(MatDesc* mats, const int32_t* prep_map, int64_t tile) {
  TileRef2 tr;
  tr.md = mats + prep_map[tile];
  const int local = static_cast<int>(tile - tr.md->prep_begin);
  tr.r0 = (local / tr.md->prep_tiles_c) * PREP_TILE;
  tr.c0 = (local % tr.md->prep_tiles_c) * PREP_TILE;
  tr.full = tr.md->vec != 0 && tr.r0 + PREP_TILE <= tr.md->rows && tr.c0 + PREP_TILE <= tr.md->cols;
  return tr;
}

__device__ __forceinline__ int64_t vec_offset(const TileRef2& tr, int i) {
  return static_cast<int64_t>(tr.r0 + i * 16 + (threadIdx.x >> 4)) * tr.md->cols + tr.c0 + (threadIdx.x & 15) * 4;
}

// Momentum update and store of a full tile whose loads are in `r`; xv
// receives the (Nesterov) update u.
template <typename TM>
__device__ __forceinline__ void finish_full(const TileRef2& tr, TileRegs& r, float (&xv)[4][4], const PrepScalars& s) {
  constexpr bool BF16 = sizeof(TM) == 2;
  TM* __restrict__ mom = static_cast<TM*>(tr.md->mom);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    xv[i][0] = prep_update<BF16>(r.g[i].x, r.m[i].x, s);
    xv[i][1] = prep_update<BF16>(r.g[i].y, r.m[i].y, s);
    xv[i][2] = prep_update<BF16>(r.g[i].z, r.m[i].z, s);
    xv[i][3] = prep_update<BF16>(r.g[i].w, r.m[i].w, s);
    st4(mom + vec_offset(tr, i), 0, r.m[i]);
  }
}

// The other tiles: edges, unaligned rows, or gradients summed over ranks.
// TM is the momentum's type (bf16 momentum rounds the glue to bf16), TG the
// gradient's (a float32 master takes a bf16 gradient).
template <typename TM, typename TG, bool REDUCE>
__device__ __forceinline__ void values_general(const TileRef2& tr, float (&xv)[4][4], const PrepScalars& s) {
  constexpr bool BF16 = sizeof(TM) == 2;
  const MatDesc* md = tr.md;
  const int rows = md->rows, cols = md->cols, t = threadIdx.x;
  const TG* __restrict__ g = static_cast<const TG*>(md->g);
  TM* __restrict__ mom = static_cast<TM*>(md->mom);
  const int cl = (t & 15) * 4;
  if (REDUCE && tr.full) {
    // Each row's copies from every rank in flight together, one row at a time.
    float4 gv[4], mv[4];
    int64_t offs[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      offs[i] = vec_offset(tr, i);
      mv[i] = ld4(mom + offs[i], 0);
    }
    ld4_ranks_rows<TG, 4>(g, offs, gv, s.red);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      xv[i][0] = prep_update<BF16>(gv[i].x, mv[i].x, s);
      xv[i][1] = prep_update<BF16>(gv[i].y, mv[i].y, s);
      xv[i][2] = prep_update<BF16>(gv[i].z, mv[i].z, s);
      xv[i][3] = prep_update<BF16>(gv[i].w, mv[i].w, s);
      st4(mom + offs[i], 0, mv[i]);
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = tr.r0 + i * 16 + (t >> 4), c = tr.c0 + cl;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      xv[i][k] = 0.f;
      if (r < rows && c + k < cols) {
        const int64_t off = static_cast<int64_t>(r) * cols + c + k;
        float mvv = ld1(mom, off);
        const float gg = REDUCE ? ld1_ranks(g, off, s.red) : ld1(g, off);
        xv[i][k] = prep_update<BF16>(gg, mvv, s);
        st1(mom, off, mvv);
      }
    }
  }
}

template <bool REDUCE>
__device__ __forceinline__ void values_general_any(const TileRef2& tr, float (&xv)[4][4], const PrepScalars& s) {
  if (tr.md->dtype == MAD_DTYPE_BF16)
    values_general<__nv_bfloat16, __nv_bfloat16, REDUCE>(tr, xv, s);
  else if (tr.md->dtype == MAD_DTYPE_F32_MASTER)
    values_general<float, __nv_bfloat16, REDUCE>(tr, xv, s);
  else
    values_general<float, float, REDUCE>(tr, xv, s);
}

__device__ __forceinline__ uint32_t pack2(__nv_bfloat16 lo, __nv_bfloat16 hi) {
  return static_cast<uint32_t>(__bfloat16_as_ushort(lo)) | (static_cast<uint32_t>(__bfloat16_as_ushort(hi)) << 16);
}

// bf16 cast of u, this thread's sum of squares, and the X store (direct, or
// through shared memory for tall matrices).
__device__ __forceinline__ void write_x(const TileRef2& tr, const float (&xv)[4][4], float& ss,
                                        __nv_bfloat16 (*tile_t)[PREP_TILE + 2]) {
  const MatDesc* md = tr.md;
  const int t = threadIdx.x, rows = md->rows, cols = md->cols, ld_x = md->ld_x;
  const int cl = (t & 15) * 4;
  __nv_bfloat16* __restrict__ x = md->x[0];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int rl = i * 16 + (t >> 4);
    const int r = tr.r0 + rl, c = tr.c0 + cl;
    __nv_bfloat16 xb[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      xb[k] = __float2bfloat16_rn(xv[i][k]);
      const float q = __bfloat162float(xb[k]);
      ss = fmaf(q, q, ss);
    }
    if (!md->transposed) {
      if (r < rows) {
        __nv_bfloat16* dst = x + static_cast<int64_t>(r) * ld_x + c;
        if (c + 4 <= cols) {
          uint2 packed;
          packed.x = pack2(xb[0], xb[1]);
          packed.y = pack2(xb[2], xb[3]);
          *reinterpret_cast<uint2*>(dst) = packed;
        } else {
          for (int k = 0; k < 4 && c + k < cols; ++k) dst[k] = xb[k];
        }
      }
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) tile_t[cl + k][rl] = xb[k];
    }
  }
  if (!md->transposed) return;
  __syncthreads();  // the tile is complete
  // X row = parameter column, X column = parameter row.
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int xr = i * 16 + (t >> 4);
    const int xc = (t & 15) * 4;
    const int row = tr.c0 + xr, col = tr.r0 + xc;
    if (row < cols) {
      __nv_bfloat16* dst = x + static_cast<int64_t>(row) * ld_x + col;
      if (col + 4 <= rows) {
        uint2 packed;
        packed.x = *reinterpret_cast<const uint32_t*>(&tile_t[xr][xc]);
        packed.y = *reinterpret_cast<const uint32_t*>(&tile_t[xr][xc + 2]);
        *reinterpret_cast<uint2*>(dst) = packed;
      } else {
        for (int k = 0; k < 4 && col + k < rows; ++k) dst[k] = tile_t[xr][xc + k];
      }
    }
  }
  __syncthreads();  // every thread has read the tile before the next one is written
}

// ---------------------------------------------------------------- local gradients: cp.async ring
// Each CTA strides over the tiles; the gradient and momentum of its tile
// k + PREP_STAGES - 1 are copied into shared memory (cp.async, one 16-byte
// slot per thread, row and array) while tile k is computed, so PREP_STAGES - 1
// tiles of loads stay in flight per CTA without holding registers.  A thread
// reads back only the slots it copied: no barrier guards the ring.
constexpr int PREP_STAGES = 3;
constexpr int PREP_SLOTS = 8;  // per thread and tile: 4 rows x (gradient, momentum)
constexpr int PREP_STAGE_BYTES = PREP_SLOTS * PREP_THREADS * 16;
constexpr int PREP_T_PITCH = PREP_TILE + 2;  // bf16 transpose tile row pitch (132 B: 4-byte reads, 2-way writes)
constexpr int PREP_SMEM_BYTES = PREP_STAGES * PREP_STAGE_BYTES + PREP_TILE * PREP_T_PITCH * 2;

template <typename TM, typename TG>
__device__ __forceinline__ void issue_tile_typed(const TileRef2& tr, float4* stage) {
  const TG* g = static_cast<const TG*>(tr.md->g);
  const TM* mom = static_cast<const TM*>(tr.md->mom);
  const int t = threadIdx.x;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t off = vec_offset(tr, i);
    cp_async_vec(smem_addr_u32(stage + i * PREP_THREADS + t), g + off);
    cp_async_vec(smem_addr_u32(stage + (4 + i) * PREP_THREADS + t), mom + off);
  }
}

// Copies of one full tile into a ring stage, then one commit group (empty for
// tiles the general path handles, so the group count stays uniform).
__device__ __forceinline__ void issue_tile(const TileRef2& tr, bool valid, float4* stage) {
  if (valid && tr.full) {
    if (tr.md->dtype == MAD_DTYPE_BF16)
      issue_tile_typed<__nv_bfloat16, __nv_bfloat16>(tr, stage);
    else if (tr.md->dtype == MAD_DTYPE_F32_MASTER)
      issue_tile_typed<float, __nv_bfloat16>(tr, stage);
    else
      issue_tile_typed<float, float>(tr, stage);
  }
  cp_async_commit();
}

template <typename TM, typename TG>
__device__ __forceinline__ void read_tile_typed(const float4* stage, TileRegs& r) {
  const int t = threadIdx.x;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    r.g[i] = slot_vec(stage + i * PREP_THREADS + t, static_cast<const TG*>(nullptr));
    r.m[i] = slot_vec(stage + (4 + i) * PREP_THREADS + t, static_cast<const TM*>(nullptr));
  }
}

__global__ void __launch_bounds__(PREP_THREADS, 2) muon_prep_ring_kernel(MatDesc* __restrict__ mats,
                                                                          const int32_t* __restrict__ prep_map,
                                                                          float* __restrict__ partials,
                                                                          int64_t n_tiles, PrepScalars s) {
  extern __shared__ __align__(16) uint8_t prep_smem[];
  float4* ring = reinterpret_cast<float4*>(prep_smem);
  auto tile_t = reinterpret_cast<__nv_bfloat16 (*)[PREP_T_PITCH]>(prep_smem + PREP_STAGES * PREP_STAGE_BYTES);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t G = gridDim.x;
  int64_t tile = blockIdx.x;
  if (tile >= n_tiles) return;

  // Tiles k, k+1, k+2 of this CTA: a (being computed), b, c (in flight).
  TileRef2 a = locate(mats, prep_map, tile);
  TileRef2 b = a;
  const bool b_ok = tile + G < n_tiles;
  if (b_ok) b = locate(mats, prep_map, tile + G);
  issue_tile(a, true, ring);
  issue_tile(b, b_ok, ring + PREP_SLOTS * PREP_THREADS);
  int st = 0;
  for (; tile < n_tiles; tile += G) {
    const int64_t far = tile + 2 * G;
    TileRef2 c = b;
    const bool c_ok = far < n_tiles;
    if (c_ok) c = locate(mats, prep_map, far);
    const int st_far = st == 0 ? 2 : st - 1;  // (st + 2) % 3
    issue_tile(c, c_ok, ring + st_far * PREP_SLOTS * PREP_THREADS);
    cp_async_wait<PREP_STAGES - 1>();  // this thread's copies of tile k have landed

    float xv[4][4];
    if (a.full) {
      TileRegs r;
      const float4* stage = ring + st * PREP_SLOTS * PREP_THREADS;
      if (a.md->dtype == MAD_DTYPE_BF16) {
        read_tile_typed<__nv_bfloat16, __nv_bfloat16>(stage, r);
        finish_full<__nv_bfloat16>(a, r, xv, s);
      } else if (a.md->dtype == MAD_DTYPE_F32_MASTER) {
        read_tile_typed<float, __nv_bfloat16>(stage, r);
        finish_full<float>(a, r, xv, s);
      } else {
        read_tile_typed<float, float>(stage, r);
        finish_full<float>(a, r, xv, s);
      }
    } else {
      values_general_any<false>(a, xv, s);
    }
    float ss = 0.f;
    write_x(a, xv, ss, tile_t);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) partials[tile * PREP_WARPS + warp] = ss;
    a = b;
    b = c;
    st = st == 2 ? 0 : st + 1;
  }
  cp_async_wait<0>();
}

// ---------------------------------------------------------------- gradients summed over ranks
// Every rank's copy is read over NVLink with two ranks' vectors in flight per
// thread (ld4_ranks_rows); those loads bound this path, so it reads directly.
__global__ void __launch_bounds__(PREP_THREADS, 2) muon_prep_reduce_kernel(MatDesc* __restrict__ mats,
                                                                            const int32_t* __restrict__ prep_map,
                                                                            float* __restrict__ partials,
                                                                            int64_t n_tiles, PrepScalars s) {
  __shared__ __nv_bfloat16 tile_t[PREP_TILE][PREP_T_PITCH];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
    const TileRef2 cur = locate(mats, prep_map, tile);
    float xv[4][4];
    values_general_any<true>(cur, xv, s);
    float ss = 0.f;
    write_x(cur, xv, ss, tile_t);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) partials[tile * PREP_WARPS + warp] = ss;
  }
}

// One CTA per matrix: the sum of its tiles' partial sums of squares, in a
// fixed order (per-thread strided sums, then the warp tree, then the warps in
// order) in double precision; the norm is rounded to bf16 as the reference's
// X.norm() on a bf16 tensor is, clamped with bf16(eps), and stored inverted.
__global__ void __launch_bounds__(FINALIZE_THREADS) muon_norm_kernel(MatDesc* __restrict__ mats,
                                                                     const float* __restrict__ partials,
                                                                     float eps_bf16) {
  __shared__ double red[FINALIZE_THREADS / 32];
  MatDesc* md = mats + blockIdx.x;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const float* p = partials + static_cast<int64_t>(md->prep_begin) * PREP_WARPS;
  const int64_t count = static_cast<int64_t>(md->prep_count) * PREP_WARPS;
  double acc = 0.0;
  int64_t k = t;
  for (; k + 3 * FINALIZE_THREADS < count; k += 4 * FINALIZE_THREADS) {
    const float a = p[k], b = p[k + FINALIZE_THREADS], c = p[k + 2 * FINALIZE_THREADS], d = p[k + 3 * FINALIZE_THREADS];
    acc += static_cast<double>(a);
    acc += static_cast<double>(b);
    acc += static_cast<double>(c);
    acc += static_cast<double>(d);
  }
  for (; k < count; k += FINALIZE_THREADS) acc += static_cast<double>(p[k]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) red[warp] = acc;
  __syncthreads();
  if (t == 0) {
    double tot = 0.0;
    for (int w = 0; w < FINALIZE_THREADS / 32; ++w) tot += red[w];
    float norm = bf16_round(static_cast<float>(sqrt(tot)));
    if (!(norm >= eps_bf16)) norm = (norm != norm) ? norm : eps_bf16;  // clamp(min=eps), NaN kept
    md->inv_norm = 1.0f / norm;
  }
}

int launch_muon_prep(MatDesc* mats, int32_t n_mats, const int32_t* prep_map, float* partials, int64_t n_tiles,
                     double beta, int nesterov, float eps, const GradReduce& red, cudaStream_t stream) {
  if (n_tiles <= 0 || n_mats <= 0) return MAD_OK;
  PrepScalars s;
  s.red = red;
  // The reference passes Python floats: beta is rounded to float32 by the
  // multiply, alpha = 1 - beta is formed in double and then rounded.
  s.beta = static_cast<float>(beta);
  s.one_m_beta = static_cast<float>(1.0 - beta);
  s.eps_bf16 = bf16_round(eps);
  s.nesterov = nesterov ? 1 : 0;
  // Two resident CTAs per SM (the ring's shared memory; the rank-summing
  // kernel's registers); every CTA strides over the tiles.
  const int64_t cap = static_cast<int64_t>(num_sms()) * 2;
  const int grid = static_cast<int>(n_tiles < cap ? n_tiles : cap);
  if (red.n > 0) {
    muon_prep_reduce_kernel<<<grid, PREP_THREADS, 0, stream>>>(mats, prep_map, partials, n_tiles, s);
    if (int rc = check_launch("muon_prep_reduce_kernel")) return rc;
  } else {
    if (cudaFuncSetAttribute(muon_prep_ring_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PREP_SMEM_BYTES) !=
        cudaSuccess)
      return fail_cuda("cudaFuncSetAttribute(muon_prep_ring_kernel)");
    muon_prep_ring_kernel<<<grid, PREP_THREADS, PREP_SMEM_BYTES, stream>>>(mats, prep_map, partials, n_tiles, s);
    if (int rc = check_launch("muon_prep_ring_kernel")) return rc;
  }
  muon_norm_kernel<<<n_mats, FINALIZE_THREADS, 0, stream>>>(mats, partials, s.eps_bf16);
  return check_launch("muon_norm_kernel");
}

}  // namespace mad
