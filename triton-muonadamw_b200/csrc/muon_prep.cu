// Muon prologue, one pass over every planned matrix (triton_muon.py:346-356):
//   mom = beta*mom + (1-beta)*g              (buffer updated in place, fp32 or bf16)
//   u   = g + beta*(mom - g)  if nesterov    (the buffer itself is untouched)
//   X   = bf16(u), transposed when rows > cols, so X is m x n with m <= n
//   s   = 1 / max(bf16(||X||_F), bf16(eps))  (the reference's bf16 norm)
// X is written unnormalised; s is folded into the first Gram and update
// epilogues.
//
// The pass is HBM-bound: 14 B per element with float32 buffers (read g, mom;
// write mom, X), 8 B with bf16 buffers.  It runs in the optimizer step at the
// SM clock the power-capped Newton-Schulz GEMMs leave, where resident warps,
// not per-thread pipelining, keep the bytes in flight:
//  * one 64x64 tile per 256-thread CTA over a grid of every tile, four CTAs
//    per SM, all of a tile's loads issued before its arithmetic;
//  * each warp writes the sum of squares of its part of the tile to its own
//    slot (no block-wide reduction, no atomics, no fences); a second launch,
//    one CTA per matrix, adds a matrix's slots in a fixed order in double
//    precision -- the norm is deterministic;
//  * tall matrices are transposed through a bf16 shared-memory tile (the
//    kernel's only block barriers).
// With a gradient reduction the other ranks' gradient copies are read over
// NVLink as well (its own instantiation: the summed loads keep two ranks'
// vectors in flight per thread).
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
constexpr int PREP_T_PITCH = PREP_TILE + 2;  // bf16 transpose tile row pitch (132 B: 4-byte reads, 2-way writes)

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
                                        __nv_bfloat16 (*tile_t)[PREP_T_PITCH]) {
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

// ---------------------------------------------------------------- the prep kernel
template <typename TM, typename TG>
__device__ __forceinline__ void load_full_typed(const TileRef2& tr, TileRegs& r) {
  const TG* __restrict__ g = static_cast<const TG*>(tr.md->g);
  const TM* __restrict__ mom = static_cast<const TM*>(tr.md->mom);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t off = vec_offset(tr, i);
    r.g[i] = ld4(g + off, 0);
    r.m[i] = ld4(mom + off, 0);
  }
}

// One 64x64 tile per CTA; the grid covers every tile and the hardware keeps
// four CTAs per SM resident.  A full tile's loads are all issued before any
// arithmetic.  REDUCE: the gradient summed over ranks (its own instantiation
// and register budget).  Each warp stores its sum of squares to
// partials[tile * PREP_WARPS + warp].
template <bool REDUCE>
__global__ void __launch_bounds__(PREP_THREADS, REDUCE ? 2 : 4) muon_prep_kernel(MatDesc* __restrict__ mats,
                                                                                const int32_t* __restrict__ prep_map,
                                                                                float* __restrict__ partials,
                                                                                int64_t n_tiles, PrepScalars s) {
  __shared__ __nv_bfloat16 tile_t[PREP_TILE][PREP_T_PITCH];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t tile = blockIdx.x;
  if (tile >= n_tiles) return;
  const TileRef2 cur = locate(mats, prep_map, tile);
  float xv[4][4];
  if (!REDUCE && cur.full) {
    TileRegs r;
    if (cur.md->dtype == MAD_DTYPE_BF16) {
      load_full_typed<__nv_bfloat16, __nv_bfloat16>(cur, r);
      finish_full<__nv_bfloat16>(cur, r, xv, s);
    } else if (cur.md->dtype == MAD_DTYPE_F32_MASTER) {
      load_full_typed<float, __nv_bfloat16>(cur, r);
      finish_full<float>(cur, r, xv, s);
    } else {
      load_full_typed<float, float>(cur, r);
      finish_full<float>(cur, r, xv, s);
    }
  } else {
    values_general_any<REDUCE>(cur, xv, s);
  }
  float ss = 0.f;
  write_x(cur, xv, ss, tile_t);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if (lane == 0) partials[tile * PREP_WARPS + warp] = ss;
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
  // One CTA per tile (a plan never has more than 2^31 - 1 prep tiles).
  const int grid = static_cast<int>(n_tiles);
  if (red.n > 0)
    muon_prep_kernel<true><<<grid, PREP_THREADS, 0, stream>>>(mats, prep_map, partials, n_tiles, s);
  else
    muon_prep_kernel<false><<<grid, PREP_THREADS, 0, stream>>>(mats, prep_map, partials, n_tiles, s);
  if (int rc = check_launch("muon_prep_kernel")) return rc;
  muon_norm_kernel<<<n_mats, FINALIZE_THREADS, 0, stream>>>(mats, partials, s.eps_bf16);
  return check_launch("muon_norm_kernel");
}

}  // namespace mad
