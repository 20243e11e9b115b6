// Muon prologue, one pass over every planned matrix (triton_muon.py:346-356):
//   mom = beta*mom + (1-beta)*g              (buffer updated in place, fp32 or bf16)
//   u   = g + beta*(mom - g)  if nesterov    (the buffer itself is untouched)
//   X   = bf16(u), transposed when rows > cols, so X is m x n with m <= n
//   s   = 1 / max(bf16(||X||_F), bf16(eps))  (the reference's bf16 norm)
// X is written unnormalised; s is folded into the first Gram and update
// epilogues.  The norm is reduced deterministically: every 64x64 tile writes
// its partial sum of squares, and the last tile of a matrix to finish (found
// with a per-matrix arrival counter, which it resets) adds the partials in a
// fixed order in double precision.
//
// Traffic per element: read g, mom (8 B), write mom (4 B) and X (2 B) with
// float32 buffers; 4 + 2 + 2 B with bf16 buffers.  With a gradient reduction
// the other ranks' gradient copies are read over NVLink as well.
#include <cuda_runtime.h>

#include "capi_common.h"
#include "elem_io.cuh"
#include "plan.cuh"
#include "ptx_sm100.cuh"

namespace mad {

constexpr int PREP_THREADS = 256;

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

// Momentum update of one 64x64 tile; xv receives the (Nesterov) update u for
// the thread's 4 rows x 4 consecutive columns, 0 outside the matrix.  TM is
// the momentum's type (bf16 momentum rounds the glue to bf16), TG the
// gradient's (a float32 master takes a bf16 gradient).
template <typename TM, typename TG, bool REDUCE>
__device__ __forceinline__ void prep_values(const MatDesc* md, int r0, int c0, bool full, float (&xv)[4][4],
                                            const PrepScalars& s) {
  constexpr bool BF16 = sizeof(TM) == 2;
  const int rows = md->rows, cols = md->cols, t = threadIdx.x;
  const TG* __restrict__ g = static_cast<const TG*>(md->g);
  TM* __restrict__ mom = static_cast<TM*>(md->mom);
  const int cl = (t & 15) * 4;  // 4 consecutive columns per thread
  if (full) {
    // All loads of the tile first (8 vectors in flight per thread), then compute and store.
    // Summed over ranks, each row's copies are in flight together, one row at a time.
    float4 gv[4], mv[4];
    if (REDUCE) {
      int64_t offs[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        offs[i] = static_cast<int64_t>(r0 + i * 16 + (t >> 4)) * cols + c0 + cl;
        mv[i] = ld4(mom + offs[i], 0);
      }
      ld4_ranks_rows<TG, 4>(g, offs, gv, s.red);
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int64_t off = static_cast<int64_t>(r0 + i * 16 + (t >> 4)) * cols + c0 + cl;
        gv[i] = ld4(g + off, 0);
        mv[i] = ld4(mom + off, 0);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t off = static_cast<int64_t>(r0 + i * 16 + (t >> 4)) * cols + c0 + cl;
      xv[i][0] = prep_update<BF16>(gv[i].x, mv[i].x, s);
      xv[i][1] = prep_update<BF16>(gv[i].y, mv[i].y, s);
      xv[i][2] = prep_update<BF16>(gv[i].z, mv[i].z, s);
      xv[i][3] = prep_update<BF16>(gv[i].w, mv[i].w, s);
      st4(mom + off, 0, mv[i]);
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int r = r0 + i * 16 + (t >> 4), c = c0 + cl;
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

// REDUCE: the gradient summed over ranks (a separate instantiation, so the
// local path keeps its register budget and occupancy).
template <bool REDUCE>
__global__ void __launch_bounds__(PREP_THREADS, REDUCE ? 2 : 4) muon_prep_kernel(MatDesc* __restrict__ mats,
                                                                 const int32_t* __restrict__ prep_map,
                                                                 float* __restrict__ partials, int64_t n_tiles,
                                                                 PrepScalars s) {
  __shared__ float tile_t[PREP_TILE][PREP_TILE + 1];
  __shared__ double red[PREP_THREADS / 32];
  __shared__ int is_last;
  const int t = threadIdx.x;
  const int lane = t & 31, warp = t >> 5;

  for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
    const int mi = prep_map[tile];
    MatDesc* md = mats + mi;
    const int rows = md->rows, cols = md->cols, ld_x = md->ld_x;
    const int transposed = md->transposed;
    const int local = static_cast<int>(tile - md->prep_begin);
    const int r0 = (local / md->prep_tiles_c) * PREP_TILE;
    const int c0 = (local % md->prep_tiles_c) * PREP_TILE;
    __nv_bfloat16* __restrict__ x = md->x[0];
    const bool full = md->vec != 0 && r0 + PREP_TILE <= rows && c0 + PREP_TILE <= cols;

    float ss = 0.f;
    const int cl = (t & 15) * 4;  // 4 consecutive columns per thread
    float xv[4][4];
    if (md->dtype == MAD_DTYPE_BF16)
      prep_values<__nv_bfloat16, __nv_bfloat16, REDUCE>(md, r0, c0, full, xv, s);
    else if (md->dtype == MAD_DTYPE_F32_MASTER)
      prep_values<float, __nv_bfloat16, REDUCE>(md, r0, c0, full, xv, s);
    else
      prep_values<float, float, REDUCE>(md, r0, c0, full, xv, s);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int rl = i * 16 + (t >> 4);
      const int r = r0 + rl, c = c0 + cl;
      __nv_bfloat16 xb[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        xb[k] = __float2bfloat16_rn(xv[i][k]);
        const float q = __bfloat162float(xb[k]);
        ss = fmaf(q, q, ss);
      }
      if (!transposed) {
        if (r < rows) {
          __nv_bfloat16* dst = x + static_cast<int64_t>(r) * ld_x + c;
          if (c + 4 <= cols) {
            uint2 packed;
            packed.x = static_cast<uint32_t>(__bfloat16_as_ushort(xb[0])) |
                       (static_cast<uint32_t>(__bfloat16_as_ushort(xb[1])) << 16);
            packed.y = static_cast<uint32_t>(__bfloat16_as_ushort(xb[2])) |
                       (static_cast<uint32_t>(__bfloat16_as_ushort(xb[3])) << 16);
            *reinterpret_cast<uint2*>(dst) = packed;
          } else {
            for (int k = 0; k < 4 && c + k < cols; ++k) dst[k] = xb[k];
          }
        }
      } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) tile_t[cl + k][rl] = __bfloat162float(xb[k]);
      }
    }

    if (transposed) {
      __syncthreads();
      // X row = parameter column, X column = parameter row.
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int xr = i * 16 + (t >> 4);
        const int xc = (t & 15) * 4;
        const int row = c0 + xr, col = r0 + xc;
        if (row < cols) {
          __nv_bfloat16* dst = x + static_cast<int64_t>(row) * ld_x + col;
          if (col + 4 <= rows) {
            uint2 packed;
            packed.x = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(tile_t[xr][xc + 0]))) |
                       (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(tile_t[xr][xc + 1]))) << 16);
            packed.y = static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(tile_t[xr][xc + 2]))) |
                       (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(tile_t[xr][xc + 3]))) << 16);
            *reinterpret_cast<uint2*>(dst) = packed;
          } else {
            for (int k = 0; k < 4 && col + k < rows; ++k) dst[k] = __float2bfloat16_rn(tile_t[xr][xc + k]);
          }
        }
      }
    }

    // Block sum of squares -> this tile's partial.
    float w = ss;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) w += __shfl_xor_sync(0xffffffffu, w, o);
    if (lane == 0) red[warp] = w;
    __syncthreads();
    if (t == 0) {
      float tot = 0.f;
      for (int k = 0; k < PREP_THREADS / 32; ++k) tot += static_cast<float>(red[k]);
      partials[tile] = tot;
      __threadfence();
      const unsigned prev = atomicAdd(&md->done, 1u);
      is_last = (prev == static_cast<unsigned>(md->prep_count) - 1u);
    }
    __syncthreads();
    if (is_last) {
      __threadfence();
      double acc = 0.0;
      const int begin = md->prep_begin, count = md->prep_count;
      for (int k = t; k < count; k += PREP_THREADS) acc += static_cast<double>(__ldcg(partials + begin + k));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0) red[warp] = acc;
      __syncthreads();
      if (t == 0) {
        double tot = 0.0;
        for (int k = 0; k < PREP_THREADS / 32; ++k) tot += red[k];
        float norm = bf16_round(static_cast<float>(sqrt(tot)));
        if (!(norm >= s.eps_bf16)) norm = (norm != norm) ? norm : s.eps_bf16;  // clamp(min=eps), NaN kept
        md->inv_norm = 1.0f / norm;
        md->done = 0u;
      }
    }
    __syncthreads();
  }
}

int launch_muon_prep(MatDesc* mats, const int32_t* prep_map, float* partials, int64_t n_tiles, double beta,
                     int nesterov, float eps, const GradReduce& red, cudaStream_t stream) {
  if (n_tiles <= 0) return MAD_OK;
  PrepScalars s;
  s.red = red;
  // The reference passes Python floats: beta is rounded to float32 by the
  // multiply, alpha = 1 - beta is formed in double and then rounded.
  s.beta = static_cast<float>(beta);
  s.one_m_beta = static_cast<float>(1.0 - beta);
  s.eps_bf16 = bf16_round(eps);
  s.nesterov = nesterov ? 1 : 0;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 8;
  const int grid = static_cast<int>(n_tiles < cap ? n_tiles : cap);
  if (red.n > 0)
    muon_prep_kernel<true><<<grid, PREP_THREADS, 0, stream>>>(mats, prep_map, partials, n_tiles, s);
  else
    muon_prep_kernel<false><<<grid, PREP_THREADS, 0, stream>>>(mats, prep_map, partials, n_tiles, s);
  return check_launch("muon_prep_kernel");
}

}  // namespace mad
