// Newton-Schulz GEMMs on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// One persistent, warp-specialised kernel template serves the three products of
// an iteration (triton_muon.py:313-325), each launched once over the tiles of
// ALL planned matrices:
//
//   GRAM   A  = bf16(s² · X Xᵀ)        m x m, K = n   (ns_kernel_1, triton_muon.py:35-93)
//   POLY   B  = bf16(b A + c · A A)    m x m, K = m   (ns_kernel_2, triton_muon.py:119-188)
//   UPDATE X' = bf16(s (a X + B X))    m x n, K = m   (ns_kernel_3, triton_muon.py:215-278)
//
// s = 1/||X||_F on iteration 0 (prep writes X unnormalised) and 1 afterwards.
// GRAM and POLY outputs are symmetric: only tiles touching the upper triangle
// are computed, and every strictly-upper 128x128 block is also stored
// transposed.  On the last iteration UPDATE writes the fp32 parameter instead
// of X' (triton_muon.py:365-372): p -= (lr·wd)·p ; p -= scaled_lr·bf16(X'),
// transposed back for tall matrices.
//
// CTA tile 128 x 256, K step 64 (one 128-byte swizzle atom of bf16), 4-stage
// TMA ring (48 KB/stage), accumulators double-buffered in TMEM (2 x 256 of
// the 512 columns) so the epilogue of tile i overlaps the MMAs of tile i+1.
// Warp 0 issues TMA, warp 1 issues tcgen05.mma (one thread), warps 2-5 drain
// TMEM (one accumulator row per thread).  Operands: X Xᵀ and A A read two
// K-major tiles; B X reads B K-major and X MN-major (its rows are the K index).
#include <cuda_runtime.h>

#include "capi_common.h"
#include "plan.cuh"
#include "ptx_sm100.cuh"

namespace mad {
namespace ns {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_BYTES = BN * BK * 2;  // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int TMEM_COLS = 2 * BN;
constexpr int NUM_THREADS = 192;
constexpr int EPI_THREADS = 128;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 1024;  // ring + barriers + alignment slack

enum Mode { GRAM = 0, POLY = 1, UPDATE = 2 };

struct GemmArgs {
  const MatDesc* mats;
  const CUtensorMap* tmaps;
  const TileRef* tiles;
  int n_tiles;
  int iter;
  int last;
  float a, b, c;
  float lr_wd;
  double lr;
  unsigned int* status;
};

__device__ __forceinline__ int k_extent(int mode, const MatDesc& md) { return mode == GRAM ? md.n : md.m; }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  return static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(lo))) |
         (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(hi))) << 16);
}

// 32 consecutive bf16 (64 bytes, 16-byte aligned) -> float.
__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16* src, float (&out)[32]) {
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 u = s4[q];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      out[q * 8 + 2 * k] = __bfloat162float(__ushort_as_bfloat16(static_cast<unsigned short>(w[k] & 0xFFFFu)));
      out[q * 8 + 2 * k + 1] = __bfloat162float(__ushort_as_bfloat16(static_cast<unsigned short>(w[k] >> 16)));
    }
  }
}

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const float (&v)[32]) {
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 u;
    u.x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
    u.y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
    u.z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
    u.w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
    d4[q] = u;
  }
}

template <int MODE>
__device__ __forceinline__ void producer_loop(const GemmArgs& args, uint8_t* ring, uint64_t* full, uint64_t* empty,
                                              volatile int* abort_flag) {
  int stage = 0, issued = 0;
  uint32_t phase = 0;
  const int cur = args.iter & 1;
  bool ok = true;
  for (int t = blockIdx.x; t < args.n_tiles && ok; t += gridDim.x) {
    const TileRef tr = args.tiles[t];
    const MatDesc& md = args.mats[tr.mat];
    const CUtensorMap* maps = args.tmaps + md.tmap_base;
    const CUtensorMap* tmA;
    const CUtensorMap* tmB;
    if (MODE == GRAM) {
      tmA = tmB = maps + (TM_XK0 + cur);
    } else if (MODE == POLY) {
      tmA = tmB = maps + TM_GRAM;
    } else {
      tmA = maps + TM_POLY;
      tmB = maps + (TM_XMN0 + cur);
    }
    tma_acquire_desc(tmA);
    if (tmB != tmA) tma_acquire_desc(tmB);
    const int nkb = (k_extent(MODE, md) + BK - 1) / BK;
    for (int kb = 0; kb < nkb; ++kb) {
      if (!mbar_wait(&empty[stage], phase ^ 1u, args.status, DEV_ERR_MBAR_TIMEOUT_PRODUCER) || *abort_flag) {
        *abort_flag = 1;
        ok = false;
        break;
      }
      uint8_t* sa = ring + stage * STAGE_BYTES;
      uint8_t* sb = sa + A_BYTES;
      mbar_arrive_expect_tx(&full[stage], STAGE_BYTES);
      tma_load_2d(sa, tmA, &full[stage], kb * BK, tr.tm * BM);
      if (MODE == UPDATE) {
#pragma unroll
        for (int j = 0; j < BN / 64; ++j) tma_load_2d(sb + j * (64 * BK * 2), tmB, &full[stage], tr.tn * BN + j * 64, kb * BK);
      } else {
        tma_load_2d(sb, tmB, &full[stage], kb * BK, tr.tn * BN);
        tma_load_2d(sb + BM * BK * 2, tmB, &full[stage], kb * BK, tr.tn * BN + BM);
      }
      ++issued;
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
  }
  // Make sure no copy into this CTA's shared memory is still in flight when it
  // exits (only possible after an abort): wait for the last fills to land.
  for (int j = issued > STAGES ? issued - STAGES : 0; j < issued; ++j)
    mbar_wait(&full[j % STAGES], static_cast<uint32_t>((j / STAGES) & 1), args.status, DEV_ERR_MBAR_TIMEOUT_DRAIN);
}

template <int MODE>
__device__ __forceinline__ void mma_loop(const GemmArgs& args, uint8_t* ring, uint64_t* full, uint64_t* empty,
                                         uint64_t* tfull, uint64_t* tempty, uint64_t* drain, uint32_t tmem_base,
                                         volatile int* abort_flag) {
  constexpr uint32_t IDESC = idesc_bf16_f32(BM, BN, false, MODE == UPDATE);
  int stage = 0, lt = 0;
  uint32_t phase = 0;
  bool ok = true;
  for (int t = blockIdx.x; t < args.n_tiles && ok; t += gridDim.x, ++lt) {
    const TileRef tr = args.tiles[t];
    const MatDesc& md = args.mats[tr.mat];
    const int nkb = (k_extent(MODE, md) + BK - 1) / BK;
    const int acc = lt & 1;
    const uint32_t acc_phase = static_cast<uint32_t>((lt >> 1) & 1);
    if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, args.status, DEV_ERR_MBAR_TIMEOUT_MMA) || *abort_flag) {
      *abort_flag = 1;
      break;
    }
    tc_fence_after();
    const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
    for (int kb = 0; kb < nkb; ++kb) {
      if (!mbar_wait(&full[stage], phase, args.status, DEV_ERR_MBAR_TIMEOUT_MMA) || *abort_flag) {
        *abort_flag = 1;
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t sa = smem_u32(ring + stage * STAGE_BYTES);
      const uint32_t sb = sa + A_BYTES;
#pragma unroll
      for (int kk = 0; kk < BK / 16; ++kk) {
        const uint64_t ad = smem_desc_sw128(sa + kk * 32, 16, 1024);
        const uint64_t bd = (MODE == UPDATE) ? smem_desc_sw128(sb + kk * 2048, 64 * BK * 2, 1024)
                                             : smem_desc_sw128(sb + kk * 32, 16, 1024);
        tc_mma_bf16(d_tmem, ad, bd, IDESC, (kb | kk) != 0 ? 1u : 0u);
      }
      tc_commit(&empty[stage]);
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
    if (ok) tc_commit(&tfull[acc]);
  }
  // Every MMA this thread issued must finish before TMEM is released.
  tc_commit(drain);
  mbar_wait(drain, 0u, args.status, DEV_ERR_MBAR_TIMEOUT_DRAIN);
}

template <int MODE>
__device__ __forceinline__ void epilogue_loop(const GemmArgs& args, uint64_t* tfull, uint64_t* tempty,
                                              uint32_t tmem_base, volatile int* abort_flag) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quad = warp & 3;  // TMEM lanes this warp may access: 32*quad .. 32*quad+31
  const int row_in_tile = quad * 32 + lane;
  const int cur = args.iter & 1;
  int lt = 0;
  for (int t = blockIdx.x; t < args.n_tiles; t += gridDim.x, ++lt) {
    const TileRef tr = args.tiles[t];
    const MatDesc& md = args.mats[tr.mat];
    const int acc = lt & 1;
    const uint32_t acc_phase = static_cast<uint32_t>((lt >> 1) & 1);
    if (!mbar_wait(&tfull[acc], acc_phase, args.status, DEV_ERR_MBAR_TIMEOUT_EPILOGUE) || *abort_flag) {
      *abort_flag = 1;
      break;
    }
    tc_fence_after();
    const int m = md.m;
    const int grow = tr.tm * BM + row_in_tile;
    const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + static_cast<uint32_t>(acc * BN);

    if (MODE == GRAM || MODE == POLY) {
      const float s2 = (MODE == GRAM && args.iter == 0) ? md.inv_norm * md.inv_norm : 1.0f;
      __nv_bfloat16* out = (MODE == GRAM) ? md.gram : md.poly;
      const __nv_bfloat16* ain = md.gram;
      const int ld = md.ld_mm;
#pragma unroll 1
      for (int ch = 0; ch < BN / 32; ++ch) {
        const int gcol0 = tr.tn * BN + ch * 32;
        const int jblk = gcol0 / BM;
        if (jblk < tr.tm || gcol0 >= m) continue;  // below the diagonal, or past the matrix
        float v[32];
        tmem_ld_32cols(tbase + ch * 32, v);
        if (grow < m) {
          if (MODE == GRAM) {
#pragma unroll
            for (int k = 0; k < 32; ++k) v[k] *= s2;
          } else {
            float av[32];
            load_bf16x32(ain + static_cast<int64_t>(grow) * ld + gcol0, av);
#pragma unroll
            for (int k = 0; k < 32; ++k) v[k] = __fadd_rn(__fmul_rn(args.b, av[k]), __fmul_rn(args.c, v[k]));
          }
          store_bf16x32(out + static_cast<int64_t>(grow) * ld + gcol0, v);
          if (jblk > tr.tm) {
            // Mirror: element (grow, col) also lands at (col, grow).
#pragma unroll
            for (int k = 0; k < 32; ++k) {
              const int col = gcol0 + k;
              if (col < m) out[static_cast<int64_t>(col) * ld + grow] = __float2bfloat16_rn(v[k]);
            }
          }
        }
      }
    } else {  // UPDATE
      const float s = (args.iter == 0) ? md.inv_norm : 1.0f;
      const int n = md.n, ld = md.ld_x;
      const __nv_bfloat16* xin = md.x[cur];
      __nv_bfloat16* xout = md.x[cur ^ 1];
#pragma unroll 1
      for (int ch = 0; ch < BN / 32; ++ch) {
        const int gcol0 = tr.tn * BN + ch * 32;
        if (gcol0 >= n) break;
        float v[32];
        tmem_ld_32cols(tbase + ch * 32, v);
        if (grow < m) {
          float xv[32];
          load_bf16x32(xin + static_cast<int64_t>(grow) * ld + gcol0, xv);
#pragma unroll
          for (int k = 0; k < 32; ++k) v[k] = __fmul_rn(s, __fadd_rn(__fmul_rn(args.a, xv[k]), v[k]));
          if (!args.last) {
            store_bf16x32(xout + static_cast<int64_t>(grow) * ld + gcol0, v);
          } else {
            // scaled_lr = lr * shape factor, formed in double and rounded once (triton_muon.py:424-431).
            const float slr = static_cast<float>(args.lr * md.lr_scale), lr_wd = args.lr_wd;
            float* __restrict__ p = md.p;
            if (!md.transposed) {
              // X' row grow is parameter row grow (parameter is m x n).
              float* prow = p + static_cast<int64_t>(grow) * n + gcol0;
              if (md.vec && gcol0 + 32 <= n) {
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                  float4 pv = reinterpret_cast<float4*>(prow)[q];
                  float* e = reinterpret_cast<float*>(&pv);
#pragma unroll
                  for (int k = 0; k < 4; ++k) {
                    const float o = bf16_round(v[q * 4 + k]);
                    const float p1 = __fsub_rn(e[k], __fmul_rn(lr_wd, e[k]));
                    e[k] = __fsub_rn(p1, __fmul_rn(slr, o));
                  }
                  reinterpret_cast<float4*>(prow)[q] = pv;
                }
              } else {
                for (int k = 0; k < 32 && gcol0 + k < n; ++k) {
                  const float o = bf16_round(v[k]);
                  const float p1 = __fsub_rn(prow[k], __fmul_rn(lr_wd, prow[k]));
                  prow[k] = __fsub_rn(p1, __fmul_rn(slr, o));
                }
              }
            } else {
              // Parameter is n x m; X'[grow][col] is p[col][grow]: lanes write consecutive grow.
#pragma unroll 4
              for (int k = 0; k < 32; ++k) {
                const int col = gcol0 + k;
                if (col < n) {
                  float* pe = p + static_cast<int64_t>(col) * m + grow;
                  const float o = bf16_round(v[k]);
                  const float p1 = __fsub_rn(*pe, __fmul_rn(lr_wd, *pe));
                  *pe = __fsub_rn(p1, __fmul_rn(slr, o));
                }
              }
            }
          }
        }
      }
    }
    tc_fence_before();
    mbar_arrive(&tempty[acc]);
  }
}

template <int MODE>
__global__ void __launch_bounds__(NUM_THREADS, 1) ns_gemm_kernel(const __grid_constant__ GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], EPI_THREADS);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) producer_loop<MODE>(args, ring, full, empty, abort_flag);
  } else if (warp == 1) {
    if (lane == 0) mma_loop<MODE>(args, ring, full, empty, tfull, tempty, drain, tmem_base, abort_flag);
  } else {
    epilogue_loop<MODE>(args, tfull, tempty, tmem_base, abort_flag);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

template <int MODE>
static int launch(const GemmArgs& args, cudaStream_t stream, const char* name) {
  if (args.n_tiles <= 0) return MAD_OK;
  if (cudaFuncSetAttribute(ns_gemm_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
      cudaSuccess)
    return fail_cuda("cudaFuncSetAttribute(ns_gemm_kernel)");
  const int grid = args.n_tiles < num_sms() ? args.n_tiles : num_sms();
  ns_gemm_kernel<MODE><<<grid, NUM_THREADS, SMEM_BYTES, stream>>>(args);
  return check_launch(name);
}

}  // namespace ns

int launch_ns_gemm(int mode, const MatDesc* mats, const CUtensorMap* tmaps, const TileRef* tiles, int64_t n_tiles,
                   int iter, int last, float a, float b, float c, double lr, float lr_wd, unsigned int* status,
                   cudaStream_t stream) {
  ns::GemmArgs args;
  args.mats = mats;
  args.tmaps = tmaps;
  args.tiles = tiles;
  args.n_tiles = static_cast<int>(n_tiles);
  args.iter = iter;
  args.last = last;
  args.a = a;
  args.b = b;
  args.c = c;
  args.lr_wd = lr_wd;
  args.lr = lr;
  args.status = status;
  switch (mode) {
    case ns::GRAM:
      return ns::launch<ns::GRAM>(args, stream, "ns_gemm_kernel<GRAM>");
    case ns::POLY:
      return ns::launch<ns::POLY>(args, stream, "ns_gemm_kernel<POLY>");
    default:
      return ns::launch<ns::UPDATE>(args, stream, "ns_gemm_kernel<UPDATE>");
  }
}

}  // namespace mad
