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
// transposed.  On the last iteration UPDATE writes the parameter (float32 or
// bf16) instead of X' (triton_muon.py:365-372): p -= (lr·wd)·p ; p -= scaled_lr·bf16(X'),
// transposed back for tall matrices.
//
// CTA pairs (clusters of 2) compute 256 x 256 tiles with tcgen05.mma.cta_group::2:
// each CTA loads its own 128 rows of the A operand and half (128 columns) of
// the B operand per K step of 64, so an SM moves 32 KB per step instead of
// the 48 KB a single-CTA 128 x 256 tile needs -- a third less operand traffic
// per flop, with no multicast load anywhere.  6-stage TMA ring per CTA;
// accumulators (each CTA: its 128 rows x 256 columns) double-buffered in TMEM
// so the epilogue of tile i overlaps the MMAs of tile i+1.  Warp 0 issues TMA
// (both CTAs; completion counted on the leader's barrier), warp 1 of the
// leader issues the pair MMAs (one thread), warps 2-9 of both CTAs drain TMEM
// (one accumulator row and half the columns per thread).  Operands: X Xᵀ and
// A A read two K-major tiles; B X reads B K-major and X MN-major (its rows are
// the K index).
//
// Tiles are handed out dynamically: the leader's producer thread takes the
// next tile index from a counter in the plan header (one atomic per tile) and
// publishes it to both CTAs of its pair through a small ring in shared
// memory, so a pair that starts late -- its SMs held by a kernel running
// beside the GEMM, such as a collective -- takes fewer tiles instead of
// finishing its share after everyone else.  Tile results do not depend on
// which pair computes them.
#include <cuda_runtime.h>

#include <atomic>
#include <cstddef>

#include "capi_common.h"
#include "elem_io.cuh"
#include "plan.cuh"
#include "ptx_sm100.cuh"

namespace mad {
namespace ns {

constexpr int BM = 128, BN = 256, BK = 64, MAX_STAGES = 6;
constexpr int PAIR_M = 2 * BM;          // rows of a pair tile
constexpr int A_BYTES = BM * BK * 2;    // 16 KB: this CTA's 128 rows of A
constexpr int B_BYTES = (BN / 2) * BK * 2;  // 16 KB: this CTA's 128 columns of B
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr uint32_t PAIR_TX_BYTES = 2 * STAGE_BYTES;  // both CTAs' fills, counted on the leader's barrier
constexpr int TMEM_COLS = 2 * BN;
constexpr int EPI_WARPS = 8;
constexpr int EPI_THREADS = EPI_WARPS * 32;
constexpr int NUM_THREADS = 64 + EPI_THREADS;  // producer warp, MMA warp, epilogue warps
enum Mode { GRAM = 0, POLY = 1, UPDATE = 2, UPDATE_LAST = 3 };

// Shared memory per mode.  Each epilogue warp has a staging area: GRAM/POLY
// stage their 32x32 output block and its transposed mirror (2 x 2 KB), UPDATE
// its output block and the X block of the a*X term (2 x 2 KB).  UPDATE_LAST
// also moves the parameter block (a 32x32 box, 4 KB float32) and the bf16
// shadow by TMA: 8 KB per warp, paid for with one ring stage fewer.
template <int MODE>
struct Smem {
  static constexpr int STAGES = MODE == UPDATE_LAST ? 5 : 6;
  static constexpr int STAGE_OUT = MODE == UPDATE_LAST ? 8192 : 4096;
  static constexpr int BYTES = STAGES * STAGE_BYTES + EPI_WARPS * STAGE_OUT + 1024 + 1024;  // + barriers, alignment
};
static_assert(Smem<GRAM>::BYTES <= 227 * 1024 && Smem<UPDATE_LAST>::BYTES <= 227 * 1024, "shared memory per CTA");
// Offsets inside a warp's staging area: the X block of the update kernels'
// a*X term, and UPDATE_LAST's bf16 shadow and parameter blocks.
constexpr int X_IN_OFF = 2048, LAST_SHADOW_OFF = 0, LAST_P_OFF = 4096;
static_assert(X_IN_OFF + 2048 <= LAST_P_OFF && LAST_SHADOW_OFF + 2048 <= X_IN_OFF, "staging areas overlap");

// UPDATE_LAST is the update of the final iteration, which writes the
// parameters; it is a separate instantiation so the common path can keep two
// chunks in flight without exceeding the register budget (168 per thread with
// ten warps).
template <int MODE>
__host__ __device__ constexpr bool is_update() { return MODE == UPDATE || MODE == UPDATE_LAST; }

struct GemmArgs {
  const MatDesc* mats;
  const CUtensorMap* tmaps;
  const TileRef* tiles;
  int n_tiles;
  int iter;
  float a, b, c;
  float lr_wd;
  double lr;
  unsigned int* status;
  int32_t* sched;        // {next tile, retired pairs}: zero at launch, reset by the last pair
  long long wait_limit;  // SM cycles before a barrier wait gives up
  int idle_producer;     // test launches only: the producer issues no loads, so the waits expire
};


// ---------------------------------------------------------------- tile scheduler
// Ring of tile indices, one copy in each CTA of the pair.  Entry j is written
// by the leader's producer (a tile index, or -1 when none is left, and the
// tile's K-block count) and read by every other role of the pair: the leader's
// MMA thread and epilogue warps, the peer's producer and epilogue warps.  Each
// reader arrives on the leader's `empty` barrier of the entry; the producer
// reuses it after all of them.  The MMA thread needs nothing else of a tile,
// so it issues the next tile's MMAs without a global-memory round trip.
constexpr int SCHED_DEPTH = 8;
constexpr uint32_t SCHED_READERS = 1 + EPI_WARPS + 1 + EPI_WARPS;

struct Sched {
  int32_t* slot;     // [SCHED_DEPTH] tile index
  int32_t* kblk;     // [SCHED_DEPTH] its TileRef::nkb
  uint64_t* full;    // [SCHED_DEPTH], one arrival (the leader's producer)
  uint64_t* empty;   // [SCHED_DEPTH], SCHED_READERS arrivals; only the leader's are used
};

// Leader producer: takes the next tile, reads its TileRef and publishes both as
// entry j.  False if the entry's previous readers did not release it in time.
__device__ __forceinline__ bool sched_publish(const GemmArgs& args, const Sched& sc, int j, int* tile, TileRef* tr) {
  const int s = j % SCHED_DEPTH;
  const uint32_t ph = static_cast<uint32_t>((j / SCHED_DEPTH) & 1);
  if (!mbar_wait_cluster(&sc.empty[s], ph ^ 1u, args.status, DEV_ERR_MBAR_TIMEOUT_PRODUCER, args.wait_limit))
    return false;
  int t = atomicAdd(&args.sched[0], 1);
  int nkb = 0;
  if (t >= args.n_tiles) {
    t = -1;
  } else {
    *tr = args.tiles[t];
    nkb = tr->nkb;
  }
  sc.slot[s] = t;
  sc.kblk[s] = nkb;
  st_shared_cluster_u32(mapa_shared(smem_u32(&sc.slot[s]), 1), t);
  st_shared_cluster_u32(mapa_shared(smem_u32(&sc.kblk[s]), 1), nkb);
  mbar_arrive(&sc.full[s]);
  mbar_arrive_cluster(mapa_shared(smem_u32(&sc.full[s]), 1));
  *tile = t;
  return true;
}

// Any other role: waits for entry j and reads it (every lane of a warp may
// call this; `release` then runs on one lane after the warp has read it).
__device__ __forceinline__ bool sched_take(const GemmArgs& args, const Sched& sc, int j, unsigned int err_bit,
                                           int* tile, int* nkb = nullptr) {
  const int s = j % SCHED_DEPTH;
  const uint32_t ph = static_cast<uint32_t>((j / SCHED_DEPTH) & 1);
  if (!mbar_wait_cluster(&sc.full[s], ph, args.status, err_bit, args.wait_limit)) return false;
  *tile = *reinterpret_cast<volatile int32_t*>(&sc.slot[s]);
  if (nkb) *nkb = *reinterpret_cast<volatile int32_t*>(&sc.kblk[s]);
  return true;
}

__device__ __forceinline__ void sched_release(const Sched& sc, int j) {
  mbar_arrive_cluster(mapa_shared(smem_u32(&sc.empty[j % SCHED_DEPTH]), 0));
}

// Leader producer, once per launch on every path: the last pair to finish
// taking tiles resets the counter for the next launch on the stream.
__device__ __forceinline__ void sched_retire(const GemmArgs& args) {
  __threadfence();
  const int done = atomicAdd(&args.sched[1], 1);
  if (done == static_cast<int>(gridDim.x >> 1) - 1) {
    __threadfence();
    atomicExch(&args.sched[0], 0);
    atomicExch(&args.sched[1], 0);
  }
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  return static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(lo))) |
         (static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(hi))) << 16);
}

template <int MODE>
__device__ __forceinline__ void producer_loop(const GemmArgs& args, uint8_t* ring, uint64_t* full, uint64_t* empty,
                                              const Sched& sc, uint32_t rank, volatile int* abort_flag) {
  int stage = 0;
  uint32_t phase = 0;
  const int cur = args.iter & 1;
  if (args.idle_producer) {
    // Test launches: one tile is handed out and nothing is loaded, so the
    // MMA and epilogue waits of that tile expire.
    int t;
    TileRef tr;
    if (rank == 0) {
      sched_publish(args, sc, 0, &t, &tr);
      sched_retire(args);
    }
    return;
  }
  bool ok = true;
  int acquired = -1;  // matrix whose tensor maps this thread has acquired
  for (int j = 0; ok; ++j) {
    int t;
    TileRef tr;
    if (rank == 0) {
      if (!sched_publish(args, sc, j, &t, &tr)) {
        *abort_flag = 1;
        break;
      }
    } else {
      if (!sched_take(args, sc, j, DEV_ERR_MBAR_TIMEOUT_PRODUCER, &t)) {
        *abort_flag = 1;
        break;
      }
      sched_release(sc, j);
      if (t >= 0) tr = args.tiles[t];
    }
    if (t < 0) break;
    const CUtensorMap* maps = args.tmaps + tr.mat * TMAPS_PER_MAT;
    const CUtensorMap* tmA;
    const CUtensorMap* tmB;
    if (MODE == GRAM) {
      tmA = tmB = maps + (TM_XK0 + cur);
    } else if (MODE == POLY) {
      tmA = tmB = maps + TM_GRAM;
    } else {  // UPDATE, UPDATE_LAST
      tmA = maps + TM_POLY;
      tmB = maps + (TM_XMN0 + cur);
    }
    if (tr.mat != acquired) {  // once per matrix: later uses by this thread are ordered after it
      tma_acquire_desc(tmA);
      if (tmB != tmA) tma_acquire_desc(tmB);
      acquired = tr.mat;
    }
    const int arow = tr.tm * PAIR_M + static_cast<int>(rank) * BM;     // this CTA's A rows
    const int bcol = tr.tn * BN + static_cast<int>(rank) * (BN / 2);   // this CTA's B columns
    const int nkb = tr.nkb;
    for (int kb = 0; kb < nkb; ++kb) {
      if (!mbar_wait(&empty[stage], phase ^ 1u, args.status, DEV_ERR_MBAR_TIMEOUT_PRODUCER, args.wait_limit) ||
          *abort_flag) {
        *abort_flag = 1;
        ok = false;
        break;
      }
      uint8_t* sa = ring + stage * STAGE_BYTES;
      uint8_t* sb = sa + A_BYTES;
      // Both CTAs' fills complete on the leader's barrier; the leader arms it for both.
      const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
      if (rank == 0) mbar_arrive_expect_tx(&full[stage], PAIR_TX_BYTES);
      tma_load_2d_pair(sa, tmA, bar, kb * BK, arow);
      if (is_update<MODE>()) {
        tma_load_2d_pair(sb, tmB, bar, bcol, kb * BK);
        tma_load_2d_pair(sb + 64 * BK * 2, tmB, bar, bcol + 64, kb * BK);
      } else {
        tma_load_2d_pair(sb, tmB, bar, kb * BK, bcol);
      }
      if (++stage == Smem<MODE>::STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
  }
  if (rank == 0) sched_retire(args);
}

// Leader CTA only: one thread issues the pair MMAs and returns each smem stage
// and each finished accumulator to both CTAs (two commits, one per CTA).
template <int MODE>
__device__ __forceinline__ void mma_loop(const GemmArgs& args, uint8_t* ring, uint64_t* full, uint64_t* empty,
                                         uint64_t* tfull, uint64_t* tempty, uint64_t* drain, uint32_t tmem_base,
                                         const Sched& sc, volatile int* abort_flag) {
  constexpr uint32_t IDESC = idesc_bf16_f32(PAIR_M, BN, false, is_update<MODE>());
  int stage = 0;
  uint32_t phase = 0;
  bool ok = true;
  for (int lt = 0; ok; ++lt) {
    int t, nkb;
    if (!sched_take(args, sc, lt, DEV_ERR_MBAR_TIMEOUT_MMA, &t, &nkb)) {
      *abort_flag = 1;
      break;
    }
    sched_release(sc, lt);
    if (t < 0) break;
    const int acc = lt & 1;
    const uint32_t acc_phase = static_cast<uint32_t>((lt >> 1) & 1);
    if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, args.status, DEV_ERR_MBAR_TIMEOUT_MMA, args.wait_limit) ||
        *abort_flag) {
      *abort_flag = 1;
      break;
    }
    tc_fence_after();
    const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
    for (int kb = 0; kb < nkb; ++kb) {
      if (!mbar_wait(&full[stage], phase, args.status, DEV_ERR_MBAR_TIMEOUT_MMA, args.wait_limit) || *abort_flag) {
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
        const uint64_t bd = is_update<MODE>() ? smem_desc_sw128(sb + kk * 2048, 64 * BK * 2, 1024)
                                              : smem_desc_sw128(sb + kk * 32, 16, 1024);
        tc_mma_bf16_pair(d_tmem, ad, bd, IDESC, (kb | kk) != 0 ? 1u : 0u);
      }
      const uint32_t e = smem_u32(&empty[stage]);
      tc_commit_pair(mapa_shared(e, 0));
      tc_commit_pair(mapa_shared(e, 1));
      if (++stage == Smem<MODE>::STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
    if (ok) {
      const uint32_t f = smem_u32(&tfull[acc]);
      tc_commit_pair(mapa_shared(f, 0));
      tc_commit_pair(mapa_shared(f, 1));
    }
  }
  // Every MMA this thread issued must finish before TMEM is released.
  tc_commit_pair(mapa_shared(smem_u32(drain), 0));
  mbar_wait(drain, 0u, args.status, DEV_ERR_MBAR_TIMEOUT_DRAIN);
}

// Global input one epilogue chunk (32 columns of one accumulator row) reads
// ahead of time: the bf16 row segment of A (POLY) or X (UPDATE).
struct ChunkIn {
  uint4 q[4];  // 32 bf16
};

template <int MODE>
__device__ __forceinline__ void chunk_prefetch(const GemmArgs& args, const MatDesc& md, int grow, int gcol0,
                                               ChunkIn& in) {
  if (MODE == GRAM) return;
  const __nv_bfloat16* src = (MODE == POLY) ? md.gram : md.x[args.iter & 1];
  const int ld = (MODE == POLY) ? md.ld_mm : md.ld_x;
  const uint4* s4 = reinterpret_cast<const uint4*>(src + static_cast<int64_t>(grow) * ld + gcol0);
#pragma unroll
  for (int q = 0; q < 4; ++q) in.q[q] = s4[q];
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr)
               : "memory");
  return v;
}

// Update kernels fetch the epilogue's X block with TMA instead of per-thread
// loads: lane 0 loads the warp's 32 rows x 32 columns (2 KB, 64-byte swizzle)
// into the second half of the warp's staging buffer (the half the mirror
// block uses in the symmetric kernels).  Per-thread 16-byte loads of 32
// different rows cost ~12% of tensor throughput per clock and, together with
// the output stores, pushed the kernel into the power cap.
__device__ __forceinline__ void in_issue(uint8_t* stage, uint64_t* bar, const CUtensorMap* map, int x, int y) {
  if ((threadIdx.x & 31) == 0) {
    mbar_arrive_expect_tx(bar, 2048);
    tma_load_2d(stage + X_IN_OFF, map, bar, x, y);
  }
}

// Waits for the block and copies this lane's row (32 bf16) into registers;
// after the warp-wide sync the buffer may be refilled.
__device__ __forceinline__ void in_take(uint8_t* stage, uint64_t* bar, uint32_t& phase, uint4 (&q)[4],
                                        unsigned int* status, volatile int* abort_flag) {
  if (!mbar_wait(bar, phase, status, DEV_ERR_MBAR_TIMEOUT_EPILOGUE)) *abort_flag = 1;
  phase ^= 1u;
  const int lane = threadIdx.x & 31;
  const uint32_t base = smem_u32(stage + X_IN_OFF);
#pragma unroll
  for (int j = 0; j < 4; ++j) q[j] = ld_shared_v4(base + static_cast<uint32_t>(lane * 64 + 16 * (j ^ ((lane >> 1) & 3))));
  // These generic-proxy reads must be ordered before the next TMA (async-proxy)
  // write into the buffer, which lane 0 issues after the warp sync.
  fence_proxy_async_smem();
  __syncwarp();
}

__device__ __forceinline__ float bf16_at(const uint4 (&q)[4], int k) {
  const uint4& u = q[k >> 3];
  const uint32_t w = ((k >> 1) & 3) == 0 ? u.x : ((k >> 1) & 3) == 1 ? u.y : ((k >> 1) & 3) == 2 ? u.z : u.w;
  return __bfloat162float(__ushort_as_bfloat16(static_cast<unsigned short>((k & 1) ? (w >> 16) : (w & 0xFFFFu))));
}

// Shared-memory address of 16-byte unit `j` of row `r` in a 32-row x 64-byte
// block under the TMA 64-byte swizzle (16-byte units XOR'ed with bits 7-8).
__device__ __forceinline__ uint32_t sw64_offset(int r, int j) { return r * 64 + 16 * (j ^ ((r >> 1) & 3)); }

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void st_shared_u16(uint32_t addr, unsigned short v) {
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"(v) : "memory");
}

// Stage this warp's 32x32 bf16 block (lane = row) and, for strictly upper
// blocks of a symmetric output, its transpose; then one lane stores both with TMA.
// Elements outside the matrix are clipped by the tensor map.
__device__ __forceinline__ void stage_and_store(uint8_t* stage, const float (&v)[32], const CUtensorMap* map,
                                                int x, int y, bool mirror) {
  const int lane = threadIdx.x & 31;
  if (lane == 0) bulk_wait_read_all();  // the previous chunk's stores are done reading the buffer
  __syncwarp();
  const uint32_t base = smem_u32(stage);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    uint4 u;
    u.x = pack_bf16x2(v[8 * j + 0], v[8 * j + 1]);
    u.y = pack_bf16x2(v[8 * j + 2], v[8 * j + 3]);
    u.z = pack_bf16x2(v[8 * j + 4], v[8 * j + 5]);
    u.w = pack_bf16x2(v[8 * j + 6], v[8 * j + 7]);
    st_shared_v4(base + sw64_offset(lane, j), u);
  }
  if (mirror) {
    // Transposed block: element (row k, column lane).
    const uint32_t mbase = base + 2048;
#pragma unroll
    for (int k = 0; k < 32; ++k)
      st_shared_u16(mbase + sw64_offset(k, lane >> 3) + 2 * (lane & 7), __bfloat16_as_ushort(__float2bfloat16_rn(v[k])));
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_2d(map, stage, x, y);
    if (mirror) tma_store_2d(map, stage + 2048, y, x);
    bulk_commit_group();
  }
}

// p -= (lr*wd)*p ; p -= scaled_lr*o  (triton_muon.py:370-372): two float32
// subtractions; with bf16 parameters every eager op's result is rounded to
// bf16 (the products too, since `out` is then bf16).
template <typename T>
__device__ __forceinline__ float param_new(float p, float x, float slr, float lr_wd) {
  const float o = bf16_round(x);
  if (sizeof(T) == 2) {
    const float w = bf16_round(__fsub_rn(p, bf16_round(__fmul_rn(lr_wd, p))));
    return bf16_round(__fsub_rn(w, bf16_round(__fmul_rn(slr, o))));
  }
  return __fsub_rn(__fsub_rn(p, __fmul_rn(lr_wd, p)), __fmul_rn(slr, o));
}

// Parameter write of one epilogue row chunk (32 columns of X' row `grow`), in
// pieces of CW columns (16 for float32; 8 for bf16, whose longer rounding
// chain needs more registers, and for a float32 master, which also stores its
// bf16 shadow): within a piece all loads are issued before any
// store (a store could otherwise alias a later load and serialise the chunk).
template <typename T, bool SHADOW>
__device__ __forceinline__ void write_params(const MatDesc& md, const float (&v)[32], int grow, int gcol0, int m,
                                             float slr, float lr_wd) {
  constexpr int CW = (sizeof(T) == 2 || SHADOW) ? 8 : 16;
  const int n = md.n;
  T* __restrict__ p = static_cast<T*>(md.p);
  __nv_bfloat16* __restrict__ sh = SHADOW ? static_cast<__nv_bfloat16*>(md.shadow) : nullptr;
#pragma unroll
  for (int h = 0; h < 32 / CW; ++h) {
    const int c0 = gcol0 + CW * h;
    float pv[CW];
    if (!md.transposed) {
      const int64_t rbase = static_cast<int64_t>(grow) * n + c0;
      T* prow = p + rbase;
      const bool vec = md.vec && c0 + CW <= n;
      if (vec) {
#pragma unroll
        for (int q = 0; q < CW / 4; ++q) {
          const float4 t = ld4(prow, q);
          pv[4 * q] = t.x;
          pv[4 * q + 1] = t.y;
          pv[4 * q + 2] = t.z;
          pv[4 * q + 3] = t.w;
        }
      } else {
#pragma unroll
        for (int k = 0; k < CW; ++k) pv[k] = (c0 + k < n) ? ld1(prow, k) : 0.f;
      }
#pragma unroll
      for (int k = 0; k < CW; ++k) pv[k] = param_new<T>(pv[k], v[CW * h + k], slr, lr_wd);
      if (vec) {
#pragma unroll
        for (int q = 0; q < CW / 4; ++q) {
          const float4 w = make_float4(pv[4 * q], pv[4 * q + 1], pv[4 * q + 2], pv[4 * q + 3]);
          st4(prow, q, w);
          if (SHADOW) st4(sh + rbase, q, w);
        }
      } else {
#pragma unroll
        for (int k = 0; k < CW; ++k)
          if (c0 + k < n) {
            st1(prow, k, pv[k]);
            if (SHADOW) st1(sh + rbase, k, pv[k]);
          }
      }
    } else {
      // Parameter is n x m: X'[grow][col] lives at p[col][grow]; per k a warp touches 32 contiguous elements.
      const int64_t cbase = static_cast<int64_t>(c0) * m + grow;
      T* pcol = p + cbase;
#pragma unroll
      for (int k = 0; k < CW; ++k) pv[k] = (c0 + k < n) ? ld1(pcol, static_cast<int64_t>(k) * m) : 0.f;
#pragma unroll
      for (int k = 0; k < CW; ++k) pv[k] = param_new<T>(pv[k], v[CW * h + k], slr, lr_wd);
#pragma unroll
      for (int k = 0; k < CW; ++k)
        if (c0 + k < n) {
          st1(pcol, static_cast<int64_t>(k) * m, pv[k]);
          if (SHADOW) st1(sh + cbase, static_cast<int64_t>(k) * m, pv[k]);
        }
    }
  }
}

// ---------------------------------------------------------------- UPDATE_LAST: parameter blocks by TMA
// The last update rewrites the parameter.  Where the plan could describe it
// with a tensor map (MatDesc::p_tma), each epilogue warp moves its 32x32
// parameter block for a chunk -- X' rows grow0.., columns gcol0.., i.e. the
// box at (gcol0, grow0) of the parameter, or (grow0, gcol0) for a tall one --
// with one TMA load into its staging area, updates it there in place, and
// writes it back (and the bf16 shadow of a float32 master) with TMA stores:
// no per-thread global traffic, and an evict-first L2 policy so the
// parameter stream does not displace the B and X operands the other tiles
// still read.  One parameter buffer per warp: the next chunk's block is
// loaded as soon as the previous block's stores have read it.
struct LastIo {
  uint64_t* bar;   // this warp's parameter-load barrier
  uint32_t phase;
  uint32_t on;     // this tile's chunks take the TMA path
  uint32_t failed; // a parameter-load wait gave up
};

__device__ __forceinline__ float ld_shared_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void st_shared_f32(uint32_t addr, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ unsigned short ld_shared_u16(uint32_t addr) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ float bf16_bits_to_float(uint32_t bits16) { return __uint_as_float(bits16 << 16); }
__device__ __forceinline__ unsigned short float_to_bf16_bits(float x) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}

// TMA load of the parameter block of the chunk at X' columns gcol0.. (lane 0).
__device__ __forceinline__ void last_p_issue(const MatDesc& md, const CUtensorMap* maps, uint8_t* stage, LastIo& io,
                                             int grow0, int gcol0) {
  if ((threadIdx.x & 31) == 0) {
    bulk_wait_read_all();  // the previous block's stores have finished reading the staging area
    mbar_arrive_expect_tx(io.bar, md.dtype == MAD_DTYPE_BF16 ? 2048u : 4096u);
    const int x = md.transposed ? grow0 : gcol0, y = md.transposed ? gcol0 : grow0;
    tma_load_2d_hint(stage + LAST_P_OFF, maps + TM_P, io.bar, x, y, l2_policy_evict_first());
  }
}

// The chunk's parameter update on the staged block, then its TMA store(s).
// Lane l owns X' row grow0 + l: parameter row grow0 + l (block row l) or, for
// a tall parameter, parameter column grow0 + l (block column l).  Float32
// blocks use the 128-byte swizzle (16-byte unit u of row r at r*128 +
// 16*(u ^ (r & 7))), bf16 blocks and the shadow the 64-byte one.  Elements
// outside the parameter are zero-filled on the load and clipped on the store.
template <typename T, bool SHADOW>
__device__ __forceinline__ void write_params_tma(const MatDesc& md, const CUtensorMap* maps, const float (&v)[32],
                                                 int grow0, int gcol0, float slr, float lr_wd, uint8_t* stage,
                                                 LastIo& io, unsigned int* status, long long limit) {
  const int lane = threadIdx.x & 31;
  if (!mbar_wait(io.bar, io.phase, status, DEV_ERR_MBAR_TIMEOUT_EPILOGUE, limit)) {
    io.failed = 1;
    return;
  }
  io.phase ^= 1u;
  const uint32_t pb = smem_u32(stage + LAST_P_OFF), sb = smem_u32(stage + LAST_SHADOW_OFF);
  if (sizeof(T) == 4) {
    if (!md.transposed) {
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const uint32_t a = pb + lane * 128 + 16 * (u ^ (lane & 7));
        uint4 q = ld_shared_v4(a);
        float w0 = param_new<T>(__uint_as_float(q.x), v[4 * u + 0], slr, lr_wd);
        float w1 = param_new<T>(__uint_as_float(q.y), v[4 * u + 1], slr, lr_wd);
        float w2 = param_new<T>(__uint_as_float(q.z), v[4 * u + 2], slr, lr_wd);
        float w3 = param_new<T>(__uint_as_float(q.w), v[4 * u + 3], slr, lr_wd);
        q.x = __float_as_uint(w0);
        q.y = __float_as_uint(w1);
        q.z = __float_as_uint(w2);
        q.w = __float_as_uint(w3);
        st_shared_v4(a, q);
        if (SHADOW) {
          // bf16 columns 4u..4u+3 of shadow row `lane`: half of a 16-byte unit
          const uint32_t sa = sb + sw64_offset(lane, u >> 1) + 8 * (u & 1);
          asm volatile("st.shared.v2.b32 [%0], {%1, %2};" ::"r"(sa), "r"(pack_bf16x2(w0, w1)), "r"(pack_bf16x2(w2, w3))
                       : "memory");
        }
      }
    } else {
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const uint32_t a = pb + k * 128 + 16 * ((lane >> 2) ^ (k & 7)) + 4 * (lane & 3);
        const float w = param_new<T>(ld_shared_f32(a), v[k], slr, lr_wd);
        st_shared_f32(a, w);
        if (SHADOW) st_shared_u16(sb + sw64_offset(k, lane >> 3) + 2 * (lane & 7), float_to_bf16_bits(w));
      }
    }
  } else {
    if (!md.transposed) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t a = pb + sw64_offset(lane, u);
        uint4 q = ld_shared_v4(a);
        uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float lo = param_new<T>(bf16_bits_to_float(w[j] & 0xFFFFu), v[8 * u + 2 * j], slr, lr_wd);
          const float hi = param_new<T>(bf16_bits_to_float(w[j] >> 16), v[8 * u + 2 * j + 1], slr, lr_wd);
          w[j] = pack_bf16x2(lo, hi);
        }
        q.x = w[0];
        q.y = w[1];
        q.z = w[2];
        q.w = w[3];
        st_shared_v4(a, q);
      }
    } else {
#pragma unroll
      for (int k = 0; k < 32; ++k) {
        const uint32_t a = pb + sw64_offset(k, lane >> 3) + 2 * (lane & 7);
        const float w = param_new<T>(bf16_bits_to_float(ld_shared_u16(a)), v[k], slr, lr_wd);
        st_shared_u16(a, float_to_bf16_bits(w));
      }
    }
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    const int x = md.transposed ? grow0 : gcol0, y = md.transposed ? gcol0 : grow0;
    const uint64_t pol = l2_policy_evict_first();
    tma_store_2d_hint(maps + TM_P, stage + LAST_P_OFF, x, y, pol);
    if (SHADOW) tma_store_2d_hint(maps + TM_SH, stage + LAST_SHADOW_OFF, x, y, pol);
    bulk_commit_group();
  }
}

template <int MODE>
__device__ __forceinline__ void chunk_finish(const GemmArgs& args, const MatDesc& md, int grow0, int grow, bool row_ok,
                                             int gcol0, bool mirror, uint32_t (&acc)[32], const ChunkIn& in,
                                             uint8_t* stage, LastIo& io, int next_gcol0) {
  float (&v)[32] = reinterpret_cast<float (&)[32]>(acc);
  const int m = md.m;
  if (grow0 >= m) return;  // the warp's rows lie past the matrix: nothing to store (warp-uniform)
  const CUtensorMap* maps = args.tmaps + md.tmap_base;
  if (MODE == GRAM || MODE == POLY) {
    if (MODE == GRAM) {
      const float s2 = (args.iter == 0) ? md.inv_norm * md.inv_norm : 1.0f;
#pragma unroll
      for (int k = 0; k < 32; ++k) v[k] *= s2;
    } else {
#pragma unroll
      for (int k = 0; k < 32; ++k) v[k] = __fadd_rn(__fmul_rn(args.b, bf16_at(in.q, k)), __fmul_rn(args.c, v[k]));
    }
    stage_and_store(stage, v, maps + (MODE == GRAM ? TM_GRAM_ST : TM_POLY_ST), gcol0, grow0, mirror);
    return;
  }
  // UPDATE
  const float s = (args.iter == 0) ? md.inv_norm : 1.0f;
#pragma unroll
  for (int k = 0; k < 32; ++k) v[k] = __fmul_rn(s, __fadd_rn(__fmul_rn(args.a, bf16_at(in.q, k)), v[k]));
  if (MODE == UPDATE) {
    stage_and_store(stage, v, maps + (TM_X0_ST + ((args.iter & 1) ^ 1)), gcol0, grow0, false);
    return;
  }
  // scaled_lr = lr * shape factor, formed in double and rounded once (triton_muon.py:424-431).
  const float slr = static_cast<float>(args.lr * md.lr_scale);
  if (io.on) {  // warp-uniform: every lane takes part in the staged update
    if (md.dtype == MAD_DTYPE_BF16)
      write_params_tma<__nv_bfloat16, false>(md, maps, v, grow0, gcol0, slr, args.lr_wd, stage, io, args.status,
                                             args.wait_limit);
    else if (md.dtype == MAD_DTYPE_F32_MASTER)
      write_params_tma<float, true>(md, maps, v, grow0, gcol0, slr, args.lr_wd, stage, io, args.status,
                                    args.wait_limit);
    else
      write_params_tma<float, false>(md, maps, v, grow0, gcol0, slr, args.lr_wd, stage, io, args.status,
                                     args.wait_limit);
    if (!io.failed && next_gcol0 >= 0) last_p_issue(md, maps, stage, io, grow0, next_gcol0);
    return;
  }
  if (!row_ok) return;
  if (md.dtype == MAD_DTYPE_BF16)
    write_params<__nv_bfloat16, false>(md, v, grow, gcol0, m, slr, args.lr_wd);
  else if (md.dtype == MAD_DTYPE_F32_MASTER)
    write_params<float, true>(md, v, grow, gcol0, m, slr, args.lr_wd);
  else
    write_params<float, false>(md, v, grow, gcol0, m, slr, args.lr_wd);
}

// Eight epilogue warps: warp w reads TMEM lanes 32*(w%4).. (the hardware
// rule) and columns [128*half, 128*half+128) of the tile, half = (w-2)/4.
// The inputs of the first chunk are fetched before waiting for the
// accumulator, and each later chunk's inputs and TMEM load are in flight
// while the previous chunk is finished (update kernels: TMA into shared
// memory; polynomial: registers).
template <int MODE>
__device__ __forceinline__ void epilogue_loop(const GemmArgs& args, uint64_t* tfull, uint64_t* tempty,
                                              uint32_t tmem_base, uint8_t* stage, uint64_t* in_bar, uint64_t* p_bar,
                                              const Sched& sc, uint32_t rank, volatile int* abort_flag) {
  constexpr bool TMA_IN = is_update<MODE>();
  uint32_t in_phase = 0;
  LastIo io;
  io.bar = p_bar;
  io.phase = 0;
  io.on = 0;
  io.failed = 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int quad = warp & 3;
  const int half = (warp - 2) >> 2;
  const uint32_t tempty_leader[2] = {mapa_shared(smem_u32(&tempty[0]), 0), mapa_shared(smem_u32(&tempty[1]), 0)};
  int acquired = -1, acquired_p = -1;  // matrices whose store/input and parameter maps lane 0 has acquired
  for (int lt = 0;; ++lt) {
    // Lane 0 takes the tile for the warp (warp-uniform from here on).
    int t = -1, got = 0;
    if (lane == 0) {
      got = sched_take(args, sc, lt, DEV_ERR_MBAR_TIMEOUT_EPILOGUE, &t) ? 1 : 0;
      if (got) sched_release(sc, lt);
    }
    got = __shfl_sync(0xffffffffu, got, 0);
    t = __shfl_sync(0xffffffffu, t, 0);
    if (!got) {
      *abort_flag = 1;
      break;
    }
    if (t < 0) break;
    const TileRef tr = args.tiles[t];
    const MatDesc& md = args.mats[tr.mat];
    const int acc_buf = lt & 1;
    const uint32_t acc_phase = static_cast<uint32_t>((lt >> 1) & 1);
    const int rowblk = (tr.tm * PAIR_M + static_cast<int>(rank) * BM) / BM;  // this CTA's 128-row block
    const int grow0 = rowblk * BM + quad * 32;
    const int grow = grow0 + lane;
    const bool row_ok = grow < md.m;
    const int col0 = tr.tn * BN + half * 128;
    // Chunks of this warp that exist (warp-uniform): GRAM/POLY skip blocks below the diagonal.
    const int limit = is_update<MODE>() ? md.n : md.m;
    const int blk = col0 / BM;
    int nch = (col0 < limit) ? (limit - col0 + 31) / 32 : 0;
    if (nch > 4) nch = 4;
    if (!is_update<MODE>() && blk < rowblk) nch = 0;
    const bool mirror = !is_update<MODE>() && blk > rowblk;
    const bool warp_rows = grow0 < md.m;  // some of this warp's rows exist (warp-uniform)
    const CUtensorMap* in_map = args.tmaps + md.tmap_base + TM_X0_ST + (args.iter & 1);

    if (lane == 0 && tr.mat != acquired) {  // once per matrix: later uses by this thread are ordered after it
      if (MODE != UPDATE_LAST) {
        const int st = MODE == GRAM ? TM_GRAM_ST : MODE == POLY ? TM_POLY_ST : TM_X0_ST + ((args.iter & 1) ^ 1);
        tma_acquire_desc(args.tmaps + md.tmap_base + st);
      }
      if (TMA_IN) tma_acquire_desc(in_map);
      acquired = tr.mat;
    }
    io.on = (MODE == UPDATE_LAST && md.p_tma && warp_rows && nch > 0) ? 1u : 0u;
    if (io.on) {
      const CUtensorMap* maps = args.tmaps + md.tmap_base;
      if (lane == 0 && tr.mat != acquired_p) {
        tma_acquire_desc(maps + TM_P);
        if (md.dtype == MAD_DTYPE_F32_MASTER) tma_acquire_desc(maps + TM_SH);
        acquired_p = tr.mat;
      }
      last_p_issue(md, maps, stage, io, grow0, col0);  // chunk 0's block arrives while the accumulator completes
    }
    ChunkIn in[2];
    if (TMA_IN) {
      if (nch > 0 && warp_rows) in_issue(stage, in_bar, in_map, col0, grow0);
    } else if (nch > 0 && row_ok) {
      chunk_prefetch<MODE>(args, md, grow, col0, in[0]);
    }
    if (!mbar_wait(&tfull[acc_buf], acc_phase, args.status, DEV_ERR_MBAR_TIMEOUT_EPILOGUE, args.wait_limit) ||
        *abort_flag) {
      *abort_flag = 1;
      break;
    }
    tc_fence_after();
    const uint32_t tbase = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                           static_cast<uint32_t>(acc_buf * BN + half * 128);
    uint32_t acc[2][32];
    if (nch > 0) {
      tmem_ld32_issue(tbase, acc[0]);
      tmem_ld_wait(acc[0]);
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      if (TMA_IN && c < nch && warp_rows) {
        in_take(stage, in_bar, in_phase, in[c & 1].q, args.status, abort_flag);
        if (c + 1 < nch) in_issue(stage, in_bar, in_map, col0 + 32 * (c + 1), grow0);
      }
      if (c + 1 < nch) {
        if (!TMA_IN && row_ok) chunk_prefetch<MODE>(args, md, grow, col0 + 32 * (c + 1), in[(c + 1) & 1]);
        tmem_ld32_issue(tbase + 32 * (c + 1), acc[(c + 1) & 1]);
      }
      if (c < nch)
        chunk_finish<MODE>(args, md, grow0, grow, row_ok, col0 + 32 * c, mirror, acc[c & 1], in[c & 1], stage, io,
                           c + 1 < nch ? col0 + 32 * (c + 1) : -1);
      if (c + 1 < nch) tmem_ld_wait(acc[(c + 1) & 1]);
    }
    if (MODE == UPDATE_LAST && io.failed) *abort_flag = 1;
    // Accumulator drained: one arrival per warp on the leader's barrier.
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive_cluster(tempty_leader[acc_buf]);
    if (*abort_flag) break;
  }
  if (lane == 0) bulk_wait_all();  // every output store has landed before the CTA retires
}

template <int MODE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(NUM_THREADS, 1)
    ns_gemm_kernel(const __grid_constant__ GemmArgs args) {
  extern __shared__ uint8_t smem_raw[];
  // Same layout in both CTAs of the pair: the pair MMA and the leader-side
  // barriers are addressed by identical shared-memory offsets.
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stage_out = ring + Smem<MODE>::STAGES * STAGE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(stage_out + EPI_WARPS * Smem<MODE>::STAGE_OUT);
  uint64_t* empty = full + MAX_STAGES;
  uint64_t* tfull = empty + MAX_STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* epi_in = drain + 1;          // one per epilogue warp: TMA fills of its X block
  uint64_t* epi_p = epi_in + EPI_WARPS;  // one per epilogue warp: TMA fills of its parameter block (UPDATE_LAST)
  Sched sc;
  sc.full = epi_p + EPI_WARPS;
  sc.empty = sc.full + SCHED_DEPTH;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sc.empty + SCHED_DEPTH);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  sc.slot = reinterpret_cast<int32_t*>(tmem_slot + 2);
  sc.kblk = sc.slot + SCHED_DEPTH;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  if (threadIdx.x == 0) {
    for (int s = 0; s < Smem<MODE>::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * EPI_WARPS);  // one arrival per epilogue warp of both CTAs
    }
    mbar_init(drain, 1);
    for (int w = 0; w < EPI_WARPS; ++w) {
      mbar_init(&epi_in[w], 1);
      mbar_init(&epi_p[w], 1);
    }
    for (int e = 0; e < SCHED_DEPTH; ++e) {
      mbar_init(&sc.full[e], 1);
      mbar_init(&sc.empty[e], SCHED_READERS);
    }
    *abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) producer_loop<MODE>(args, ring, full, empty, sc, rank, abort_flag);
  } else if (warp == 1) {
    if (lane == 0 && rank == 0)
      mma_loop<MODE>(args, ring, full, empty, tfull, tempty, drain, tmem_base, sc, abort_flag);
  } else {
    epilogue_loop<MODE>(args, tfull, tempty, tmem_base, stage_out + (warp - 2) * Smem<MODE>::STAGE_OUT,
                        &epi_in[warp - 2], &epi_p[warp - 2], sc, rank, abort_flag);
  }
  __syncthreads();
  if (*abort_flag && threadIdx.x == 0) {
    // After an abort a peer may still have copies in flight into this CTA's
    // shared memory: give them time to land (bounded) before retiring.
    const long long t0 = clock64();
    while (clock64() - t0 < 400000) {
    }
  }
  tc_fence_before();
  cluster_sync();  // neither CTA retires while the pair still uses its memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// SMs the persistent GEMM leaves free for kernels that must run beside it
// (the NCCL all-gather of a sharded step): set by mad_set_gemm_sm_reserve.
std::atomic<int> g_reserved_sms{0};

template <int MODE>
static int launch(const GemmArgs& args, cudaStream_t stream, const char* name) {
  if (args.n_tiles <= 0) return MAD_OK;
  constexpr int SMEM_BYTES = Smem<MODE>::BYTES;
  if (cudaFuncSetAttribute(ns_gemm_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES) !=
      cudaSuccess)
    return fail_cuda("cudaFuncSetAttribute(ns_gemm_kernel)");
  // One CTA pair per two SMs: as many pairs as can be co-resident, capped by the tile count.
  static int max_pairs[16] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  int pairs = (dev < 16) ? max_pairs[dev] : 0;
  if (pairs == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * (num_sms() / 2));
    cfg.blockDim = dim3(NUM_THREADS);
    cfg.dynamicSmemBytes = SMEM_BYTES;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&pairs, ns_gemm_kernel<MODE>, &cfg) != cudaSuccess || pairs <= 0)
      return fail_cuda("cudaOccupancyMaxActiveClusters(ns_gemm_kernel)");
    if (dev < 16) max_pairs[dev] = pairs;
  }
  // SMs left to other kernels (mad_set_gemm_sm_reserve): whole CTA pairs fewer.
  const int reserve_pairs = (g_reserved_sms.load(std::memory_order_relaxed) + 1) / 2;
  if (reserve_pairs > 0) pairs = pairs - reserve_pairs > 1 ? pairs - reserve_pairs : 1;
  const int grid_pairs = args.n_tiles < pairs ? args.n_tiles : pairs;
  ns_gemm_kernel<MODE><<<2 * grid_pairs, NUM_THREADS, SMEM_BYTES, stream>>>(args);
  return check_launch(name);
}

// Gram launches still to run with an idle producer and a short wait limit
// (mad_debug_expire_next_waits).  The Gram epilogue reads no input and the idle
// producer issues no load, so when the waits of such a launch expire nothing
// is in flight: the error path runs without any risk to the GPU.
std::atomic<int> g_expire_gram_launches{0};

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
  args.a = a;
  args.b = b;
  args.c = c;
  args.lr_wd = lr_wd;
  args.lr = lr;
  args.status = status;
  // The status word is the first field of the plan header; the scheduler's counters follow it.
  static_assert(offsetof(PlanHeader, sched_next) == 8 && offsetof(PlanHeader, sched_retired) == 12,
                "PlanHeader scheduler fields");
  args.sched = reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(status) + offsetof(PlanHeader, sched_next));
  args.wait_limit = MBAR_WAIT_LIMIT_CYCLES;
  args.idle_producer = 0;
  if (mode == ns::GRAM && ns::g_expire_gram_launches.load(std::memory_order_relaxed) > 0 &&
      ns::g_expire_gram_launches.fetch_sub(1) > 0) {
    args.wait_limit = MBAR_WAIT_LIMIT_TEST_CYCLES;
    args.idle_producer = 1;
  }
  switch (mode) {
    case ns::GRAM:
      return ns::launch<ns::GRAM>(args, stream, "ns_gemm_kernel<GRAM>");
    case ns::POLY:
      return ns::launch<ns::POLY>(args, stream, "ns_gemm_kernel<POLY>");
    default:
      return last ? ns::launch<ns::UPDATE_LAST>(args, stream, "ns_gemm_kernel<UPDATE_LAST>")
                  : ns::launch<ns::UPDATE>(args, stream, "ns_gemm_kernel<UPDATE>");
  }
}

}  // namespace mad

// Arms the next n_launches Newton-Schulz Gram launches of this process so that
// their barrier waits expire (see g_expire_gram_launches).
extern "C" int mad_debug_expire_next_waits(int32_t n_launches) {
  mad::clear_error();
  if (n_launches < 0) return mad::fail(MAD_ERR_INVALID, "mad_debug_expire_next_waits: negative count");
  mad::ns::g_expire_gram_launches.store(n_launches);
  return MAD_OK;
}

// The Newton-Schulz GEMMs of this process run on (SMs - sms) SMs from the next
// launch on, rounded to CTA pairs, so kernels launched beside them on other
// streams find SMs free.  0 (the default) uses every SM.
extern "C" int mad_set_gemm_sm_reserve(int32_t sms) {
  mad::clear_error();
  if (sms < 0 || sms > 1024) return mad::fail(MAD_ERR_INVALID, "mad_set_gemm_sm_reserve: %d SMs out of range", sms);
  mad::ns::g_reserved_sms.store(sms);
  return MAD_OK;
}
