// Device-side plan tables shared by the host planner and the kernels.
//
// A Muon plan is one contiguous device buffer (the "table") holding, in order:
//   PlanHeader | MatDesc[n] | CUtensorMap[6n] | TileRef lists (gram, poly,
//   update) | prep tile -> matrix map | prep partial sums
// plus a second buffer (the "work") with each matrix's bf16 Newton-Schulz
// operands: two X buffers (ping-pong), the Gram matrix A and the polynomial B.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>

namespace mad {

// ---------------------------------------------------------------- AdamW
// One tensor of the multi-tensor AdamW launch.  `vec` is 1 when every pointer
// is 16-byte aligned, so 4-element vector loads/stores are legal.
struct AdamEntry {
  void* p;             // parameter: float32, or bf16 for dtype 1
  const void* g;       // gradient: float32 for dtype 0, else bf16
  float* m;
  float* v;
  int64_t numel;
  int64_t tile_begin;  // first global tile index of this tensor
  int32_t vec;
  int32_t dtype;       // MAD_DTYPE_*: 0 float32, 1 bf16, 2 float32 master + bf16 grad/shadow
  void* shadow;        // dtype 2: bf16 copy of the updated parameter
};
static_assert(sizeof(AdamEntry) == 64, "AdamEntry layout");

constexpr int ADAM_THREADS = 128;
constexpr int ADAM_VECS = 1;                           // 4-element vectors per thread and stream in a tile
constexpr int ADAM_TILE = ADAM_THREADS * 4 * ADAM_VECS;  // elements per tile: 512

// ---------------------------------------------------------------- Muon
constexpr int TM_XK0 = 0;   // X ping buffer, K-major box {64, 128}
constexpr int TM_XK1 = 1;   // X pong buffer, K-major box {64, 128}
constexpr int TM_XMN0 = 2;  // X ping buffer, MN-major box {64, 64}
constexpr int TM_XMN1 = 3;  // X pong buffer, MN-major box {64, 64}
constexpr int TM_GRAM = 4;  // A = X Xᵀ, K-major box {64, 128}
constexpr int TM_POLY = 5;  // B = bA + cA², K-major box {64, 128}
// Epilogue stores: 32x32 boxes, 64-byte swizzle (one epilogue warp's chunk).
constexpr int TM_GRAM_ST = 6;
constexpr int TM_POLY_ST = 7;
constexpr int TM_X0_ST = 8;
constexpr int TM_X1_ST = 9;
// Parameter write of the last update: 32x32 boxes of the parameter (its own
// type and orientation; 128-byte swizzle for float32, 64-byte for bf16) and
// of the bf16 shadow of a float32 master.  Valid when MatDesc::p_tma is set.
constexpr int TM_P = 10;
constexpr int TM_SH = 11;
constexpr int TMAPS_PER_MAT = 12;

constexpr int PREP_TILE = 64;  // prep works on 64x64 tiles of the parameter
constexpr int PREP_PARTIALS_PER_TILE = 8;  // one partial sum of squares per prep warp

struct MatDesc {
  void* p;               // parameter, rows x cols, row-major: float32, or bf16 for dtype 1
  const void* g;         // gradient, same layout: float32 for dtype 0, else bf16
  void* mom;             // momentum buffer, same layout and type as p
  __nv_bfloat16* x[2];   // Newton-Schulz iterate, m x n (ld_x), ping-pong
  __nv_bfloat16* gram;   // A, m x m (ld_mm)
  __nv_bfloat16* poly;   // B, m x m (ld_mm)
  double lr_scale;       // shape factor: scaled_lr = float(lr * lr_scale)
  int32_t rows, cols;    // parameter shape
  int32_t m, n;          // wide shape: m = min(rows, cols), n = max(rows, cols)
  int32_t ld_x, ld_mm;   // leading dimensions (elements), multiples of 64
  int32_t transposed;    // rows > cols: X = uᵀ
  float inv_norm;        // 1 / max(bf16(||X||_F), bf16(eps)), written by prep
  int32_t prep_begin;    // first prep tile of this matrix
  int32_t prep_tiles_c;  // prep tiles along cols
  int32_t prep_count;    // number of prep tiles
  uint32_t done;         // unused (kept for the layout)
  int32_t tmap_base;     // index of this matrix's first tensor map
  int32_t vec;           // 4-element vectors legal for p, g, mom (and shadow) on every row
  int32_t dtype;         // MAD_DTYPE_*: 0 float32, 1 bf16, 2 float32 master + bf16 grad/shadow
  int32_t p_tma;         // 1: TM_P (and TM_SH for dtype 2) describe the parameter; else per-thread writes
  void* shadow;          // dtype 2: bf16 copy of the updated parameter, same layout as p
};
static_assert(sizeof(MatDesc) == 136, "MatDesc layout");

// One 256x256 output tile of a Newton-Schulz product.  The tile lists are
// built with MatDesc::tmap_base == mat * TMAPS_PER_MAT, so a kernel can find a
// tile's tensor maps without reading its MatDesc.
struct TileRef {
  int32_t mat;
  int32_t tm;   // row block (256 rows: a CTA pair's two 128-row halves)
  int32_t tn;   // column block (256 columns)
  int32_t nkb;  // 64-wide blocks of this product's K extent (n for X Xᵀ, m otherwise)
};

struct PlanHeader {
  uint32_t status;   // device error bits, sticky until the host clears them
  int32_t n_mats;
  // Tile scheduler of the Newton-Schulz GEMM launches: the next tile to hand
  // out and the CTA pairs that have finished taking tiles.  Zero between
  // launches (the last pair of each launch resets both).
  int32_t sched_next;
  int32_t sched_retired;
  int32_t pad[60];
};
static_assert(sizeof(PlanHeader) == 256, "PlanHeader size");

}  // namespace mad
