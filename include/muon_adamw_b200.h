/*
 * muon_adamw_b200.h -- C ABI of the B200 MuonAdamW optimizer step.
 *
 * Plain pointers and sizes only.  All pointers named param/grad/exp_avg/
 * exp_avg_sq/momentum/dev_* are CUDA device pointers; `stream` is a
 * cudaStream_t passed as void*.  Every function returns 0 (MAD_OK) on success
 * or a MAD_ERR_* code, with a message from mad_last_error().  Apart from
 * mad_ipc_alloc (device buffers other processes of the node map, for the
 * multi-GPU paths), no function allocates device memory: callers size
 * buffers with the *_bytes / *_plan_size functions and pass them in.
 *
 * Each entry point replaces one piece of the reference's Python/Triton path
 * (reference paths relative to its "MuonAdamW package/" directory):
 *
 *   mad_adamw_step         triton_muon_adamw/adamw/triton_adam.py:66-103  solve_adamw_step
 *   mad_adamw_plan         triton_muon_adamw/adamw/triton_adam.py:106-130 TritonAdamW.__init__ (state binding)
 *   mad_adamw_step_multi   triton_muon_adamw/adamw/triton_adam.py:132-153 TritonAdamW.step (per-tensor loop)
 *   mad_muon_plan_size,
 *   mad_muon_plan          triton_muon_adamw/muon/triton_muon.py:375-412 TritonMuon.__init__ and the
 *                          per-call workspaces of :319-321 (newton_shultz_step) and :358-359 (muon_step)
 *   mad_muon_prep          triton_muon_adamw/muon/triton_muon.py:346-356 muon_step prologue
 *   mad_ns_gram            triton_muon_adamw/muon/triton_muon.py:95-117  solve_ns_kernel_1
 *   mad_ns_poly            triton_muon_adamw/muon/triton_muon.py:191-212 solve_ns_kernel_2
 *   mad_ns_update          triton_muon_adamw/muon/triton_muon.py:281-310 solve_ns_kernel_3, and on the
 *                          last iteration the muon_step epilogue :365-372
 *   mad_muon_step_multi    triton_muon_adamw/muon/triton_muon.py:414-448 TritonMuon.step
 *   mad_adamw_set_grads,
 *   mad_muon_set_grads     the reference reads p.grad afresh on every step (triton_adam.py:137-153,
 *                          triton_muon.py:414-448); these follow new gradient tensors without re-planning
 */
#ifndef MUON_ADAMW_B200_H
#define MUON_ADAMW_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  MAD_OK = 0,
  MAD_ERR_INVALID = 1,     /* bad argument: shape, count, null pointer */
  MAD_ERR_ALIGN = 2,       /* pointer alignment the kernel needs is not met */
  MAD_ERR_CUDA = 3,        /* a CUDA runtime/driver call failed */
  MAD_ERR_WORKSPACE = 4,   /* caller buffer too small */
  MAD_ERR_DEVICE = 5       /* a kernel reported an error in its status word */
};

/* Element types of parameters, gradients and Muon momentum (the AdamW moments
 * are always float32, as in the reference, triton_adam.py:128-130):
 *   MAD_DTYPE_F32         param, grad, momentum float32
 *   MAD_DTYPE_BF16        param, grad, momentum bf16
 *   MAD_DTYPE_F32_MASTER  param float32 (a master copy), momentum float32, grad
 *                         bf16; the updated value is also stored, rounded to
 *                         bf16, to `shadow` (the model's bf16 parameter, same
 *                         layout as param) -- mixed-precision training. */
enum { MAD_DTYPE_F32 = 0, MAD_DTYPE_BF16 = 1, MAD_DTYPE_F32_MASTER = 2 };

/* Message describing the last failure on the calling thread ("" if none). */
const char* mad_last_error(void);

/* ABI version of this library (2: dtype fields in mad_adamw_tensor and mad_muon_matrix;
 * 3: gradient reduction over ranks, CUDA IPC buffers; 4: shadow pointers, F32_MASTER). */
int32_t mad_abi_version(void);

/* Data-parallel gradients summed over the ranks of one node (no counterpart in
 * the single-GPU reference).  Every rank's gradient buffer is mapped into this
 * process (mad_ipc_open); rank k's copy of a gradient element at address g is
 * read at g + delta[k] bytes (delta[own rank] = 0).  The kernels sum the
 * copies in rank order in float32, multiply by `scale` (1/n_ranks for the
 * mean), round to the gradient's element type and use the result as the
 * gradient: the reduce-scatter of the gradients fused into the step. */
#define MAD_MAX_RANKS 8
typedef struct mad_grad_reduce {
  int32_t n_ranks; /* 1..MAD_MAX_RANKS */
  float scale;
  int64_t delta[MAD_MAX_RANKS];
} mad_grad_reduce;

/* ------------------------------------------------------------------ AdamW */

/* One tensor of the AdamW branch (flattened; any shape).  param and grad have
 * the types `dtype` gives; exp_avg and exp_avg_sq are float32.  bf16
 * parameters are updated in float32 and rounded once on the store. */
typedef struct mad_adamw_tensor {
  void* param;       /* element type: float32, or bf16 for MAD_DTYPE_BF16 */
  const void* grad;  /* element type: float32 for MAD_DTYPE_F32, else bf16 */
  float* exp_avg;
  float* exp_avg_sq;
  int64_t numel;
  int32_t dtype;     /* MAD_DTYPE_* */
  int32_t pad;
  void* shadow;      /* MAD_DTYPE_F32_MASTER: bf16 copy of the updated param; else unused */
} mad_adamw_tensor;

/* One AdamW update of one float32 tensor, in place (replaces solve_adamw_step,
 * triton_adam.py:66-103; same argument meaning).  bias1/bias2 are the host
 * bias corrections 1-beta^t. */
int mad_adamw_step(float* param, const float* grad, float* exp_avg, float* exp_avg_sq, int64_t numel, float lr,
                   float bias1, float bias2, float beta1, float beta2, float weight_decay, float eps, void* stream);

/* Device bytes of the table mad_adamw_plan writes for these tensors. */
int mad_adamw_table_bytes(const mad_adamw_tensor* tensors, int32_t n_tensors, int64_t* table_bytes);

/* Writes the multi-tensor table for `tensors` into dev_table and returns its
 * tile count.  Re-plan whenever any pointer changes (e.g. new .grad tensors).
 * Synchronises `stream` once (the host staging buffer is freed on return). */
int mad_adamw_plan(const mad_adamw_tensor* tensors, int32_t n_tensors, void* dev_table, int64_t table_bytes,
                   int64_t* n_tiles, void* stream);

/* Replaces the gradient address of every planned tensor (grads[i] for the
 * tensor planned i-th) without re-planning: one small kernel on `stream`,
 * ordered after the work already queued there, no synchronisation.  For
 * gradients re-allocated between steps (the reference reads p.grad afresh on
 * every step, triton_adam.py:137-153).  Every address must be 16-byte aligned
 * (MAD_ERR_ALIGN otherwise: re-plan with mad_adamw_plan). */
int mad_adamw_set_grads(void* dev_table, int64_t n_tiles, const void* const* grads, int32_t n_tensors, void* stream);

/* One AdamW update of every planned tensor in one launch (replaces the
 * TritonAdamW.step per-tensor loop, triton_adam.py:132-153). */
int mad_adamw_step_multi(const void* dev_table, int64_t n_tiles, float lr, float beta1, float beta2, float eps,
                         float weight_decay, float bias1, float bias2, void* stream);

/* mad_adamw_step_multi with each gradient element summed over the ranks of `reduce`. */
int mad_adamw_step_multi_reduce(const void* dev_table, int64_t n_tiles, float lr, float beta1, float beta2,
                                float eps, float weight_decay, float bias1, float bias2,
                                const mad_grad_reduce* reduce, void* stream);

/* ------------------------------------------------------------------ Muon */

/* One Muon matrix (rows x cols, row-major, contiguous); param, grad and
 * momentum have the types `dtype` gives.  With bf16 the momentum/Nesterov glue
 * and the parameter update round to bf16 after every operation, as the
 * reference's eager ops on bf16 tensors do (triton_muon.py:346-349, 370-372). */
typedef struct mad_muon_matrix {
  void* param;       /* float32, or bf16 for MAD_DTYPE_BF16 */
  const void* grad;  /* float32 for MAD_DTYPE_F32, else bf16 */
  void* momentum;    /* the param's type */
  int64_t rows;
  int64_t cols;
  double lr_scale; /* shape adjustment: scaled_lr = float(lr * lr_scale) (triton_muon.py:424-431) */
  int32_t dtype;   /* MAD_DTYPE_* */
  int32_t pad;
  void* shadow;    /* MAD_DTYPE_F32_MASTER: bf16 copy of the updated param (rows x cols); else unused */
} mad_muon_matrix;

/* Sizes and launch counts of a Muon plan; filled by mad_muon_plan_size and
 * passed back unchanged to every Muon call. */
typedef struct mad_muon_plan_info {
  int32_t n_mats;
  int32_t num_sms;
  int64_t table_bytes;
  int64_t work_bytes;
  int64_t prep_tiles;
  int64_t gram_tiles;
  int64_t poly_tiles;
  int64_t update_tiles;
  int64_t off_mats;
  int64_t off_tmaps;
  int64_t off_gram_tiles;
  int64_t off_poly_tiles;
  int64_t off_update_tiles;
  int64_t off_prep_map;
  int64_t off_partials;
} mad_muon_plan_info;

/* Where one matrix's Newton-Schulz operands live inside the work buffer. */
typedef struct mad_muon_buffers {
  void* x[2];       /* bf16 m x n iterate (ping, pong), leading dim ld_x */
  void* gram;       /* bf16 m x m, leading dim ld_mm */
  void* poly;       /* bf16 m x m, leading dim ld_mm */
  int64_t m, n, ld_x, ld_mm;
  int32_t transposed;
} mad_muon_buffers;

/* Computes table/work sizes and tile counts for these matrices. */
int mad_muon_plan_size(const mad_muon_matrix* mats, int32_t n_mats, mad_muon_plan_info* info);

/* Writes the plan (matrix descriptors, TMA tensor maps, tile lists) into
 * dev_table and lays the bf16 workspaces out in dev_work.  If `buffers` is
 * non-null it receives n_mats entries describing the workspace layout.
 * Synchronises `stream` once. */
int mad_muon_plan(const mad_muon_matrix* mats, int32_t n_mats, void* dev_table, void* dev_work,
                  const mad_muon_plan_info* info, mad_muon_buffers* buffers, void* stream);

/* mad_adamw_set_grads for a Muon plan: the gradient address of each planned
 * matrix (grads[i] for matrix i), 16-byte aligned; no re-planning, no
 * synchronisation (the reference reads p.grad afresh, triton_muon.py:414-448). */
int mad_muon_set_grads(const mad_muon_plan_info* info, void* dev_table, const void* const* grads, void* stream);

/* Momentum EMA, Nesterov, bf16 cast, transpose-to-wide and the Frobenius
 * norm of every planned matrix, in one launch. */
int mad_muon_prep(const mad_muon_plan_info* info, void* dev_table, double beta, int32_t nesterov, float eps,
                  void* stream);

/* mad_muon_prep with each gradient element summed over the ranks of `reduce`. */
int mad_muon_prep_reduce(const mad_muon_plan_info* info, void* dev_table, double beta, int32_t nesterov, float eps,
                         const mad_grad_reduce* reduce, void* stream);

/* Newton-Schulz iteration `iter` (0-based), one launch each:
 *   gram:   A  = s² X Xᵀ          upper-triangle tiles, mirrored
 *   poly:   B  = b A + c A A      upper-triangle tiles, mirrored
 *   update: X' = s (a X + B X)    s = 1/||X|| on iteration 0, else 1
 * With last != 0 the update writes the parameters instead of X':
 *   p = p - float(lr*weight_decay) p ;  p = p - float(lr*lr_scale) * bf16(X')
 * with X' transposed back to the parameter's orientation for tall matrices. */
int mad_ns_gram(const mad_muon_plan_info* info, void* dev_table, int32_t iter, void* stream);
int mad_ns_poly(const mad_muon_plan_info* info, void* dev_table, int32_t iter, float b, float c, void* stream);
int mad_ns_update(const mad_muon_plan_info* info, void* dev_table, int32_t iter, int32_t last, float a, double lr,
                  double weight_decay, void* stream);

/* The whole Muon branch for every planned matrix: prep, then ns_steps x
 * (gram, poly, update), the last update writing the parameters. */
int mad_muon_step_multi(const mad_muon_plan_info* info, void* dev_table, double beta, int32_t nesterov, float a,
                        float b, float c, int32_t ns_steps, float eps, double lr, double weight_decay, void* stream);

/* mad_muon_step_multi with the prep's gradient summed over the ranks of `reduce`. */
int mad_muon_step_multi_reduce(const mad_muon_plan_info* info, void* dev_table, double beta, int32_t nesterov,
                               float a, float b, float c, int32_t ns_steps, float eps, double lr,
                               double weight_decay, const mad_grad_reduce* reduce, void* stream);

/* The Muon step of ONE matrix without any allocation (no counterpart in the
 * reference).  For callers that cannot allocate at step time -- code under a
 * custom or pre-sized allocator, or a foreign-language host with no allocator
 * binding: the plan and the bf16 workspaces live in a static device array of
 * about 9.3 MB that every GPU loading this library keeps until exit.
 * Limit: rows*cols <= 1,048,576 and min(rows, cols) <= 1024 (MAD_ERR_INVALID
 * otherwise).  Same arguments and results as planning the one matrix with
 * mad_muon_plan and calling mad_muon_step_multi; lr_scale as in
 * mad_muon_matrix.  The first call on a device resolves the array's address
 * for that device.  Each call uploads
 * its plan synchronously and, once its kernels have finished, reads their
 * status word back: MAD_ERR_DEVICE if one gave up waiting on a barrier (the
 * parameter and momentum it wrote are then invalid).  Calls that overlap on
 * the GPU race on the array. */
int mad_muon_step_noalloc(float* param, const float* grad, float* momentum, int64_t rows, int64_t cols,
                          double lr_scale, double beta, int32_t nesterov, float a, float b, float c, int32_t ns_steps,
                          float eps, double lr, double weight_decay, void* stream);

/* ------------------------------------------------------------------ peer buffers */

/* Device memory the other processes of this node can map (CUDA IPC), for the
 * gradient buffers mad_grad_reduce reads.  The only entry points that
 * allocate.  mad_ipc_alloc: `bytes` of device memory on the current device
 * (zeroed) and its MAD_IPC_HANDLE_BYTES-byte handle for the peers.
 * mad_ipc_open: maps a peer's allocation (peer access enabled) and returns its
 * address in this process.  Close every mapping (all ranks) before the owner
 * frees its allocation. */
#define MAD_IPC_HANDLE_BYTES 64
int mad_ipc_alloc(int64_t bytes, void** dev_ptr, void* handle);
int mad_ipc_free(void* dev_ptr);
int mad_ipc_open(const void* handle, void** peer_ptr);
int mad_ipc_close(void* peer_ptr);

/* Copies `bytes` from src to dst -- device buffers of this node, local or
 * mapped with mad_ipc_open -- on `stream`, by the copy engines (one
 * cudaMemcpyAsync; no SM is used).  The sharded step pushes each rank's
 * updated parameters into the other ranks' replicas with it. */
int mad_copy_async(void* dst, const void* src, int64_t bytes, void* stream);

/* Other ranks' copies of a buffer: rank k's copy of the byte at address a is
 * at a + delta[k] (mapped with mad_ipc_open). */
typedef struct mad_peer_set {
  int32_t n_peers; /* 0..MAD_MAX_RANKS */
  int32_t pad;
  int64_t delta[MAD_MAX_RANKS];
} mad_peer_set;

/* Writes the `bytes` at src (16-byte aligned, a multiple of 16) into every
 * peer's copy with one small kernel on `stream`: each 16-byte vector is read
 * once and stored to all peers over NVLink.  Its CTAs (128 threads, no shared
 * memory) fit beside the persistent GEMM's, so the broadcast runs during the
 * Newton-Schulz work: the all-gather of the sharded step. */
int mad_peer_push(const void* src, int64_t bytes, const mad_peer_set* peers, void* stream);

/* Copies the plan's device status word to *status (synchronises `stream`)
 * and, if clear != 0, resets it.  Non-zero bits mean a kernel gave up
 * waiting on a barrier; the step's results are then invalid. */
int mad_muon_read_status(const mad_muon_plan_info* info, void* dev_table, uint32_t* status, int32_t clear,
                         void* stream);

/* The Newton-Schulz GEMMs (persistent: one CTA per SM) leave `sms` SMs free
 * from the next launch on, rounded up to whole CTA pairs (no counterpart in
 * the single-GPU reference).  A sharded step's exchange kernels (NCCL's
 * all-gather) launched beside the GEMMs on other streams then run at once
 * instead of taking SMs the GEMM's next launch is waiting for.  0 (default):
 * every SM. */
int mad_set_gemm_sm_reserve(int32_t sms);

/* Test hook (no counterpart in the reference): the next n_launches
 * Newton-Schulz Gram launches of this process run with an idle TMA producer
 * and a ~10 ms barrier-wait limit, so their waits expire with no copy or MMA
 * in flight.  Lets a test drive the kernels' error path -- status bits
 * DEV_ERR_MBAR_TIMEOUT_MMA and _EPILOGUE, MAD_ERR_DEVICE from
 * mad_muon_step_noalloc -- without faulting or hanging the GPU.  0 disarms. */
int mad_debug_expire_next_waits(int32_t n_launches);

#ifdef __cplusplus
}
#endif

#endif /* MUON_ADAMW_B200_H */
