/*
 * bell.h — C ABI of the B200 (sm_100a) Block-ELL SwiGLU library (libbell_b200.so).
 *
 * Plain C: device pointers, sizes and a stream handle (a cudaStream_t passed
 * as void*).  No torch types.  Every entry point is stream-ordered on the
 * caller's stream, never synchronises (except bell_read_status), and never
 * allocates or frees device memory: the caller owns inputs, outputs and the
 * workspace buffers named in the descriptors.
 *
 * Return value: 0 (BELL_OK) or a negative BELL_ERR_* code; the message of the
 * last failure on the calling thread is available from bell_last_error().
 * Device-side problems (a column index out of range, a wait that timed out)
 * never trap: the kernels record a BELL_ERR_* bit in the status word
 * (BellFFNDesc.status, or the library's own word when NULL) and skip the work;
 * bell_read_status() returns and clears it.
 *
 * T = 0 (no tokens) is a valid call: the weights and shapes are checked, the
 * token-sized buffers (activations, outputs, h, plan) may be NULL, nothing is
 * launched and the result is BELL_OK.
 *
 * Block-ELL weight (looped_blockell/layers/block_ell.py:1-9,53-66 of the
 * reference): values [R, K, B, B] dense tiles and col_indices [R, K] int32.
 * The logical weight is [R*B, C*B]; y = x @ W^T.  Tile layout
 * BELL_TILE_IN_OUT (default) stores values[r,k] as [B_in, B_out], the
 * JAX/Flax convention (block_ell.py:96-99); BELL_TILE_OUT_IN stores
 * [B_out, B_in], the reference CUDA kernels' convention
 * (csrc/block_ell/swiglu_fwd.cu:273-284).  A column index of -1 marks a dead
 * slot (looped_blockell/opt/column_reorder.py:131-136) that contributes
 * nothing.  B is 16, 32, 64 or 128 for the bf16 and fp32 entry points; the
 * ternary path, the persistent loop kernel and bell_down_silu_bwd_bf16 name
 * their own tile sizes below.
 */
#ifndef BELL_H_
#define BELL_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BELL_ABI_VERSION 2

enum {
  BELL_OK = 0,
  BELL_ERR_DTYPE = -1,   /* unsupported dtype / kind */
  BELL_ERR_SHAPE = -2,   /* inconsistent or unsupported shape */
  BELL_ERR_ALIGN = -3,   /* pointer or stride not 16-byte aligned */
  BELL_ERR_ARCH = -4,    /* device is not sm_100 */
  BELL_ERR_LAUNCH = -5,  /* CUDA API / launch failure */
  BELL_ERR_TIMEOUT = -6, /* a device-side bounded wait gave up */
  BELL_ERR_COLIDX = -7,  /* column index outside [-1, C) */
  BELL_ERR_ARG = -8      /* NULL pointer or bad argument */
};

/* device status-word bits (OR-ed by kernels) */
enum {
  BELL_STATUS_COLIDX = 1,
  BELL_STATUS_TIMEOUT = 2,
  BELL_STATUS_INTERNAL = 4
};

enum { BELL_TILE_IN_OUT = 0, BELL_TILE_OUT_IN = 1 };
enum { BELL_DTYPE_BF16 = 0, BELL_DTYPE_F32 = 1 };

/* One Block-ELL weight. */
typedef struct BellEll {
  const void* values;          /* [R, K, B, B] bf16 or f32 tiles            */
  const int32_t* col_indices;  /* [R, K]                                    */
  int32_t R, C, K, B;          /* block-rows, block-cols, slots/row, tile   */
  int32_t layout;              /* BELL_TILE_IN_OUT / BELL_TILE_OUT_IN        */
  int32_t flags;               /* BELL_ELL_* hints (0 = none)                 */
} BellEll;

/* BellFFNDesc.gate.flags: the gate and up col_indices hold the same columns
 * (the reference MLPBlock's default, looped_blockell/layers/mlp.py:84-95).
 * Identical col_indices pointers imply it.  The forward then loads each
 * activation tile once for both projections. */
#define BELL_ELL_SAME_COLS_AS_UP 1

/*
 * SwiGLU feed-forward: out = W_down(silu(W_gate x) * W_up x) (+ residual).
 * x, residual, out: [T, d_model]; h, gate_pre, up_out: [T, d_ff]; row-major,
 * contiguous, element type = dtype (bf16 or f32).  `plan` is caller-owned
 * workspace of bell_plan_bytes() bytes (16-byte aligned).
 */
typedef struct BellFFNDesc {
  int64_t T;
  int32_t d_model, d_ff;
  int32_t dtype;               /* BELL_DTYPE_BF16 / BELL_DTYPE_F32           */
  int32_t add_residual;        /* add `residual` (or x when NULL) to out    */
  const void* x;
  const void* residual;        /* NULL -> x                                  */
  void* h;                     /* workspace/output: silu(gate) * up          */
  void* gate_pre;              /* optional output: gate projection (or NULL) */
  void* up_out;                /* optional output: up projection (or NULL)   */
  void* out;
  void* plan;                  /* workspace                                  */
  BellEll gate, up, down;
  int32_t* status;             /* optional device status word (or NULL)      */
  int32_t max_ctas;            /* cap on each persistent grid (0 = all SMs);
                                  leaves SMs free for concurrent work such as a
                                  collective on another stream               */
  int32_t reserved;
} BellFFNDesc;

/* y = x @ W^T (+ residual): one Block-ELL linear. */
typedef struct BellLinearDesc {
  int64_t T;
  int32_t dtype;               /* element type of x and the weight tiles     */
  int32_t out_dtype;           /* element type of out (bf16 inputs: BF16/F32) */
  int32_t add_residual;
  int32_t max_ctas;            /* cap on the persistent grid (0 = all SMs)   */
  const void* x;               /* [T, C*B]                                   */
  const void* residual;        /* [T, R*B], element type = dtype              */
  void* out;                   /* [T, R*B]                                   */
  void* plan;                  /* workspace, bell_plan_bytes(0,0,0,R,K)      */
  BellEll w;
  int32_t* status;
  /* bf16 only: with add_residual, the residual is added to output rows
   * [residual_row_lo, residual_row_hi) only (both 0: every row).  At tile
   * size 128 both bounds are multiples of 256 or equal to T. */
  int64_t residual_row_lo, residual_row_hi;
} BellLinearDesc;

/* Workspace bytes for the tile-schedule plan of one forward. */
size_t bell_plan_bytes(int32_t R_gu, int32_t K_gate, int32_t K_up, int32_t R_down, int32_t K_down);

/*
 * Fused Block-ELL SwiGLU forward, bf16 in/out, fp32 accumulation in TMEM.
 * Replaces titan::block_ell_swiglu_fwd / _with_intermediate
 * (reference csrc/block_ell/block_ell_ops.cpp:51-76, swiglu_fwd.cu:565-733).
 */
int bell_swiglu_fwd_bf16(const BellFFNDesc* desc, void* stream);

/*
 * Same forward for callers that cannot allocate device memory (an FFI host
 * whose runtime owns all device memory, or a server that sizes its memory
 * once at start-up).  No counterpart in the reference.  The plan and h come
 * from a static scratch array inside the library (BELL_NOALLOC_SCRATCH_BYTES,
 * reserved on every GPU that loads it); desc->h and desc->plan must be NULL.
 * Rejects problems needing more than that (see bell_noalloc_scratch_bytes)
 * with BELL_ERR_SHAPE.  The first call on a device looks up the array's
 * address; make it before any stream capture.  That address is kept for the
 * life of the process's primary context on the device: do not keep using the
 * library across a cudaDeviceReset.  Calls share the array, so calls that
 * overlap on the GPU race.  Allocates nothing.
 */
#define BELL_NOALLOC_SCRATCH_BYTES (32u << 20)
int bell_swiglu_fwd_bf16_noalloc(const BellFFNDesc* desc, void* stream);
size_t bell_noalloc_scratch_bytes(int64_t T, int32_t d_ff, int32_t R_gu, int32_t K_gate, int32_t K_up,
                                  int32_t R_down, int32_t K_down);

/* Gate/up half only: h = silu(x Wg) * (x Wu) (+ gate_pre/up_out).
 * Replaces the reference's first launch, block_ell_gate_up_silu_kernel
 * (swiglu_fwd.cu:140-402, launched at :652). */
int bell_gate_up_bf16(const BellFFNDesc* desc, void* stream);

/* Down half only: out = h Wd (+ residual, or + x when residual is NULL and
 * add_residual is set), reading the h a bell_gate_up_bf16 call left in
 * desc->h.  Replaces the reference's second launch,
 * block_ell_down_residual_kernel (swiglu_fwd.cu:413-559, launched at :690). */
int bell_down_bf16(const BellFFNDesc* desc, void* stream);

/* One Block-ELL linear (the down projection with residual epilogue, or any
 * block_ell_matmul).  Replaces block_ell_down_residual_kernel
 * (swiglu_fwd.cu:413-559, launched at :690) and the JAX block_ell_matmul
 * (looped_blockell/layers/block_ell.py:149-182). */
int bell_linear_bf16(const BellLinearDesc* desc, void* stream);

/* fp32 SwiGLU forward (all tensors f32; accuracy target rel-L2 <= 1e-5).
 * FFMA on the CUDA cores.  Replaces the fp32 evaluation of the reference's
 * block_ell_matmul / MLPBlock (looped_blockell/layers/block_ell.py:149-182,
 * mlp.py:119-145), which the reference runs in fp32 (config.py dtype). */
int bell_swiglu_fwd_f32(const BellFFNDesc* desc, void* stream);
int bell_linear_f32(const BellLinearDesc* desc, void* stream);

/*
 * The same fp32 forward on the bf16 tensor cores ("bf16x6": every fp32
 * operand split into three bf16 parts, the six leading cross products
 * accumulated in fp32; Henry, Tang & Heinecke, ARITH 2019).  Same semantics
 * and accuracy target as bell_swiglu_fwd_f32 (block_ell.py:149-182,
 * mlp.py:119-145).
 *
 * The weights are first expanded once by bell_f32x_expand_ell into bf16
 * Block-ELL matrices over one activation matrix A = [h parts | x parts]
 * ([T, 3 d_ff + 3 d_model] bf16, column blocks CA = 3 d_ff/B + 3 d_model/B):
 *   gate, up: col_base = 3 d_ff/B, part_cols = d_model/B, ident_base = -1;
 *   down:     col_base = 0, part_cols = d_ff/B, ident_base = 3 d_ff/B,
 *             ident_stride = d_model/B (three identity slots per block-row
 *             that add the residual inside the accumulator; ident_base = -1
 *             leaves them out, and then add_residual must be 0).
 * values6 holds [R, K6, B, B] bf16 and cols6 [R, K6] int32 with
 * K6 = bell_f32x_slots(K, with_identity) = 6K (+3), at most 254.
 *
 * bell_swiglu_fwd_f32x takes a BellFFNDesc with dtype F32: x, residual
 * (NULL -> x), out, and the optional h / gate_pre / up_out outputs are fp32;
 * gate / up / down are the expanded matrices (C = CA, tile size B); desc->plan
 * is unused.  `workspace` holds bell_f32x_workspace_bytes() bytes (256-byte
 * aligned).  Stream-ordered; allocates nothing.
 */
int32_t bell_f32x_slots(int32_t K, int32_t with_identity);
int bell_f32x_expand_ell(const BellEll* w_f32, int32_t col_base, int32_t part_cols, int32_t ident_base,
                         int32_t ident_stride, void* values6, int32_t* cols6, void* stream);
size_t bell_f32x_workspace_bytes(int64_t T, int32_t d_model, int32_t d_ff, int32_t B, int32_t K_gate6,
                                 int32_t K_up6, int32_t K_down6);
int bell_swiglu_fwd_f32x(const BellFFNDesc* desc, void* workspace, void* stream);

/* One fp32 Block-ELL linear the same way (replaces the fp32 evaluation of
 * block_ell_matmul, looped_blockell/layers/block_ell.py:149-182).  Activation
 * matrix A = [x parts | residual parts] ([T, 3 in + 3 out] bf16; [T, 3 in]
 * when the weight has no identity slots).  Expand the weight with
 * col_base = 0, part_cols = C (= in/B) and, for a residual, ident_base = 3 C,
 * ident_stride = R; desc->w is the expanded matrix (its C counts A's column
 * blocks), dtype and out_dtype are F32, residual_row_lo/hi must be 0, plan is
 * unused.  `workspace` holds bell_f32x_linear_workspace_bytes() bytes. */
/* Split fp32 rows into their three bf16 parts: src [T, n] (row stride
 * ld_src) -> dst[t, col0 + p n + j], p = 0, 1, 2 (row stride ld_dst, bf16).
 * The operand form of the fp32 tile gradients on the tensor cores (six
 * bell_sddmm_bf16 calls over part slices, accumulated in fp32), which replace
 * the fp32 evaluation of the reference's weight gradients
 * (csrc/block_ell/swiglu_bwd.cu:13-14, 29-30). */
int bell_f32x_split_rows(int64_t T, int32_t n, const float* src, int64_t ld_src, void* dst, int64_t ld_dst,
                         int64_t col0, void* stream);
size_t bell_f32x_linear_workspace_bytes(int64_t T, int32_t in_features, int32_t out_features, int32_t R,
                                        int32_t K6);
int bell_linear_f32x(const BellLinearDesc* desc, void* workspace, void* stream);

/* ---------------------------------------------------------------- ternary */

/*
 * Ternary Block-ELL weight: 2-bit packed tiles and one fp32 scale per tile.
 * packed: [R, K, B, B/4] bytes; tile (r,k) stored output-column major
 * ([B_out][B_in]); each little-endian uint32 holds 16 consecutive B_in
 * entries of one output column, entry i at bits 2*(i%16); codes 00 = 0,
 * 01 = +1, 11 = -1.  scales: [R, K] fp32 (per-tile AbsMean,
 * bonsai-test/bitlinear.py:34-55 with group = one tile).  Tile size B = 64.
 */
typedef struct BellTernaryEll {
  const uint8_t* packed;
  const float* scales;
  const int32_t* col_indices;
  int32_t R, C, K, B;
} BellTernaryEll;

/*
 * Ternary SwiGLU forward.  x: [T, d_model] bf16.  Activations are quantised
 * per token to int8 by absmax (bitlinear.py:58-69, Qb = 128, clamp 127);
 * tile products accumulate exactly in int32 (tcgen05 kind::i8), are combined
 * per tile as acc = fma(scale, float(sum), acc) in fp32 in ascending slot
 * order, and divided by the token scale;
 * h = silu(gate) * up in fp32 is re-quantised per token over all of d_ff for
 * the down projection.  out: [T, d_model] fp32 (+ x when add_residual).
 * Workspaces (caller-owned): q_x int8 [T, d_model], s_x f32 [T],
 * h f32 [T, d_ff], q_h int8 [T, d_ff], s_h f32 [T], plan.
 * gate_pre / up_out: optional fp32 [T, d_ff] outputs.
 */
typedef struct BellTernaryFFNDesc {
  int64_t T;
  int32_t d_model, d_ff;
  int32_t add_residual;
  int32_t reserved;
  const void* x;               /* bf16 */
  int8_t* q_x;
  float* s_x;
  float* h;
  int8_t* q_h;
  float* s_h;
  float* gate_pre;             /* optional */
  float* up_out;               /* optional */
  float* out;
  void* plan;
  BellTernaryEll gate, up, down;
  int32_t* status;
} BellTernaryFFNDesc;

int bell_swiglu_fwd_ternary(const BellTernaryFFNDesc* desc, void* stream);

/* ------------------------------------------------------------------- loop */

/*
 * L shared-weight iterations of  h <- h + FFN(RMSNorm(h))  (bf16), as one
 * persistent kernel (BELL_LOOP_PERSISTENT) or stream-ordered kernel launches
 * (BELL_LOOP_LAUNCHES).  Replaces titan::persistent_mlp_step's per-block host
 * loop (csrc/loop/persistent_core.cu:273-337, loop_ops.cpp:52-66) for the
 * shared-weight case.  h_in, h_out: [T, d_model]; norm_gain: [d_model] bf16;
 * workspaces: hn [T, d_model] bf16, h_mid [T, d_ff] bf16, plan, and
 * `workspace` (bell_loop_workspace_bytes() bytes, 16-byte aligned).  At tile
 * size 64 the RMSNorm is folded into the GEMMs: the gain multiplies the
 * gate/up tiles (copies in the workspace), the down epilogue keeps per-row
 * sums of squares of the new state, and the gate/up epilogue scales each
 * token row by its 1/rms; other tile sizes run a separate RMSNorm kernel.
 */
typedef struct BellLoopDesc {
  int64_t T;
  int32_t d_model, d_ff;
  int32_t L;
  float eps;
  const void* h_in;
  void* h_out;
  const void* norm_gain;
  void* hn;
  void* h_mid;
  void* plan;
  void* workspace;             /* bell_loop_workspace_bytes() bytes          */
  BellEll gate, up, down;
  int32_t* status;
  int32_t mode;                /* BELL_LOOP_*                                 */
  int32_t reserved;
} BellLoopDesc;

/* BellLoopDesc.mode: which implementation runs the L iterations. */
enum {
  BELL_LOOP_AUTO = 0,          /* the library's choice (the fastest it has)   */
  BELL_LOOP_LAUNCHES = 1,      /* 1 + 3L stream-ordered kernel launches       */
  BELL_LOOP_PERSISTENT = 2     /* one persistent kernel (tile size 64)        */
};

int bell_loop_fwd_bf16(const BellLoopDesc* desc, void* stream);
size_t bell_loop_workspace_bytes(int64_t T, int32_t d_model, int32_t R_gu, int32_t K_gate, int32_t K_up,
                                 int32_t B);

/* Diagonal SSM injection h = exp(-softplus(log_dt) exp(log_A)) h + softplus(log_dt) e
 * (bf16 h/e, fp32 log_A/log_dt [d]); replaces diagonal_injection_cuda
 * (csrc/loop/persistent_core.cu:53-83). */
int bell_diag_injection_bf16(int64_t T, int32_t d_model, const void* h, const void* e,
                             const float* log_A, const float* log_dt, void* out, void* stream);

/* Injection fused with the first RMSNorm of persistent_mlp_step:
 * h_out = injection(h, e) (bf16, the residual base) and
 * normed = RMSNorm(h_out) * gain, in one pass; bit-identical to
 * bell_diag_injection_bf16 followed by bell_rmsnorm_bf16.  d_model % 8 == 0,
 * bf16 pointers 16-byte aligned. */
int bell_inject_rmsnorm_bf16(int64_t T, int32_t d_model, const void* h, const void* e, const float* log_A,
                             const float* log_dt, const void* gain, float eps, void* h_out, void* normed,
                             void* stream);

/* RMSNorm (bf16 in/out, fp32 math); replaces rmsnorm_cuda
 * (csrc/loop/persistent_core.cu:97-154,224-264). */
int bell_rmsnorm_bf16(int64_t T, int32_t d_model, const void* x, const void* gain, float eps,
                      void* out, void* stream);

/* RMSNorm in fp32 (fp32 x, gain and out; d_model % 4 == 0, pointers 16-byte
 * aligned): the reference RMSNorm layer on fp32 activations
 * (looped_blockell/layers/norms.py:8-15). */
int bell_rmsnorm_f32(int64_t T, int32_t d_model, const float* x, const float* gain, float eps, float* out,
                     void* stream);

/* --------------------------------------------------------------- backward */

/*
 * The backward of the bf16 SwiGLU (reference titan::block_ell_swiglu_bwd,
 * csrc/block_ell/block_ell_ops.cpp:83-97, swiglu_bwd.cu:7-35) is built from:
 *   [d_g | d_u] = bell_down_silu_bwd_bf16(grad_out, W_down transposed,
 *                 gate_pre, up_out)  (or bell_linear_bf16 for d_h followed
 *                 by bell_silu_mul_bwd_bf16)
 *   d_x  = bell_linear_bf16([d_g | d_u], [W_gate ; W_up] transposed,
 *                           residual = grad_out)
 *   d_W  = bell_sddmm_bf16 for each of gate (x, d_g), up (x, d_u) and
 *          down (h, grad_out).
 * A transposed Block-ELL holds the same tile bytes, regrouped by column and
 * read in the other tile layout.
 */

/* SiLU*up backward (swiglu_bwd.cu:305-334): d_gate = d_h * up * silu'(gate),
 * d_up = d_h * silu(gate).  d_h, gate_pre, up_out: [T, d_ff] contiguous bf16;
 * d_gate, d_up: [T, d_ff] bf16 with rows ld_out elements apart (d_ff % 8 == 0,
 * ld_out % 8 == 0, all pointers 16-byte aligned). */
int bell_silu_mul_bwd_bf16(int64_t T, int32_t d_ff, const void* d_h, const void* gate_pre, const void* up_out,
                           void* d_gate, void* d_up, int64_t ld_out, void* stream);

/*
 * d_h = grad_out @ W_down fused with the SiLU*up backward: the linear
 * kernel's epilogue turns each fp32 d_h tile into d_gate and d_up, so d_h
 * never reaches memory (replaces the reference's d_h product and
 * silu_mul_backward, swiglu_bwd.cu:7-12, 305-334).  w_t is the transposed
 * down weight (R = d_ff / B block-rows over C = d_model / B column blocks).
 * grad_out: [T, d_model]; gate_pre, up_out: [T, d_ff]; d_gate_up: [T, 2 d_ff]
 * with d_gate in columns [0, d_ff) and d_up in [d_ff, 2 d_ff); all bf16.
 * plan: bell_plan_bytes(0, 0, 0, w_t.R, w_t.K) bytes.  Tile size 64 or 128
 * (smaller tiles: bell_linear_bf16, then bell_silu_mul_bwd_bf16).
 */
typedef struct BellDownBwdDesc {
  int64_t T;
  const void* grad_out;
  const void* gate_pre;
  const void* up_out;
  void* d_gate_up;
  void* plan;
  BellEll w_t;
  int32_t* status;
} BellDownBwdDesc;

int bell_down_silu_bwd_bf16(const BellDownBwdDesc* desc, void* stream);

/*
 * Tile gradients of one Block-ELL weight (sampled dense-dense product):
 *   grad[r, k] += a[:, c*B:(c+1)*B]^T b[:, r*B:(r+1)*B]  over all T tokens,
 * c = col_indices[r, k], stored in `layout` ([B_in, B_out] or [B_out, B_in]).
 * Dead slots (-1) keep a zero tile.  Replaces block_ell_down_backward_dw and
 * block_ell_proj_backward_dw (swiglu_bwd.cu:13-14, 29-30).  a: [T, C*B],
 * b: [T, R*B] bf16, rows lda / ldb elements apart (multiples of 8).
 * grad: [R, K, B, B] fp32, zeroed first unless `accumulate`; grad_bf16
 * (optional) receives a bf16 copy, as the reference returns.
 */
typedef struct BellSddmmDesc {
  int64_t T;
  const void* a;
  const void* b;
  int64_t lda, ldb;
  const int32_t* col_indices;  /* [R, K] */
  int32_t R, C, K, B;
  int32_t layout;
  int32_t accumulate;
  float* grad;
  void* grad_bf16;             /* optional */
  int32_t* status;
} BellSddmmDesc;

int bell_sddmm_bf16(const BellSddmmDesc* desc, void* stream);

/* The same tile gradients for fp32 a and b (the fp32 training path; fp32
 * accumulation on the CUDA cores, any tile size).  Rows lda / ldb elements
 * apart (multiples of 4); grad_bf16 must be NULL. */
int bell_sddmm_f32(const BellSddmmDesc* desc, void* stream);

/* ------------------------------------------------------------- conversion */

/*
 * Dense weight [out_features, in_features] -> Block-ELL keeping, per block-row,
 * the K tiles of largest Frobenius norm (ties: the lower column first), kept
 * columns ascending.  Replaces create_block_ell_from_dense
 * (looped_blockell/layers/block_ell.py:79-116; K = max(1, int(C * density))
 * is the caller's).  dense: bf16 or f32 row-major, 16-byte aligned; values:
 * [R, K, B, B] same type, in `layout`; col_indices: [R, K]; norms: [R, C]
 * f32 workspace that receives the tile norms.  B is 64 or 128, C <= 2048.
 */
typedef struct BellDenseToEllDesc {
  const void* dense;
  int32_t dtype;               /* BELL_DTYPE_BF16 / BELL_DTYPE_F32 */
  int32_t out_features, in_features;
  int32_t B, K, layout;
  void* values;
  int32_t* col_indices;
  float* norms;
} BellDenseToEllDesc;

int bell_dense_to_ell(const BellDenseToEllDesc* desc, void* stream);

/* --------------------------------------------------- sharded exchange */

/* Owner-side sum of the d_ff-sharded forward (no reference counterpart: the
 * reference has no multi-GPU path).  out[r, c] = bf16(fp32 sum over slices
 * s = 0 .. n_slices-1 in ascending order, then + residual[r, c] when residual
 * is non-NULL), rounded once.  Slice s, row r is at slices + s * slice_stride
 * + r * ld_slice, except slice local_slot (-1: none), read from local + r *
 * ld_local.  All bf16; d % 8 == 0; pointers 16-byte aligned; strides in
 * elements, multiples of 8.  max_ctas > 0 caps the grid (the SMs that
 * concurrent GEMM launches leave free). */
int bell_sum_slices_bf16(const void* slices, int64_t slice_stride, int64_t ld_slice, int32_t n_slices,
                         int32_t local_slot, const void* local, int64_t ld_local, const void* residual,
                         int64_t ld_res, void* out, int64_t ld_out, int64_t rows, int32_t d, int32_t max_ctas,
                         void* stream);
/* One stream-ordered copy of `bytes` between two device addresses (a peer
 * GPU's memory mapped into this process included: copy engines over NVLink). */
int bell_memcpy_async(void* dst, const void* src, size_t bytes, void* stream);
/* Enable direct access from the current device to `peer` (already enabled is
 * success); without it a copy between them is staged through the host. */
int bell_enable_peer_access(int32_t peer);
/* CUDA IPC for the sharded exchange's inboxes: the 64-byte handle of the
 * allocation holding `ptr` and ptr's offset in it; mapping such a handle of
 * another process into the current device's address space (peer access
 * enabled as needed; *ptr_out = mapped base + offset); unmapping a base. */
int bell_ipc_handle(const void* ptr, void* handle_out, uint64_t* offset_out);
int bell_ipc_open(const void* handle, uint64_t offset, void** ptr_out, void** base_out);
int bell_ipc_close(void* base);

/* ---------------------------------------------------------------- L2 pins */

/* Persisting-L2 window over [base, base+bytes) on `stream`; replaces
 * pin_weights_l2 / unpin_weights_l2 (csrc/loop/l2_policy.cu:48-155). */
int bell_pin_l2(const void* base, size_t bytes, void* stream);
int bell_unpin_l2(void* stream);

/* ------------------------------------------------------------------- misc */

int bell_abi_version(void);
/* Copies the last error message of this thread into buf; returns its code. */
int bell_last_error(char* buf, size_t len);
/* Reads (and clears when `clear`) the library's status word on `stream`;
 * this call synchronises the stream. */
int bell_read_status(int32_t* value, int32_t clear, void* stream);
/* Number of SMs of the current device and whether it is sm_100 (1/0). */
int bell_device_info(int32_t* sm_count, int32_t* is_sm100);

#ifdef __cplusplus
}
#endif

#endif /* BELL_H_ */
