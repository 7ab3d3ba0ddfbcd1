/*
 * llmc_b200.h -- C ABI of the B200 (sm_100a) kernels for llm-compressor's
 * post-training-quantization hot path.
 *
 * Conventions
 *  - Every entry point is `extern "C"`, takes plain device pointers, int64
 *    sizes and a `cudaStream_t` passed as `void*`, and returns an LlmcStatus.
 *    Nothing here allocates memory visible to the caller; scratch space is a
 *    caller-provided workspace whose size a *_workspace_size() call reports.
 *  - Nothing synchronises the stream.  Errors detected on the device (a
 *    non-positive-definite Hessian, a bounded wait that ran out) are written
 *    to a caller-provided device status word, never raised as a trap.
 *  - Tensors are row-major and contiguous unless a leading dimension is given.
 *  - bf16 values travel as uint16 bit patterns, fp8 as uint8.
 *
 * Each declaration names the reference interface it replaces
 * (S/ = llm-compressor src/llmcompressor/, CT/ = compressed-tensors).
 */
#ifndef LLMC_B200_H
#define LLMC_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum LlmcStatus {
  LLMC_OK = 0,
  LLMC_EINVAL_SHAPE = 1, /* maps to ValueError (shape / divisibility)          */
  LLMC_EINVAL_DTYPE = 2, /* maps to ValueError (dtype)                          */
  LLMC_ENOT_PD = 3,      /* Hessian not positive definite -> RTN fallback        */
  LLMC_ETIMEOUT = 4,     /* a bounded device-side wait ran out                   */
  LLMC_ECUDA = 5,        /* a CUDA runtime call failed                           */
  LLMC_EINVAL_ARG = 6,   /* bad argument (null pointer, unsupported option)      */
  LLMC_ENOSUPPORT = 7    /* combination not supported by this build -> NotImplementedError */
} LlmcStatus;

/* QuantizationStrategy (CT/quantization/quant_args.py QuantizationStrategy) */
enum { LLMC_STRAT_TENSOR = 0, LLMC_STRAT_CHANNEL = 1, LLMC_STRAT_GROUP = 2,
       LLMC_STRAT_TENSOR_GROUP = 3, LLMC_STRAT_BLOCK = 4 };
/* scale storage dtype (QuantizationArgs.scale_dtype; NONE = the weight dtype, bf16) */
enum { LLMC_SCALE_NONE = 0, LLMC_SCALE_FP8 = 1, LLMC_SCALE_U8 = 2, LLMC_SCALE_F32 = 3 };
/* zero-point dtype (QuantizationArgs.zp_dtype) */
enum { LLMC_ZP_INT8 = 0, LLMC_ZP_FP8 = 1, LLMC_ZP_UINT8 = 2 };

/* The QuantizationArgs fields the hot path reads (CT/quantization/quant_args.py). */
typedef struct LlmcQuantArgs {
  int32_t num_bits;    /* 4 or 8                                   */
  int32_t type;        /* 0 = int, 1 = float                       */
  int32_t symmetric;   /* 1 = symmetric                            */
  int32_t strategy;    /* LLMC_STRAT_*                              */
  int64_t group_size;  /* GROUP / TENSOR_GROUP                      */
  int64_t block_rows;  /* BLOCK: block_structure[0]                 */
  int64_t block_cols;  /* BLOCK: block_structure[1]                 */
  int32_t scale_dtype; /* LLMC_SCALE_*                              */
  int32_t zp_dtype;    /* LLMC_ZP_*                                 */
} LlmcQuantArgs;

/* Output formats of the compressors (CT/compressors/*). */
enum { LLMC_FMT_PACK_INT32 = 0, /* pack_quantized: int codes, 32/num_bits per int32 */
       LLMC_FMT_FP8 = 1,        /* naive/float_quantized: float8_e4m3fn weight       */
       LLMC_FMT_NVFP4 = 2,      /* nvfp4_pack_quantized: E2M1 pairs + fp8 scales     */
       LLMC_FMT_MXFP4 = 3,      /* mxfp4_pack_quantized: E2M1 pairs + E8M0 scales    */
       LLMC_FMT_INT8 = 4 };     /* int8 codes, unpacked                               */

/* Library version (major*10000 + minor*100 + patch). */
int llmc_version(void);
/* Number of kernels this library has launched in the process so far (host
 * counter, incremented at each launch site); lets a caller count the device
 * work issued by a region of code.  No counterpart in the reference. */
int64_t llmc_kernel_launches(void);
/* Static description of a status code. */
const char* llmc_status_string(int status);
/* The CUDA call that last made an entry point of this library return
 * LLMC_ECUDA on the calling host thread, with CUDA's error string ("" if
 * none).  No counterpart in the reference (its errors are Python
 * exceptions carrying torch's message). */
const char* llmc_last_cuda_error(void);
/* Status raised on the current device by kernels whose entry points take no
 * status word (the streaming casts): LLMC_ETIMEOUT if a bounded wait ran out
 * since the last clear, else LLMC_OK.  Synchronises the device (it reads a
 * device variable); clear != 0 resets it.  No counterpart in the reference. */
int llmc_device_status(int clear, int* status);

/* ---------------------------------------------------------------- observers
 * Memoryless min-max statistics of a bf16 weight (rows x cols):
 * S/observers/min_max.py:16-25,106-110 (`_get_min_max` over the view built by
 * `_flatten_weight`, S/observers/helpers.py:63-102).  Outputs are bf16 with
 * shapes: TENSOR (1), CHANNEL (rows,1), GROUP/TENSOR_GROUP (rows, cols/group),
 * BLOCK (ceil(rows/bh), ceil(cols/bw)) -- blocks zero-padded as
 * `maybe_pad_tensor_for_block_quant`. */
int llmc_observe_minmax(const void* w_bf16, int64_t rows, int64_t cols, const LlmcQuantArgs* args,
                        void* min_bf16, void* max_bf16, void* stream);

/* MSE grid-search statistics of a bf16 weight (the `memoryless_mse` weight
 * observer): S/observers/mse.py:12-45 -> S/observers/mse_quant.py:19-141
 * (`_grid_search_mse`, eager search) and :235-273 (`_calculate_error`),
 * observer_kwargs maxshrink / patience / grid / norm (reference defaults 0.2,
 * 5, 100, 2.4).  Outputs as llmc_observe_minmax (the chosen shrunk range);
 * feed them to llmc_calculate_qparams as `get_qparams` does.  GROUP and
 * TENSOR_GROUP need a group of 32 * {1,2,4,8,16,32} or a power of two below
 * 32; CHANNEL, BLOCK and TENSOR groups up to 32768 values; at most 64 grid
 * steps.  `workspace`: llmc_observe_mse_workspace_size bytes of device
 * memory (8 bytes per group + 8).  The first call on a device, and a call
 * with a new `norm`, synchronises `stream` to upload the power table. */
int llmc_observe_mse_workspace_size(int64_t rows, int64_t cols, const LlmcQuantArgs* args, int64_t* bytes);
int llmc_observe_mse(const void* w_bf16, int64_t rows, int64_t cols, const LlmcQuantArgs* args, float maxshrink,
                     int patience, float grid, float norm, void* min_bf16, void* max_bf16, void* workspace,
                     void* stream);

/* Activation observers of static activation schemes: one calibration batch
 * folded into the running min/max statistics.  Replaces
 * `Observer.forward` -> `update_statistics_from_observed` of
 * MemorylessMinMaxObserver (mode 0), StaticMinMaxObserver (mode 1) and
 * MinMaxObserver (mode 2, moving average `lerp(prev, new, c)`)
 * (S/observers/min_max.py:16-110, S/observers/helpers.py:219-221) on the
 * activation layouts of flatten_for_calibration
 * (S/observers/helpers.py:104-153):
 *   x        n_tok x hidden activations (batch and sequence flattened), bf16
 *            (dtype 0) or float32 (dtype 1), contiguous, 16-byte aligned,
 *            hidden % 8 == 0;
 *   group    0: TENSOR (one statistic; also the q/k/v TENSOR layout);
 *            > 0: GROUP / TENSOR_GROUP, hidden / group statistics, each over
 *            `group` consecutive features of every token (group a multiple
 *            of 8 and a power-of-two multiple up to 256);
 *   min_io, max_io  the statistics in the activation dtype, updated in place;
 *            has_prev = 0 when the observer holds none yet (they are then
 *            written, whatever the mode);
 *   avg_w0, avg_w1  mode 2: float(1 - c) and float(c) (c: averaging_constant).
 * NaN inputs are skipped by the reduction (torch.amin would propagate them).
 * workspace: llmc_observe_activation_workspace_size bytes of device memory. */
int llmc_observe_activation_workspace_size(int64_t hidden, int64_t group, int64_t* bytes);
int llmc_observe_activation(const void* x, int64_t n_tok, int64_t hidden, int dtype, int64_t group, int mode,
                            float avg_w0, float avg_w1, int has_prev, void* min_io, void* max_io, void* workspace,
                            void* stream);

/* Absolute maximum of `n` bf16 values, max-accumulated into *absmax_f32
 * (initialise it to 0).  Used for fused-set NVFP4 global scales:
 * `Observer.get_global_scale`, S/observers/base.py:78-96. */
int llmc_absmax_accumulate(const void* w_bf16, int64_t n, float* absmax_f32, void* stream);

/* generate_gparam (CT/quantization/utils/helpers.py:309-338) from an absmax:
 * writes the float32 global scale. */
int llmc_global_scale(const float* absmax_f32, float* global_scale_f32, void* stream);

/* calculate_qparams (CT/quantization/utils/helpers.py:50-137) over `n`
 * groups from bf16 min/max.  scale_out dtype: float32 when a global scale
 * is given, else bf16 (the statistics' dtype; values on the fp8 grid for
 * scale_dtype FP8, power-of-two values for MX).  zp_out: int8 for
 * LLMC_ZP_INT8, uint8 for UINT8, float32 zeros for FP8.  global_scale may be
 * NULL. */
int llmc_calculate_qparams(const void* min_bf16, const void* max_bf16, int64_t n, const LlmcQuantArgs* args,
                           const float* global_scale, void* scale_out, void* zp_out, void* stream);

/* llmc_calculate_qparams with the statistics' dtype given: f32_stats != 0
 * evaluates calculate_qparams for statistics of a float32 tensor (every
 * step in float32, float32 eps for zero scales, float32 scale_out) -- the
 * re-observation of the permuted float32 weight under activation ordering
 * GROUP (S/modifiers/gptq/gptq_quantize.py:141-145).  The min/max values
 * still come as bf16 (the weight's values, exact in bf16).  Not for MX. */
int llmc_calculate_qparams_ex(const void* min_bf16, const void* max_bf16, int64_t n, const LlmcQuantArgs* args,
                              const float* global_scale, int f32_stats, void* scale_out, void* zp_out, void* stream);

/* ---------------------------------------------------------------- casts
 * Quantize a bf16 weight with given parameters and pack it in a
 * compressed-tensors format: `compress` of PackedQuantizationCompressor
 * (CT/compressors/pack_quantized/base.py:29-78), NaiveQuantizationCompressor
 * (CT/compressors/naive_quantized/base.py), NVFP4PackedCompressor
 * (CT/compressors/nvfp4/base.py:23-73) and MXFP4PackedCompressor
 * (CT/compressors/mxfp4/base.py:20-34).
 *   scale: bf16 (scale_is_f32 = 0) or float32 (scale_is_f32 = 1), laid out as
 *          llmc_observe_minmax's statistics; zp: int8 or NULL (symmetric);
 *   global_scale: float32 scalar or NULL (NVFP4).
 *   out: PACK_INT32 -> int32 (rows, ceil(cols*bits/32)); FP8 -> uint8 (rows, cols);
 *        NVFP4/MXFP4 -> uint8 (rows, cols/2); INT8 -> int8 (rows, cols). */
int llmc_quantize_pack(const void* w_bf16, int64_t rows, int64_t cols, const LlmcQuantArgs* args,
                       const void* scale, int scale_is_f32, const void* zp_int8, const float* global_scale,
                       int out_format, void* out, void* stream);

/* Model-free fused path: observe + calculate_qparams + quantize + pack in one
 * streaming pass over the bf16 weight (S/entrypoints/model_free/lifecycle.py:38-60
 * then `compress_module`, CT/compressors/base.py:145-166).
 *   scale_out: bf16 (INT/FP8 schemes), fp8 bytes (NVFP4), E8M0 bytes (MXFP4);
 *   zp_out: int8 (rows, groups) for asymmetric INT, else NULL;
 *   global_scale: float32 device scalar, required for TENSOR_GROUP (NVFP4). */
int llmc_modelfree_quantize(const void* w_bf16, int64_t rows, int64_t cols, const LlmcQuantArgs* args,
                            const float* global_scale, int out_format, void* packed_out, void* scale_out,
                            void* zp_out, void* stream);

/* int8 tensors holding int4 values (-8..7) -> two per byte, the even column
 * in the low nibble: `_pack_int4_to_int8` of the reference's checkpoint
 * repacker (S/utils/pack_int4_to_int8.py:13-28).  in: int8 (rows x cols),
 * cols even; out: int8 (rows x cols/2). */
int llmc_pack_int4_to_int8(const int8_t* in, int64_t rows, int64_t cols, int8_t* out, void* stream);

/* Several tensors through llmc_modelfree_quantize in as few launches as
 * possible (all with the same args and format): a batched launch for up to 48
 * tensors at a time, each with its own pointers; tensors whose shape or
 * alignment the batched kernels do not take get their own launch.  Used for
 * MoE expert sets and whole shards (S/entrypoints/model_free/process.py:104-121
 * per tensor). */
typedef struct {
  const void* w;              /* bf16 (rows x cols) */
  int64_t rows, cols;
  const float* global_scale;  /* NVFP4: float32 scalar; else NULL */
  void* out;                  /* as llmc_modelfree_quantize */
  void* scale_out;
  void* zp_out;               /* asymmetric only */
} LlmcCastJob;
int llmc_modelfree_quantize_batch(const LlmcCastJob* jobs, int njobs, const LlmcQuantArgs* args, int out_format,
                                  void* stream);

/* pack_to_int32(zero_point, num_bits, packed_dim=0)
 * (CT/compressors/pack_quantized/helpers.py:20-89): int8 (rows, groups) ->
 * int32 (ceil(rows*bits/32), groups). */
int llmc_pack_zero_point(const int8_t* zp, int64_t rows, int64_t groups, int num_bits, int32_t* out, void* stream);

/* ---------------------------------------------------------------- GPTQ Hessian
 * H += alpha * X^T X over X (n_tokens, d) bf16 with row stride ld; H is a
 * float32 (d, d) row-major matrix kept fully symmetric.  Replaces
 * `accumulate_hessian` / `_hessian_update` (S/modifiers/gptq/gptq_quantize.py:22-32,
 * 63-97; alpha = 2 reproduces the sqrt(2) input scaling).  Tensor cores
 * (tcgen05, TMEM accumulators, TMA) when d and ld are multiples of 8; a
 * CUDA-core kernel otherwise.  The tensor-core accumulators are drained into
 * float32 running sums every LLMC_HESSIAN_FOLD_TOKENS tokens, so the error
 * against the exact sum does not grow with the tokens of one call.  If
 * num_samples is non-NULL, *num_samples += num_add on the device in the same
 * stream (the reference's batch count, `:70-73,91`).  status (optional device
 * int) receives LLMC_ETIMEOUT if a bounded wait in the kernel ran out (the
 * kernel then stops early and H holds a partial sum). */
int llmc_hessian_accumulate(const void* x_bf16, int64_t n_tokens, int64_t d, int64_t ld, float* H, float alpha,
                            float* num_samples, float num_add, int* status, void* stream);

#define LLMC_HESSIAN_FOLD_TOKENS 1024

/* Options of llmc_hessian_accumulate_grouped (zero fields take the defaults). */
typedef struct LlmcHessianOpts {
  int64_t fold_tokens;  /* tokens per tensor-core partial sum (a multiple of 64); 0: LLMC_HESSIAN_FOLD_TOKENS */
  int64_t wait_ns;      /* limit of every bounded device-side wait; 0: 4 s                                   */
  int32_t test_stall;   /* 1: the MMA issuer waits on a barrier nothing arrives on, so the launch ends with
                           LLMC_ETIMEOUT after wait_ns (tests of the timeout path; H is left unchanged)     */
  int32_t reserved;
} LlmcHessianOpts;

/* Block-diagonal Hessians of `ngroups` column groups of X in one launch:
 * group g accumulates H_g += alpha * X_g^T X_g with X_g = columns
 * [g*d, (g+1)*d) of X (n_tokens, ngroups*d; row stride ld) into rows
 * [g*d, (g+1)*d) of H (ngroups*d, d).  Replaces the per-expert calls of
 * `accumulate_hessian` for the down projections of an MoE layer whose experts
 * all see every token (S/modeling/moe/linear_experts.py:244-277 ->
 * S/modifiers/gptq/base.py:255-289).  ngroups = 1 is llmc_hessian_accumulate
 * with options.  Tensor cores when d % 32 == 0 (any d % 8 == 0 for one
 * group). */
int llmc_hessian_accumulate_grouped(const void* x_bf16, int64_t n_tokens, int64_t ngroups, int64_t d, int64_t ld,
                                    float* H, float alpha, float* num_samples, float num_add, int* status,
                                    const LlmcHessianOpts* opts, void* stream);

/* Number of 256x256 output tiles the tensor-core Hessian computes for size d
 * (tiles touching the lower triangle). */
int llmc_hessian_tiles(int64_t d);

/* ---------------------------------------------------------------- GPTQ solve
 * Replaces `quantize_weight` (S/modifiers/gptq/gptq_quantize.py:100-296) in
 * three steps so that modules sharing one Hessian (q/k/v, gate/up) factor it
 * once:
 *   1. llmc_gptq_prepare_hessian: `_mask_dead_hessian` (:35-38) -- diag == 0 ->
 *      1, dead[i] = 1 -- then damp = percdamp * mean(diag), diag += damp
 *      (:181-185).  H (d x d float32) is modified in place.
 *   2. llmc_gptq_hinv: Hinv = upper Cholesky factor of H^-1 (:185-188), in
 *      float32, and (if HinvT is not NULL) its transpose, which lets step 3 run
 *      its trailing updates on the tensor cores; a non-positive pivot sets *status = LLMC_ENOT_PD (the
 *      reference's LinAlgError) and later steps then use the identity
 *      (:189-196, round-to-nearest fallback).  workspace: see
 *      llmc_gptq_hinv_workspace_size.
 *   3. llmc_gptq_quantize: the blockwise column loop (:199-277) for one weight
 *      (rows x cols bf16) with stored bf16 scales / int8 zero points (int
 *      types; TENSOR, CHANNEL, GROUP or BLOCK; other options below), writing the fake-quantized bf16
 *      weight and the summed loss (float32 scalar).  Dead columns are zeroed
 *      first (:38).  HinvT (optional) is the transposed factor from step 2.  workspace: see llmc_gptq_quantize_workspace_size.
 * Nothing synchronises; *status is read by the caller when it needs it.  The
 * tensor-core GEMMs of steps 2 and 3 raise *status to LLMC_ETIMEOUT (the
 * largest code, so it is never masked by LLMC_ENOT_PD) if one of their
 * bounded waits runs out; the results are then unusable. */
int llmc_gptq_prepare_hessian(float* H, int64_t d, float percdamp, uint8_t* dead, void* stream);
int llmc_gptq_hinv_workspace_size(int64_t d, int64_t* bytes);
int llmc_gptq_hinv(const float* H, int64_t d, float* Hinv, float* HinvT, void* workspace, int* status,
                   void* stream);
int llmc_gptq_quantize_workspace_size(int64_t rows, int64_t cols, int64_t* bytes);
int llmc_gptq_quantize(const void* w_bf16, int64_t rows, int64_t cols, const float* Hinv, const float* HinvT,
                       const uint8_t* dead, const LlmcQuantArgs* args, const void* scale_bf16, const int8_t* zp,
                       int64_t blocksize, void* wq_bf16, float* loss, void* workspace, int* status,
                       void* stream);

/* Activation ordering and the other quantization options of the block loop
 * (S/modifiers/gptq/gptq_quantize.py:120-166,209-256,279-293).
 *
 * llmc_gptq_actorder_perm: perm = argsort(diag(H), descending) -- equal
 *   diagonal values keep index order (torch's sort leaves their order
 *   unspecified).  d int32 outputs.
 * llmc_gptq_permute_hessian: Hp = H[perm][:, perm] (Hp must not alias H).
 *   The permuted Hessian then goes through llmc_gptq_prepare_hessian and
 *   llmc_gptq_hinv as usual (dead columns and damping in the permuted order).
 * llmc_permute_columns_bf16: dst[:, j] = src[:, perm[j]] -- the permuted
 *   weight that activation ordering GROUP re-observes (:141-145).
 * llmc_gptq_quantize_ex: llmc_gptq_quantize for TENSOR, CHANNEL, GROUP,
 *   TENSOR_GROUP and BLOCK strategies, int (2..8 bits), FP8 (E4M3) and FP4
 *   (E2M1) types, any block size >= 1 (blocks of more than 128 columns run
 *   as 128-column steps, the same arithmetic in exact terms), with:
 *     perm          solve column j is weight column perm[j] (order != 0); the
 *                   output weight is in the weight's own column order.  perm
 *                   must be a permutation of 0..cols-1 (entries outside
 *                   [0, cols) are clamped, giving wrong results, not faults);
 *     order         0: none; 1: WEIGHT / STATIC -- solve column j uses the
 *                   scales of weight column perm[j]'s group (g_idx[perm]);
 *                   2: GROUP -- solve column j uses group j / group_size
 *                   (scales observed on the permuted weight) and g_idx_out
 *                   receives weight column c's group (cols int32);
 *     scale_is_f32  scales are float32 and dequantization runs in float32
 *                   (else bf16 scales, bf16 products);
 *     global_scale  TENSOR_GROUP (NVFP4): float32 device scalar; the
 *                   effective scale is scale / global_scale in float32 and
 *                   scales are float32.
 *   Scale layouts: TENSOR (1), CHANNEL (rows), GROUP / TENSOR_GROUP
 *   (rows, cols / group_size), BLOCK (ceil(rows / block_rows),
 *   ceil(cols / block_cols)).  zp: int8, asymmetric int types only.
 *   cx may be NULL (no ordering, bf16 scales). */
typedef struct {
  const int32_t* perm;
  int32_t order;
  int32_t scale_is_f32;
  const float* global_scale;
  int32_t* g_idx_out;
  float* row_loss_out;  /* optional (rows floats): each row's share of the loss, so callers that run several
                           modules' rows in one call (modules sharing a Hessian) can report each module's loss */
} LlmcGptqColumns;
int llmc_gptq_actorder_perm(const float* H, int64_t d, int32_t* perm, void* stream);
int llmc_gptq_permute_hessian(const float* H, int64_t d, const int32_t* perm, float* Hp, void* stream);
int llmc_permute_columns_bf16(const void* src, int64_t rows, int64_t cols, const int32_t* perm, void* dst,
                              void* stream);
int llmc_gptq_quantize_ex(const void* w_bf16, int64_t rows, int64_t cols, const float* Hinv, const float* HinvT,
                          const uint8_t* dead, const LlmcQuantArgs* args, const void* scale, const int8_t* zp,
                          const LlmcGptqColumns* cx, int64_t blocksize, void* wq_bf16, float* loss,
                          void* workspace, int* status, void* stream);

/* GPTQ for E weights of one shape, each with its own Hessian (the down
 * projections of an MoE layer's experts, S/modifiers/gptq/base.py:591-597 once
 * per expert): for every expert e, llmc_gptq_prepare_hessian and
 * llmc_gptq_hinv on H[e] and the block loop (llmc_gptq_quantize) on W[e]
 * with its scales, in column order.  The experts are issued across
 * `nstreams` (1..16) library-owned streams joined to `stream`, so their
 * small, latency-bound kernels overlap; one host call for all experts.
 *   H       (E, d, d) float32, the averaged Hessians (clobbered);
 *   w_bf16  (E, rows, d); scale_bf16 / zp: each expert's qparams laid out as
 *           llmc_calculate_qparams gives them (CHANNEL, GROUP, TENSOR or
 *           BLOCK; TENSOR_GROUP -> LLMC_ENOSUPPORT), experts back to back;
 *           zp NULL for symmetric / float types;
 *   wq_bf16 (E, rows, d) out; loss (E) float32 out; status (E) int32 out
 *           (zeroed here; LLMC_ENOT_PD: that expert fell back to
 *           round-to-nearest; LLMC_ETIMEOUT: a bounded wait ran out);
 *   workspace: llmc_gptq_solve_batch_workspace_size bytes, 256-byte aligned. */
int llmc_gptq_solve_batch_workspace_size(int64_t E, int64_t rows, int64_t d, int nstreams, int64_t* bytes);
int llmc_gptq_solve_batch(float* H, int64_t E, int64_t d, float percdamp, const void* w_bf16, int64_t rows,
                          const LlmcQuantArgs* args, const void* scale_bf16, const int8_t* zp, int64_t blocksize,
                          void* wq_bf16, float* loss, int* status, void* workspace, int nstreams, void* stream);

/* Float32-accurate GEMM on the tensor cores (3xTF32 split):
 *   C (m x n, ldc) = A*B^T (mode 0), C - A*B^T (mode 1) or -A*B^T (mode 2),
 * A row-major m x k, B row-major n x k -- the shape of the GPTQ trailing update
 * `W[:, i2:] -= Err1.matmul(Hinv[i1:i2, i2:])` (S/modifiers/gptq/gptq_quantize.py:276-277,
 * with B = the transposed factor) and of the factorisation updates.
 * Pointers 16-byte aligned and lda/ldb multiples of 4, else LLMC_ENOSUPPORT. */
int llmc_gemm_f32_nt(int64_t m, int64_t n, int64_t k, const float* A, int64_t lda, const float* B, int64_t ldb,
                     float* C, int64_t ldc, int mode, void* stream);

/* ---------------------------------------------------------------- calibration forward
 * Fused elementwise parts of a Llama-family decoder layer, used by the
 * sequential calibration pipeline's forward passes (the reference runs the
 * HF modules eagerly: S/pipelines/sequential/pipeline.py:70-118 calling
 * transformers' LlamaDecoderLayer.forward).  bf16 in and out, 16-byte
 * aligned pointers and strides in elements that are multiples of 8, else
 * LLMC_EINVAL_SHAPE.
 *
 * RMSNorm of `rows` rows of `cols` values (LlamaRMSNorm.forward): float32
 * mean of squares, rsqrt(mean + eps), bf16(x*r), bf16(weight * that).  With
 * `residual` non-NULL the normalised value is h = bf16(residual + x), also
 * written to residual_out (the decoder layer's post-attention
 * `residual + hidden_states` fused with post_attention_layernorm). */
int llmc_rmsnorm_bf16(const void* x, const void* residual, int64_t rows, int64_t cols, const void* weight, float eps,
                      void* out, void* residual_out, void* stream);
/* Rotary embedding (apply_rotary_pos_emb: x*cos + rotate_half(x)*sin, each
 * product and the sum rounded to bf16) of x (batch, heads, seq, head_dim)
 * with element strides sb, sh, ss (unit stride inside a head) into out laid
 * out (batch, seq, heads, head_dim) contiguous.  cos / sin: (batch or 1, seq,
 * head_dim), rows contiguous, batch stride cos_batch_stride (0: shared). */
int llmc_rotary_bf16(const void* x, int64_t batch, int64_t heads, int64_t seq, int64_t head_dim, int64_t sb,
                     int64_t sh, int64_t ss, const void* cos, const void* sin, int64_t cos_batch_stride, void* out,
                     void* stream);
/* out = bf16(bf16(silu(gate)) * up) over n contiguous values (LlamaMLP's
 * act_fn(gate_proj(x)) * up_proj(x) with act_fn = SiLU). */
int llmc_silu_mul_bf16(const void* gate, const void* up, int64_t n, void* out, void* stream);
/* Mixture-of-experts layers in all-expert mode (every expert on every token,
 * the reference's moe_calibrate_all_experts; S/modeling/moe/linear_experts.py:244-277)
 * with the experts' projections stacked: gate / up are (rows, cols) with
 * cols = experts * group, expert e owning columns [e*group, (e+1)*group).
 * out = bf16(bf16(silu(gate)) * up) (may be NULL) and out_scaled =
 * bf16(out * weights[row, e]) (may be NULL; weights float32, row stride
 * weights_ld: the dense routing weights, zero where the token is not routed
 * to expert e, which gives an exact zero).  llmc_scale_groups_bf16 applies
 * the same scaling to a given x. */
int llmc_silu_mul_scaled_bf16(const void* gate, const void* up, int64_t rows, int64_t cols, int64_t group,
                              const float* weights, int64_t weights_ld, void* out, void* out_scaled, void* stream);
int llmc_scale_groups_bf16(const void* x, int64_t rows, int64_t cols, int64_t group, const float* weights,
                           int64_t weights_ld, void* out, void* stream);
/* Routed MoE combine (transformers' Qwen3MoeExperts.forward: each expert's
 * output times the token's routing weight, rounded to bf16 and index_add_-ed
 * into a zero bf16 tensor, experts in increasing index):
 * out[t] = sum_k bf16(y[pos[t*top_k + k]] * weights[t*top_k + k]) with a bf16
 * rounding after every add, k in the given order.  y: (y_rows, hidden) bf16
 * expert outputs; pos: int32 rows of y (an index outside [0, y_rows)
 * contributes nothing); weights float32; top_k <= 64. */
int llmc_moe_combine_bf16(const void* y, int64_t y_rows, const int* pos, const float* weights, int64_t tokens,
                          int64_t top_k, int64_t hidden, void* out, void* stream);

/* ---------------------------------------------------------------- no-allocation variant
 * llmc_gptq_quantize for callers that cannot allocate device memory -- code
 * running during CUDA stream capture (where cudaMalloc is not allowed),
 * hosts that own all device memory and expose no allocator, bare FFI
 * bindings.  It takes the same inputs and outputs but no workspace: the
 * scratch is a fixed array of LLMC_GPTQ_NOALLOC_SCRATCH_BYTES compiled into
 * the library, held on every GPU that loads the library's device code until
 * the process exits.  No counterpart in the reference.
 *  - Size limit: returns LLMC_EINVAL_SHAPE, launching nothing, when
 *    llmc_gptq_quantize_workspace_size(rows, cols) exceeds the array
 *    (rows*cols*4 + rows*2052 + 272 bytes > 32 MiB; e.g. 1024 x 4096 fits,
 *    4096 x 4096 does not).
 *  - Each call made outside stream capture looks up the array's device
 *    address (cudaGetSymbolAddress) with the current device; a call during
 *    capture uses the address found by the last call outside capture on that
 *    device, so make the first call on a device before any stream capture
 *    (a first call during capture returns LLMC_EINVAL_ARG).
 *  - Every call shares the one array: calls whose kernels overlap on the GPU
 *    (other streams, other host threads) race and corrupt each other.
 *    Calls ordered on one stream are safe; nothing from a previous call's
 *    contents is read.
 *  - Allocates nothing (no cudaMalloc/cudaFree). */
#define LLMC_GPTQ_NOALLOC_SCRATCH_BYTES (32ll << 20)
int llmc_gptq_quantize_noalloc(const void* w_bf16, int64_t rows, int64_t cols, const float* Hinv,
                               const float* HinvT, const uint8_t* dead, const LlmcQuantArgs* args, const void* scale_bf16,
                               const int8_t* zp, int64_t blocksize, void* wq_bf16, float* loss, int* status,
                               void* stream);

#ifdef __cplusplus
}
#endif
#endif /* LLMC_B200_H */
