/*
 * opendm_muon.h - C ABI of the B200 (sm_100a) MuonAdamW optimizer step.
 *
 * The reference implements this path as one PyTorch file,
 * opendm/optimizer/muon_adamw.py, with no native code. Each entry point below
 * replaces a group of torch ops from that file; the citation beside each
 * names the reference lines it stands in for. The Python host
 * (opendm_b200.optimizer.MuonAdamW) keeps the reference's torch.optim surface
 * and calls these functions through ctypes.
 *
 * Conventions
 *  - Every function returns an int status: MUON_OK (0) or a MUON_ERR_* code.
 *    The message of the last failure on the calling thread is returned by
 *    muon_last_error().
 *  - Every buffer is caller-owned device memory given as a plain pointer with
 *    sizes and leading dimensions in elements. The library allocates no device
 *    memory, performs no host synchronisation (muon_read_error, which waits
 *    for its stream to read the error word, is the one exception) and issues
 *    no collectives. (muon_ns_plan_create allocates only the host-side plan
 *    object.)
 *  - `stream` is a cudaStream_t passed as void*. NULL means the legacy
 *    default stream.
 *  - Device kernels bound every spin-wait. A wait that times out writes a
 *    nonzero code to the caller's device error word (`err_dev`), which the
 *    host reads after the stream completes (muon_read_error).
 */
#ifndef OPENDM_MUON_H_
#define OPENDM_MUON_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MUON_ABI_VERSION 4

enum muon_status {
  MUON_OK = 0,
  MUON_ERR_ARG = 1,         /* invalid argument (shape, dtype, pointer, alignment) */
  MUON_ERR_CUDA = 2,        /* a CUDA runtime or driver call failed */
  MUON_ERR_DEVICE = 3,      /* the current device is not sm_100 */
  MUON_ERR_UNSUPPORTED = 4, /* the request is valid but not implemented */
  MUON_ERR_KERNEL = 5       /* a kernel recorded an error (bounded wait expired) */
};

enum muon_dtype {
  MUON_BF16 = 0, /* bfloat16 storage */
  MUON_F32 = 1,  /* float32 storage */
  MUON_TF32 = 2, /* float32 storage holding values rounded to tf32 (NS operands) */
  MUON_F16 = 3,  /* float16 storage (NS operands, scaled by powers of two) */
  MUON_F16X3 = 4 /* NS operands as float16 pairs hi + lo (hi = fp16(x), lo = fp16(x - hi)), each
                    product as hi*hi + hi*lo + lo*hi: ~22-bit operands for 3x the MMA work */
};

enum muon_ns_algo {
  MUON_NS_STANDARD = 0, /* Newton-Schulz iteration on X */
  MUON_NS_GRAM = 1      /* iteration on the gram matrix, X updated every 3 iterations */
};

/* ------------------------------------------------------------------ misc */

/* ABI version of the loaded library (MUON_ABI_VERSION). */
int muon_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char* muon_last_error(void);

/* MUON_OK when `device` is an sm_100 GPU this library can run on. */
int muon_device_check(int device);

/* Copy the device error word to *host_code (synchronises `stream`).
 * Returns MUON_ERR_KERNEL when the word is nonzero, and clears it. */
int muon_read_error(int* err_dev, int* host_code, void* stream);

/* Failure-detection self test (no counterpart in the reference): launches a
 * kernel whose bounded wait on a barrier that nothing completes expires after
 * `timeout_us` (1..1e6) and records code 0x1ff in *err_dev, leaving the
 * context usable. Read the result with muon_read_error. */
int muon_selftest_bounded_wait(int* err_dev, int timeout_us, void* stream);

/* --------------------------------------------- (a) momentum + Nesterov
 * Replaces muon_adamw.py:381-394 (step += 1 is done by the host):
 *   g = grad.float() (zeros when grad is absent)
 *   exp_avg = momentum * exp_avg + g
 *   d = g + momentum * exp_avg   (nesterov)   |   d = exp_avg   (otherwise)
 * and the Frobenius norm of muon_adamw.py:118-121, fused: each segment's
 * sum of d^2 is reduced and turned into the Newton-Schulz input scale
 *   scale = 0                       if the norm is 0 or not finite
 *   scale = 1 / max(norm, eps)      otherwise.
 * d is written rounded to `dir_dtype` into `direction` with row stride `ld`
 * (the matrix keeps the parameter's layout): MUON_BF16 / MUON_TF32 write the
 * Newton-Schulz operand directly; MUON_F32 writes d unrounded (fp32
 * directions of FSDP shards, exchanged before the owner orthogonalises).
 */
typedef struct muon_momentum_seg {
  const void* grad;    /* [rows*cols] of grad_dtype, or NULL for an absent grad */
  float* exp_avg;      /* [rows*cols] fp32, updated in place */
  void* direction;     /* [rows][ld] of dir_dtype, or NULL: update exp_avg only */
  int64_t rows;
  int64_t cols;
  int64_t ld;          /* >= cols */
  int64_t chunk_begin; /* prefix sum of muon_momentum_chunks() over previous segments */
} muon_momentum_seg;

/* Number of work chunks the momentum kernel uses for a rows x cols segment. */
int64_t muon_momentum_chunks(int64_t rows, int64_t cols);

int muon_momentum(const muon_momentum_seg* segs_dev, int n_segs, int64_t total_chunks,
                  int grad_dtype, int dir_dtype, float momentum, int nesterov, float eps,
                  float* partials_dev /* [total_chunks] scratch */,
                  float* scales_dev /* [n_segs] out */, void* stream);

/* Allocation-free variant of muon_momentum for one matrix. It has no
 * counterpart in the reference. It exists for callers that cannot allocate
 * device memory: code that runs inside a host framework whose memory pool
 * owns every allocation, or inside a region where cudaMalloc is not allowed.
 * The caller passes only inputs and outputs (grad may be NULL; scale_out is
 * one device float); the per-chunk scratch is a 64 KiB array inside the
 * library that every GPU which loads the library keeps until the process
 * exits. Limit: rows * cols <= MUON_NOALLOC_MAX_ELEMENTS; larger matrices are
 * rejected with MUON_ERR_ARG. The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress), so make that first call
 * before any stream capture; the address is kept for the life of the
 * process, so do not call this entry point on a device after a
 * cudaDeviceReset of it. All calls on one device share its copy of the
 * array, which keeps the last call's contents: calls that overlap on that GPU
 * (for example on two streams) race with each other. Each call writes every
 * scratch value it reads, so nothing needs clearing between calls. Results
 * equal muon_momentum's for the same matrix. */
#define MUON_NOALLOC_MAX_ELEMENTS (16384LL * 16384LL)
int muon_momentum_single_noalloc(const void* grad, float* exp_avg, void* direction, int64_t rows, int64_t cols,
                                 int64_t ld, int grad_dtype, int dir_dtype, float momentum, int nesterov,
                                 float eps, float* scale_out, void* stream);

/* ------------------------------------------- fp16 operand preparation
 * fp16 operands in the momentum pass itself. Replaces muon_adamw.py:381-394
 * (momentum + Nesterov) and the normalisation of :118-121, like muon_momentum,
 * but also writes the fp16 Newton-Schulz input, so each element is read and
 * written once (12 bytes per element for bf16 gradients; a momentum pass
 * followed by a second pass writing the operand would take 18):
 *   x0 = fp16(d * p),  p = pscale[scale_index], a power of two
 * chosen from the previous step's norm of the same matrix, and
 *   scales[scale_index] = (1 / max(||d||, eps)) * mul / p
 * (mul = muon_ns_operand_scale(rows, cols, 0, MUON_F16)), the factor that
 * turns the stored x0 into the normalised input times mul. A Newton-Schulz
 * class with the MUON_NS_INPUT_SCALED flag applies it in its first
 * iteration. A matrix whose p is 0 (first step) or out of the safe range for
 * this step's norm is rewritten by a fix-up pass with a new p (redo[i] = 1);
 * pscale is updated for the next step either way. A zero or non-finite norm
 * gives scales = 0 (a zero update). pscale: [n] device floats kept by the
 * caller between steps, zero before the first; scales and redo: [n] outputs;
 * partials: [total_chunks] scratch (chunks from muon_momentum_chunks). */
typedef struct muon_momentum_f16_seg {
  const void* grad;    /* [rows*cols] of grad_dtype, or NULL */
  float* exp_avg;      /* [rows*cols] fp32, updated in place */
  void* dst;           /* [rows][ld] fp16 (a class's x0 slot) */
  int64_t rows;
  int64_t cols;
  int64_t ld;
  int64_t chunk_begin;
  int64_t lo_offset;   /* MUON_F16X3 classes: elements from dst to the lo half (its x0 batch slot
                          2g + 1); lo = fp16(x - fp16(x)) is written there. 0: no lo half */
  float mul;           /* muon_ns_operand_scale(rows, cols, 0, MUON_F16) */
  int32_t scale_index;
} muon_momentum_f16_seg;

int muon_momentum_f16(const muon_momentum_f16_seg* segs_dev, int n_segs, int64_t total_chunks, int grad_dtype,
                      float momentum, int nesterov, float eps, float* partials_dev, float* pscale_dev,
                      float* scales_dev, int* redo_dev, const float* grad_scale_dev, void* stream);

/* Power-of-two scale of the stored operand X at Newton-Schulz iteration
 * `iteration` for op_dtype MUON_F16 (1.0 for the other types). */
float muon_ns_operand_scale(int32_t rows, int32_t cols, int iteration, int op_dtype);

/* ------------------------------------ (b) Newton-Schulz orthogonalisation
 * Replaces zeropower_via_newtonschulz5 (muon_adamw.py:101-128) for a set of
 * same-shape matrices ("class"), and optionally the update of
 * muon_adamw.py:395-398 and :407-414.
 *
 * The quintic iteration X <- a X + (b A + c A A) X, A = X X^T, is evaluated
 * in the algebraically identical form
 *   A' = X X^T - I,   B' = gamma A' + beta I,   M = alpha I + A' B',   X <- M X,
 *   alpha = a + b + c, beta = b + 2c, gamma = c,
 * which avoids cancellation between a X and (b A + c A A) X when the operands
 * are rounded (tf32, fp16 or bf16) for the tensor cores, and lets every
 * epilogue work from its accumulator alone. A matrix with rows > cols is
 * orthogonalised through its transpose, as in the reference; here the
 * transpose is expressed by operand majorness, so X keeps the parameter's
 * layout and no transposed copy is made.
 *
 * Two algorithms (muon_ns_class.algo):
 *   MUON_NS_STANDARD  every iteration on X: gram, poly and apply launches.
 *   MUON_NS_GRAM      the iteration on the m x m gram matrix A = X X^T: each
 *                     P_j = a + b A_j + c A_j^2 is a polynomial of A_j, so
 *                     A_{j+1} = P_j (P_j A_j) and X_k = (P_{k-1} ... P_s) X_s;
 *                     the product is applied to X once per segment of
 *                     muon_ns_gram_segment() = 3 iterations, after which A is
 *                     recomputed from X (a restart that keeps the rounding of
 *                     the m x m products from growing; split fp16 operands
 *                     need it too: without it rank-1 inputs reach 2.5e-2).
 *                     At 5 iterations it executes at least 10% fewer FLOPs
 *                     for n >~ 1.4 m (1.16x fewer at n = 1.5 m, 1.6-1.85x
 *                     at n >= 4 m); it needs MUON_F16, MUON_F16X3 or
 *                     MUON_TF32 operands.
 *                     muon_ns_choose_algo returns the cheaper one for a shape.
 * Both give the same result up to operand rounding.
 *
 * Each class owns caller-provided buffers of op dtype (MUON_BF16 and
 * MUON_F16: 2 bytes, MUON_TF32: 4 bytes per element):
 *   x0, x1:     [count][rows][ld_x]  (x0 holds the direction written by
 *               muon_momentum, or by muon_momentum_f16 for the fp16
 *               types; x1 is the ping-pong partner)
 *   ap, bp, mm: [count][m][ld_m]     m = min(rows, cols)
 *   aa, pa, qa, qb: [count][m][ld_m] (MUON_NS_GRAM only; NULL otherwise)
 * The m x m buffers hold symmetric matrices as their 256 x 256 blocks on and
 * above the diagonal; the blocks below it are never written or read.
 * ld_x and ld_m must make rows 16-byte aligned (multiple of 8 for 2-byte,
 * of 4 for 4-byte types), and every buffer must be 16-byte aligned.
 * `scales` holds the per-matrix input scale produced by muon_momentum.
 *
 * The last iteration writes U, the orthogonalised update, to u_out
 * ([count][rows][ld_u], 16-byte aligned, ld_u * element size a multiple of
 * 16 bytes) rounded to u_dtype: MUON_F32 for the
 * exact fp32 result, or the parameter dtype (MUON_BF16), which is the value
 * the reference adds to a bf16 parameter (muon_adamw.py:414 casts the update
 * to the parameter's dtype first). muon_apply_update then applies it.
 */
/* muon_ns_class.flags: with MUON_F16 (or MUON_F16X3) operands, x0 holds the direction times
 * an arbitrary per-matrix factor and scales[i] turns it into the normalised
 * input times muon_ns_operand_scale(rows, cols, 0, MUON_F16) (what
 * muon_momentum_f16 writes). Without it, fp16 x0 must hold that scaled,
 * normalised input itself and scales is not read. tf32 and bf16 classes always apply scales (x0 holds the raw
 * direction). */
#define MUON_NS_INPUT_SCALED 1

typedef struct muon_ns_class {
  int32_t rows;
  int32_t cols;
  int32_t count;
  int32_t u_dtype; /* MUON_F32 or MUON_BF16 */
  void* x0;
  void* x1;
  int64_t ld_x;
  void* ap;
  void* bp;
  void* mm;
  int64_t ld_m;
  const float* scales; /* [count] device */
  void* u_out;         /* [count][rows][ld_u] of u_dtype */
  int64_t ld_u;
  int32_t algo;        /* MUON_NS_STANDARD or MUON_NS_GRAM */
  int32_t flags;       /* MUON_NS_INPUT_SCALED or 0 */
  void* aa;            /* MUON_NS_GRAM: A, P A and the two Q buffers */
  void* pa;
  void* qa;
  void* qb;
} muon_ns_class;

typedef struct muon_ns_plan muon_ns_plan;

/* Build launch descriptors (tensor maps, tile schedules) for `n_classes`
 * classes iterated `steps` times with operands of `op_dtype`
 * (MUON_TF32, MUON_F16, MUON_F16X3 or MUON_BF16). The plan stores pointers, not data: buffers must
 * outlive it and stay at the same addresses. */
int muon_ns_plan_create(const muon_ns_class* classes, int n_classes, int op_dtype, int steps,
                        muon_ns_plan** plan_out);

/* Run the plan: 3 grouped GEMM launches per iteration, plus one per 3
 * iterations when a class uses MUON_NS_GRAM. `err_dev` is a device int (0
 * before the call). */
int muon_ns_plan_run(const muon_ns_plan* plan, int* err_dev, void* stream);

void muon_ns_plan_destroy(muon_ns_plan* plan);

/* Kernel launches one muon_ns_plan_run issues (-1 for a null plan). */
int muon_ns_plan_launches(const muon_ns_plan* plan);

/* Let the plan's launches use at most `sms` SMs (0: all, the default), so a
 * collective launched on another stream finds SMs free while the plan runs
 * (each Newton-Schulz CTA takes a whole SM). No counterpart in the
 * reference, which runs its collectives and GEMMs one after the other. */
int muon_ns_plan_set_sm_limit(muon_ns_plan* plan, int sms);

/* Bytes of one class's workspace when its buffers are carved from a single
 * buffer with muon_ns_class_layout (each part 256-byte aligned). */
int64_t muon_ns_class_workspace_bytes(int32_t rows, int32_t cols, int32_t count, int op_dtype, int algo);

/* The algorithm with fewer executed FLOPs for a rows x cols class iterated
 * `steps` times (MUON_NS_STANDARD for MUON_BF16 operands or steps < 3). */
int muon_ns_choose_algo(int32_t rows, int32_t cols, int op_dtype, int steps);

/* Iterations per MUON_NS_GRAM segment of the reference's 5-step loop
 * (muon_adamw.py:124-127; the product of the segment's P is applied to X,
 * and A recomputed, at the end of each): 3 for MUON_F16, MUON_F16X3 and
 * MUON_TF32; 0 for an op_dtype without the gram form. Segments alternate the
 * x0 / x1 buffers, so a caller that reuses the X buffer the last apply does
 * not read (as U's destination) needs it. */
int muon_ns_gram_segment(int op_dtype);

/* Fill the buffer pointers and ld_x/ld_m of `cls` (rows, cols, count and
 * algo set by the caller) from one workspace buffer `base` of
 * muon_ns_class_workspace_bytes() bytes. */
int muon_ns_class_layout(muon_ns_class* cls, void* base, int op_dtype);

/* ------------------------------------------- (e) gradient-norm clipping
 * Replaces the clipping the reference's trainer runs before every step
 * (opendm/trainer/trainer.py:213, max_grad_norm = 1.0, through
 * torch.nn.utils.clip_grad_norm_), folded into the step: muon_clip_grad_norm
 * reads the gradients once and computes, on the device, torch's total norm
 * (per-tensor norms rounded to each gradient's dtype, their 2-norm rounded to
 * bf16 when every gradient is bf16, else fp32) and the coefficient
 * min(max_norm / (total + 1e-6), 1) with torch's rounding; out_dev[0] = total,
 * out_dev[1] = coefficient. muon_momentum_scaled and muon_adamw_scaled then
 * multiply each gradient by *grad_scale_dev as they read it (coefficient and
 * product in the gradient's dtype, as torch's CUDA in-place multiply of a
 * gradient list by a 0-d tensor computes it), so the gradients are never
 * rewritten. partials_dev: total_chunks floats (total_chunks = the
 * sum of muon_norm_chunks(numel) over the segments; chunk_begin its prefix). */
typedef struct muon_norm_seg {
  const void* grad; /* numel elements of dtype */
  int64_t numel;
  int64_t chunk_begin;
  int32_t dtype; /* MUON_BF16 or MUON_F32 */
  int32_t reserved;
} muon_norm_seg;

int64_t muon_norm_chunks(int64_t numel);
int muon_clip_grad_norm(const muon_norm_seg* segs_dev, int n_segs, int64_t total_chunks, float max_norm,
                        float* partials_dev, float* out_dev, void* stream);
int muon_momentum_scaled(const muon_momentum_seg* segs_dev, int n_segs, int64_t total_chunks, int grad_dtype,
                         int dir_dtype, float momentum, int nesterov, float eps, float* partials_dev,
                         float* scales_dev, const float* grad_scale_dev, void* stream);

/* ------------------------------- (d') cross-GPU flags for the all-gather
 * The sharded step moves the owners' updated parameters between GPUs with
 * cudaMemcpyAsync over NVLink (copy engines, no SMs) out of peer-mapped
 * buffers. These calls order the copies: no counterpart in the reference,
 * which gathers with torch.distributed collectives (muon_adamw.py:503-535).
 * A flag is a 4-byte-aligned uint32 in device memory of this GPU or of a peer
 * mapped into its address space.
 *
 * muon_flags_set: after all work queued before it on `stream`, stores `value`
 * to each flag with release semantics at system scope.
 * muon_flags_wait: work queued after it on `stream` starts once every flag
 * reaches `value` (compared in wrap-around order), read with acquire
 * semantics. The wait is bounded by `timeout_us`; on expiry it records 0x106
 * in the device int `err_dev` and lets the stream go on (the host reads the
 * word with muon_read_error). */
#define MUON_MAX_FLAGS 32
typedef struct muon_flag_list {
  uint32_t* ptr[MUON_MAX_FLAGS];
  int32_t n;
} muon_flag_list;

int muon_flags_set(const muon_flag_list* list, uint32_t value, void* stream);
int muon_flags_wait(const muon_flag_list* list, uint32_t value, int64_t timeout_us, int* err_dev, void* stream);

/* ------------------------------------------- (c) weight decay + update
 * Replaces muon_adamw.py:395-398 and :407-414 for whole matrices, with the
 * reference's rounding order:
 *   p = p * wd_factor            rounded to the param dtype (skipped when 1)
 *   p = p + (-eff) * u           one fused multiply-add, rounded to the param dtype
 * where u is U already rounded to the param dtype (muon_ns_class.u_dtype) and
 * eff = lr * lr_scale * coefficient * sqrt(max(rows, cols)) per matrix.
 * wd_factor = 1 - lr * weight_decay and eff are read at launch time, so a
 * learning-rate scheduler may change them between steps.
 */
typedef struct muon_update_seg {
  void* param;         /* [rows][cols] of param_dtype, updated in place */
  const void* update;  /* [rows][ld] of param_dtype */
  int64_t rows;
  int64_t cols;
  int64_t ld;          /* >= cols */
  int64_t chunk_begin; /* prefix sum of muon_momentum_chunks(rows, cols) */
  float eff;
  int32_t param_dtype; /* MUON_BF16 or MUON_F32 */
} muon_update_seg;

int muon_apply_update(const muon_update_seg* segs_dev, int n_segs, int64_t total_chunks, float wd_factor,
                      void* stream);

/* ------------------------------------------------- AdamW fallback group
 * Replaces _adamw_step / _call_adamw_functional (muon_adamw.py:131-175,
 * :333-343), i.e. torch.optim.adamw single-tensor AdamW with decoupled weight
 * decay, fused into one pass per element:
 *   p = p * (1 - lr*wd)            (skipped when wd == 0)
 *   m = lerp(m, g, 1 - beta1)
 *   v = beta2 * v + (1 - beta2) * g * g
 *   p = p - step_size * m / (sqrt(v) / bc2_sqrt + eps)
 * step_size = lr / (1 - beta1^step) and bc2_sqrt = sqrt(1 - beta2^step) are
 * computed by the host per segment from its step count.
 */
typedef struct muon_adamw_seg {
  void* param;        /* [numel] of param_dtype */
  const void* grad;   /* [numel] of grad_dtype */
  float* exp_avg;     /* [numel] fp32 */
  float* exp_avg_sq;  /* [numel] fp32 */
  int64_t numel;
  int64_t chunk_begin;/* prefix sum of muon_adamw_chunks() */
  float step_size;
  float bc2_sqrt;
  int32_t param_dtype;
  int32_t grad_dtype;
} muon_adamw_seg;

int64_t muon_adamw_chunks(int64_t numel);

int muon_adamw(const muon_adamw_seg* segs_dev, int n_segs, int64_t total_chunks, double beta1,
               double beta2, float eps, float wd_factor, void* stream);

/* muon_adamw with each gradient multiplied by *grad_scale_dev as it is read
 * (gradient-norm clipping, section (e)). */
int muon_adamw_scaled(const muon_adamw_seg* segs_dev, int n_segs, int64_t total_chunks, double beta1, double beta2,
                      float eps, float wd_factor, const float* grad_scale_dev, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* OPENDM_MUON_H_ */
