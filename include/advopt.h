/*
 * advopt.h — C ABI of the B200 (sm_100a) optimizer-step library
 * (libadvopt.so, built from advanced_optimizers_b200/csrc).
 *
 * The library replaces the per-parameter eager step of adv_optm 2.5.4
 * (Koratahiu/Advanced_Optimizers).  The reference has no native interface of
 * its own: its boundary is the Python method `Optimizer.step()` of each class,
 * which loops `step_parameter(p, group, i)` over the parameters.  Each entry
 * point below replaces one cluster of that loop's tensor ops for a whole
 * parameter group at once; the Python classes in advanced_optimizers_b200/
 * call them through ctypes.
 *
 * Conventions
 *  - All pointers inside the structs are DEVICE pointers unless stated.
 *  - Every entry point is asynchronous on `stream` (a cudaStream_t passed as
 *    void*), allocates nothing, and returns 0 on success or a negative
 *    ADVOPT_E* code; advopt_last_error() then describes the failure.
 *  - Tensors are contiguous; parameters and their gradients share a dtype.
 */
#ifndef ADVOPT_H_
#define ADVOPT_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ADVOPT_ABI_VERSION 5

/* ---- error codes ---- */
#define ADVOPT_OK 0
#define ADVOPT_E_INVALID (-1)   /* bad argument (null table, unsupported mode, size) */
#define ADVOPT_E_CUDA (-2)      /* a CUDA runtime call failed */
#define ADVOPT_E_UNSUPPORTED (-3)

/* ---- element / storage codes ---- */
#define ADVOPT_DT_F32 0
#define ADVOPT_DT_BF16 1

/* state precision (group['actual_state_precision'] of the reference) */
#define ADVOPT_PREC_FP32 0     /* fp32 states, fp32 math                      */
#define ADVOPT_PREC_BF16_SR 1  /* bf16 states written by stochastic rounding  */
#define ADVOPT_PREC_INT8_SR 2  /* int8 m / uint8 v, 2048-element block scales */
#define ADVOPT_PREC_AUTO 3     /* states in the param dtype, math in it too   */

/* algorithm */
#define ADVOPT_ALGO_ADAMW 0    /* AdamW_adv._step_parameter (v before m)           */
#define ADVOPT_ALGO_AUXADAM 1  /* Muon_AuxAdam._adam_step_parameter (m before v)   */
#define ADVOPT_ALGO_PRODIGY 2  /* Prodigy_adv._step_parameter (d-scaled moments)   */
#define ADVOPT_ALGO_LION 3     /* Lion_adv in the general kernel (Lion_adv.py:214-278): no second
                                  moment; ADVOPT_PREC_FP32 (factored tensors: ADVOPT_T_FACTORED |
                                  ADVOPT_T_FACT_M) or ADVOPT_PREC_AUTO (m in the param dtype);
                                  beta1 = the lerp weight of the update, w_m = 1 - beta2 */

/* launch flags */
#define ADVOPT_F_NESTEROV (1u << 0)
#define ADVOPT_F_ATAN2 (1u << 1)
#define ADVOPT_F_NORMED (1u << 2)      /* normed_momentum (AdamW only) */
#define ADVOPT_F_CAUTIOUS (1u << 3)
#define ADVOPT_F_SR (1u << 4)          /* stochastic rounding of bf16 params */
#define ADVOPT_F_NOISE_IN (1u << 5)    /* read SR noise from the tensors' noise_* arrays */
#define ADVOPT_F_HAS_M (1u << 6)       /* betas[0] > 0 */
#define ADVOPT_F_PRODIGY_STATS (1u << 7)
#define ADVOPT_F_FISHER (1u << 8)      /* Fisher weight decay (needs a stats pass) */
#define ADVOPT_F_FISHER_STATS (1u << 9)/* this launch only accumulates sum((p*ws)^2) */
#define ADVOPT_F_ANCHORS (1u << 10)    /* some tensor carries a centered-WD anchor */
#define ADVOPT_F_NO_WD (1u << 11)      /* no tensor of the launch has weight decay (optional hint) */
#define ADVOPT_F_GRAD_SQ (1u << 12)    /* also write each piece's sum of g*g to piece_gsq (Kourkoutas-beta) */
#define ADVOPT_F_EMIT_UPDATE (1u << 13)/* write each tensor's unscaled update to update_out and leave the
                                          param alone (spectral normalisation finishes the step); with
                                          stages > 0 (fast kernel) every update_out has the param dtype */
#define ADVOPT_F_FACT_M (1u << 14)     /* every tensor carries ADVOPT_T_FACT_M and ADVOPT_T_FACTORED
                                          (needs ADVOPT_PREC_FP32 and ADVOPT_F_HAS_M).  General kernel
                                          (stages 0): dynamic shared memory in two equal halves, the
                                          second for the |m| sums; fast kernel (stages > 0, every row
                                          on the fast layout): 2 x gen_offset floats of column sums,
                                          then the stage ring */

/* per-tensor flags */
#define ADVOPT_T_FACTORED (1u << 0)    /* second moment as rank-1 factors (factored_2nd) */
#define ADVOPT_T_VEC (1u << 1)         /* all pointers 16-byte aligned: vector path allowed */
#define ADVOPT_T_P0_SCALAR (1u << 2)   /* Prodigy p0 is the scalar 0 (all-zero param at init) */
#define ADVOPT_T_FACT_M (1u << 3)      /* first moment as signed rank-1 factors + 1-bit signs
                                          (state_precision='factored'; fp32 launches only) */
#define ADVOPT_T_UPD_BF16 (1u << 7)    /* update_out holds bf16 (else float32) */
#define ADVOPT_T_ANCHOR_SHIFT 4        /* 3 bits: centered-WD anchor storage */
#define ADVOPT_ANCHOR_NONE 0
#define ADVOPT_ANCHOR_FULL 1           /* anchor in the param dtype      */
#define ADVOPT_ANCHOR_FP8 2            /* float8_e4m3fn                   */
#define ADVOPT_ANCHOR_INT8 3           /* int8, block 128, scale/min in the param dtype */
#define ADVOPT_ANCHOR_INT4 4           /* int4 pairs (high, low), block 32 */

/*
 * One parameter tensor of an Adam-family group (AdamW_adv, Muon's auxiliary
 * Adam, Prodigy_adv).  Field order is fixed: 8-byte fields, then 4-byte ones.
 * Replaces the per-tensor state of AdamW_adv.py:221-277 / Prodigy_adv.py:271-331.
 */
typedef struct advopt_adam_tensor {
  void* param;               /* p (f32 or bf16), updated in place             */
  const void* grad;          /* p.grad                                        */
  void* exp_avg;             /* m: f32 / bf16 / int8, NULL without momentum   */
  float* exp_avg_scale;      /* int8 block scales [ceil(n/2048)]              */
  void* exp_avg_sq;          /* v: f32 / bf16 / uint8, NULL when factored     */
  float* exp_avg_sq_scale;   /* uint8 block scales                            */
  float* row_factor;         /* factored: mu_v_nmf [d1] (rewritten in place)  */
  float* col_factor;         /* factored: mv_v_nmf [d2] (rewritten by finish) */
  float* col_partial;        /* factored: scratch [n_slots][d2]               */
  void* aux0;                /* Prodigy s | anchor data                       */
  void* aux1;                /* Prodigy p0 | anchor scale                     */
  void* aux2;                /* anchor min                                    */
  const int32_t* noise_v;    /* injected SR noise for v  (ADVOPT_F_NOISE_IN)  */
  const int32_t* noise_m;    /* injected SR noise for m                       */
  const int32_t* noise_p;    /* injected SR noise for the param               */
  float* m_row_factor;       /* ADVOPT_T_FACT_M: mu_m_nmf [d1] (rewritten in place) */
  float* m_col_factor;       /* mv_m_nmf [d2] (rewritten by the finish)       */
  float* m_col_partial;      /* scratch [n_slots][d2]                         */
  uint8_t* m_sign;           /* sign [d1][ceil(d2/8)], bit j of byte b = column 8b+j; its
                                storage is a whole number of 4-byte words, 4-byte aligned */
  void* update_out;          /* ADVOPT_F_EMIT_UPDATE: the update before its step-size
                                scaling, f32 or bf16 (ADVOPT_T_UPD_BF16), [numel] */
  int64_t numel;
  int64_t d1;                /* factored effective shape (d1, d2)             */
  int64_t d2;
  float step_size;           /* lr/bc1 (AdamW), dlr (Prodigy); x4/pi under atan2 */
  float sqrt_bc2;            /* sqrt(1 - beta2^t), 1 without bias correction  */
  float eps;                 /* eps or 1/sqrt(numel) (eps=None); Prodigy: d*eps */
  float wd;                  /* weight_decay * lr (0: none)                   */
  float cwd;                 /* centered_wd * lr (0: none)                    */
  float fisher_clip;         /* Fisher: max(1, rms(p/denom)) written by advopt_fisher_finish */
  uint32_t tensor_id;        /* stable id of the param inside the optimizer   */
  uint32_t step;             /* Philox counter word (per-tensor step)         */
  uint32_t flags;            /* ADVOPT_T_*                                    */
  uint32_t slice_p;          /* Prodigy slice stride                          */
  int32_t slot_base;         /* first partial slot of this tensor             */
  int32_t n_slots;           /* partial slots of this tensor                  */
} advopt_adam_tensor;

/* A contiguous run [begin, end) of one tensor's flat elements, processed by
 * one CTA.  begin is a multiple of 2048; for factored tensors both ends sit on
 * row boundaries of the effective shape.  `slot` indexes the tensor's
 * col_partial rows (factored) and the launch's per-piece statistics. */
typedef struct advopt_piece {
  int64_t begin;
  int64_t end;
  int32_t tensor;
  int32_t slot;
} advopt_piece;

/* Prodigy's d estimate, resident in device memory (one per optimizer).  The
 * doubles are the param group's Python floats d, d0, d_max, d_numerator;
 * sums are the running d_numerator (carried, times beta3) and d_denom of the
 * current step (Prodigy_adv.py:246-257, 333-335); the five floats are the
 * step's launch scalars written by advopt_prodigy_scalars. */
typedef struct advopt_prodigy_dev {
  double d;
  double d0;
  double d_max;
  double d_numerator;
  float sums[2];
  float c_v;                 /* float(d * d * (1 - beta2))                     */
  float c_m;                 /* float(d * (1 - beta1))                         */
  float d_f;                 /* float(d)                                       */
  float s_alpha;             /* float((d / d0) * d) or float((d / d0) * dlr)  */
  float coef;                /* float((d / d0) * dlr): d_numerator's add       */
  float pad;
} advopt_prodigy_dev;

/* One launch over one parameter group (all scalars already rounded to fp32
 * the way the reference's scalar arguments are). */
typedef struct advopt_adam_launch {
  const advopt_adam_tensor* tensors;  /* [n_tensors]                          */
  const advopt_piece* pieces;         /* [n_pieces], grouped by CTA           */
  const int32_t* cta_offsets;         /* [grid + 1]: CTA c runs pieces [off[c], off[c+1]) */
  double* piece_stats;                /* [n_pieces * 2] Prodigy / Fisher partials */
  int32_t* err;                       /* set to 1 if a bounded wait gave up (may be NULL) */
  int32_t n_tensors;
  int32_t n_pieces;
  int32_t grid;                       /* CTAs (= length of cta_offsets - 1)   */
  int32_t smem_floats;                /* dynamic shared memory, floats        */
  int32_t gen_offset;                 /* floats before the stage ring: column accumulator (fast path: factored tensors with larger d2 accumulate in col_partial) */
  int32_t algo;                       /* ADVOPT_ALGO_*                        */
  int32_t precision;                  /* ADVOPT_PREC_*                        */
  int32_t param_dtype;                /* ADVOPT_DT_*                          */
  uint32_t flags;                     /* ADVOPT_F_*                           */
  float beta1;                        /* mul_(beta1) (Prodigy m)              */
  float beta2;                        /* mul_(beta2)                          */
  float w_m;                          /* lerp weight 1 - beta1                */
  float w_nest;                       /* lerp weight 1 - nesterov coef        */
  float c_v;                          /* addcmul value: 1-beta2 (Prodigy: d*d*(1-beta2)) */
  float c_m;                          /* Prodigy add alpha d*(1-beta1)        */
  float d_eps;                        /* unused (Prodigy's d*eps is per tensor) */
  float beta3;                        /* Prodigy s decay                      */
  float s_alpha;                      /* Prodigy s add alpha                  */
  float d;                            /* Prodigy d (grad.mul(d) without momentum) */
  int32_t stages;                     /* fast path: shared-memory ring depth (2..4); 0 = general kernel */
  uint64_t seed;                      /* Philox key                           */
  /* Kourkoutas-beta (both NULL otherwise): tensor t's v update uses
   * beta2 = layer_beta2[2 * layer_of_tensor[t]] and (1 - beta2) =
   * layer_beta2[2 * layer_of_tensor[t] + 1] instead of beta2 / c_v. */
  const float* layer_beta2;           /* [n_layers][2], written by advopt_kourkoutas_prepare */
  const int32_t* layer_of_tensor;     /* [n_tensors]                          */
  double* piece_gsq;                  /* ADVOPT_F_GRAD_SQ: [n_pieces] sum of g*g of the grad the step uses */
  /* Prodigy with d on the device: c_v, c_m, d and s_alpha are read from here
   * instead of the fields above (NULL: the fields above) */
  const advopt_prodigy_dev* prodigy;
} advopt_adam_launch;

/* Adam-family step for one group.  Replaces AdamW_adv.step/_step_parameter
 * (AdamW_adv.py:279-465), Muon_AuxAdam._adam_step_parameter
 * (Muon_AuxAdam.py:70-192), Prodigy_adv._step_parameter
 * (Prodigy_adv.py:372-519), and param_update.apply_parameter_update
 * (param_update.py:77-156) for every tensor of the group. */
int advopt_adam_step(const advopt_adam_launch* launch, void* stream);

/*
 * Spectral normalisation (scaled_optm.py:35-72, 160-168, 255-295), the step's
 * last part when a group sets spectral_normalization: advopt_adam_step with
 * ADVOPT_F_EMIT_UPDATE writes each tensor's unscaled update U to update_out;
 * advopt_spectral_step then
 *   - for a 2-D update (d_out x d_in, in the singular vectors' dtype): one
 *     power-iteration step v = norm(U^T u), u = norm(U v), sigma = u . (U v),
 *     scale = lr * (target / max(sigma, 1/(sqrt(d_out)+sqrt(d_in)))), with
 *     each torch op's rounding to that dtype; u and v are updated in place;
 *   - for a 1-D update: scale = lr / max(max|U|, 1e-12) in the update's dtype;
 * and applies p = apply_parameter_update(p, U * scale) (param_update.py:77-156)
 * with the launch's weight decay, cautious mask, centered anchors and bf16
 * stochastic rounding.  lr is each tensor's step_size in the launch's table.
 */
#define ADVOPT_S_UPD_BF16 (1u << 0)    /* update_out holds bf16 (else float32) */
#define ADVOPT_S_VEC_BF16 (1u << 1)    /* u, v are bf16 (else float32) */
#define ADVOPT_S_MAXABS (1u << 2)      /* 1-D update: max-abs scaling, no u / v */

typedef struct advopt_spectral_tensor {
  const void* update;        /* U [d_out][d_in] (the adam table's update_out)     */
  void* u;                   /* spectral_u [d_out]                               */
  void* v;                   /* spectral_v [d_in]                                */
  float* v_partial;          /* scratch [n_slabs][d_in]                          */
  float* u_raw;              /* scratch [d_out]                                  */
  float* scalars;            /* scratch [4], 8-byte aligned: the step's scale, max|U| (1-D),
                                then |U^T u|^2 as a double                       */
  int64_t d_out;             /* 1-D: 1                                           */
  int64_t d_in;              /* 1-D: numel                                       */
  float target;              /* sqrt(d_out / d_in) (1 for LoRA A factors)        */
  uint32_t flags;            /* ADVOPT_S_*                                       */
  int32_t n_slabs;           /* row slabs of the U^T u pass                      */
  int32_t pad;
} advopt_spectral_tensor;

/* `launch` is the step's launch (its table, pieces, grid, flags, seed);
 * `tensors` has launch->n_tensors entries in the same order.  col_items: one
 * advopt_piece per row slab of each 2-D update (begin/end = rows, slot = slab
 * index, at most 64 rows); row_items: pieces of rows (2-D, at most 64 rows)
 * or of elements (1-D) for the U v and max|U| passes. */
int advopt_spectral_step(const advopt_adam_launch* launch, const advopt_spectral_tensor* tensors,
                         const advopt_piece* col_items, int32_t n_col_items,
                         const advopt_piece* row_items, int32_t n_row_items, void* stream);

/* Second half of factored_2nd / 'factored': reduce the column partials into
 * mv_v_nmf (and mv_m_nmf for ADVOPT_T_FACT_M tensors) and normalise one factor
 * of each (factorization_util.py:60-80).  `tensor_index` lists the factored
 * tensors of the launch. */
int advopt_factored_finish(const advopt_adam_launch* launch, const int32_t* tensor_index,
                           int32_t n_factored, int32_t max_d2, void* stream);

/*
 * Kourkoutas-beta (Kourkoutas.py:6-257), layer-wise dynamic beta2.  A layer is
 * a set of tensors (by default those of one shape); its state is a float32
 * EMA of the pooled grad norm.
 *   prepare (once per optimizer step, before the launches): for each layer
 *     pooled = sqrt(acc); ema = ema*alpha + pooled*(1-alpha);
 *     raw = pooled / (ema + tiny_spike); sun = raw / (1 + raw);
 *     target = beta2_max - (beta2_max - beta2_min) * sun;
 *     beta2 = (1-w)*beta2_max + w*target  (w = min(1, step / k_warmup_steps));
 *     layer_beta2[l] = (beta2, float(1 - double(beta2))); acc = 0;
 *     all in float32 with each Python-double scalar rounded to float32 first,
 *     as the reference's 0-dim tensor ops do (Kourkoutas.py:131-187);
 *   accumulate (after each launch that set ADVOPT_F_GRAD_SQ): for each tensor
 *     in order, the sum of its pieces' piece_gsq (rounded to float32, or to
 *     bf16 when the step squares and sums a bf16 grad) is added to its layer's
 *     acc: the next step's pooled norm (Kourkoutas.py:231-247).
 */
typedef struct advopt_kourkoutas_args {
  float* acc;                   /* [n_layers] pooled squared-norm accumulators  */
  float* ema;                   /* [n_layers] kourkoutas_r_ema                   */
  float* layer_beta2;           /* [n_layers][2] (beta2, 1 - beta2)              */
  const int32_t* layer_of_tensor; /* accumulate: [n_tensors] of the launch      */
  const double* piece_gsq;      /* accumulate: the launch's per-piece sums        */
  const advopt_piece* pieces;   /* accumulate: the launch's pieces                */
  int32_t n_layers;
  int32_t n_tensors;
  int32_t n_pieces;
  int32_t gsq_bf16;             /* accumulate: the step squares a bf16 grad       */
  float beta2_max, beta2_min_gap; /* beta2_max, float(beta2_max - beta2_min)     */
  float ema_alpha, one_minus_alpha; /* float(alpha), float(1 - alpha)            */
  float tiny_spike;
  float w, one_minus_w_bmax;    /* float(w), float((1 - w) * beta2_max)            */
  float pad;
  double cv_scale;              /* prepare: layer_beta2[2l+1] = float(cv_scale * (1 - beta2));
                                   1 for AdamW, d*d for Prodigy (Prodigy_adv.py:413) */
  const double* d_dev;          /* prepare: when set, cv_scale = d_dev[0] * d_dev[0] (Prodigy's d on the device) */
} advopt_kourkoutas_args;

int advopt_kourkoutas_prepare(const advopt_kourkoutas_args* args, void* stream);
int advopt_kourkoutas_accumulate(const advopt_kourkoutas_args* args, void* stream);

/* Prodigy: fold the per-piece statistics into the group's running sums in
 * parameter order (Prodigy_adv.py:505-509).  `sums` (device, 2 floats) holds
 * d_numerator (already decayed by beta3) and d_denom on entry and exit.
 * `coef` = (d/d0)*dlr as float (taken from launch->prodigy->coef when that is
 * set), `s_is_bf16` says whether s is stored in bf16. */
int advopt_prodigy_finish(const advopt_adam_launch* launch, float* sums, float coef,
                          int32_t s_is_bf16, void* stream);

/* Fisher weight decay: turn the per-piece sums of (p/denom)^2 into each
 * tensor's 1/max(1, rms) (update_util.py:26-36), written to fisher_clip of a
 * device copy of the tensor table. */
int advopt_fisher_finish(const advopt_adam_launch* launch, advopt_adam_tensor* tensors_rw, void* stream);

/* Prodigy with d on the device, step part: from dev->d, the launch scalars
 * into dev (c_v, c_m, d_f, s_alpha, coef) and the d-dependent fields of the
 * group's device tensor table, in the reference's double arithmetic
 * (Prodigy_adv.py:345-346, 404-520): step_size = float(dlr [* 4/pi]),
 * eps = float(d * eps_t), wd = float(wd_t * dlr), cwd = float(cwd_t * dlr),
 * with dlr = d * lr.  One thread; launched after the table upload. */
typedef struct advopt_prodigy_scalar_args {
  advopt_prodigy_dev* dev;
  advopt_adam_tensor* tensors;    /* device table of the launch              */
  const double* tensor_consts;    /* device [n_tensors][3]: eps_t (eps or 1/sqrt(numel)), wd_t, cwd_t */
  int32_t n_tensors;
  int32_t safeguard_warmup;
  double lr, beta1, beta2;
  double step_scale;              /* 4/pi under atan2, else 1               */
} advopt_prodigy_scalar_args;

int advopt_prodigy_scalars(const advopt_prodigy_scalar_args* args, void* stream);

/* Prodigy with d on the device, end of step: calculate_d (Prodigy_adv.py:
 * 540-572) when `active`, in double precision with Python's min/max, then
 * init_step's carry (Prodigy_adv.py:246-257): sums = {float(d_numerator *
 * beta3) * carry_scale, 0}.  One thread. */
typedef struct advopt_prodigy_d_args {
  advopt_prodigy_dev* dev;
  int32_t active;                 /* prodigy_steps <= 0 or k < prodigy_steps */
  int32_t d_limiter;
  double d_coef, growth_rate;
  double limiter_factor;          /* 2 ** 0.25                               */
  double beta3;
  double carry_scale;             /* 1, or 0 on the ranks that do not carry the numerator */
} advopt_prodigy_d_args;

int advopt_prodigy_update_d(const advopt_prodigy_d_args* args, void* stream);

/* Lion_adv step for one group (Lion_adv.py:213-278, lion_k.py:23-24). */
typedef struct advopt_lion_tensor {
  void* param;
  const void* grad;
  void* exp_avg;             /* param dtype */
  const int32_t* noise_p;
  int64_t numel;
  float lr;
  float wd;                  /* weight_decay * lr */
  uint32_t tensor_id;
  uint32_t step;
  uint32_t flags;            /* ADVOPT_T_VEC */
  uint32_t pad;
} advopt_lion_tensor;

int advopt_lion_step(const advopt_lion_tensor* tensors, int32_t n_tensors, const advopt_piece* pieces,
                     int32_t n_pieces, int32_t param_dtype, float w1, float w2, uint32_t flags,
                     uint64_t seed, void* stream);

/* Adam-family step of ONE tensor that allocates nothing.  No counterpart in
 * the reference (whose step is eager PyTorch): it exists for callers that
 * cannot allocate device memory during a step — a runtime with its own
 * fixed device arena and no allocator hook, or code that must not call
 * cudaMalloc or a caching allocator mid-step.  The scratch that
 * advopt_adam_step takes from the caller (descriptor table, CTA plan,
 * factored column partials) lives instead in a file-scope __device__ array of
 * ADVOPT_NOALLOC_SCRATCH_BYTES that every GPU loading the library holds until
 * exit.  `tensor` and `launch` are HOST structs: the caller's device buffers
 * and the hyperparameters/flags (their table, plan, grid, shared-memory and
 * stage fields are ignored; launch->err, if set, receives a bounded-wait
 * give-up).  AdamW and the auxiliary Adam only (no Prodigy, no Fisher).
 * Factored tensors whose d2 column partials would not fit the array are
 * rejected with ADVOPT_E_INVALID.  The first call on a device looks up the
 * array's address (cudaGetSymbolAddress, that device current): make it before
 * any stream capture.  Calls share the array and it keeps the last call's
 * contents; calls whose kernels overlap on the GPU race and must be
 * serialised by the caller. */
#define ADVOPT_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)
int advopt_adam_step_noalloc(const advopt_adam_tensor* tensor, const advopt_adam_launch* launch, void* stream);

/* Newton–Schulz GEMM on the 5th-generation tensor cores (tcgen05 + TMEM,
 * TMA operand loads): D = bf16(alpha * A @ B + beta * C), bf16 in, fp32
 * accumulate.  A is [M][K] (K contiguous, leading dimension lda); B is [N][K]
 * (b_mn_major = 0) or [K][N] (b_mn_major = 1); C and D are [M][N].  M must be
 * a multiple of 128, N of 256, K of 64; pointers 16-byte aligned, leading
 * dimensions multiples of 8.  Replaces the torch.addmm calls of
 * Muon_util._newton_schulz_iteration (Muon_util.py:98-114).  `err`, if set,
 * receives 1 when a bounded wait gave up. */
int advopt_ns_gemm(void* D, int32_t ldd, const void* A, int32_t lda, const void* B, int32_t ldb, int32_t b_mn_major,
                   const void* C, int32_t ldc, int32_t M, int32_t N, int32_t K, float alpha, float beta,
                   int32_t* err, void* stream);

/*
 * Muon_adv / AdaMuon_adv: the elementwise work around the Newton–Schulz
 * GEMMs for ONE 2-D (or flattened) matrix.  The host runs, in order:
 *   stage 0  momentum (+ Nesterov, + AdaMuon's sign projection), the
 *            momentum_buffer store, X0 = bf16(update), ||X0|| (bf16) and
 *            X = bf16(X0 / max(||X0||, ns_eps)) into the zero-padded
 *            workspace `ns` ([m_pad][n_pad], transposed when rows > cols);
 *   the Newton–Schulz chain with advopt_ns_gemm on the workspace;
 *   Muon:    stage 1 (U = result in the param's layout, RMS scale), stage 2
 *            (param update);
 *   AdaMuon: stage 3 (U), stage 4 (second moment statistics + RMS scale),
 *            stage 5 (second_momentum_buffer store + param update).
 * Replaces Muon_adv._muon_step_parameter (Muon_adv.py:443-555) and
 * AdaMuon_adv._muon_step_parameter (AdaMuon_adv.py:492-659) for non-factored
 * matrices, with Muon_util.rms_adjustment (Muon_util.py:362-372) and
 * param_update.apply_parameter_update (param_update.py:77-156).
 */
#define ADVOPT_MU_NESTEROV (1u << 0)
#define ADVOPT_MU_SIGN (1u << 1)      /* AdaMuon kappa_p = 1: sign(update) before NS */
#define ADVOPT_MU_SR (1u << 2)        /* stochastic rounding of bf16 params */
#define ADVOPT_MU_CAUTIOUS (1u << 3)
#define ADVOPT_MU_NOISE_IN (1u << 4)  /* read SR noise from noise_* */
#define ADVOPT_MU_RMS (1u << 5)       /* rms_rescaling */
#define ADVOPT_MU_TRANSPOSED (1u << 6)/* rows > cols: the workspace holds X^T */
#define ADVOPT_MU_ATAN2 (1u << 7)     /* AdaMuon use_atan2 */
#define ADVOPT_MU_MARS (1u << 8)      /* approx_mars: g' = (g - last_grad) * mars_factor + g */
#define ADVOPT_MU_NORMUON (1u << 9)   /* normuon_variant: stages 7, 8, 9 */
#define ADVOPT_MU_VFACT (1u << 10)    /* AdaMuon factored_2nd: stages 10, 11 */
#define ADVOPT_MU_LOWRANK (1u << 11)  /* low_rank_ortho: stage 0 stops after X0 (no norm, no workspace load) */

/* storage codes of momentum_buffer / second_momentum_buffer */
#define ADVOPT_ST_F32 0
#define ADVOPT_ST_BF16 1      /* bf16, round to nearest ('auto' with bf16 params) */
#define ADVOPT_ST_BF16_SR 2   /* bf16, stochastic rounding ('bf16_sr')           */
#define ADVOPT_ST_Q8 3        /* int8 / uint8 codes + 2048-element block scales   */

typedef struct advopt_muon_args {
  void* param;               /* p (f32 or bf16), [rows][cols] flattened          */
  const void* grad;
  void* m;                   /* momentum_buffer                                  */
  float* m_scale;            /* momentum_buffer_scale (ADVOPT_ST_Q8)             */
  void* v;                   /* AdaMuon second_momentum_buffer                   */
  float* v_scale;
  uint16_t* x0;              /* scratch bf16 [numel]                             */
  uint16_t* ns;              /* workspace X, bf16 [m_pad][ld_ns]                 */
  const uint16_t* ns_result; /* the chain's final X (stages 1 and 3)             */
  uint16_t* u;               /* scratch bf16 [numel]: U in the param's layout    */
  double* partial;           /* scratch [max(ceil(numel/2048), tiles32)]         */
  float* scalars;            /* scratch [4]: ||X0|| (bf16 value), update scale   */
  const int32_t* noise_m;
  const int32_t* noise_v;
  const int32_t* noise_p;
  int64_t numel;
  int64_t rows;              /* p.shape[0]                                       */
  int64_t cols;              /* numel / rows                                     */
  int64_t ld_ns;             /* workspace leading dimension (= n_pad)            */
  int64_t m_pad;             /* workspace rows: min(rows, cols) rounded up to 256 */
  int64_t n_pad;             /* workspace cols: max(rows, cols) rounded up to 256 */
  uint64_t seed;             /* Philox key                                       */
  float w_m;                 /* 1 - beta1                                        */
  float w_nest;              /* Nesterov coefficient (grad.lerp(m, coef))        */
  float beta2;               /* AdaMuon                                          */
  float c_v;                 /* AdaMuon 1 - beta2                                */
  float eps;                 /* AdaMuon eps (or 1/sqrt(numel))                   */
  float ns_eps;              /* Newton–Schulz norm clamp                         */
  float wd;                  /* weight_decay * lr (0: none)                      */
  float scale_const;         /* rms: step_scale*0.2*sqrt(numel); else lr*sqrt(max(1, r/c)) */
  uint32_t tensor_id;
  uint32_t step;
  uint32_t flags;            /* ADVOPT_MU_*                                      */
  int32_t m_storage;         /* ADVOPT_ST_*                                      */
  int32_t v_storage;
  int32_t param_bf16;        /* 1: bf16 params, 0: f32                           */
  int32_t math_bf16;         /* 1: momentum and AdaMuon math in bf16 ('auto', bf16 params) */
  int32_t update_bf16;       /* 1: the orthogonalised update is bf16 (else f32)  */
  /* approx MARS-M (Muon_util.py:333-347) */
  void* last_grad;           /* state['last_grad'] (param dtype), rewritten      */
  float mars_factor;         /* float(mars_gamma * beta1 / (1 - beta1))          */
  /* NorMuon (Muon_util.py:349-360): row-wise second moment after the chain */
  float nm_w;                /* lerp weight 1 - beta2 (Muon: beta2_normuon)      */
  float nm_eps;              /* normuon_eps (AdaMuon: eps)                        */
  int32_t pad0;
  float* row_v;              /* state['normuon_v'] [rows] f32, rewritten          */
  float* row_den;            /* scratch [rows]: sqrt(v) + eps                    */
  /* AdaMuon factored_2nd (AdaMuon_adv.py:617-631): v = outer(v_row, v_col) */
  float* v_row;              /* mu_vbuf_nmf [d1], rewritten                      */
  float* v_col;              /* mv_vbuf_nmf [d2], rewritten                      */
  float* v_full;             /* scratch f32 [numel]: the updated v               */
  double* v_sums;            /* scratch f64 [d1 + kVColSplit * d2]: row sums, column partials */
  int64_t d1, d2;            /* effective shape (factorization_util.py:43-50)    */
} advopt_muon_args;

/* column partial sums of the AdaMuon factored v: d1 rows are cut into this
 * many row ranges, each summed per column; the finish adds them in order */
#define ADVOPT_VCOL_SPLIT 16

/* Low-rank Newton–Schulz (Muon_util.py:239-270), bf16 operands, float32
 * accumulation, one rounding of each product to bf16:
 *   advopt_lr_sketch  S [n][r] ~ N(0, 1) (Philox4x32-10, Box–Muller), the sketch
 *   advopt_lr_gemm    D [M][N] = op(A) B; op(A) = A [M][K], or A^T with A stored [K][M] (trans_a)
 *   advopt_lr_qr      Q [m][r] = the Q factor of A [m][r] (shifted CholeskyQR3 in float64;
 *                     `work` holds advopt_lr_qr_work(m, r) doubles)
 * The host chain: MG = M S, Q = qr(MG), P = Q^T M, the ordinary chain on P
 * (stage 6 with P as its input, then stage 3), U = Q NS(P). */
int advopt_lr_sketch(uint16_t* S, int64_t n, int64_t r, uint64_t seed, uint32_t tensor_id, uint32_t step,
                     void* stream);
int advopt_lr_gemm(uint16_t* D, const uint16_t* A, const uint16_t* B, int64_t M, int64_t N, int64_t K,
                   int32_t trans_a, void* stream);
int64_t advopt_lr_qr_work(int64_t m, int64_t r);
int advopt_lr_qr(uint16_t* Q, const uint16_t* A, int64_t m, int64_t r, double* work, void* stream);

/* Peer copies for the sharded parameter gather (copy engines, no SMs):
 *   advopt_ipc_get_handle  the CUDA IPC handle (64 bytes) of the allocation holding
 *                          ptr, and ptr's byte offset in it
 *   advopt_ipc_open        map another process's allocation; advopt_ipc_close unmaps it
 *   advopt_enable_peer     peer access to another device of this process
 *   advopt_copy_async      device-to-device cudaMemcpyAsync on `stream` */
int advopt_ipc_get_handle(const void* ptr, void* handle_out, uint64_t* offset_out);
int advopt_ipc_open(const void* handle, void** base_out);
int advopt_ipc_close(void* base);
int advopt_enable_peer(int32_t peer_device);
int advopt_copy_async(void* dst, const void* src, uint64_t bytes, void* stream);

/* Stages (one matrix per call sequence):
 *   0 momentum / X0 / norm / workspace load     6 the same for a bare Newton–Schulz call
 *   1 U store + RMS scale, 2 Muon update        3 U store only
 *   4 AdaMuon statistics + scale, 5 AdaMuon second moment + update
 *   7 NorMuon rows (v, sqrt(v) + eps per row), 8 NorMuon statistics + scale, 9 NorMuon update
 *   10 AdaMuon factored statistics + scale + new factors, 11 AdaMuon factored update
 *   13 sum(U^2) of the U already in `u` + RMS scale (Muon after a low-rank chain) */
int advopt_muon_stage(const advopt_muon_args* args, int32_t stage, void* stream);

/* The stochastic-rounding noise generator.  No reference counterpart: the
 * reference draws torch.randint from a generator seeded 42
 * (param_update.py:159-204); the kernels draw counter-based Philox4x32-10
 * instead (or the reference's own integers in the test mode).
 *   advopt_philox4x32_10: n raw evaluations; counters_keys holds n records
 *     {c0, c1, c2, c3, k0, k1}, out receives n x 4 words (device pointers).
 *   advopt_noise_fill: the n 16-bit values a kernel draws for elements
 *     0 .. n-1 of tensor `tensor_id` at `step` from noise stream `stream_id`
 *     (0 = v, 1 = m, 2 = param); counter = (k >> 3, stream_id << 24,
 *     tensor_id, step), key = seed, element k takes half (k & 1) of word
 *     (k & 7) >> 1. */
int advopt_philox4x32_10(const uint32_t* counters_keys, uint32_t* out, int64_t n, void* stream);
int advopt_noise_fill(uint16_t* out, int64_t n, uint64_t seed, uint32_t tensor_id, uint32_t step,
                      uint32_t stream_id, void* stream);

/* advopt_ns_gemm for a product the caller knows to be symmetric (D = D^T:
 * A @ B symmetric and C symmetric or unused), M == N a multiple of 256: only
 * the 256 x 256 blocks on or above the diagonal are computed; every
 * off-diagonal block is also stored transposed below the diagonal.  Replaces
 * the two symmetric addmm calls of each quintic iteration, A = X X^T and
 * B = b A + c A A (Muon_util.py:108-112). */
int advopt_ns_gemm_sym(void* D, int32_t ldd, const void* A, int32_t lda, const void* B, int32_t ldb,
                       int32_t b_mn_major, const void* C, int32_t ldc, int32_t M, int32_t K, float alpha, float beta,
                       int32_t* err, void* stream);

/* The whole Newton–Schulz chain on a loaded workspace with advopt_ns_gemm:
 * x, c are [m_pad][n_pad] bf16 (x holds the normalised input), a, b are
 * [m_pad][m_pad] (b unused for CANS).  Quintic: `steps` iterations of
 * A = X X^T, B = coef_b A + coef_c A A, X = coef_a X + B X.  CANS (cns != 0):
 * A = X X^T, X = c1 X + c3 A X with (c1, c3) from the bounds starting at
 * [cns_lower_bound, 1], computed in double as Muon_util.py:69-105 does.
 * *final_x receives the buffer holding the result (x or c).  Replaces the
 * loops of Muon_util._newton_schulz_iteration (Muon_util.py:78-114). */
int advopt_ns_chain(void* x, void* c, void* a, void* b, int32_t m_pad, int32_t n_pad, int32_t steps, int32_t cns,
                    double coef_a, double coef_b, double coef_c, double cns_lower_bound, void** final_x,
                    int32_t* err, void* stream);

/* Layout checks for bindings: sizeof of each struct. */
size_t advopt_sizeof(int which); /* 0 adam_tensor, 1 piece, 2 adam_launch, 3 lion_tensor, 4 muon_args */
int advopt_abi_version(void);
/* Last error message of the calling thread ("" if none). */
const char* advopt_last_error(void);
/* Number of SMs and the Adam kernel's resident CTAs per SM for a given
 * dynamic shared-memory size (floats), for the general (fast = 0) or the
 * fast-path (fast = 1) kernel; used by the host planner. */
int advopt_adam_occupancy(int32_t precision, int32_t param_dtype, int32_t algo, int32_t smem_floats,
                          int32_t fast, int32_t* sm_count, int32_t* ctas_per_sm);

#ifdef __cplusplus
}
#endif
#endif /* ADVOPT_H_ */
