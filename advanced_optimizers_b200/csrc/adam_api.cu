// Adam-family host dispatch, the factored/Prodigy/Fisher finishing kernels
// and the C entry points (include/advopt.h).
#include "adam_impl.cuh"

namespace advopt {

// ---------------------------------------------------------------------------
// factored_2nd / 'factored' finish: column sums from the partials, then
// normalise one factor (factorization_util.py:60-80).  Kernel A sums partial
// rows in slot order (float64) into mv; kernel B normalises mu (d1 < d2) or
// mv by its total.  blockIdx.z / blockIdx.y = 1 does the same for the signed
// momentum's |m| factors of ADVOPT_T_FACT_M tensors.  Both leave the factors
// untouched when the step's error word is set: a CTA whose bounded wait gave
// up has not written its column partials.
// ---------------------------------------------------------------------------
__global__ void factored_cols_kernel(const advopt_adam_tensor* tensors, const int32_t* index, const int32_t* err) {
  if (err && *err) return;
  const advopt_adam_tensor* t = tensors + index[blockIdx.y];
  const bool mom = blockIdx.z == 1;
  if (mom && (!(t->flags & ADVOPT_T_FACT_M) || !t->m_col_partial)) return;
  if (!mom && !t->col_partial) return;     // factored Lion: no second moment
  const int64_t d2 = t->d2;
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= d2) return;
  double acc = 0.0;
  const float* src = (mom ? t->m_col_partial : t->col_partial) + j;
  for (int s = 0; s < t->n_slots; ++s) acc += (double)src[(int64_t)s * d2];
  (mom ? t->m_col_factor : t->col_factor)[j] = (float)acc;
}

__global__ void factored_norm_kernel(const advopt_adam_tensor* tensors, const int32_t* index, const int32_t* err) {
  if (err && *err) return;
  const advopt_adam_tensor* t = tensors + index[blockIdx.x];
  const bool mom = blockIdx.y == 1;
  if (mom && (!(t->flags & ADVOPT_T_FACT_M) || !t->m_col_partial)) return;
  if (!mom && !t->col_partial) return;
  const int64_t d1 = t->d1, d2 = t->d2;
  float* vec = mom ? (d1 < d2 ? t->m_row_factor : t->m_col_factor) : (d1 < d2 ? t->row_factor : t->col_factor);
  const int64_t n = d1 < d2 ? d1 : d2;
  __shared__ double part[32];
  double acc = 0.0;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) acc += (double)vec[i];
  acc = warp_sum_d(acc);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  __shared__ float scale_s;
  if (threadIdx.x == 0) {
    double tot = 0.0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += part[w];
    float sc = (float)tot;
    scale_s = sc < 1e-12f ? 1e-12f : sc;     // scale.clamp_min_(1e-12)
  }
  __syncthreads();
  const float sc = scale_s;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) vec[i] = __fdiv_rn(vec[i], sc);
}

// Prodigy: per-tensor sums of the piece statistics, folded in param order.
__global__ void prodigy_finish_kernel(const advopt_adam_launch L, float* sums, float coef, int s_is_bf16) {
  __shared__ double dot_s[256], abs_s[256];
  if (L.prodigy) coef = L.prodigy->coef;
  float num = sums[0], den = sums[1];
  // pieces of tensor t are found by scanning all pieces (launch sizes are small)
  for (int t = 0; t < L.n_tensors; ++t) {
    double a = 0.0, b = 0.0;
    for (int i = threadIdx.x; i < L.n_pieces; i += blockDim.x) {
      if (L.pieces[i].tensor == t) {
        a += L.piece_stats[2 * i];
        b += L.piece_stats[2 * i + 1];
      }
    }
    dot_s[threadIdx.x] = a;
    abs_s[threadIdx.x] = b;
    __syncthreads();
    for (int o = blockDim.x / 2; o > 0; o >>= 1) {
      if ((int)threadIdx.x < o) {
        dot_s[threadIdx.x] += dot_s[threadIdx.x + o];
        abs_s[threadIdx.x] += abs_s[threadIdx.x + o];
      }
      __syncthreads();
    }
    if (threadIdx.x == 0) {
      const float dot = (float)dot_s[0];
      num = __fadd_rn(num, __fmul_rn(coef, dot));              // d_numerator.add_((d/d0)*dlr*dot)
      float sabs = (float)abs_s[0];
      if (s_is_bf16) sabs = round_bf16(sabs);                 // s.abs().sum() is bf16 for bf16 s
      den = __fadd_rn(den, sabs);
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    sums[0] = num;
    sums[1] = den;
  }
}

// Python's two-argument min / max: the first argument unless the second is
// strictly smaller / larger.
__device__ __forceinline__ double py_min(double a, double b) { return b < a ? b : a; }
__device__ __forceinline__ double py_max(double a, double b) { return b > a ? b : a; }

// Prodigy step scalars from the device d (Prodigy_adv.py:345-346, 404-520).
__global__ void prodigy_scalars_kernel(const advopt_prodigy_scalar_args a) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  advopt_prodigy_dev* P = a.dev;
  const double d = P->d, d0 = P->d0;
  const double dlr = d * a.lr;
  P->c_v = (float)(d * d * (1.0 - a.beta2));
  P->c_m = (float)(d * (1.0 - a.beta1));
  P->d_f = (float)d;
  P->s_alpha = (float)(a.safeguard_warmup ? (d / d0) * d : (d / d0) * dlr);
  P->coef = (float)((d / d0) * dlr);
  const float ss = (float)(a.step_scale == 1.0 ? dlr : dlr * a.step_scale);
  for (int t = 0; t < a.n_tensors; ++t) {
    advopt_adam_tensor& T = a.tensors[t];
    const double* c = a.tensor_consts + 3 * t;
    T.step_size = ss;
    T.eps = (float)(d * c[0]);
    T.wd = c[1] != 0.0 ? (float)(c[1] * dlr) : 0.0f;
    T.cwd = c[2] != 0.0 ? (float)(c[2] * dlr) : 0.0f;
  }
}

// calculate_d + init_step's carry (Prodigy_adv.py:246-257, 540-572).
__global__ void prodigy_update_d_kernel(const advopt_prodigy_d_args a) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  advopt_prodigy_dev* P = a.dev;
  if (a.active) {
    const double gn = (double)P->sums[0], gd = (double)P->sums[1];
    double d = P->d, d_max = P->d_max;
    if (gd > 0.0) {
      double d_hat = a.d_coef * gn / gd;
      if (a.d_limiter) d_hat = py_min(d * a.limiter_factor, d_hat);
      if (d == P->d0) d = py_max(d, d_hat);
      d_max = py_max(d_max, d_hat);
      d = py_min(d_max, d * a.growth_rate);
    }
    P->d = d;
    P->d_max = d_max;
    P->d_numerator = gn;
  }
  P->sums[0] = (float)(P->d_numerator * a.beta3) * (float)a.carry_scale;
  P->sums[1] = 0.0f;
}

// Kourkoutas-beta: per-layer EMA and dynamic beta2 (Kourkoutas.py:131-187).
__global__ void kourkoutas_prepare_kernel(const advopt_kourkoutas_args a) {
  const int l = blockIdx.x * blockDim.x + threadIdx.x;
  if (l >= a.n_layers) return;
  const float pooled = __fsqrt_rn(a.acc[l]);
  float e = __fmul_rn(a.ema[l], a.ema_alpha);
  e = __fmaf_rn(a.one_minus_alpha, pooled, e);           // add_(pooled, alpha=1 - ema_alpha)
  a.ema[l] = e;
  const float raw = __fdiv_rn(pooled, __fadd_rn(e, a.tiny_spike));
  const float sun = __fdiv_rn(raw, __fadd_rn(1.0f, raw));
  const float target = __fsub_rn(a.beta2_max, __fmul_rn(a.beta2_min_gap, sun));
  const float b2 = __fadd_rn(a.one_minus_w_bmax, __fmul_rn(a.w, target));
  a.layer_beta2[2 * l] = b2;
  // value=1.0 - beta2 (AdamW) or d * d * (1.0 - beta2) (Prodigy) with beta2 a Python float
  const double cv = a.d_dev ? a.d_dev[0] * a.d_dev[0] : a.cv_scale;
  a.layer_beta2[2 * l + 1] = (float)(cv * (1.0 - (double)b2));
  a.acc[l] = 0.0f;
}

// Kourkoutas-beta: each tensor's sum of g*g (its pieces, in order) into its
// layer's accumulator, tensors in launch order (Kourkoutas.py:231-247).
__global__ void kourkoutas_accumulate_kernel(const advopt_kourkoutas_args a) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  // the planner lays the tensors end to end, so one tensor's pieces are
  // consecutive and the tensors come in launch order
  int i = 0;
  while (i < a.n_pieces) {
    const int t = a.pieces[i].tensor;
    double s = 0.0;
    for (; i < a.n_pieces && a.pieces[i].tensor == t; ++i) s += a.piece_gsq[i];
    float v = (float)s;
    if (a.gsq_bf16) v = round_bf16(v);
    const int l = a.layer_of_tensor[t];
    if (l >= 0) a.acc[l] = __fadd_rn(a.acc[l], v);
  }
}

// Fisher: rms of p*ws per tensor -> 1/max(1, rms) stored as fisher_clip (the
// divisor clip_coef itself; update_util.py:26-36).
__global__ void fisher_finish_kernel(const advopt_adam_launch L, advopt_adam_tensor* tensors_rw) {
  const int t = blockIdx.x;
  __shared__ double part[256];
  double a = 0.0;
  for (int i = threadIdx.x; i < L.n_pieces; i += blockDim.x)
    if (L.pieces[i].tensor == t) a += L.piece_stats[2 * i];
  part[threadIdx.x] = a;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if ((int)threadIdx.x < o) part[threadIdx.x] += part[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const double n = (double)tensors_rw[t].numel;
    const float mean = (float)(part[0] / n);
    const float rms = __fsqrt_rn(mean);
    tensors_rw[t].fisher_clip = rms > 1.0f ? rms : 1.0f;
  }
}


cudaError_t run_adam(const advopt_adam_launch& L, cudaStream_t s) {
  switch (L.precision) {
    case ADVOPT_PREC_FP32: return launch_adam_fp32(L, s);
    case ADVOPT_PREC_BF16_SR: return launch_adam_bf16sr(L, s);
    case ADVOPT_PREC_INT8_SR: return launch_adam_int8(L, s);
    default:  // AUTO: f32 params are exactly the FP32 path
      return L.param_dtype == ADVOPT_DT_BF16 ? launch_adam_auto(L, s) : launch_adam_fp32(L, s);
  }
}

cudaError_t run_occupancy(int prec, int pdt, int algo, int smem_floats, int* ctas, int fast) {
  switch (prec) {
    case ADVOPT_PREC_FP32: return occupancy_adam_fp32(pdt, algo, smem_floats, ctas, fast);
    case ADVOPT_PREC_BF16_SR: return occupancy_adam_bf16sr(pdt, algo, smem_floats, ctas, fast);
    case ADVOPT_PREC_INT8_SR: return occupancy_adam_int8(pdt, algo, smem_floats, ctas, fast);
    default: return pdt == ADVOPT_DT_BF16 ? occupancy_adam_auto(pdt, algo, smem_floats, ctas, fast)
                                          : occupancy_adam_fp32(pdt, algo, smem_floats, ctas, fast);
  }
}

}  // namespace advopt

using namespace advopt;

extern "C" int advopt_adam_step(const advopt_adam_launch* L, void* stream) {
  if (!L || !L->tensors || !L->pieces || !L->cta_offsets || L->grid <= 0)
    return set_error(ADVOPT_E_INVALID, "advopt_adam_step: null table or empty grid");
  if (L->precision < 0 || L->precision > 3 || L->algo < 0 || L->algo > 3 || L->param_dtype < 0 || L->param_dtype > 1)
    return set_error(ADVOPT_E_INVALID, "advopt_adam_step: bad precision/algo/dtype code");
  if ((L->flags & (ADVOPT_F_PRODIGY_STATS | ADVOPT_F_FISHER_STATS)) && !L->piece_stats)
    return set_error(ADVOPT_E_INVALID, "advopt_adam_step: statistics requested without piece_stats");
  if ((L->flags & ADVOPT_F_GRAD_SQ) && !L->piece_gsq)
    return set_error(ADVOPT_E_INVALID, "advopt_adam_step: ADVOPT_F_GRAD_SQ without piece_gsq");
  if ((L->layer_beta2 != nullptr) != (L->layer_of_tensor != nullptr))
    return set_error(ADVOPT_E_INVALID, "advopt_adam_step: layer_beta2 and layer_of_tensor go together");
  if (L->smem_floats < 0 || L->smem_floats > 56832)
    return set_error(ADVOPT_E_INVALID, "advopt_adam_step: shared memory request above 227 KB (factored d2 too large)");
  if (L->stages < 0 || L->stages > 4) return set_error(ADVOPT_E_INVALID, "advopt_adam_step: stages must be 0..4");
  if (L->algo == ADVOPT_ALGO_LION &&
      ((L->precision != ADVOPT_PREC_FP32 && L->precision != ADVOPT_PREC_AUTO) || !(L->flags & ADVOPT_F_HAS_M) ||
       L->stages != 0 || (L->flags & (ADVOPT_F_ATAN2 | ADVOPT_F_NORMED | ADVOPT_F_FISHER | ADVOPT_F_FISHER_STATS))))
    return set_error(ADVOPT_E_INVALID, "advopt_adam_step: Lion launches are float32 or 'auto', general-kernel only");
  if ((L->flags & ADVOPT_F_FACT_M) && (L->precision != ADVOPT_PREC_FP32 || !(L->flags & ADVOPT_F_HAS_M) ||
                                       (L->smem_floats % 2) != 0))
    return set_error(ADVOPT_E_INVALID,
                     "advopt_adam_step: factored momentum needs ADVOPT_PREC_FP32, ADVOPT_F_HAS_M and an even "
                     "shared-memory split");
  if ((L->flags & ADVOPT_F_EMIT_UPDATE) && (L->flags & (ADVOPT_F_FISHER | ADVOPT_F_FISHER_STATS)))
    return set_error(ADVOPT_E_INVALID, "advopt_adam_step: update emission with Fisher weight decay");
  return check_cuda(run_adam(*L, static_cast<cudaStream_t>(stream)), "advopt_adam_step");
}

namespace advopt {
cudaError_t run_factored_finish(const advopt_adam_tensor* tensors, const int32_t* index, int n_factored, int max_d2,
                                const int32_t* err, cudaStream_t s) {
  dim3 ga((unsigned)((max_d2 + 255) / 256), (unsigned)n_factored, 2u);
  factored_cols_kernel<<<ga, 256, 0, s>>>(tensors, index, err);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  factored_norm_kernel<<<dim3((unsigned)n_factored, 2u), 1024, 0, s>>>(tensors, index, err);
  return cudaGetLastError();
}
}  // namespace advopt

extern "C" int advopt_factored_finish(const advopt_adam_launch* L, const int32_t* index, int32_t n_factored,
                                      int32_t max_d2, void* stream) {
  if (!L || (n_factored > 0 && !index)) return set_error(ADVOPT_E_INVALID, "advopt_factored_finish: null argument");
  if (n_factored <= 0) return ADVOPT_OK;
  return check_cuda(run_factored_finish(L->tensors, index, n_factored, max_d2, L->err,
                                        static_cast<cudaStream_t>(stream)),
                    "advopt_factored_finish");
}

extern "C" int advopt_kourkoutas_prepare(const advopt_kourkoutas_args* a, void* stream) {
  if (!a || !a->acc || !a->ema || !a->layer_beta2 || a->n_layers < 0)
    return set_error(ADVOPT_E_INVALID, "advopt_kourkoutas_prepare: null argument");
  if (a->n_layers == 0) return ADVOPT_OK;
  kourkoutas_prepare_kernel<<<(a->n_layers + 127) / 128, 128, 0, static_cast<cudaStream_t>(stream)>>>(*a);
  return check_cuda(cudaGetLastError(), "advopt_kourkoutas_prepare");
}

extern "C" int advopt_kourkoutas_accumulate(const advopt_kourkoutas_args* a, void* stream) {
  if (!a || !a->acc || !a->layer_of_tensor || !a->piece_gsq || !a->pieces || a->n_tensors < 0 || a->n_pieces < 0)
    return set_error(ADVOPT_E_INVALID, "advopt_kourkoutas_accumulate: null argument");
  kourkoutas_accumulate_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(*a);
  return check_cuda(cudaGetLastError(), "advopt_kourkoutas_accumulate");
}

extern "C" int advopt_prodigy_finish(const advopt_adam_launch* L, float* sums, float coef, int32_t s_is_bf16,
                                     void* stream) {
  if (!L || !sums || !L->piece_stats) return set_error(ADVOPT_E_INVALID, "advopt_prodigy_finish: null argument");
  prodigy_finish_kernel<<<1, 256, 0, static_cast<cudaStream_t>(stream)>>>(*L, sums, coef, s_is_bf16);
  return check_cuda(cudaGetLastError(), "advopt_prodigy_finish");
}

extern "C" int advopt_prodigy_scalars(const advopt_prodigy_scalar_args* a, void* stream) {
  if (!a || !a->dev || a->n_tensors < 0 || (a->n_tensors > 0 && (!a->tensors || !a->tensor_consts)))
    return set_error(ADVOPT_E_INVALID, "advopt_prodigy_scalars: null argument");
  prodigy_scalars_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(*a);
  return check_cuda(cudaGetLastError(), "advopt_prodigy_scalars");
}

extern "C" int advopt_prodigy_update_d(const advopt_prodigy_d_args* a, void* stream) {
  if (!a || !a->dev) return set_error(ADVOPT_E_INVALID, "advopt_prodigy_update_d: null argument");
  prodigy_update_d_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(*a);
  return check_cuda(cudaGetLastError(), "advopt_prodigy_update_d");
}

extern "C" int advopt_fisher_finish(const advopt_adam_launch* L, advopt_adam_tensor* tensors_rw, void* stream) {
  if (!L || !tensors_rw || !L->piece_stats) return set_error(ADVOPT_E_INVALID, "advopt_fisher_finish: null argument");
  fisher_finish_kernel<<<L->n_tensors, 256, 0, static_cast<cudaStream_t>(stream)>>>(*L, tensors_rw);
  return check_cuda(cudaGetLastError(), "advopt_fisher_finish");
}

extern "C" int advopt_adam_occupancy(int32_t precision, int32_t param_dtype, int32_t algo, int32_t smem_floats,
                                     int32_t fast, int32_t* sm_count, int32_t* ctas_per_sm) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return check_cuda(e, "advopt_adam_occupancy");
  int sms = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return check_cuda(e, "advopt_adam_occupancy");
  int ctas = 0;
  e = run_occupancy(precision, param_dtype, algo, smem_floats, &ctas, fast);
  if (e != cudaSuccess) return check_cuda(e, "advopt_adam_occupancy");
  if (sm_count) *sm_count = sms;
  if (ctas_per_sm) *ctas_per_sm = ctas;
  return ADVOPT_OK;
}
