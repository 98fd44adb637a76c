/*
 * ORACLE — test infrastructure only.
 *
 * Plain-C restatement of the per-element arithmetic that adv_optm 2.5.4 gets
 * from PyTorch's CPU kernels (ATen, torch 2.11).  Only tests/, the smoke check
 * and bench.py's CPU-baseline leg load this library, and only as the checker /
 * the CPU baseline: the product never links or calls it.
 *
 * Compile with -ffp-contract=off (see oracle/Makefile): every fused
 * multiply-add below is an explicit fmaf(), matching the ATen vectorised CPU
 * kernels, and nothing else may be contracted.  The FMA placement of each
 * primitive was pinned against torch's CPU output bit for bit
 * (tests/golden/make_golden.py records the reference's own outputs).
 *
 * Values that the reference keeps in bfloat16 travel here as float32 arrays
 * holding exactly-representable bf16 values, plus explicit bf16 rounding
 * (orc_round_bf16) at the points where ATen rounds.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

static inline uint32_t f2u(float x) { uint32_t u; memcpy(&u, &x, 4); return u; }
static inline float u2f(uint32_t u) { float x; memcpy(&x, &u, 4); return x; }

/* float -> bf16 bits, round-to-nearest-even, NaN -> 0x7FC0
 * (c10::BFloat16 round_to_nearest_even, used by every ATen float->bf16 cast). */
static inline uint16_t bf16_rne(float x) {
  if (x != x) return 0x7FC0u;
  uint32_t u = f2u(x);
  uint32_t bias = ((u >> 16) & 1u) + 0x7FFFu;
  return (uint16_t)((u + bias) >> 16);
}
static inline float bf16_to_f(uint16_t b) { return u2f(((uint32_t)b) << 16); }

/* torch.lerp(self, end, w) with a scalar weight.  ATen's CPU kernel
 * (LerpKernel.cpp, lerp_vec) evaluates fmadd(coeff, end - self, base) with
 * coeff = w, base = self when |w| < 0.5, else coeff = w - 1, base = end.
 * Used by AdamW_adv.py:437,443, Muon_adv.py:513,518, AdaMuon_adv.py:584,588,
 * Lion_adv.py:262,265. */
static inline float lerp1(float self, float end, float w) {
  if (fabsf(w) < 0.5f) return fmaf(w, end - self, self);
  return fmaf(w - 1.0f, end - self, end);
}

void orc_lerp(float* out, const float* self, const float* end, float w, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = lerp1(self[i], end[i], w);
}

/* self.addcmul_(t1, t2, value=s): fmadd(s * t1, t2, self)
 * (PointwiseOpsKernel.cpp; AdamW_adv.py:417, AdaMuon_adv.py:637). */
void orc_addcmul(float* out, const float* self, const float* t1, const float* t2, float s, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = fmaf(s * t1[i], t2[i], self[i]);
}

/* self.add_(other, alpha=a): fmadd(other, a, self) (ufunc/add.h vectorised
 * path; param_update.py:48, Prodigy_adv.py:442). */
void orc_add_alpha(float* out, const float* self, const float* other, float a, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = fmaf(other[i], a, self[i]);
}

/* Round float32 values to bf16 (returns the bf16 values widened to float32). */
void orc_round_bf16(float* out, const float* x, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = bf16_to_f(bf16_rne(x[i]));
}

/* float32 -> bf16 bits (RNE). */
void orc_to_bf16_bits(uint16_t* out, const float* x, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = bf16_rne(x[i]);
}

/* Stochastic rounding to bf16 (param_update.py:206-219): add the 16-bit
 * random integer to the float's bit pattern (int32, wrapping), clear the low
 * 16 bits, and keep the high half.  The masked pattern converts to bf16
 * exactly except for NaN, which ATen's cast canonicalises to 0x7FC0. */
void orc_sr_bf16_bits(uint16_t* out, const float* x, const int32_t* r, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    uint32_t u = (f2u(x[i]) + (uint32_t)r[i]) & 0xFFFF0000u;
    float y = u2f(u);
    out[i] = (y != y) ? (uint16_t)0x7FC0u : (uint16_t)(u >> 16);
  }
}

/* Block-wise int8 stochastic quantisation over the flat index with
 * replicate padding (state_util.py:59-106,124-157 and
 * param_update.py:271-307,329-363).
 *   signed:   scale = absmax/127,  q = clamp(floor(x/max(scale,1e-12) + r/65536), -127, 127)
 *   non_neg:  scale = max/255,     q = clamp(floor(x/max(scale,1e-12) + r/65536),    0, 255)
 * Replicate padding repeats the last element, so the padded block's max equals
 * the max over the block's real elements.  `r` has one entry per padded
 * element (the reference draws randint over the padded numel,
 * param_update.py:256); element i uses r[i]. */
void orc_quant_block(void* q_out, float* scale_out, const float* x, const int32_t* r,
                     int64_t n, int64_t block, int non_neg) {
  int64_t nb = (n + block - 1) / block;
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nb; ++b) {
    int64_t s = b * block, e = s + block < n ? s + block : n;
    float mx = -INFINITY;
    int has_nan = 0;
    for (int64_t i = s; i < e; ++i) {
      float a = non_neg ? x[i] : fabsf(x[i]);
      if (a != a) has_nan = 1;
      else if (a > mx) mx = a;
    }
    if (has_nan) mx = NAN; /* amax propagates NaN */
    float scale = mx / (non_neg ? 255.0f : 127.0f);
    scale_out[b] = scale;
    float safe = scale < 1e-12f ? 1e-12f : scale; /* clamp_min(1e-12) */
    if (scale != scale) safe = scale;
    for (int64_t i = s; i < e; ++i) {
      float noise = (float)r[i] * (1.0f / 65536.0f);
      float y = floorf(x[i] / safe + noise);
      if (y != y) y = 0.0f; /* NaN casts to an unspecified code in ATen; pin it to 0 */
      if (non_neg) {
        y = y < 0.0f ? 0.0f : (y > 255.0f ? 255.0f : y);
        ((uint8_t*)q_out)[i] = (uint8_t)(int)y;
      } else {
        y = y < -127.0f ? -127.0f : (y > 127.0f ? 127.0f : y);
        ((int8_t*)q_out)[i] = (int8_t)(int)y;
      }
    }
  }
}

/* Dequantisation: q * scale[block] (state_util.py:40-52). */
void orc_dequant_block(float* out, const void* q, const float* scale, int64_t n, int64_t block, int non_neg) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    float qv = non_neg ? (float)((const uint8_t*)q)[i] : (float)((const int8_t*)q)[i];
    out[i] = qv * scale[i / block];
  }
}

/* torch.outer(row, col) in float32 (factorization_util.py:53-57). */
void orc_outer(float* out, const float* row, const float* col, int64_t d1, int64_t d2) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < d1; ++i)
    for (int64_t j = 0; j < d2; ++j) out[i * d2 + j] = row[i] * col[j];
}

/* Row and column sums of a (d1, d2) float32 matrix accumulated in float64
 * (the reference sums in float32 with ATen's cascade order; the float64 sum
 * is the exact value that both the reference and the device kernels
 * approximate). factorization_util.py:68-69. */
void orc_row_col_sums(double* rows, double* cols, const float* m, int64_t d1, int64_t d2) {
  for (int64_t j = 0; j < d2; ++j) cols[j] = 0.0;
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < d1; ++i) {
    double acc = 0.0;
    for (int64_t j = 0; j < d2; ++j) acc += (double)m[i * d2 + j];
    rows[i] = acc;
  }
  for (int64_t i = 0; i < d1; ++i)
    for (int64_t j = 0; j < d2; ++j) cols[j] += (double)m[i * d2 + j];
}

/* fmaf over arrays (used for one-off scalar chains that ATen fuses). */
void orc_fma(float* out, const float* a, const float* b, const float* c, int64_t n) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = fmaf(a[i], b[i], c[i]);
}

int orc_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* Threads of the OpenMP loops above (overrides OMP_NUM_THREADS, which a
 * launcher such as torchrun sets to 1). */
void orc_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
