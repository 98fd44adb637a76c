// Multi-tensor Adam-family step (AdamW_adv, Muon's auxiliary Adam, Prodigy_adv)
// for sm_100a.  One persistent launch covers a whole parameter group: the host
// planner cuts the group's tensors into "pieces" (contiguous, 2048-aligned
// element ranges; row-aligned for factored tensors) and gives every CTA a
// contiguous run of pieces with an equal share of elements.
//
// Per CTA iteration a chunk of 2048 consecutive elements of one tensor — one
// int8_sr quantisation block (state_util.py:10) — is held in registers, 8
// elements per thread, loaded with 128-bit accesses.  Everything the reference
// does to those elements in ~30 eager passes happens in this one pass:
//   moment updates (AdamW_adv.py:401-453, Muon_AuxAdam.py:135-180,
//   Prodigy_adv.py:436-483), bias correction, the block absmax / max and the
//   stochastic re-quantisation of int8/uint8 states (state_util.py:109-163),
//   bf16 stochastic rounding (param_update.py:206-219), the rank-1 factor row
//   sums and column partials of factored_2nd (factorization_util.py:60-80),
//   weight decay incl. cautious/centered/Fisher (param_update.py:15-156), and
//   Prodigy's slice statistics (Prodigy_adv.py:495-511).
#include "advopt.h"
#include "common.cuh"
#include "capi_internal.h"

namespace advopt {

template <int PREC, bool PBF>
struct StateTraits {
  // m / v storage: 0 f32, 1 bf16, 2 int8 (m) / uint8 (v)
  static constexpr int kStore = PREC == ADVOPT_PREC_FP32 ? 0
                              : PREC == ADVOPT_PREC_BF16_SR ? 1
                              : PREC == ADVOPT_PREC_INT8_SR ? 2
                              : (PBF ? 1 : 0);
  // math in bf16 (each tensor op rounds to bf16): 'auto' with bf16 params
  static constexpr bool kMathBF = PREC == ADVOPT_PREC_AUTO && PBF;
  // states written with stochastic rounding (bf16_sr) rather than RNE
  static constexpr bool kSRStates = PREC == ADVOPT_PREC_BF16_SR;
};

struct TensorRegs {
  const void* grad;
  void* param;
  void* m;
  float* m_scale;
  void* v;
  float* v_scale;
  float* row;
  float* col;
  float* colpart;
  void* aux0;
  void* aux1;
  void* aux2;
  const int32_t* nz_v;
  const int32_t* nz_m;
  const int32_t* nz_p;
  int64_t numel, d1, d2;
  float step_size, sqrt_bc2, eps, wd, cwd, fisher_clip;
  uint32_t tensor_id, step, flags, slice_p;
};

__device__ __forceinline__ void load_tensor(const advopt_adam_tensor* t, TensorRegs& r) {
  r.grad = t->grad; r.param = t->param; r.m = t->exp_avg; r.m_scale = t->exp_avg_scale;
  r.v = t->exp_avg_sq; r.v_scale = t->exp_avg_sq_scale; r.row = t->row_factor; r.col = t->col_factor;
  r.colpart = t->col_partial; r.aux0 = t->aux0; r.aux1 = t->aux1; r.aux2 = t->aux2;
  r.nz_v = t->noise_v; r.nz_m = t->noise_m; r.nz_p = t->noise_p;
  r.numel = t->numel; r.d1 = t->d1; r.d2 = t->d2;
  r.step_size = t->step_size; r.sqrt_bc2 = t->sqrt_bc2; r.eps = t->eps; r.wd = t->wd; r.cwd = t->cwd;
  r.fisher_clip = t->fisher_clip;
  r.tensor_id = t->tensor_id; r.step = t->step; r.flags = t->flags; r.slice_p = t->slice_p;
}

// Noise for 8 elements: injected int32 array or Philox.
__device__ __forceinline__ void noise8(const advopt_adam_launch& L, const TensorRegs& T, const int32_t* arr,
                                       uint32_t stream, int64_t k0, int nv, uint32_t (&r)[8]) {
  if (L.flags & ADVOPT_F_NOISE_IN) {
#pragma unroll
    for (int e = 0; e < 8; ++e) r[e] = e < nv ? (uint32_t)arr[k0 + e] : 0u;
  } else {
    philox_u16x8(L.seed, T.tensor_id, T.step, stream, k0, r);
  }
}

// Centered-WD anchor value of element k as float (centered_decay.py:219-261).
__device__ __forceinline__ float anchor_value(const TensorRegs& T, int64_t k, bool pbf) {
  const uint32_t mode = (T.flags >> ADVOPT_T_ANCHOR_SHIFT) & 7u;
  if (mode == ADVOPT_ANCHOR_FULL) {
    return pbf ? bf16_to_f(static_cast<const uint16_t*>(T.aux0)[k]) : static_cast<const float*>(T.aux0)[k];
  }
  if (mode == ADVOPT_ANCHOR_FP8) {
    return fp8e4m3_to_f(static_cast<const uint8_t*>(T.aux0)[k]);
  }
  int q;
  int64_t blk;
  float qmin;
  if (mode == ADVOPT_ANCHOR_INT8) {
    q = (int)static_cast<const int8_t*>(T.aux0)[k];
    blk = k >> 7;
    qmin = -128.0f;
  } else {
    const int b = (int)static_cast<const int8_t*>(T.aux0)[k >> 1];
    q = (k & 1) ? ((int)(int8_t)(b << 4) >> 4) : (b >> 4);
    blk = k >> 5;
    qmin = -8.0f;
  }
  float s, mn;
  if (pbf) {
    s = bf16_to_f(static_cast<const uint16_t*>(T.aux1)[blk]);
    mn = bf16_to_f(static_cast<const uint16_t*>(T.aux2)[blk]);
  } else {
    s = static_cast<const float*>(T.aux1)[blk];
    mn = static_cast<const float*>(T.aux2)[blk];
  }
  return __fadd_rn(__fmul_rn(__fsub_rn((float)q, qmin), s), mn);
}

// _apply_weight_decay for one element (param_update.py:15-75).  `pc` is the
// working param value; `rb` rounds to the working dtype (bf16 for the
// non-SR bf16 path).  wd/cwd are already scaled by lr (and by the Fisher
// scaler `ws` when ws_on).
template <bool RB>
__device__ __forceinline__ float weight_decay(float pc, float u, float wd, float cwd, bool cautious, bool has_anchor,
                                              float anchor, bool ws_on, float ws) {
  auto R = [](float x) { return RB ? round_bf16(x) : x; };
  if (wd != 0.0f) {
    const float tgt = pc;
    if (cautious) {
      const float mask = R(__fmul_rn(u, tgt)) >= 0.0f ? 1.0f : 0.0f;
      if (ws_on) {
        const float sw = __fmul_rn(ws, wd);                       // wd_scaler * scaled_wd
        pc = R(__fmaf_rn(__fmul_rn(-1.0f, tgt), __fmul_rn(mask, sw), pc));
      } else {
        pc = R(__fmaf_rn(__fmul_rn(-wd, tgt), mask, pc));
      }
    } else {
      if (ws_on) {
        pc = R(__fmaf_rn(__fmul_rn(-1.0f, tgt), __fmul_rn(ws, wd), pc));
      } else {
        pc = R(__fmaf_rn(tgt, -wd, pc));
      }
    }
  }
  if (cwd != 0.0f && has_anchor) {
    const float tgt = R(__fsub_rn(pc, R(anchor)));
    if (cautious) {
      const float mask = R(__fmul_rn(u, tgt)) >= 0.0f ? 1.0f : 0.0f;
      if (ws_on) {
        const float sw = __fmul_rn(ws, cwd);
        pc = R(__fmaf_rn(__fmul_rn(-1.0f, tgt), __fmul_rn(mask, sw), pc));
      } else {
        pc = R(__fmaf_rn(__fmul_rn(-cwd, tgt), mask, pc));
      }
    } else {
      if (ws_on) {
        pc = R(__fmaf_rn(__fmul_rn(-1.0f, tgt), __fmul_rn(ws, cwd), pc));
      } else {
        pc = R(__fmaf_rn(tgt, -cwd, pc));
      }
    }
  }
  return pc;
}

// The denominator the Fisher scaler sees (update_util.py:15-36): the
// reference passes `denom` before its cast to the update dtype, which only
// differs from the cast value for factored tensors under bf16 'auto' math.
template <int ALGO>
__device__ __forceinline__ float fisher_den(float v, float den_u, const TensorRegs& T, bool fact, bool mbf) {
  if (!(mbf && fact)) return den_u;
  float den = __fsqrt_rn(v);
  if (ALGO == ADVOPT_ALGO_PRODIGY) return __fadd_rn(den, T.eps);
  return __fadd_rn(__fdiv_rn(den, T.sqrt_bc2), T.eps);
}

template <int PREC, bool PBF, int ALGO, bool EXT>
__global__ void __launch_bounds__(kThreads, 3) adam_kernel(const advopt_adam_launch L) {
  using TR = StateTraits<PREC, PBF>;
  constexpr int kStore = TR::kStore;
  constexpr bool kMBF = TR::kMathBF;
  // dynamic shared memory: [0, max d2) column accumulators of the factored
  // tensor in progress; from gen_offset, the generic factored path's staged
  // chunk (2048 floats) and row-segment sums (2049 floats)
  extern __shared__ float dsm[];
  float* colacc = dsm;
  float* vbuf = dsm + L.gen_offset;
  float* segs = vbuf + kChunk;
  __shared__ float red[2][kWarps][4];         // per-chunk block reductions (double-buffered)
  __shared__ double dred[kWarps][2];

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t F = L.flags;
  const bool has_m = F & ADVOPT_F_HAS_M;
  const bool nest = F & ADVOPT_F_NESTEROV;
  const bool atan2m = EXT && (F & ADVOPT_F_ATAN2);
  const bool normed = EXT && (ALGO == ADVOPT_ALGO_ADAMW) && (F & ADVOPT_F_NORMED);
  const bool cautious = F & ADVOPT_F_CAUTIOUS;
  const bool sr = PBF && (F & ADVOPT_F_SR);
  const bool fisher = EXT && (F & ADVOPT_F_FISHER);
  const bool fstats = EXT && (F & ADVOPT_F_FISHER_STATS);
  // the Fisher statistics pass writes nothing but piece_stats
  const bool pstats = (ALGO == ADVOPT_ALGO_PRODIGY) && (F & ADVOPT_F_PRODIGY_STATS) && !fstats;
  auto Rm = [](float x) { return kMBF ? round_bf16(x) : x; };  // rounding of m / update / grad ops
  int parity = 0;

  const int pbeg = L.cta_offsets[blockIdx.x], pend = L.cta_offsets[blockIdx.x + 1];
  __shared__ TensorRegs T;  // descriptor of the piece's tensor, read field by field when needed
  for (int pi = pbeg; pi < pend; ++pi) {
    const advopt_piece pc = L.pieces[pi];
    __syncthreads();  // previous piece finished with T
    if (tid == 0) load_tensor(L.tensors + pc.tensor, T);
    __syncthreads();
    const bool fact = T.flags & ADVOPT_T_FACTORED;
    const bool vec = T.flags & ADVOPT_T_VEC;
    const bool has_anchor = EXT && (((T.flags >> ADVOPT_T_ANCHOR_SHIFT) & 7u) != 0);
    // factored row/column sums are skipped in the Fisher statistics pass
    const bool fact_sums = fact && !fstats;
    const int64_t d2 = fact ? T.d2 : 1;
    // fast factored path: every chunk holds each column at most once and each
    // thread's 8 elements sit in one row with 8 aligned factor columns
    const bool ffast = fact && d2 >= kChunk && (d2 % 8) == 0;
    const bool vbf = kMBF && !fact;  // v math in bf16 ('auto' bf16, not factored)
    if (fact_sums) {
      for (int j = tid; j < (int)d2; j += kThreads) colacc[j] = 0.0f;
      __syncthreads();
    }
    int64_t r0 = fact ? pc.begin / d2 : 0;
    int64_t c0 = fact ? pc.begin - r0 * d2 : 0;
    double row_carry = 0.0;  // thread 0: running sum of the row in progress
    double st0 = 0.0, st1 = 0.0;
    const uint32_t slice_p = T.slice_p ? T.slice_p : 1u;

    for (int64_t cs = pc.begin; cs < pc.end; cs += kChunk) {
      const int clen = (int)min((int64_t)kChunk, pc.end - cs);
      const int64_t k0 = cs + tid * kVec;
      const int nv = max(0, min(kVec, clen - tid * kVec));
      const bool v8 = vec && nv == kVec;
      const int64_t blk = cs / kChunk;

      float g[8], p[8], m[8], vh[8];
      load8<PBF>(T.grad, k0, nv, v8, g);
      load8<PBF>(T.param, k0, nv, v8, p);
      if (has_m) {
        if (kStore == 2) {
          const float sc = T.m_scale[blk];
          load8_q<true>(T.m, k0, nv, v8, m);
#pragma unroll
          for (int e = 0; e < 8; ++e) m[e] = __fmul_rn(m[e], sc);
        } else if (kStore == 1) {
          load8<true>(T.m, k0, nv, v8, m);
        } else {
          load8<false>(T.m, k0, nv, v8, m);
        }
      }
      if (fact) {
        // v_hat = outer(mu, mv) (factorization_util.py:53-57)
        if (ffast) {
          const int64_t cc = c0 + tid * kVec;
          const bool second = cc >= d2;
          const int64_t col = second ? cc - d2 : cc;
          float mv[8];
          load8<false>(T.col, col, 8, (reinterpret_cast<uintptr_t>(T.col) & 15) == 0, mv);
          const float mu = nv > 0 ? T.row[r0 + (second ? 1 : 0)] : 0.0f;
#pragma unroll
          for (int e = 0; e < 8; ++e) vh[e] = __fmul_rn(mu, mv[e]);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            vh[e] = 0.0f;
            if (e < nv) {
              const int64_t cc = c0 + tid * kVec + e;
              const int64_t dr = cc / d2;
              vh[e] = __fmul_rn(T.row[r0 + dr], T.col[cc - dr * d2]);
            }
          }
        }
      } else {
        if (kStore == 2) {
          const float sc = T.v_scale[blk];
          load8_q<false>(T.v, k0, nv, v8, vh);
#pragma unroll
          for (int e = 0; e < 8; ++e) vh[e] = __fmul_rn(vh[e], sc);
        } else if (kStore == 1) {
          load8<true>(T.v, k0, nv, v8, vh);
        } else {
          load8<false>(T.v, k0, nv, v8, vh);
        }
      }
      uint32_t rp[8];
      if (sr && !fstats) noise8(L, T, T.nz_p, kNoiseP, k0, nv, rp);
      int slice_off = 0;  // offset of the next Prodigy slice point from k0
      if (pstats) slice_off = (int)((slice_p - (uint32_t)(k0 % slice_p)) % slice_p);

      // ---- per-element arithmetic, in the reference's op order; the param
      // update does not depend on the block statistics and is done here ----
      float m_new[8], v[8];
      float amax_m = 0.0f, vmax = 0.0f;
      uint32_t pout[8];
      float pout_f[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const bool ok = e < nv;
        float gi = g[e];
        // v = v*beta2 + c_v*g*g   (mul_ then addcmul_, AdamW_adv.py:417, Prodigy_adv.py:469)
        float vi = __fmul_rn(vh[e], L.beta2);
        if (vbf) vi = round_bf16(vi);
        vi = __fmaf_rn(__fmul_rn(L.c_v, gi), gi, vi);
        if (vbf) vi = round_bf16(vi);
        if (fact) vi = fabsf(vi);       // _factorize_state's abs_ (factorization_util.py:35)
        v[e] = ok ? vi : 0.0f;
        // denominator (AdamW_adv.py:424-431, Prodigy_adv.py:477-482)
        float den = __fsqrt_rn(vi);
        if (vbf) den = round_bf16(den);
        if (ALGO != ADVOPT_ALGO_PRODIGY) {
          den = __fdiv_rn(den, T.sqrt_bc2);
          if (vbf) den = round_bf16(den);
        }
        if (!atan2m) {
          den = __fadd_rn(den, T.eps);   // Prodigy: T.eps holds d*eps
          if (vbf) den = round_bf16(den);
        }
        const float du = kMBF ? round_bf16(den) : den;   // denom.to(update.dtype)
        if (normed) gi = atan2m ? Rm(atan2f(gi, du)) : Rm(__fdiv_rn(gi, du));
        // first moment and the update direction
        float ui;
        if (has_m) {
          float mi;
          if (ALGO == ADVOPT_ALGO_PRODIGY) {
            mi = Rm(__fmaf_rn(gi, L.c_m, Rm(__fmul_rn(m[e], L.beta1))));
          } else {
            mi = Rm(lerp_t(m[e], gi, L.w_m));
          }
          m_new[e] = ok ? mi : 0.0f;
          ui = nest ? Rm(lerp_t(mi, gi, L.w_nest)) : mi;
        } else {
          m_new[e] = 0.0f;
          ui = (ALGO == ADVOPT_ALGO_PRODIGY) ? Rm(__fmul_rn(gi, L.d)) : gi;
        }
        if (!normed) ui = atan2m ? Rm(atan2f(ui, du)) : Rm(__fdiv_rn(ui, du));
        ui = Rm(__fmul_rn(ui, T.step_size));
        amax_m = fmaxf(amax_m, fabsf(m_new[e]));
        vmax = fmaxf(vmax, v[e]);

        // Prodigy slice statistics on p before its update (Prodigy_adv.py:501-509)
        if (pstats && ok && e >= slice_off && ((e - slice_off) % (int)slice_p) == 0) {
          const int64_t si = (k0 + e) / slice_p;
          float p0v = 0.0f;
          if (!(T.flags & ADVOPT_T_P0_SCALAR))
            p0v = PBF ? bf16_to_f(static_cast<const uint16_t*>(T.aux1)[si]) : static_cast<const float*>(T.aux1)[si];
          st0 += (double)gi * (double)__fsub_rn(p0v, p[e]);
          const float s_old = PBF ? bf16_to_f(static_cast<const uint16_t*>(T.aux0)[si])
                                  : static_cast<const float*>(T.aux0)[si];
          float s1 = __fmul_rn(s_old, L.beta3);
          if (PBF) s1 = round_bf16(s1);
          float s2 = __fmaf_rn(gi, L.s_alpha, s1);
          if (PBF) {
            const uint32_t b = f_to_bf16_rne(s2);
            static_cast<uint16_t*>(T.aux0)[si] = (uint16_t)b;
            s2 = bf16_to_f(b);
          } else {
            static_cast<float*>(T.aux0)[si] = s2;
          }
          st1 += (double)fabsf(s2);
        }

        // Fisher weight decay scaler (update_util.py:15-36)
        float ws = 0.0f;
        if (fisher || fstats) {
          const float dn = fisher_den<ALGO>(vi, du, T, fact, kMBF);
          if (fstats) {
            const float pw = __fmul_rn(p[e], __fdiv_rn(1.0f, dn));
            if (ok) st0 += (double)__fmul_rn(pw, pw);
          } else if (atan2m) {
            ws = __fmul_rn(atan2f(1.0f, dn), (float)(4.0 / 3.14159265358979323846));
          } else {
            ws = __fdiv_rn(__fdiv_rn(1.0f, dn), T.fisher_clip);
          }
        }
        // parameter update (param_update.py:77-156)
        const float anc = (has_anchor && ok) ? anchor_value(T, k0 + e, PBF) : 0.0f;
        if (PBF && !sr) {
          const float pcv = weight_decay<true>(p[e], ui, T.wd, T.cwd, cautious, has_anchor, anc, fisher, ws);
          pout[e] = f_to_bf16_rne(__fadd_rn(pcv, -ui));
        } else {
          const float pcv = weight_decay<false>(p[e], ui, T.wd, T.cwd, cautious, has_anchor, anc, fisher, ws);
          const float pn = __fadd_rn(pcv, -ui);
          if (PBF) pout[e] = f_to_bf16_sr(pn, rp[e]);
          else pout_f[e] = pn;
        }
      }
      if (!fstats) {
        if (PBF) store8_bf16(T.param, k0, nv, v8, pout);
        else store8_f32(T.param, k0, nv, v8, pout_f);
      }

      // ---- factored second moment: row sums and column partials ----
      float rsum0 = 0.0f, rsum1 = 0.0f;
      if (fact_sums) {
        if (ffast) {
          const int64_t cc = c0 + tid * kVec;
          const bool second = cc >= d2;
          const int64_t col = second ? cc - d2 : cc;
          float s = 0.0f;
          if (nv > 0) {
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              s = __fadd_rn(s, v[e]);
              colacc[col + e] = __fadd_rn(colacc[col + e], v[e]);
            }
          }
          if (second) rsum1 = s; else rsum0 = s;
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (e < nv) vbuf[tid * kVec + e] = v[e];
        }
      }

      // ---- block reductions (one barrier per chunk) ----
      {
        const float a = warp_max(amax_m), b = warp_max(vmax), c = warp_sum(rsum0), d = warp_sum(rsum1);
        if (lane == 0) {
          red[parity][warp][0] = a;
          red[parity][warp][1] = b;
          red[parity][warp][2] = c;
          red[parity][warp][3] = d;
        }
      }
      __syncthreads();

      if (fact_sums) {
        if (ffast) {
          if (tid == 0) {
            float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) {
              s0 = __fadd_rn(s0, red[parity][w][2]);
              s1 = __fadd_rn(s1, red[parity][w][3]);
            }
            row_carry += (double)s0;
            if (clen >= d2 - c0) {         // row r0 completes in this chunk
              T.row[r0] = (float)row_carry;
              row_carry = (double)s1;
            }
          }
        } else {
          // generic: each column's elements in this chunk, summed in order by
          // the thread that owns its first occurrence
          const int ncol = (int)min((int64_t)clen, d2);
          for (int pp = tid; pp < ncol; pp += kThreads) {
            float acc = 0.0f;
            for (int q = pp; q < clen; q += (int)d2) acc = __fadd_rn(acc, vbuf[q]);
            int64_t j = c0 + pp;
            if (j >= d2) j -= d2;
            colacc[j] = __fadd_rn(colacc[j], acc);
          }
          // rows: segment s covers chunk positions [max(0, s*d2-c0), min(clen, (s+1)*d2-c0))
          const int nseg = (int)((c0 + clen - 1) / d2) + 1;
          for (int s = warp; s < nseg; s += kWarps) {
            const int64_t lo = max((int64_t)0, (int64_t)s * d2 - c0);
            const int64_t hi = min((int64_t)clen, (int64_t)(s + 1) * d2 - c0);
            float acc = 0.0f;
            for (int64_t q = lo + lane; q < hi; q += 32) acc = __fadd_rn(acc, vbuf[q]);
            acc = warp_sum(acc);
            if (lane == 0) segs[s] = acc;
          }
          __syncthreads();
          if (tid == 0) {
            for (int s = 0; s < nseg; ++s) {
              row_carry += (double)segs[s];
              if ((int64_t)(s + 1) * d2 - c0 <= clen) {   // row r0+s ends in this chunk
                T.row[r0 + s] = (float)row_carry;
                row_carry = 0.0;
              }
            }
          }
          __syncthreads();
        }
      }

      // ---- store the new moments (they need the block max) ----
      if (!fstats) {
        if (has_m) {
          if (kStore == 2) {
            float bmax = 0.0f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) bmax = fmaxf(bmax, red[parity][w][0]);
            const float scale = __fdiv_rn(bmax, 127.0f);
            const float safe = scale < 1e-12f ? 1e-12f : scale;
            uint32_t r[8], c[8];
            noise8(L, T, T.nz_m, kNoiseM, k0, nv, r);
#pragma unroll
            for (int e = 0; e < 8; ++e) c[e] = quant_code(m_new[e], safe, r[e], false);
            store8_q(T.m, k0, nv, v8, c);
            if (tid == 0) T.m_scale[blk] = scale;
          } else if (kStore == 1) {
            uint32_t b[8];
            if (TR::kSRStates) {
              uint32_t r[8];
              noise8(L, T, T.nz_m, kNoiseM, k0, nv, r);
#pragma unroll
              for (int e = 0; e < 8; ++e) b[e] = f_to_bf16_sr(m_new[e], r[e]);
            } else {
#pragma unroll
              for (int e = 0; e < 8; ++e) b[e] = f_to_bf16_rne(m_new[e]);
            }
            store8_bf16(T.m, k0, nv, v8, b);
          } else {
            store8_f32(T.m, k0, nv, v8, m_new);
          }
        }
        if (!fact) {
          if (kStore == 2) {
            float bmax = 0.0f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) bmax = fmaxf(bmax, red[parity][w][1]);
            const float scale = __fdiv_rn(bmax, 255.0f);
            const float safe = scale < 1e-12f ? 1e-12f : scale;
            uint32_t r[8], c[8];
            noise8(L, T, T.nz_v, kNoiseV, k0, nv, r);
#pragma unroll
            for (int e = 0; e < 8; ++e) c[e] = quant_code(v[e], safe, r[e], true);
            store8_q(T.v, k0, nv, v8, c);
            if (tid == 0) T.v_scale[blk] = scale;
          } else if (kStore == 1) {
            uint32_t b[8];
            if (TR::kSRStates) {
              uint32_t r[8];
              noise8(L, T, T.nz_v, kNoiseV, k0, nv, r);
#pragma unroll
              for (int e = 0; e < 8; ++e) b[e] = f_to_bf16_sr(v[e], r[e]);
            } else {
#pragma unroll
              for (int e = 0; e < 8; ++e) b[e] = f_to_bf16_rne(v[e]);
            }
            store8_bf16(T.v, k0, nv, v8, b);
          } else {
            store8_f32(T.v, k0, nv, v8, v);
          }
        }
      }

      // advance the factored row/column position by one chunk
      if (fact) {
        c0 += clen;
        if (c0 >= d2) {
          const int64_t dr = c0 / d2;
          r0 += dr;
          c0 -= dr * d2;
        }
      }
      parity ^= 1;
    }

    // ---- end of piece: flush column partials and statistics ----
    if (fact_sums) {
      __syncthreads();
      float* dst = T.colpart + (int64_t)pc.slot * d2;
      for (int j = tid; j < (int)d2; j += kThreads) dst[j] = colacc[j];
      __syncthreads();
    }
    if (pstats || fstats) {
      const double a = warp_sum_d(st0), b = warp_sum_d(st1);
      if (lane == 0) {
        dred[warp][0] = a;
        dred[warp][1] = b;
      }
      __syncthreads();
      if (tid == 0) {
        double sa = 0.0, sb = 0.0;
        for (int w = 0; w < kWarps; ++w) {
          sa += dred[w][0];
          sb += dred[w][1];
        }
        L.piece_stats[2 * pi] = sa;
        L.piece_stats[2 * pi + 1] = sb;
      }
      __syncthreads();
    }
  }
}


// ---------------------------------------------------------------------------
// factored_2nd finish: column sums from the partials, then normalise one
// factor (factorization_util.py:60-80).  Kernel A sums partial rows in slot
// order (float64) into mv; kernel B normalises mu (d1 < d2) or mv by its total.
// ---------------------------------------------------------------------------
__global__ void factored_cols_kernel(const advopt_adam_tensor* tensors, const int32_t* index) {
  const advopt_adam_tensor* t = tensors + index[blockIdx.y];
  const int64_t d2 = t->d2;
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= d2) return;
  double acc = 0.0;
  const float* src = t->col_partial + j;
  for (int s = 0; s < t->n_slots; ++s) acc += (double)src[(int64_t)s * d2];
  t->col_factor[j] = (float)acc;
}

__global__ void factored_norm_kernel(const advopt_adam_tensor* tensors, const int32_t* index) {
  const advopt_adam_tensor* t = tensors + index[blockIdx.x];
  const int64_t d1 = t->d1, d2 = t->d2;
  float* vec = d1 < d2 ? t->row_factor : t->col_factor;
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

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
template <int PREC, bool PBF, int ALGO>
static cudaError_t launch_one(const advopt_adam_launch& L, cudaStream_t s) {
  const bool ext = L.flags & (ADVOPT_F_ATAN2 | ADVOPT_F_NORMED | ADVOPT_F_FISHER | ADVOPT_F_FISHER_STATS |
                              ADVOPT_F_ANCHORS);
  auto k = ext ? adam_kernel<PREC, PBF, ALGO, true> : adam_kernel<PREC, PBF, ALGO, false>;
  const size_t smem = (size_t)L.smem_floats * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  k<<<L.grid, kThreads, smem, s>>>(L);
  return cudaGetLastError();
}

template <int PREC, bool PBF, int ALGO>
static cudaError_t occupancy_one(int smem_floats, int* ctas) {
  auto k = adam_kernel<PREC, PBF, ALGO, false>;
  const size_t smem = (size_t)smem_floats * sizeof(float);
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(ctas, k, kThreads, smem);
}

#define ADVOPT_DISPATCH(FN, PREC, PBF, ALGO, ...)                                                  \
  [&]() -> cudaError_t {                                                                           \
    switch (ALGO) {                                                                                \
      case ADVOPT_ALGO_ADAMW: return FN<PREC, PBF, ADVOPT_ALGO_ADAMW>(__VA_ARGS__);                \
      case ADVOPT_ALGO_AUXADAM: return FN<PREC, PBF, ADVOPT_ALGO_AUXADAM>(__VA_ARGS__);            \
      default: return FN<PREC, PBF, ADVOPT_ALGO_PRODIGY>(__VA_ARGS__);                             \
    }                                                                                              \
  }()

template <class Fn>
static cudaError_t dispatch(int prec, int pdt, Fn&& fn) {
  return fn(prec, pdt);
}

static cudaError_t run_adam(const advopt_adam_launch& L, cudaStream_t s) {
  const bool pbf = L.param_dtype == ADVOPT_DT_BF16;
  switch (L.precision) {
    case ADVOPT_PREC_FP32:
      return pbf ? ADVOPT_DISPATCH(launch_one, ADVOPT_PREC_FP32, true, L.algo, L, s)
                 : ADVOPT_DISPATCH(launch_one, ADVOPT_PREC_FP32, false, L.algo, L, s);
    case ADVOPT_PREC_BF16_SR:
      return pbf ? ADVOPT_DISPATCH(launch_one, ADVOPT_PREC_BF16_SR, true, L.algo, L, s)
                 : ADVOPT_DISPATCH(launch_one, ADVOPT_PREC_BF16_SR, false, L.algo, L, s);
    case ADVOPT_PREC_INT8_SR:
      return pbf ? ADVOPT_DISPATCH(launch_one, ADVOPT_PREC_INT8_SR, true, L.algo, L, s)
                 : ADVOPT_DISPATCH(launch_one, ADVOPT_PREC_INT8_SR, false, L.algo, L, s);
    default:  // AUTO: f32 params are exactly the FP32 path
      return pbf ? ADVOPT_DISPATCH(launch_one, ADVOPT_PREC_AUTO, true, L.algo, L, s)
                 : ADVOPT_DISPATCH(launch_one, ADVOPT_PREC_FP32, false, L.algo, L, s);
  }
}

static cudaError_t run_occupancy(int prec, int pdt, int algo, int smem_floats, int* ctas) {
  const bool pbf = pdt == ADVOPT_DT_BF16;
  switch (prec) {
    case ADVOPT_PREC_FP32:
      return pbf ? ADVOPT_DISPATCH(occupancy_one, ADVOPT_PREC_FP32, true, algo, smem_floats, ctas)
                 : ADVOPT_DISPATCH(occupancy_one, ADVOPT_PREC_FP32, false, algo, smem_floats, ctas);
    case ADVOPT_PREC_BF16_SR:
      return pbf ? ADVOPT_DISPATCH(occupancy_one, ADVOPT_PREC_BF16_SR, true, algo, smem_floats, ctas)
                 : ADVOPT_DISPATCH(occupancy_one, ADVOPT_PREC_BF16_SR, false, algo, smem_floats, ctas);
    case ADVOPT_PREC_INT8_SR:
      return pbf ? ADVOPT_DISPATCH(occupancy_one, ADVOPT_PREC_INT8_SR, true, algo, smem_floats, ctas)
                 : ADVOPT_DISPATCH(occupancy_one, ADVOPT_PREC_INT8_SR, false, algo, smem_floats, ctas);
    default:
      return pbf ? ADVOPT_DISPATCH(occupancy_one, ADVOPT_PREC_AUTO, true, algo, smem_floats, ctas)
                 : ADVOPT_DISPATCH(occupancy_one, ADVOPT_PREC_FP32, false, algo, smem_floats, ctas);
  }
}

}  // namespace advopt

using namespace advopt;

extern "C" int advopt_adam_step(const advopt_adam_launch* L, void* stream) {
  if (!L || !L->tensors || !L->pieces || !L->cta_offsets || L->grid <= 0)
    return set_error(ADVOPT_E_INVALID, "advopt_adam_step: null table or empty grid");
  if (L->precision < 0 || L->precision > 3 || L->algo < 0 || L->algo > 2 || L->param_dtype < 0 || L->param_dtype > 1)
    return set_error(ADVOPT_E_INVALID, "advopt_adam_step: bad precision/algo/dtype code");
  if ((L->flags & (ADVOPT_F_PRODIGY_STATS | ADVOPT_F_FISHER_STATS)) && !L->piece_stats)
    return set_error(ADVOPT_E_INVALID, "advopt_adam_step: statistics requested without piece_stats");
  if (L->smem_floats < 0 || L->smem_floats > 49152)
    return set_error(ADVOPT_E_INVALID, "advopt_adam_step: factored d2 above 49152 columns is not supported");
  return check_cuda(run_adam(*L, static_cast<cudaStream_t>(stream)), "advopt_adam_step");
}

extern "C" int advopt_factored_finish(const advopt_adam_launch* L, const int32_t* index, int32_t n_factored,
                                      int32_t max_d2, void* stream) {
  if (!L || (n_factored > 0 && !index)) return set_error(ADVOPT_E_INVALID, "advopt_factored_finish: null argument");
  if (n_factored <= 0) return ADVOPT_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  dim3 ga((unsigned)((max_d2 + 255) / 256), (unsigned)n_factored);
  factored_cols_kernel<<<ga, 256, 0, s>>>(L->tensors, index);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return check_cuda(e, "advopt_factored_finish");
  factored_norm_kernel<<<n_factored, 1024, 0, s>>>(L->tensors, index);
  return check_cuda(cudaGetLastError(), "advopt_factored_finish");
}

extern "C" int advopt_prodigy_finish(const advopt_adam_launch* L, float* sums, float coef, int32_t s_is_bf16,
                                     void* stream) {
  if (!L || !sums || !L->piece_stats) return set_error(ADVOPT_E_INVALID, "advopt_prodigy_finish: null argument");
  prodigy_finish_kernel<<<1, 256, 0, static_cast<cudaStream_t>(stream)>>>(*L, sums, coef, s_is_bf16);
  return check_cuda(cudaGetLastError(), "advopt_prodigy_finish");
}

extern "C" int advopt_fisher_finish(const advopt_adam_launch* L, advopt_adam_tensor* tensors_rw, void* stream) {
  if (!L || !tensors_rw || !L->piece_stats) return set_error(ADVOPT_E_INVALID, "advopt_fisher_finish: null argument");
  fisher_finish_kernel<<<L->n_tensors, 256, 0, static_cast<cudaStream_t>(stream)>>>(*L, tensors_rw);
  return check_cuda(cudaGetLastError(), "advopt_fisher_finish");
}

extern "C" int advopt_adam_occupancy(int32_t precision, int32_t param_dtype, int32_t algo, int32_t smem_floats,
                                     int32_t* sm_count, int32_t* ctas_per_sm) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return check_cuda(e, "advopt_adam_occupancy");
  int sms = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return check_cuda(e, "advopt_adam_occupancy");
  int ctas = 0;
  e = run_occupancy(precision, param_dtype, algo, smem_floats, &ctas);
  if (e != cudaSuccess) return check_cuda(e, "advopt_adam_occupancy");
  if (sm_count) *sm_count = sms;
  if (ctas_per_sm) *ctas_per_sm = ctas;
  return ADVOPT_OK;
}
