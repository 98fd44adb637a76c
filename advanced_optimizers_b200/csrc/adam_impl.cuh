// Multi-tensor Adam-family step kernel template (included by adam_<precision>.cu) (AdamW_adv, Muon's auxiliary Adam, Prodigy_adv)
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
#pragma once

#include "advopt.h"
#include "capi_internal.h"
#include "common.cuh"

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
  float* mrow;
  float* mcol;
  float* mcolpart;
  uint8_t* msign;
  void* upd;
  int64_t numel, d1, d2;
  float step_size, sqrt_bc2, eps, wd, cwd, fisher_clip;
  uint32_t tensor_id, step, flags, slice_p;
};

__device__ __forceinline__ void load_tensor(const advopt_adam_tensor* t, TensorRegs& r) {
  r.grad = t->grad; r.param = t->param; r.m = t->exp_avg; r.m_scale = t->exp_avg_scale;
  r.v = t->exp_avg_sq; r.v_scale = t->exp_avg_sq_scale; r.row = t->row_factor; r.col = t->col_factor;
  r.colpart = t->col_partial; r.aux0 = t->aux0; r.aux1 = t->aux1; r.aux2 = t->aux2;
  r.nz_v = t->noise_v; r.nz_m = t->noise_m; r.nz_p = t->noise_p;
  r.mrow = t->m_row_factor; r.mcol = t->m_col_factor; r.mcolpart = t->m_col_partial; r.msign = t->m_sign;
  r.upd = t->update_out;
  r.numel = t->numel; r.d1 = t->d1; r.d2 = t->d2;
  r.step_size = t->step_size; r.sqrt_bc2 = t->sqrt_bc2; r.eps = t->eps; r.wd = t->wd; r.cwd = t->cwd;
  r.fisher_clip = t->fisher_clip;
  r.tensor_id = t->tensor_id; r.step = t->step; r.flags = t->flags; r.slice_p = t->slice_p;
}

// Centered-WD anchor value of element k as float (centered_decay.py:78-119).
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
// scaler `ws` when ws_on).  The non-cautious decay is add_(target, alpha=-wd),
// which on a bf16 tensor rounds alpha to bf16 first; addcmul_'s value stays
// float32.
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
        pc = R(__fmaf_rn(tgt, -R(wd), pc));
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
        pc = R(__fmaf_rn(tgt, -R(cwd), pc));
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


// ---------------------------------------------------------------------------
// Correctly rounded square root and division for the general kernel: the
// Newton–Markstein sequences of the fast kernel (Markstein 1990; Muller et
// al., Handbook of Floating-Point Arithmetic, ch. 5), used inside the ranges
// where they were checked against __fsqrt_rn / __fdiv_rn on B200
// (v in [2^-100, FLT_MAX]; 2^-50 <= d <= 2^24 and 2^-100 <= |u| <= 2^64),
// IEEE division / square root outside them.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float sqrt_cr(float v) {
  if (!(v >= 0x1p-100f && v <= 3.402823466e38f)) return __fsqrt_rn(v);
  float y;
  asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(v));
  const float s = __fmul_rn(v, y);
  const float r = __fmaf_rn(-s, s, v);
  return __fmaf_rn(r, __fmul_rn(y, 0.5f), s);
}
__device__ __forceinline__ float div_cr(float u, float d) {
  const float au = fabsf(u);
  if (!(d >= 0x1p-50f && d <= 0x1p24f && au >= 0x1p-100f && au <= 0x1p64f)) return __fdiv_rn(u, d);
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(d));
  const float e = __fmaf_rn(-d, y, 1.0f);
  const float y1 = __fmaf_rn(e, y, y);
  const float q = __fmul_rn(u, y1);
  const float r = __fmaf_rn(-q, d, u);
  return __fmaf_rn(r, y1, q);
}

// ---------------------------------------------------------------------------
// Raw words of one thread's 8 elements of one chunk, as loaded from HBM; the
// next chunk's words are loaded while the current chunk is computed.
// ---------------------------------------------------------------------------
template <int BPE>
struct Words {
  static constexpr int N = 2 * BPE;  // 32-bit words for 8 elements
  uint32_t w[N];
};

template <int BPE>
__device__ __forceinline__ void ld_words(const void* base, int64_t k0, int nv, bool v8, Words<BPE>& out) {
  const unsigned char* p = static_cast<const unsigned char*>(base) + k0 * BPE;
  if (v8) {
    if (BPE == 1) {
      const uint2 q = __ldg(reinterpret_cast<const uint2*>(p));
      out.w[0] = q.x; out.w[1] = q.y;
    } else if (BPE == 2) {
      const uint4 q = __ldg(reinterpret_cast<const uint4*>(p));
      out.w[0] = q.x; out.w[1] = q.y; out.w[2] = q.z; out.w[3] = q.w;
    } else {
      const uint4 a = __ldg(reinterpret_cast<const uint4*>(p));
      const uint4 b = __ldg(reinterpret_cast<const uint4*>(p) + 1);
      out.w[0] = a.x; out.w[1] = a.y; out.w[2] = a.z; out.w[3] = a.w;
      out.w[4] = b.x; out.w[5] = b.y; out.w[6] = b.z; out.w[7] = b.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < Words<BPE>::N; ++i) out.w[i] = 0u;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      if (e < nv) {
        if (BPE == 1) out.w[e >> 2] |= (uint32_t)p[e] << (8 * (e & 3));
        else if (BPE == 2) out.w[e >> 1] |= (uint32_t)reinterpret_cast<const uint16_t*>(p)[e] << (16 * (e & 1));
        else out.w[e] = reinterpret_cast<const uint32_t*>(p)[e];
      }
    }
  }
}

// Unpack 8 elements to float: BPE 4 = f32, 2 = bf16, 1 = int8 (SIGNED) / uint8.
template <int BPE, bool SIGNED = true>
__device__ __forceinline__ void unpack8(const Words<BPE>& in, float (&x)[8]) {
  if (BPE == 4) {
#pragma unroll
    for (int e = 0; e < 8; ++e) x[e] = __uint_as_float(in.w[e]);
  } else if (BPE == 2) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      x[2 * i] = __uint_as_float(in.w[i] << 16);
      x[2 * i + 1] = __uint_as_float(in.w[i] & 0xFFFF0000u);
    }
  } else {
    codes4_to_f<SIGNED>(in.w[0], x);
    codes4_to_f<SIGNED>(in.w[1], x + 4);
  }
}

template <int kStore>
struct StoreBytes {
  static constexpr int v = kStore == 2 ? 1 : (kStore == 1 ? 2 : 4);
};

// Per-thread raw data of one chunk.
template <bool PBF, int kStore>
struct Raw {
  Words<PBF ? 2 : 4> g, p;
  Words<StoreBytes<kStore>::v> m, v;
  float mv[8];
  float mu, ms, vs;
  // signed rank-1 momentum (fast factored path): the thread's sign byte and factors
  float fmv[8];
  float fmu;
  uint32_t fsgn;
};

struct ChunkPos {
  int64_t cs;    // first element of the chunk
  int clen;      // elements in the chunk
  int64_t r0;    // factored: row of the chunk's first element
  int64_t c0;    // factored: its column
};

template <int PREC, bool PBF, int ALGO, bool EXT>
__device__ __forceinline__ void load_raw(const TensorRegs& T, const ChunkPos& cp, int tid, bool fact, bool ffast,
                                         bool has_m, bool vec, bool factm,
                                         Raw<PBF, StateTraits<PREC, PBF>::kStore>& R) {
  constexpr int kStore = StateTraits<PREC, PBF>::kStore;
  constexpr int SB = StoreBytes<kStore>::v;
  const int64_t k0 = cp.cs + tid * kVec;
  const int nv = max(0, min(kVec, cp.clen - tid * kVec));
  const bool v8 = vec && nv == kVec;
  const int64_t blk = cp.cs >> 11;
  ld_words<PBF ? 2 : 4>(T.grad, k0, nv, v8, R.g);
  ld_words<PBF ? 2 : 4>(T.param, k0, nv, v8, R.p);
  if (factm) {
    // signed rank-1 momentum: the generic path reads its factors per element
    if (ffast) {
      const int64_t cc = cp.c0 + tid * kVec;
      const bool second = cc >= T.d2;
      const int64_t col = second ? cc - T.d2 : cc;
      R.fmu = nv > 0 ? T.mrow[cp.r0 + (second ? 1 : 0)] : 0.0f;
      R.fsgn = nv > 0 ? (uint32_t)T.msign[k0 >> 3] : 0u;    // 8 elements = one sign byte
      const float4 a = *reinterpret_cast<const float4*>(T.mcol + col);
      const float4 b = *(reinterpret_cast<const float4*>(T.mcol + col) + 1);
      R.fmv[0] = a.x; R.fmv[1] = a.y; R.fmv[2] = a.z; R.fmv[3] = a.w;
      R.fmv[4] = b.x; R.fmv[5] = b.y; R.fmv[6] = b.z; R.fmv[7] = b.w;
    }
  } else if (has_m) {
    ld_words<SB>(T.m, k0, nv, v8, R.m);
    if (kStore == 2) R.ms = T.m_scale[blk];
  }
  if (ALGO == ADVOPT_ALGO_LION) {
    // Lion: no second moment
  } else if (fact) {
    if (ffast) {
      const int64_t cc = cp.c0 + tid * kVec;
      const bool second = cc >= T.d2;
      const int64_t col = second ? cc - T.d2 : cc;
      R.mu = nv > 0 ? T.row[cp.r0 + (second ? 1 : 0)] : 0.0f;
      const float4 a = *reinterpret_cast<const float4*>(T.col + col);
      const float4 b = *(reinterpret_cast<const float4*>(T.col + col) + 1);
      R.mv[0] = a.x; R.mv[1] = a.y; R.mv[2] = a.z; R.mv[3] = a.w;
      R.mv[4] = b.x; R.mv[5] = b.y; R.mv[6] = b.z; R.mv[7] = b.w;
    }
  } else {
    ld_words<SB>(T.v, k0, nv, v8, R.v);
    if (kStore == 2) R.vs = T.v_scale[blk];
  }
}

template <bool NOISE_IN>
__device__ __forceinline__ U4 noise_words(const advopt_adam_launch& L, const TensorRegs& T, const int32_t* arr,
                                          uint32_t stream, int64_t k0, int nv) {
  if (NOISE_IN) {
    uint32_t r[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) r[e] = e < nv ? ((uint32_t)arr[k0 + e] & 0xFFFFu) : 0u;
    return U4{r[0] | (r[1] << 16), r[2] | (r[3] << 16), r[4] | (r[5] << 16), r[6] | (r[7] << 16)};
  }
  const uint64_t grp = (uint64_t)k0 >> 3;
  U4 c{(uint32_t)grp, (uint32_t)(grp >> 32) | (stream << 24), T.tensor_id, T.step};
  return philox4x32_10(c, (uint32_t)L.seed, (uint32_t)(L.seed >> 32));
}
// noise_words with the Philox round keys from a kernel-parameter table.
template <bool NOISE_IN>
__device__ __forceinline__ U4 noise_words_k(const PhiloxKeys& K, const TensorRegs& T, const int32_t* arr,
                                            uint32_t stream, int64_t k0, int nv) {
  if (NOISE_IN) {
    uint32_t r[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) r[e] = e < nv ? ((uint32_t)arr[k0 + e] & 0xFFFFu) : 0u;
    return U4{r[0] | (r[1] << 16), r[2] | (r[3] << 16), r[4] | (r[5] << 16), r[6] | (r[7] << 16)};
  }
  const uint64_t grp = (uint64_t)k0 >> 3;
  U4 c{(uint32_t)grp, (uint32_t)(grp >> 32) | (stream << 24), T.tensor_id, T.step};
  return philox4x32_10_k(c, K);
}
__device__ __forceinline__ uint32_t noise_at(const U4& n, int e) {
  const uint32_t w = (e >> 1) == 0 ? n.x : (e >> 1) == 1 ? n.y : (e >> 1) == 2 ? n.z : n.w;
  return (e & 1) ? (w >> 16) : (w & 0xFFFFu);
}

// Stochastic quantisation of 8 values with a per-block divisor (set_state,
// state_util.py:124-157 and param_update.py:271-363), packed into 2 words.
template <bool SIGNED>
__device__ __forceinline__ uint2 quantize8(const float (&x)[8], float bmax, const U4& nz) {
  const float scale = __fdiv_rn(bmax, SIGNED ? 127.0f : 255.0f);
  const float safe = scale < 1e-12f ? 1e-12f : scale;
  const float rs = __frcp_rn(safe);
  int c[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const float y = __fadd_rn(div_const(x[e], safe, rs), noise_unit(noise_at(nz, e)));
    const int f = floor_int(y);
    c[e] = SIGNED ? min(max(f, -127), 127) : min(max(f, 0), 255);
  }
  return make_uint2(pack4_bytes(c[0], c[1], c[2], c[3]), pack4_bytes(c[4], c[5], c[6], c[7]));
}

// ---------------------------------------------------------------------------
// Prodigy slice statistics (Prodigy_adv.py:494-509): every slice_p-th
// element k of a tensor adds g_k * (p0[k / slice_p] - p_k) to d_numerator's
// dot product and updates s[k / slice_p] = s * beta3 + g_k * s_alpha, whose
// |.| goes to d_denom.  A thread's slice point in a chunk has its s and p0
// entries fetched before the chunk's arithmetic (their latency then overlaps
// it) and is applied once per thread, not once per unrolled element, so the
// lanes of a warp that hold a slice point do it together.
// ---------------------------------------------------------------------------
struct SliceAt {
  int e;          // offset in the thread's 8 elements (>= 8: none)
  int64_t si;     // slice index k / slice_p
  float p0;
  float s;
};

template <bool PBF>
__device__ __forceinline__ void slice_fetch(const TensorRegs& T, int64_t k0, int e, uint32_t slice_p, bool si32,
                                            SliceAt& S) {
  S.e = e;
  S.si = si32 ? (int64_t)((uint32_t)(k0 + e) / slice_p) : (k0 + e) / (int64_t)slice_p;
  S.p0 = 0.0f;
  if (!(T.flags & ADVOPT_T_P0_SCALAR))
    S.p0 = PBF ? bf16_to_f(static_cast<const uint16_t*>(T.aux1)[S.si]) : static_cast<const float*>(T.aux1)[S.si];
  S.s = PBF ? bf16_to_f(static_cast<const uint16_t*>(T.aux0)[S.si]) : static_cast<const float*>(T.aux0)[S.si];
}

template <bool PBF>
__device__ __forceinline__ void slice_apply(const TensorRegs& T, const SliceAt& S, float gv, float pv, float beta3,
                                            float s_alpha, double& st0, double& st1) {
  st0 += (double)gv * (double)__fsub_rn(S.p0, pv);
  float s1 = __fmul_rn(S.s, beta3);
  if (PBF) s1 = round_bf16(s1);
  float s2 = __fmaf_rn(gv, s_alpha, s1);
  if (PBF) {
    const uint32_t b = f_to_bf16_rne(s2);
    static_cast<uint16_t*>(T.aux0)[S.si] = (uint16_t)b;
    s2 = bf16_to_f(b);
  } else {
    static_cast<float*>(T.aux0)[S.si] = s2;
  }
  st1 += (double)fabsf(s2);
}

template <int PREC, bool PBF, int ALGO, bool EXT, bool NOISE_IN, bool FM = false>
__global__ void __launch_bounds__(kThreads, 2) adam_kernel(const advopt_adam_launch L) {
  using TR = StateTraits<PREC, PBF>;
  constexpr int kStore = TR::kStore;
  constexpr bool kMBF = TR::kMathBF;
  constexpr int SB = StoreBytes<kStore>::v;
  // dynamic shared memory: [0, max d2) column accumulators of the factored
  // tensor in progress; from gen_offset, the generic factored path's staged
  // chunk (2048 floats) and row-segment sums (2049 floats)
  extern __shared__ float4 dsm4[];
  float* colacc = reinterpret_cast<float*>(dsm4);
  float* vbuf = colacc + L.gen_offset;
  float* segs = vbuf + kChunk;
  // FM: a launch of signed rank-1 momentum tensors only ('factored', fp32);
  // the same areas again for |m| in the second half of shared memory
  static_assert(!FM || PREC == ADVOPT_PREC_FP32, "factored momentum is float32");
  float* colacc_m = colacc + (FM ? L.smem_floats / 2 : 0);
  float* mbuf = colacc_m + L.gen_offset;
  float* msegs = mbuf + kChunk;
  __shared__ float red[2][kWarps][6];         // per-chunk block reductions (double-buffered)
  __shared__ double dred[kWarps][2];
  __shared__ TensorRegs Ts;                   // the piece's tensor descriptor

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
  // Prodigy with d on the device reads its launch scalars from there
  const bool pdev = ALGO == ADVOPT_ALGO_PRODIGY && L.prodigy != nullptr;
  const float c_v0 = pdev ? L.prodigy->c_v : L.c_v;
  const float d_f = pdev ? L.prodigy->d_f : L.d;
  const float s_alpha = pdev ? L.prodigy->s_alpha : L.s_alpha;
  // Prodigy's m.add_(grad, alpha=d*(1-beta1)): alpha rounded to bf16 under bf16 math
  const float c_m_raw = pdev ? L.prodigy->c_m : L.c_m;
  const float beta1 = L.beta1, w_m = L.w_m, w_nest = L.w_nest, c_m = kMBF ? round_bf16(c_m_raw) : c_m_raw;
  float beta2 = L.beta2, c_v = c_v0;      // per tensor under Kourkoutas-beta
  const bool gsq = (F & ADVOPT_F_GRAD_SQ) && !fstats;
  const bool emit = F & ADVOPT_F_EMIT_UPDATE;
  __shared__ double gred[kWarps];
  auto Rm = [](float x) { return kMBF ? round_bf16(x) : x; };  // rounding of m / update / grad ops
  int parity = 0;

  const int pbeg = L.cta_offsets[blockIdx.x], pend = L.cta_offsets[blockIdx.x + 1];
  for (int pi = pbeg; pi < pend; ++pi) {
    const advopt_piece pc = L.pieces[pi];
    __syncthreads();  // the previous piece is done with Ts
    if (tid == 0) load_tensor(L.tensors + pc.tensor, Ts);
    __syncthreads();
    const TensorRegs& T = Ts;  // fields are re-read from shared memory where registers are short
    if (L.layer_beta2) {
      // Kourkoutas-beta: the tensor's layer's dynamic beta2 (Kourkoutas.py:249-257)
      const int l = L.layer_of_tensor[pc.tensor];
      beta2 = l >= 0 ? L.layer_beta2[2 * l] : L.beta2;
      c_v = l >= 0 ? L.layer_beta2[2 * l + 1] : c_v0;
    }
    double gacc = 0.0;     // Kourkoutas-beta: this thread's sum of g*g over the piece
    const bool fact = FM || (T.flags & ADVOPT_T_FACTORED);
    const bool vec = T.flags & ADVOPT_T_VEC;
    const bool has_anchor = EXT && (((T.flags >> ADVOPT_T_ANCHOR_SHIFT) & 7u) != 0);
    const bool fact_sums = fact && !fstats;   // factored row/column sums (skipped by the Fisher pass)
    constexpr bool kHasV = ALGO != ADVOPT_ALGO_LION;
    const bool v_sums = fact_sums && kHasV;
    // signed rank-1 momentum (state_precision='factored', AdamW_adv.py:342-399)
    const bool factm = FM && has_m;
    const bool fm_sums = factm && !fstats;
    const int64_t d2 = fact ? T.d2 : 1;
    const int64_t pd2 = (d2 + 7) >> 3;        // sign bytes per row
    // fast factored path: each column at most once per chunk, each thread's 8
    // elements in one row (one sign byte), 8-aligned factor columns
    const bool ffast = fact && d2 >= kChunk && (d2 % 8) == 0 && ((reinterpret_cast<uintptr_t>(T.col) & 15) == 0) &&
                       (!factm || (reinterpret_cast<uintptr_t>(T.mcol) & 15) == 0);
    const bool upd_bf16 = T.flags & ADVOPT_T_UPD_BF16;
    const bool vbf = kMBF && !fact;  // v math in bf16 ('auto' bf16, not factored)
    const float rcp_sbc2 = __frcp_rn(T.sqrt_bc2);
    const float step_size = T.step_size, eps = T.eps, sbc2 = T.sqrt_bc2, wd = T.wd, cwd = T.cwd;
    if (fact_sums) {
      if (kHasV)
        for (int j = tid; j < (int)d2; j += kThreads) colacc[j] = 0.0f;
      if (fm_sums)
        for (int j = tid; j < (int)d2; j += kThreads) colacc_m[j] = 0.0f;
      __syncthreads();
    }
    double row_carry = 0.0;  // thread 0: running sum of the row in progress
    double row_carry_m = 0.0;
    double st0 = 0.0, st1 = 0.0;
    const uint32_t slice_p = T.slice_p ? T.slice_p : 1u;
    // Prodigy: running remainder of this thread's first element mod slice_p
    // (one 64-bit division per piece, none per element)
    uint32_t srem = pstats ? (uint32_t)((uint64_t)(pc.begin + tid * kVec) % slice_p) : 0u;
    const uint32_t srem_step = (uint32_t)kChunk % slice_p;
    const bool si32 = T.numel < (int64_t(1) << 32);

    ChunkPos cp;
    cp.cs = pc.begin;
    cp.clen = (int)min((int64_t)kChunk, pc.end - pc.begin);
    cp.r0 = fact ? pc.begin / d2 : 0;
    cp.c0 = fact ? pc.begin - cp.r0 * d2 : 0;
    Raw<PBF, kStore> cur;
    load_raw<PREC, PBF, ALGO, EXT>(T, cp, tid, fact, ffast, has_m, vec, factm, cur);

    while (true) {
      // next chunk's position, and its loads in flight during this chunk
      ChunkPos np = cp;
      np.cs = cp.cs + kChunk;
      const bool has_next = np.cs < pc.end;
      if (fact) {
        np.c0 = cp.c0 + cp.clen;
        if (ffast) {
          if (np.c0 >= d2) { np.c0 -= d2; np.r0 += 1; }
        } else if (np.c0 >= d2) {
          const int64_t dr = np.c0 / d2;
          np.r0 += dr;
          np.c0 -= dr * d2;
        }
      }
      Raw<PBF, kStore> nxt;
      if (has_next) {
        np.clen = (int)min((int64_t)kChunk, pc.end - np.cs);
        load_raw<PREC, PBF, ALGO, EXT>(T, np, tid, fact, ffast, has_m, vec, factm, nxt);
      }

      const int clen = cp.clen;
      const int64_t k0 = cp.cs + tid * kVec;
      const int nv = max(0, min(kVec, clen - tid * kVec));
      const bool v8 = vec && nv == kVec;
      const int64_t blk = cp.cs >> 11;
      const int64_t r0 = cp.r0, c0 = cp.c0;

      float g[8], p[8], m[8], vh[8];
      unpack8<PBF ? 2 : 4>(cur.g, g);
      unpack8<PBF ? 2 : 4>(cur.p, p);
      if (factm) {
        // _reconstruct_state(signed=True): outer(mu, mv), negated where the
        // sign bit is clear (factorization_util.py:9-19)
        if (ffast) {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float a = __fmul_rn(cur.fmu, cur.fmv[e]);
            m[e] = ((cur.fsgn >> e) & 1u) ? a : -a;
          }
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            m[e] = 0.0f;
            if (e < nv) {
              const int64_t cc = c0 + tid * kVec + e;
              const int64_t dr = cc / d2;
              const int64_t col = cc - dr * d2;
              const float a = __fmul_rn(T.mrow[r0 + dr], T.mcol[col]);
              const uint32_t byte = T.msign[(r0 + dr) * pd2 + (col >> 3)];
              m[e] = ((byte >> (col & 7)) & 1u) ? a : -a;
            }
          }
        }
      } else if (has_m) {
        unpack8<SB, true>(cur.m, m);
        if (kStore == 2) {
#pragma unroll
          for (int e = 0; e < 8; ++e) m[e] = __fmul_rn(m[e], cur.ms);
        }
      }
      if (!kHasV) {
#pragma unroll
        for (int e = 0; e < 8; ++e) vh[e] = 0.0f;
      } else if (fact) {
        if (ffast) {
#pragma unroll
          for (int e = 0; e < 8; ++e) vh[e] = __fmul_rn(cur.mu, cur.mv[e]);   // outer(mu, mv)
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
        unpack8<SB, false>(cur.v, vh);
        if (kStore == 2) {
#pragma unroll
          for (int e = 0; e < 8; ++e) vh[e] = __fmul_rn(vh[e], cur.vs);
        }
      }
      U4 nzp{0u, 0u, 0u, 0u};
      if (sr && !fstats) nzp = noise_words<NOISE_IN>(L, T, T.nz_p, kNoiseP, k0, nv);
      SliceAt sl;          // this thread's first Prodigy slice point in the chunk
      sl.e = kVec;
      if (pstats) {
        const int first = srem ? (int)(slice_p - srem) : 0;
        if (first < nv) slice_fetch<PBF>(T, k0, first, slice_p, si32, sl);
        srem += srem_step;
        if (srem >= slice_p) srem -= slice_p;
      }

      // ---- per-element arithmetic in the reference's op order; the param
      // update does not need the block statistics and happens here ----
      float m_new[8], v[8];
      float amax_m = 0.0f, vmax = 0.0f;
      uint32_t pout[8];
      float uemit[8];
      if (gsq) {
        // torch.sum(grad.pow(2)) of the grad the step uses: squares in bf16
        // for a bf16 grad under 'auto' (Kourkoutas.py:241-245)
        float s8 = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (e < nv) s8 = __fadd_rn(s8, kMBF ? round_bf16(__fmul_rn(g[e], g[e])) : __fmul_rn(g[e], g[e]));
        gacc += (double)s8;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const bool ok = e < nv;
        float gi = g[e];
        float vi = 0.0f, du = 1.0f, ui;
        if constexpr (ALGO == ADVOPT_ALGO_LION) {
          // Lion_adv.py:236-247 on the float32 grad: c = lerp(g, m, beta1),
          // m = lerp(m, g, 1 - beta2), update = sign(c) (lion_k.py:23-24)
          const float c = Rm(lerp_t(gi, m[e], beta1));
          m_new[e] = ok ? Rm(lerp_t(m[e], gi, w_m)) : 0.0f;
          v[e] = 0.0f;
          ui = c > 0.0f ? 1.0f : (c < 0.0f ? -1.0f : c);
        } else {
        // v = v*beta2 + c_v*g*g   (mul_ then addcmul_, AdamW_adv.py:417, Prodigy_adv.py:469)
        vi = __fmul_rn(vh[e], beta2);
        if (vbf) vi = round_bf16(vi);
        vi = __fmaf_rn(__fmul_rn(c_v, gi), gi, vi);
        if (vbf) vi = round_bf16(vi);
        if (fact) vi = fabsf(vi);       // _factorize_state's abs_ (factorization_util.py:35)
        v[e] = ok ? vi : 0.0f;
        // denominator (AdamW_adv.py:424-431, Prodigy_adv.py:477-482)
        float den = sqrt_cr(vi);
        if (vbf) den = round_bf16(den);
        if (ALGO != ADVOPT_ALGO_PRODIGY) {
          den = div_rcp(den, sbc2, rcp_sbc2);   // den >= 2^-75 or 0: always in div_rcp's exact range
          if (vbf) den = round_bf16(den);
        }
        if (!atan2m) {
          den = __fadd_rn(den, eps);   // Prodigy: eps holds d*eps
          if (vbf) den = round_bf16(den);
        }
        du = kMBF ? round_bf16(den) : den;   // denom.to(update.dtype)
        if (normed) gi = atan2m ? Rm(atan2f(gi, du)) : Rm(div_cr(gi, du));
        // first moment and the update direction
        if (has_m) {
          float mi;
          if (ALGO == ADVOPT_ALGO_PRODIGY) {
            mi = Rm(__fmaf_rn(gi, c_m, Rm(__fmul_rn(m[e], beta1))));
          } else {
            mi = Rm(lerp_t(m[e], gi, w_m));
          }
          m_new[e] = ok ? mi : 0.0f;
          ui = nest ? Rm(lerp_t(mi, gi, w_nest)) : mi;
        } else {
          m_new[e] = 0.0f;
          ui = (ALGO == ADVOPT_ALGO_PRODIGY) ? Rm(__fmul_rn(gi, d_f)) : gi;
        }
        if (!normed) ui = atan2m ? Rm(atan2f(ui, du)) : Rm(div_cr(ui, du));
        }
        if (emit) uemit[e] = ui;   // the update before its scaling (AdamW_adv.py:459-461)
        ui = Rm(__fmul_rn(ui, step_size));
        amax_m = fmaxf(amax_m, fabsf(m_new[e]));
        vmax = fmaxf(vmax, v[e]);

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
          const float pcv = weight_decay<true>(p[e], ui, wd, cwd, cautious, has_anchor, anc, fisher, ws);
          pout[e] = f_to_bf16_rne(__fadd_rn(pcv, -ui));
        } else {
          const float pcv = weight_decay<false>(p[e], ui, wd, cwd, cautious, has_anchor, anc, fisher, ws);
          const float pn = __fadd_rn(pcv, -ui);
          // bf16 + SR: add the noise to the bit pattern; the pack below keeps the high half
          pout[e] = PBF ? (__float_as_uint(pn) + noise_at(nzp, e)) : __float_as_uint(pn);
        }
      }
      // Prodigy slice statistics on g and p before its update (Prodigy_adv.py:501-509):
      // the prefetched first point, then any further ones (slice_p < 8)
      if (pstats) {
        for (int e = sl.e; e < nv;) {
          float gv = 0.0f, pv = 0.0f;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (j == e) { gv = g[j]; pv = p[j]; }
          slice_apply<PBF>(T, sl, gv, pv, L.beta3, s_alpha, st0, st1);
          e += (int)slice_p;
          if (e < nv) slice_fetch<PBF>(T, k0, e, slice_p, si32, sl);
        }
      }
      if (emit) {
        if (upd_bf16) {
          uint32_t b[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) b[e] = f_to_bf16_rne(uemit[e]);
          store8_bf16(T.upd, k0, nv, v8, b);
        } else {
          store8_f32(T.upd, k0, nv, v8, uemit);
        }
      } else if (!fstats) {
        if (PBF) {
          Words<2> o;
#pragma unroll
          for (int i = 0; i < 4; ++i)
            o.w[i] = sr ? __byte_perm(pout[2 * i], pout[2 * i + 1], 0x7632) : (pout[2 * i] | (pout[2 * i + 1] << 16));
          uint16_t* dst = static_cast<uint16_t*>(T.param) + k0;
          if (v8) {
            *reinterpret_cast<uint4*>(dst) = make_uint4(o.w[0], o.w[1], o.w[2], o.w[3]);
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e)
              if (e < nv) dst[e] = (uint16_t)(o.w[e >> 1] >> (16 * (e & 1)));
          }
        } else {
          float* dst = static_cast<float*>(T.param) + k0;
          if (v8) {
            reinterpret_cast<uint4*>(dst)[0] = make_uint4(pout[0], pout[1], pout[2], pout[3]);
            reinterpret_cast<uint4*>(dst)[1] = make_uint4(pout[4], pout[5], pout[6], pout[7]);
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e)
              if (e < nv) dst[e] = __uint_as_float(pout[e]);
          }
        }
      }
      // noise for the quantised / SR'd states, drawn before the barrier
      U4 nzm{0u, 0u, 0u, 0u}, nzv{0u, 0u, 0u, 0u};
      if (!fstats && TR::kStore != 0 && (kStore == 2 || TR::kSRStates)) {
        if (has_m) nzm = noise_words<NOISE_IN>(L, T, T.nz_m, kNoiseM, k0, nv);
        if (!fact && kHasV) nzv = noise_words<NOISE_IN>(L, T, T.nz_v, kNoiseV, k0, nv);
      }

      // ---- factored second moment: row sums and column partials ----
      float rsum0 = 0.0f, rsum1 = 0.0f;
      if (v_sums) {
        if (ffast) {
          const int64_t cc = c0 + tid * kVec;
          const bool second = cc >= d2;
          const int64_t col = second ? cc - d2 : cc;
          if (nv > 0) {
            float4* ca = reinterpret_cast<float4*>(colacc + col);
            float4 a = ca[0], b = ca[1];
            a.x = __fadd_rn(a.x, v[0]); a.y = __fadd_rn(a.y, v[1]); a.z = __fadd_rn(a.z, v[2]); a.w = __fadd_rn(a.w, v[3]);
            b.x = __fadd_rn(b.x, v[4]); b.y = __fadd_rn(b.y, v[5]); b.z = __fadd_rn(b.z, v[6]); b.w = __fadd_rn(b.w, v[7]);
            ca[0] = a;
            ca[1] = b;
          }
          const float s = __fadd_rn(__fadd_rn(__fadd_rn(v[0], v[1]), __fadd_rn(v[2], v[3])),
                                    __fadd_rn(__fadd_rn(v[4], v[5]), __fadd_rn(v[6], v[7])));
          if (second) rsum1 = s; else rsum0 = s;
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (e < nv) vbuf[tid * kVec + e] = v[e];
        }
      }

      // ---- signed rank-1 momentum: sign bits, |m| row sums and column partials
      // (_factorize_state(signed=True), factorization_util.py:25-32) ----
      float mrs0 = 0.0f, mrs1 = 0.0f;
      if (fm_sums) {
        if (ffast) {
          const int64_t cc = c0 + tid * kVec;
          const bool second = cc >= d2;
          const int64_t col = second ? cc - d2 : cc;
          float am[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) am[e] = fabsf(m_new[e]);
          if (nv > 0) {
            uint32_t sb = 0u;
#pragma unroll
            for (int e = 0; e < 8; ++e) sb |= (m_new[e] > 0.0f ? 1u : 0u) << e;
            T.msign[k0 >> 3] = (uint8_t)sb;
            float4* ca = reinterpret_cast<float4*>(colacc_m + col);
            float4 a = ca[0], b = ca[1];
            a.x = __fadd_rn(a.x, am[0]); a.y = __fadd_rn(a.y, am[1]); a.z = __fadd_rn(a.z, am[2]); a.w = __fadd_rn(a.w, am[3]);
            b.x = __fadd_rn(b.x, am[4]); b.y = __fadd_rn(b.y, am[5]); b.z = __fadd_rn(b.z, am[6]); b.w = __fadd_rn(b.w, am[7]);
            ca[0] = a;
            ca[1] = b;
          }
          const float s = __fadd_rn(__fadd_rn(__fadd_rn(am[0], am[1]), __fadd_rn(am[2], am[3])),
                                    __fadd_rn(__fadd_rn(am[4], am[5]), __fadd_rn(am[6], am[7])));
          if (second) mrs1 = s; else mrs0 = s;
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            if (e < nv) {
              mbuf[tid * kVec + e] = fabsf(m_new[e]);
              // one atomic per element on the 4-byte word that holds its sign byte
              const int64_t cc = c0 + tid * kVec + e;
              const int64_t dr = cc / d2;
              const int64_t col = cc - dr * d2;
              const int64_t byte = (r0 + dr) * pd2 + (col >> 3);
              unsigned int* w = reinterpret_cast<unsigned int*>(T.msign) + (byte >> 2);
              const unsigned int bit = 1u << (((unsigned)(byte & 3) << 3) + (unsigned)(col & 7));
              if (m_new[e] > 0.0f) atomicOr(w, bit); else atomicAnd(w, ~bit);
            }
          }
        }
      }

      // ---- block reductions (one barrier per chunk) ----
      {
        const float a = (has_m && kStore == 2) ? warp_max(amax_m) : 0.0f;
        const float b = (!fact && kStore == 2) ? warp_max(vmax) : 0.0f;
        const float c = ffast ? warp_sum(rsum0) : 0.0f;
        const float d = ffast ? warp_sum(rsum1) : 0.0f;
        const float e5 = (ffast && fm_sums) ? warp_sum(mrs0) : 0.0f;
        const float f6 = (ffast && fm_sums) ? warp_sum(mrs1) : 0.0f;
        if (lane == 0) {
          red[parity][warp][0] = a;
          red[parity][warp][1] = b;
          red[parity][warp][2] = c;
          red[parity][warp][3] = d;
          red[parity][warp][4] = e5;
          red[parity][warp][5] = f6;
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
            if (kHasV && clen >= d2 - c0) {         // row r0 completes in this chunk
              T.row[r0] = (float)row_carry;
              row_carry = (double)s1;
            }
            if (fm_sums) {
              float m0 = 0.0f, m1 = 0.0f;
#pragma unroll
              for (int w = 0; w < kWarps; ++w) {
                m0 = __fadd_rn(m0, red[parity][w][4]);
                m1 = __fadd_rn(m1, red[parity][w][5]);
              }
              row_carry_m += (double)m0;
              if (clen >= d2 - c0) {
                T.mrow[r0] = (float)row_carry_m;
                row_carry_m = (double)m1;
              }
            }
          }
        } else {
          // generic: each column's elements in this chunk, summed in order by
          // the thread that owns its first occurrence; rows by segment
          auto gen_sums = [&](const float* buf, float* cacc, float* sg, float* rowp, double& carry) {
            const int ncol = (int)min((int64_t)clen, d2);
            for (int pp = tid; pp < ncol; pp += kThreads) {
              float acc = 0.0f;
              for (int q = pp; q < clen; q += (int)d2) acc = __fadd_rn(acc, buf[q]);
              int64_t j = c0 + pp;
              if (j >= d2) j -= d2;
              cacc[j] = __fadd_rn(cacc[j], acc);
            }
            // rows: segment s covers chunk positions [max(0, s*d2-c0), min(clen, (s+1)*d2-c0))
            const int nseg = (int)((c0 + clen - 1) / d2) + 1;
            for (int s = warp; s < nseg; s += kWarps) {
              const int64_t lo = max((int64_t)0, (int64_t)s * d2 - c0);
              const int64_t hi = min((int64_t)clen, (int64_t)(s + 1) * d2 - c0);
              float acc = 0.0f;
              for (int64_t q = lo + lane; q < hi; q += 32) acc = __fadd_rn(acc, buf[q]);
              acc = warp_sum(acc);
              if (lane == 0) sg[s] = acc;
            }
            __syncthreads();
            if (tid == 0) {
              for (int s = 0; s < nseg; ++s) {
                carry += (double)sg[s];
                if ((int64_t)(s + 1) * d2 - c0 <= clen) {   // row r0+s ends in this chunk
                  rowp[r0 + s] = (float)carry;
                  carry = 0.0;
                }
              }
            }
            __syncthreads();
          };
          if (kHasV) gen_sums(vbuf, colacc, segs, T.row, row_carry);
          if (fm_sums) gen_sums(mbuf, colacc_m, msegs, T.mrow, row_carry_m);
        }
      }

      // ---- store the new moments (they need the block max) ----
      if (!fstats) {
        if (has_m && !factm) {
          if (kStore == 2) {
            float bmax = 0.0f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) bmax = fmaxf(bmax, red[parity][w][0]);
            const uint2 q = quantize8<true>(m_new, bmax, nzm);
            uint8_t* dst = static_cast<uint8_t*>(T.m) + k0;
            if (v8) {
              *reinterpret_cast<uint2*>(dst) = q;
            } else {
#pragma unroll
              for (int e = 0; e < 8; ++e)
                if (e < nv) dst[e] = (uint8_t)((e < 4 ? q.x : q.y) >> (8 * (e & 3)));
            }
            if (tid == 0) T.m_scale[blk] = __fdiv_rn(bmax, 127.0f);
          } else if (kStore == 1) {
            uint32_t b[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) b[e] = TR::kSRStates ? f_to_bf16_sr(m_new[e], noise_at(nzm, e)) : f_to_bf16_rne(m_new[e]);
            store8_bf16(T.m, k0, nv, v8, b);
          } else {
            store8_f32(T.m, k0, nv, v8, m_new);
          }
        }
        if (!fact && kHasV) {        // (Lion has no second moment)
          if (kStore == 2) {
            float bmax = 0.0f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) bmax = fmaxf(bmax, red[parity][w][1]);
            const uint2 q = quantize8<false>(v, bmax, nzv);
            uint8_t* dst = static_cast<uint8_t*>(T.v) + k0;
            if (v8) {
              *reinterpret_cast<uint2*>(dst) = q;
            } else {
#pragma unroll
              for (int e = 0; e < 8; ++e)
                if (e < nv) dst[e] = (uint8_t)((e < 4 ? q.x : q.y) >> (8 * (e & 3)));
            }
            if (tid == 0) T.v_scale[blk] = __fdiv_rn(bmax, 255.0f);
          } else if (kStore == 1) {
            uint32_t b[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) b[e] = TR::kSRStates ? f_to_bf16_sr(v[e], noise_at(nzv, e)) : f_to_bf16_rne(v[e]);
            store8_bf16(T.v, k0, nv, v8, b);
          } else {
            store8_f32(T.v, k0, nv, v8, v);
          }
        }
      }
      parity ^= 1;
      if (!has_next) break;
      cp = np;
      cur = nxt;
    }

    // ---- end of piece: flush column partials and statistics ----
    if (fact_sums) {
      __syncthreads();
      if (kHasV) {
        float* dst = T.colpart + (int64_t)pc.slot * d2;
        for (int j = tid; j < (int)d2; j += kThreads) dst[j] = colacc[j];
      }
      if (fm_sums) {
        float* dm = T.mcolpart + (int64_t)pc.slot * d2;
        for (int j = tid; j < (int)d2; j += kThreads) dm[j] = colacc_m[j];
      }
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
    if (gsq) {
      const double a = warp_sum_d(gacc);
      if (lane == 0) gred[warp] = a;
      __syncthreads();
      if (tid == 0) {
        double sa = 0.0;
        for (int w = 0; w < kWarps; ++w) sa += gred[w];
        L.piece_gsq[pi] = sa;
      }
      __syncthreads();
    }
  }
}

}  // namespace advopt

#include "adam_fast.cuh"

namespace advopt {

// Host launchers, instantiated per precision in adam_<precision>.cu.  A
// launch with L.stages > 0 (and none of the extended options) runs the fast
// kernel; everything else runs the general one.
// Option flags compiled into a specialised fast kernel for this launch, or
// kCfDyn.  Specialisations exist for the int8_sr / bf16 AdamW step (every
// tensor with momentum and stochastic rounding, lerp weights below 1/2, no
// cautious decay): with and without Nesterov, with and without decay.
template <int PREC, bool PBF, int ALGO>
int fast_config(const advopt_adam_launch& L) {
  if (!(PREC == ADVOPT_PREC_INT8_SR && PBF && ALGO == ADVOPT_ALGO_ADAMW)) return kCfDyn;
  const uint32_t F = L.flags;
  if (!(F & ADVOPT_F_HAS_M) || !(F & ADVOPT_F_SR) || (F & (ADVOPT_F_CAUTIOUS | ADVOPT_F_NOISE_IN | ADVOPT_F_EMIT_UPDATE)))
    return kCfDyn;
  if (!(fabsf(L.w_m) < 0.5f)) return kCfDyn;
  int cf = kCfHasM | kCfSR | kCfMSmall;
  if (F & ADVOPT_F_NESTEROV) {
    if (!(fabsf(L.w_nest) < 0.5f)) return kCfDyn;
    cf |= kCfNest | kCfNSmall;
  }
  if (!(F & ADVOPT_F_NO_WD)) cf |= kCfWd;
  return cf;
}

template <int PREC, bool PBF, int ALGO, int CF>
cudaError_t launch_fast(const advopt_adam_launch& L, size_t smem, cudaStream_t s) {
  auto kf = adam_fast_kernel<PREC, PBF, ALGO, false, CF>;
  cudaError_t e = cudaFuncSetAttribute(kf, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kf<<<L.grid, kThreads, smem, s>>>(L, philox_keys(L.seed));
  return cudaGetLastError();
}

// Host launchers, instantiated per precision in adam_<precision>.cu.  A
// launch with L.stages > 0 (and none of the extended options) runs the fast
// kernel; everything else runs the general one.
template <int PREC, bool PBF, int ALGO>
cudaError_t launch_adam_algo(const advopt_adam_launch& L, cudaStream_t s) {
  const bool ext = L.flags & (ADVOPT_F_ATAN2 | ADVOPT_F_NORMED | ADVOPT_F_FISHER | ADVOPT_F_FISHER_STATS |
                              ADVOPT_F_ANCHORS);
  const bool nin = L.flags & ADVOPT_F_NOISE_IN;
  const size_t smem = (size_t)L.smem_floats * sizeof(float);
  // signed rank-1 momentum on the fast layout (planned with stages > 0):
  // the fast kernel's FM variant
  if constexpr (PREC == ADVOPT_PREC_FP32 && ALGO != ADVOPT_ALGO_LION) {
    if ((L.flags & ADVOPT_F_FACT_M) && !ext && L.stages > 0 && !(L.flags & ADVOPT_F_EMIT_UPDATE)) {
      auto kf = nin ? adam_fast_kernel<PREC, PBF, ALGO, true, kCfDyn, true>
                    : adam_fast_kernel<PREC, PBF, ALGO, false, kCfDyn, true>;
      cudaError_t e = cudaFuncSetAttribute(kf, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      kf<<<L.grid, kThreads, smem, s>>>(L, philox_keys(L.seed));
      return cudaGetLastError();
    }
  }
  // Lion, and signed rank-1 momentum otherwise, live in the general kernel;
  // update emission runs in either (the fast kernel's only when planned)
  const bool general_only = ALGO == ADVOPT_ALGO_LION || (L.flags & ADVOPT_F_FACT_M);
  if constexpr (ALGO != ADVOPT_ALGO_LION) {
  if (!ext && !general_only && L.stages > 0) {
    const bool emit = L.flags & ADVOPT_F_EMIT_UPDATE;
    if (nin) {
      auto kf = emit ? adam_fast_kernel<PREC, PBF, ALGO, true, kCfDynEmit> : adam_fast_kernel<PREC, PBF, ALGO, true, kCfDyn>;
      cudaError_t e = cudaFuncSetAttribute(kf, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      kf<<<L.grid, kThreads, smem, s>>>(L, philox_keys(L.seed));
      return cudaGetLastError();
    }
    if constexpr (PREC == ADVOPT_PREC_INT8_SR && PBF && ALGO == ADVOPT_ALGO_ADAMW) {
      constexpr int B = kCfHasM | kCfSR | kCfMSmall, N = kCfNest | kCfNSmall;
      switch (fast_config<PREC, PBF, ALGO>(L)) {
        case B: return launch_fast<PREC, PBF, ALGO, B>(L, smem, s);
        case B | kCfWd: return launch_fast<PREC, PBF, ALGO, B | kCfWd>(L, smem, s);
        case B | N: return launch_fast<PREC, PBF, ALGO, B | N>(L, smem, s);
        case B | N | kCfWd: return launch_fast<PREC, PBF, ALGO, B | N | kCfWd>(L, smem, s);
        default: break;
      }
    }
    if (emit) return launch_fast<PREC, PBF, ALGO, kCfDynEmit>(L, smem, s);
    return launch_fast<PREC, PBF, ALGO, kCfDyn>(L, smem, s);
  }
  }
  if (L.flags & ADVOPT_F_FACT_M) {
    // every tensor of the launch holds signed rank-1 momentum
    if constexpr (PREC == ADVOPT_PREC_FP32) {
      auto kf = ext ? (nin ? adam_kernel<PREC, PBF, ALGO, true, true, true> : adam_kernel<PREC, PBF, ALGO, true, false, true>)
                    : (nin ? adam_kernel<PREC, PBF, ALGO, false, true, true> : adam_kernel<PREC, PBF, ALGO, false, false, true>);
      cudaError_t e = cudaFuncSetAttribute(kf, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      kf<<<L.grid, kThreads, smem, s>>>(L);
      return cudaGetLastError();
    }
    return cudaErrorInvalidValue;
  }
  auto k = ext ? (nin ? adam_kernel<PREC, PBF, ALGO, true, true> : adam_kernel<PREC, PBF, ALGO, true, false>)
               : (nin ? adam_kernel<PREC, PBF, ALGO, false, true> : adam_kernel<PREC, PBF, ALGO, false, false>);
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  k<<<L.grid, kThreads, smem, s>>>(L);
  return cudaGetLastError();
}

template <int PREC, bool PBF, int ALGO>
cudaError_t occupancy_adam_algo(int smem_floats, int* ctas, int fast) {
  const size_t smem = (size_t)smem_floats * sizeof(float);
  if (fast) {
    auto k = adam_fast_kernel<PREC, PBF, ALGO, false, kCfDyn>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(ctas, k, kThreads, smem);
  }
  auto k = adam_kernel<PREC, PBF, ALGO, false, false>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(ctas, k, kThreads, smem);
}

template <int PREC>
cudaError_t launch_adam_prec(const advopt_adam_launch& L, cudaStream_t s) {
  const bool pbf = L.param_dtype == ADVOPT_DT_BF16;
  switch (L.algo) {
    case ADVOPT_ALGO_ADAMW:
      return pbf ? launch_adam_algo<PREC, true, ADVOPT_ALGO_ADAMW>(L, s) : launch_adam_algo<PREC, false, ADVOPT_ALGO_ADAMW>(L, s);
    case ADVOPT_ALGO_AUXADAM:
      return pbf ? launch_adam_algo<PREC, true, ADVOPT_ALGO_AUXADAM>(L, s) : launch_adam_algo<PREC, false, ADVOPT_ALGO_AUXADAM>(L, s);
    case ADVOPT_ALGO_LION:
      // Lion: float32 (factored, or float32 params) and 'auto' launches
      // (checked by advopt_adam_step)
      if constexpr (PREC == ADVOPT_PREC_FP32 || PREC == ADVOPT_PREC_AUTO)
        return pbf ? launch_adam_algo<PREC, true, ADVOPT_ALGO_LION>(L, s) : launch_adam_algo<PREC, false, ADVOPT_ALGO_LION>(L, s);
      return cudaErrorInvalidValue;
    default:
      return pbf ? launch_adam_algo<PREC, true, ADVOPT_ALGO_PRODIGY>(L, s) : launch_adam_algo<PREC, false, ADVOPT_ALGO_PRODIGY>(L, s);
  }
}

template <int PREC>
cudaError_t occupancy_adam_prec(int pdt, int algo, int smem_floats, int* ctas, int fast) {
  const bool pbf = pdt == ADVOPT_DT_BF16;
  switch (algo) {
    case ADVOPT_ALGO_ADAMW:
      return pbf ? occupancy_adam_algo<PREC, true, ADVOPT_ALGO_ADAMW>(smem_floats, ctas, fast) : occupancy_adam_algo<PREC, false, ADVOPT_ALGO_ADAMW>(smem_floats, ctas, fast);
    case ADVOPT_ALGO_AUXADAM:
      return pbf ? occupancy_adam_algo<PREC, true, ADVOPT_ALGO_AUXADAM>(smem_floats, ctas, fast) : occupancy_adam_algo<PREC, false, ADVOPT_ALGO_AUXADAM>(smem_floats, ctas, fast);
    default:
      return pbf ? occupancy_adam_algo<PREC, true, ADVOPT_ALGO_PRODIGY>(smem_floats, ctas, fast) : occupancy_adam_algo<PREC, false, ADVOPT_ALGO_PRODIGY>(smem_floats, ctas, fast);
  }
}

// declared here, defined (instantiated) in adam_fp32.cu, adam_bf16sr.cu, adam_int8.cu, adam_auto.cu
cudaError_t launch_adam_fp32(const advopt_adam_launch& L, cudaStream_t s);
cudaError_t launch_adam_bf16sr(const advopt_adam_launch& L, cudaStream_t s);
cudaError_t launch_adam_int8(const advopt_adam_launch& L, cudaStream_t s);
cudaError_t launch_adam_auto(const advopt_adam_launch& L, cudaStream_t s);
cudaError_t occupancy_adam_fp32(int pdt, int algo, int smem_floats, int* ctas, int fast);
cudaError_t occupancy_adam_bf16sr(int pdt, int algo, int smem_floats, int* ctas, int fast);
cudaError_t occupancy_adam_int8(int pdt, int algo, int smem_floats, int* ctas, int fast);
cudaError_t occupancy_adam_auto(int pdt, int algo, int smem_floats, int* ctas, int fast);

}  // namespace advopt
