// Fast path of the Adam-family step (included by adam_impl.cuh users).
//
// Same arithmetic as adam_kernel (op for op, same roundings), restricted to
// the common configurations: no atan2 / normed momentum / Fisher / centered
// anchors, and factored tensors only with d2 >= 2048, d2 % 8 == 0 (every
// Llama-shaped effective shape).  Differences in structure:
//   * each chunk's inputs (grad, param, m codes, v codes) stream into a ring
//     of shared-memory stages with cp.async.bulk (TMA bulk copies, no
//     multicast) completed on mbarriers, `stages` chunks ahead;
//   * element arithmetic runs on fp32x2 lanes (sm_100 packed FFMA2/FADD2/FMUL2);
//   * the per-element square root and division use Newton–Markstein
//     sequences (below) that are correctly rounded on the value ranges a
//     thread checks for; a warp with any element outside them recomputes its
//     chunk with the IEEE intrinsics;
//   * block maxima use warp max-reductions of the float bit patterns
//     (redux.sync), factored row sums are reduced across the CTA once per row;
//   * waits are bounded: a wait that gives up sets *L.err and the CTA stops.
#pragma once

#include <type_traits>

namespace advopt {

// ---------------------------------------------------------------------------
// Correctly rounded sqrt and division by Newton–Markstein iteration
// (P. Markstein, "Computation of elementary functions on the IBM RISC
// System/6000 processor", IBM J. Res. Dev. 34(1), 1990; J.-M. Muller et al.,
// Handbook of Floating-Point Arithmetic, ch. 5):
//   sqrt(v): y ~ 1/sqrt(v) (hardware estimate), s = v*y, r = v - s*s (exact
//            by FMA), s' = s + r*(y/2);
//   u / d:   y ~ 1/d (hardware estimate), y1 = y + y*(1 - d*y), q = u*y1,
//            r = u - q*d (exact by FMA), q' = q + r*y1.
// Checked on B200 against __fsqrt_rn / __fdiv_rn: the square root matches for
// every float in [2^-102, FLT_MAX]; the quotient matches (every divisor
// mantissa x 64 dividend mantissas per exponent pair, dividends down to the
// subnormals) whenever |u| >= 2^-102 or u = 0, and the quotient is normal.
// The fast path therefore requires v >= 2^-100 (so d >= 2^-50), d <= 2^24 and
// |u| >= 2^-100 (so 2^-124 <= |q| <= |u| * 2^50; |u| large enough to overflow
// comes only with an infinite v, which fails d <= 2^24); a warp with any
// element outside takes the IEEE path.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float rsqrt_est(float x) {
  float y;
  asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_est(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float min3f(float a, float b, float c) {
  float r;
  asm("min.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ float2 neg2(float2 a) { return make_float2(-a.x, -a.y); }

__device__ __forceinline__ float2 sqrt_nm2(float2 v) {
  const float2 y = make_float2(rsqrt_est(v.x), rsqrt_est(v.y));
  const float2 s = mul2(v, y);
  const float2 h = mul2(y, splat2(0.5f));
  const float2 r = fma2(neg2(s), s, v);
  return fma2(r, h, s);
}
__device__ __forceinline__ float2 div_nm2(float2 u, float2 d) {
  const float2 y = make_float2(rcp_est(d.x), rcp_est(d.y));
  const float2 e = fma2(neg2(d), y, splat2(1.0f));
  const float2 y1 = fma2(e, y, y);
  const float2 q = mul2(u, y1);
  const float2 r = fma2(neg2(q), d, u);
  return fma2(r, y1, q);
}

template <int PREC, bool PBF>
struct FastLayout {
  static constexpr int kStore = StateTraits<PREC, PBF>::kStore;
  static constexpr int BPP = PBF ? 2 : 4;                         // param / grad bytes
  static constexpr int BPS = kStore == 2 ? 1 : (kStore == 1 ? 2 : 4);  // state bytes
  static constexpr int G = 0;
  static constexpr int P = kChunk * BPP;
  static constexpr int M = 2 * kChunk * BPP;
  static constexpr int V = M + kChunk * BPS;
  static constexpr int BYTES = V + kChunk * BPS;                  // one stage
};

// Descriptor fields of the current piece with its first element folded in
// (written by thread 0 at the start of each piece; the chunks index them with
// 32-bit offsets).
struct PieceRegs {
  unsigned char* p;     // param bytes of the piece
  unsigned char* u;     // emitted update of the piece (ADVOPT_F_EMIT_UPDATE: the param dtype)
  unsigned char* m;     // first-moment storage of the piece
  float* ms;            // block scales of m from the piece's first block
  float* vs;            // block scales of v
  float* row;           // factored row factor
  const float* col;     // factored column factor
  float* mrow;          // signed rank-1 momentum (FM): row factor, column factor, sign bytes
  const float* mcol;
  uint8_t* msign;
  uint32_t gbase;       // Philox element group of the piece's first element
  uint32_t tensor_id, step;
};

template <int PREC, bool PBF>
__device__ __forceinline__ void piece_regs(const TensorRegs& T, int64_t pb, PieceRegs& P) {
  using LY = FastLayout<PREC, PBF>;
  P.p = static_cast<unsigned char*>(T.param) + pb * LY::BPP;
  P.u = T.upd ? static_cast<unsigned char*>(T.upd) + pb * LY::BPP : nullptr;
  P.m = T.m ? static_cast<unsigned char*>(T.m) + pb * LY::BPS : nullptr;
  P.ms = T.m_scale ? T.m_scale + (pb >> 11) : nullptr;
  P.vs = T.v_scale ? T.v_scale + (pb >> 11) : nullptr;
  P.row = T.row;
  P.col = T.col;
  P.mrow = T.mrow;
  P.mcol = T.mcol;
  P.msign = T.msign;
  P.gbase = (uint32_t)((uint64_t)pb >> 3);
  P.tensor_id = T.tensor_id;
  P.step = T.step;
}

struct Cursor {      // producer position (thread 0)
  int pi;            // piece index
  int64_t cs;        // chunk start
  int64_t pend;      // piece end
  int tensor;        // tensor of the cached descriptor fields
  const void* g;
  const void* p;
  const void* m;
  const void* v;
  uint32_t flags;
};

template <int PREC, bool PBF>
__device__ __forceinline__ void cursor_load_piece(const advopt_adam_launch& L, Cursor& c) {
  const advopt_piece pc = L.pieces[c.pi];
  c.cs = pc.begin;
  c.pend = pc.end;
  if (pc.tensor != c.tensor) {
    const advopt_adam_tensor* t = L.tensors + pc.tensor;
    c.tensor = pc.tensor;
    c.g = t->grad;
    c.p = t->param;
    c.m = t->exp_avg;
    c.v = t->exp_avg_sq;
    c.flags = t->flags;
  }
}

// Issue the copies of the cursor's chunk into `stage`; records whether the
// consumers must read this chunk from global memory instead (tails,
// misaligned tensors).  Thread 0 only.
template <int PREC, bool PBF>
__device__ __forceinline__ void issue_chunk(const Cursor& c, unsigned char* stage, uint64_t* bar, int* direct,
                                            bool has_m) {
  using LY = FastLayout<PREC, PBF>;
  const int clen = (int)min((int64_t)kChunk, c.pend - c.cs);
  const bool fact = c.flags & ADVOPT_T_FACTORED;
  const uint32_t bp = (uint32_t)clen * LY::BPP, bs = (uint32_t)clen * LY::BPS;
  const bool ok = (c.flags & ADVOPT_T_VEC) && (bp % 16 == 0) && (bs % 16 == 0);
  if (!ok) {
    *direct = 1;
    mbar_arrive_tx(bar, 0);
    return;
  }
  *direct = 0;
  const uint32_t total = 2 * bp + (has_m ? bs : 0) + (fact ? 0 : bs);
  mbar_arrive_tx(bar, total);
  bulk_g2s(stage + LY::G, static_cast<const unsigned char*>(c.g) + c.cs * LY::BPP, bp, bar);
  bulk_g2s(stage + LY::P, static_cast<const unsigned char*>(c.p) + c.cs * LY::BPP, bp, bar);
  if (has_m) bulk_g2s(stage + LY::M, static_cast<const unsigned char*>(c.m) + c.cs * LY::BPS, bs, bar);
  if (!fact) bulk_g2s(stage + LY::V, static_cast<const unsigned char*>(c.v) + c.cs * LY::BPS, bs, bar);
}

// Move the cursor to the first chunk of the first non-empty piece at or after
// c.pi (empty pieces have no chunks on the consumer side either).
template <int PREC, bool PBF>
__device__ __forceinline__ bool cursor_seek(const advopt_adam_launch& L, Cursor& c, int pend_piece) {
  for (; c.pi < pend_piece; ++c.pi) {
    cursor_load_piece<PREC, PBF>(L, c);
    if (c.cs < c.pend) return true;
  }
  return false;
}

// Advance the cursor by one chunk; false when the CTA has no more chunks.
template <int PREC, bool PBF>
__device__ __forceinline__ bool cursor_next(const advopt_adam_launch& L, Cursor& c, int pend_piece) {
  c.cs += kChunk;
  if (c.cs < c.pend) return true;
  ++c.pi;
  return cursor_seek<PREC, PBF>(L, c, pend_piece);
}

template <int BPE>
__device__ __forceinline__ void lds_words(const unsigned char* s, Words<BPE>& out) {
  if (BPE == 1) {
    const uint2 q = *reinterpret_cast<const uint2*>(s);
    out.w[0] = q.x; out.w[1] = q.y;
  } else if (BPE == 2) {
    const uint4 q = *reinterpret_cast<const uint4*>(s);
    out.w[0] = q.x; out.w[1] = q.y; out.w[2] = q.z; out.w[3] = q.w;
  } else {
    const uint4 a = *reinterpret_cast<const uint4*>(s);
    const uint4 b = *(reinterpret_cast<const uint4*>(s) + 1);
    out.w[0] = a.x; out.w[1] = a.y; out.w[2] = a.z; out.w[3] = a.w;
    out.w[4] = b.x; out.w[5] = b.y; out.w[6] = b.z; out.w[7] = b.w;
  }
}

// Eight values as four fp32 pairs: BPE 4 = f32, 2 = bf16, 1 = int8 (SIGNED) /
// uint8 codes (exact via 2^23 + byte, minus the bias on packed lanes).
template <int BPE, bool SIGNED>
__device__ __forceinline__ void unpack8x2(const Words<BPE>& in, float2 (&x)[4]) {
  if (BPE == 4) {
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = make_float2(__uint_as_float(in.w[2 * i]), __uint_as_float(in.w[2 * i + 1]));
  } else if (BPE == 2) {
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = make_float2(__uint_as_float(in.w[i] << 16), __uint_as_float(in.w[i] & 0xFFFF0000u));
  } else {
    const float bias = SIGNED ? -8388736.0f : -8388608.0f;  // -(2^23 + 128) | -2^23
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t w = SIGNED ? (in.w[h] ^ 0x80808080u) : in.w[h];
      const float2 a = make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7440)),
                                   __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7441)));
      const float2 b = make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7442)),
                                   __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7443)));
      x[2 * h] = add2(a, splat2(bias));
      x[2 * h + 1] = add2(b, splat2(bias));
    }
  }
}

// Stochastic quantisation of 8 values with the block divisor (set_state,
// state_util.py:124-157): code = clamp(floor(x/safe + r/65536)) with
// scale = bmax/127 (int8) or bmax/255 (uint8) and safe = max(scale, 1e-12).
// scale is the Markstein quotient with the correctly rounded reciprocal of
// the constant (exact for bmax >= 2^-90; below that every code is 0 or -1
// by the sign, and the block scale is written by the IEEE division).  x/safe
// is the Newton–Markstein quotient (exact for |x| >= 2^-102 with |x/safe| <=
// 127; for smaller |x| only the quotient's sign reaches the floor).  floor(y)
// comes from y + 1.5*2^23 rounded down, whose low byte is the
// two's-complement code.
template <bool SIGNED>
__device__ __forceinline__ float block_scale(float bmax) {
  // RN(1/127), RN(1/255) as exact float literals
  return bmax >= 0x1p-90f ? div_rcp(bmax, SIGNED ? 127.0f : 255.0f, SIGNED ? 0x1.020408p-7f : 0x1.010102p-8f)
                           : __fdiv_rn(bmax, SIGNED ? 127.0f : 255.0f);
}

template <bool SIGNED>
__device__ __forceinline__ uint2 quantize8x2(const float2 (&x)[4], float scale, const U4& nz) {
  const float safe = scale < 1e-12f ? 1e-12f : scale;
  const float y0 = rcp_est(safe);
  const float y1 = __fmaf_rn(__fmaf_rn(-safe, y0, 1.0f), y0, y0);
  const uint32_t nw[4] = {nz.x, nz.y, nz.z, nz.w};
  uint32_t f[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 q0 = mul2(x[i], splat2(y1));
    const float2 q = fma2(fma2(neg2(q0), splat2(safe), x[i]), splat2(y1), q0);
    // noise r * 2^-16 from bits: the 16 bits placed under the exponent of 1
    // give 1 + r*2^-23 (one byte permute), minus 1 exactly, then r*2^-23 * 128
    // = r*2^-16 enters a single rounding: y = RN(q + r*2^-16)
    const float2 n1 = make_float2(__uint_as_float(__byte_perm(nw[i], 0x3F80u, 0x5410)),
                                  __uint_as_float(__byte_perm(nw[i], 0x3F80u, 0x5432)));
    float2 y = fma2(add2(n1, splat2(-1.0f)), splat2(128.0f), q);
    // int8: floor(y) >= -128 needs the lower clamp only (y < 128 when
    // |x| <= bmax); uint8: y can reach 256.0 exactly, so clamp above too
    if (SIGNED) y = make_float2(fmaxf(y.x, -127.0f), fmaxf(y.y, -127.0f));
    else y = make_float2(fminf(fmaxf(y.x, 0.0f), 255.5f), fminf(fmaxf(y.y, 0.0f), 255.5f));
    const float2 F = __fadd2_rd(y, splat2(12582912.0f));   // 1.5*2^23 + floor(y)
    f[2 * i] = __float_as_uint(F.x);
    f[2 * i + 1] = __float_as_uint(F.y);
  }
  const uint32_t a0 = __byte_perm(f[0], f[1], 0x0040), a1 = __byte_perm(f[2], f[3], 0x0040);
  const uint32_t b0 = __byte_perm(f[4], f[5], 0x0040), b1 = __byte_perm(f[6], f[7], 0x0040);
  return make_uint2(__byte_perm(a0, a1, 0x5410), __byte_perm(b0, b1, 0x5410));
}

// One thread's inputs of one chunk as loaded (packed words: bf16 pairs,
// int8 quads, ...); the element math unpacks one pair at a time, which keeps
// the live register set small.
template <int PREC, bool PBF>
struct FastIn {
  using LY = FastLayout<PREC, PBF>;
  Words<LY::BPP> g, p;
  Words<LY::BPS> m, v;
  float ms, vs, mu;
  float4 mva, mvb;
  // FM: the momentum's row factor, eight column factors and the sign byte
  float fmu;
  float4 fma, fmb;
  uint32_t fsg;
};

template <int PREC, bool PBF>
__device__ __forceinline__ void fast_load(const TensorRegs& T, const unsigned char* st, bool dir, int64_t k0, int nv,
                                          bool v8, bool has_m, bool fact, FastIn<PREC, PBF>& in) {
  using LY = FastLayout<PREC, PBF>;
  constexpr int SB = LY::BPS;
  const int tid = threadIdx.x;
  if (dir) {
    ld_words<LY::BPP>(T.grad, k0, nv, v8, in.g);
    ld_words<LY::BPP>(T.param, k0, nv, v8, in.p);
    if (has_m) ld_words<SB>(T.m, k0, nv, v8, in.m);
    if (!fact) ld_words<SB>(T.v, k0, nv, v8, in.v);
  } else {
    lds_words<LY::BPP>(st + LY::G + tid * kVec * LY::BPP, in.g);
    lds_words<LY::BPP>(st + LY::P + tid * kVec * LY::BPP, in.p);
    if (has_m) lds_words<SB>(st + LY::M + tid * kVec * SB, in.m);
    if (!fact) lds_words<SB>(st + LY::V + tid * kVec * SB, in.v);
  }
}

// Pair i (elements 2i, 2i+1) of 8 packed values: BPE 4 = f32, 2 = bf16,
// 1 = int8 (SIGNED) / uint8 codes (exact via 2^23 + byte, minus the bias).
template <int BPE, bool SIGNED>
__device__ __forceinline__ float2 pair_of(const Words<BPE>& in, int i) {
  if (BPE == 4) return make_float2(__uint_as_float(in.w[2 * i]), __uint_as_float(in.w[2 * i + 1]));
  // bf16 pair: low half moved up by a byte permute (ALU pipe rather than a
  // shift on the FMA pipe), high half masked
  if (BPE == 2) return make_float2(__uint_as_float(__byte_perm(in.w[i], 0u, 0x1044)), __uint_as_float(in.w[i] & 0xFFFF0000u));
  const uint32_t w0 = in.w[i >> 1];
  const uint32_t w = SIGNED ? (w0 ^ 0x80808080u) : w0;
  const uint32_t sel = (i & 1) ? 0x7442u : 0x7440u;
  const float2 a = make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, sel)),
                               __uint_as_float(__byte_perm(w, 0x4B000000u, sel + 1)));
  return add2(a, splat2(SIGNED ? -8388736.0f : -8388608.0f));   // -(2^23 + 128) | -2^23
}

// Uniform scalars of the element math.
struct FastScalars {
  float beta1, beta2, c_v, c_m, w_m, w_m1, w_n, w_n1, d;
  float sbc2, rcp_sbc2, eps, step_size, wd;
  bool w_m_small, w_n_small, has_m, nest, cautious, sr;
};

// Option flags of the element math.  A kernel instantiated with CF = kCfDyn
// reads them from the launch; the others have them compiled in (the host
// picks such a kernel only when the launch matches it exactly).  Compiled-in
// flags remove a uniform branch per element pair and let the scheduler
// interleave the pairs.
// kCfDynEmit: the dynamic-flag kernel that also writes the unscaled update
// (ADVOPT_F_EMIT_UPDATE) instead of the param; a variant of its own, so that
// the other kernels carry none of that code
enum : int { kCfDynEmit = -2, kCfDyn = -1, kCfHasM = 1, kCfNest = 2, kCfWd = 4, kCfSR = 8, kCfMSmall = 16,
             kCfNSmall = 32 };
template <int CF> __device__ __forceinline__ bool cf_has_m(const FastScalars& S) { return CF < 0 ? S.has_m : (CF & kCfHasM) != 0; }
template <int CF> __device__ __forceinline__ bool cf_nest(const FastScalars& S) { return CF < 0 ? S.nest : (CF & kCfNest) != 0; }
template <int CF> __device__ __forceinline__ bool cf_wd(const FastScalars& S) { return CF < 0 ? S.wd != 0.0f : (CF & kCfWd) != 0 && S.wd != 0.0f; }
template <int CF> __device__ __forceinline__ bool cf_cautious(const FastScalars& S) { return CF < 0 ? S.cautious : false; }
template <int CF> __device__ __forceinline__ bool cf_sr(const FastScalars& S) { return CF < 0 ? S.sr : (CF & kCfSR) != 0; }
template <int CF> __device__ __forceinline__ bool cf_msmall(const FastScalars& S) { return CF < 0 ? S.w_m_small : (CF & kCfMSmall) != 0; }
template <int CF> __device__ __forceinline__ bool cf_nsmall(const FastScalars& S) { return CF < 0 ? S.w_n_small : (CF & kCfNSmall) != 0; }

// Moments of one thread's 8 values (AdamW_adv.py:401-440,
// Muon_AuxAdam.py:148-175, Prodigy_adv.py:430-470): the new m and the new v
// (factored: before the factor rebuild).  No square root or division is
// involved, so these are exact whichever update path follows.
template <int PREC, bool PBF, int ALGO, int CF, bool FACT, bool FM = false>
__device__ __forceinline__ void fast_moments(const FastIn<PREC, PBF>& in, const FastScalars& S, float2 (&m_new)[4],
                                             float2 (&v)[4]) {
  using TR = StateTraits<PREC, PBF>;
  using LY = FastLayout<PREC, PBF>;
  constexpr bool kMBF = TR::kMathBF;
  constexpr int kStore = TR::kStore;
  auto Rm2 = [](float2 x) { return kMBF ? make_float2(round_bf16(x.x), round_bf16(x.y)) : x; };
  constexpr bool vbf = kMBF && !FACT;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 gi = pair_of<LY::BPP, true>(in.g, i);
    float2 vh;
    if (FACT) {
      const float2 mv = (i == 0) ? make_float2(in.mva.x, in.mva.y) : (i == 1) ? make_float2(in.mva.z, in.mva.w)
                      : (i == 2) ? make_float2(in.mvb.x, in.mvb.y) : make_float2(in.mvb.z, in.mvb.w);
      vh = mul2(splat2(in.mu), mv);
    } else {
      vh = pair_of<LY::BPS, false>(in.v, i);
      if (kStore == 2) vh = mul2(vh, splat2(in.vs));
    }
    // v = v*beta2 + c_v*g*g  (factored v is >= 0, so its abs() is the identity)
    float2 vi = mul2(vh, splat2(S.beta2));
    if (vbf) vi = make_float2(round_bf16(vi.x), round_bf16(vi.y));
    vi = fma2(mul2(splat2(S.c_v), gi), gi, vi);
    if (vbf) vi = make_float2(round_bf16(vi.x), round_bf16(vi.y));
    v[i] = vi;
    if (cf_has_m<CF>(S)) {
      float2 m0;
      if (FM) {
        // _reconstruct_state(signed=True): outer(mu, mv), negated where the
        // sign bit is clear (factorization_util.py:9-19)
        const float2 mv = (i == 0) ? make_float2(in.fma.x, in.fma.y) : (i == 1) ? make_float2(in.fma.z, in.fma.w)
                        : (i == 2) ? make_float2(in.fmb.x, in.fmb.y) : make_float2(in.fmb.z, in.fmb.w);
        const float2 a = mul2(splat2(in.fmu), mv);
        m0 = make_float2(((in.fsg >> (2 * i)) & 1u) ? a.x : -a.x, ((in.fsg >> (2 * i + 1)) & 1u) ? a.y : -a.y);
      } else {
        m0 = pair_of<LY::BPS, true>(in.m, i);
        if (kStore == 2) m0 = mul2(m0, splat2(in.ms));
      }
      if (ALGO == ADVOPT_ALGO_PRODIGY) m_new[i] = Rm2(fma2(gi, splat2(S.c_m), Rm2(mul2(m0, splat2(S.beta1)))));
      else m_new[i] = Rm2(lerp2(m0, gi, S.w_m, S.w_m1, cf_msmall<CF>(S)));
    } else {
      m_new[i] = splat2(0.0f);
    }
  }
}

// Parameter update from the moments (AdamW_adv.py:441-465,
// Muon_AuxAdam.py:176-192, Prodigy_adv.py:471-519, param_update.py:77-156):
// packed param words (bf16 pairs after stochastic rounding or RNE; f32
// values).  FAST: Newton–Markstein sqrt / division; `hard` reports elements
// outside their exact range, for which the caller reruns this function with
// the IEEE operations.
template <int PREC, bool PBF, int ALGO, int CF, bool FACT, bool FAST>
__device__ __forceinline__ void fast_update(const Words<FastLayout<PREC, PBF>::BPP>& g,
                                            const Words<FastLayout<PREC, PBF>::BPP>& p, const float2 (&m_new)[4],
                                            const float2 (&v)[4], const FastScalars& S, const uint32_t (&npw)[4],
                                            uint32_t (&pw)[PBF ? 4 : 8], bool& hard, bool emit) {
  using TR = StateTraits<PREC, PBF>;
  using LY = FastLayout<PREC, PBF>;
  constexpr bool kMBF = TR::kMathBF;
  auto Rm2 = [](float2 x) { return kMBF ? make_float2(round_bf16(x.x), round_bf16(x.y)) : x; };
  constexpr bool vbf = kMBF && !FACT;
  float lo = 0x1p100f, hi = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 gi = pair_of<LY::BPP, true>(g, i);
    const float2 vi = v[i];
    float2 ui;
    if (cf_has_m<CF>(S)) {
      const float2 mi = m_new[i];
      ui = cf_nest<CF>(S) ? Rm2(lerp2(mi, gi, S.w_n, S.w_n1, cf_nsmall<CF>(S))) : mi;
    } else {
      ui = (ALGO == ADVOPT_ALGO_PRODIGY) ? Rm2(mul2(gi, splat2(S.d))) : gi;
    }
    // denominator
    float2 den;
    if (FAST) {
      lo = min3f(lo, vi.x, vi.y);
      lo = min3f(lo, fabsf(ui.x), fabsf(ui.y));
      den = sqrt_nm2(vi);
    } else {
      den = make_float2(__fsqrt_rn(vi.x), __fsqrt_rn(vi.y));
    }
    if (vbf) den = make_float2(round_bf16(den.x), round_bf16(den.y));
    if (ALGO != ADVOPT_ALGO_PRODIGY) {
      den = div_rcp2(den, S.sbc2, S.rcp_sbc2);
      if (vbf) den = make_float2(round_bf16(den.x), round_bf16(den.y));
    }
    den = add2(den, splat2(S.eps));
    if (vbf) den = make_float2(round_bf16(den.x), round_bf16(den.y));
    const float2 du = kMBF ? make_float2(round_bf16(den.x), round_bf16(den.y)) : den;
    if (FAST) hi = max3f(hi, du.x, du.y);
    ui = FAST ? div_nm2(ui, du) : make_float2(__fdiv_rn(ui.x, du.x), __fdiv_rn(ui.y, du.y));
    ui = Rm2(ui);
    if (emit) {
      // spectral normalisation: the update before its scaling, in the param
      // dtype (AdamW_adv.py:459-461; scaled_optm.py:269 casts it there)
      if (PBF) {
        pw[i] = f_to_bf16_rne(ui.x) | (f_to_bf16_rne(ui.y) << 16);
      } else {
        pw[2 * i] = __float_as_uint(ui.x);
        pw[2 * i + 1] = __float_as_uint(ui.y);
      }
      continue;
    }
    ui = Rm2(mul2(ui, splat2(S.step_size)));
    // parameter update (param_update.py:77-156)
    float2 pc2 = pair_of<LY::BPP, true>(p, i);
    if (cf_wd<CF>(S)) {
      if (cf_cautious<CF>(S)) {
        float2 prod = mul2(ui, pc2);
        if (PBF && !cf_sr<CF>(S)) prod = make_float2(round_bf16(prod.x), round_bf16(prod.y));
        const float2 mask = make_float2(prod.x >= 0.0f ? 1.0f : 0.0f, prod.y >= 0.0f ? 1.0f : 0.0f);
        pc2 = fma2(mul2(splat2(-S.wd), pc2), mask, pc2);
      } else {
        // add_(p, alpha=-wd): alpha rounded to bf16 on a bf16 tensor (no SR)
        pc2 = fma2(pc2, splat2(-((PBF && !cf_sr<CF>(S)) ? round_bf16(S.wd) : S.wd)), pc2);
      }
      if (PBF && !cf_sr<CF>(S)) pc2 = make_float2(round_bf16(pc2.x), round_bf16(pc2.y));
    }
    const float2 pn = add2(pc2, neg2(ui));
    if (PBF) {
      if (cf_sr<CF>(S))
        pw[i] = __byte_perm(__float_as_uint(pn.x) + (npw[i] & 0xFFFFu), __float_as_uint(pn.y) + (npw[i] >> 16), 0x7632);
      else
        pw[i] = f_to_bf16_rne(pn.x) | (f_to_bf16_rne(pn.y) << 16);
    } else {
      pw[2 * i] = __float_as_uint(pn.x);
      pw[2 * i + 1] = __float_as_uint(pn.y);
    }
  }
  // NaN inputs fail both comparisons and take the IEEE path as well
  hard = FAST && !(lo >= 0x1p-100f && hi <= 0x1p24f);
}

__device__ __forceinline__ uint32_t fbits_max_warp(float a) {
  return __reduce_max_sync(0xffffffffu, __float_as_uint(a));
}

// Resident CTAs per SM the register budget is sized for: three for the
// int8_sr / bf16 Adam step (the Llama configuration), two elsewhere.
template <int PREC, bool PBF, int ALGO>
struct FastOcc {
  static constexpr int v = (PREC == ADVOPT_PREC_INT8_SR && PBF && ALGO != ADVOPT_ALGO_PRODIGY) ? 3 : 2;
};

// FM: a launch of signed rank-1 momentum tensors only ('factored', float32
// launches): m is rebuilt from its factors and sign bytes instead of being
// streamed through the ring, and its |m| row sums and column partials use a
// second accumulator area after the second moment's.
template <int PREC, bool PBF, int ALGO, bool NOISE_IN, int CF, bool FM = false>
__global__ void __launch_bounds__(kThreads, (FastOcc<PREC, PBF, ALGO>::v))
    adam_fast_kernel(const advopt_adam_launch L, const PhiloxKeys K) {
  using TR = StateTraits<PREC, PBF>;
  using LY = FastLayout<PREC, PBF>;
  constexpr int kStore = TR::kStore;
  constexpr int kMaxStages = 4;
  extern __shared__ float4 dsm4[];
  float* colacc = reinterpret_cast<float*>(dsm4);
  static_assert(!FM || PREC == ADVOPT_PREC_FP32, "factored momentum is float32");
  float* colacc_m = colacc + (FM ? L.gen_offset : 0);
  unsigned char* stages = reinterpret_cast<unsigned char*>(colacc + (FM ? 2 : 1) * L.gen_offset);
  __shared__ uint64_t bars[kMaxStages];
  __shared__ int direct[kMaxStages];
  __shared__ int abort_flag;
  __shared__ uint32_t redm[2][kWarps], redv[2][kWarps];
  __shared__ float redr[2][kWarps];
  __shared__ float redrm[2][kWarps];
  __shared__ double dred[kWarps][2];
  __shared__ double gred[kWarps];
  __shared__ TensorRegs Ts;
  __shared__ PieceRegs Ps;
  __shared__ Cursor cur;          // producer state (thread 0 only)
  __shared__ int cur_valid;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int S = L.stages;
  const uint32_t F = L.flags;
  const bool has_m = CF < 0 ? (F & ADVOPT_F_HAS_M) != 0 : (CF & kCfHasM) != 0;
  const bool ring_m = has_m && !FM;    // m streamed through the stage ring
  const bool pstats = (ALGO == ADVOPT_ALGO_PRODIGY) && (F & ADVOPT_F_PRODIGY_STATS);
  // spectral normalisation (the kCfDynEmit variant): write the unscaled
  // update where the param would be written, and leave the param alone
  constexpr bool emit = CF == kCfDynEmit;
  const bool gsq = F & ADVOPT_F_GRAD_SQ;
  FastScalars SC;
  SC.beta1 = L.beta1;
  SC.beta2 = L.beta2;
  // Prodigy with d on the device reads its launch scalars from there
  const bool pdev = ALGO == ADVOPT_ALGO_PRODIGY && L.prodigy != nullptr;
  const float c_v0 = pdev ? L.prodigy->c_v : L.c_v;
  const float s_alpha = pdev ? L.prodigy->s_alpha : L.s_alpha;
  SC.c_v = c_v0;
  SC.c_m = pdev ? L.prodigy->c_m : L.c_m;
  // Prodigy's m.add_(grad, alpha=...) rounds alpha to bf16 under bf16 math
  if (StateTraits<PREC, PBF>::kMathBF) SC.c_m = round_bf16(SC.c_m);
  SC.w_m = L.w_m;
  SC.w_m1 = __fsub_rn(L.w_m, 1.0f);
  SC.w_n = L.w_nest;
  SC.w_n1 = __fsub_rn(L.w_nest, 1.0f);
  SC.d = pdev ? L.prodigy->d_f : L.d;
  SC.w_m_small = fabsf(L.w_m) < 0.5f;
  SC.w_n_small = fabsf(L.w_nest) < 0.5f;
  SC.has_m = has_m;
  SC.nest = F & ADVOPT_F_NESTEROV;
  SC.cautious = F & ADVOPT_F_CAUTIOUS;
  SC.sr = PBF && (F & ADVOPT_F_SR);

  const int pbeg = L.cta_offsets[blockIdx.x], pend = L.cta_offsets[blockIdx.x + 1];
  if (pbeg >= pend) return;

  // ---- producer prologue: fill the ring ----
  if (tid == 0) {
    abort_flag = 0;
    for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
    mbar_fence_init();
    cur.pi = pbeg;
    cur.tensor = -1;
    cur_valid = cursor_seek<PREC, PBF>(L, cur, pend);
    for (int s = 0; s < S && cur_valid; ++s) {
      issue_chunk<PREC, PBF>(cur, stages + (size_t)s * LY::BYTES, &bars[s], &direct[s], ring_m);
      cur_valid = cursor_next<PREC, PBF>(L, cur, pend);
    }
  }
  __syncthreads();

  int parity = 0;
  int slot = 0;         // consumer position in the ring
  uint32_t par = 0u;    // its mbarrier phase
  for (int pi = pbeg; pi < pend; ++pi) {
    const advopt_piece pc = L.pieces[pi];
    __syncthreads();
    if (tid == 0) {
      load_tensor(L.tensors + pc.tensor, Ts);
      piece_regs<PREC, PBF>(Ts, pc.begin, Ps);
    }
    __syncthreads();
    const TensorRegs& T = Ts;
    const bool fact = T.flags & ADVOPT_T_FACTORED;
    const bool vec = T.flags & ADVOPT_T_VEC;
    const int64_t d2 = fact ? T.d2 : 1;
    // factored tensors wider than the shared-memory accumulator keep their
    // column partials in their own global slot row (read-modify-write)
    const bool col_global = fact && d2 > (int64_t)L.gen_offset;
    float* colrow = fact ? (col_global ? T.colpart + (int64_t)pc.slot * d2 : colacc) : nullptr;
    float* colrow_m = FM ? (col_global ? T.mcolpart + (int64_t)pc.slot * d2 : colacc_m) : nullptr;
    if (L.layer_beta2) {
      // Kourkoutas-beta: the tensor's layer's dynamic beta2 (Kourkoutas.py:249-257)
      const int l = L.layer_of_tensor[pc.tensor];
      SC.beta2 = l >= 0 ? L.layer_beta2[2 * l] : L.beta2;
      SC.c_v = l >= 0 ? L.layer_beta2[2 * l + 1] : c_v0;
    }
    double gacc = 0.0;     // Kourkoutas-beta: this thread's sum of g*g over the piece
    SC.sbc2 = T.sqrt_bc2;
    SC.rcp_sbc2 = __frcp_rn(T.sqrt_bc2);
    SC.eps = T.eps;
    SC.step_size = T.step_size;
    SC.wd = T.wd;
    if (fact) {
      for (int j2 = tid * 4; j2 < (int)d2; j2 += kThreads * 4)
        *reinterpret_cast<float4*>(colrow + j2) = make_float4(0.f, 0.f, 0.f, 0.f);
      if (FM)
        for (int j2 = tid * 4; j2 < (int)d2; j2 += kThreads * 4)
          *reinterpret_cast<float4*>(colrow_m + j2) = make_float4(0.f, 0.f, 0.f, 0.f);
      __syncthreads();
    }
    // Per-piece constants: the descriptor fields the chunks use, read once
    // from shared memory, with the piece's first element folded in.  Offsets
    // inside a piece fit 32 bits (the host sends tensors of 2^34 or more
    // elements to the general kernel), as do the Philox element groups.
    const int64_t pb = pc.begin;          // a multiple of the 2048-element block
    const int plen = (int)(pc.end - pc.begin);
    const PieceRegs& P = Ps;
    const int d2i = (int)d2;
    int r0 = fact ? (int)(pb / d2) : 0;
    int c0 = fact ? (int)(pb - (int64_t)r0 * d2) : 0;
    float racc0 = 0.0f, racc1 = 0.0f;   // this thread's part of rows r0 and r0 + 1
    float raccm0 = 0.0f, raccm1 = 0.0f; // FM: the same for |m|
    double st0 = 0.0, st1 = 0.0;
    const uint32_t slice_p = T.slice_p ? T.slice_p : 1u;
    // Prodigy: this thread's first element's remainder mod slice_p, advanced
    // by one chunk's remainder per chunk (one 64-bit division per piece, none
    // per element); slice indices below 2^32 divide in 32 bits
    uint32_t srem = pstats ? (uint32_t)((uint64_t)(pb + tid * kVec) % slice_p) : 0u;
    const uint32_t srem_step = (uint32_t)kChunk % slice_p;
    const bool si32 = T.numel < (int64_t(1) << 32);

    // Scalars of a chunk (factored row / column factors, block scales),
    // loaded one chunk ahead so their L2 latency overlaps the current chunk.
    float pre_mu = 0.0f, pre_ms = 0.0f, pre_vs = 0.0f;
    float4 pre_a = make_float4(0.f, 0.f, 0.f, 0.f), pre_b = pre_a;
    float pre_fmu = 0.0f;
    float4 pre_fa = pre_a, pre_fb = pre_a;
    uint32_t pre_sg = 0u;
    auto prefetch = [&](int off, int c0n, int r0n, auto fact_tag) {
      constexpr bool fct = decltype(fact_tag)::value;
      if (fct) {
        const int nvn = min(kVec, plen - off - tid * kVec);
        const int cc = c0n + tid * kVec;
        const bool sec = cc >= d2i;
        const int col = sec ? cc - d2i : cc;
        pre_mu = nvn > 0 ? P.row[r0n + (sec ? 1 : 0)] : 0.0f;
        pre_a = *reinterpret_cast<const float4*>(P.col + col);
        pre_b = *(reinterpret_cast<const float4*>(P.col + col) + 1);
        if (FM) {
          pre_fmu = nvn > 0 ? P.mrow[r0n + (sec ? 1 : 0)] : 0.0f;
          pre_fa = *reinterpret_cast<const float4*>(P.mcol + col);
          pre_fb = *(reinterpret_cast<const float4*>(P.mcol + col) + 1);
          // the thread's 8 elements are one sign byte (8-aligned columns)
          pre_sg = nvn > 0 ? (uint32_t)P.msign[(pb + off + tid * kVec) >> 3] : 0u;
        }
      }
      if (kStore == 2 && has_m) pre_ms = P.ms[off >> 11];
      if (kStore == 2 && !fct) pre_vs = P.vs[off >> 11];
    };
    if (fact) prefetch(0, c0, r0, std::true_type{});
    else prefetch(0, c0, r0, std::false_type{});

    // One chunk at piece offset `off`; FULL: all 2048 elements present and
    // 16-byte aligned (the common case, with the tail predicates compiled
    // out).  Returns false when a bounded wait gave up.
    auto chunk = [&](int off, auto full_tag, auto fact_tag) -> bool {
      constexpr bool kFull = decltype(full_tag)::value;
      constexpr bool fact = decltype(fact_tag)::value;   // shadows the piece's flag
      const int clen = kFull ? kChunk : min(kChunk, plen - off);
      const int toff = off + tid * kVec;                 // this thread's first element in the piece
      const int64_t k0 = pb + toff;
      const int nv = kFull ? kVec : max(0, min(kVec, clen - tid * kVec));
      const bool v8 = kFull ? true : (vec && nv == kVec);
      int col = 0;
      bool second = false;
      if (fact) {
        const int cc = c0 + tid * kVec;
        second = cc >= d2i;
        col = second ? cc - d2i : cc;
      }
      // Philox words of one noise stream for this thread's 8 elements
      auto noise = [&](const int32_t* arr, uint32_t stream) -> U4 {
        if (NOISE_IN) return noise_words_k<true>(K, T, arr, stream, k0, nv);
        return philox4x32_10_k(U4{P.gbase + ((uint32_t)toff >> 3), stream << 24, P.tensor_id, P.step}, K);
      };
      SliceAt sl;          // this thread's first Prodigy slice point in the chunk
      sl.e = kVec;
      if (pstats) {
        const int first = srem ? (int)(slice_p - srem) : 0;
        if (first < nv) slice_fetch<PBF>(T, k0, first, slice_p, si32, sl);
      }
      FastIn<PREC, PBF> in;
      in.mu = pre_mu;
      in.mva = pre_a;
      in.mvb = pre_b;
      in.ms = pre_ms;
      in.vs = pre_vs;
      in.fmu = pre_fmu;
      in.fma = pre_fa;
      in.fmb = pre_fb;
      in.fsg = pre_sg;
      if (!mbar_wait(&bars[slot], par)) {
        // the copies never arrived: report, finish this chunk on whatever is
        // in the stage, and leave uniformly after the next barrier
        abort_flag = 1;
        if (L.err) atomicExch(L.err, 1);
      }
      const unsigned char* st = stages + (size_t)slot * LY::BYTES;
      const bool dir = kFull ? false : (direct[slot] != 0);
      fast_load<PREC, PBF>(T, st, dir, k0, nv, v8, ring_m, fact, in);
      U4 nzp{0u, 0u, 0u, 0u};
      if (cf_sr<CF>(SC)) nzp = noise(T.nz_p, kNoiseP);
      if (gsq) {
        // torch.sum(grad.pow(2)) of the grad the step uses: squares in bf16
        // for a bf16 grad under 'auto' (Kourkoutas.py:241-245)
        float s8 = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 gp = pair_of<LY::BPP, true>(in.g, i);
          float q0 = __fmul_rn(gp.x, gp.x), q1 = __fmul_rn(gp.y, gp.y);
          if (TR::kMathBF) { q0 = round_bf16(q0); q1 = round_bf16(q1); }
          if (2 * i < nv) s8 = __fadd_rn(s8, q0);
          if (2 * i + 1 < nv) s8 = __fadd_rn(s8, q1);
        }
        gacc += (double)s8;
      }
      float2 m_new[4], v[4];
      uint32_t pw[PBF ? 4 : 8];
      fast_moments<PREC, PBF, ALGO, CF, fact, FM>(in, SC, m_new, v);
      {
        const uint32_t npw[4] = {nzp.x, nzp.y, nzp.z, nzp.w};
        bool hard = false;
        fast_update<PREC, PBF, ALGO, CF, fact, true>(in.g, in.p, m_new, v, SC, npw, pw, hard, emit);
        if (__any_sync(0xffffffffu, hard)) {
          // some lane of the warp is outside the Newton–Markstein ranges:
          // redo the warp's parameter update with the IEEE operations (the
          // moments are exact either way); its grad / param words and noise
          // are fetched again rather than kept live through the fast path
          FastIn<PREC, PBF> in2;
          fast_load<PREC, PBF>(T, st, dir, k0, nv, v8, false, true, in2);
          U4 nz2{0u, 0u, 0u, 0u};
          if (cf_sr<CF>(SC)) nz2 = noise(T.nz_p, kNoiseP);
          const uint32_t npw2[4] = {nz2.x, nz2.y, nz2.z, nz2.w};
          bool h2;
          fast_update<PREC, PBF, ALGO, CF, fact, false>(in2.g, in2.p, m_new, v, SC, npw2, pw, h2, emit);
        }
      }
      if (!kFull) {
        // elements past the tensor's end stay out of the block maxima and sums
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (!(2 * i < nv)) { m_new[i].x = 0.0f; v[i].x = 0.0f; }
          if (!(2 * i + 1 < nv)) { m_new[i].y = 0.0f; v[i].y = 0.0f; }
        }
      }

      if (pstats) {
        // Prodigy slice statistics on g and p before the update
        // (Prodigy_adv.py:494-509): the prefetched first point, then any
        // further ones (slice_p < 8)
        for (int e = sl.e; e < nv;) {
          float gv = 0.0f, pv = 0.0f;
#pragma unroll
          for (int j = 0; j < 8; j += 2) {
            const float2 gp = pair_of<LY::BPP, true>(in.g, j >> 1), pp = pair_of<LY::BPP, true>(in.p, j >> 1);
            if (e == j) { gv = gp.x; pv = pp.x; }
            if (e == j + 1) { gv = gp.y; pv = pp.y; }
          }
          slice_apply<PBF>(T, sl, gv, pv, L.beta3, s_alpha, st0, st1);
          e += (int)slice_p;
          if (e < nv) slice_fetch<PBF>(T, k0, e, slice_p, si32, sl);
        }
        srem += srem_step;
        if (srem >= slice_p) srem -= slice_p;
      }

      // param store
      if (PBF) {
        uint16_t* dst = reinterpret_cast<uint16_t*>(emit ? P.u : P.p) + toff;
        if (v8) {
          *reinterpret_cast<uint4*>(dst) = make_uint4(pw[0], pw[1], pw[2], pw[3]);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (e < nv) dst[e] = (uint16_t)(pw[e >> 1] >> (16 * (e & 1)));
        }
      } else {
        float* dst = reinterpret_cast<float*>(emit ? P.u : P.p) + toff;
        if (v8) {
          reinterpret_cast<uint4*>(dst)[0] = make_uint4(pw[0], pw[1], pw[2], pw[3]);
          reinterpret_cast<uint4*>(dst)[1] = make_uint4(pw[4], pw[5], pw[6], pw[7]);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (e < nv) dst[e] = __uint_as_float(pw[e]);
        }
      }

      // block maxima of the quantised states (bit patterns of non-negative
      // floats order like the values)
      if (has_m && kStore == 2) {
        float a = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) a = max3f(a, fabsf(m_new[i].x), fabsf(m_new[i].y));
        const uint32_t wm = fbits_max_warp(a);
        if (lane == 0) redm[parity][warp] = wm;
      }
      if (!fact && kStore == 2) {
        float b = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) b = max3f(b, v[i].x, v[i].y);
        const uint32_t wv = fbits_max_warp(b);
        if (lane == 0) redv[parity][warp] = wv;
      }
      // factored: column partials and this thread's row parts
      bool row_done = false;
      if (fact) {
        if (nv > 0) {
          float4* ca = reinterpret_cast<float4*>(colrow + col);
          float4 a = ca[0], b = ca[1];
          const float2 a01 = add2(make_float2(a.x, a.y), v[0]), a23 = add2(make_float2(a.z, a.w), v[1]);
          const float2 b01 = add2(make_float2(b.x, b.y), v[2]), b23 = add2(make_float2(b.z, b.w), v[3]);
          ca[0] = make_float4(a01.x, a01.y, a23.x, a23.y);
          ca[1] = make_float4(b01.x, b01.y, b23.x, b23.y);
        }
        const float2 s01 = add2(v[0], v[1]), s23 = add2(v[2], v[3]);
        const float2 s = add2(s01, s23);
        const float sum = __fadd_rn(s.x, s.y);
        if (second) racc1 = __fadd_rn(racc1, sum);
        else racc0 = __fadd_rn(racc0, sum);
        row_done = clen >= d2i - c0;   // row r0 ends inside this chunk (uniform)
        if (FM) {
          // _factorize_state(signed=True) (factorization_util.py:25-32): the
          // sign bits of m > 0, |m| row sums and column partials
          float2 am[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) am[i] = make_float2(fabsf(m_new[i].x), fabsf(m_new[i].y));
          if (nv > 0) {
            uint32_t sb = 0u;
#pragma unroll
            for (int i = 0; i < 4; ++i)
              sb |= ((m_new[i].x > 0.0f ? 1u : 0u) << (2 * i)) | ((m_new[i].y > 0.0f ? 1u : 0u) << (2 * i + 1));
            P.msign[k0 >> 3] = (uint8_t)sb;
            float4* cm = reinterpret_cast<float4*>(colrow_m + col);
            float4 a = cm[0], b = cm[1];
            const float2 a01 = add2(make_float2(a.x, a.y), am[0]), a23 = add2(make_float2(a.z, a.w), am[1]);
            const float2 b01 = add2(make_float2(b.x, b.y), am[2]), b23 = add2(make_float2(b.z, b.w), am[3]);
            cm[0] = make_float4(a01.x, a01.y, a23.x, a23.y);
            cm[1] = make_float4(b01.x, b01.y, b23.x, b23.y);
          }
          const float2 t = add2(add2(am[0], am[1]), add2(am[2], am[3]));
          const float tsum = __fadd_rn(t.x, t.y);
          if (second) raccm1 = __fadd_rn(raccm1, tsum);
          else raccm0 = __fadd_rn(raccm0, tsum);
        }
        if (row_done) {
          const float w = warp_sum(racc0);
          if (lane == 0) redr[parity][warp] = w;
          if (FM) {
            const float wm = warp_sum(raccm0);
            if (lane == 0) redrm[parity][warp] = wm;
          }
        }
      }
      __syncthreads();
      if (abort_flag) return false;   // every thread reads the same flag after the barrier
      // every thread is done with this stage: refill it with the chunk S ahead
      if (tid == 0 && cur_valid) {
        issue_chunk<PREC, PBF>(cur, stages + (size_t)slot * LY::BYTES, &bars[slot], &direct[slot], ring_m);
        cur_valid = cursor_next<PREC, PBF>(L, cur, pend);
      }
      // noise of the quantised states
      U4 nzm{0u, 0u, 0u, 0u}, nzv{0u, 0u, 0u, 0u};
      if (kStore == 2 || TR::kSRStates) {
        if (ring_m) nzm = noise(T.nz_m, kNoiseM);
        if (!fact) nzv = noise(T.nz_v, kNoiseV);
      }
      if (row_done) {
        if (tid == 0) {
          double t = 0.0;
#pragma unroll
          for (int w = 0; w < kWarps; ++w) t += (double)redr[parity][w];
          P.row[r0] = (float)t;
          if (FM) {
            double tm = 0.0;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) tm += (double)redrm[parity][w];
            P.mrow[r0] = (float)tm;
          }
        }
        racc0 = racc1;
        racc1 = 0.0f;
        raccm0 = raccm1;
        raccm1 = 0.0f;
      }
      if (ring_m) {
        if (kStore == 2) {
          const float bmax = __uint_as_float(__reduce_max_sync(0xffffffffu, redm[parity][lane & (kWarps - 1)]));
          const float scale = block_scale<true>(bmax);
          const uint2 q = quantize8x2<true>(m_new, scale, nzm);
          uint8_t* dst = P.m + toff;
          if (v8) {
            *reinterpret_cast<uint2*>(dst) = q;
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e)
              if (e < nv) dst[e] = (uint8_t)((e < 4 ? q.x : q.y) >> (8 * (e & 3)));
          }
          if (tid == 0) P.ms[off >> 11] = scale;
        } else if (kStore == 1) {
          uint32_t b[8];
          const uint32_t nmw[4] = {nzm.x, nzm.y, nzm.z, nzm.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            b[2 * i] = TR::kSRStates ? f_to_bf16_sr(m_new[i].x, nmw[i] & 0xFFFFu) : f_to_bf16_rne(m_new[i].x);
            b[2 * i + 1] = TR::kSRStates ? f_to_bf16_sr(m_new[i].y, nmw[i] >> 16) : f_to_bf16_rne(m_new[i].y);
          }
          store8_bf16(T.m, k0, nv, v8, b);
        } else {
          const float mf[8] = {m_new[0].x, m_new[0].y, m_new[1].x, m_new[1].y,
                               m_new[2].x, m_new[2].y, m_new[3].x, m_new[3].y};
          store8_f32(T.m, k0, nv, v8, mf);
        }
      }
      if (!fact) {
        if (kStore == 2) {
          const float bmax = __uint_as_float(__reduce_max_sync(0xffffffffu, redv[parity][lane & (kWarps - 1)]));
          const float scale = block_scale<false>(bmax);
          const uint2 q = quantize8x2<false>(v, scale, nzv);
          uint8_t* dst = static_cast<uint8_t*>(T.v) + k0;
          if (v8) {
            *reinterpret_cast<uint2*>(dst) = q;
          } else {
#pragma unroll
            for (int e = 0; e < 8; ++e)
              if (e < nv) dst[e] = (uint8_t)((e < 4 ? q.x : q.y) >> (8 * (e & 3)));
          }
          if (tid == 0) P.vs[off >> 11] = scale;
        } else if (kStore == 1) {
          uint32_t b[8];
          const uint32_t nvw[4] = {nzv.x, nzv.y, nzv.z, nzv.w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            b[2 * i] = TR::kSRStates ? f_to_bf16_sr(v[i].x, nvw[i] & 0xFFFFu) : f_to_bf16_rne(v[i].x);
            b[2 * i + 1] = TR::kSRStates ? f_to_bf16_sr(v[i].y, nvw[i] >> 16) : f_to_bf16_rne(v[i].y);
          }
          store8_bf16(T.v, k0, nv, v8, b);
        } else {
          const float vf[8] = {v[0].x, v[0].y, v[1].x, v[1].y, v[2].x, v[2].y, v[3].x, v[3].y};
          store8_f32(T.v, k0, nv, v8, vf);
        }
      }
      if (fact) {
        c0 += clen;
        if (c0 >= d2i) {
          c0 -= d2i;
          r0 += 1;
        }
      }
      if (off + kChunk < plen) prefetch(off + kChunk, c0, r0, fact_tag);
      parity ^= 1;
      if (++slot == S) {
        slot = 0;
        par ^= 1u;
      }
      return true;
    };
    for (int off = 0; off < plen; off += kChunk) {
      const bool full = vec && (plen - off >= kChunk);
      const bool ok = full ? (fact ? chunk(off, std::true_type{}, std::true_type{})
                                   : chunk(off, std::true_type{}, std::false_type{}))
                           : (fact ? chunk(off, std::false_type{}, std::true_type{})
                                   : chunk(off, std::false_type{}, std::false_type{}));
      if (!ok) return;
    }

    if (fact) {
      __syncthreads();
      if (!col_global) {
        float* dstp = T.colpart + (int64_t)pc.slot * d2;
        for (int j2 = tid * 4; j2 < (int)d2; j2 += kThreads * 4)
          *reinterpret_cast<float4*>(dstp + j2) = *reinterpret_cast<const float4*>(colacc + j2);
        if (FM) {
          float* dstm = T.mcolpart + (int64_t)pc.slot * d2;
          for (int j2 = tid * 4; j2 < (int)d2; j2 += kThreads * 4)
            *reinterpret_cast<float4*>(dstm + j2) = *reinterpret_cast<const float4*>(colacc_m + j2);
        }
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
    if (pstats) {
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

}  // namespace advopt
