// Fast path of the Adam-family step (included by adam_impl.cuh users).
//
// Same arithmetic as adam_kernel (op for op), restricted to the common
// configurations: no atan2 / normed momentum / Fisher / centered anchors, and
// factored tensors only with d2 >= 2048, d2 % 8 == 0 (every Llama-shaped
// effective shape).  Differences in structure:
//   * each chunk's inputs (grad, param, m codes, v codes) stream into a ring
//     of shared-memory stages with cp.async.bulk (TMA bulk copies, no
//     multicast) completed on mbarriers, `stages` chunks ahead, so memory
//     latency is hidden without holding prefetched data in registers;
//   * element arithmetic runs on fp32x2 lanes (sm_100 packed FFMA2/FADD2/FMUL2);
//   * waits are bounded: a wait that gives up sets *L.err and the CTA stops.
#pragma once

namespace advopt {

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

template <int BPE, bool SIGNED>
__device__ __forceinline__ void unpack8x2(const Words<BPE>& in, float2 (&x)[4]) {
  float t[8];
  unpack8<BPE, SIGNED>(in, t);
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = make_float2(t[2 * i], t[2 * i + 1]);
}

// Two-lane stochastic quantisation with a per-block divisor; returns the
// packed codes of 8 values.
template <bool SIGNED>
__device__ __forceinline__ uint2 quantize8x2(const float2 (&x)[4], float bmax, const U4& nz) {
  const float scale = __fdiv_rn(bmax, SIGNED ? 127.0f : 255.0f);
  const float safe = scale < 1e-12f ? 1e-12f : scale;
  const float rs = __frcp_rn(safe);
  bool tiny = false;
#pragma unroll
  // zeros are exact through div_rcp2 (and the noise add absorbs a -0); only
  // nonzero magnitudes below 2^-100 need the IEEE division
  for (int i = 0; i < 4; ++i)
    tiny |= (fabsf(x[i].x) < 0x1p-100f && x[i].x != 0.0f) | (fabsf(x[i].y) < 0x1p-100f && x[i].y != 0.0f);
  const bool any_tiny = __any_sync(0xffffffffu, tiny);
  const uint32_t nw[4] = {nz.x, nz.y, nz.z, nz.w};
  int c[8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 q = div_rcp2(x[i], safe, rs);
    if (any_tiny) {
      if (fabsf(x[i].x) < 0x1p-100f && x[i].x != 0.0f) q.x = __fdiv_rn(x[i].x, safe);
      if (fabsf(x[i].y) < 0x1p-100f && x[i].y != 0.0f) q.y = __fdiv_rn(x[i].y, safe);
    }
    // noise r * 2^-16 from bits: (1 + r*2^-16) - 1
    const float2 n1 = make_float2(__uint_as_float(0x3F800000u | ((nw[i] & 0xFFFFu) << 7)),
                                  __uint_as_float(0x3F800000u | ((nw[i] >> 16) << 7)));
    const float2 noise = add2(n1, splat2(-1.0f));
    const float2 y = add2(q, noise);
    const float2 f = __fadd2_rd(y, splat2(12582912.0f));   // 1.5*2^23 + floor(y)
    const int f0 = (int)(__float_as_uint(f.x) - 0x4B400000u), f1 = (int)(__float_as_uint(f.y) - 0x4B400000u);
    c[2 * i] = SIGNED ? min(max(f0, -127), 127) : min(max(f0, 0), 255);
    c[2 * i + 1] = SIGNED ? min(max(f1, -127), 127) : min(max(f1, 0), 255);
  }
  return make_uint2(pack4_bytes(c[0], c[1], c[2], c[3]), pack4_bytes(c[4], c[5], c[6], c[7]));
}

template <int PREC, bool PBF, int ALGO, bool NOISE_IN>
__global__ void __launch_bounds__(kThreads, 2) adam_fast_kernel(const advopt_adam_launch L) {
  using TR = StateTraits<PREC, PBF>;
  using LY = FastLayout<PREC, PBF>;
  constexpr int kStore = TR::kStore;
  constexpr bool kMBF = TR::kMathBF;
  constexpr int SB = LY::BPS;
  constexpr int kMaxStages = 4;
  extern __shared__ float4 dsm4[];
  float* colacc = reinterpret_cast<float*>(dsm4);
  unsigned char* stages = reinterpret_cast<unsigned char*>(colacc + L.gen_offset);
  __shared__ uint64_t bars[kMaxStages];
  __shared__ int direct[kMaxStages];
  __shared__ int abort_flag;
  __shared__ float red[2][kWarps][4];
  __shared__ double dred[kWarps][2];
  __shared__ TensorRegs Ts;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int S = L.stages;
  const uint32_t F = L.flags;
  const bool has_m = F & ADVOPT_F_HAS_M;
  const bool nest = F & ADVOPT_F_NESTEROV;
  const bool cautious = F & ADVOPT_F_CAUTIOUS;
  const bool sr = PBF && (F & ADVOPT_F_SR);
  const bool pstats = (ALGO == ADVOPT_ALGO_PRODIGY) && (F & ADVOPT_F_PRODIGY_STATS);
  const float beta1 = L.beta1, beta2 = L.beta2, c_v = L.c_v, c_m = L.c_m;
  const float w_m = L.w_m, w_m1 = __fsub_rn(L.w_m, 1.0f), w_n = L.w_nest, w_n1 = __fsub_rn(L.w_nest, 1.0f);
  const bool w_m_small = fabsf(w_m) < 0.5f, w_n_small = fabsf(w_n) < 0.5f;
  auto Rm = [](float x) { return kMBF ? round_bf16(x) : x; };
  auto Rm2 = [](float2 x) { return kMBF ? make_float2(round_bf16(x.x), round_bf16(x.y)) : x; };

  const int pbeg = L.cta_offsets[blockIdx.x], pend = L.cta_offsets[blockIdx.x + 1];
  if (pbeg >= pend) return;

  // ---- producer prologue: fill the ring ----
  Cursor cur{};
  bool cur_valid = false;
  if (tid == 0) {
    abort_flag = 0;
    for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
    mbar_fence_init();
    cur.pi = pbeg;
    cur.tensor = -1;
    cur_valid = cursor_seek<PREC, PBF>(L, cur, pend);
    for (int s = 0; s < S && cur_valid; ++s) {
      issue_chunk<PREC, PBF>(cur, stages + (size_t)s * LY::BYTES, &bars[s], &direct[s], has_m);
      cur_valid = cursor_next<PREC, PBF>(L, cur, pend);
    }
  }
  __syncthreads();

  int parity = 0;
  uint32_t j = 0;   // chunk counter (consumer)
  for (int pi = pbeg; pi < pend; ++pi) {
    const advopt_piece pc = L.pieces[pi];
    __syncthreads();
    if (tid == 0) load_tensor(L.tensors + pc.tensor, Ts);
    __syncthreads();
    const TensorRegs& T = Ts;
    const bool fact = T.flags & ADVOPT_T_FACTORED;
    const bool vec = T.flags & ADVOPT_T_VEC;
    const int64_t d2 = fact ? T.d2 : 1;
    const bool vbf = kMBF && !fact;
    const float sbc2 = T.sqrt_bc2, rcp_sbc2 = __frcp_rn(T.sqrt_bc2), eps = T.eps, step_size = T.step_size, wd = T.wd;
    if (fact) {
      for (int j2 = tid * 4; j2 < (int)d2; j2 += kThreads * 4)
        *reinterpret_cast<float4*>(colacc + j2) = make_float4(0.f, 0.f, 0.f, 0.f);
      __syncthreads();
    }
    int64_t r0 = fact ? pc.begin / d2 : 0;
    int64_t c0 = fact ? pc.begin - r0 * d2 : 0;
    double row_carry = 0.0, st0 = 0.0, st1 = 0.0;
    const uint32_t slice_p = T.slice_p ? T.slice_p : 1u;

    for (int64_t cs = pc.begin; cs < pc.end; cs += kChunk, ++j) {
      const int slot = (int)(j % (uint32_t)S);
      const uint32_t par = (j / (uint32_t)S) & 1u;
      const int clen = (int)min((int64_t)kChunk, pc.end - cs);
      const int64_t k0 = cs + tid * kVec;
      const int nv = max(0, min(kVec, clen - tid * kVec));
      const bool v8 = vec && nv == kVec;
      const int64_t blk = cs >> 11;
      // factored column factors of this chunk (L2-resident; issued before the wait)
      float mu = 0.0f;
      float4 mva = make_float4(0.f, 0.f, 0.f, 0.f), mvb = mva;
      int64_t col = 0;
      bool second = false;
      if (fact) {
        const int64_t cc = c0 + tid * kVec;
        second = cc >= d2;
        col = second ? cc - d2 : cc;
        mu = nv > 0 ? T.row[r0 + (second ? 1 : 0)] : 0.0f;
        mva = *reinterpret_cast<const float4*>(T.col + col);
        mvb = *(reinterpret_cast<const float4*>(T.col + col) + 1);
      }
      const float ms = (has_m && kStore == 2) ? T.m_scale[blk] : 0.0f;
      const float vs = (!fact && kStore == 2) ? T.v_scale[blk] : 0.0f;
      if (!mbar_wait(&bars[slot], par)) {
        // the copies never arrived: report, finish this chunk on whatever is
        // in the stage, and leave uniformly after the next barrier
        abort_flag = 1;
        if (L.err) atomicExch(L.err, 1);
      }
      const unsigned char* st = stages + (size_t)slot * LY::BYTES;
      const bool dir = direct[slot] != 0;
      Words<LY::BPP> wg, wp;
      Words<SB> wm, wv;
      if (dir) {
        ld_words<LY::BPP>(T.grad, k0, nv, v8, wg);
        ld_words<LY::BPP>(T.param, k0, nv, v8, wp);
        if (has_m) ld_words<SB>(T.m, k0, nv, v8, wm);
        if (!fact) ld_words<SB>(T.v, k0, nv, v8, wv);
      } else {
        lds_words<LY::BPP>(st + LY::G + tid * kVec * LY::BPP, wg);
        lds_words<LY::BPP>(st + LY::P + tid * kVec * LY::BPP, wp);
        if (has_m) lds_words<SB>(st + LY::M + tid * kVec * SB, wm);
        if (!fact) lds_words<SB>(st + LY::V + tid * kVec * SB, wv);
      }
      float2 g[4], p[4], m[4], vh[4];
      unpack8x2<LY::BPP, true>(wg, g);
      unpack8x2<LY::BPP, true>(wp, p);
      if (has_m) {
        unpack8x2<SB, true>(wm, m);
        if (kStore == 2) {
#pragma unroll
          for (int i = 0; i < 4; ++i) m[i] = mul2(m[i], splat2(ms));
        }
      }
      if (fact) {
        const float2 mu2 = splat2(mu);
        vh[0] = mul2(mu2, make_float2(mva.x, mva.y));
        vh[1] = mul2(mu2, make_float2(mva.z, mva.w));
        vh[2] = mul2(mu2, make_float2(mvb.x, mvb.y));
        vh[3] = mul2(mu2, make_float2(mvb.z, mvb.w));
      } else {
        unpack8x2<SB, false>(wv, vh);
        if (kStore == 2) {
#pragma unroll
          for (int i = 0; i < 4; ++i) vh[i] = mul2(vh[i], splat2(vs));
        }
      }
      U4 nzp{0u, 0u, 0u, 0u};
      if (sr) nzp = noise_words<NOISE_IN>(L, T, T.nz_p, kNoiseP, k0, nv);
      const uint32_t npw[4] = {nzp.x, nzp.y, nzp.z, nzp.w};
      int slice_off = 0;
      if (pstats) slice_off = (int)((slice_p - (uint32_t)(k0 % slice_p)) % slice_p);

      float2 m_new[4], v[4];
      float amax_m = 0.0f, vmax = 0.0f;
      uint32_t pout[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 gi = g[i];
        // v = v*beta2 + c_v*g*g
        float2 vi = mul2(vh[i], splat2(beta2));
        if (vbf) vi = make_float2(round_bf16(vi.x), round_bf16(vi.y));
        vi = fma2(mul2(splat2(c_v), gi), gi, vi);
        if (vbf) vi = make_float2(round_bf16(vi.x), round_bf16(vi.y));
        if (fact) vi = make_float2(fabsf(vi.x), fabsf(vi.y));
        v[i] = vi;
        // denominator
        float2 den = make_float2(__fsqrt_rn(vi.x), __fsqrt_rn(vi.y));
        if (vbf) den = make_float2(round_bf16(den.x), round_bf16(den.y));
        if (ALGO != ADVOPT_ALGO_PRODIGY) {
          den = div_rcp2(den, sbc2, rcp_sbc2);
          if (vbf) den = make_float2(round_bf16(den.x), round_bf16(den.y));
        }
        den = add2(den, splat2(eps));
        if (vbf) den = make_float2(round_bf16(den.x), round_bf16(den.y));
        const float2 du = kMBF ? make_float2(round_bf16(den.x), round_bf16(den.y)) : den;
        float2 ui;
        if (has_m) {
          float2 mi;
          if (ALGO == ADVOPT_ALGO_PRODIGY) mi = Rm2(fma2(gi, splat2(c_m), Rm2(mul2(m[i], splat2(beta1)))));
          else mi = Rm2(lerp2(m[i], gi, w_m, w_m1, w_m_small));
          m_new[i] = mi;
          ui = nest ? Rm2(lerp2(mi, gi, w_n, w_n1, w_n_small)) : mi;
        } else {
          m_new[i] = splat2(0.0f);
          ui = (ALGO == ADVOPT_ALGO_PRODIGY) ? Rm2(mul2(gi, splat2(L.d))) : gi;
        }
        ui = make_float2(Rm(__fdiv_rn(ui.x, du.x)), Rm(__fdiv_rn(ui.y, du.y)));
        ui = Rm2(mul2(ui, splat2(step_size)));
        const bool ok0 = 2 * i < nv, ok1 = 2 * i + 1 < nv;
        if (!ok0) { m_new[i].x = 0.0f; v[i].x = 0.0f; }
        if (!ok1) { m_new[i].y = 0.0f; v[i].y = 0.0f; }
        amax_m = fmaxf(amax_m, fmaxf(fabsf(m_new[i].x), fabsf(m_new[i].y)));
        vmax = fmaxf(vmax, fmaxf(v[i].x, v[i].y));

        if (pstats) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int e = 2 * i + h;
            if (e < nv && e >= slice_off && ((e - slice_off) % (int)slice_p) == 0) {
              const float gv = h ? gi.y : gi.x, pv = h ? p[i].y : p[i].x;
              const int64_t si = (k0 + e) / slice_p;
              float p0v = 0.0f;
              if (!(T.flags & ADVOPT_T_P0_SCALAR))
                p0v = PBF ? bf16_to_f(static_cast<const uint16_t*>(T.aux1)[si]) : static_cast<const float*>(T.aux1)[si];
              st0 += (double)gv * (double)__fsub_rn(p0v, pv);
              const float s_old = PBF ? bf16_to_f(static_cast<const uint16_t*>(T.aux0)[si])
                                      : static_cast<const float*>(T.aux0)[si];
              float s1 = __fmul_rn(s_old, L.beta3);
              if (PBF) s1 = round_bf16(s1);
              float s2 = __fmaf_rn(gv, L.s_alpha, s1);
              if (PBF) {
                const uint32_t b = f_to_bf16_rne(s2);
                static_cast<uint16_t*>(T.aux0)[si] = (uint16_t)b;
                s2 = bf16_to_f(b);
              } else {
                static_cast<float*>(T.aux0)[si] = s2;
              }
              st1 += (double)fabsf(s2);
            }
          }
        }
        // parameter update (param_update.py:77-156)
        float2 pc2 = p[i];
        if (wd != 0.0f) {
          if (cautious) {
            float2 prod = mul2(ui, pc2);
            if (PBF && !sr) prod = make_float2(round_bf16(prod.x), round_bf16(prod.y));
            const float2 mask = make_float2(prod.x >= 0.0f ? 1.0f : 0.0f, prod.y >= 0.0f ? 1.0f : 0.0f);
            pc2 = fma2(mul2(splat2(-wd), pc2), mask, pc2);
          } else {
            pc2 = fma2(pc2, splat2(-wd), pc2);
          }
          if (PBF && !sr) pc2 = make_float2(round_bf16(pc2.x), round_bf16(pc2.y));
        }
        const float2 pn = add2(pc2, make_float2(-ui.x, -ui.y));
        if (PBF) {
          if (sr) {
            pout[2 * i] = __float_as_uint(pn.x) + (npw[i] & 0xFFFFu);
            pout[2 * i + 1] = __float_as_uint(pn.y) + (npw[i] >> 16);
          } else {
            pout[2 * i] = f_to_bf16_rne(pn.x);
            pout[2 * i + 1] = f_to_bf16_rne(pn.y);
          }
        } else {
          pout[2 * i] = __float_as_uint(pn.x);
          pout[2 * i + 1] = __float_as_uint(pn.y);
        }
      }
      // param store
      if (PBF) {
        uint32_t o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          o[i] = sr ? __byte_perm(pout[2 * i], pout[2 * i + 1], 0x7632) : (pout[2 * i] | (pout[2 * i + 1] << 16));
        uint16_t* dst = static_cast<uint16_t*>(T.param) + k0;
        if (v8) {
          *reinterpret_cast<uint4*>(dst) = make_uint4(o[0], o[1], o[2], o[3]);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (e < nv) dst[e] = (uint16_t)(o[e >> 1] >> (16 * (e & 1)));
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

      // factored: column partials (vector smem) and this thread's row part
      float rsum0 = 0.0f, rsum1 = 0.0f;
      if (fact) {
        if (nv > 0) {
          float4* ca = reinterpret_cast<float4*>(colacc + col);
          float4 a = ca[0], b = ca[1];
          const float2 a01 = add2(make_float2(a.x, a.y), v[0]), a23 = add2(make_float2(a.z, a.w), v[1]);
          const float2 b01 = add2(make_float2(b.x, b.y), v[2]), b23 = add2(make_float2(b.z, b.w), v[3]);
          ca[0] = make_float4(a01.x, a01.y, a23.x, a23.y);
          ca[1] = make_float4(b01.x, b01.y, b23.x, b23.y);
        }
        // same association as the general kernel: ((v0+v1)+(v2+v3)) + ((v4+v5)+(v6+v7))
        const float2 pairs = add2(make_float2(v[0].x, v[2].x), make_float2(v[0].y, v[2].y));   // v0+v1, v4+v5
        const float2 pairs2 = add2(make_float2(v[1].x, v[3].x), make_float2(v[1].y, v[3].y));  // v2+v3, v6+v7
        const float2 halves = add2(pairs, pairs2);
        const float sum = __fadd_rn(halves.x, halves.y);
        if (second) rsum1 = sum; else rsum0 = sum;
      }
      // noise of the quantised states, drawn before the barrier
      U4 nzm{0u, 0u, 0u, 0u}, nzv{0u, 0u, 0u, 0u};
      if (kStore == 2 || TR::kSRStates) {
        if (has_m) nzm = noise_words<NOISE_IN>(L, T, T.nz_m, kNoiseM, k0, nv);
        if (!fact) nzv = noise_words<NOISE_IN>(L, T, T.nz_v, kNoiseV, k0, nv);
      }
      {
        const float a = (has_m && kStore == 2) ? warp_max(amax_m) : 0.0f;
        const float b = (!fact && kStore == 2) ? warp_max(vmax) : 0.0f;
        const float c = fact ? warp_sum(rsum0) : 0.0f;
        const float d = fact ? warp_sum(rsum1) : 0.0f;
        if (lane == 0) {
          red[parity][warp][0] = a;
          red[parity][warp][1] = b;
          red[parity][warp][2] = c;
          red[parity][warp][3] = d;
        }
      }
      __syncthreads();
      if (abort_flag) return;   // every thread reads the same flag after the barrier
      // every thread is done with this stage: refill it with the chunk S ahead
      if (tid == 0 && cur_valid) {
        issue_chunk<PREC, PBF>(cur, stages + (size_t)slot * LY::BYTES, &bars[slot], &direct[slot], has_m);
        cur_valid = cursor_next<PREC, PBF>(L, cur, pend);
      }
      if (fact && tid == 0) {
        float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) {
          s0 = __fadd_rn(s0, red[parity][w][2]);
          s1 = __fadd_rn(s1, red[parity][w][3]);
        }
        row_carry += (double)s0;
        if (clen >= d2 - c0) {
          T.row[r0] = (float)row_carry;
          row_carry = (double)s1;
        }
      }
      if (has_m) {
        if (kStore == 2) {
          float bmax = 0.0f;
#pragma unroll
          for (int w = 0; w < kWarps; ++w) bmax = fmaxf(bmax, red[parity][w][0]);
          const uint2 q = quantize8x2<true>(m_new, bmax, nzm);
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
          float bmax = 0.0f;
#pragma unroll
          for (int w = 0; w < kWarps; ++w) bmax = fmaxf(bmax, red[parity][w][1]);
          const uint2 q = quantize8x2<false>(v, bmax, nzv);
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
        if (c0 >= d2) {
          c0 -= d2;
          r0 += 1;
        }
      }
      parity ^= 1;
    }

    if (fact) {
      __syncthreads();
      float* dstp = T.colpart + (int64_t)pc.slot * d2;
      for (int j2 = tid * 4; j2 < (int)d2; j2 += kThreads * 4)
        *reinterpret_cast<float4*>(dstp + j2) = *reinterpret_cast<const float4*>(colacc + j2);
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
