// Shared device primitives for the optimizer-step kernels (sm_100a).
//
// The whole library is compiled with -fmad=false: no multiply-add is fused
// unless written as __fmaf_rn, so every rounding below happens exactly where
// PyTorch's CPU kernels round in the reference (the fused forms are the ATen
// vectorised lerp, addcmul and add-with-alpha).  Division and square root are
// the IEEE-rounded __fdiv_rn / __fsqrt_rn.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace advopt {

constexpr int kThreads = 256;       // threads per CTA of the elementwise kernels
constexpr int kVec = 8;             // elements per thread per chunk
constexpr int kChunk = kThreads * kVec;  // 2048 = the int8_sr block (state_util.py:10)
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ uint32_t f2u(float x) { return __float_as_uint(x); }
__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }

__device__ __forceinline__ float bf16_to_f(uint32_t b16) { return u2f(b16 << 16); }

// float -> bf16 bits, round to nearest even; NaN -> 0x7FC0 (c10::BFloat16).
__device__ __forceinline__ uint32_t f_to_bf16_rne(float x) {
  const uint32_t u = f2u(x);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7FC0u;
  return (u + 0x7FFFu + ((u >> 16) & 1u)) >> 16;
}
__device__ __forceinline__ float round_bf16(float x) { return bf16_to_f(f_to_bf16_rne(x)); }

// Stochastic rounding to bf16 (param_update.py:206-219): add the 16-bit random
// integer to the bit pattern (wrapping int32 add), keep the high half.  A NaN
// result is canonicalised to 0x7FC0 as ATen's float->bf16 cast does.
__device__ __forceinline__ uint32_t f_to_bf16_sr(float x, uint32_t r16) {
  const uint32_t v = (f2u(x) + r16) >> 16;
  if ((v & 0x7F80u) == 0x7F80u && (v & 0x7Fu)) return 0x7FC0u;
  return v;
}

// torch.lerp with a scalar weight (ATen CPU lerp_vec): fmadd(coeff, end-self, base).
__device__ __forceinline__ float lerp_t(float self, float end, float w) {
  const float d = __fsub_rn(end, self);
  return (fabsf(w) < 0.5f) ? __fmaf_rn(w, d, self) : __fmaf_rn(__fsub_rn(w, 1.0f), d, end);
}

// ---------------------------------------------------------------------------
// Philox4x32-10 (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as easy
// as 1, 2, 3", SC'11).  Counter-based: every element's noise is a pure
// function of (seed, tensor, step, stream, element index).
// ---------------------------------------------------------------------------
struct U4 {
  uint32_t x, y, z, w;
};

__device__ __forceinline__ U4 philox4x32_10(U4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int i = 0; i < 10; ++i) {
    // one 32x32->64 multiply per lane word (hi and lo from a single wide
    // product; written as mul.wide so it stays one instruction)
    uint64_t p0, p1;
    asm("mul.wide.u32 %0, %1, %2;" : "=l"(p0) : "r"(c.x), "r"(0xD2511F53u));
    asm("mul.wide.u32 %0, %1, %2;" : "=l"(p1) : "r"(c.z), "r"(0xCD9E8D57u));
    c = U4{(uint32_t)(p1 >> 32) ^ c.y ^ k0, (uint32_t)p1, (uint32_t)(p0 >> 32) ^ c.w ^ k1, (uint32_t)p0};
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return c;
}

// The ten round keys of a Philox4x32-10 key, computed once on the host and
// passed as a kernel parameter: the rounds then read them from the constant
// bank instead of re-deriving the Weyl sequence per call.
struct PhiloxKeys {
  uint32_t k[20];   // round i uses k[2i], k[2i+1]
};

inline PhiloxKeys philox_keys(uint64_t seed) {
  PhiloxKeys K;
  uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
  for (int i = 0; i < 10; ++i) {
    K.k[2 * i] = k0;
    K.k[2 * i + 1] = k1;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return K;
}

// Same rounds as philox4x32_10 with the keys from the table.
__device__ __forceinline__ U4 philox4x32_10_k(U4 c, const PhiloxKeys& K) {
#pragma unroll
  for (int i = 0; i < 10; ++i) {
    uint64_t p0, p1;
    asm("mul.wide.u32 %0, %1, %2;" : "=l"(p0) : "r"(c.x), "r"(0xD2511F53u));
    asm("mul.wide.u32 %0, %1, %2;" : "=l"(p1) : "r"(c.z), "r"(0xCD9E8D57u));
    c = U4{(uint32_t)(p1 >> 32) ^ c.y ^ K.k[2 * i], (uint32_t)p1, (uint32_t)(p0 >> 32) ^ c.w ^ K.k[2 * i + 1],
           (uint32_t)p0};
  }
  return c;
}

// Noise streams (counter word y carries the stream id in its top byte).
enum NoiseStream : uint32_t { kNoiseV = 0, kNoiseM = 1, kNoiseP = 2, kNoiseAux = 3 };

// Eight 16-bit uniform integers in [0, 65536) for elements k0 .. k0+7 of a
// tensor (k0 a multiple of 8), the same values the injected-noise path reads
// from an int32 array.
__device__ __forceinline__ void philox_u16x8(uint64_t seed, uint32_t tensor_id, uint32_t step, uint32_t stream,
                                             int64_t k0, uint32_t (&r)[8]) {
  const uint64_t grp = (uint64_t)k0 >> 3;
  U4 c{(uint32_t)grp, (uint32_t)(grp >> 32) | (stream << 24), tensor_id, step};
  const U4 o = philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  r[0] = o.x & 0xFFFFu; r[1] = o.x >> 16;
  r[2] = o.y & 0xFFFFu; r[3] = o.y >> 16;
  r[4] = o.z & 0xFFFFu; r[5] = o.z >> 16;
  r[6] = o.w & 0xFFFFu; r[7] = o.w >> 16;
}

// ---------------------------------------------------------------------------
// Vector loads / stores of 8 consecutive elements (16-byte aligned when `vec`).
// ---------------------------------------------------------------------------
template <bool BF16>
__device__ __forceinline__ void load8(const void* base, int64_t k0, int nv, bool vec, float (&x)[8]) {
  if (BF16) {
    const uint16_t* p = static_cast<const uint16_t*>(base) + k0;
    if (vec) {
      const uint4 q = __ldg(reinterpret_cast<const uint4*>(p));
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        x[2 * i] = u2f(w[i] << 16);
        x[2 * i + 1] = u2f(w[i] & 0xFFFF0000u);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = e < nv ? bf16_to_f(p[e]) : 0.0f;
    }
  } else {
    const float* p = static_cast<const float*>(base) + k0;
    if (vec) {
      const float4 a = __ldg(reinterpret_cast<const float4*>(p));
      const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
      x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
      x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = e < nv ? p[e] : 0.0f;
    }
  }
}

// Store: bf16 values given as 16-bit patterns in u[], or floats in x[].
__device__ __forceinline__ void store8_bf16(void* base, int64_t k0, int nv, bool vec, const uint32_t (&u)[8]) {
  uint16_t* p = static_cast<uint16_t*>(base) + k0;
  if (vec) {
    uint4 q;
    q.x = u[0] | (u[1] << 16);
    q.y = u[2] | (u[3] << 16);
    q.z = u[4] | (u[5] << 16);
    q.w = u[6] | (u[7] << 16);
    *reinterpret_cast<uint4*>(p) = q;
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (e < nv) p[e] = (uint16_t)u[e];
  }
}

__device__ __forceinline__ void store8_f32(void* base, int64_t k0, int nv, bool vec, const float (&x)[8]) {
  float* p = static_cast<float*>(base) + k0;
  if (vec) {
    reinterpret_cast<float4*>(p)[0] = make_float4(x[0], x[1], x[2], x[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(x[4], x[5], x[6], x[7]);
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (e < nv) p[e] = x[e];
  }
}

// 8 int8 / uint8 codes.
template <bool SIGNED>
__device__ __forceinline__ void load8_q(const void* base, int64_t k0, int nv, bool vec, float (&x)[8]) {
  const uint8_t* p = static_cast<const uint8_t*>(base) + k0;
  if (vec) {
    const uint2 q = __ldg(reinterpret_cast<const uint2*>(p));
    const uint32_t w[2] = {q.x, q.y};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t b = (w[i >> 2] >> (8 * (i & 3))) & 0xFFu;
      x[i] = SIGNED ? (float)(int)(int8_t)b : (float)b;
    }
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t b = e < nv ? p[e] : 0u;
      x[e] = SIGNED ? (float)(int)(int8_t)b : (float)b;
    }
  }
}

__device__ __forceinline__ void store8_q(void* base, int64_t k0, int nv, bool vec, const uint32_t (&c)[8]) {
  uint8_t* p = static_cast<uint8_t*>(base) + k0;
  if (vec) {
    uint2 q;
    q.x = (c[0] & 0xFF) | ((c[1] & 0xFF) << 8) | ((c[2] & 0xFF) << 16) | ((c[3] & 0xFF) << 24);
    q.y = (c[4] & 0xFF) | ((c[5] & 0xFF) << 8) | ((c[6] & 0xFF) << 16) | ((c[7] & 0xFF) << 24);
    *reinterpret_cast<uint2*>(p) = q;
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (e < nv) p[e] = (uint8_t)c[e];
  }
}

// Block-wise stochastic quantisation of one value (param_update.py:296-304,
// 352-360): q = clamp(floor(x / safe_scale + r/65536), lo, hi).
__device__ __forceinline__ uint32_t quant_code(float x, float safe_scale, uint32_t r16, bool non_neg) {
  const float noise = __fmul_rn((float)r16, 1.0f / 65536.0f);
  float y = floorf(__fadd_rn(__fdiv_rn(x, safe_scale), noise));
  if (y != y) y = 0.0f;
  if (non_neg) {
    y = fminf(fmaxf(y, 0.0f), 255.0f);
  } else {
    y = fminf(fmaxf(y, -127.0f), 127.0f);
  }
  return (uint32_t)(int)y;
}

// float8_e4m3fn -> float (exact): 1 sign, 4 exponent (bias 7), 3 mantissa
// bits; 0x7F / 0xFF are NaN, no infinities.
__device__ __forceinline__ float fp8e4m3_to_f(uint32_t b) {
  const uint32_t s = (b & 0x80u) << 24;
  const uint32_t e = (b >> 3) & 0xFu, m = b & 0x7u;
  if (e == 0xFu && m == 0x7u) return u2f(s | 0x7FC00000u);
  if (e == 0) {  // subnormal: m * 2^-9
    return u2f(s | f2u((float)m * 0.001953125f));
  }
  return u2f(s | ((e + 120u) << 23) | (m << 20));
}

// Warp reductions.
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace advopt

namespace advopt {

// RN(x / d) from r = RN(1/d): q0 = x*r, then two residual corrections
// q <- q + r*(x - q*d) (Markstein, "Computation of elementary functions on
// the IBM RISC System/6000 processor", IBM J. Res. Dev. 34, 1990).  After
// the first correction q is faithful; the second then yields the correctly
// rounded quotient, provided the residuals stay normal.  Callers use it only
// for |x| >= 2^-100 with a normal divisor and fall back to __fdiv_rn below.
__device__ __forceinline__ float div_rcp(float x, float d, float r) {
  float q = __fmul_rn(x, r);
  float e = __fmaf_rn(-q, d, x);
  q = __fmaf_rn(e, r, q);
  e = __fmaf_rn(-q, d, x);
  return __fmaf_rn(e, r, q);
}
__device__ __forceinline__ float div_const(float x, float d, float r) {
  return fabsf(x) >= 0x1p-100f ? div_rcp(x, d, r) : __fdiv_rn(x, d);
}

// r16 * 2^-16 exactly, without the conversion pipe: 1 + r*2^-16 built from
// bits, minus 1 (exact by Sterbenz).
__device__ __forceinline__ float noise_unit(uint32_t r16) {
  return __fsub_rn(__uint_as_float(0x3F800000u | (r16 << 7)), 1.0f);
}

// floor(y) as an int for |y| < 2^22: y + 1.5*2^23 rounded toward -inf lands on
// the integer grid of that binade, so its low bits are 2^22 + floor(y).
__device__ __forceinline__ int floor_int(float y) {
  return (int)(__float_as_uint(__fadd_rd(y, 12582912.0f)) - 0x4B400000u);
}

// Four int8 (SIGNED) or uint8 codes of w as exact floats, via 2^23 + byte.
template <bool SIGNED>
__device__ __forceinline__ void codes4_to_f(uint32_t w, float* out) {
  const uint32_t x = SIGNED ? (w ^ 0x80808080u) : w;
  const float bias = SIGNED ? 8388736.0f : 8388608.0f;  // 2^23 + 128 | 2^23
  out[0] = __fsub_rn(__uint_as_float(__byte_perm(x, 0x4B000000u, 0x7440)), bias);
  out[1] = __fsub_rn(__uint_as_float(__byte_perm(x, 0x4B000000u, 0x7441)), bias);
  out[2] = __fsub_rn(__uint_as_float(__byte_perm(x, 0x4B000000u, 0x7442)), bias);
  out[3] = __fsub_rn(__uint_as_float(__byte_perm(x, 0x4B000000u, 0x7443)), bias);
}

// Pack the low bytes of four ints.
__device__ __forceinline__ uint32_t pack4_bytes(int c0, int c1, int c2, int c3) {
  const uint32_t lo = __byte_perm((uint32_t)c0, (uint32_t)c1, 0x0040);
  const uint32_t hi = __byte_perm((uint32_t)c2, (uint32_t)c3, 0x0040);
  return __byte_perm(lo, hi, 0x5410);
}

}  // namespace advopt

namespace advopt {

// ---------------------------------------------------------------------------
// Packed fp32x2 arithmetic (sm_100): one instruction, two IEEE-rounded lanes.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return __fadd2_rn(a, b); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return __fmul2_rn(a, b); }
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) { return __ffma2_rn(a, b, c); }
__device__ __forceinline__ float2 splat2(float a) { return make_float2(a, a); }
// end - self, exactly as one fused op: fma(self, -1, end)
__device__ __forceinline__ float2 sub2(float2 end, float2 self) { return __ffma2_rn(self, splat2(-1.0f), end); }

// torch.lerp, two lanes (weight uniform): fmadd(coeff, end-self, base).
__device__ __forceinline__ float2 lerp2(float2 self, float2 end, float w, float wm1, bool small) {
  const float2 d = sub2(end, self);
  return small ? fma2(splat2(w), d, self) : fma2(splat2(wm1), d, end);
}

// Two-lane div_rcp (same Markstein sequence as div_rcp).
__device__ __forceinline__ float2 div_rcp2(float2 x, float d, float r) {
  const float2 D = splat2(-d), Rr = splat2(r);
  float2 q = mul2(x, Rr);
  float2 e = fma2(q, D, x);
  q = fma2(e, Rr, q);
  e = fma2(q, D, x);
  return fma2(e, Rr, q);
}

// ---------------------------------------------------------------------------
// mbarrier + bulk asynchronous copy (global -> shared, no multicast).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// Arrive + expect_tx; relaxed: announcing the bytes of the copies issued
// next needs no ordering of this thread's earlier memory operations.
__device__ __forceinline__ void mbar_arrive_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.relaxed.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: gives up after `limit` polls (each try_wait itself suspends
// for a hardware-defined interval) and reports it instead of hanging.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t limit = (1u << 24)) {
  for (uint32_t i = 0; i < limit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}

}  // namespace advopt
