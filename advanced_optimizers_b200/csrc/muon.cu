// Elementwise kernels around the Newton–Schulz GEMMs of Muon_adv / AdaMuon_adv
// (Muon_adv.py:443-555, AdaMuon_adv.py:492-659, Muon_util.py:7-121,362-372).
//
//   stage 0  prep_kernel    momentum lerp, Nesterov, AdaMuon's sign projection,
//                           momentum_buffer store (f32 / bf16 RNE / bf16 SR /
//                           int8 blocks), X0 = bf16(update), per-chunk sum(X0^2)
//            norm_kernel    ||X0||_F as the reference's bf16 norm, clamped at eps
//            load_kernel    workspace = bf16(X0 / norm), transposed when
//                           rows > cols, zero padding to [m_pad][n_pad]
//   stage 1  store_kernel   U = NS result in the param's layout, per-tile sum(U^2)
//            scale_kernel   rms_adjustment's scale in the update's dtype
//   stage 2  apply_kernel   p = apply_parameter_update(p, U * scale)
//   stage 3  store_kernel only (AdaMuon)
//   stage 4  adamuon_stats  per-chunk sum(u'^2), u' = u / (sqrt(v') + eps), and
//            scale_kernel   (nothing else written: v' is recomputed in stage 5)
//   stage 5  adamuon_apply  second_momentum_buffer store + param update
//   stage 6  prep_kernel<RAW> X0 = bf16(grad) for a bare Newton–Schulz call,
//            then norm_kernel and load_kernel as in stage 0
//   stage 7  normuon_rows   NorMuon: per-row lerp of mean(u^2) into normuon_v,
//                           sqrt(v) + eps per row (Muon_util.py:349-360)
//   stage 8  normuon_stats  per-chunk sum(u'^2), u' = u / den[row], and scale_kernel
//   stage 9  normuon_apply  param update with u' * scale
//   stage 10 vfact_*        AdaMuon factored_2nd: v = outer(row, col) * beta2 +
//                           (1-beta2) u^2 into a scratch, sum(u'^2) and
//                           scale_kernel, then the new row / column factors
//   stage 11 vfact_apply    param update with u' * scale
//   stage 13 u_stats        sum(U^2) of U already in `u` (low-rank chain) and scale_kernel
//   MARS-M (flag) corrects the grad inside stage 0; with ADVOPT_MU_LOWRANK
//   stage 0 ends after X0 (the chain runs on the low-rank projection).
//
// One launch sequence handles one matrix.  Chunks of 2048 elements (the int8
// block) map to CTAs of 256 threads x 8 consecutive elements, so one Philox
// call gives a thread all eight of its noise values.
#include "advopt.h"
#include "capi_internal.h"
#include "common.cuh"

namespace advopt {
namespace muon {

using Args = advopt_muon_args;

__device__ __forceinline__ void noise8(const Args& a, const int32_t* arr, uint32_t stream, int64_t k0, int64_t n,
                                       uint32_t (&r)[8]) {
  if (a.flags & ADVOPT_MU_NOISE_IN) {
#pragma unroll
    for (int e = 0; e < 8; ++e) r[e] = (k0 + e < n) ? ((uint32_t)arr[k0 + e] & 0xFFFFu) : 0u;
  } else {
    philox_u16x8(a.seed, a.tensor_id, a.step, stream, k0, r);
  }
}

__device__ __forceinline__ float load_state(const void* base, int64_t k, int st, const float* scale, bool non_neg) {
  switch (st) {
    case ADVOPT_ST_F32: return static_cast<const float*>(base)[k];
    case ADVOPT_ST_BF16:
    case ADVOPT_ST_BF16_SR: return bf16_to_f(static_cast<const uint16_t*>(base)[k]);
    default: {
      const float q = non_neg ? (float)static_cast<const uint8_t*>(base)[k] : (float)static_cast<const int8_t*>(base)[k];
      return __fmul_rn(q, scale[k >> 11]);
    }
  }
}

// Store with the state's rounding.  For ADVOPT_ST_Q8 `safe` is the block's
// max(scale, 1e-12) (state_util.py:109-163).
__device__ __forceinline__ void store_state(void* base, int64_t k, int st, float x, float safe, bool non_neg,
                                            uint32_t r16) {
  switch (st) {
    case ADVOPT_ST_F32: static_cast<float*>(base)[k] = x; break;
    case ADVOPT_ST_BF16: static_cast<uint16_t*>(base)[k] = (uint16_t)f_to_bf16_rne(x); break;
    case ADVOPT_ST_BF16_SR: static_cast<uint16_t*>(base)[k] = (uint16_t)f_to_bf16_sr(x, r16); break;
    default: static_cast<uint8_t*>(base)[k] = (uint8_t)quant_code(x, safe, r16, non_neg); break;
  }
}

__device__ __forceinline__ float block_max256(float v, float* red) {
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float m = red[0];
#pragma unroll
  for (int i = 1; i < kWarps; ++i) m = fmaxf(m, red[i]);
  __syncthreads();
  return m;
}

// Sum over the CTA; the result is valid in thread 0.
__device__ __forceinline__ double block_sum_d(double v, double* red, int nthreads) {
  v = warp_sum_d(v);
  const int t = threadIdx.y * blockDim.x + threadIdx.x;
  if ((t & 31) == 0) red[t >> 5] = v;
  __syncthreads();
  double s = 0.0;
  if (t == 0)
    for (int i = 0; i < nthreads / 32; ++i) s += red[i];
  __syncthreads();
  return s;
}

__device__ __forceinline__ float load_grad(const Args& a, int64_t k) {
  return a.param_bf16 ? bf16_to_f(static_cast<const uint16_t*>(a.grad)[k]) : static_cast<const float*>(a.grad)[k];
}

// approx MARS-M (Muon_util.py:333-347): c = (g - last).mul_(f).add_(g), each
// op rounding to the grad's dtype (bf16 under 'auto' with bf16 params, else
// f32); last_grad (the param's dtype) takes g.
template <bool MBF>
__device__ __forceinline__ float mars(const Args& a, int64_t k, float g) {
  const bool pbf = a.param_bf16 != 0;
  const float lg = pbf ? bf16_to_f(static_cast<const uint16_t*>(a.last_grad)[k])
                       : static_cast<const float*>(a.last_grad)[k];
  float t = __fsub_rn(g, lg);
  if (MBF) t = round_bf16(t);
  t = __fmul_rn(t, a.mars_factor);
  if (MBF) t = round_bf16(t);
  t = __fadd_rn(t, g);
  if (MBF) t = round_bf16(t);
  if (pbf)
    static_cast<uint16_t*>(a.last_grad)[k] = (uint16_t)f_to_bf16_rne(g);
  else
    static_cast<float*>(a.last_grad)[k] = g;
  return t;
}

// ---- stage 0: momentum, Nesterov, sign, momentum store, X0, sum(X0^2) ----
// RAW (stage 6): X0 = bf16(grad) only, for a bare Newton–Schulz call.
template <bool MBF, bool RAW>
__global__ void __launch_bounds__(256) prep_kernel(const Args a) {
  __shared__ float redf[kWarps];
  __shared__ double redd[kWarps];
  const int64_t nchunks = (a.numel + kChunk - 1) / kChunk;
  const int st = a.m_storage;
  for (int64_t c = blockIdx.x; c < nchunks; c += gridDim.x) {
    const int64_t k0 = c * kChunk + threadIdx.x * 8;
    float mn[8];
    float amax = 0.0f;
    double ss = 0.0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int64_t k = k0 + e;
      mn[e] = 0.0f;
      if (k < a.numel) {
        float g = load_grad(a, k);
        if (!RAW && (a.flags & ADVOPT_MU_MARS)) g = mars<MBF>(a, k, g);
        float u = g;
        if (!RAW) {
          const float m0 = load_state(a.m, k, st, a.m_scale, false);
          float m1 = lerp_t(m0, g, a.w_m);
          if (MBF) m1 = round_bf16(m1);
          mn[e] = m1;
          amax = fmaxf(amax, fabsf(m1));
          u = m1;
          if (a.flags & ADVOPT_MU_NESTEROV) {
            u = lerp_t(g, m1, a.w_nest);
            if (MBF) u = round_bf16(u);
          }
          if (a.flags & ADVOPT_MU_SIGN) u = u > 0.0f ? 1.0f : (u < 0.0f ? -1.0f : u);
        }
        const uint32_t xb = f_to_bf16_rne(u);
        a.x0[k] = (uint16_t)xb;
        const float xf = bf16_to_f(xb);
        ss += (double)xf * (double)xf;
      }
    }
    if (!RAW) {
      float safe = 0.0f;
      if (st == ADVOPT_ST_Q8) {
        const float bmax = block_max256(amax, redf);
        const float scale = __fdiv_rn(bmax, 127.0f);
        safe = scale < 1e-12f ? 1e-12f : scale;
        if (threadIdx.x == 0) a.m_scale[c] = scale;
      }
      uint32_t r[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (st >= ADVOPT_ST_BF16_SR) noise8(a, a.noise_m, kNoiseM, k0, a.numel, r);
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (k0 + e < a.numel) store_state(a.m, k0 + e, st, mn[e], safe, false, r[e]);
    }
    const double s = block_sum_d(ss, redd, 256);
    if (threadIdx.x == 0) a.partial[c] = s;
  }
}

// ---- vectorised stage 0 for the common layout: bf16 grads, f32 / bf16 /
// bf16-SR momentum, numel a multiple of 8, 16-byte aligned buffers.  Same
// element arithmetic, noise and summation order as prep_kernel (each thread
// sums its 8 squares in float64 in element order, then the CTA sum).
__device__ __forceinline__ void unpack_bf16x8(const uint4 w, float (&x)[8]) {
  const uint32_t q[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[2 * i] = bf16_to_f(q[i] & 0xFFFFu);
    x[2 * i + 1] = bf16_to_f(q[i] >> 16);
  }
}
__device__ __forceinline__ uint4 pack_bf16x8(const uint32_t (&b)[8]) {
  return make_uint4(b[0] | (b[1] << 16), b[2] | (b[3] << 16), b[4] | (b[5] << 16), b[6] | (b[7] << 16));
}

template <bool MBF, bool RAW, int ST>
__global__ void __launch_bounds__(256) prep_vec_kernel(const Args a) {
  __shared__ double redd[kWarps];
  const int64_t nchunks = (a.numel + kChunk - 1) / kChunk;
  for (int64_t c = blockIdx.x; c < nchunks; c += gridDim.x) {
    const int64_t k0 = c * kChunk + threadIdx.x * 8;
    double ss = 0.0;
    if (k0 < a.numel) {
      float g[8], m0[8];
      unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.grad) + k0)), g);
      if (!RAW) {
        if (ST == ADVOPT_ST_F32) {
          const float4 lo = *reinterpret_cast<const float4*>(static_cast<const float*>(a.m) + k0);
          const float4 hi = *(reinterpret_cast<const float4*>(static_cast<const float*>(a.m) + k0) + 1);
          m0[0] = lo.x; m0[1] = lo.y; m0[2] = lo.z; m0[3] = lo.w;
          m0[4] = hi.x; m0[5] = hi.y; m0[6] = hi.z; m0[7] = hi.w;
        } else {
          unpack_bf16x8(*reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.m) + k0), m0);
        }
      }
      uint32_t r[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (!RAW && ST == ADVOPT_ST_BF16_SR) noise8(a, a.noise_m, kNoiseM, k0, a.numel, r);
      uint32_t xb[8], mb[8];
      float mf[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float u = g[e];
        if (!RAW) {
          float m1 = lerp_t(m0[e], g[e], a.w_m);
          if (MBF) m1 = round_bf16(m1);
          mf[e] = m1;
          u = m1;
          if (a.flags & ADVOPT_MU_NESTEROV) {
            u = lerp_t(g[e], m1, a.w_nest);
            if (MBF) u = round_bf16(u);
          }
          if (a.flags & ADVOPT_MU_SIGN) u = u > 0.0f ? 1.0f : (u < 0.0f ? -1.0f : u);
          mb[e] = ST == ADVOPT_ST_BF16_SR ? f_to_bf16_sr(m1, r[e]) : f_to_bf16_rne(m1);
        }
        xb[e] = f_to_bf16_rne(u);
        const float xf = bf16_to_f(xb[e]);
        ss += (double)xf * (double)xf;
      }
      *reinterpret_cast<uint4*>(a.x0 + k0) = pack_bf16x8(xb);
      if (!RAW) {
        if (ST == ADVOPT_ST_F32) {
          float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.m) + k0);
          dst[0] = make_float4(mf[0], mf[1], mf[2], mf[3]);
          dst[1] = make_float4(mf[4], mf[5], mf[6], mf[7]);
        } else {
          *reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.m) + k0) = pack_bf16x8(mb);
        }
      }
    }
    const double s = block_sum_d(ss, redd, 256);
    if (threadIdx.x == 0) a.partial[c] = s;
  }
}

// ||X0||_F -> bf16, clamped at bf16(ns_eps): scalars[0].  One CTA of 1024.
__global__ void __launch_bounds__(1024) norm_kernel(const Args a, int64_t nparts) {
  __shared__ double red[32];
  double s = 0.0;
  for (int64_t i = threadIdx.x; i < nparts; i += blockDim.x) s += a.partial[i];
  s = block_sum_d(s, red, 1024);
  if (threadIdx.x == 0) {
    float n = round_bf16((float)sqrt(s));
    const float e = round_bf16(a.ns_eps);
    if (n < e) n = e;
    a.scalars[0] = n;
  }
}

// Workspace tile (32 x 32, 32 x 8 threads) = bf16(X0 / norm), transposed
// when rows > cols, zeros in the padding.
__global__ void __launch_bounds__(256) load_kernel(const Args a) {
  __shared__ uint16_t tile[32][33];
  const float nrm = a.scalars[0];
  const float rn = __frcp_rn(nrm);
  const int64_t i0 = (int64_t)blockIdx.y * 32, j0 = (int64_t)blockIdx.x * 32;
  const int tx = threadIdx.x;
  if (!(a.flags & ADVOPT_MU_TRANSPOSED)) {
    for (int ii = threadIdx.y; ii < 32; ii += 8) {
      const int64_t i = i0 + ii, j = j0 + tx;
      uint16_t v = 0;
      if (i < a.rows && j < a.cols)
        v = (uint16_t)f_to_bf16_rne(div_const(bf16_to_f(a.x0[i * a.cols + j]), nrm, rn));
      a.ns[i * a.ld_ns + j] = v;
    }
    return;
  }
  // workspace (i, j) = X0[j][i]: read source rows j0.., cols i0.. coalesced
  for (int ii = threadIdx.y; ii < 32; ii += 8) {
    const int64_t r = j0 + ii, c = i0 + tx;
    uint16_t v = 0;
    if (r < a.rows && c < a.cols)
      v = (uint16_t)f_to_bf16_rne(div_const(bf16_to_f(a.x0[r * a.cols + c]), nrm, rn));
    tile[ii][tx] = v;
  }
  __syncthreads();
  for (int ii = threadIdx.y; ii < 32; ii += 8) a.ns[(i0 + ii) * a.ld_ns + j0 + tx] = tile[tx][ii];
}

// Vectorised load for cols a multiple of 8.  Not transposed: one thread per
// 8 consecutive workspace columns.  Transposed: 64 x 64 tiles through shared
// memory (row stride 66 elements keeps 32-bit stores aligned and limits bank
// conflicts of the column reads to two ways).
constexpr int kTile = 64, kTileLd = 66;

__global__ void __launch_bounds__(256) load_vec_kernel(const Args a) {
  const float nrm = a.scalars[0];
  const float rn = __frcp_rn(nrm);
  const int64_t gpr = a.n_pad / 8;
  const int64_t groups = a.m_pad * gpr;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < groups; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = t / gpr, j = (t - i * gpr) * 8;
    uint4 out = make_uint4(0u, 0u, 0u, 0u);
    if (i < a.rows && j < a.cols) {   // cols % 8 == 0: the group is all inside
      float x[8];
      unpack_bf16x8(*reinterpret_cast<const uint4*>(a.x0 + i * a.cols + j), x);
      uint32_t b[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) b[e] = f_to_bf16_rne(div_const(x[e], nrm, rn));
      out = pack_bf16x8(b);
    }
    *reinterpret_cast<uint4*>(a.ns + i * a.ld_ns + j) = out;
  }
}

__global__ void __launch_bounds__(256) load_vec_t_kernel(const Args a) {
  __shared__ __align__(16) uint16_t tile[kTile * kTileLd];
  const float nrm = a.scalars[0];
  const float rn = __frcp_rn(nrm);
  // workspace tile rows i0.. (= source columns), columns j0.. (= source rows)
  const int64_t i0 = (int64_t)blockIdx.y * kTile, j0 = (int64_t)blockIdx.x * kTile;
  for (int t = threadIdx.x; t < kTile * 8; t += blockDim.x) {
    const int jj = t >> 3, ig = (t & 7) * 8;
    const int64_t r = j0 + jj, c = i0 + ig;
    uint32_t b[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (r < a.rows && c < a.cols) {
      float x[8];
      unpack_bf16x8(*reinterpret_cast<const uint4*>(a.x0 + r * a.cols + c), x);
#pragma unroll
      for (int e = 0; e < 8; ++e) b[e] = f_to_bf16_rne(div_const(x[e], nrm, rn));
    }
    uint32_t* row = reinterpret_cast<uint32_t*>(tile + jj * kTileLd + ig);
#pragma unroll
    for (int e = 0; e < 4; ++e) row[e] = b[2 * e] | (b[2 * e + 1] << 16);
  }
  __syncthreads();
  for (int t = threadIdx.x; t < kTile * 8; t += blockDim.x) {
    const int ii = t >> 3, jg = (t & 7) * 8;
    uint32_t b[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) b[e] = tile[(jg + e) * kTileLd + ii];
    *reinterpret_cast<uint4*>(a.ns + (i0 + ii) * a.ld_ns + j0 + jg) = pack_bf16x8(b);
  }
}

// ---- stage 1/3: U in the param's layout, per-tile sum(U^2) ----
__global__ void __launch_bounds__(256) store_kernel(const Args a) {
  __shared__ uint16_t tile[32][33];
  __shared__ double red[8];
  const uint16_t* x = a.ns_result;
  const bool tr = a.flags & ADVOPT_MU_TRANSPOSED;
  const int64_t r0 = (int64_t)blockIdx.y * 32, c0 = (int64_t)blockIdx.x * 32;
  const int tx = threadIdx.x;
  if (tr) {
    // x holds [cols][rows]: read x rows c0.., cols r0.. coalesced
    for (int ii = threadIdx.y; ii < 32; ii += 8) {
      const int64_t c = c0 + ii, r = r0 + tx;
      tile[ii][tx] = (r < a.rows && c < a.cols) ? x[c * a.ld_ns + r] : (uint16_t)0;
    }
    __syncthreads();
  }
  double ss = 0.0;
  for (int ii = threadIdx.y; ii < 32; ii += 8) {
    const int64_t r = r0 + ii, c = c0 + tx;
    if (r < a.rows && c < a.cols) {
      const uint16_t v = tr ? tile[tx][ii] : x[r * a.ld_ns + c];
      a.u[r * a.cols + c] = v;
      const float f = bf16_to_f(v);
      ss += (double)f * (double)f;
    }
  }
  const double s = block_sum_d(ss, red, 256);
  if (tx == 0 && threadIdx.y == 0) a.partial[(int64_t)blockIdx.y * gridDim.x + blockIdx.x] = s;
}

// Vectorised stage 1/3 for cols a multiple of 8: U in the param's layout and
// per-CTA sum(U^2) (each thread in element order, float64).  Not transposed:
// a grid-stride loop over 8-element groups; transposed: 64 x 64 tiles.
__global__ void __launch_bounds__(256) store_vec_kernel(const Args a) {
  __shared__ double red[8];
  const int64_t gpr = a.cols / 8, groups = a.rows * gpr;
  double ss = 0.0;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < groups; t += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = t / gpr, c = (t - r * gpr) * 8;
    const uint4 w = *reinterpret_cast<const uint4*>(a.ns_result + r * a.ld_ns + c);
    *reinterpret_cast<uint4*>(a.u + r * a.cols + c) = w;
    float x[8];
    unpack_bf16x8(w, x);
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += (double)x[e] * (double)x[e];
  }
  const double s = block_sum_d(ss, red, 256);
  if (threadIdx.x == 0) a.partial[blockIdx.x] = s;
}

__global__ void __launch_bounds__(256) store_vec_t_kernel(const Args a) {
  __shared__ __align__(16) uint16_t tile[kTile * kTileLd];
  __shared__ double red[8];
  // param tile rows r0.. (= workspace columns), columns c0.. (= workspace rows)
  const int64_t r0 = (int64_t)blockIdx.y * kTile, c0 = (int64_t)blockIdx.x * kTile;
  for (int t = threadIdx.x; t < kTile * 8; t += blockDim.x) {
    const int cc = t >> 3, rg = (t & 7) * 8;
    // the workspace is [m_pad][n_pad] with zero padding: always readable
    const uint4 w = *reinterpret_cast<const uint4*>(a.ns_result + (c0 + cc) * a.ld_ns + r0 + rg);
    uint32_t* row = reinterpret_cast<uint32_t*>(tile + cc * kTileLd + rg);
    row[0] = w.x; row[1] = w.y; row[2] = w.z; row[3] = w.w;
  }
  __syncthreads();
  double ss = 0.0;
  for (int t = threadIdx.x; t < kTile * 8; t += blockDim.x) {
    const int rr = t >> 3, cg = (t & 7) * 8;
    const int64_t r = r0 + rr, c = c0 + cg;
    if (r < a.rows && c < a.cols) {
      uint32_t b[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) b[e] = tile[(cg + e) * kTileLd + rr];
      *reinterpret_cast<uint4*>(a.u + r * a.cols + c) = pack_bf16x8(b);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float f = bf16_to_f(b[e]);
        ss += (double)f * (double)f;
      }
    }
  }
  const double s = block_sum_d(ss, red, 256);
  if (threadIdx.x == 0) a.partial[(int64_t)blockIdx.y * gridDim.x + blockIdx.x] = s;
}

// rms_adjustment (Muon_util.py:362-372) in the update's dtype:
//   rms:   scale = bf16?(bf16?(1 / bf16?(max(||U||, 1e-8))) * scale_const)
//          (python float / 0-dim tensor = reciprocal, then a scalar multiply)
//   plain: scale = scale_const
__global__ void __launch_bounds__(1024) scale_kernel(const Args a, int64_t nparts) {
  __shared__ double red[32];
  const bool ubf = a.update_bf16 != 0;
  double s = 0.0;
  if (a.flags & ADVOPT_MU_RMS)
    for (int64_t i = threadIdx.x; i < nparts; i += blockDim.x) s += a.partial[i];
  s = block_sum_d(s, red, 1024);
  if (threadIdx.x == 0) {
    float sc = a.scale_const;
    if (a.flags & ADVOPT_MU_RMS) {
      float n = (float)sqrt(s);
      if (ubf) n = round_bf16(n);
      const float lo = ubf ? round_bf16(1e-8f) : 1e-8f;
      if (n < lo) n = lo;
      float rcp = __fdiv_rn(1.0f, n);
      if (ubf) rcp = round_bf16(rcp);
      sc = __fmul_rn(rcp, a.scale_const);
      if (ubf) sc = round_bf16(sc);
    }
    a.scalars[1] = sc;
  }
}

// param_update.apply_parameter_update for one element (param_update.py:77-156).
__device__ __forceinline__ void apply_one(const Args& a, int64_t k, float u, uint32_t r16) {
  const bool pbf = a.param_bf16 != 0;
  float p = pbf ? bf16_to_f(static_cast<const uint16_t*>(a.param)[k]) : static_cast<const float*>(a.param)[k];
  const bool sr = pbf && (a.flags & ADVOPT_MU_SR);
  if (a.wd != 0.0f) {
    if (a.flags & ADVOPT_MU_CAUTIOUS) {
      const float mask = __fmul_rn(u, p) >= 0.0f ? 1.0f : 0.0f;
      p = __fmaf_rn(__fmul_rn(-a.wd, p), mask, p);
    } else {
      // add_(p, alpha=-wd) on a bf16 tensor rounds alpha to bf16
      p = __fmaf_rn(p, -((pbf && !sr) ? round_bf16(a.wd) : a.wd), p);
    }
    if (pbf && !sr) p = round_bf16(p);
  }
  const float pn = __fadd_rn(p, -u);
  if (pbf)
    static_cast<uint16_t*>(a.param)[k] = (uint16_t)(sr ? f_to_bf16_sr(pn, r16) : f_to_bf16_rne(pn));
  else
    static_cast<float*>(a.param)[k] = pn;
}

// ---- stage 2 (Muon): p -= U * scale; eight consecutive elements a thread ----
__global__ void __launch_bounds__(256) apply_kernel(const Args a) {
  const float sc = a.scalars[1];
  const bool ubf = a.update_bf16 != 0;
  const bool need_r = a.param_bf16 && (a.flags & ADVOPT_MU_SR);
  const int64_t groups = (a.numel + 7) / 8;
  for (int64_t gi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; gi < groups; gi += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k0 = gi * 8;
    uint32_t r[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (need_r) noise8(a, a.noise_p, kNoiseP, k0, a.numel, r);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int64_t k = k0 + e;
      if (k < a.numel) {
        float u = __fmul_rn(bf16_to_f(a.u[k]), sc);
        if (ubf) u = round_bf16(u);
        apply_one(a, k, u, r[e]);
      }
    }
  }
}

// Vectorised stage 2 for bf16 params, numel a multiple of 8 (same arithmetic as apply_kernel).
__global__ void __launch_bounds__(256) apply_vec_kernel(const Args a) {
  const float sc = a.scalars[1];
  const bool ubf = a.update_bf16 != 0;
  const bool sr = a.flags & ADVOPT_MU_SR;
  const int64_t groups = a.numel / 8;
  for (int64_t gi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; gi < groups; gi += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k0 = gi * 8;
    uint32_t r[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (sr) noise8(a, a.noise_p, kNoiseP, k0, a.numel, r);
    float u[8], p[8];
    unpack_bf16x8(*reinterpret_cast<const uint4*>(a.u + k0), u);
    uint16_t* pp = static_cast<uint16_t*>(a.param) + k0;
    unpack_bf16x8(*reinterpret_cast<const uint4*>(pp), p);
    uint32_t b[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float ue = __fmul_rn(u[e], sc);
      if (ubf) ue = round_bf16(ue);
      float pe = p[e];
      if (a.wd != 0.0f) {
        if (a.flags & ADVOPT_MU_CAUTIOUS) {
          const float mask = __fmul_rn(ue, pe) >= 0.0f ? 1.0f : 0.0f;
          pe = __fmaf_rn(__fmul_rn(-a.wd, pe), mask, pe);
        } else {
          pe = __fmaf_rn(pe, -(sr ? a.wd : round_bf16(a.wd)), pe);
        }
        if (!sr) pe = round_bf16(pe);
      }
      const float pn = __fadd_rn(pe, -ue);
      b[e] = sr ? f_to_bf16_sr(pn, r[e]) : f_to_bf16_rne(pn);
    }
    *reinterpret_cast<uint4*>(pp) = pack_bf16x8(b);
  }
}

// AdaMuon second moment on U (AdaMuon_adv.py:620-631):
//   v' = v*beta2 + (1-beta2)*u*u;  u' = u / (sqrt(v') + eps)   (atan2: atan2(u, sqrt(v')))
// in bf16 when MBF ('auto' precision with bf16 params), else fp32.
template <bool MBF>
__device__ __forceinline__ float adamuon_u(const Args& a, float u, float v0, float& v1) {
  float v = __fmul_rn(v0, a.beta2);
  if (MBF) v = round_bf16(v);
  v = __fmaf_rn(__fmul_rn(a.c_v, u), u, v);
  if (MBF) v = round_bf16(v);
  v1 = v;
  float den = __fsqrt_rn(v);
  if (MBF) den = round_bf16(den);
  float q;
  if (a.flags & ADVOPT_MU_ATAN2) {
    q = atan2f(u, den);
  } else {
    den = __fadd_rn(den, a.eps);
    if (MBF) den = round_bf16(den);
    q = __fdiv_rn(u, den);
  }
  return MBF ? round_bf16(q) : q;
}

// ---- stage 4: per-chunk sum(u'^2); nothing written ----
template <bool MBF>
__global__ void __launch_bounds__(256) adamuon_stats_kernel(const Args a) {
  __shared__ double redd[kWarps];
  const int64_t nchunks = (a.numel + kChunk - 1) / kChunk;
  for (int64_t c = blockIdx.x; c < nchunks; c += gridDim.x) {
    const int64_t k0 = c * kChunk + threadIdx.x * 8;
    double ss = 0.0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int64_t k = k0 + e;
      if (k < a.numel) {
        float v1;
        const float up = adamuon_u<MBF>(a, bf16_to_f(a.u[k]), load_state(a.v, k, a.v_storage, a.v_scale, true), v1);
        ss += (double)up * (double)up;
      }
    }
    const double s = block_sum_d(ss, redd, 256);
    if (threadIdx.x == 0) a.partial[c] = s;
  }
}

// ---- stage 5: v' stored, p updated with u' * scale ----
template <bool MBF>
__global__ void __launch_bounds__(256) adamuon_apply_kernel(const Args a) {
  __shared__ float redf[kWarps];
  const int64_t nchunks = (a.numel + kChunk - 1) / kChunk;
  const float sc = a.scalars[1];
  const bool ubf = a.update_bf16 != 0;
  const int vst = a.v_storage;
  const bool need_rp = a.param_bf16 && (a.flags & ADVOPT_MU_SR);
  for (int64_t c = blockIdx.x; c < nchunks; c += gridDim.x) {
    const int64_t k0 = c * kChunk + threadIdx.x * 8;
    float vn[8], up[8];
    float vmax = 0.0f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int64_t k = k0 + e;
      vn[e] = 0.0f;
      up[e] = 0.0f;
      if (k < a.numel) {
        up[e] = adamuon_u<MBF>(a, bf16_to_f(a.u[k]), load_state(a.v, k, vst, a.v_scale, true), vn[e]);
        vmax = fmaxf(vmax, vn[e]);
      }
    }
    float safe = 0.0f;
    if (vst == ADVOPT_ST_Q8) {
      const float bmax = block_max256(vmax, redf);
      const float scale = __fdiv_rn(bmax, 255.0f);
      safe = scale < 1e-12f ? 1e-12f : scale;
      if (threadIdx.x == 0) a.v_scale[c] = scale;
    }
    uint32_t rv[8] = {0, 0, 0, 0, 0, 0, 0, 0}, rp[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (vst >= ADVOPT_ST_BF16_SR) noise8(a, a.noise_v, kNoiseV, k0, a.numel, rv);
    if (need_rp) noise8(a, a.noise_p, kNoiseP, k0, a.numel, rp);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int64_t k = k0 + e;
      if (k < a.numel) {
        store_state(a.v, k, vst, vn[e], safe, true, rv[e]);
        float u = __fmul_rn(up[e], sc);
        if (ubf) u = round_bf16(u);
        apply_one(a, k, u, rp[e]);
      }
    }
  }
}

// Row index of element k0 of the flattened [rows][cols] update, advanced one
// element at a time (8 consecutive elements a thread; a row may end inside).
struct RowCursor {
  int64_t r, c, cols;
  __device__ __forceinline__ RowCursor(int64_t k0, int64_t cols_) : cols(cols_) {
    r = k0 / cols_;
    c = k0 - r * cols_;
  }
  __device__ __forceinline__ void next() {
    if (++c == cols) { c = 0; ++r; }
  }
};

// ---- stage 7: NorMuon row statistics (Muon_util.py:349-360) ----
//   v[r] = lerp(v[r], mean_c(u^2), 1 - beta2)  (u^2 in the update's dtype, the
//   mean in float32);  den[r] = sqrt(v[r]) + eps.  One warp per row.
__global__ void __launch_bounds__(256) normuon_rows_kernel(const Args a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool ubf = a.update_bf16 != 0;
  for (int64_t r = (int64_t)blockIdx.x * kWarps + warp; r < a.rows; r += (int64_t)gridDim.x * kWarps) {
    const uint16_t* row = a.u + r * a.cols;
    double s = 0.0;
    for (int64_t c = lane; c < a.cols; c += 32) {
      const float x = bf16_to_f(row[c]);
      float q = __fmul_rn(x, x);
      if (ubf) q = round_bf16(q);
      s += (double)q;
    }
    s = warp_sum_d(s);
    if (lane == 0) {
      const float mean = __fdiv_rn((float)s, (float)a.cols);
      const float v = lerp_t(a.row_v[r], mean, a.nm_w);
      a.row_v[r] = v;
      a.row_den[r] = __fadd_rn(__fsqrt_rn(v), a.nm_eps);
    }
  }
}

// u' = u / den[row], computed in float32 and stored in the update's dtype
__device__ __forceinline__ float normuon_u(const Args& a, float u, int64_t r) {
  const float q = __fdiv_rn(u, a.row_den[r]);
  return a.update_bf16 ? round_bf16(q) : q;
}

// ---- stage 8: per-chunk sum(u'^2) of the NorMuon update ----
__global__ void __launch_bounds__(256) normuon_stats_kernel(const Args a) {
  __shared__ double redd[kWarps];
  const int64_t nchunks = (a.numel + kChunk - 1) / kChunk;
  for (int64_t c = blockIdx.x; c < nchunks; c += gridDim.x) {
    const int64_t k0 = c * kChunk + threadIdx.x * 8;
    double ss = 0.0;
    if (k0 < a.numel) {
      RowCursor rc(k0, a.cols);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (k0 + e < a.numel) {
          const float up = normuon_u(a, bf16_to_f(a.u[k0 + e]), rc.r);
          ss += (double)up * (double)up;
        }
        rc.next();
      }
    }
    const double s = block_sum_d(ss, redd, 256);
    if (threadIdx.x == 0) a.partial[c] = s;
  }
}

// ---- stage 13: per-chunk sum(U^2) of U in `u` (after a low-rank chain) ----
__global__ void __launch_bounds__(256) u_stats_kernel(const Args a) {
  __shared__ double redd[kWarps];
  const int64_t nchunks = (a.numel + kChunk - 1) / kChunk;
  for (int64_t c = blockIdx.x; c < nchunks; c += gridDim.x) {
    const int64_t k0 = c * kChunk + threadIdx.x * 8;
    double ss = 0.0;
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (k0 + e < a.numel) {
        const float f = bf16_to_f(a.u[k0 + e]);
        ss += (double)f * (double)f;
      }
    const double s = block_sum_d(ss, redd, 256);
    if (threadIdx.x == 0) a.partial[c] = s;
  }
}

// ---- stage 9: p updated with u' * scale (NorMuon) ----
__global__ void __launch_bounds__(256) normuon_apply_kernel(const Args a) {
  const float sc = a.scalars[1];
  const bool ubf = a.update_bf16 != 0;
  const bool need_r = a.param_bf16 && (a.flags & ADVOPT_MU_SR);
  const int64_t groups = (a.numel + 7) / 8;
  for (int64_t gi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; gi < groups; gi += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k0 = gi * 8;
    uint32_t r[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (need_r) noise8(a, a.noise_p, kNoiseP, k0, a.numel, r);
    RowCursor rc(k0, a.cols);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int64_t k = k0 + e;
      if (k < a.numel) {
        float u = __fmul_rn(normuon_u(a, bf16_to_f(a.u[k]), rc.r), sc);
        if (ubf) u = round_bf16(u);
        apply_one(a, k, u, r[e]);
      }
      rc.next();
    }
  }
}

// AdaMuon factored second moment (AdaMuon_adv.py:617-631), in float32:
//   v = outer(v_row, v_col)[i][j] * beta2 + (1 - beta2) * u * u
//   u' = u / R(sqrt(v) + eps)   (atan2: atan2(u, R(sqrt(v))))
// with R the update's dtype; (i, j) = divmod(k, d2) in the effective shape.
__device__ __forceinline__ float vfact_u(const Args& a, float u, float v) {
  const bool ubf = a.update_bf16 != 0;
  float den = __fsqrt_rn(v);
  float q;
  if (a.flags & ADVOPT_MU_ATAN2) {
    if (ubf) den = round_bf16(den);
    q = atan2f(u, den);
  } else {
    den = __fadd_rn(den, a.eps);
    if (ubf) den = round_bf16(den);
    q = __fdiv_rn(u, den);
  }
  return ubf ? round_bf16(q) : q;
}

// ---- stage 10a: v (into v_full) and per-chunk sum(u'^2) ----
__global__ void __launch_bounds__(256) vfact_stats_kernel(const Args a) {
  __shared__ double redd[kWarps];
  const int64_t nchunks = (a.numel + kChunk - 1) / kChunk;
  for (int64_t c = blockIdx.x; c < nchunks; c += gridDim.x) {
    const int64_t k0 = c * kChunk + threadIdx.x * 8;
    double ss = 0.0;
    if (k0 < a.numel) {
      RowCursor rc(k0, a.d2);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int64_t k = k0 + e;
        if (k < a.numel) {
          const float u = bf16_to_f(a.u[k]);
          float v = __fmul_rn(__fmul_rn(a.v_row[rc.r], a.v_col[rc.c]), a.beta2);
          v = __fmaf_rn(__fmul_rn(a.c_v, u), u, v);
          a.v_full[k] = v;
          const float up = vfact_u(a, u, v);
          ss += (double)up * (double)up;
        }
        rc.next();
      }
    }
    const double s = block_sum_d(ss, redd, 256);
    if (threadIdx.x == 0) a.partial[c] = s;
  }
}

// ---- stage 10b: row sums of v (one warp per row of the effective shape) ----
__global__ void __launch_bounds__(256) vfact_rows_kernel(const Args a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int64_t i = (int64_t)blockIdx.x * kWarps + warp; i < a.d1; i += (int64_t)gridDim.x * kWarps) {
    const float* row = a.v_full + i * a.d2;
    double s = 0.0;
    for (int64_t j = lane; j < a.d2; j += 32) s += (double)row[j];
    s = warp_sum_d(s);
    if (lane == 0) a.v_sums[i] = s;
  }
}

// ---- stage 10c: column partial sums over ADVOPT_VCOL_SPLIT row ranges ----
__global__ void __launch_bounds__(256) vfact_cols_kernel(const Args a) {
  const int64_t j = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int split = blockIdx.y;
  if (j >= a.d2) return;
  const int64_t i0 = a.d1 * split / ADVOPT_VCOL_SPLIT, i1 = a.d1 * (split + 1) / ADVOPT_VCOL_SPLIT;
  double s = 0.0;
  for (int64_t i = i0; i < i1; ++i) s += (double)a.v_full[i * a.d2 + j];
  a.v_sums[a.d1 + (int64_t)split * a.d2 + j] = s;
}

// ---- stage 10d: the new factors (factorization_util.py:60-80): row and
// column sums as float32, the factor of the smaller dimension divided by
// max(its total, 1e-12).  One CTA of 1024. ----
__global__ void __launch_bounds__(1024) vfact_finish_kernel(const Args a) {
  __shared__ double red[32];
  __shared__ float scale_s;
  const double* rows = a.v_sums;
  const double* cols = a.v_sums + a.d1;
  const bool by_rows = a.d1 < a.d2;
  double t = 0.0;
  if (by_rows) {
    for (int64_t i = threadIdx.x; i < a.d1; i += blockDim.x) t += rows[i];
  } else {
    for (int64_t j = threadIdx.x; j < a.d2; j += blockDim.x) {
      double cj = 0.0;
      for (int sp = 0; sp < ADVOPT_VCOL_SPLIT; ++sp) cj += cols[(int64_t)sp * a.d2 + j];
      t += cj;
    }
  }
  t = block_sum_d(t, red, 1024);
  if (threadIdx.x == 0) {
    const float tf = (float)t;
    scale_s = tf > 1e-12f ? tf : 1e-12f;
  }
  __syncthreads();
  const float sc = scale_s;
  for (int64_t i = threadIdx.x; i < a.d1; i += blockDim.x) {
    const float r = (float)rows[i];
    a.v_row[i] = by_rows ? __fdiv_rn(r, sc) : r;
  }
  for (int64_t j = threadIdx.x; j < a.d2; j += blockDim.x) {
    double cj = 0.0;
    for (int sp = 0; sp < ADVOPT_VCOL_SPLIT; ++sp) cj += cols[(int64_t)sp * a.d2 + j];
    const float c = (float)cj;
    a.v_col[j] = by_rows ? c : __fdiv_rn(c, sc);
  }
}

// ---- stage 11: p updated with u' * scale (AdaMuon factored) ----
__global__ void __launch_bounds__(256) vfact_apply_kernel(const Args a) {
  const float sc = a.scalars[1];
  const bool ubf = a.update_bf16 != 0;
  const bool need_r = a.param_bf16 && (a.flags & ADVOPT_MU_SR);
  const int64_t groups = (a.numel + 7) / 8;
  for (int64_t gi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; gi < groups; gi += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k0 = gi * 8;
    uint32_t r[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (need_r) noise8(a, a.noise_p, kNoiseP, k0, a.numel, r);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int64_t k = k0 + e;
      if (k < a.numel) {
        float u = __fmul_rn(vfact_u(a, bf16_to_f(a.u[k]), a.v_full[k]), sc);
        if (ubf) u = round_bf16(u);
        apply_one(a, k, u, r[e]);
      }
    }
  }
}

}  // namespace muon
}  // namespace advopt

using namespace advopt;
using namespace advopt::muon;

static int sm_count() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

static unsigned grid_for(int64_t units) {
  const int64_t cap = (int64_t)sm_count() * 8;
  const int64_t g = units < cap ? units : cap;
  return (unsigned)(g > 0 ? g : 1);
}

extern "C" int advopt_muon_stage(const advopt_muon_args* ap, int32_t stage, void* stream) {
  if (!ap) return set_error(ADVOPT_E_INVALID, "advopt_muon_stage: null arguments");
  const Args& a = *ap;
  if (a.numel <= 0 || a.rows <= 0 || a.cols <= 0 || a.rows * a.cols != a.numel)
    return set_error(ADVOPT_E_INVALID, "advopt_muon_stage: rows * cols must equal numel > 0");
  if (!a.grad || !a.x0 || !a.u || !a.partial || !a.scalars || (stage != 6 && stage != 3 && (!a.param || !a.m)))
    return set_error(ADVOPT_E_INVALID, "advopt_muon_stage: null buffer");
  const int64_t m = a.rows < a.cols ? a.rows : a.cols, n = a.rows < a.cols ? a.cols : a.rows;
  const bool tr = (a.flags & ADVOPT_MU_TRANSPOSED) != 0;
  if (tr != (a.rows > a.cols) || a.m_pad < m || a.n_pad < n || a.m_pad % 256 || a.n_pad % 256 || a.ld_ns < a.n_pad)
    return set_error(ADVOPT_E_INVALID, "advopt_muon_stage: workspace shape does not match the matrix");
  if (a.m_storage == ADVOPT_ST_Q8 && !a.m_scale) return set_error(ADVOPT_E_INVALID, "advopt_muon_stage: no m scale");
  if ((a.flags & ADVOPT_MU_NOISE_IN) && ((a.m_storage >= ADVOPT_ST_BF16_SR && !a.noise_m) ||
                                         (a.param_bf16 && (a.flags & ADVOPT_MU_SR) && !a.noise_p)))
    return set_error(ADVOPT_E_INVALID, "advopt_muon_stage: injected noise missing");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t nchunks = (a.numel + kChunk - 1) / kChunk;
  const dim3 tb(32, 8);
  // the vectorised kernels read and write 8 elements (16 bytes of bf16) at a time
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  const bool vec = a.numel % 8 == 0 && al16(a.grad) && al16(a.x0) && al16(a.u) && (!a.ns || al16(a.ns)) &&
                   (!a.param || al16(a.param)) && (!a.m || al16(a.m)) && (!a.ns_result || al16(a.ns_result)) &&
                   a.ld_ns % 8 == 0;
  switch (stage) {
    case 0:
    case 6: {
      if (!a.ns) return set_error(ADVOPT_E_INVALID, "advopt_muon_stage: null workspace");
      const unsigned gp = grid_for(nchunks);
      if (vec && a.param_bf16 && (stage == 6 || (a.m_storage != ADVOPT_ST_Q8 && !(a.flags & ADVOPT_MU_MARS)))) {
        if (stage == 6) prep_vec_kernel<false, true, ADVOPT_ST_BF16><<<gp, 256, 0, s>>>(a);
        else if (a.m_storage == ADVOPT_ST_F32)
          a.math_bf16 ? prep_vec_kernel<true, false, ADVOPT_ST_F32><<<gp, 256, 0, s>>>(a)
                      : prep_vec_kernel<false, false, ADVOPT_ST_F32><<<gp, 256, 0, s>>>(a);
        else if (a.m_storage == ADVOPT_ST_BF16)
          a.math_bf16 ? prep_vec_kernel<true, false, ADVOPT_ST_BF16><<<gp, 256, 0, s>>>(a)
                      : prep_vec_kernel<false, false, ADVOPT_ST_BF16><<<gp, 256, 0, s>>>(a);
        else
          a.math_bf16 ? prep_vec_kernel<true, false, ADVOPT_ST_BF16_SR><<<gp, 256, 0, s>>>(a)
                      : prep_vec_kernel<false, false, ADVOPT_ST_BF16_SR><<<gp, 256, 0, s>>>(a);
      } else if (stage == 6) {
        prep_kernel<false, true><<<gp, 256, 0, s>>>(a);
      } else if (a.math_bf16) {
        prep_kernel<true, false><<<gp, 256, 0, s>>>(a);
      } else {
        prep_kernel<false, false><<<gp, 256, 0, s>>>(a);
      }
      // low-rank: X0 feeds the sketch products; the chain runs on the projection
      if (a.flags & ADVOPT_MU_LOWRANK) break;
      norm_kernel<<<1, 1024, 0, s>>>(a, nchunks);
      if (vec && a.cols % 8 == 0 && tr)
        load_vec_t_kernel<<<dim3((unsigned)(a.n_pad / kTile), (unsigned)(a.m_pad / kTile)), 256, 0, s>>>(a);
      else if (vec && a.cols % 8 == 0)
        load_vec_kernel<<<grid_for(a.m_pad * a.n_pad / 2048), 256, 0, s>>>(a);
      else
        load_kernel<<<dim3((unsigned)(a.n_pad / 32), (unsigned)(a.m_pad / 32)), tb, 0, s>>>(a);
      break;
    }
    case 1:
    case 3: {
      if (!a.ns_result) return set_error(ADVOPT_E_INVALID, "advopt_muon_stage: null Newton-Schulz result");
      int64_t nparts;
      if (vec && a.cols % 8 == 0 && tr) {
        const dim3 tg((unsigned)((a.cols + kTile - 1) / kTile), (unsigned)((a.rows + kTile - 1) / kTile));
        store_vec_t_kernel<<<tg, 256, 0, s>>>(a);
        nparts = (int64_t)tg.x * tg.y;
      } else if (vec && a.cols % 8 == 0) {
        const unsigned g = grid_for(a.numel / 2048 + 1);
        store_vec_kernel<<<g, 256, 0, s>>>(a);
        nparts = g;
      } else {
        const dim3 tg((unsigned)((a.cols + 31) / 32), (unsigned)((a.rows + 31) / 32));
        store_kernel<<<tg, tb, 0, s>>>(a);
        nparts = (int64_t)tg.x * tg.y;
      }
      if (stage == 1) scale_kernel<<<1, 1024, 0, s>>>(a, nparts);
      break;
    }
    case 2:
      if (vec && a.param_bf16)
        apply_vec_kernel<<<grid_for((a.numel + 8 * 256 - 1) / (8 * 256)), 256, 0, s>>>(a);
      else
        apply_kernel<<<grid_for((a.numel + 8 * 256 - 1) / (8 * 256)), 256, 0, s>>>(a);
      break;
    case 4:
    case 5: {
      if (!a.v || (a.v_storage == ADVOPT_ST_Q8 && !a.v_scale))
        return set_error(ADVOPT_E_INVALID, "advopt_muon_stage: AdaMuon second moment missing");
      if (stage == 5 && (a.flags & ADVOPT_MU_NOISE_IN) && a.v_storage >= ADVOPT_ST_BF16_SR && !a.noise_v)
        return set_error(ADVOPT_E_INVALID, "advopt_muon_stage: injected noise missing");
      if (stage == 4) {
        if (a.math_bf16) adamuon_stats_kernel<true><<<grid_for(nchunks), 256, 0, s>>>(a);
        else adamuon_stats_kernel<false><<<grid_for(nchunks), 256, 0, s>>>(a);
        scale_kernel<<<1, 1024, 0, s>>>(a, nchunks);
      } else {
        if (a.math_bf16) adamuon_apply_kernel<true><<<grid_for(nchunks), 256, 0, s>>>(a);
        else adamuon_apply_kernel<false><<<grid_for(nchunks), 256, 0, s>>>(a);
      }
      break;
    }
    case 7:
    case 8:
    case 9:
      if (!a.row_v || !a.row_den) return set_error(ADVOPT_E_INVALID, "advopt_muon_stage: NorMuon buffers missing");
      if (stage == 7) {
        normuon_rows_kernel<<<grid_for((a.rows + kWarps - 1) / kWarps), 256, 0, s>>>(a);
      } else if (stage == 8) {
        normuon_stats_kernel<<<grid_for(nchunks), 256, 0, s>>>(a);
        scale_kernel<<<1, 1024, 0, s>>>(a, nchunks);
      } else {
        normuon_apply_kernel<<<grid_for((a.numel + 8 * 256 - 1) / (8 * 256)), 256, 0, s>>>(a);
      }
      break;
    case 13:
      u_stats_kernel<<<grid_for(nchunks), 256, 0, s>>>(a);
      scale_kernel<<<1, 1024, 0, s>>>(a, nchunks);
      break;
    case 10:
    case 11:
      if (!a.v_row || !a.v_col || !a.v_full || !a.v_sums || a.d1 <= 0 || a.d2 <= 0 || a.d1 * a.d2 != a.numel)
        return set_error(ADVOPT_E_INVALID, "advopt_muon_stage: AdaMuon factored second moment missing");
      if (stage == 10) {
        vfact_stats_kernel<<<grid_for(nchunks), 256, 0, s>>>(a);
        scale_kernel<<<1, 1024, 0, s>>>(a, nchunks);
        vfact_rows_kernel<<<grid_for((a.d1 + kWarps - 1) / kWarps), 256, 0, s>>>(a);
        vfact_cols_kernel<<<dim3((unsigned)((a.d2 + 255) / 256), ADVOPT_VCOL_SPLIT), 256, 0, s>>>(a);
        vfact_finish_kernel<<<1, 1024, 0, s>>>(a);
      } else {
        vfact_apply_kernel<<<grid_for((a.numel + 8 * 256 - 1) / (8 * 256)), 256, 0, s>>>(a);
      }
      break;
    default:
      return set_error(ADVOPT_E_INVALID, "advopt_muon_stage: unknown stage");
  }
  return check_cuda(cudaGetLastError(), "advopt_muon_stage");
}
