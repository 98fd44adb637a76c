// Lion_adv step (Lion_adv.py:213-278 with lion_k.py:23-24, kappa_p = 1) for
// a whole parameter group: one grid-stride pass over the pieces, 8 elements
// per thread.
//   update = sign(lerp(g, m, beta1)) * lr        (computed in the param dtype)
//   m      = lerp(m, g, 1 - beta2)
//   p      = apply_parameter_update(p, update)   (param_update.py:77-156)
#include "advopt.h"
#include "capi_internal.h"
#include "common.cuh"

namespace advopt {

template <bool PBF>
__global__ void __launch_bounds__(kThreads) lion_kernel(const advopt_lion_tensor* tensors, const advopt_piece* pieces,
                                                        int n_pieces, float w1, float w2, uint32_t flags,
                                                        uint64_t seed) {
  const bool sr = PBF && (flags & ADVOPT_F_SR);
  const bool cautious = flags & ADVOPT_F_CAUTIOUS;
  const bool noise_in = flags & ADVOPT_F_NOISE_IN;
  auto R = [](float x) { return PBF ? round_bf16(x) : x; };
  for (int pi = blockIdx.x; pi < n_pieces; pi += gridDim.x) {
    const advopt_piece pc = pieces[pi];
    const advopt_lion_tensor T = tensors[pc.tensor];
    const bool vec = T.flags & ADVOPT_T_VEC;
    for (int64_t cs = pc.begin; cs < pc.end; cs += kChunk) {
      const int clen = (int)min((int64_t)kChunk, pc.end - cs);
      const int64_t k0 = cs + threadIdx.x * kVec;
      const int nv = max(0, min(kVec, clen - (int)threadIdx.x * kVec));
      if (nv == 0) continue;
      const bool v8 = vec && nv == kVec;
      float g[8], p[8], m[8];
      load8<PBF>(T.grad, k0, nv, v8, g);
      load8<PBF>(T.param, k0, nv, v8, p);
      load8<PBF>(T.exp_avg, k0, nv, v8, m);
      float u[8], mn[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float c = R(lerp_t(g[e], m[e], w1));         // torch.lerp(grad, exp_avg, beta1)
        mn[e] = R(lerp_t(m[e], g[e], w2));                 // exp_avg.lerp_(grad, 1 - beta2)
        const float sg = c > 0.0f ? 1.0f : (c < 0.0f ? -1.0f : c);
        u[e] = R(__fmul_rn(sg, T.lr));                     // update.mul_(lr)
      }
      uint32_t r[8];
      if (sr) {
        if (noise_in) {
#pragma unroll
          for (int e = 0; e < 8; ++e) r[e] = e < nv ? (uint32_t)T.noise_p[k0 + e] : 0u;
        } else {
          philox_u16x8(seed, T.tensor_id, T.step, kNoiseP, k0, r);
        }
      }
      if (PBF) {
        uint32_t mb[8], pb[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          mb[e] = f_to_bf16_rne(mn[e]);
          float pcv = p[e];
          if (T.wd != 0.0f) {
            if (cautious) {
              const float mask = (sr ? __fmul_rn(u[e], pcv) : round_bf16(__fmul_rn(u[e], pcv))) >= 0.0f ? 1.0f : 0.0f;
              pcv = __fmaf_rn(__fmul_rn(-T.wd, pcv), mask, pcv);
            } else {
              // add_(p, alpha=-wd) on a bf16 tensor rounds alpha to bf16
              pcv = __fmaf_rn(pcv, -(sr ? T.wd : round_bf16(T.wd)), pcv);
            }
            if (!sr) pcv = round_bf16(pcv);
          }
          pcv = __fadd_rn(pcv, -u[e]);
          pb[e] = sr ? f_to_bf16_sr(pcv, r[e]) : f_to_bf16_rne(pcv);
        }
        store8_bf16(T.exp_avg, k0, nv, v8, mb);
        store8_bf16(T.param, k0, nv, v8, pb);
      } else {
        float pf[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          float pcv = p[e];
          if (T.wd != 0.0f) {
            if (cautious) {
              const float mask = __fmul_rn(u[e], pcv) >= 0.0f ? 1.0f : 0.0f;
              pcv = __fmaf_rn(__fmul_rn(-T.wd, pcv), mask, pcv);
            } else {
              pcv = __fmaf_rn(pcv, -T.wd, pcv);
            }
          }
          pf[e] = __fadd_rn(pcv, -u[e]);
        }
        store8_f32(T.exp_avg, k0, nv, v8, mn);
        store8_f32(T.param, k0, nv, v8, pf);
      }
    }
  }
}

}  // namespace advopt

extern "C" int advopt_lion_step(const advopt_lion_tensor* tensors, int32_t n_tensors, const advopt_piece* pieces,
                                int32_t n_pieces, int32_t param_dtype, float w1, float w2, uint32_t flags,
                                uint64_t seed, void* stream) {
  using namespace advopt;
  if (!tensors || !pieces || n_tensors <= 0 || n_pieces <= 0)
    return set_error(ADVOPT_E_INVALID, "advopt_lion_step: empty tables");
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = n_pieces < sms * 8 ? n_pieces : sms * 8;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (param_dtype == ADVOPT_DT_BF16)
    lion_kernel<true><<<grid, kThreads, 0, s>>>(tensors, pieces, n_pieces, w1, w2, flags, seed);
  else
    lion_kernel<false><<<grid, kThreads, 0, s>>>(tensors, pieces, n_pieces, w1, w2, flags, seed);
  return check_cuda(cudaGetLastError(), "advopt_lion_step");
}
