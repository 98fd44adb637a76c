// Spectral normalisation of Adam-family and Lion updates (scaled_optm.py:35-72,
// 160-168, 255-295) and the parameter update that follows it
// (param_update.py:77-156).  The step kernel has written each tensor's
// unscaled update U (ADVOPT_F_EMIT_UPDATE); six launches finish the step:
//   1. spec_vpart_kernel   U^T u per row slab (column partials, float32)
//   2. spec_vsum_kernel    U^T u from the slabs, column-parallel (float64),
//      and its squared norm; spec_vfinish_kernel v = U^T u / |U^T u|
//   3. spec_rows_kernel    U v per row (a warp per row), or max|U| for 1-D
//   4. spec_ufinish_kernel u = U v / |U v|, sigma = u . U v, the scale
//   5. spec_apply_kernel   p = apply_parameter_update(p, U * scale)
// Every value the reference rounds to a torch dtype (the singular vectors'
// dtype for 2-D updates, the update's for 1-D) is rounded here at the same
// op; sums run in float32 per thread and float64 across threads, in an order
// of their own.  All passes are HBM-bound: U is read three times (passes 1, 3
// and 5) and written once by the step kernel.
#include "adam_impl.cuh"

namespace advopt {
namespace {

constexpr int kSThreads = 256;
constexpr int kSCols = kSThreads * 8;      // columns per block pass of the U^T u kernel
constexpr int kSlabMax = 64;               // rows per slab / row item

__device__ __forceinline__ float ld_val(const void* base, int64_t k, bool bf) {
  return bf ? bf16_to_f(static_cast<const uint16_t*>(base)[k]) : static_cast<const float*>(base)[k];
}
__device__ __forceinline__ float rnd(float x, bool bf) { return bf ? round_bf16(x) : x; }
__device__ __forceinline__ void st_val(void* base, int64_t k, float x, bool bf) {
  if (bf)
    static_cast<uint16_t*>(base)[k] = (uint16_t)f_to_bf16_rne(x);
  else
    static_cast<float*>(base)[k] = x;
}
// 8 consecutive update values starting at element k0 (nv of them valid)
__device__ __forceinline__ void ld8(const void* base, int64_t k0, int nv, bool bf, bool vec, float (&x)[8]) {
  if (bf)
    load8<true>(base, k0, nv, vec && nv == 8, x);
  else
    load8<false>(base, k0, nv, vec && nv == 8, x);
}

__device__ double block_sum_d(double v, double* red) {
  v = warp_sum_d(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double t = 0.0;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
  return t;
}

// 1. v_partial[slab][j] = sum over the slab's rows i of U[i][j] * u[i]
__global__ void __launch_bounds__(kSThreads) spec_vpart_kernel(const advopt_spectral_tensor* S,
                                                               const advopt_piece* items) {
  const advopt_piece it = items[blockIdx.x];
  const advopt_spectral_tensor& T = S[it.tensor];
  const bool ub = T.flags & ADVOPT_S_UPD_BF16, vb = T.flags & ADVOPT_S_VEC_BF16;
  const int64_t d_in = T.d_in;
  const int nrow = (int)(it.end - it.begin);
  __shared__ float us[kSlabMax];
  for (int r = threadIdx.x; r < nrow; r += blockDim.x) us[r] = ld_val(T.u, it.begin + r, vb);
  // the squared-norm accumulator of pass 2 starts at zero (pass 2 runs after this launch)
  if (it.slot == 0 && threadIdx.x == 0) *reinterpret_cast<double*>(T.scalars + 2) = 0.0;
  __syncthreads();
  const bool vec = (d_in % 8) == 0 && ((reinterpret_cast<uintptr_t>(T.update) & 15) == 0);
  float* dst = T.v_partial + (int64_t)it.slot * d_in;
  for (int64_t j0 = (int64_t)threadIdx.x * 8; j0 < d_in; j0 += kSCols) {
    const int nj = (int)min((int64_t)8, d_in - j0);
    float acc[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
    for (int r = 0; r < nrow; ++r) {
      float x[8];
      ld8(T.update, (it.begin + r) * d_in + j0, nj, ub, vec, x);
      const float ur = us[r];
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = __fmaf_rn(x[e], ur, acc[e]);
    }
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (e < nj) dst[j0 + e] = acc[e];
  }
}

// 2a. v_raw[j] = sum over slabs (float64, rounded to the vectors' dtype), one
//     thread per column over a grid of (kVsumBlocks, tensor) striding over the
//     columns, and the squared norm accumulated per block into a float64 word.
constexpr int kVsumThreads = 256;
constexpr int kVsumBlocks = 64;
__global__ void __launch_bounds__(kVsumThreads) spec_vsum_kernel(const advopt_spectral_tensor* S) {
  const advopt_spectral_tensor& T = S[blockIdx.y];
  if (T.flags & ADVOPT_S_MAXABS) return;
  const int64_t d_in = T.d_in;
  if ((int64_t)blockIdx.x * kVsumThreads >= d_in) return;        // whole block past the columns
  const bool vb = T.flags & ADVOPT_S_VEC_BF16;
  double sq = 0.0;
  for (int64_t j = (int64_t)blockIdx.x * kVsumThreads + threadIdx.x; j < d_in;
       j += (int64_t)kVsumBlocks * kVsumThreads) {
    double a = 0.0;
    for (int s = 0; s < T.n_slabs; ++s) a += (double)T.v_partial[(int64_t)s * d_in + j];
    const float vr = rnd((float)a, vb);              // torch.mv's output dtype
    T.v_partial[j] = vr;                             // slab 0 now holds v_raw
    sq += (double)vr * (double)vr;
  }
  __shared__ double red[kVsumThreads / 32];
  sq = warp_sum_d(sq);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < kVsumThreads / 32; ++w) t += red[w];
    atomicAdd(reinterpret_cast<double*>(T.scalars + 2), t);
  }
}

// 2b. |v_raw|, v = v_raw / max(|v_raw|, 1e-8) where |v_raw| >= 1e-6
//     (scaled_optm.py:274-279).  1-D tensors: clear the max|U| word.
__global__ void __launch_bounds__(1024) spec_vfinish_kernel(const advopt_spectral_tensor* S) {
  const advopt_spectral_tensor& T = S[blockIdx.x];
  __shared__ float norm_s;
  if (T.flags & ADVOPT_S_MAXABS) {
    if (threadIdx.x == 0) reinterpret_cast<unsigned int*>(T.scalars)[1] = 0u;
    return;
  }
  const bool vb = T.flags & ADVOPT_S_VEC_BF16;
  const int64_t d_in = T.d_in;
  if (threadIdx.x == 0) norm_s = rnd((float)sqrt(*reinterpret_cast<const double*>(T.scalars + 2)), vb);
  __syncthreads();
  const float nrm = norm_s;
  if (!(nrm >= 1e-6f)) return;                       // keep v (torch.where(v_norm >= 1e-6, ...))
  const float den = rnd(fmaxf(nrm, 1e-8f), vb);      // v_norm.clamp_min(1e-8)
  for (int64_t j = threadIdx.x; j < d_in; j += blockDim.x)
    st_val(T.v, j, rnd(__fdiv_rn(T.v_partial[j], den), vb), vb);
}

// 3. u_raw[i] = U[i] . v (a warp per row; scaled_optm.py:282), or, for 1-D
//    updates, max|U| over the item's elements (scaled_optm.py:167).
__global__ void __launch_bounds__(kSThreads) spec_rows_kernel(const advopt_spectral_tensor* S,
                                                              const advopt_piece* items) {
  const advopt_piece it = items[blockIdx.x];
  const advopt_spectral_tensor& T = S[it.tensor];
  const bool ub = T.flags & ADVOPT_S_UPD_BF16, vb = T.flags & ADVOPT_S_VEC_BF16;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (T.flags & ADVOPT_S_MAXABS) {
    const bool vec = (reinterpret_cast<uintptr_t>(T.update) & 15) == 0 && (it.begin % 8) == 0;
    float mx = 0.0f;
    for (int64_t k0 = it.begin + (int64_t)threadIdx.x * 8; k0 < it.end; k0 += (int64_t)blockDim.x * 8) {
      float x[8];
      const int nv = (int)min((int64_t)8, it.end - k0);
      ld8(T.update, k0, nv, ub, vec, x);
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (e < nv) mx = fmaxf(mx, fabsf(x[e]));
    }
    mx = warp_max(mx);
    // non-negative floats order like their bit patterns
    if (lane == 0) atomicMax(reinterpret_cast<unsigned int*>(T.scalars) + 1, __float_as_uint(mx));
    return;
  }
  const int64_t d_in = T.d_in;
  const bool vec = (d_in % 8) == 0 && ((reinterpret_cast<uintptr_t>(T.update) & 15) == 0);
  const bool vvec = (d_in % 8) == 0 && ((reinterpret_cast<uintptr_t>(T.v) & 15) == 0);
  for (int64_t i = it.begin + warp; i < it.end; i += kSThreads / 32) {
    float acc0 = 0.0f, acc1 = 0.0f;
    // two column blocks of 256 in flight per lane; v in 16-byte loads
    for (int64_t j0 = (int64_t)lane * 8; j0 < d_in; j0 += 512) {
      const int64_t j1 = j0 + 256;
      const int n0 = (int)min((int64_t)8, d_in - j0);
      const int n1 = j1 < d_in ? (int)min((int64_t)8, d_in - j1) : 0;
      float x0[8], x1[8], v0[8], v1[8];
      ld8(T.update, i * d_in + j0, n0, ub, vec, x0);
      ld8(T.v, j0, n0, vb, vvec, v0);
      if (n1 > 0) {
        ld8(T.update, i * d_in + j1, n1, ub, vec, x1);
        ld8(T.v, j1, n1, vb, vvec, v1);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (e < n0) acc0 = __fmaf_rn(x0[e], v0[e], acc0);
#pragma unroll
      for (int e = 0; e < 8; ++e)
        if (e < n1) acc1 = __fmaf_rn(x1[e], v1[e], acc1);
    }
    const float acc = warp_sum(__fadd_rn(acc0, acc1));
    if (lane == 0) T.u_raw[i] = rnd(acc, vb);
  }
}

// 4. u = u_raw / max(|u_raw|, 1e-8) where |u_raw| >= 1e-6, sigma = u . u_raw,
//    scale = lr * (target / max(sigma, eps)) (scaled_optm.py:285-294: a
//    scalar over a tensor is reciprocal(t) * scalar); 1-D: lr / max(max|U|, 1e-12).
__global__ void __launch_bounds__(1024) spec_ufinish_kernel(const advopt_adam_tensor* tensors,
                                                            const advopt_spectral_tensor* S) {
  const advopt_spectral_tensor& T = S[blockIdx.x];
  const float lr = tensors[blockIdx.x].step_size;
  __shared__ double red[32];
  __shared__ float norm_s;
  if (T.flags & ADVOPT_S_MAXABS) {
    if (threadIdx.x == 0) {
      const bool ub = T.flags & ADVOPT_S_UPD_BF16;
      const float mx = __uint_as_float(reinterpret_cast<const unsigned int*>(T.scalars)[1]);
      const float nrm = rnd(fmaxf(rnd(mx, ub), 1e-12f), ub);     // vector_norm(inf).clamp_min(1e-12)
      const float r = rnd(__fdiv_rn(1.0f, nrm), ub);
      T.scalars[0] = rnd(__fmul_rn(r, lr), ub);
    }
    return;
  }
  const bool vb = T.flags & ADVOPT_S_VEC_BF16;
  const int64_t d_out = T.d_out;
  double ss = 0.0;
  for (int64_t i = threadIdx.x; i < d_out; i += blockDim.x) ss += (double)T.u_raw[i] * (double)T.u_raw[i];
  ss = block_sum_d(ss, red);
  if (threadIdx.x == 0) norm_s = rnd((float)sqrt(ss), vb);
  __syncthreads();
  const float nrm = norm_s;
  const bool upd = nrm >= 1e-6f;
  const float den = rnd(fmaxf(nrm, 1e-8f), vb);
  double dot = 0.0;
  for (int64_t i = threadIdx.x; i < d_out; i += blockDim.x) {
    float nu;
    if (upd) {
      nu = rnd(__fdiv_rn(T.u_raw[i], den), vb);
      st_val(T.u, i, nu, vb);
    } else {
      nu = ld_val(T.u, i, vb);
    }
    dot += (double)rnd(__fmul_rn(nu, T.u_raw[i]), vb);   // vecdot = (u * u_raw).sum(): products in the dtype
  }
  dot = block_sum_d(dot, red);
  if (threadIdx.x == 0) {
    const float sigma = rnd((float)dot, vb);                      // vecdot(u, u_raw)
    const float eps = (float)(1.0 / (sqrt((double)d_out) + sqrt((double)T.d_in)));
    const float sc = rnd(sigma >= eps ? sigma : eps, vb);         // sigma.clamp_min_(eps)
    const float r = rnd(__fdiv_rn(1.0f, sc), vb);
    const float s1 = rnd(__fmul_rn(r, T.target), vb);
    T.scalars[0] = rnd(__fmul_rn(s1, lr), vb);
  }
}

// 5. p = apply_parameter_update(p, U * scale) over the launch's pieces: CTA b
//    takes every kApplySplit-th chunk of piece b / kApplySplit, so the pass has
//    kApplySplit times as many CTAs as the step (enough loads in flight for HBM).
constexpr int kApplySplit = 8;
template <bool PBF, bool NOISE_IN>
__global__ void __launch_bounds__(kThreads, 4) spec_apply_kernel(const advopt_adam_launch L,
                                                                 const advopt_spectral_tensor* S) {
  const int tid = threadIdx.x;
  const uint32_t F = L.flags;
  const bool cautious = F & ADVOPT_F_CAUTIOUS;
  const bool sr = PBF && (F & ADVOPT_F_SR);
  const bool anchors = F & ADVOPT_F_ANCHORS;
  __shared__ TensorRegs Ts;
  const int pi = blockIdx.x / kApplySplit, part = blockIdx.x % kApplySplit;
  const advopt_piece pc = L.pieces[pi];
  if (tid == 0) load_tensor(L.tensors + pc.tensor, Ts);
  __syncthreads();
  const TensorRegs& T = Ts;
  const advopt_spectral_tensor& ST = S[pc.tensor];
  const bool ub = ST.flags & ADVOPT_S_UPD_BF16;
  const float sc = ST.scalars[0];
  const bool vec = T.flags & ADVOPT_T_VEC;
  const bool has_anchor = anchors && (((T.flags >> ADVOPT_T_ANCHOR_SHIFT) & 7u) != 0);
  const float wd = T.wd, cwd = T.cwd;
  for (int64_t cs = pc.begin + (int64_t)part * kChunk; cs < pc.end; cs += (int64_t)kApplySplit * kChunk) {
    const int clen = (int)min((int64_t)kChunk, pc.end - cs);
    const int64_t k0 = cs + tid * kVec;
    const int nv = max(0, min(kVec, clen - tid * kVec));
    if (nv == 0) continue;
    const bool v8 = vec && nv == kVec;
    float p[8], u[8];
    load8<PBF>(T.param, k0, nv, v8, p);
    ld8(ST.update, k0, nv, ub, v8, u);
    U4 nzp{0u, 0u, 0u, 0u};
    if (sr) nzp = noise_words<NOISE_IN>(L, T, T.nz_p, kNoiseP, k0, nv);
    uint32_t pout[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float ui = rnd(__fmul_rn(u[e], sc), ub);            // update.mul_(scale)
      const float anc = (has_anchor && e < nv) ? anchor_value(T, k0 + e, PBF) : 0.0f;
      if (PBF && !sr) {
        const float pcv = weight_decay<true>(p[e], ui, wd, cwd, cautious, has_anchor, anc, false, 0.0f);
        pout[e] = f_to_bf16_rne(__fadd_rn(pcv, -ui));
      } else {
        const float pcv = weight_decay<false>(p[e], ui, wd, cwd, cautious, has_anchor, anc, false, 0.0f);
        const float pn = __fadd_rn(pcv, -ui);
        pout[e] = PBF ? (__float_as_uint(pn) + noise_at(nzp, e)) : __float_as_uint(pn);
      }
    }
    if (PBF) {
      uint32_t b[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) b[e] = sr ? (pout[e] >> 16) : pout[e];
      store8_bf16(T.param, k0, nv, v8, b);
    } else {
      float x[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = __uint_as_float(pout[e]);
      store8_f32(T.param, k0, nv, v8, x);
    }
  }
}

}  // namespace
}  // namespace advopt

extern "C" int advopt_spectral_step(const advopt_adam_launch* L, const advopt_spectral_tensor* S,
                                    const advopt_piece* col_items, int32_t n_col_items,
                                    const advopt_piece* row_items, int32_t n_row_items, void* stream) {
  using namespace advopt;
  if (!L || !S || !L->tensors || !L->pieces || L->n_tensors <= 0 || L->n_pieces <= 0)
    return set_error(ADVOPT_E_INVALID, "advopt_spectral_step: null or empty launch");
  if ((n_col_items > 0 && !col_items) || (n_row_items > 0 && !row_items) || n_col_items < 0 || n_row_items < 0)
    return set_error(ADVOPT_E_INVALID, "advopt_spectral_step: null item list");
  if (L->flags & (ADVOPT_F_FISHER | ADVOPT_F_FISHER_STATS))
    return set_error(ADVOPT_E_INVALID, "advopt_spectral_step: Fisher weight decay is not supported here");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (n_col_items > 0) {
    spec_vpart_kernel<<<n_col_items, kSThreads, 0, s>>>(S, col_items);
    spec_vsum_kernel<<<dim3(kVsumBlocks, (unsigned)L->n_tensors), kVsumThreads, 0, s>>>(S);
  }
  spec_vfinish_kernel<<<L->n_tensors, 1024, 0, s>>>(S);
  if (n_row_items > 0) spec_rows_kernel<<<n_row_items, kSThreads, 0, s>>>(S, row_items);
  spec_ufinish_kernel<<<L->n_tensors, 1024, 0, s>>>(L->tensors, S);
  const bool pbf = L->param_dtype == ADVOPT_DT_BF16, nin = L->flags & ADVOPT_F_NOISE_IN;
  const unsigned ga = (unsigned)L->n_pieces * kApplySplit;
  if (pbf)
    nin ? spec_apply_kernel<true, true><<<ga, kThreads, 0, s>>>(*L, S)
        : spec_apply_kernel<true, false><<<ga, kThreads, 0, s>>>(*L, S);
  else
    nin ? spec_apply_kernel<false, true><<<ga, kThreads, 0, s>>>(*L, S)
        : spec_apply_kernel<false, false><<<ga, kThreads, 0, s>>>(*L, S);
  return check_cuda(cudaGetLastError(), "advopt_spectral_step");
}
