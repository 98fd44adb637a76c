// Low-rank Newton–Schulz for Muon_adv / AdaMuon_adv (Muon_util.py:239-270):
//
//   MG = M @ S          S: Gaussian sketch [cols][r], M the [rows][cols] update
//   Q  = qr(MG).Q       in float32 by the reference; here shifted CholeskyQR3 in
//                       float64 (Fukaya, Kannan, Nakatsukasa, Yamamoto and
//                       Yanagisawa, "Shifted Cholesky QR for computing the QR
//                       factorization of ill-conditioned matrices", SIAM J. Sci.
//                       Comput. 42 (2020)), then cast to the update's dtype
//   P  = Q^T @ M        [r][cols], orthogonalised by the ordinary chain
//   U  = Q @ NS(P)      [rows][cols]
//
// QR is unique up to the signs of Q's columns, and U does not depend on them:
// with Q' = Q D (D diagonal, entries +-1), NS(D P) = D NS(P) because every
// iteration is a polynomial in P P^T applied to P, so Q' NS(Q'^T M) = Q NS(P).
//
// The three products are thin (one dimension is r <= a few hundred) and take
// under 2 r / min(rows, cols) of the full chain's FLOPs; they run as tiled
// SIMT kernels with float32 accumulation and one rounding of the output, as
// torch's bf16 matmul does.  The sketch is drawn from Philox4x32-10 with the
// Box–Muller transform (the reference draws torch.randn from its own
// generator; the test mode injects the reference's sketch instead).
#include <math.h>

#include "advopt.h"
#include "capi_internal.h"
#include "common.cuh"

namespace advopt {
namespace lowrank {

constexpr int kTM = 64, kTN = 64, kTK = 16;   // output tile and k step of the products

// D[M][N] = bf16(sum_k opA[m][k] * B[k][n]); opA = A [M][K] (row-major) or,
// with TRANS_A, A^T with A stored [K][M].  B is [K][N] row-major.  256
// threads, each 4 x 4 outputs.
template <bool TRANS_A>
__global__ void __launch_bounds__(256) gemm_kernel(uint16_t* __restrict__ D, const uint16_t* __restrict__ A,
                                                  const uint16_t* __restrict__ B, int64_t M, int64_t N, int64_t K) {
  __shared__ float As[kTK][kTM + 4];
  __shared__ float Bs[kTK][kTN + 4];
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  const int64_t m0 = (int64_t)blockIdx.y * kTM, n0 = (int64_t)blockIdx.x * kTN;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
  for (int64_t k0 = 0; k0 < K; k0 += kTK) {
    // 16 x 64 elements of each operand: 4 per thread
    for (int t = threadIdx.x; t < kTK * kTM; t += 256) {
      int kk, mm;
      if (TRANS_A) { kk = t / kTM; mm = t % kTM; } else { mm = t / kTK; kk = t % kTK; }
      const int64_t gm = m0 + mm, gk = k0 + kk;
      float v = 0.0f;
      if (gm < M && gk < K) v = bf16_to_f(TRANS_A ? A[gk * M + gm] : A[gm * K + gk]);
      As[kk][mm] = v;
    }
    for (int t = threadIdx.x; t < kTK * kTN; t += 256) {
      const int kk = t / kTN, nn = t % kTN;
      const int64_t gk = k0 + kk, gn = n0 + nn;
      Bs[kk][nn] = (gk < K && gn < N) ? bf16_to_f(B[gk * N + gn]) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kTK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t gm = m0 + ty * 4 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t gn = n0 + tx * 4 + j;
      if (gn < N) D[gm * N + gn] = (uint16_t)f_to_bf16_rne(acc[i][j]);
    }
  }
}

// ---- shifted CholeskyQR3 in float64 on A [m][r] ----
constexpr int kGramSplit = 32;   // row ranges of the Gram partial sums

// Gram partials: part[s][i][j] = sum over rows of range s of A[row][i] * A[row][j]
// (i <= j computed, both halves written).  Grid (ceil(r/16)^2, kGramSplit), 16 x 16 threads.
__global__ void __launch_bounds__(256) gram_kernel(const double* __restrict__ A, double* __restrict__ part,
                                                  int64_t m, int64_t r) {
  const int tiles = (int)((r + 15) / 16);
  const int ti = blockIdx.x / tiles, tj = blockIdx.x % tiles;
  const int64_t i = (int64_t)ti * 16 + (threadIdx.x >> 4), j = (int64_t)tj * 16 + (threadIdx.x & 15);
  const int s = blockIdx.y;
  const int64_t r0 = m * s / kGramSplit, r1 = m * (s + 1) / kGramSplit;
  if (i >= r || j >= r || j < i) return;
  double acc = 0.0;
  for (int64_t row = r0; row < r1; ++row) acc = fma(A[row * r + i], A[row * r + j], acc);
  part[((int64_t)s * r + i) * r + j] = acc;
  part[((int64_t)s * r + j) * r + i] = acc;
}

// G = sum of the partials (+ shift on the diagonal), then its Cholesky factor
// in place (lower triangle of G holds L, G = L L^T).  One CTA of 1024.  A
// non-positive pivot (a rank-deficient A after the shifted pass) leaves its
// column of L zero and the solve below leaves that column of Q zero.
__global__ void __launch_bounds__(1024) chol_kernel(const double* __restrict__ part, double* __restrict__ G,
                                                   int64_t m, int64_t r, int shifted) {
  __shared__ double shift_s;
  const int64_t rr = r * r;
  for (int64_t t = threadIdx.x; t < rr; t += blockDim.x) {
    double s = 0.0;
    for (int sp = 0; sp < kGramSplit; ++sp) s += part[(int64_t)sp * rr + t];
    G[t] = s;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // s = 11 (m r + r (r + 1)) u ||A||^2, ||A||_2^2 <= trace(A^T A)
    double tr = 0.0;
    for (int64_t i = 0; i < r; ++i) tr += G[i * r + i];
    shift_s = shifted ? 11.0 * ((double)m * (double)r + (double)r * (double)(r + 1)) * 0x1p-53 * tr : 0.0;
  }
  __syncthreads();
  for (int64_t i = threadIdx.x; i < r; i += blockDim.x) G[i * r + i] += shift_s;
  __syncthreads();
  for (int64_t k = 0; k < r; ++k) {
    __shared__ double dk;
    if (threadIdx.x == 0) {
      const double a = G[k * r + k];
      dk = a > 0.0 ? sqrt(a) : 0.0;
      G[k * r + k] = dk;
    }
    __syncthreads();
    const double d = dk;
    for (int64_t i = k + 1 + threadIdx.x; i < r; i += blockDim.x) G[i * r + k] = d > 0.0 ? G[i * r + k] / d : 0.0;
    __syncthreads();
    // trailing update of the lower triangle: G[i][j] -= L[i][k] L[j][k], j <= i
    const int64_t n = r - k - 1;
    for (int64_t t = threadIdx.x; t < n * n; t += blockDim.x) {
      const int64_t i = k + 1 + t / n, j = k + 1 + t % n;
      if (j <= i) G[i * r + j] -= G[i * r + k] * G[j * r + k];
    }
    __syncthreads();
  }
}

// Q = A L^{-T} row by row (forward substitution q L^T = a), one thread per row.
__global__ void __launch_bounds__(256) solve_kernel(double* __restrict__ A, const double* __restrict__ L,
                                                   int64_t m, int64_t r) {
  const int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= m) return;
  double* a = A + row * r;
  for (int64_t j = 0; j < r; ++j) {
    double s = a[j];
    for (int64_t i = 0; i < j; ++i) s -= a[i] * L[j * r + i];
    const double d = L[j * r + j];
    a[j] = d > 0.0 ? s / d : 0.0;
  }
}

__global__ void widen_kernel(double* __restrict__ out, const uint16_t* __restrict__ in, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = (double)bf16_to_f(in[i]);
}

// float64 -> float32 (QR's dtype in the reference) -> bf16 (the update's)
__global__ void narrow_kernel(uint16_t* __restrict__ out, const double* __restrict__ in, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = (uint16_t)f_to_bf16_rne((float)in[i]);
}

// Gaussian sketch [n][r] in bf16: element e of the flat array takes the
// Box–Muller pair of Philox word pair (e >> 1) of counter (e >> 2, stream
// kNoiseAux << 24 | 1, tensor_id, step).
__global__ void sketch_kernel(uint16_t* __restrict__ S, int64_t count, uint64_t seed, uint32_t tensor_id,
                              uint32_t step) {
  for (int64_t q = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; q * 4 < count;
       q += (int64_t)gridDim.x * blockDim.x) {
    const U4 w = philox4x32_10(U4{(uint32_t)q, ((uint32_t)kNoiseAux << 24) | 1u, tensor_id, step}, (uint32_t)seed,
                               (uint32_t)(seed >> 32));
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      // u1 in (0, 1], u2 in [0, 1): 24-bit uniforms
      const float u1 = ((float)(words[2 * h] >> 8) + 1.0f) * 0x1p-24f;
      const float u2 = (float)(words[2 * h + 1] >> 8) * 0x1p-24f;
      const float rad = sqrtf(-2.0f * logf(u1));
      float sn, cs;
      sincospif(2.0f * u2, &sn, &cs);
      const int64_t e = q * 4 + 2 * h;
      if (e < count) S[e] = (uint16_t)f_to_bf16_rne(rad * cs);
      if (e + 1 < count) S[e + 1] = (uint16_t)f_to_bf16_rne(rad * sn);
    }
  }
}

}  // namespace lowrank
}  // namespace advopt

using namespace advopt;
using namespace advopt::lowrank;

static unsigned lr_grid(int64_t n, int per = 256) {
  const int64_t g = (n + per - 1) / per;
  return (unsigned)(g < 1 ? 1 : (g > 65535 * 4 ? 65535 * 4 : g));
}

extern "C" int advopt_lr_gemm(uint16_t* D, const uint16_t* A, const uint16_t* B, int64_t M, int64_t N, int64_t K,
                              int32_t trans_a, void* stream) {
  if (!D || !A || !B || M <= 0 || N <= 0 || K <= 0) return set_error(ADVOPT_E_INVALID, "advopt_lr_gemm: bad argument");
  if ((M + kTM - 1) / kTM > 65535) return set_error(ADVOPT_E_INVALID, "advopt_lr_gemm: M too large");
  const dim3 grid((unsigned)((N + kTN - 1) / kTN), (unsigned)((M + kTM - 1) / kTM));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (trans_a) gemm_kernel<true><<<grid, 256, 0, s>>>(D, A, B, M, N, K);
  else gemm_kernel<false><<<grid, 256, 0, s>>>(D, A, B, M, N, K);
  return check_cuda(cudaGetLastError(), "advopt_lr_gemm");
}

extern "C" int64_t advopt_lr_qr_work(int64_t m, int64_t r) {
  return m * r + (int64_t)kGramSplit * r * r + r * r;
}

extern "C" int advopt_lr_qr(uint16_t* Q, const uint16_t* A, int64_t m, int64_t r, double* work, void* stream) {
  if (!Q || !A || !work || m <= 0 || r <= 0 || r > m) return set_error(ADVOPT_E_INVALID, "advopt_lr_qr: bad argument");
  const int64_t tiles = (r + 15) / 16;
  if (tiles * tiles > 65535) return set_error(ADVOPT_E_INVALID, "advopt_lr_qr: rank too large");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  double* Ad = work;
  double* part = work + m * r;
  double* G = part + (int64_t)kGramSplit * r * r;
  widen_kernel<<<lr_grid(m * r), 256, 0, s>>>(Ad, A, m * r);
  for (int pass = 0; pass < 3; ++pass) {
    gram_kernel<<<dim3((unsigned)(tiles * tiles), kGramSplit), 256, 0, s>>>(Ad, part, m, r);
    chol_kernel<<<1, 1024, 0, s>>>(part, G, m, r, pass == 0 ? 1 : 0);
    solve_kernel<<<lr_grid(m), 256, 0, s>>>(Ad, G, m, r);
  }
  narrow_kernel<<<lr_grid(m * r), 256, 0, s>>>(Q, Ad, m * r);
  return check_cuda(cudaGetLastError(), "advopt_lr_qr");
}

extern "C" int advopt_lr_sketch(uint16_t* S, int64_t n, int64_t r, uint64_t seed, uint32_t tensor_id, uint32_t step,
                                void* stream) {
  if (!S || n <= 0 || r <= 0) return set_error(ADVOPT_E_INVALID, "advopt_lr_sketch: bad argument");
  const int64_t count = n * r;
  sketch_kernel<<<lr_grid((count + 3) / 4), 256, 0, static_cast<cudaStream_t>(stream)>>>(S, count, seed, tensor_id,
                                                                                          step);
  return check_cuda(cudaGetLastError(), "advopt_lr_sketch");
}
