// Direct access to the counter-based generator the kernels draw their
// stochastic-rounding noise from (Philox4x32-10, Salmon et al., SC'11), for
// known-answer and distribution tests and for reproducing a step's noise.
#include "advopt.h"
#include "capi_internal.h"
#include "common.cuh"

namespace advopt {
namespace {

__global__ void philox_raw_kernel(const uint32_t* in, uint32_t* out, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint32_t* q = in + 6 * i;
  const U4 o = philox4x32_10(U4{q[0], q[1], q[2], q[3]}, q[4], q[5]);
  out[4 * i + 0] = o.x;
  out[4 * i + 1] = o.y;
  out[4 * i + 2] = o.z;
  out[4 * i + 3] = o.w;
}

__global__ void noise_kernel(uint16_t* out, int64_t n, uint64_t seed, uint32_t tensor_id, uint32_t step,
                             uint32_t stream) {
  const int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t k0 = g * 8;
  if (k0 >= n) return;
  uint32_t r[8];
  philox_u16x8(seed, tensor_id, step, stream, k0, r);
#pragma unroll
  for (int e = 0; e < 8; ++e)
    if (k0 + e < n) out[k0 + e] = (uint16_t)r[e];
}

}  // namespace
}  // namespace advopt

using namespace advopt;

extern "C" int advopt_philox4x32_10(const uint32_t* counters_keys, uint32_t* out, int64_t n, void* stream) {
  if (n < 0 || (n > 0 && (!counters_keys || !out))) return set_error(ADVOPT_E_INVALID, "advopt_philox4x32_10: bad arguments");
  if (n == 0) return ADVOPT_OK;
  const int64_t blocks = (n + 255) / 256;
  philox_raw_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(counters_keys, out, n);
  return check_cuda(cudaGetLastError(), "advopt_philox4x32_10");
}

extern "C" int advopt_noise_fill(uint16_t* out, int64_t n, uint64_t seed, uint32_t tensor_id, uint32_t step,
                                 uint32_t stream_id, void* stream) {
  if (n < 0 || (n > 0 && !out) || stream_id > 255) return set_error(ADVOPT_E_INVALID, "advopt_noise_fill: bad arguments");
  if (n == 0) return ADVOPT_OK;
  const int64_t groups = (n + 7) / 8;
  noise_kernel<<<(unsigned)((groups + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(out, n, seed, tensor_id,
                                                                                               step, stream_id);
  return check_cuda(cudaGetLastError(), "advopt_noise_fill");
}
