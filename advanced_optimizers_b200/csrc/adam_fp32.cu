// Adam-family kernels instantiated for state precision ADVOPT_PREC_FP32.
#include "adam_impl.cuh"

namespace advopt {
cudaError_t launch_adam_fp32(const advopt_adam_launch& L, cudaStream_t s) { return launch_adam_prec<ADVOPT_PREC_FP32>(L, s); }
cudaError_t occupancy_adam_fp32(int pdt, int algo, int smem_floats, int* ctas, int fast) {
  return occupancy_adam_prec<ADVOPT_PREC_FP32>(pdt, algo, smem_floats, ctas, fast);
}
}  // namespace advopt
