// Adam-family kernels instantiated for state precision ADVOPT_PREC_BF16_SR.
#include "adam_impl.cuh"

namespace advopt {
cudaError_t launch_adam_bf16sr(const advopt_adam_launch& L, cudaStream_t s) { return launch_adam_prec<ADVOPT_PREC_BF16_SR>(L, s); }
cudaError_t occupancy_adam_bf16sr(int pdt, int algo, int smem_floats, int* ctas, int fast) {
  return occupancy_adam_prec<ADVOPT_PREC_BF16_SR>(pdt, algo, smem_floats, ctas, fast);
}
}  // namespace advopt
