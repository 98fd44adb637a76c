// Error reporting shared by the C entry points.
#pragma once

#include <cuda_runtime.h>

#include "advopt.h"

namespace advopt {
// Records `msg` as the calling thread's last error and returns `code`.
int set_error(int code, const char* msg);
// ADVOPT_OK when e == cudaSuccess, else records "<where>: <cuda error>" and
// returns ADVOPT_E_CUDA.
int check_cuda(cudaError_t e, const char* where);

// Launch helpers shared by the C entry points (adam_api.cu).
cudaError_t run_adam(const advopt_adam_launch& L, cudaStream_t s);
cudaError_t run_occupancy(int prec, int pdt, int algo, int smem_floats, int* ctas, int fast);
cudaError_t run_factored_finish(const advopt_adam_tensor* tensors, const int32_t* index, int n_factored, int max_d2,
                                const int32_t* err, cudaStream_t s);
}  // namespace advopt
