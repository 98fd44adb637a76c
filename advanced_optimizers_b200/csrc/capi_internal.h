// Error reporting shared by the C entry points.
#pragma once

#include <cuda_runtime.h>

namespace advopt {
// Records `msg` as the calling thread's last error and returns `code`.
int set_error(int code, const char* msg);
// ADVOPT_OK when e == cudaSuccess, else records "<where>: <cuda error>" and
// returns ADVOPT_E_CUDA.
int check_cuda(cudaError_t e, const char* where);
}  // namespace advopt
