// C entry points that are not kernels: error state, ABI/layout queries.
#include <cstdio>
#include <cstring>

#include "advopt.h"
#include "capi_internal.h"

namespace advopt {
static thread_local char g_last_error[512] = "";

int set_error(int code, const char* msg) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s", msg);
  return code;
}

int check_cuda(cudaError_t e, const char* where) {
  if (e == cudaSuccess) return ADVOPT_OK;
  std::snprintf(g_last_error, sizeof(g_last_error), "%s: %s (%s)", where, cudaGetErrorString(e), cudaGetErrorName(e));
  return ADVOPT_E_CUDA;
}
}  // namespace advopt

extern "C" const char* advopt_last_error(void) { return advopt::g_last_error; }

extern "C" int advopt_abi_version(void) { return ADVOPT_ABI_VERSION; }

extern "C" size_t advopt_sizeof(int which) {
  switch (which) {
    case 0: return sizeof(advopt_adam_tensor);
    case 1: return sizeof(advopt_piece);
    case 2: return sizeof(advopt_adam_launch);
    case 3: return sizeof(advopt_lion_tensor);
    case 4: return sizeof(advopt_muon_args);
    case 5: return sizeof(advopt_kourkoutas_args);
    case 6: return sizeof(advopt_prodigy_dev);
    case 7: return sizeof(advopt_prodigy_scalar_args);
    case 8: return sizeof(advopt_prodigy_d_args);
    case 9: return sizeof(advopt_spectral_tensor);
    default: return 0;
  }
}
