// Peer copies for the sharded parameter gather: device memory of another
// rank (opened through a CUDA IPC handle) read by this GPU's copy engines,
// so the gather takes no SMs from the step's kernels.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "advopt.h"
#include "capi_internal.h"

using namespace advopt;

static PFN_cuMemGetAddressRange_v3020 g_range = nullptr;
static std::once_flag g_range_once;

extern "C" int advopt_ipc_get_handle(const void* ptr, void* handle_out, uint64_t* offset_out) {
  if (!ptr || !handle_out || !offset_out) return set_error(ADVOPT_E_INVALID, "advopt_ipc_get_handle: null argument");
  // the handle names the whole allocation: report where ptr sits inside it
  std::call_once(g_range_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_range = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
  });
  if (!g_range) return set_error(ADVOPT_E_CUDA, "advopt_ipc_get_handle: cuMemGetAddressRange is unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (g_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return set_error(ADVOPT_E_CUDA, "advopt_ipc_get_handle: cuMemGetAddressRange failed");
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return check_cuda(e, "advopt_ipc_get_handle");
  std::memcpy(handle_out, &h, sizeof(h));
  *offset_out = reinterpret_cast<uint64_t>(ptr) - static_cast<uint64_t>(base);
  return ADVOPT_OK;
}

extern "C" int advopt_ipc_open(const void* handle, void** base_out) {
  if (!handle || !base_out) return set_error(ADVOPT_E_INVALID, "advopt_ipc_open: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return check_cuda(cudaIpcOpenMemHandle(base_out, h, cudaIpcMemLazyEnablePeerAccess), "advopt_ipc_open");
}

extern "C" int advopt_ipc_close(void* base) {
  if (!base) return ADVOPT_OK;
  return check_cuda(cudaIpcCloseMemHandle(base), "advopt_ipc_close");
}

extern "C" int advopt_enable_peer(int32_t peer_device) {
  const cudaError_t e = cudaDeviceEnablePeerAccess(peer_device, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();
    return ADVOPT_OK;
  }
  return check_cuda(e, "advopt_enable_peer");
}

extern "C" int advopt_copy_async(void* dst, const void* src, uint64_t bytes, void* stream) {
  if (bytes == 0) return ADVOPT_OK;
  if (!dst || !src) return set_error(ADVOPT_E_INVALID, "advopt_copy_async: null pointer");
  return check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream)),
                    "advopt_copy_async");
}
