// Peer buffers for the multi-GPU paths: CUDA IPC handles of device memory,
// exchanged by the caller between ranks (one process per GPU) and opened here
// so that a kernel on this GPU can store into another GPU's buffer over
// NVLink. A handle names a whole allocation, so the pointer's offset inside
// its allocation travels with it (framework tensors are sub-allocations).
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstring>

#include "nplk_host.h"

namespace nplk {
namespace {

PFN_cuMemGetAddressRange_v3020 address_range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<PFN_cuMemGetAddressRange_v3020>(nullptr);
    return reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  }();
  return fn;
}

}  // namespace
}  // namespace nplk

using namespace nplk;

extern "C" size_t nplk_ipc_handle_size(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int nplk_ipc_get_handle(const void *dev_ptr, void *handle, uint64_t *offset) {
  if (!dev_ptr || !handle || !offset) return kErrInvalidArg;
  auto range = address_range_fn();
  if (!range) return kErrInternal;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(dev_ptr)) != CUDA_SUCCESS)
    return kErrInvalidArg;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
  if (e != cudaSuccess) return map_cuda_error(e);
  std::memcpy(handle, &h, sizeof(h));
  *offset = static_cast<uint64_t>(reinterpret_cast<CUdeviceptr>(dev_ptr) - base);
  return kOk;
}

extern "C" int nplk_ipc_open_handle(const void *handle, uint64_t offset, void **dev_ptr) {
  if (!handle || !dev_ptr) return kErrInvalidArg;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void *base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return map_cuda_error(e);
  *dev_ptr = static_cast<uint8_t *>(base) + offset;
  return kOk;
}

extern "C" int nplk_ipc_close_handle(void *dev_ptr, uint64_t offset) {
  if (!dev_ptr) return kErrInvalidArg;
  const cudaError_t e = cudaIpcCloseMemHandle(static_cast<uint8_t *>(dev_ptr) - offset);
  return e == cudaSuccess ? kOk : map_cuda_error(e);
}
