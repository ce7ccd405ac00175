// Fused conv2d + bias + BN + activation for callers that cannot allocate
// device memory.
//
// The regular entry point (nplk_conv2d_fused) needs a caller-provided device
// workspace for the tf32-split weights and the per-channel epilogue
// constants. Some callers cannot make that allocation: hosts that reserve
// their whole device-memory budget at start-up and must not grow it while
// serving a request, code running inside another allocator's callback, and
// foreign-language callers that must avoid cudaMalloc/cudaFree because those
// calls can synchronise the whole device. This variant keeps that workspace in
// a fixed array in the library's own device memory instead.
//
// Properties a caller must know:
//   * Capacity: the array holds kNoAllocScratchBytes (8 MiB). Geometries whose
//     minimum workspace (split weights + epilogue constants) would exceed it
//     are rejected with NPL_ERR_UNSUPPORTED and a message on stderr. When the
//     full workspace (which adds the NHWC input planes) does not fit, the
//     conv runs on the direct-gather kernel, with identical results.
//   * Footprint: every GPU on which the library is loaded keeps the 8 MiB
//     (plus one status word) until the process exits.
//   * Set-up: the first call on each device looks up the array's device
//     address (cudaGetSymbolAddress) with that device current. That first
//     call should therefore come before any stream capture.
//   * Status: with status == NULL the kernels report a bounded-wait timeout
//     to a word kept beside the array; nplk_read_status() reads and clears it
//     (together with the library's other status word) without allocating.
//     Each call clears that word before its kernels run, so read it after
//     every call whose outcome matters.
//   * Sharing: all calls on a device use the same array, which keeps whatever
//     the last call wrote. Each call rewrites every byte it later reads, and
//     clears the status word it uses, before its kernels run. Calls whose
//     execution overlaps on the GPU (different streams, no ordering between
//     them) race on the array and produce undefined results.
//   * Nothing here allocates: no cudaMalloc, cudaFree or allocating library
//     routine is called.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "nplk_host.h"

namespace nplk {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
static __device__ __align__(256) int g_noalloc_status;

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void *g_scratch_ptr[kMaxDevices];
int *g_status_ptr[kMaxDevices];

// Device addresses of the static arrays for the current device (looked up
// once per device).
int noalloc_setup(void **scratch, int **status) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return kErrInternal;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_scratch_ptr[dev]) {
    void *p = nullptr;
    int *q = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      std::fprintf(stderr, "[NPL] no-alloc conv: cudaGetSymbolAddress(scratch) failed: %s\n",
                   cudaGetErrorString(e));
      return map_cuda_error(e);
    }
    e = cudaGetSymbolAddress(reinterpret_cast<void **>(&q), g_noalloc_status);
    if (e != cudaSuccess) {
      std::fprintf(stderr, "[NPL] no-alloc conv: cudaGetSymbolAddress(status) failed: %s\n",
                   cudaGetErrorString(e));
      return map_cuda_error(e);
    }
    g_scratch_ptr[dev] = p;
    g_status_ptr[dev] = q;
  }
  *scratch = g_scratch_ptr[dev];
  *status = g_status_ptr[dev];
  return kOk;
}

}  // namespace

int *noalloc_status_word_if_set_up() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  return g_status_ptr[dev];
}

}  // namespace nplk

using namespace nplk;

extern "C" int nplk_conv2d_fused_noalloc(void *stream, const nplk_conv_geom_t *g,
                                         const float *x, const float *w, const float *bias,
                                         const float *bn_mean, const float *bn_var,
                                         const float *bn_gamma, const float *bn_beta,
                                         float bn_eps, int act, float act_alpha, float *out,
                                         int *status) {
  if (!g || !x || !w || !out) return kErrInvalidArg;
  const size_t need = nplk_conv_workspace_min_size(g);
  if (need == 0) return kErrInvalidArg;
  if (need > kNoAllocScratchBytes) {
    std::fprintf(stderr,
                 "[NPL] no-alloc conv: this geometry needs %zu bytes of scratch; the "
                 "no-allocation entry point holds %zu (use nplk_conv2d_fused with a "
                 "caller workspace)\n",
                 need, kNoAllocScratchBytes);
    return kErrUnsupported;
  }
  void *scratch = nullptr;
  int *own_status = nullptr;
  int rc = noalloc_setup(&scratch, &own_status);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (!status) {
    status = own_status;
    if (cudaMemsetAsync(status, 0, sizeof(int), s) != cudaSuccess) return launch_result();
  }
  rc = nplk_conv2d_prepare(stream, g, w, bias, bn_mean, bn_var, bn_gamma, bn_beta, bn_eps,
                           scratch, kNoAllocScratchBytes);
  if (rc) return rc;
  return nplk_conv2d_run(stream, g, x, act, act_alpha, out, scratch, kNoAllocScratchBytes,
                         status);
}
