// Host runtime behind the npl_* API: library state bound to one CUDA device,
// argument validation with the reference's error codes, and the per-call
// context that turns tensor descriptors into device pointers.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstddef>
#include <cstdint>
#include <mutex>
#include <vector>

#include "neural_primitives.h"
#include "npl_kernels.h"

namespace npl {

struct State {
  std::mutex mu;
  std::atomic<bool> initialized{false};  // read without the mutex by calls on any thread
  npl_config_t config{};
  int device = 0;
  cudaStream_t stream = nullptr;
  int concurrent_managed = 0;
  std::atomic<size_t> total_ops{0};
  std::atomic<size_t> total_fused{0};
};

State &state();

// Element count (product of shape) and the reference's tensor check
// (ValidateTensor, npl_tensor_ops.cpp:743-769): NULL descriptor, NULL data,
// ndim outside [1, 8], or a zero dimension -> NPL_ERR_INVALID_ARG with a
// message on stderr.
size_t element_count(const npl_tensor_t *t);
int validate_tensor(const npl_tensor_t *t, const char *name);

// True when NPL_TF32_FAST=1 selects one-pass TF32 for the dense contractions.
bool tf32_fast_mode();

// True when NPL_AUTOTUNE=1: npl_* calls tune a shape that has no entry in the
// tile-configuration cache (nplk_conv2d_tune / nplk_gemm_tune) on its first
// call.
bool autotune_mode();
// Whether the cache holds an entry for the conv geometry / GEMM shape.
bool conv_tuned(const nplk_conv_geom_t *g);
bool gemm_tuned(int64_t M, int64_t N, int64_t K);

// One API call: resolves tensor pointers to device memory on the library's
// device, stages plain host memory through the stream-ordered pool, times the
// launched kernels with CUDA events, copies staged outputs back, synchronises
// and reports kernel status.
class Call {
 public:
  Call();
  ~Call();
  Call(const Call &) = delete;
  Call &operator=(const Call &) = delete;

  int status() const { return status_; }
  cudaStream_t stream() const { return stream_; }

  // Device view of a tensor's first `bytes` bytes. Inputs are copied to the
  // device when staged; outputs are copied back by finish(). The same host
  // pointer seen twice in one call maps to the same device buffer, so
  // in-place operations work.
  float *input(const void *host_or_dev, size_t bytes);
  float *output(void *host_or_dev, size_t bytes, bool read_before_write = false);
  // Small parameter array (batch-norm statistics and the like), NULL stays NULL.
  const float *param(const float *p, size_t count);
  // Writable parameter array that must be copied back (running statistics).
  float *param_out(float *p, size_t count);
  // Device scratch for this call.
  void *scratch(size_t bytes);
  // Like scratch(), but an allocation failure returns nullptr without failing
  // the call (for callers with a path that needs no scratch).
  void *try_scratch(size_t bytes);

  void start_timer();
  void stop_timer();

  // Finishes the call; returns NPL_OK or an error. Fills stats if non-NULL.
  int finish(npl_perf_stats_t *stats, double flops, double bytes, const char *backend,
             int fused_ops = 0);

  // Records a kernel-launch error code (first one wins).
  void fail(int rc) {
    if (rc != 0 && status_ == 0) status_ = rc;
  }

 private:
  struct Buf {
    const void *user;
    void *dev;
    size_t bytes;
    bool staged;
    bool copy_back;
  };
  void *resolve(const void *p, size_t bytes, bool copy_in, bool copy_back);

  int status_ = 0;
  cudaStream_t stream_ = nullptr;
  std::vector<Buf> bufs_;
  std::vector<void *> scratch_;
  cudaEvent_t ev0_ = nullptr, ev1_ = nullptr;
  bool timed_ = false;
};

// Copy/compute overlap within one call: two auxiliary non-blocking streams
// (host-to-device and device-to-host copies) and a pool of events without
// timing, created once per thread for the library's device.
struct CopyLanes {
  cudaStream_t in = nullptr;
  cudaStream_t out = nullptr;
  std::vector<cudaEvent_t> events;
};
// The calling thread's lanes with at least `events` events, or NULL on error.
// Leaves the library's device current.
CopyLanes *copy_lanes(size_t events);
// True for page-locked host memory (asynchronous copies overlap compute).
bool is_pinned_host(const void *p);

// Reference-compatible helpers shared by several operators.
int validate_conv_params(const npl_conv_params_t *p);

}  // namespace npl
