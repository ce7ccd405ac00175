// Host runtime for the npl_* API (see npl_runtime.h).
#include "npl_runtime.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>

namespace nplk {
int *device_status_word();
}

namespace npl {

State &state() {
  static State s;
  return s;
}

size_t element_count(const npl_tensor_t *t) {
  size_t n = 1;
  for (size_t i = 0; i < t->ndim; ++i) n *= t->shape[i];
  return n;
}

int validate_tensor(const npl_tensor_t *t, const char *name) {
  if (!t) {
    std::fprintf(stderr, "[NPL] Error: %s tensor is NULL\n", name);
    return NPL_ERR_INVALID_ARG;
  }
  if (!t->data) {
    std::fprintf(stderr, "[NPL] Error: %s tensor data is NULL\n", name);
    return NPL_ERR_INVALID_ARG;
  }
  if (t->ndim == 0 || t->ndim > NPL_MAX_DIMS) {
    std::fprintf(stderr, "[NPL] Error: %s tensor has invalid ndim: %zu\n", name, t->ndim);
    return NPL_ERR_INVALID_ARG;
  }
  for (size_t i = 0; i < t->ndim; ++i) {
    if (t->shape[i] == 0) {
      std::fprintf(stderr, "[NPL] Error: %s tensor has zero dimension at axis %zu\n", name, i);
      return NPL_ERR_INVALID_ARG;
    }
  }
  return NPL_OK;
}

bool tf32_fast_mode() {
  const char *e = std::getenv("NPL_TF32_FAST");
  return e && e[0] == '1';
}

bool autotune_mode() {
  const char *e = std::getenv("NPL_AUTOTUNE");
  return e && e[0] == '1';
}

bool conv_tuned(const nplk_conv_geom_t *g) {
  char key[256];
  nplk_tuning_key_conv(g, key, sizeof(key));
  return nplk_tuning_cache_get(key, nullptr, nullptr) == 1;
}

bool gemm_tuned(int64_t M, int64_t N, int64_t K) {
  char key[256];
  nplk_tuning_key_gemm(M, N, K, key, sizeof(key));
  return nplk_tuning_cache_get(key, nullptr, nullptr) == 1;
}

int validate_conv_params(const npl_conv_params_t *p) {
  // ValidateConvParams, npl_convolution.cpp:1347-1365.
  if (!p) return NPL_ERR_INVALID_ARG;
  if (p->kernel_h == 0 || p->kernel_w == 0) return NPL_ERR_INVALID_ARG;
  if (p->stride_h == 0 || p->stride_w == 0) return NPL_ERR_INVALID_ARG;
  if (p->groups == 0) return NPL_ERR_INVALID_ARG;
  return NPL_OK;
}

namespace {

struct ThreadEvents {
  int device = -1;
  cudaEvent_t a = nullptr, b = nullptr;
  int *pinned_status = nullptr;
};
thread_local ThreadEvents t_ev;

int map_err(cudaError_t e) {
  if (e == cudaSuccess) return NPL_OK;
  if (e == cudaErrorMemoryAllocation) return NPL_ERR_OOM;
  return NPL_ERR_INTERNAL;
}

// Fault injection (nplk_debug_fail_next_allocations): allocations still to
// fail as out of memory.
std::atomic<int> g_fail_allocs{0};

// cudaMallocAsync, or an injected out-of-memory failure.
cudaError_t device_alloc(void **p, size_t bytes, cudaStream_t s) {
  int n = g_fail_allocs.load(std::memory_order_relaxed);
  while (n > 0) {
    if (g_fail_allocs.compare_exchange_weak(n, n - 1)) return cudaErrorMemoryAllocation;
  }
  return cudaMallocAsync(p, bytes, s);
}

// Kept for the thread's lifetime (no destructor: CUDA may already be shut
// down when thread-local objects die at process exit).
struct ThreadLanes {
  int device = -1;
  CopyLanes lanes;
  void release() {
    if (device < 0) return;
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(device);
    for (cudaEvent_t e : lanes.events) cudaEventDestroy(e);
    if (lanes.in) cudaStreamDestroy(lanes.in);
    if (lanes.out) cudaStreamDestroy(lanes.out);
    cudaSetDevice(cur);
    lanes = CopyLanes{};
    device = -1;
  }
};
thread_local ThreadLanes t_lanes;

}  // namespace

CopyLanes *copy_lanes(size_t events) {
  const int dev = state().device;
  // Streams and events belong to the current device: make it the library's
  // (a thread's first call may come with another device current).
  if (cudaSetDevice(dev) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (t_lanes.device != dev) {
    t_lanes.release();
    if (cudaStreamCreateWithFlags(&t_lanes.lanes.in, cudaStreamNonBlocking) != cudaSuccess ||
        cudaStreamCreateWithFlags(&t_lanes.lanes.out, cudaStreamNonBlocking) != cudaSuccess) {
      cudaGetLastError();
      t_lanes.device = dev;
      t_lanes.release();
      return nullptr;
    }
    t_lanes.device = dev;
  }
  while (t_lanes.lanes.events.size() < events) {
    cudaEvent_t e = nullptr;
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    t_lanes.lanes.events.push_back(e);
  }
  return &t_lanes.lanes;
}

bool is_pinned_host(const void *p) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return a.type == cudaMemoryTypeHost;
}

Call::Call() {
  State &s = state();
  if (!s.initialized) {
    status_ = NPL_ERR_NOT_INITIALIZED;
    return;
  }
  if (cudaSetDevice(s.device) != cudaSuccess) {
    status_ = NPL_ERR_INTERNAL;
    return;
  }
  stream_ = s.stream;
  if (t_ev.device != s.device) {
    if (t_ev.a) cudaEventDestroy(t_ev.a);
    if (t_ev.b) cudaEventDestroy(t_ev.b);
    if (t_ev.pinned_status) cudaFreeHost(t_ev.pinned_status);
    t_ev = ThreadEvents{};
    if (cudaEventCreate(&t_ev.a) != cudaSuccess || cudaEventCreate(&t_ev.b) != cudaSuccess ||
        cudaMallocHost(reinterpret_cast<void **>(&t_ev.pinned_status), sizeof(int)) !=
            cudaSuccess) {
      status_ = NPL_ERR_INTERNAL;
      return;
    }
    t_ev.device = s.device;
  }
  ev0_ = t_ev.a;
  ev1_ = t_ev.b;
}

Call::~Call() {
  // finish() normally releases everything; this covers early error returns.
  for (auto &b : bufs_)
    if (b.staged && b.dev) cudaFreeAsync(b.dev, stream_);
  for (void *p : scratch_) cudaFreeAsync(p, stream_);
  if (!bufs_.empty() || !scratch_.empty()) cudaStreamSynchronize(stream_);
}

void *Call::resolve(const void *p, size_t bytes, bool copy_in, bool copy_back) {
  if (!p || status_) return nullptr;
  for (auto &b : bufs_) {
    if (b.user == p) {
      if (bytes > b.bytes) {
        fail(NPL_ERR_INTERNAL);
        return nullptr;
      }
      b.copy_back = b.copy_back || copy_back;
      return b.dev;
    }
  }
  cudaPointerAttributes a{};
  cudaError_t e = cudaPointerGetAttributes(&a, p);
  if (e != cudaSuccess) {
    cudaGetLastError();
    a.type = cudaMemoryTypeUnregistered;
  }
  Buf b{p, nullptr, bytes, false, false};
  if (a.type == cudaMemoryTypeDevice) {
    if (a.device != state().device) {
      std::fprintf(stderr, "[NPL] Error: tensor lives on device %d, library is bound to %d\n",
                   a.device, state().device);
      fail(NPL_ERR_INVALID_ARG);
      return nullptr;
    }
    b.dev = const_cast<void *>(p);
  } else if (a.type == cudaMemoryTypeManaged) {
    b.dev = const_cast<void *>(p);
    if (state().concurrent_managed) {
#if CUDART_VERSION >= 13000
      cudaMemLocation loc{cudaMemLocationTypeDevice, state().device};
      cudaMemPrefetchAsync(p, bytes, loc, 0, stream_);
#else
      cudaMemPrefetchAsync(p, bytes, state().device, stream_);
#endif
      cudaGetLastError();
    }
  } else {
    // Plain or pinned host memory: stage through the device pool.
    e = device_alloc(&b.dev, bytes, stream_);
    if (e != cudaSuccess) {
      fail(map_err(e));
      return nullptr;
    }
    b.staged = true;
    b.copy_back = copy_back;
    if (copy_in) {
      e = cudaMemcpyAsync(b.dev, p, bytes, cudaMemcpyHostToDevice, stream_);
      if (e != cudaSuccess) {
        cudaFreeAsync(b.dev, stream_);
        fail(map_err(e));
        return nullptr;
      }
    }
  }
  bufs_.push_back(b);
  return b.dev;
}

float *Call::input(const void *p, size_t bytes) {
  return static_cast<float *>(resolve(p, bytes, true, false));
}

float *Call::output(void *p, size_t bytes, bool read_before_write) {
  return static_cast<float *>(resolve(p, bytes, read_before_write, true));
}

const float *Call::param(const float *p, size_t count) {
  if (!p) return nullptr;
  return static_cast<const float *>(resolve(p, count * sizeof(float), true, false));
}

float *Call::param_out(float *p, size_t count) {
  if (!p) return nullptr;
  return static_cast<float *>(resolve(p, count * sizeof(float), true, true));
}

void *Call::scratch(size_t bytes) {
  if (status_) return nullptr;
  void *d = nullptr;
  cudaError_t e = device_alloc(&d, bytes < 256 ? 256 : bytes, stream_);
  if (e != cudaSuccess) {
    fail(map_err(e));
    return nullptr;
  }
  scratch_.push_back(d);
  return d;
}

void *Call::try_scratch(size_t bytes) {
  if (status_) return nullptr;
  void *d = nullptr;
  if (device_alloc(&d, bytes < 256 ? 256 : bytes, stream_) != cudaSuccess) {
    cudaGetLastError();  // an allocation failure is not sticky; clear it
    return nullptr;
  }
  scratch_.push_back(d);
  return d;
}

void Call::start_timer() {
  if (!status_ && cudaEventRecord(ev0_, stream_) == cudaSuccess) timed_ = true;
}

void Call::stop_timer() {
  if (timed_ && cudaEventRecord(ev1_, stream_) != cudaSuccess) timed_ = false;
}

int Call::finish(npl_perf_stats_t *stats, double flops, double bytes, const char *backend,
                 int fused_ops) {
  int *dev_status = nplk::device_status_word();
  if (!status_ && dev_status) {
    // Kernel status word -> pinned host int, then clear it, in stream order.
    *t_ev.pinned_status = 0;
    if (cudaMemcpyAsync(t_ev.pinned_status, dev_status, sizeof(int), cudaMemcpyDeviceToHost,
                        stream_) != cudaSuccess ||
        cudaMemsetAsync(dev_status, 0, sizeof(int), stream_) != cudaSuccess)
      fail(NPL_ERR_INTERNAL);
  }
  if (!status_) {
    for (auto &b : bufs_) {
      if (b.staged && b.copy_back) {
        cudaError_t e = cudaMemcpyAsync(const_cast<void *>(b.user), b.dev, b.bytes,
                                        cudaMemcpyDeviceToHost, stream_);
        if (e != cudaSuccess) {
          fail(map_err(e));
          break;
        }
      }
    }
  }
  for (auto &b : bufs_)
    if (b.staged && b.dev) cudaFreeAsync(b.dev, stream_);
  for (void *p : scratch_) cudaFreeAsync(p, stream_);
  bufs_.clear();
  scratch_.clear();
  cudaError_t e = cudaStreamSynchronize(stream_);
  if (e != cudaSuccess) fail(map_err(e));
  e = cudaGetLastError();
  if (e != cudaSuccess) fail(map_err(e));
  if (!status_ && dev_status && *t_ev.pinned_status != 0) {
    std::fprintf(stderr, "[NPL] Error: kernel pipeline wait expired (status %d)\n",
                 *t_ev.pinned_status);
    fail(NPL_ERR_INTERNAL);
  }
  float ms = 0.0f;
  if (timed_ && !status_) cudaEventElapsedTime(&ms, ev0_, ev1_);
  if (stats) {
    stats->elapsed_ms = ms;
    stats->gflops = (ms > 0.0f && flops > 0.0) ? flops / 1e9 / (ms / 1e3) : 0.0;
    stats->bandwidth_gbps = (ms > 0.0f && bytes > 0.0) ? bytes / 1e9 / (ms / 1e3) : 0.0;
    stats->operations_fused = fused_ops > 1 ? static_cast<size_t>(fused_ops) : 0;
    stats->memory_saved_bytes = 0;
    stats->backend_used = backend;
    stats->was_fused = fused_ops > 1 ? 1 : 0;
  }
  if (!status_) {
    state().total_ops++;
    if (fused_ops > 1) state().total_fused++;
  }
  return status_;
}

}  // namespace npl

extern "C" int nplk_debug_fail_next_allocations(int count) {
  return npl::g_fail_allocs.exchange(count > 0 ? count : 0);
}
