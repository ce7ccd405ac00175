// npl_* lifecycle, configuration and utility entry points
// (reference: advanced/neural_layer/src/npl_core.cpp:23-189, 402-468).
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "npl_runtime.h"

namespace nplk {
int *device_status_word();
}

static_assert(sizeof(npl_tensor_t) == 168, "npl_tensor_t layout");
static_assert(offsetof(npl_tensor_t, ndim) == 8, "npl_tensor_t.ndim");
static_assert(offsetof(npl_tensor_t, shape) == 16, "npl_tensor_t.shape");
static_assert(offsetof(npl_tensor_t, strides) == 80, "npl_tensor_t.strides");
static_assert(offsetof(npl_tensor_t, dtype) == 144, "npl_tensor_t.dtype");
static_assert(offsetof(npl_tensor_t, layout) == 148, "npl_tensor_t.layout");
static_assert(offsetof(npl_tensor_t, size_bytes) == 152, "npl_tensor_t.size_bytes");
static_assert(offsetof(npl_tensor_t, is_contiguous) == 160, "npl_tensor_t.is_contiguous");
static_assert(sizeof(npl_config_t) == 56, "npl_config_t layout");
static_assert(offsetof(npl_config_t, workspace_size_mb) == 40, "npl_config_t.workspace");
static_assert(offsetof(npl_config_t, verbose) == 48, "npl_config_t.verbose");
static_assert(sizeof(npl_perf_stats_t) == 56, "npl_perf_stats_t layout");
static_assert(offsetof(npl_perf_stats_t, backend_used) == 40, "npl_perf_stats_t.backend");

using npl::state;

extern "C" int npl_get_default_config(npl_config_t *c) {
  if (!c) return NPL_ERR_INVALID_ARG;
  // Same defaults as the reference (npl_core.cpp:172-189).
  c->num_threads = 0;
  c->enable_fusion = 1;
  c->enable_graph_optimization = 1;
  c->enable_jit = 1;
  c->enable_poly = 1;
  c->enable_vectorization = 1;
  c->enable_numa = 1;
  c->enable_memory_pooling = 1;
  c->workspace_size_mb = 256;
  c->verbose = 0;
  return NPL_OK;
}

extern "C" int npl_init(const npl_config_t *config) {
  npl::State &s = state();
  std::lock_guard<std::mutex> lock(s.mu);
  if (s.initialized) return NPL_OK;
  if (config)
    s.config = *config;
  else
    npl_get_default_config(&s.config);

  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();
    std::fprintf(stderr, "[NPL] Error: no CUDA device available\n");
    return NPL_ERR_INTERNAL;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return NPL_ERR_INTERNAL;
  cudaDeviceProp prop{};
  if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return NPL_ERR_INTERNAL;
  if (prop.major != 10 || prop.minor != 0) {
    std::fprintf(stderr,
                 "[NPL] Error: device %d is sm_%d%d; this library is built for sm_100a (B200)\n",
                 dev, prop.major, prop.minor);
    return NPL_ERR_UNSUPPORTED;
  }
  if (cudaSetDevice(dev) != cudaSuccess || cudaFree(nullptr) != cudaSuccess)
    return NPL_ERR_INTERNAL;
  cudaStream_t stream = nullptr;
  if (cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking) != cudaSuccess)
    return NPL_ERR_INTERNAL;
  // Keep freed pool memory cached for reuse by later calls.
  cudaMemPool_t pool;
  if (cudaDeviceGetDefaultMemPool(&pool, dev) == cudaSuccess) {
    uint64_t threshold = UINT64_MAX;
    cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold);
  }
  int cma = 0;
  cudaDeviceGetAttribute(&cma, cudaDevAttrConcurrentManagedAccess, dev);
  if (!nplk::device_status_word()) {
    cudaStreamDestroy(stream);
    return NPL_ERR_INTERNAL;
  }
  s.device = dev;
  s.stream = stream;
  s.concurrent_managed = cma;
  s.total_ops = 0;
  s.total_fused = 0;
  s.initialized = true;
  // The tile-configuration cache file, if one is named and present (a file
  // from another device or format version is reported and skipped).
  const char *cache_path = std::getenv("NPL_TUNING_CACHE");
  if (cache_path && cache_path[0]) {
    if (FILE *f = std::fopen(cache_path, "r")) {
      std::fclose(f);
      const int n = nplk_tuning_cache_load(cache_path);
      if (s.config.verbose && n >= 0)
        std::printf("[NPL] Loaded %d tuning entries from %s\n", n, cache_path);
    }
  }
  if (s.config.verbose) {
    std::printf("[NPL] Initialized on device %d (%s, %d SMs)\n", dev, prop.name,
                prop.multiProcessorCount);
  }
  return NPL_OK;
}

extern "C" void npl_shutdown(void) {
  npl::State &s = state();
  std::lock_guard<std::mutex> lock(s.mu);
  if (!s.initialized) return;
  if (s.config.verbose) {
    std::printf("[NPL] Shutting down...\n  Total operations: %zu\n  Operations fused: %zu\n",
                s.total_ops.load(), s.total_fused.load());
  }
  cudaSetDevice(s.device);
  cudaStreamSynchronize(s.stream);
  const char *cache_path = std::getenv("NPL_TUNING_CACHE");
  nplk_tuning_stats_t ts{};
  if (cache_path && cache_path[0] && nplk_tuning_cache_stats(&ts) == 0 && ts.entries > 0)
    nplk_tuning_cache_save(cache_path);
  cudaStreamDestroy(s.stream);
  s.stream = nullptr;
  s.initialized = false;
  s.total_ops = 0;
  s.total_fused = 0;
}

extern "C" int npl_is_initialized(void) { return state().initialized ? 1 : 0; }

extern "C" const char *npl_strerror(int error) {
  switch (error) {
    case NPL_OK:
      return "Success";
    case NPL_ERR_NOT_INITIALIZED:
      return "Not initialized";
    case NPL_ERR_INVALID_ARG:
      return "Invalid argument";
    case NPL_ERR_NO_MEMORY:
      return "Out of memory";
    case NPL_ERR_INTERNAL:
      return "Internal error";
    case NPL_ERR_UNSUPPORTED:
      return "Unsupported operation";
    case NPL_ERR_SHAPE_MISMATCH:
      return "Tensor shape mismatch";
    case NPL_ERR_OOM:
      return "Out of memory during execution";
    default:
      return "Unknown error";
  }
}

extern "C" const char *npl_get_system_info(void) {
  static thread_local char buf[1024];
  npl::State &s = state();
  if (!s.initialized) {
    std::snprintf(buf, sizeof(buf), "JCore Neural Primitives Layer: Not initialized");
    return buf;
  }
  cudaDeviceProp prop{};
  cudaGetDeviceProperties(&prop, s.device);
  size_t free_b = 0, total_b = 0;
  cudaSetDevice(s.device);
  cudaMemGetInfo(&free_b, &total_b);
  std::snprintf(buf, sizeof(buf),
                "JCore Neural Primitives Layer (B200 backend)\n"
                "  Status: Initialized\n"
                "  Device: %d %s (sm_%d%d, %d SMs)\n"
                "  HBM: %.1f GB total, %.1f GB free\n"
                "  Dense ops: tcgen05 3xTF32 GEMM / implicit-GEMM conv%s\n"
                "  Statistics:\n"
                "    Total Operations: %zu\n"
                "    Fused Operations: %zu\n",
                s.device, prop.name, prop.major, prop.minor, prop.multiProcessorCount,
                total_b / 1e9, free_b / 1e9,
                npl::tf32_fast_mode() ? " (TF32 fast mode)" : "", s.total_ops.load(),
                s.total_fused.load());
  return buf;
}

// Known-answer checks of the reference self test (npl_test.cpp:104-555),
// run on the device through the public API.
extern "C" int npl_self_test(int verbose) {
  if (!state().initialized) return NPL_ERR_NOT_INITIALIZED;
  int failures = 0;
  auto report = [&](const char *name, bool ok) {
    if (!ok) ++failures;
    if (verbose) std::printf("[%s] %s\n", ok ? "PASS" : "FAIL", name);
  };
  auto make = [](npl_tensor_t *t, size_t nd, const size_t *shape) {
    npl_create_tensor(nullptr, nd, shape, NPL_DTYPE_FP32, NPL_LAYOUT_NCHW, t);
    return npl_allocate_tensor(t);
  };
  {  // matmul 32^3 of ones -> 32
    const size_t s2[] = {32, 32};
    npl_tensor_t A, B, C;
    bool ok = make(&A, 2, s2) == NPL_OK && make(&B, 2, s2) == NPL_OK && make(&C, 2, s2) == NPL_OK;
    if (ok) {
      for (int i = 0; i < 1024; ++i) {
        static_cast<float *>(A.data)[i] = 1.0f;
        static_cast<float *>(B.data)[i] = 1.0f;
      }
      ok = npl_matmul(&A, &B, &C, 1.0f, 0.0f, nullptr) == NPL_OK;
      for (int i = 0; ok && i < 1024; ++i)
        ok = std::fabs(static_cast<float *>(C.data)[i] - 32.0f) < 1e-3f;
    }
    report("MatMul", ok);
    npl_free_tensor(&A);
    npl_free_tensor(&B);
    npl_free_tensor(&C);
  }
  {  // conv 1x3x8x8 ones, 2x3x3x3 ones, bias 0.5, VALID -> 27.5
    const size_t si[] = {1, 3, 8, 8}, sw[] = {2, 3, 3, 3}, sb[] = {2}, so[] = {1, 2, 6, 6};
    npl_tensor_t in, w, b, out;
    bool ok = make(&in, 4, si) == NPL_OK && make(&w, 4, sw) == NPL_OK &&
              make(&b, 1, sb) == NPL_OK && make(&out, 4, so) == NPL_OK;
    if (ok) {
      for (int i = 0; i < 192; ++i) static_cast<float *>(in.data)[i] = 1.0f;
      for (int i = 0; i < 54; ++i) static_cast<float *>(w.data)[i] = 1.0f;
      static_cast<float *>(b.data)[0] = static_cast<float *>(b.data)[1] = 0.5f;
      npl_conv_params_t p{};
      p.kernel_h = p.kernel_w = 3;
      p.stride_h = p.stride_w = 1;
      p.dilation_h = p.dilation_w = 1;
      p.groups = 1;
      p.padding = NPL_PAD_VALID;
      ok = npl_conv2d(&in, &w, &b, &p, &out, nullptr) == NPL_OK;
      for (int i = 0; ok && i < 72; ++i)
        ok = std::fabs(static_cast<float *>(out.data)[i] - 27.5f) < 0.01f;
    }
    report("Conv2D", ok);
    npl_free_tensor(&in);
    npl_free_tensor(&w);
    npl_free_tensor(&b);
    npl_free_tensor(&out);
  }
  {  // relu on [-2, 2), softmax rows sum to 1, GAP of ones -> 1
    const size_t s1[] = {1024};
    npl_tensor_t x, y;
    bool ok = make(&x, 1, s1) == NPL_OK && make(&y, 1, s1) == NPL_OK;
    if (ok) {
      float *xd = static_cast<float *>(x.data);
      for (int i = 0; i < 1024; ++i) xd[i] = -2.0f + 4.0f * i / 1024;
      ok = npl_relu(&x, &y, nullptr) == NPL_OK;
      for (int i = 0; ok && i < 1024; ++i)
        ok = std::fabs(static_cast<float *>(y.data)[i] - (xd[i] > 0 ? xd[i] : 0.0f)) < 1e-3f;
    }
    report("ReLU", ok);
    npl_free_tensor(&x);
    npl_free_tensor(&y);

    const size_t ss[] = {2, 10};
    ok = make(&x, 2, ss) == NPL_OK && make(&y, 2, ss) == NPL_OK;
    if (ok) {
      for (int i = 0; i < 20; ++i) static_cast<float *>(x.data)[i] = static_cast<float>(i % 10);
      ok = npl_softmax(&x, 1, &y, nullptr) == NPL_OK;
      for (int r = 0; ok && r < 2; ++r) {
        float sum = 0.0f;
        for (int i = 0; i < 10; ++i) sum += static_cast<float *>(y.data)[r * 10 + i];
        ok = std::fabs(sum - 1.0f) < 1e-3f;
      }
    }
    report("Softmax", ok);
    npl_free_tensor(&x);
    npl_free_tensor(&y);

    const size_t sg[] = {2, 64, 7, 7}, sgo[] = {2, 64, 1, 1};
    ok = make(&x, 4, sg) == NPL_OK && make(&y, 4, sgo) == NPL_OK;
    if (ok) {
      for (int i = 0; i < 2 * 64 * 49; ++i) static_cast<float *>(x.data)[i] = 1.0f;
      ok = npl_global_avg_pool(&x, &y, nullptr) == NPL_OK;
      for (int i = 0; ok && i < 128; ++i)
        ok = std::fabs(static_cast<float *>(y.data)[i] - 1.0f) < 1e-3f;
    }
    report("GlobalAvgPool", ok);
    npl_free_tensor(&x);
    npl_free_tensor(&y);
  }
  return failures == 0 ? NPL_OK : NPL_ERR_INTERNAL;
}
