// Streaming elementwise kernels: inference batch norm, activations, binary
// add/mul and the column-shard relayout. All are HBM-bound: they move each
// element once in and once out with 16-byte accesses where the layout allows,
// and use grid-stride loops sized to a few CTAs per SM.
#include <cuda_runtime.h>

#include "nplk_device.cuh"
#include "nplk_host.h"

namespace nplk {

namespace {
constexpr int kThreads = 256;

int stream_grid(int64_t work_items) {
  const int64_t max_blocks = static_cast<int64_t>(sm_count()) * 8;
  int64_t b = ceil_div(work_items, kThreads);
  if (b > max_blocks) b = max_blocks;
  if (b < 1) b = 1;
  return static_cast<int>(b);
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
}  // namespace

// ---------------------------------------------------------------------------
// Batch norm (inference): y = gamma*(x-mean)*inv_std + beta per NCHW channel,
// inv_std = 1/sqrt(var+eps) (npl_activation_norm.cpp:389-398). Each block
// first computes the per-channel constants into shared memory.
// ---------------------------------------------------------------------------
constexpr int kBnMaxSmemChannels = 3072;  // 48 KB of float4: the default smem limit

template <bool kVec>
__global__ void bn_infer_kernel(const float *__restrict__ x, float *__restrict__ y,
                                int64_t total, uint32_t channels, FastDiv div_hw,
                                FastDiv div_c, const float *__restrict__ mean,
                                const float *__restrict__ var,
                                const float *__restrict__ gamma,
                                const float *__restrict__ beta, float eps) {
  extern __shared__ float4 prm[];  // {gamma, mean, inv_std, beta} per channel
  for (uint32_t c = threadIdx.x; c < channels; c += blockDim.x) {
    prm[c] = make_float4(gamma ? gamma[c] : 1.0f, mean[c], 1.0f / sqrtf(var[c] + eps),
                         beta ? beta[c] : 0.0f);
  }
  __syncthreads();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  if (kVec) {
    const int64_t n4 = total / 4;
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    float4 *y4 = reinterpret_cast<float4 *>(y);
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
         i += stride) {
      const uint32_t plane = fdiv(static_cast<uint32_t>(i * 4), div_hw);
      const uint32_t c = plane - fdiv(plane, div_c) * channels;
      const float4 q = prm[c];
      float4 v = x4[i];
      v.x = q.x * (v.x - q.y) * q.z + q.w;
      v.y = q.x * (v.y - q.y) * q.z + q.w;
      v.z = q.x * (v.z - q.y) * q.z + q.w;
      v.w = q.x * (v.w - q.y) * q.z + q.w;
      y4[i] = v;
    }
  } else {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += stride) {
      const uint32_t plane = fdiv(static_cast<uint32_t>(i), div_hw);
      const uint32_t c = plane - fdiv(plane, div_c) * channels;
      const float4 q = prm[c];
      y[i] = q.x * (x[i] - q.y) * q.z + q.w;
    }
  }
}

// Fallback for very large tensors or channel counts: plain 64-bit indexing.
__global__ void bn_infer_generic_kernel(const float *__restrict__ x, float *__restrict__ y,
                                        int64_t total, int64_t channels, int64_t hw,
                                        const float *__restrict__ mean,
                                        const float *__restrict__ var,
                                        const float *__restrict__ gamma,
                                        const float *__restrict__ beta, float eps) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += stride) {
    const int64_t c = (i / hw) % channels;
    const float g = gamma ? gamma[c] : 1.0f;
    const float b = beta ? beta[c] : 0.0f;
    const float inv = 1.0f / sqrtf(var[c] + eps);
    y[i] = g * (x[i] - mean[c]) * inv + b;
  }
}

// ---------------------------------------------------------------------------
// Activations
// ---------------------------------------------------------------------------
__global__ void act_vec_kernel(const float4 *__restrict__ x, float4 *__restrict__ y, int64_t n4,
                               int act, float alpha) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += stride) {
    float4 v = x[i];
    v.x = apply_act(v.x, act, alpha);
    v.y = apply_act(v.y, act, alpha);
    v.z = apply_act(v.z, act, alpha);
    v.w = apply_act(v.w, act, alpha);
    y[i] = v;
  }
}

__global__ void act_scalar_kernel(const float *__restrict__ x, float *__restrict__ y,
                                  int64_t begin, int64_t n, int act, float alpha) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = begin + static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride)
    y[i] = apply_act(x[i], act, alpha);
}

// ---------------------------------------------------------------------------
// Binary ops (npl_tensor_ops.cpp:440-662): 0 = add, 1 = mul.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bin_op(int op, float a, float b) {
  return op == 0 ? a + b : a * b;
}

__global__ void binary_kernel(int op, int64_t n, const float *__restrict__ a,
                              const float *__restrict__ b, float *__restrict__ c, int b_mode,
                              int64_t channels, int64_t inner) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += stride) {
    float av, bv;
    switch (b_mode) {
      case 1:
        av = a[i];
        bv = b[0];
        break;
      case 2:
        av = a[0];
        bv = b[i];
        break;
      case 3:
        av = a[i];
        bv = b[(i / inner) % channels];
        break;
      default:
        av = a[i];
        bv = b[i];
        break;
    }
    c[i] = bin_op(op, av, bv);
  }
}

__global__ void binary_vec_kernel(int op, int64_t n4, const float4 *__restrict__ a,
                                  const float4 *__restrict__ b, float4 *__restrict__ c) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n4;
       i += stride) {
    const float4 u = a[i], v = b[i];
    c[i] = make_float4(bin_op(op, u.x, v.x), bin_op(op, u.y, v.y), bin_op(op, u.z, v.z),
                       bin_op(op, u.w, v.w));
  }
}

// ---------------------------------------------------------------------------
// [g][rows][cps] -> [rows][g*cps]
// ---------------------------------------------------------------------------
__global__ void colshard_relayout_kernel(const float *__restrict__ src, float *__restrict__ dst,
                                         int64_t g, int64_t rows, int64_t cps, bool vec) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  if (vec) {
    const int64_t cps4 = cps / 4;
    const int64_t total = g * rows * cps4;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += stride) {
      const int64_t j = i % cps4;
      const int64_t r = (i / cps4) % rows;
      const int64_t s = i / (cps4 * rows);
      const float4 v = reinterpret_cast<const float4 *>(src)[i];
      reinterpret_cast<float4 *>(dst + r * g * cps + s * cps)[j] = v;
    }
  } else {
    const int64_t total = g * rows * cps;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += stride) {
      const int64_t j = i % cps;
      const int64_t r = (i / cps) % rows;
      const int64_t s = i / (cps * rows);
      dst[r * g * cps + s * cps + j] = src[i];
    }
  }
}

}  // namespace nplk

using namespace nplk;

extern "C" int nplk_batch_norm_infer(void *stream, int64_t n, int64_t c, int64_t hw,
                                     const float *x, float *y, const float *mean,
                                     const float *var, const float *gamma, const float *beta,
                                     float eps) {
  if (n <= 0 || c <= 0 || hw <= 0 || !x || !y || !mean || !var) return kErrInvalidArg;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t total = n * c * hw;
  const bool small = total < (int64_t(1) << 31) && c <= kBnMaxSmemChannels;
  if (small) {
    const bool vec = (hw % 4 == 0) && aligned16(x) && aligned16(y);
    const int grid = stream_grid(vec ? total / 4 : total);
    const size_t smem = static_cast<size_t>(c) * sizeof(float4);
    const FastDiv dhw = make_fastdiv(static_cast<uint32_t>(hw));
    const FastDiv dc = make_fastdiv(static_cast<uint32_t>(c));
    if (vec)
      bn_infer_kernel<true><<<grid, kThreads, smem, s>>>(x, y, total, static_cast<uint32_t>(c),
                                                         dhw, dc, mean, var, gamma, beta, eps);
    else
      bn_infer_kernel<false><<<grid, kThreads, smem, s>>>(
          x, y, total, static_cast<uint32_t>(c), dhw, dc, mean, var, gamma, beta, eps);
  } else {
    bn_infer_generic_kernel<<<stream_grid(total), kThreads, 0, s>>>(x, y, total, c, hw, mean,
                                                                   var, gamma, beta, eps);
  }
  count_launch();
  return launch_result();
}

extern "C" int nplk_activation(void *stream, int64_t n, const float *x, float *y, int act,
                               float alpha, int scalar_semantics) {
  if (n <= 0 || !x || !y) return kErrInvalidArg;
  if (scalar_semantics) {
    if (act == 1) act = kActReluScalar;
    else if (act == 2) act = kActRelu6Scalar;
    else if (act == 10) act = kActSoftplusScalar;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int64_t done = 0;
  if (aligned16(x) && aligned16(y) && n >= 4) {
    const int64_t n4 = n / 4;
    act_vec_kernel<<<stream_grid(n4), kThreads, 0, s>>>(reinterpret_cast<const float4 *>(x),
                                                       reinterpret_cast<float4 *>(y), n4, act,
                                                       alpha);
    count_launch();
    done = n4 * 4;
    int rc = launch_result();
    if (rc) return rc;
  }
  if (done < n) {
    act_scalar_kernel<<<stream_grid(n - done), kThreads, 0, s>>>(x, y, done, n, act, alpha);
    count_launch();
  }
  return launch_result();
}

extern "C" int nplk_binary(void *stream, int op, int64_t n, const float *a, const float *b,
                           float *c, int b_mode, int64_t channels, int64_t inner) {
  if (n <= 0 || !a || !b || !c || (op != 0 && op != 1)) return kErrInvalidArg;
  if (b_mode == 3 && (channels <= 0 || inner <= 0)) return kErrInvalidArg;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (b_mode == 0 && n % 4 == 0 && aligned16(a) && aligned16(b) && aligned16(c)) {
    binary_vec_kernel<<<stream_grid(n / 4), kThreads, 0, s>>>(
        op, n / 4, reinterpret_cast<const float4 *>(a), reinterpret_cast<const float4 *>(b),
        reinterpret_cast<float4 *>(c));
  } else {
    binary_kernel<<<stream_grid(n), kThreads, 0, s>>>(op, n, a, b, c, b_mode, channels, inner);
  }
  count_launch();
  return launch_result();
}

extern "C" int nplk_colshard_relayout(void *stream, int64_t g, int64_t rows,
                                      int64_t cols_per_shard, const float *src, float *dst) {
  if (g <= 0 || rows <= 0 || cols_per_shard <= 0 || !src || !dst) return kErrInvalidArg;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec = cols_per_shard % 4 == 0 && aligned16(src) && aligned16(dst);
  const int64_t work = g * rows * (vec ? cols_per_shard / 4 : cols_per_shard);
  colshard_relayout_kernel<<<stream_grid(work), kThreads, 0, s>>>(src, dst, g, rows,
                                                                  cols_per_shard, vec);
  count_launch();
  return launch_result();
}
