// Row reductions: softmax, layer norm and global average pooling.
// Rows are read from HBM once: the warp/CTA keeps them in registers while it
// reduces (max and sum for softmax, mean then centred variance for layer
// norm), using warp shuffles and one shared-memory exchange across warps.
#include <cuda_runtime.h>
#include <math_constants.h>

#include "nplk_host.h"
#include "ptx_sm100.cuh"

namespace nplk {

namespace {
bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Sum over the CTA; every thread gets the result. `red` holds >= 32 floats.
__device__ __forceinline__ float block_sum(float v, float *red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = lane < nw ? red[lane] : 0.0f;
  return warp_sum(t);
}
}  // namespace

// ---------------------------------------------------------------------------
// Softmax over contiguous rows (inner == 1), one warp per row, the row held in
// registers as NV float4 per lane: max, exp(x - max), sum, exp / sum
// (ExecuteSoftmaxAxis, npl_activation_norm.cpp:322-350).
// ---------------------------------------------------------------------------
template <int NV>
__global__ void softmax_rows_warp_kernel(const float *__restrict__ x, float *__restrict__ y,
                                         int64_t rows, int cols) {
  // Launched as a programmatic dependent: the kernel before it (when it
  // allows an early launch) has completed and its writes are visible past
  // this wait; after any other kernel it returns at once.
  griddep_wait();
  const int lane = threadIdx.x & 31;
  const int64_t warp_id = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  const int c4 = cols >> 2;
  for (int64_t r = warp_id; r < rows; r += nwarps) {
    const float4 *xr = reinterpret_cast<const float4 *>(x + r * cols);
    float4 v[NV];
    float mx = -CUDART_INF_F;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int j = lane + 32 * i;
      if (j < c4) {
        v[i] = xr[j];
        mx = fmaxf(mx, fmaxf(fmaxf(v[i].x, v[i].y), fmaxf(v[i].z, v[i].w)));
      }
    }
    mx = warp_max(mx);
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int j = lane + 32 * i;
      if (j < c4) {
        v[i].x = expf(v[i].x - mx);
        v[i].y = expf(v[i].y - mx);
        v[i].z = expf(v[i].z - mx);
        v[i].w = expf(v[i].w - mx);
        sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
      }
    }
    sum = warp_sum(sum);
    float4 *yr = reinterpret_cast<float4 *>(y + r * cols);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int j = lane + 32 * i;
      if (j < c4)
        yr[j] = make_float4(v[i].x / sum, v[i].y / sum, v[i].z / sum, v[i].w / sum);
    }
  }
}

// General softmax: one thread per (outer, inner) line, strided along the
// axis; consecutive threads take consecutive inner indices (coalesced).
__global__ void softmax_strided_kernel(const float *__restrict__ x, float *__restrict__ y,
                                       int64_t outer, int64_t axis_len, int64_t inner) {
  griddep_wait();  // as in softmax_rows_warp_kernel
  const int64_t lines = outer * inner;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t l = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; l < lines;
       l += stride) {
    const int64_t o = l / inner, in = l - o * inner;
    const float *xp = x + o * axis_len * inner + in;
    float *yp = y + o * axis_len * inner + in;
    float mx = -CUDART_INF_F;
    for (int64_t i = 0; i < axis_len; ++i) mx = fmaxf(mx, xp[i * inner]);
    float sum = 0.0f;
    for (int64_t i = 0; i < axis_len; ++i) {
      const float e = expf(xp[i * inner] - mx);
      yp[i * inner] = e;
      sum += e;
    }
    for (int64_t i = 0; i < axis_len; ++i) yp[i * inner] = yp[i * inner] / sum;
  }
}

// ---------------------------------------------------------------------------
// Layer norm, one CTA per row, row in registers (NV float4 per thread):
// mean = sum/n; var = sum((x-mean)^2)/n; y = gamma*((x-mean)*inv_std)+beta
// (ExecuteLayerNormGeneric, npl_activation_norm.cpp:482-512).
// ---------------------------------------------------------------------------
template <int NV>
__global__ void layernorm_rows_kernel(const float *__restrict__ x, float *__restrict__ y,
                                      int64_t rows, int cols, const float *__restrict__ gamma,
                                      const float *__restrict__ beta, float eps) {
  __shared__ float red[32];
  const int c4 = cols >> 2;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float4 *xr = reinterpret_cast<const float4 *>(x + r * cols);
    float4 v[NV];
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int j = threadIdx.x + blockDim.x * i;
      if (j < c4) {
        v[i] = xr[j];
        s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
      }
    }
    const float mean = block_sum(s, red) / static_cast<float>(cols);
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int j = threadIdx.x + blockDim.x * i;
      if (j < c4) {
        const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean,
                    d = v[i].w - mean;
        q += (a * a + b * b) + (c * c + d * d);
      }
    }
    const float var = block_sum(q, red) / static_cast<float>(cols);
    const float inv = 1.0f / sqrtf(var + eps);
    float4 *yr = reinterpret_cast<float4 *>(y + r * cols);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int j = threadIdx.x + blockDim.x * i;
      if (j < c4) {
        float4 o;
        const float g0 = gamma ? gamma[4 * j] : 1.0f, g1 = gamma ? gamma[4 * j + 1] : 1.0f,
                    g2 = gamma ? gamma[4 * j + 2] : 1.0f, g3 = gamma ? gamma[4 * j + 3] : 1.0f;
        const float b0 = beta ? beta[4 * j] : 0.0f, b1 = beta ? beta[4 * j + 1] : 0.0f,
                    b2 = beta ? beta[4 * j + 2] : 0.0f, b3 = beta ? beta[4 * j + 3] : 0.0f;
        o.x = g0 * ((v[i].x - mean) * inv) + b0;
        o.y = g1 * ((v[i].y - mean) * inv) + b1;
        o.z = g2 * ((v[i].z - mean) * inv) + b2;
        o.w = g3 * ((v[i].w - mean) * inv) + b3;
        yr[j] = o;
      }
    }
  }
}

// Long rows (2 K..16 K elements, a multiple of 4, 16-byte aligned): the
// arithmetic of layernorm_rows_kernel fed by a warp-specialised ring. One
// producer lane stages whole rows (one bulk copy each) into `stages`
// shared-memory stages; the 16 consumer warps form G groups (kG = 1, 2 or 4)
// that each take every G-th row: a group reads its row into registers,
// releases the stage at once (its own named barrier), reduces and writes,
// while the other groups and the next rows' copies proceed. With G = 1 (16 K
// rows) the thread-to-element mapping is layernorm_rows_kernel's with 512
// threads, so the results agree bit for bit.
constexpr int kLnWarps = 16;
constexpr int kLnThreads = (kLnWarps + 1) * 32;

template <int kG>
__device__ __forceinline__ void ln_group_sync(int group) {
  asm volatile("bar.sync %0, %1;" ::"r"(1 + group), "n"(kLnWarps * 32 / kG) : "memory");
}

// Sum over the group's warps; every thread of the group gets the result.
template <int kG>
__device__ __forceinline__ float ln_group_sum(float v, float *red, int group) {
  constexpr int kGW = kLnWarps / kG;  // warps per group
  const int lane = threadIdx.x & 31, gw = (threadIdx.x >> 5) % kGW;
  v = warp_sum(v);
  if (lane == 0) red[group * kGW + gw] = v;
  ln_group_sync<kG>(group);
  float t = lane < kGW ? red[group * kGW + lane] : 0.0f;
  t = warp_sum(t);
  ln_group_sync<kG>(group);  // red is written again by the next reduction
  return t;
}

template <int NV, int kG>
__global__ void __launch_bounds__(kLnThreads, 1)
    layernorm_ring_kernel(const float *__restrict__ x, float *__restrict__ y, int64_t rows,
                          int cols, const float *__restrict__ gamma,
                          const float *__restrict__ beta, float eps, int stages, int *status) {
  extern __shared__ __align__(128) uint8_t smem_ln[];
  float *st = reinterpret_cast<float *>(smem_ln);
  uint64_t *full = reinterpret_cast<uint64_t *>(st + static_cast<int64_t>(stages) * cols);
  uint64_t *empty = full + stages;
  float *red = reinterpret_cast<float *>(empty + stages);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(red + 32);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  const int64_t nk = rows > blockIdx.x ? (rows - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const uint32_t row_bytes = static_cast<uint32_t>(cols) * 4u;
  if (warp == kLnWarps) {
    // ---------------- producer ----------------
    if (lane == 0) {
      int64_t k = 0;
      for (; k < nk; ++k) {
        const int s = static_cast<int>(k % stages);
        const uint32_t ph = static_cast<uint32_t>(k / stages) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, status, kStatusTimeoutProducer)) break;
        mbar_arrive_expect_tx(&full[s], row_bytes);
        bulk_load_g2s(st + static_cast<int64_t>(s) * cols,
                      x + (blockIdx.x + k * gridDim.x) * static_cast<int64_t>(cols), row_bytes,
                      &full[s]);
      }
      for (int64_t j = k > stages ? k - stages : 0; j < k; ++j)
        mbar_drain(&full[j % stages], static_cast<uint32_t>(j / stages) & 1u);
    }
    return;
  }
  // ---------------- consumers ----------------
  constexpr int kGT = kLnWarps * 32 / kG;  // threads per group
  const int group = threadIdx.x / kGT;
  const int t = threadIdx.x - group * kGT;
  const int c4 = cols >> 2;
  for (int64_t k = group; k < nk; k += kG) {
    const int s = static_cast<int>(k % stages);
    const uint32_t ph = static_cast<uint32_t>(k / stages) & 1u;
    if (!mbar_wait(&full[s], ph, abort_flag, status, kStatusTimeoutStage)) break;
    const float4 *xr = reinterpret_cast<const float4 *>(st + static_cast<int64_t>(s) * cols);
    float4 v[NV];
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int j = t + kGT * i;
      if (j < c4) {
        v[i] = xr[j];
        sum += (v[i].x + v[i].y) + (v[i].z + v[i].w);
      }
    }
    ln_group_sync<kG>(group);  // every thread of the group holds its part of the row
    if (t == 0) mbar_arrive(&empty[s]);
    const float mean = ln_group_sum<kG>(sum, red, group) / static_cast<float>(cols);
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int j = t + kGT * i;
      if (j < c4) {
        const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean,
                    d = v[i].w - mean;
        q += (a * a + b * b) + (c * c + d * d);
      }
    }
    const float var = ln_group_sum<kG>(q, red, group) / static_cast<float>(cols);
    const float inv = 1.0f / sqrtf(var + eps);
    float4 *yr = reinterpret_cast<float4 *>(
        y + (blockIdx.x + k * gridDim.x) * static_cast<int64_t>(cols));
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int j = t + kGT * i;
      if (j < c4) {
        float4 o;
        const float g0 = gamma ? gamma[4 * j] : 1.0f, g1 = gamma ? gamma[4 * j + 1] : 1.0f,
                    g2 = gamma ? gamma[4 * j + 2] : 1.0f, g3 = gamma ? gamma[4 * j + 3] : 1.0f;
        const float b0 = beta ? beta[4 * j] : 0.0f, b1 = beta ? beta[4 * j + 1] : 0.0f,
                    b2 = beta ? beta[4 * j + 2] : 0.0f, b3 = beta ? beta[4 * j + 3] : 0.0f;
        o.x = g0 * ((v[i].x - mean) * inv) + b0;
        o.y = g1 * ((v[i].y - mean) * inv) + b1;
        o.z = g2 * ((v[i].z - mean) * inv) + b2;
        o.w = g3 * ((v[i].w - mean) * inv) + b3;
        yr[j] = o;
      }
    }
  }
}

// Any row length: three passes over the row from global memory (L2-resident
// for one CTA's row).
__global__ void layernorm_generic_kernel(const float *__restrict__ x, float *__restrict__ y,
                                         int64_t rows, int64_t cols,
                                         const float *__restrict__ gamma,
                                         const float *__restrict__ beta, float eps) {
  __shared__ float red[32];
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float *xr = x + r * cols;
    float s = 0.0f;
    for (int64_t j = threadIdx.x; j < cols; j += blockDim.x) s += xr[j];
    const float mean = block_sum(s, red) / static_cast<float>(cols);
    float q = 0.0f;
    for (int64_t j = threadIdx.x; j < cols; j += blockDim.x) {
      const float d = xr[j] - mean;
      q += d * d;
    }
    const float var = block_sum(q, red) / static_cast<float>(cols);
    const float inv = 1.0f / sqrtf(var + eps);
    for (int64_t j = threadIdx.x; j < cols; j += blockDim.x) {
      const float g = gamma ? gamma[j] : 1.0f, b = beta ? beta[j] : 0.0f;
      y[r * cols + j] = g * ((xr[j] - mean) * inv) + b;
    }
  }
}

// ---------------------------------------------------------------------------
// Global average pool: one warp per contiguous plane of hw elements.
// ---------------------------------------------------------------------------
// A warp reduces kGapPlanes planes per iteration, issuing all their loads
// before the reductions, so several 16-byte loads per lane are in flight.
constexpr int kGapPlanes = 4;

// kGapPlanes planes per warp and iteration, J float4 per lane per plane: every
// load is issued (predicated, no branches) before the first add, so all of
// them are in flight together.
template <int J>
__device__ __forceinline__ void gap_planes(const float *__restrict__ x, float *__restrict__ y,
                                           int64_t planes, int64_t hw, int hw4, int64_t warp_id,
                                           int64_t nwarps, int lane) {
  for (int64_t p0 = warp_id * kGapPlanes; p0 < planes; p0 += nwarps * kGapPlanes) {
    float4 v[kGapPlanes][J];
#pragma unroll
    for (int k = 0; k < kGapPlanes; ++k) {
      const float4 *x4 = reinterpret_cast<const float4 *>(x + (p0 + k) * hw);
      const bool okp = p0 + k < planes;
#pragma unroll
      for (int j = 0; j < J; ++j)
        v[k][j] = (okp && lane + 32 * j < hw4) ? __ldg(x4 + lane + 32 * j)
                                               : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
#pragma unroll
    for (int k = 0; k < kGapPlanes; ++k) {
      float s = 0.0f;
#pragma unroll
      for (int j = 0; j < J; ++j) s += (v[k][j].x + v[k][j].y) + (v[k][j].z + v[k][j].w);
      const float t = warp_sum(s);
      if (lane == 0 && p0 + k < planes) y[p0 + k] = t / static_cast<float>(hw);
    }
  }
}

// J > 0: planes of at most J * 128 elements, 16-byte aligned (J float4 per
// lane per plane; a kernel per J, so the common J = 2 keeps its register count
// and occupancy: 64 registers against 96 with the J = 4 path in the same
// kernel, 22.5 vs 30.7 us on [256,512,14,14]). J = 0: any plane.
template <int J>
__global__ void gap_kernel(const float *__restrict__ x, float *__restrict__ y, int64_t planes,
                           int64_t hw, bool vec) {
  const int lane = threadIdx.x & 31;
  const int64_t warp_id = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
  if constexpr (J > 0) {
    gap_planes<J>(x, y, planes, hw, static_cast<int>(hw / 4), warp_id, nwarps, lane);
  } else {
    for (int64_t p = warp_id; p < planes; p += nwarps) {
      const float *xp = x + p * hw;
      float s = 0.0f;
      if (vec) {
        const float4 *x4 = reinterpret_cast<const float4 *>(xp);
        for (int64_t j = lane; j < hw / 4; j += 32) {
          const float4 v = x4[j];
          s += (v.x + v.y) + (v.z + v.w);
        }
      } else {
        for (int64_t j = lane; j < hw; j += 32) s += xp[j];
      }
      s = warp_sum(s);
      if (lane == 0) y[p] = s / static_cast<float>(hw);
    }
  }
}

// ---------------------------------------------------------------------------
// Batch statistics for training-mode batch norm: one CTA per channel, mean
// over N*HW, then the biased variance from the centred values
// (ComputeBatchStatistics, npl_activation_norm.cpp:524-552).
// ---------------------------------------------------------------------------
__global__ void bn_stats_kernel(const float *__restrict__ x, int64_t n, int64_t c, int64_t hw,
                                float *__restrict__ mean, float *__restrict__ var) {
  __shared__ float red[32];
  const int64_t ch = blockIdx.x;
  const float count = static_cast<float>(n * hw);
  float s = 0.0f;
  for (int64_t b = 0; b < n; ++b) {
    const float *p = x + (b * c + ch) * hw;
    for (int64_t j = threadIdx.x; j < hw; j += blockDim.x) s += p[j];
  }
  const float m = block_sum(s, red) / count;
  float q = 0.0f;
  for (int64_t b = 0; b < n; ++b) {
    const float *p = x + (b * c + ch) * hw;
    for (int64_t j = threadIdx.x; j < hw; j += blockDim.x) {
      const float d = p[j] - m;
      q += d * d;
    }
  }
  const float v = block_sum(q, red) / count;
  if (threadIdx.x == 0) {
    mean[ch] = m;
    var[ch] = v;
  }
}

__global__ void bn_update_running_kernel(int64_t c, float *run_mean, float *run_var,
                                         const float *mean, const float *var, float momentum) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < c) {
    run_mean[i] = momentum * run_mean[i] + (1.0f - momentum) * mean[i];
    run_var[i] = momentum * run_var[i] + (1.0f - momentum) * var[i];
  }
}

}  // namespace nplk

using namespace nplk;

extern "C" int nplk_batch_norm_stats(void *stream, int64_t n, int64_t c, int64_t hw,
                                     const float *x, float *mean, float *var) {
  if (n <= 0 || c <= 0 || hw <= 0 || !x || !mean || !var) return kErrInvalidArg;
  if (c > 2147483647) return kErrUnsupported;
  bn_stats_kernel<<<static_cast<unsigned>(c), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, n, c, hw, mean, var);
  count_launch();
  return launch_result();
}

extern "C" int nplk_bn_update_running(void *stream, int64_t c, float *run_mean, float *run_var,
                                      const float *mean, const float *var, float momentum) {
  if (c <= 0 || !run_mean || !run_var || !mean || !var) return kErrInvalidArg;
  bn_update_running_kernel<<<static_cast<unsigned>(ceil_div(c, 256)), 256, 0,
                             static_cast<cudaStream_t>(stream)>>>(c, run_mean, run_var, mean,
                                                                  var, momentum);
  count_launch();
  return launch_result();
}

namespace {
int grid_for(int64_t items, int per_block) {
  const int64_t max_blocks = static_cast<int64_t>(sm_count()) * 16;
  int64_t b = ceil_div(items, per_block);
  if (b > max_blocks) b = max_blocks;
  return static_cast<int>(b < 1 ? 1 : b);
}
}  // namespace

extern "C" int nplk_softmax(void *stream, int64_t outer, int64_t axis_len, int64_t inner,
                            const float *x, float *y) {
  if (outer <= 0 || axis_len <= 0 || inner <= 0 || !x || !y) return kErrInvalidArg;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (inner == 1 && axis_len % 4 == 0 && axis_len <= 32 * 4 * 16 && aligned16(x) &&
      aligned16(y)) {
    const int c4 = static_cast<int>(axis_len / 4);
    const int threads = 256;
    // One warp per row and a grid that covers every row: block scheduling
    // keeps the loads of many rows in flight (rows of 1000: 120.8 us against
    // 156.7 us for a grid of 16 blocks per SM whose warps each pipelined
    // several rows).
    const int64_t blocks = ceil_div(outer, static_cast<int64_t>(threads / 32));
    const int grid = static_cast<int>(blocks < (int64_t(1) << 30) ? blocks : (int64_t(1) << 30));
    const int cols = static_cast<int>(axis_len);
    // Programmatic launches (the kernels wait for their predecessor first):
    // behind a kernel that allows it -- the bandwidth chain's one-pass kernel
    // -- the softmax's launch overlaps that kernel's last wave.
    if (c4 <= 32 * 4)
      return launch_programmatic(softmax_rows_warp_kernel<4>, dim3(grid), dim3(threads), 0, s, x,
                                 y, outer, cols);
    if (c4 <= 32 * 8)
      return launch_programmatic(softmax_rows_warp_kernel<8>, dim3(grid), dim3(threads), 0, s, x,
                                 y, outer, cols);
    return launch_programmatic(softmax_rows_warp_kernel<16>, dim3(grid), dim3(threads), 0, s, x, y,
                               outer, cols);
  }
  return launch_programmatic(softmax_strided_kernel, dim3(grid_for(outer * inner, 256)), dim3(256),
                             0, s, x, y, outer, axis_len, inner);
}

extern "C" int nplk_layer_norm(void *stream, int64_t rows, int64_t cols, const float *x,
                               float *y, const float *gamma, const float *beta, float eps) {
  if (rows <= 0 || cols <= 0 || !x || !y) return kErrInvalidArg;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t rows_grid = rows < 65535 * 16 ? rows : 65535 * 16;
  if (cols % 4 == 0 && aligned16(x) && aligned16(y) && cols >= 2048 && cols <= 16384) {
    // Rows of 8..64 KB through the ring: up to 8 stages in ~200 KB (3 for
    // 64 KB rows); the grid is as many CTAs as are resident.
    const int64_t row_bytes = cols * 4;
    int stages = static_cast<int>(200 * 1024 / row_bytes);
    if (stages > 8) stages = 8;
    const size_t smem = static_cast<size_t>(stages) * row_bytes + 2 * 8 * 8 + 32 * 4 + 16;
    // Groups: 16 K rows take all 16 warps; 8 K rows two groups of 8; shorter
    // rows four groups of 4 (each thread then holds up to 8 float4).
    const int G = cols > 8192 ? 1 : cols > 4096 ? 2 : 4;
    const int nv = static_cast<int>(ceil_div(cols / 4, int64_t(kLnWarps * 32 / G)));
    int *status = device_status_word();
    const int ci = static_cast<int>(cols);
    auto go = [&](auto kernel) -> int {
      if (int rc = ensure_dynamic_smem(reinterpret_cast<const void *>(kernel),
                                       static_cast<int>(smem)))
        return rc;
      int per_sm = 0;
      if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kLnThreads, smem) !=
              cudaSuccess ||
          per_sm < 1)
        per_sm = 1;
      int64_t blocks = static_cast<int64_t>(sm_count()) * per_sm;
      if (blocks > rows) blocks = rows;
      kernel<<<static_cast<unsigned>(blocks), kLnThreads, smem, s>>>(x, y, rows, ci, gamma, beta,
                                                                     eps, stages, status);
      return 0;
    };
    int rc;
    if (G == 1)
      rc = go(layernorm_ring_kernel<8, 1>);
    else if (G == 2)
      rc = go(layernorm_ring_kernel<8, 2>);
    else
      rc = nv <= 4 ? go(layernorm_ring_kernel<4, 4>) : go(layernorm_ring_kernel<8, 4>);
    if (rc) return rc;
  } else if (cols % 4 == 0 && aligned16(x) && aligned16(y) && cols <= 512 * 4 * 16) {
    const int64_t c4 = cols / 4;
    int threads = 512;
    while (threads > 32 && threads / 2 >= c4) threads /= 2;
    const int64_t nv = ceil_div(c4, threads);
    const int grid = static_cast<int>(rows_grid);
    if (nv <= 1)
      layernorm_rows_kernel<1><<<grid, threads, 0, s>>>(x, y, rows, static_cast<int>(cols),
                                                        gamma, beta, eps);
    else if (nv <= 2)
      layernorm_rows_kernel<2><<<grid, threads, 0, s>>>(x, y, rows, static_cast<int>(cols),
                                                        gamma, beta, eps);
    else if (nv <= 4)
      layernorm_rows_kernel<4><<<grid, threads, 0, s>>>(x, y, rows, static_cast<int>(cols),
                                                        gamma, beta, eps);
    else if (nv <= 8)
      layernorm_rows_kernel<8><<<grid, threads, 0, s>>>(x, y, rows, static_cast<int>(cols),
                                                        gamma, beta, eps);
    else
      layernorm_rows_kernel<16><<<grid, threads, 0, s>>>(x, y, rows, static_cast<int>(cols),
                                                         gamma, beta, eps);
  } else {
    layernorm_generic_kernel<<<static_cast<int>(rows_grid), 256, 0, s>>>(x, y, rows, cols,
                                                                        gamma, beta, eps);
  }
  count_launch();
  return launch_result();
}

extern "C" int nplk_global_avg_pool(void *stream, int64_t planes, int64_t hw, const float *x,
                                    float *y) {
  if (planes <= 0 || hw <= 0 || !x || !y) return kErrInvalidArg;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool vec = hw % 4 == 0 && aligned16(x);
  // Planes of up to 512 elements: one pass, every warp takes kGapPlanes planes
  // and the grid covers them all (block scheduling overlaps the warps' load
  // round trips; a grid capped at a few blocks per SM made warps loop and wait
  // on one round trip per iteration: 28.7 vs 22.5 us on [256,512,14,14]).
  if (vec && hw <= 4 * 32 * 4) {
    const int64_t blocks = ceil_div(planes, static_cast<int64_t>(8 * kGapPlanes));
    const int grid = static_cast<int>(blocks < (int64_t(1) << 30) ? blocks : (int64_t(1) << 30));
    if (hw <= 2 * 32 * 4)
      gap_kernel<2><<<grid, 256, 0, s>>>(x, y, planes, hw, vec);
    else
      gap_kernel<4><<<grid, 256, 0, s>>>(x, y, planes, hw, vec);
  } else {
    gap_kernel<0><<<grid_for(planes, 8), 256, 0, s>>>(x, y, planes, hw, vec);
  }
  count_launch();
  return launch_result();
}
