// Sliding-window kernels over NCHW planes: depthwise convolution and max /
// average pooling.
//
// plane_window_kernel (planes of at most 24 K elements): a CTA stages a batch
// of whole input planes in shared memory with 16-byte loads (consecutive
// planes are contiguous in NCHW, so the batch is one contiguous range and
// many bytes are in flight per SM), then each thread computes 4 adjacent
// outputs of one row from shared memory. window_kernel (larger planes): one
// thread per output, consecutive threads on consecutive output columns, so
// the window reads of a warp hit a few cache lines and are served from L1
// after the first touch. Both compute every output with the same expression
// in the same order (the reference's: kh outer, kw inner, padded cells
// skipped), so they agree bit for bit; each input element crosses HBM about
// once.
#include <cuda_runtime.h>
#include <math_constants.h>

#include "nplk_device.cuh"
#include "nplk_host.h"

namespace nplk {

namespace {
int window_grid(int64_t items) {
  const int64_t max_blocks = static_cast<int64_t>(sm_count()) * 16;
  int64_t b = ceil_div(items, 256);
  if (b > max_blocks) b = max_blocks;
  return static_cast<int>(b < 1 ? 1 : b);
}
}  // namespace

struct WindowGeom {
  int C, H, W, KH, KW, sh, sw, ph, pw, Ho, Wo;
  FastDiv div_wo, div_ho, div_c;
};

// Depthwise: out[n][c][oh][ow] = sum_{kh,kw} x[n][c][oh*sh+kh-ph][ow*sw+kw-pw]
// * w[c][kh][kw] (+ bias[c]) with the reference's summation order (kh outer,
// kw inner) and no dilation (npl_convolution.cpp:921-951).
__global__ void dwconv_kernel(const float *__restrict__ x, const float *__restrict__ w,
                              const float *__restrict__ bias, float *__restrict__ y,
                              uint32_t total, WindowGeom g) {
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const uint32_t q1 = fdiv(i, g.div_wo);
    const int ow = static_cast<int>(i - q1 * g.Wo);
    const uint32_t plane = fdiv(q1, g.div_ho);
    const int oh = static_cast<int>(q1 - plane * g.Ho);
    const int c = static_cast<int>(plane - fdiv(plane, g.div_c) * g.C);
    const float *xp = x + static_cast<int64_t>(plane) * g.H * g.W;
    const float *wp = w + static_cast<int64_t>(c) * g.KH * g.KW;
    float sum = 0.0f;
    for (int kh = 0; kh < g.KH; ++kh) {
      const int ih = oh * g.sh + kh - g.ph;
      if (static_cast<unsigned>(ih) >= static_cast<unsigned>(g.H)) continue;
      for (int kw = 0; kw < g.KW; ++kw) {
        const int iw = ow * g.sw + kw - g.pw;
        if (static_cast<unsigned>(iw) < static_cast<unsigned>(g.W))
          sum += __ldg(xp + ih * g.W + iw) * __ldg(wp + kh * g.KW + kw);
      }
    }
    if (bias) sum += bias[c];
    y[i] = sum;
  }
}

// Max pooling (-inf start, padded cells skipped, npl_pooling.cpp:129-219) and
// average pooling (padded cells counted only with count_include_pad,
// npl_pooling.cpp:221-315).
template <int kType>
__global__ void pool_kernel(const float *__restrict__ x, float *__restrict__ y, uint32_t total,
                            WindowGeom g, int count_include_pad) {
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const uint32_t q1 = fdiv(i, g.div_wo);
    const int ow = static_cast<int>(i - q1 * g.Wo);
    const uint32_t plane = fdiv(q1, g.div_ho);
    const int oh = static_cast<int>(q1 - plane * g.Ho);
    const float *xp = x + static_cast<int64_t>(plane) * g.H * g.W;
    if (kType == 0) {
      float m = -CUDART_INF_F;
      for (int kh = 0; kh < g.KH; ++kh) {
        const int ih = oh * g.sh + kh - g.ph;
        if (static_cast<unsigned>(ih) >= static_cast<unsigned>(g.H)) continue;
        for (int kw = 0; kw < g.KW; ++kw) {
          const int iw = ow * g.sw + kw - g.pw;
          if (static_cast<unsigned>(iw) < static_cast<unsigned>(g.W)) {
            const float v = __ldg(xp + ih * g.W + iw);
            m = (m < v) ? v : m;  // std::max(m, v)
          }
        }
      }
      y[i] = m;
    } else {
      float s = 0.0f;
      int cnt = 0;
      for (int kh = 0; kh < g.KH; ++kh) {
        const int ih = oh * g.sh + kh - g.ph;
        const bool row_in = static_cast<unsigned>(ih) < static_cast<unsigned>(g.H);
        for (int kw = 0; kw < g.KW; ++kw) {
          const int iw = ow * g.sw + kw - g.pw;
          if (row_in && static_cast<unsigned>(iw) < static_cast<unsigned>(g.W)) {
            s += __ldg(xp + ih * g.W + iw);
            ++cnt;
          } else if (count_include_pad) {
            ++cnt;
          }
        }
      }
      y[i] = cnt > 0 ? s / static_cast<float>(cnt) : 0.0f;
    }
  }
}

// One output of window operation kOp (0 depthwise, 1 max pool, 2 average
// pool) at (oh, ow) of a plane read from xp (row pitch g.W); wp: the plane's
// filter (depthwise). Same expression and order as dwconv_kernel /
// pool_kernel.
template <int kOp, int KH_, int KW_>
__device__ __forceinline__ float window_out(const float *xp, const float *wp, int oh, int ow,
                                            const WindowGeom &g, int count_include_pad) {
  const int KH = KH_ ? KH_ : g.KH, KW = KW_ ? KW_ : g.KW;
  if (kOp == 0) {
    float sum = 0.0f;
#pragma unroll
    for (int kh = 0; kh < KH; ++kh) {
      const int ih = oh * g.sh + kh - g.ph;
      if (static_cast<unsigned>(ih) >= static_cast<unsigned>(g.H)) continue;
#pragma unroll
      for (int kw = 0; kw < KW; ++kw) {
        const int iw = ow * g.sw + kw - g.pw;
        if (static_cast<unsigned>(iw) < static_cast<unsigned>(g.W))
          sum += xp[ih * g.W + iw] * wp[kh * KW + kw];
      }
    }
    return sum;
  } else if (kOp == 1) {
    float m = -CUDART_INF_F;
#pragma unroll
    for (int kh = 0; kh < KH; ++kh) {
      const int ih = oh * g.sh + kh - g.ph;
      if (static_cast<unsigned>(ih) >= static_cast<unsigned>(g.H)) continue;
#pragma unroll
      for (int kw = 0; kw < KW; ++kw) {
        const int iw = ow * g.sw + kw - g.pw;
        if (static_cast<unsigned>(iw) < static_cast<unsigned>(g.W)) {
          const float v = xp[ih * g.W + iw];
          m = (m < v) ? v : m;  // std::max(m, v)
        }
      }
    }
    return m;
  } else {
    float s = 0.0f;
    int cnt = 0;
#pragma unroll
    for (int kh = 0; kh < KH; ++kh) {
      const int ih = oh * g.sh + kh - g.ph;
      const bool row_in = static_cast<unsigned>(ih) < static_cast<unsigned>(g.H);
#pragma unroll
      for (int kw = 0; kw < KW; ++kw) {
        const int iw = ow * g.sw + kw - g.pw;
        if (row_in && static_cast<unsigned>(iw) < static_cast<unsigned>(g.W)) {
          s += xp[ih * g.W + iw];
          ++cnt;
        } else if (count_include_pad) {
          ++cnt;
        }
      }
    }
    return cnt > 0 ? s / static_cast<float>(cnt) : 0.0f;
  }
}

constexpr int kPlaneBatchBytes = 20480;   // staged input per CTA batch (target)
constexpr int kPlaneMaxBytes = 98304;     // largest plane staged whole (2 buffers)

// Asynchronous global -> shared copies (cp.async), so that the next batch of
// planes loads while the current one is computed.
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}

__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}

__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// SW_ (1 or 2): horizontal stride of the 3x3 depthwise fast path, fixed at
// compile time so that its input patch stays in registers; 0 otherwise.
template <int kOp, int KH_, int KW_, int SW_>
__global__ void __launch_bounds__(256) plane_window_kernel(const float *__restrict__ x,
                                                           const float *__restrict__ w,
                                                           const float *__restrict__ bias,
                                                           float *__restrict__ y, int64_t planes,
                                                           int np, WindowGeom g,
                                                           int count_include_pad, int vec) {
  // Two buffers, each: np input planes, then np filters (depthwise).
  extern __shared__ float smem_planes[];
  const int KH = KH_ ? KH_ : g.KH, KW = KW_ ? KW_ : g.KW;
  const int taps = KH * KW;
  const int HW = g.H * g.W, HoWo = g.Ho * g.Wo;
  const int groups = (g.Wo + 3) >> 2;  // items of 4 outputs per output row
  const int items_pp = g.Ho * groups;
  const int buf_floats = (np * (HW + (kOp == 0 ? taps : 0)) + 3) & ~3;
  const int t = threadIdx.x;
  // Issues the asynchronous copies of the batch starting at plane q0.
  auto stage = [&](int64_t q0, float *buf) {
    const int cnt = static_cast<int>(planes - q0 < np ? planes - q0 : np);
    const float *src = x + q0 * HW;
    const int n_in = cnt * HW;
    if (vec) {
      const float4 *s4 = reinterpret_cast<const float4 *>(src);
      float4 *d4 = reinterpret_cast<float4 *>(buf);
      for (int i = t; i < (n_in >> 2); i += 256) cp_async16(d4 + i, s4 + i);
    } else {
      for (int i = t; i < n_in; i += 256) cp_async4(buf + i, src + i);
    }
    if (kOp == 0) {
      float *wb = buf + np * HW;
      for (int i = t; i < cnt * taps; i += 256) {
        const int pl = i / taps;
        const int c = static_cast<int>((q0 + pl) % g.C);
        cp_async4(wb + i, w + static_cast<int64_t>(c) * taps + (i - pl * taps));
      }
    }
    cp_async_commit();
  };
  const int64_t step = static_cast<int64_t>(gridDim.x) * np;
  int64_t p0 = static_cast<int64_t>(blockIdx.x) * np;
  if (p0 < planes) stage(p0, smem_planes);
  int cur = 0;
  for (; p0 < planes; p0 += step, cur ^= 1) {
    float *sp = smem_planes + cur * buf_floats;
    float *sw = sp + np * HW;
    const int cnt = static_cast<int>(planes - p0 < np ? planes - p0 : np);
    if (p0 + step < planes) {
      stage(p0 + step, smem_planes + (cur ^ 1) * buf_floats);
      cp_async_wait<1>();  // this batch landed; the next one may still be in flight
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (kOp == 0 && KH_ == 3 && KW_ == 3 && SW_ > 0) {
      // 3x3 depthwise: threads are split evenly over the batch's planes, so a
      // thread keeps its plane's 9 weights in registers; an item of 4
      // adjacent outputs reads its 3 x (3*sw + 3) input patch once.
      const int tpp = 256 / np;
      const int pl = t / tpp;
      if (pl < cnt) {
        const float *xp = sp + pl * HW;
        const float *wp = sw + pl * 9;
        float wr[9];
#pragma unroll
        for (int k = 0; k < 9; ++k) wr[k] = wp[k];
        const float b = bias ? __ldg(bias + (p0 + pl) % g.C) : 0.0f;
        float *yp0 = y + (p0 + pl) * HoWo;
        for (int r = t - pl * tpp; r < items_pp; r += tpp) {
          const int oh = r / groups;
          const int ow0 = (r - oh * groups) << 2;
          constexpr int kCols = 3 * SW_ + 3;  // inputs under 4 adjacent outputs
          float xr[3][kCols];
          bool rok[3], cok[kCols];
#pragma unroll
          for (int kh = 0; kh < 3; ++kh) {
            const int ih = oh * g.sh + kh - g.ph;
            rok[kh] = static_cast<unsigned>(ih) < static_cast<unsigned>(g.H);
          }
#pragma unroll
          for (int j = 0; j < kCols; ++j) {
            const int iw = ow0 * SW_ - g.pw + j;
            cok[j] = static_cast<unsigned>(iw) < static_cast<unsigned>(g.W);
          }
#pragma unroll
          for (int kh = 0; kh < 3; ++kh) {
            const int ih = oh * g.sh + kh - g.ph;
#pragma unroll
            for (int j = 0; j < kCols; ++j)
              xr[kh][j] = (rok[kh] && cok[j]) ? xp[ih * g.W + ow0 * SW_ - g.pw + j] : 0.0f;
          }
          float *yp = yp0 + oh * g.Wo;
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int ow = ow0 + q;
            if (ow >= g.Wo) break;
            float sum = 0.0f;
#pragma unroll
            for (int kh = 0; kh < 3; ++kh) {
              if (!rok[kh]) continue;
#pragma unroll
              for (int kw = 0; kw < 3; ++kw) {
                const int j = q * SW_ + kw;
                if (cok[j]) sum += xr[kh][j] * wr[kh * 3 + kw];
              }
            }
            if (bias) sum += b;
            yp[ow] = sum;
          }
        }
      }
    } else {
    for (int it = t; it < cnt * items_pp; it += 256) {
      const int pl = it / items_pp;
      const int r = it - pl * items_pp;
      const int oh = r / groups;
      const int ow0 = (r - oh * groups) << 2;
      const float *xp = sp + pl * HW;
      const float *wp = sw + pl * taps;
      float *yp = y + (p0 + pl) * HoWo + oh * g.Wo;
      float b = 0.0f;
      if (kOp == 0 && bias) b = __ldg(bias + (p0 + pl) % g.C);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int ow = ow0 + q;
        if (ow < g.Wo) {
          float v = window_out<kOp, KH_, KW_>(xp, wp, oh, ow, g, count_include_pad);
          if (kOp == 0 && bias) v += b;
          yp[ow] = v;
        }
      }
    }
    }
    __syncthreads();
  }
}

namespace {

// Planes per batch for plane_window_kernel, 0 when a plane is too large.
int plane_batch(const WindowGeom &g, int taps) {
  const int64_t plane_bytes = (static_cast<int64_t>(g.H) * g.W + taps) * 4;
  if (plane_bytes > kPlaneMaxBytes) return 0;
  int np = static_cast<int>(kPlaneBatchBytes / plane_bytes);
  if (np < 1) np = 1;
  if (np > 64) np = 64;
  return np;
}

template <int kOp>
int launch_plane(cudaStream_t s, const float *x, const float *w, const float *bias, float *y,
                 int64_t planes, const WindowGeom &g, int count_include_pad, int np) {
  const int taps = g.KH * g.KW;
  const size_t buf_floats =
      (static_cast<size_t>(np) * (static_cast<size_t>(g.H) * g.W + (kOp == 0 ? taps : 0)) + 3) &
      ~size_t(3);
  const size_t smem = 2 * buf_floats * 4;  // double buffered
  const int vec = ((g.H * g.W) % 4 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15u) == 0);
  int64_t blocks = ceil_div(planes, np);
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  if (blocks > cap) blocks = cap;
  const unsigned grid = static_cast<unsigned>(blocks);
  bool done = false;
  if constexpr (kOp == 0) {
    if (g.KH == 3 && g.KW == 3 && g.sw == 1) {
      if (int rc = ensure_dynamic_smem(reinterpret_cast<const void *>(plane_window_kernel<0, 3, 3, 1>), static_cast<int>(smem))) return rc;
      plane_window_kernel<0, 3, 3, 1><<<grid, 256, smem, s>>>(x, w, bias, y, planes, np, g,
                                                             count_include_pad, vec);
      done = true;
    } else if (g.KH == 3 && g.KW == 3 && g.sw == 2) {
      if (int rc = ensure_dynamic_smem(reinterpret_cast<const void *>(plane_window_kernel<0, 3, 3, 2>), static_cast<int>(smem))) return rc;
      plane_window_kernel<0, 3, 3, 2><<<grid, 256, smem, s>>>(x, w, bias, y, planes, np, g,
                                                             count_include_pad, vec);
      done = true;
    }
  }
  if (done) {
  } else if (g.KH == 3 && g.KW == 3) {
    if (int rc = ensure_dynamic_smem(
            reinterpret_cast<const void *>(plane_window_kernel<kOp, 3, 3, 0>), static_cast<int>(smem)))
      return rc;
    plane_window_kernel<kOp, 3, 3, 0><<<grid, 256, smem, s>>>(x, w, bias, y, planes, np, g,
                                                             count_include_pad, vec);
  } else {
    if (int rc = ensure_dynamic_smem(
            reinterpret_cast<const void *>(plane_window_kernel<kOp, 0, 0, 0>), static_cast<int>(smem)))
      return rc;
    plane_window_kernel<kOp, 0, 0, 0><<<grid, 256, smem, s>>>(x, w, bias, y, planes, np, g,
                                                             count_include_pad, vec);
  }
  count_launch();
  return launch_result();
}

}  // namespace

}  // namespace nplk

using namespace nplk;

extern "C" int nplk_depthwise_conv2d(void *stream, const nplk_conv_geom_t *g, const float *x,
                                     const float *w, const float *bias, float *out) {
  if (!g || !x || !w || !out) return kErrInvalidArg;
  if (g->n <= 0 || g->c_in <= 0 || g->h <= 0 || g->w <= 0 || g->kh <= 0 || g->kw <= 0 ||
      g->stride_h <= 0 || g->stride_w <= 0 || g->h_out <= 0 || g->w_out <= 0 ||
      g->pad_top < 0 || g->pad_left < 0)
    return kErrInvalidArg;
  const int64_t total = g->n * g->c_in * g->h_out * g->w_out;
  if (total >= (int64_t(1) << 31) || g->h * g->w >= (int64_t(1) << 31)) return kErrUnsupported;
  WindowGeom wg{};
  wg.C = static_cast<int>(g->c_in);
  wg.H = static_cast<int>(g->h);
  wg.W = static_cast<int>(g->w);
  wg.KH = static_cast<int>(g->kh);
  wg.KW = static_cast<int>(g->kw);
  wg.sh = static_cast<int>(g->stride_h);
  wg.sw = static_cast<int>(g->stride_w);
  wg.ph = static_cast<int>(g->pad_top);
  wg.pw = static_cast<int>(g->pad_left);
  wg.Ho = static_cast<int>(g->h_out);
  wg.Wo = static_cast<int>(g->w_out);
  wg.div_wo = make_fastdiv(static_cast<uint32_t>(wg.Wo));
  wg.div_ho = make_fastdiv(static_cast<uint32_t>(wg.Ho));
  wg.div_c = make_fastdiv(static_cast<uint32_t>(wg.C));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int np = plane_batch(wg, wg.KH * wg.KW);
  if (np > 0) return launch_plane<0>(s, x, w, bias, out, g->n * g->c_in, wg, 0, np);
  dwconv_kernel<<<window_grid(total), 256, 0, s>>>(x, w, bias, out,
                                                   static_cast<uint32_t>(total), wg);
  count_launch();
  return launch_result();
}

extern "C" int nplk_pool2d(void *stream, int64_t n, int64_t c, int64_t h, int64_t w,
                           int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph,
                           int64_t pw, int64_t h_out, int64_t w_out, int pool_type,
                           int count_include_pad, const float *x, float *y) {
  if (n <= 0 || c <= 0 || h <= 0 || w <= 0 || kh <= 0 || kw <= 0 || sh <= 0 || sw <= 0 ||
      ph < 0 || pw < 0 || h_out <= 0 || w_out <= 0 || !x || !y)
    return kErrInvalidArg;
  if (pool_type != 0 && pool_type != 1) return kErrInvalidArg;
  const int64_t total = n * c * h_out * w_out;
  if (total >= (int64_t(1) << 31) || h * w >= (int64_t(1) << 31)) return kErrUnsupported;
  WindowGeom wg{};
  wg.C = static_cast<int>(c);
  wg.H = static_cast<int>(h);
  wg.W = static_cast<int>(w);
  wg.KH = static_cast<int>(kh);
  wg.KW = static_cast<int>(kw);
  wg.sh = static_cast<int>(sh);
  wg.sw = static_cast<int>(sw);
  wg.ph = static_cast<int>(ph);
  wg.pw = static_cast<int>(pw);
  wg.Ho = static_cast<int>(h_out);
  wg.Wo = static_cast<int>(w_out);
  wg.div_wo = make_fastdiv(static_cast<uint32_t>(wg.Wo));
  wg.div_ho = make_fastdiv(static_cast<uint32_t>(wg.Ho));
  wg.div_c = make_fastdiv(static_cast<uint32_t>(wg.C));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int np = plane_batch(wg, 0);
  if (np > 0)
    return pool_type == 0 ? launch_plane<1>(s, x, nullptr, nullptr, y, n * c, wg,
                                            count_include_pad, np)
                          : launch_plane<2>(s, x, nullptr, nullptr, y, n * c, wg,
                                            count_include_pad, np);
  if (pool_type == 0)
    pool_kernel<0><<<window_grid(total), 256, 0, s>>>(x, y, static_cast<uint32_t>(total), wg,
                                                      count_include_pad);
  else
    pool_kernel<1><<<window_grid(total), 256, 0, s>>>(x, y, static_cast<uint32_t>(total), wg,
                                                      count_include_pad);
  count_launch();
  return launch_result();
}
