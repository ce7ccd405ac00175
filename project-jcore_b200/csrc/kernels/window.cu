// Sliding-window kernels over NCHW planes: depthwise convolution and max /
// average pooling. One thread per output element; consecutive threads take
// consecutive output columns, so the window reads of a warp fall on a few
// adjacent cache lines and are served from L1 after the first touch. Each
// input element therefore crosses HBM about once.
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
  if (pool_type == 0)
    pool_kernel<0><<<window_grid(total), 256, 0, s>>>(x, y, static_cast<uint32_t>(total), wg,
                                                      count_include_pad);
  else
    pool_kernel<1><<<window_grid(total), 256, 0, s>>>(x, y, static_cast<uint32_t>(total), wg,
                                                      count_include_pad);
  count_launch();
  return launch_result();
}
