// Convolution entry points of the npl_* API
// (reference: advanced/neural_layer/src/npl_convolution.cpp:13-246, 904-991).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>

#include "npl_runtime.h"

using npl::element_count;
using npl::state;
using npl::validate_tensor;

namespace npl {
int batch_norm_training(Call &call, const npl_batchnorm_params_t *p, float *x_dev, size_t n,
                        size_t c, size_t hw, float *y_dev);
}

namespace {

// Convolution geometry exactly as PrepareConvContext derives it
// (npl_convolution.cpp:180-246): dimensions per the input's layout tag (the
// data itself is always indexed as NCHW), SAME padding from the reference's
// formula (stride-1)*in + k - stride split top/bottom, VALID and EXPLICIT
// both taking pad_h/pad_w. Returns NPL_ERR_SHAPE_MISMATCH when the padded
// input is smaller than the dilated kernel (the reference's size_t arithmetic
// would wrap there).
int conv_geometry(const npl_tensor_t *in, const npl_tensor_t *w, const npl_conv_params_t *p,
                  nplk_conv_geom_t *g) {
  if (in->ndim != 4 || w->ndim < 1) return NPL_ERR_SHAPE_MISMATCH;
  size_t N, C, H, W;
  if (in->layout == NPL_LAYOUT_NCHW) {
    N = in->shape[0];
    C = in->shape[1];
    H = in->shape[2];
    W = in->shape[3];
  } else {
    N = in->shape[0];
    H = in->shape[1];
    W = in->shape[2];
    C = in->shape[3];
  }
  size_t top, bottom, left, right;
  if (p->padding == NPL_PAD_SAME) {
    const size_t th = (p->stride_h - 1) * H + p->kernel_h - p->stride_h;
    const size_t tw = (p->stride_w - 1) * W + p->kernel_w - p->stride_w;
    top = th / 2;
    bottom = th - top;
    left = tw / 2;
    right = tw - left;
  } else {
    top = bottom = p->pad_h;
    left = right = p->pad_w;
  }
  const size_t hd = p->dilation_h * (p->kernel_h - 1) + 1;
  const size_t wd = p->dilation_w * (p->kernel_w - 1) + 1;
  if (H + top + bottom < hd || W + left + right < wd) return NPL_ERR_SHAPE_MISMATCH;
  g->n = static_cast<int64_t>(N);
  g->c_in = static_cast<int64_t>(C);
  g->h = static_cast<int64_t>(H);
  g->w = static_cast<int64_t>(W);
  g->c_out = static_cast<int64_t>(w->shape[0]);
  g->kh = static_cast<int64_t>(p->kernel_h);
  g->kw = static_cast<int64_t>(p->kernel_w);
  g->stride_h = static_cast<int64_t>(p->stride_h);
  g->stride_w = static_cast<int64_t>(p->stride_w);
  g->pad_top = static_cast<int64_t>(top);
  g->pad_left = static_cast<int64_t>(left);
  g->dil_h = static_cast<int64_t>(p->dilation_h);
  g->dil_w = static_cast<int64_t>(p->dilation_w);
  g->h_out = static_cast<int64_t>((H + top + bottom - hd) / p->stride_h + 1);
  g->w_out = static_cast<int64_t>((W + left + right - wd) / p->stride_w + 1);
  return NPL_OK;
}

bool all_fp32(const npl_tensor_t *a, const npl_tensor_t *b, const npl_tensor_t *c,
              const npl_tensor_t *d) {
  return a->dtype == NPL_DTYPE_FP32 && b->dtype == NPL_DTYPE_FP32 &&
         c->dtype == NPL_DTYPE_FP32 && (!d || d->dtype == NPL_DTYPE_FP32);
}

// Inference-mode conv on page-locked host input and output: the batch is cut
// into chunks whose host-to-device copy, conv and device-to-host copy run on
// three streams, so the PCIe transfers in both directions overlap each
// other and the kernels (a synchronous whole-batch call would copy in,
// compute and copy out one after the other). The first and last chunks are
// small (1/16 of the batch), which shortens the copy-in before the first
// conv and the copy-out after the last; the middle ones take about a quarter
// of the batch each. Same kernels and per-image results as the unchunked
// call.
constexpr size_t kPipelineMinBytes = size_t(8) << 20;
constexpr int kPipelineMaxChunks = 8;

// Chunk sizes (images) for a batch of n >= 2: {e, m, ..., m', e}.
int pipeline_chunks(int n, int *sizes) {
  const int e = n / 16 > 0 ? n / 16 : 1;
  int rest = n - 2 * e;
  int k = 0;
  sizes[k++] = e;
  if (rest > 0) {
    const int mid = (rest + 3) / 4;  // at most four middle chunks
    while (rest > 0) {
      const int c = rest < mid ? rest : mid;
      sizes[k++] = c;
      rest -= c;
    }
  }
  sizes[k++] = e;
  return k;
}

int run_conv_pipelined(const nplk_conv_geom_t &g, const npl_tensor_t *input,
                       const npl_tensor_t *weights, const npl_tensor_t *bias,
                       const npl_batchnorm_params_t *bn, int act, float act_alpha,
                       npl_tensor_t *output, npl_perf_stats_t *stats, const char *backend) {
  const size_t co = static_cast<size_t>(g.c_out);
  const size_t in_img = static_cast<size_t>(g.c_in * g.h * g.w);
  const size_t out_img = static_cast<size_t>(g.c_out * g.h_out * g.w_out);
  const size_t w_elems = static_cast<size_t>(g.c_out * g.c_in * g.kh * g.kw);
  const int n = static_cast<int>(g.n);
  int sizes[kPipelineMaxChunks];
  const int chunks = pipeline_chunks(n, sizes);
  int per = 0;
  for (int c = 0; c < chunks; ++c) per = sizes[c] > per ? sizes[c] : per;
  npl::Call call;  // binds the library's device before the lanes are made on it
  if (call.status()) return call.finish(nullptr, 0, 0, nullptr);
  npl::CopyLanes *lanes = npl::copy_lanes(2 * static_cast<size_t>(chunks) + 2);
  if (!lanes) {
    call.fail(NPL_ERR_INTERNAL);
    return call.finish(nullptr, 0, 0, nullptr);
  }
  const float *w = call.input(weights->data, w_elems * 4);
  const float *b = bias ? call.input(bias->data, co * 4) : nullptr;
  const float *mean = nullptr, *var = nullptr, *gamma = nullptr, *beta = nullptr;
  if (bn) {
    mean = call.param(bn->mean, co);
    var = call.param(bn->variance, co);
    gamma = call.param(bn->gamma, co);
    beta = call.param(bn->beta, co);
  }
  nplk_conv_geom_t gc = g;
  gc.n = per;
  const size_t ws = nplk_conv_workspace_size(&gc);
  void *work = call.scratch(ws);
  float *dx = static_cast<float *>(call.scratch(in_img * n * 4));
  float *dy = static_cast<float *>(call.scratch(out_img * n * 4));
  if (call.status()) return call.finish(nullptr, 0, 0, nullptr);
  cudaStream_t s = call.stream();
  cudaEvent_t *ev = lanes->events.data();  // [0]: buffers ready, [1]: copies out done
  cudaEvent_t *ev_in = ev + 2, *ev_done = ev + 2 + chunks;
  const float *hx = static_cast<const float *>(input->data);
  float *hy = static_cast<float *>(output->data);
  call.start_timer();
  call.fail(nplk_conv2d_prepare(s, &gc, w, b, mean, var, gamma, beta, bn ? bn->epsilon : 0.0f,
                                work, ws));
  auto ok = [&](cudaError_t e) {
    if (e != cudaSuccess) call.fail(NPL_ERR_INTERNAL);
    return e == cudaSuccess;
  };
  if (!call.status() && ok(cudaEventRecord(ev[0], s)) &&
      ok(cudaStreamWaitEvent(lanes->in, ev[0], 0)) && ok(cudaStreamWaitEvent(lanes->out, ev[0], 0))) {
    int i0 = 0;
    for (int c = 0; c < chunks && !call.status(); i0 += sizes[c], ++c) {
      const int nc = sizes[c];
      gc.n = nc;
      const size_t xo = static_cast<size_t>(i0) * in_img, yo = static_cast<size_t>(i0) * out_img;
      if (!ok(cudaMemcpyAsync(dx + xo, hx + xo, nc * in_img * 4, cudaMemcpyHostToDevice,
                              lanes->in)) ||
          !ok(cudaEventRecord(ev_in[c], lanes->in)) || !ok(cudaStreamWaitEvent(s, ev_in[c], 0)))
        break;
      call.fail(nplk_conv2d_run(s, &gc, dx + xo, act, act_alpha, dy + yo, work, ws, nullptr));
      if (call.status() || !ok(cudaEventRecord(ev_done[c], s)) ||
          !ok(cudaStreamWaitEvent(lanes->out, ev_done[c], 0)) ||
          !ok(cudaMemcpyAsync(hy + yo, dy + yo, nc * out_img * 4, cudaMemcpyDeviceToHost,
                              lanes->out)))
        break;
    }
  }
  // Everything below on the call's stream (frees, status read) waits for the
  // last copies, also after an error.
  if (cudaEventRecord(ev[1], lanes->out) != cudaSuccess || cudaStreamWaitEvent(s, ev[1], 0) != cudaSuccess) {
    cudaStreamSynchronize(lanes->out);
    cudaStreamSynchronize(lanes->in);
    call.fail(NPL_ERR_INTERNAL);
  }
  cudaEventRecord(ev[0], lanes->in);
  cudaStreamWaitEvent(s, ev[0], 0);
  call.stop_timer();
  const double flops = 2.0 * g.n * g.c_out * g.c_in * g.h_out * g.w_out * g.kh * g.kw;
  const int fused = 1 + (bn ? 1 : 0) + (act != NPLK_ACT_NONE ? 1 : 0);
  return call.finish(stats, flops, 4.0 * (in_img * n + w_elems + out_img * n), backend, fused);
}

// Runs conv (+bias) (+BN) (+act) through the implicit-GEMM kernel.
int run_conv(const npl_tensor_t *input, const npl_tensor_t *weights, const npl_tensor_t *bias,
             const npl_conv_params_t *params, const npl_batchnorm_params_t *bn, int act,
             float act_alpha, npl_tensor_t *output, npl_perf_stats_t *stats,
             const char *backend) {
  nplk_conv_geom_t g{};
  int rc = conv_geometry(input, weights, params, &g);
  if (rc) return rc;
  if (!all_fp32(input, weights, output, bias)) return NPL_ERR_UNSUPPORTED;
  const size_t in_elems = static_cast<size_t>(g.n * g.c_in * g.h * g.w);
  const size_t w_elems = static_cast<size_t>(g.c_out * g.c_in * g.kh * g.kw);
  const size_t out_elems = static_cast<size_t>(g.n * g.c_out * g.h_out * g.w_out);
  if (element_count(input) < in_elems || element_count(weights) < w_elems ||
      element_count(output) < out_elems ||
      (bias && element_count(bias) < static_cast<size_t>(g.c_out))) {
    std::fprintf(stderr, "[NPL] Error: conv tensor sizes do not match the geometry\n");
    return NPL_ERR_SHAPE_MISMATCH;
  }
  const size_t co = static_cast<size_t>(g.c_out);
  const bool train_bn = bn && bn->training;
  if (!train_bn && g.n >= 2 && in_elems * 4 >= kPipelineMinBytes &&
      npl::is_pinned_host(input->data) && npl::is_pinned_host(output->data) &&
      input->data != output->data)
    return run_conv_pipelined(g, input, weights, bias, bn, act, act_alpha, output, stats,
                              backend);
  npl::Call call;
  const float *x = call.input(input->data, in_elems * 4);
  const float *w = call.input(weights->data, w_elems * 4);
  const float *b = bias ? call.input(bias->data, co * 4) : nullptr;
  float *y = call.output(output->data, out_elems * 4);
  const float *mean = nullptr, *var = nullptr, *gamma = nullptr, *beta = nullptr;
  if (bn && !train_bn) {
    mean = call.param(bn->mean, co);
    var = call.param(bn->variance, co);
    gamma = call.param(bn->gamma, co);
    beta = call.param(bn->beta, co);
  }
  // NPL_AUTOTUNE=1: a geometry without a tile-configuration cache entry is
  // tuned on this call (every conv kernel timed, the fastest cached), which
  // needs the workspace of the largest candidate.
  const bool tune = npl::autotune_mode() && !npl::conv_tuned(&g);
  size_t ws = nplk_conv_workspace_size(&g);
  if (tune)
    for (int a = NPLK_CONV_ALGO_DIRECT; a <= NPLK_CONV_ALGO_WINDOW_PAIR; ++a)
      ws = std::max(ws, nplk_conv_workspace_size_algo(&g, a));
  void *work = call.scratch(ws);
  if (call.status()) return call.finish(nullptr, 0, 0, nullptr);
  call.start_timer();
  const float eps = bn ? bn->epsilon : 0.0f;
  const int conv_act = train_bn ? NPLK_ACT_NONE : act;
  if (tune) {
    int algo = 0;
    call.fail(nplk_conv2d_tune(call.stream(), &g, x, w, b, mean, var, gamma, beta, eps, conv_act,
                               act_alpha, y, work, ws, 3, &algo, nullptr));
  } else {
    call.fail(nplk_conv2d_fused(call.stream(), &g, x, w, b, mean, var, gamma, beta, eps,
                                conv_act, act_alpha, y, work, ws, nullptr));
  }
  int fused = 1 + (bn ? 1 : 0) + (act != NPLK_ACT_NONE ? 1 : 0);
  if (train_bn && !call.status()) {
    // Training-mode BN needs batch statistics of the conv output, so it runs
    // as separate passes after the conv.
    call.fail(npl::batch_norm_training(call, bn, y, static_cast<size_t>(g.n), co,
                                       static_cast<size_t>(g.h_out * g.w_out), y));
    if (act != NPLK_ACT_NONE && !call.status())
      call.fail(nplk_activation(call.stream(), static_cast<int64_t>(out_elems), y, y, act,
                                act_alpha, 0));
    fused = 1;
  }
  call.stop_timer();
  const double flops = 2.0 * g.n * g.c_out * g.c_in * g.h_out * g.w_out * g.kh * g.kw;
  return call.finish(stats, flops, 4.0 * (in_elems + w_elems + out_elems), backend, fused);
}

// Activation code for the fused epilogue; LeakyReLU through the enum uses the
// reference's fixed slope 0.01 (npl_activation_norm.cpp:213), and the scalar
// ReLU formulas apply when vectorisation is disabled in the config.
int epilogue_act(npl_activation_t a, float *alpha) {
  *alpha = 0.01f;
  if (!state().config.enable_vectorization) {
    if (a == NPL_ACT_RELU) return 101;
    if (a == NPL_ACT_RELU6) return 102;
    if (a == NPL_ACT_SOFTPLUS) return 110;
  }
  return static_cast<int>(a);
}

}  // namespace

extern "C" int npl_conv2d(const npl_tensor_t *input, const npl_tensor_t *weights,
                          const npl_tensor_t *bias, const npl_conv_params_t *params,
                          npl_tensor_t *output, npl_perf_stats_t *stats) {
  if (!state().initialized) return NPL_ERR_NOT_INITIALIZED;
  int rc = validate_tensor(input, "input");
  if (rc) return rc;
  rc = validate_tensor(weights, "weights");
  if (rc) return rc;
  rc = validate_tensor(output, "output");
  if (rc) return rc;
  if (bias) {
    rc = validate_tensor(bias, "bias");
    if (rc) return rc;
  }
  rc = npl::validate_conv_params(params);
  if (rc) return rc;
  // One implicit-GEMM kernel covers all of the reference's algorithms
  // (Winograd for 3x3/s1, direct, and the im2col path it cannot execute).
  return run_conv(input, weights, bias, params, nullptr, NPLK_ACT_NONE, 0.0f, output, stats,
                  "B200-tcgen05-igemm-3xTF32");
}

extern "C" int npl_conv2d_bn_activation(const npl_tensor_t *input,
                                        const npl_tensor_t *weights, const npl_tensor_t *bias,
                                        const npl_conv_params_t *conv_params,
                                        const npl_batchnorm_params_t *bn_params,
                                        npl_activation_t activation, npl_tensor_t *output,
                                        npl_perf_stats_t *stats) {
  if (!state().initialized) return NPL_ERR_NOT_INITIALIZED;
  int rc = validate_tensor(input, "input");
  if (rc) return rc;
  rc = validate_tensor(weights, "weights");
  if (rc) return rc;
  rc = validate_tensor(output, "output");
  if (rc) return rc;
  if (bias) {
    rc = validate_tensor(bias, "bias");
    if (rc) return rc;
  }
  rc = npl::validate_conv_params(conv_params);
  if (rc) return rc;
  if (bn_params && (!bn_params->mean || !bn_params->variance)) return NPL_ERR_INVALID_ARG;
  if (static_cast<int>(activation) < 0 || static_cast<int>(activation) > 10)
    return NPL_ERR_INVALID_ARG;
  float alpha = 0.0f;
  const int act = epilogue_act(activation, &alpha);
  return run_conv(input, weights, bias, conv_params, bn_params, act, alpha, output, stats,
                  "B200-tcgen05-igemm-3xTF32+BN+act");
}

extern "C" int npl_depthwise_conv2d(const npl_tensor_t *input, const npl_tensor_t *weights,
                                    const npl_tensor_t *bias, const npl_conv_params_t *params,
                                    npl_tensor_t *output, npl_perf_stats_t *stats) {
  if (!state().initialized) return NPL_ERR_NOT_INITIALIZED;
  int rc = validate_tensor(input, "input");
  if (rc) return rc;
  rc = validate_tensor(weights, "weights");
  if (rc) return rc;
  rc = validate_tensor(output, "output");
  if (rc) return rc;
  if (bias) {
    rc = validate_tensor(bias, "bias");
    if (rc) return rc;
  }
  // The reference runs without checking the parameters; zero kernel or
  // stride values would divide by zero there, here they are rejected.
  if (!params || params->kernel_h == 0 || params->kernel_w == 0 || params->stride_h == 0 ||
      params->stride_w == 0)
    return NPL_ERR_INVALID_ARG;
  nplk_conv_geom_t g{};
  rc = conv_geometry(input, weights, params, &g);
  if (rc) return rc;
  if (!all_fp32(input, weights, output, bias)) return NPL_ERR_UNSUPPORTED;
  g.c_out = g.c_in;
  const size_t in_elems = static_cast<size_t>(g.n * g.c_in * g.h * g.w);
  const size_t w_elems = static_cast<size_t>(g.c_in * g.kh * g.kw);
  const size_t out_elems = static_cast<size_t>(g.n * g.c_in * g.h_out * g.w_out);
  if (element_count(input) < in_elems || element_count(weights) < w_elems ||
      element_count(output) < out_elems ||
      (bias && element_count(bias) < static_cast<size_t>(g.c_in)))
    return NPL_ERR_SHAPE_MISMATCH;
  npl::Call call;
  const float *x = call.input(input->data, in_elems * 4);
  const float *w = call.input(weights->data, w_elems * 4);
  const float *b = bias ? call.input(bias->data, static_cast<size_t>(g.c_in) * 4) : nullptr;
  float *y = call.output(output->data, out_elems * 4);
  if (call.status()) return call.finish(nullptr, 0, 0, nullptr);
  call.start_timer();
  call.fail(nplk_depthwise_conv2d(call.stream(), &g, x, w, b, y));
  call.stop_timer();
  const double flops = 2.0 * g.n * g.c_in * g.h_out * g.w_out * g.kh * g.kw;
  return call.finish(stats, flops, 4.0 * (in_elems + w_elems + out_elems),
                     "B200-depthwise");
}

extern "C" int npl_conv2d_output_shape(const size_t *input_shape,
                                       const npl_conv_params_t *params, size_t *output_shape) {
  // npl_convolution.cpp:139-172, including its conventions: channel slot
  // copied from the input, explicit pads only for NPL_PAD_EXPLICIT.
  if (!input_shape || !params || !output_shape) return NPL_ERR_INVALID_ARG;
  const size_t N = input_shape[0], C = input_shape[1], H = input_shape[2],
               W = input_shape[3];
  const size_t ph = params->padding == NPL_PAD_EXPLICIT ? params->pad_h : 0;
  const size_t pw = params->padding == NPL_PAD_EXPLICIT ? params->pad_w : 0;
  if (params->stride_h == 0 || params->stride_w == 0) return NPL_ERR_INVALID_ARG;
  output_shape[0] = N;
  output_shape[1] = C;
  if (params->padding == NPL_PAD_SAME) {
    output_shape[2] = (H + params->stride_h - 1) / params->stride_h;
    output_shape[3] = (W + params->stride_w - 1) / params->stride_w;
  } else {
    const size_t hd = params->dilation_h * (params->kernel_h - 1) + 1;
    const size_t wd = params->dilation_w * (params->kernel_w - 1) + 1;
    output_shape[2] = (H + 2 * ph - hd) / params->stride_h + 1;
    output_shape[3] = (W + 2 * pw - wd) / params->stride_w + 1;
  }
  return NPL_OK;
}
