// Activation, normalisation and pooling entry points of the npl_* API
// (reference: advanced/neural_layer/src/npl_activation_norm.cpp:13-182 and
// npl_pooling.cpp:12-127).
#include <cuda_runtime.h>

#include <cstdio>

#include "npl_runtime.h"

using npl::element_count;
using npl::state;
using npl::validate_tensor;

namespace npl {

// Training-mode batch norm (ExecuteBatchNormTraining,
// npl_activation_norm.cpp:409-468): batch statistics over N*H*W per channel
// (biased variance), running statistics updated in place with
// momentum*old + (1-momentum)*batch, then normalisation with the batch
// statistics. Runs on the call's stream; x_dev and y_dev may alias.
int batch_norm_training(Call &call, const npl_batchnorm_params_t *p, float *x_dev, size_t n,
                        size_t c, size_t hw, float *y_dev) {
  float *stats = static_cast<float *>(call.scratch(2 * c * sizeof(float)));
  float *run_mean = call.param_out(const_cast<float *>(p->mean), c);
  float *run_var = call.param_out(const_cast<float *>(p->variance), c);
  const float *gamma = call.param(p->gamma, c);
  const float *beta = call.param(p->beta, c);
  if (call.status()) return call.status();
  int rc = nplk_batch_norm_stats(call.stream(), n, c, hw, x_dev, stats, stats + c);
  if (rc) return rc;
  rc = nplk_bn_update_running(call.stream(), c, run_mean, run_var, stats, stats + c,
                              p->momentum);
  if (rc) return rc;
  return nplk_batch_norm_infer(call.stream(), n, c, hw, x_dev, y_dev, stats, stats + c, gamma,
                               beta, p->epsilon);
}

}  // namespace npl

namespace {

int run_activation(const npl_tensor_t *input, int act, float alpha, npl_tensor_t *output,
                   npl_perf_stats_t *stats, bool scalar) {
  const size_t n = element_count(input);
  if (element_count(output) < n) return NPL_ERR_SHAPE_MISMATCH;
  if (input->dtype != NPL_DTYPE_FP32 || output->dtype != NPL_DTYPE_FP32)
    return NPL_ERR_UNSUPPORTED;
  npl::Call call;
  const float *x = call.input(input->data, n * 4);
  float *y = call.output(output->data, n * 4);
  if (call.status()) return call.finish(nullptr, 0, 0, nullptr);
  call.start_timer();
  call.fail(nplk_activation(call.stream(), static_cast<int64_t>(n), x, y, act, alpha,
                            scalar ? 1 : 0));
  call.stop_timer();
  return call.finish(stats, 0.0, 8.0 * n, "B200-elementwise");
}

}  // namespace

extern "C" int npl_activation(const npl_tensor_t *input, npl_activation_t activation,
                              npl_tensor_t *output, npl_perf_stats_t *stats) {
  if (!state().initialized) return NPL_ERR_NOT_INITIALIZED;
  int rc = validate_tensor(input, "input");
  if (rc) return rc;
  rc = validate_tensor(output, "output");
  if (rc) return rc;
  if (static_cast<int>(activation) < 0 || static_cast<int>(activation) > 10)
    return NPL_ERR_INVALID_ARG;
  if (activation == NPL_ACT_NONE) {
    // Copy when the buffers differ (npl_activation_norm.cpp:25-31).
    if (input->data == output->data) return NPL_OK;
    const size_t n = element_count(input);
    if (element_count(output) < n) return NPL_ERR_SHAPE_MISMATCH;
    npl::Call call;
    const float *x = call.input(input->data, n * 4);
    float *y = call.output(output->data, n * 4);
    if (call.status()) return call.finish(nullptr, 0, 0, nullptr);
    call.start_timer();
    call.fail(nplk_activation(call.stream(), static_cast<int64_t>(n), x, y, 0, 0.0f, 0));
    call.stop_timer();
    return call.finish(stats, 0.0, 8.0 * n, "B200-copy");
  }
  // LeakyReLU reached through the enum uses slope 0.01 (:213); the scalar
  // formulas apply when vectorisation is disabled (:34-38).
  return run_activation(input, static_cast<int>(activation), 0.01f, output, stats,
                        !state().config.enable_vectorization);
}

extern "C" int npl_relu(const npl_tensor_t *input, npl_tensor_t *output,
                        npl_perf_stats_t *stats) {
  return npl_activation(input, NPL_ACT_RELU, output, stats);
}

extern "C" int npl_leaky_relu(const npl_tensor_t *input, float alpha, npl_tensor_t *output,
                              npl_perf_stats_t *stats) {
  if (!state().initialized) return NPL_ERR_NOT_INITIALIZED;
  int rc = validate_tensor(input, "input");
  if (rc) return rc;
  rc = validate_tensor(output, "output");
  if (rc) return rc;
  return run_activation(input, NPL_ACT_LEAKY_RELU, alpha, output, stats, false);
}

extern "C" int npl_softmax(const npl_tensor_t *input, int axis, npl_tensor_t *output,
                           npl_perf_stats_t *stats) {
  if (!state().initialized) return NPL_ERR_NOT_INITIALIZED;
  int rc = validate_tensor(input, "input");
  if (rc) return rc;
  rc = validate_tensor(output, "output");
  if (rc) return rc;
  if (axis < 0) axis += static_cast<int>(input->ndim);
  if (axis < 0 || axis >= static_cast<int>(input->ndim)) return NPL_ERR_INVALID_ARG;
  size_t outer = 1, inner = 1;
  for (int i = 0; i < axis; ++i) outer *= input->shape[i];
  for (size_t i = axis + 1; i < input->ndim; ++i) inner *= input->shape[i];
  const size_t len = input->shape[axis];
  const size_t n = outer * len * inner;
  if (element_count(output) < n) return NPL_ERR_SHAPE_MISMATCH;
  npl::Call call;
  const float *x = call.input(input->data, n * 4);
  float *y = call.output(output->data, n * 4);
  if (call.status()) return call.finish(nullptr, 0, 0, nullptr);
  call.start_timer();
  call.fail(nplk_softmax(call.stream(), static_cast<int64_t>(outer),
                         static_cast<int64_t>(len), static_cast<int64_t>(inner), x, y));
  call.stop_timer();
  return call.finish(stats, 0.0, 8.0 * n, "B200-softmax");
}

extern "C" int npl_batch_norm(const npl_tensor_t *input, const npl_batchnorm_params_t *params,
                              npl_tensor_t *output, npl_perf_stats_t *stats) {
  if (!state().initialized) return NPL_ERR_NOT_INITIALIZED;
  int rc = validate_tensor(input, "input");
  if (rc) return rc;
  rc = validate_tensor(output, "output");
  if (rc) return rc;
  if (!params || !params->mean || !params->variance) return NPL_ERR_INVALID_ARG;
  if (input->ndim != 4) return NPL_ERR_SHAPE_MISMATCH;
  const size_t n = input->shape[0], c = input->shape[1], hw = input->shape[2] * input->shape[3];
  const size_t total = n * c * hw;
  if (element_count(output) < total) return NPL_ERR_SHAPE_MISMATCH;
  npl::Call call;
  float *x = call.input(input->data, total * 4);
  float *y = call.output(output->data, total * 4);
  if (call.status()) return call.finish(nullptr, 0, 0, nullptr);
  call.start_timer();
  if (params->training) {
    call.fail(npl::batch_norm_training(call, params, x, n, c, hw, y));
  } else {
    const float *mean = call.param(params->mean, c);
    const float *var = call.param(params->variance, c);
    const float *gamma = call.param(params->gamma, c);
    const float *beta = call.param(params->beta, c);
    if (!call.status())
      call.fail(nplk_batch_norm_infer(call.stream(), n, c, hw, x, y, mean, var, gamma, beta,
                                      params->epsilon));
  }
  call.stop_timer();
  return call.finish(stats, 0.0, 8.0 * total, "B200-batchnorm");
}

extern "C" int npl_layer_norm(const npl_tensor_t *input, const npl_layernorm_params_t *params,
                              npl_tensor_t *output, npl_perf_stats_t *stats) {
  if (!state().initialized) return NPL_ERR_NOT_INITIALIZED;
  int rc = validate_tensor(input, "input");
  if (rc) return rc;
  rc = validate_tensor(output, "output");
  if (rc) return rc;
  if (!params) return NPL_ERR_INVALID_ARG;
  // A zero normalized_shape divides by zero in the reference; rejected here.
  if (params->normalized_shape == 0) return NPL_ERR_INVALID_ARG;
  const size_t cols = params->normalized_shape;
  const size_t rows = element_count(input) / cols;
  if (rows == 0) return NPL_OK;
  const size_t n = rows * cols;
  if (element_count(output) < n) return NPL_ERR_SHAPE_MISMATCH;
  npl::Call call;
  const float *x = call.input(input->data, n * 4);
  float *y = call.output(output->data, n * 4);
  const float *gamma = call.param(params->gamma, cols);
  const float *beta = call.param(params->beta, cols);
  if (call.status()) return call.finish(nullptr, 0, 0, nullptr);
  call.start_timer();
  call.fail(nplk_layer_norm(call.stream(), static_cast<int64_t>(rows),
                            static_cast<int64_t>(cols), x, y, gamma, beta, params->epsilon));
  call.stop_timer();
  return call.finish(stats, 0.0, 8.0 * n, "B200-layernorm");
}

namespace {

int run_gap(const npl_tensor_t *input, npl_tensor_t *output, npl_perf_stats_t *stats) {
  if (input->ndim != 4) return NPL_ERR_SHAPE_MISMATCH;
  const size_t planes = input->shape[0] * input->shape[1];
  const size_t hw = input->shape[2] * input->shape[3];
  // The reference writes [N,C,1,1] or [N,C] outputs and nothing otherwise
  // (npl_pooling.cpp:372-375).
  if (output->ndim != 4 && output->ndim != 2) return NPL_OK;
  if (element_count(output) < planes) return NPL_ERR_SHAPE_MISMATCH;
  npl::Call call;
  const float *x = call.input(input->data, planes * hw * 4);
  float *y = call.output(output->data, planes * 4);
  if (call.status()) return call.finish(nullptr, 0, 0, nullptr);
  call.start_timer();
  call.fail(nplk_global_avg_pool(call.stream(), static_cast<int64_t>(planes),
                                 static_cast<int64_t>(hw), x, y));
  call.stop_timer();
  return call.finish(stats, 0.0, 4.0 * (planes * hw + planes), "B200-gap");
}

}  // namespace

extern "C" int npl_pooling(const npl_tensor_t *input, const npl_pooling_params_t *params,
                           npl_tensor_t *output, npl_perf_stats_t *stats) {
  if (!state().initialized) return NPL_ERR_NOT_INITIALIZED;
  int rc = validate_tensor(input, "input");
  if (rc) return rc;
  rc = validate_tensor(output, "output");
  if (rc) return rc;
  // ValidatePoolingParams (npl_pooling.cpp:407-424).
  if (!params) return NPL_ERR_INVALID_ARG;
  const bool global = params->type == NPL_POOL_GLOBAL_AVG || params->type == NPL_POOL_GLOBAL_MAX;
  if (!global && (params->kernel_h == 0 || params->kernel_w == 0 || params->stride_h == 0 ||
                  params->stride_w == 0))
    return NPL_ERR_INVALID_ARG;
  // The context below divides by the strides even for the global types; a
  // zero stride would fault in the reference and is rejected here.
  if (params->stride_h == 0 || params->stride_w == 0) return NPL_ERR_INVALID_ARG;
  // PreparePoolingContext (:95-127): NCHW input, exact output shape.
  if (input->ndim != 4) return NPL_ERR_SHAPE_MISMATCH;
  const size_t N = input->shape[0], C = input->shape[1], H = input->shape[2],
               W = input->shape[3];
  const size_t he = H + 2 * params->pad_h, we = W + 2 * params->pad_w;
  const size_t ho = (he - params->kernel_h) / params->stride_h + 1;
  const size_t wo = (we - params->kernel_w) / params->stride_w + 1;
  if (output->ndim < 4 || output->shape[0] != N || output->shape[1] != C ||
      output->shape[2] != ho || output->shape[3] != wo)
    return NPL_ERR_SHAPE_MISMATCH;
  if (params->type == NPL_POOL_GLOBAL_AVG) return run_gap(input, output, stats);
  if (params->type != NPL_POOL_MAX && params->type != NPL_POOL_AVG &&
      params->type != NPL_POOL_GLOBAL_MAX)
    return NPL_ERR_UNSUPPORTED;
  // GLOBAL_MAX falls back to windowed max pooling with the given parameters,
  // as in the reference (:40-43).
  if (he < params->kernel_h || we < params->kernel_w) return NPL_ERR_SHAPE_MISMATCH;
  const int type = params->type == NPL_POOL_AVG ? 1 : 0;
  const size_t in_n = N * C * H * W, out_n = N * C * ho * wo;
  npl::Call call;
  const float *x = call.input(input->data, in_n * 4);
  float *y = call.output(output->data, out_n * 4);
  if (call.status()) return call.finish(nullptr, 0, 0, nullptr);
  call.start_timer();
  call.fail(nplk_pool2d(call.stream(), N, C, H, W, params->kernel_h, params->kernel_w,
                        params->stride_h, params->stride_w, params->pad_h, params->pad_w, ho,
                        wo, type, params->count_include_pad, x, y));
  call.stop_timer();
  return call.finish(stats, 0.0, 4.0 * (in_n + out_n), type ? "B200-avgpool" : "B200-maxpool");
}

extern "C" int npl_global_avg_pool(const npl_tensor_t *input, npl_tensor_t *output,
                                   npl_perf_stats_t *stats) {
  if (!state().initialized) return NPL_ERR_NOT_INITIALIZED;
  int rc = validate_tensor(input, "input");
  if (rc) return rc;
  rc = validate_tensor(output, "output");
  if (rc) return rc;
  return run_gap(input, output, stats);
}
