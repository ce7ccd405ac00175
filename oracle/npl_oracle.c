/* CPU restatement of the reference NPL hot path. TEST INFRASTRUCTURE ONLY
 * (see npl_oracle.h). Parity pinned against the compiled reference
 * (oracle/_ref/libnpl_ref.so) and the golden fixtures in tests/golden/. */
#include "npl_oracle.h"

#include <math.h>
#include <omp.h>
#include <stddef.h>
#include <stdlib.h>

void oracle_set_threads(int n) { omp_set_num_threads(n > 0 ? n : 1); }

void oracle_sgemm(int64_t M, int64_t N, int64_t K, float alpha, const float *A, int64_t lda,
                  const float *B, int64_t ldb, float beta, float *C, int64_t ldc) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < M; ++i) {
    double *acc = (double *)calloc((size_t)N, sizeof(double));
    for (int64_t k = 0; k < K; ++k) {
      const double a = (double)A[i * lda + k];
      const float *b = B + k * ldb;
      for (int64_t j = 0; j < N; ++j) acc[j] += a * (double)b[j];
    }
    for (int64_t j = 0; j < N; ++j) {
      double v = (double)alpha * acc[j];
      if (beta != 0.0f) v += (double)beta * (double)C[i * ldc + j];
      C[i * ldc + j] = (float)v;
    }
    free(acc);
  }
}

void oracle_conv2d(const float *x, int64_t N, int64_t C, int64_t H, int64_t W, const float *w,
                   int64_t Cout, int64_t KH, int64_t KW, int64_t sh, int64_t sw, int64_t pt,
                   int64_t pl, int64_t dh, int64_t dw, int64_t Ho, int64_t Wo,
                   const float *bias, float *out) {
#pragma omp parallel for schedule(static)
  for (int64_t idx = 0; idx < N * Cout; ++idx) {
    const int64_t n = idx / Cout, oc = idx % Cout;
    for (int64_t oh = 0; oh < Ho; ++oh) {
      for (int64_t ow = 0; ow < Wo; ++ow) {
        float sum = 0.0f;
        for (int64_t ic = 0; ic < C; ++ic) {
          for (int64_t kh = 0; kh < KH; ++kh) {
            for (int64_t kw = 0; kw < KW; ++kw) {
              const int64_t ih = oh * sh + kh * dh - pt;
              const int64_t iw = ow * sw + kw * dw - pl;
              if (ih >= 0 && ih < H && iw >= 0 && iw < W)
                sum += x[((n * C + ic) * H + ih) * W + iw] * w[((oc * C + ic) * KH + kh) * KW + kw];
            }
          }
        }
        out[((n * Cout + oc) * Ho + oh) * Wo + ow] = sum;
      }
    }
    if (bias) {
      float *o = out + (n * Cout + oc) * Ho * Wo;
      for (int64_t i = 0; i < Ho * Wo; ++i) o[i] += bias[oc];
    }
  }
}

void oracle_depthwise_conv2d(const float *x, int64_t N, int64_t C, int64_t H, int64_t W,
                             const float *w, int64_t KH, int64_t KW, int64_t sh, int64_t sw,
                             int64_t pt, int64_t pl, int64_t Ho, int64_t Wo, const float *bias,
                             float *out) {
#pragma omp parallel for schedule(static)
  for (int64_t idx = 0; idx < N * C; ++idx) {
    const int64_t c = idx % C;
    for (int64_t oh = 0; oh < Ho; ++oh) {
      for (int64_t ow = 0; ow < Wo; ++ow) {
        float sum = 0.0f;
        for (int64_t kh = 0; kh < KH; ++kh) {
          for (int64_t kw = 0; kw < KW; ++kw) {
            const int64_t ih = oh * sh + kh - pt, iw = ow * sw + kw - pl;
            if (ih >= 0 && ih < H && iw >= 0 && iw < W)
              sum += x[(idx * H + ih) * W + iw] * w[(c * KH + kh) * KW + kw];
          }
        }
        out[(idx * Ho + oh) * Wo + ow] = sum;
      }
    }
    if (bias) {
      float *o = out + idx * Ho * Wo;
      for (int64_t i = 0; i < Ho * Wo; ++i) o[i] += bias[c];
    }
  }
}

void oracle_batch_norm(const float *x, int64_t N, int64_t C, int64_t HW, const float *mean,
                       const float *var, const float *gamma, const float *beta, float eps,
                       float *out) {
#pragma omp parallel for schedule(static)
  for (int64_t idx = 0; idx < N * C; ++idx) {
    const int64_t c = idx % C;
    const float m = mean[c], g = gamma ? gamma[c] : 1.0f, b = beta ? beta[c] : 0.0f;
    const float inv_std = 1.0f / sqrtf(var[c] + eps);
    for (int64_t i = 0; i < HW; ++i) out[idx * HW + i] = g * (x[idx * HW + i] - m) * inv_std + b;
  }
}

void oracle_batch_norm_train(const float *x, int64_t N, int64_t C, int64_t HW, float *run_mean,
                             float *run_var, const float *gamma, const float *beta, float eps,
                             float momentum, float *out) {
  float *bm = (float *)__builtin_alloca((size_t)C * sizeof(float));
  float *bv = (float *)__builtin_alloca((size_t)C * sizeof(float));
  const int64_t cnt = N * HW;
  for (int64_t c = 0; c < C; ++c) {
    float s = 0.0f;
    for (int64_t n = 0; n < N; ++n)
      for (int64_t i = 0; i < HW; ++i) s += x[(n * C + c) * HW + i];
    bm[c] = s / (float)cnt;
  }
  for (int64_t c = 0; c < C; ++c) {
    float s = 0.0f;
    for (int64_t n = 0; n < N; ++n)
      for (int64_t i = 0; i < HW; ++i) {
        const float d = x[(n * C + c) * HW + i] - bm[c];
        s += d * d;
      }
    bv[c] = s / (float)cnt;
  }
  for (int64_t c = 0; c < C; ++c) {
    run_mean[c] = momentum * run_mean[c] + (1.0f - momentum) * bm[c];
    run_var[c] = momentum * run_var[c] + (1.0f - momentum) * bv[c];
  }
  oracle_batch_norm(x, N, C, HW, bm, bv, gamma, beta, eps, out);
}

static float act_one(float x, int act, float alpha, int scalar) {
  switch (act) {
    case 1: /* vectorised: std::max(x, 0); scalar: x > 0 ? x : 0 */
      return scalar ? (x > 0.0f ? x : 0.0f) : (x < 0.0f ? 0.0f : x);
    case 2:
      if (scalar) {
        const float t = 0.0f < x ? x : 0.0f;
        return 6.0f < t ? 6.0f : t;
      } else {
        const float t = x < 0.0f ? 0.0f : x;
        return 6.0f < t ? 6.0f : t;
      }
    case 3:
      return tanhf(x);
    case 4:
      return 1.0f / (1.0f + expf(-x));
    case 5: {
      const float x3 = x * x * x;
      return 0.5f * x * (1.0f + tanhf(0.7978845608f * (x + 0.044715f * x3)));
    }
    case 6:
      return x * (1.0f / (1.0f + expf(-x)));
    case 7:
      return x > 0.0f ? x : alpha * x;
    case 8:
      return x > 0.0f ? x : 1.0f * (expf(x) - 1.0f);
    case 9:
      return 1.05070098f * (x > 0.0f ? x : 1.67326324f * (expf(x) - 1.0f));
    case 10:
      return scalar ? logf(1.0f + expf(x)) : log1pf(expf(x));
    default:
      return x;
  }
}

void oracle_activation(const float *x, int64_t n, int act, float alpha, int scalar, float *out) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) out[i] = act_one(x[i], act, alpha, scalar);
}

void oracle_softmax(const float *x, int64_t outer, int64_t axis_len, int64_t inner, float *out) {
#pragma omp parallel for schedule(static)
  for (int64_t idx = 0; idx < outer * inner; ++idx) {
    const int64_t o = idx / inner, in = idx % inner;
    float mx = -INFINITY;
    for (int64_t i = 0; i < axis_len; ++i) {
      const float v = x[(o * axis_len + i) * inner + in];
      mx = (mx < v) ? v : mx;
    }
    float sum = 0.0f;
    for (int64_t i = 0; i < axis_len; ++i) {
      const int64_t off = (o * axis_len + i) * inner + in;
      const float e = expf(x[off] - mx);
      out[off] = e;
      sum += e;
    }
    for (int64_t i = 0; i < axis_len; ++i) out[(o * axis_len + i) * inner + in] /= sum;
  }
}

void oracle_layer_norm(const float *x, int64_t rows, int64_t cols, const float *gamma,
                       const float *beta, float eps, float *out) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const float *xr = x + r * cols;
    float mean = 0.0f;
    for (int64_t j = 0; j < cols; ++j) mean += xr[j];
    mean /= (float)cols;
    float var = 0.0f;
    for (int64_t j = 0; j < cols; ++j) {
      const float d = xr[j] - mean;
      var += d * d;
    }
    var /= (float)cols;
    const float inv_std = 1.0f / sqrtf(var + eps);
    for (int64_t j = 0; j < cols; ++j) {
      const float g = gamma ? gamma[j] : 1.0f, b = beta ? beta[j] : 0.0f;
      out[r * cols + j] = g * ((xr[j] - mean) * inv_std) + b;
    }
  }
}

void oracle_pool2d(const float *x, int64_t N, int64_t C, int64_t H, int64_t W, int64_t KH,
                   int64_t KW, int64_t sh, int64_t sw, int64_t ph, int64_t pw, int64_t Ho,
                   int64_t Wo, int type, int count_include_pad, float *out) {
#pragma omp parallel for schedule(static)
  for (int64_t idx = 0; idx < N * C; ++idx) {
    const float *xp = x + idx * H * W;
    for (int64_t oh = 0; oh < Ho; ++oh) {
      for (int64_t ow = 0; ow < Wo; ++ow) {
        float m = -INFINITY, s = 0.0f;
        int cnt = 0;
        for (int64_t kh = 0; kh < KH; ++kh) {
          for (int64_t kw = 0; kw < KW; ++kw) {
            const int64_t ih = oh * sh + kh - ph, iw = ow * sw + kw - pw;
            if (ih >= 0 && ih < H && iw >= 0 && iw < W) {
              const float v = xp[ih * W + iw];
              m = (m < v) ? v : m;
              s += v;
              ++cnt;
            } else if (count_include_pad) {
              ++cnt;
            }
          }
        }
        out[(idx * Ho + oh) * Wo + ow] = type == 0 ? m : (cnt > 0 ? s / (float)cnt : 0.0f);
      }
    }
  }
}

void oracle_global_avg_pool(const float *x, int64_t planes, int64_t hw, float *out) {
  const int64_t simd = 8;
#pragma omp parallel for schedule(static)
  for (int64_t p = 0; p < planes; ++p) {
    const float *xp = x + p * hw;
    float part[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const int64_t vec_end = (hw / simd) * simd;
    for (int64_t i = 0; i < vec_end; i += simd)
      for (int64_t j = 0; j < simd; ++j) part[j] += xp[i + j];
    float sum = 0.0f;
    for (int64_t j = 0; j < simd; ++j) sum += part[j];
    for (int64_t i = vec_end; i < hw; ++i) sum += xp[i];
    out[p] = sum / (float)hw;
  }
}
