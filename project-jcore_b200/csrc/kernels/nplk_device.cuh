// Device-side helpers shared by the NPL kernels: activation formulas.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace nplk {

// Division by a loop-invariant divisor d >= 1 for dividends n < 2^31:
// q = (n * m) >> s with s = 31 + ceil(log2 d) and m = ceil(2^s / d). The
// rounding error m*d - 2^s < d and 2^s >= 2^31 * d make the quotient exact
// for every n < 2^31 (round-up method of Granlund & Montgomery, 1994).
struct FastDiv {
  uint64_t m;
  uint32_t s;
  uint32_t d;
};

inline FastDiv make_fastdiv(uint32_t d) {
  FastDiv f;
  uint32_t l = 0;
  while ((uint64_t(1) << l) < d) ++l;
  f.s = 31 + l;
  f.m = ((uint64_t(1) << f.s) + d - 1) / d;
  f.d = d;
  return f;
}

__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv &f) {
  return static_cast<uint32_t>((static_cast<uint64_t>(n) * f.m) >> f.s);
}

// Activation codes: 0..10 are npl_activation_t. Where the reference has two
// implementations that differ (vectorised path vs scalar path of
// advanced/neural_layer/src/npl_activation_norm.cpp:186-293), codes 0..10 follow
// the vectorised path (the default, enable_vectorization = 1) and the codes
// below select the scalar formulas (neural_primitives_internal.h:229-251).
enum : int {
  kActReluScalar = 101,
  kActRelu6Scalar = 102,
  kActSoftplusScalar = 110,
};

__device__ __forceinline__ float apply_act(float x, int act, float alpha) {
  switch (act) {
    case 0:
      return x;
    case 1:  // vmath_reluf: std::max(x, 0) keeps NaN and -0 (vmath_fallback.cpp:188)
      return x < 0.0f ? 0.0f : x;
    case 2: {  // vmath_relu6f: std::min(std::max(x, 0), 6) (vmath_fused.cpp:96-113)
      const float t = x < 0.0f ? 0.0f : x;
      return 6.0f < t ? 6.0f : t;
    }
    case 3:
      return tanhf(x);
    case 4:
      return 1.0f / (1.0f + expf(-x));
    case 5: {  // tanh form of GELU (vmath_fused.cpp:220-250, internal.h ScalarGELU)
      const float x3 = x * x * x;
      return 0.5f * x * (1.0f + tanhf(0.7978845608f * (x + 0.044715f * x3)));
    }
    case 6:  // x * sigmoid(x)
      return x * (1.0f / (1.0f + expf(-x)));
    case 7:
      return x > 0.0f ? x : alpha * x;
    case 8:  // ELU with alpha 1
      return x > 0.0f ? x : 1.0f * (expf(x) - 1.0f);
    case 9:
      return 1.05070098f * (x > 0.0f ? x : 1.67326324f * (expf(x) - 1.0f));
    case 10:  // vmath_softplusf: log1p(exp(x))
      return log1pf(expf(x));
    case kActReluScalar:
      return x > 0.0f ? x : 0.0f;
    case kActRelu6Scalar: {
      const float t = 0.0f < x ? x : 0.0f;
      return 6.0f < t ? 6.0f : t;
    }
    case kActSoftplusScalar:
      return logf(1.0f + expf(x));
    default:
      return x;
  }
}

}  // namespace nplk
