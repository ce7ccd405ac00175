/* CPU restatement of the reference NPL hot path. TEST INFRASTRUCTURE ONLY:
 * used by tests/, __graft_entry__.smoke() and the CPU-baseline leg of bench.py
 * as the checker; never linked into or called by the product library.
 *
 * Each function restates one loop nest of the reference
 * (advanced/neural_layer/src/*.cpp, cited per function) with the same fp32
 * arithmetic and summation order, except oracle_sgemm, which accumulates in
 * fp64 because the reference's GEMM order belongs to the BLAS it links. */
#ifndef NPL_ORACLE_H_
#define NPL_ORACLE_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

void oracle_set_threads(int n);

/* C = alpha*A@B + beta*C, row-major, fp64 accumulation; C not read if beta==0. */
void oracle_sgemm(int64_t M, int64_t N, int64_t K, float alpha, const float *A, int64_t lda,
                  const float *B, int64_t ldb, float beta, float *C, int64_t ldc);

/* ExecuteConvDirect (npl_convolution.cpp:248-378): NCHW, sum over (ic,kh,kw)
 * in that order, then + bias[oc] if bias != NULL. */
void oracle_conv2d(const float *x, int64_t N, int64_t C, int64_t H, int64_t W, const float *w,
                   int64_t Cout, int64_t KH, int64_t KW, int64_t sh, int64_t sw, int64_t pt,
                   int64_t pl, int64_t dh, int64_t dw, int64_t Ho, int64_t Wo,
                   const float *bias, float *out);

/* ExecuteDepthwiseConv (npl_convolution.cpp:904-991). */
void oracle_depthwise_conv2d(const float *x, int64_t N, int64_t C, int64_t H, int64_t W,
                             const float *w, int64_t KH, int64_t KW, int64_t sh, int64_t sw,
                             int64_t pt, int64_t pl, int64_t Ho, int64_t Wo, const float *bias,
                             float *out);

/* ExecuteBatchNormInference (npl_activation_norm.cpp:362-407). */
void oracle_batch_norm(const float *x, int64_t N, int64_t C, int64_t HW, const float *mean,
                       const float *var, const float *gamma, const float *beta, float eps,
                       float *out);

/* ExecuteBatchNormTraining (npl_activation_norm.cpp:409-468); updates
 * run_mean/run_var in place. */
void oracle_batch_norm_train(const float *x, int64_t N, int64_t C, int64_t HW, float *run_mean,
                             float *run_var, const float *gamma, const float *beta, float eps,
                             float momentum, float *out);

/* Activations: act is an npl_activation_t value; scalar != 0 selects the
 * reference's scalar formulas (ExecuteActivationScalar, :186-230) instead of
 * the vectorised path (ExecuteActivationVectorized, :232-293). */
void oracle_activation(const float *x, int64_t n, int act, float alpha, int scalar, float *out);

/* ExecuteSoftmaxAxis (npl_activation_norm.cpp:295-356). */
void oracle_softmax(const float *x, int64_t outer, int64_t axis_len, int64_t inner, float *out);

/* ExecuteLayerNormGeneric (npl_activation_norm.cpp:470-522). */
void oracle_layer_norm(const float *x, int64_t rows, int64_t cols, const float *gamma,
                       const float *beta, float eps, float *out);

/* ExecuteMaxPooling / ExecuteAvgPooling (npl_pooling.cpp:129-315);
 * type 0 = max, 1 = average. */
void oracle_pool2d(const float *x, int64_t N, int64_t C, int64_t H, int64_t W, int64_t KH,
                   int64_t KW, int64_t sh, int64_t sw, int64_t ph, int64_t pw, int64_t Ho,
                   int64_t Wo, int type, int count_include_pad, float *out);

/* ExecuteGlobalAvgPooling (npl_pooling.cpp:317-385) with 8-wide partial sums. */
void oracle_global_avg_pool(const float *x, int64_t planes, int64_t hw, float *out);

#ifdef __cplusplus
}
#endif

#endif /* NPL_ORACLE_H_ */
