/* cblas_sgemm / cblas_dgemm for the reference oracle build. TEST INFRASTRUCTURE ONLY.
 *
 * The reference reaches its GEMM arithmetic through a weak cblas_sgemm
 * (composite/mkernel_interface/src/mil_gemm.cpp:19-27, called at :298-307;
 * also composite/kernel_autoTuner/src/kernels_openblas.cpp:28). OpenBLAS is
 * not vendored by the reference and no version is pinned. Here the call is
 * forwarded to the OpenBLAS 0.3.30 that numpy ships
 * (libscipy_openblas64_*.so). That build uses a 64-bit integer interface
 * with symbol suffix "64_". CBLAS enum values are those of cblas.h:
 * RowMajor = 101, NoTrans = 111. */
#include <stdint.h>

void scipy_cblas_sgemm64_(int order, int transa, int transb, int64_t m, int64_t n,
                          int64_t k, float alpha, const float *a, int64_t lda,
                          const float *b, int64_t ldb, float beta, float *c, int64_t ldc);
void scipy_cblas_dgemm64_(int order, int transa, int transb, int64_t m, int64_t n,
                          int64_t k, double alpha, const double *a, int64_t lda,
                          const double *b, int64_t ldb, double beta, double *c,
                          int64_t ldc);
void scipy_openblas_set_num_threads64_(int n);

void cblas_sgemm(int order, int transa, int transb, int m, int n, int k, float alpha,
                 const float *a, int lda, const float *b, int ldb, float beta, float *c,
                 int ldc) {
  scipy_cblas_sgemm64_(order, transa, transb, m, n, k, alpha, a, lda, b, ldb, beta, c,
                       ldc);
}

void cblas_dgemm(int order, int transa, int transb, int m, int n, int k, double alpha,
                 const double *a, int lda, const double *b, int ldb, double beta,
                 double *c, int ldc) {
  scipy_cblas_dgemm64_(order, transa, transb, m, n, k, alpha, a, lda, b, ldb, beta, c,
                       ldc);
}

void npl_ref_blas_set_threads(int n) { scipy_openblas_set_num_threads64_(n > 0 ? n : 1); }
