/*
 * neural_primitives.h — public C ABI of the B200 NPL backend (libnpl_b200.so).
 *
 * This is a drop-in replacement for JCore's Neural Primitives Layer API
 * (reference: advanced/neural_layer/include/neural_primitives.h:44-579).
 * Every symbol, enum value and struct layout below matches the reference so
 * that existing C callers and the Java FFM bindings
 * (ffm_api/jcorex/src/main/java/net/api/kernel/Tensors.java:24-45,
 *  Config.java:19-31) link and run unchanged. The struct offsets are pinned by
 * static_asserts in the library sources and by the ABI tests.
 *
 * Semantics on the B200 backend:
 *   - All compute runs on the current CUDA device (one process per GPU).
 *   - npl_allocate_tensor returns CUDA managed memory, so callers may keep
 *     writing tensor->data from the host as they did with the CPU library.
 *     Device pointers (cudaMalloc, torch) are used in place. Plain host
 *     pointers are staged through device memory for the duration of a call.
 *   - Every call is synchronous: results are visible to the host on return.
 *   - Only NPL_DTYPE_FP32 tensors are computed (as in the reference).
 */
#ifndef NPL_B200_NEURAL_PRIMITIVES_H_
#define NPL_B200_NEURAL_PRIMITIVES_H_

#include <stddef.h>

/* Exported-symbol marker (the library is built with hidden default visibility). */
#ifndef NPL_API
#if defined(__GNUC__)
#define NPL_API __attribute__((visibility("default")))
#else
#define NPL_API
#endif
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes (reference neural_primitives.h:52-59). */
#define NPL_OK 0
#define NPL_ERR_NOT_INITIALIZED -1
#define NPL_ERR_INVALID_ARG -2
#define NPL_ERR_NO_MEMORY -3
#define NPL_ERR_INTERNAL -4
#define NPL_ERR_UNSUPPORTED -5
#define NPL_ERR_SHAPE_MISMATCH -6
#define NPL_ERR_OOM -7

/* Tensor memory layout tag (reference :65-69). */
typedef enum {
  NPL_LAYOUT_NCHW = 0,
  NPL_LAYOUT_NHWC = 1,
  NPL_LAYOUT_NCHW_VECT_C = 2
} npl_data_layout_t;

/* Element type (reference :75-81). */
typedef enum {
  NPL_DTYPE_FP32 = 0,
  NPL_DTYPE_FP16 = 1,
  NPL_DTYPE_BF16 = 2,
  NPL_DTYPE_INT8 = 3,
  NPL_DTYPE_INT32 = 4
} npl_dtype_t;

/* Activation selector (reference :87-99). */
typedef enum {
  NPL_ACT_NONE = 0,
  NPL_ACT_RELU = 1,
  NPL_ACT_RELU6 = 2,
  NPL_ACT_TANH = 3,
  NPL_ACT_SIGMOID = 4,
  NPL_ACT_GELU = 5,
  NPL_ACT_SWISH = 6,
  NPL_ACT_LEAKY_RELU = 7,
  NPL_ACT_ELU = 8,
  NPL_ACT_SELU = 9,
  NPL_ACT_SOFTPLUS = 10
} npl_activation_t;

/* Convolution padding policy (reference :105-109). */
typedef enum {
  NPL_PAD_VALID = 0,
  NPL_PAD_SAME = 1,
  NPL_PAD_EXPLICIT = 2
} npl_padding_t;

/* Pooling kind (reference :115-120). */
typedef enum {
  NPL_POOL_MAX = 0,
  NPL_POOL_AVG = 1,
  NPL_POOL_GLOBAL_AVG = 2,
  NPL_POOL_GLOBAL_MAX = 3
} npl_pooling_t;

/* Library configuration; 56 bytes (reference :126-137). On the B200 backend
 * only num_threads (host-side helper threads), enable_vectorization (selects
 * the reference's vectorised vs scalar activation semantics), workspace_size_mb
 * and verbose are read; the JIT/graph/polyhedral/NUMA switches are accepted
 * and ignored because those tiers do not exist here. */
typedef struct {
  size_t num_threads;
  int enable_fusion;
  int enable_graph_optimization;
  int enable_jit;
  int enable_poly;
  int enable_vectorization;
  int enable_numa;
  int enable_memory_pooling;
  size_t workspace_size_mb;
  int verbose;
} npl_config_t;

#define NPL_MAX_DIMS 8

/* Tensor descriptor; 168 bytes: data@0 ndim@8 shape@16 strides@80 dtype@144
 * layout@148 size_bytes@152 is_contiguous@160 (reference :145-154). Strides
 * are in elements, row-major. */
typedef struct {
  void *data;
  size_t ndim;
  size_t shape[NPL_MAX_DIMS];
  size_t strides[NPL_MAX_DIMS];
  npl_dtype_t dtype;
  npl_data_layout_t layout;
  size_t size_bytes;
  int is_contiguous;
} npl_tensor_t;

/* Per-call statistics; 56 bytes (reference :160-168). elapsed_ms is the
 * device time of the call's kernels measured with CUDA events. */
typedef struct {
  double elapsed_ms;
  double gflops;
  double bandwidth_gbps;
  size_t operations_fused;
  size_t memory_saved_bytes;
  const char *backend_used;
  int was_fused;
} npl_perf_stats_t;

/* Convolution parameters (reference :174-187). */
typedef struct {
  size_t kernel_h;
  size_t kernel_w;
  size_t stride_h;
  size_t stride_w;
  size_t pad_h;
  size_t pad_w;
  size_t dilation_h;
  size_t dilation_w;
  size_t groups;
  npl_padding_t padding;
  npl_activation_t activation;
  int use_bias;
} npl_conv_params_t;

/* Batch-norm parameters (reference :193-201). The pointers are host or
 * device arrays of length C; gamma/beta may be NULL (1 and 0). */
typedef struct {
  const float *mean;
  const float *variance;
  const float *gamma;
  const float *beta;
  float epsilon;
  int training;
  float momentum;
} npl_batchnorm_params_t;

/* Layer-norm parameters (reference :207-212). */
typedef struct {
  const float *gamma;
  const float *beta;
  float epsilon;
  size_t normalized_shape;
} npl_layernorm_params_t;

/* Pooling parameters (reference :218-227). */
typedef struct {
  size_t kernel_h;
  size_t kernel_w;
  size_t stride_h;
  size_t stride_w;
  size_t pad_h;
  size_t pad_w;
  npl_pooling_t type;
  int count_include_pad;
} npl_pooling_params_t;

/* ---- initialisation (reference npl_core.cpp:23-189) ---------------------- */
/* Binds the library to the current CUDA device, creates its stream and
 * device memory pool. NULL config = defaults. Returns NPL_ERR_INTERNAL when no
 * CUDA device is usable. */
NPL_API int npl_init(const npl_config_t *config);
NPL_API void npl_shutdown(void);
NPL_API int npl_is_initialized(void);
NPL_API int npl_get_default_config(npl_config_t *out_config);

/* ---- tensor management (reference npl_tensor_ops.cpp:16-109) -------------- */
NPL_API int npl_create_tensor(void *data, size_t ndim, const size_t *shape,
                      npl_dtype_t dtype, npl_data_layout_t layout,
                      npl_tensor_t *out_tensor);
/* Allocates CUDA managed memory (256-byte aligned) when data is NULL. */
NPL_API int npl_allocate_tensor(npl_tensor_t *tensor);
NPL_API void npl_free_tensor(npl_tensor_t *tensor);
NPL_API int npl_reshape_tensor(const npl_tensor_t *tensor, size_t new_ndim,
                       const size_t *new_shape, npl_tensor_t *out_tensor);

/* ---- convolution (reference npl_convolution.cpp:13-172) ------------------- */
/* Implicit-GEMM convolution on the tcgen05 tensor cores (3xTF32), plus bias. */
NPL_API int npl_conv2d(const npl_tensor_t *input, const npl_tensor_t *weights,
               const npl_tensor_t *bias, const npl_conv_params_t *params,
               npl_tensor_t *output, npl_perf_stats_t *stats);
NPL_API int npl_depthwise_conv2d(const npl_tensor_t *input, const npl_tensor_t *weights,
                         const npl_tensor_t *bias, const npl_conv_params_t *params,
                         npl_tensor_t *output, npl_perf_stats_t *stats);
/* conv + bias -> inference batch norm -> activation, fused in one kernel
 * epilogue (the reference runs the conv only, npl_convolution.cpp:116-126). */
NPL_API int npl_conv2d_bn_activation(const npl_tensor_t *input, const npl_tensor_t *weights,
                             const npl_tensor_t *bias,
                             const npl_conv_params_t *conv_params,
                             const npl_batchnorm_params_t *bn_params,
                             npl_activation_t activation, npl_tensor_t *output,
                             npl_perf_stats_t *stats);

/* ---- activations (reference npl_activation_norm.cpp:13-112) ---------------- */
NPL_API int npl_activation(const npl_tensor_t *input, npl_activation_t activation,
                   npl_tensor_t *output, npl_perf_stats_t *stats);
NPL_API int npl_relu(const npl_tensor_t *input, npl_tensor_t *output, npl_perf_stats_t *stats);
NPL_API int npl_leaky_relu(const npl_tensor_t *input, float alpha, npl_tensor_t *output,
                   npl_perf_stats_t *stats);
NPL_API int npl_softmax(const npl_tensor_t *input, int axis, npl_tensor_t *output,
                npl_perf_stats_t *stats);

/* ---- normalisation (reference npl_activation_norm.cpp:118-182) -------------- */
NPL_API int npl_batch_norm(const npl_tensor_t *input, const npl_batchnorm_params_t *params,
                   npl_tensor_t *output, npl_perf_stats_t *stats);
NPL_API int npl_layer_norm(const npl_tensor_t *input, const npl_layernorm_params_t *params,
                   npl_tensor_t *output, npl_perf_stats_t *stats);

/* ---- pooling (reference npl_pooling.cpp:12-87) ------------------------------ */
NPL_API int npl_pooling(const npl_tensor_t *input, const npl_pooling_params_t *params,
                npl_tensor_t *output, npl_perf_stats_t *stats);
NPL_API int npl_global_avg_pool(const npl_tensor_t *input, npl_tensor_t *output,
                        npl_perf_stats_t *stats);

/* ---- tensor ops (reference npl_tensor_ops.cpp:115-219) ----------------------- */
/* C = alpha*A@B + beta*C, fp32 row-major, on the tcgen05 tensor cores with
 * 3xTF32 split precision (max normwise relative error <= 1e-4 vs fp32). */
NPL_API int npl_matmul(const npl_tensor_t *A, const npl_tensor_t *B, npl_tensor_t *C,
               float alpha, float beta, npl_perf_stats_t *stats);
NPL_API int npl_add(const npl_tensor_t *A, const npl_tensor_t *B, npl_tensor_t *C,
            npl_perf_stats_t *stats);
NPL_API int npl_mul(const npl_tensor_t *A, const npl_tensor_t *B, npl_tensor_t *C,
            npl_perf_stats_t *stats);

/* ---- utilities (reference npl_convolution.cpp:139-172, npl_core.cpp:402-468) - */
NPL_API int npl_conv2d_output_shape(const size_t *input_shape, const npl_conv_params_t *params,
                            size_t *output_shape);
/* The reference declares npl_strerror but defines NPL_strerror
 * (npl_core.cpp:402); this library exports the declared name. */
NPL_API const char *npl_strerror(int error);
NPL_API const char *npl_get_system_info(void);
/* Runs the known-answer checks of the reference self test
 * (advanced/neural_layer/src/npl_test.cpp:56-555) on the device. */
NPL_API int npl_self_test(int verbose);

#ifdef __cplusplus
}
#endif

#endif /* NPL_B200_NEURAL_PRIMITIVES_H_ */
