/*
 * npl_kernels.h — device-level C ABI of libnpl_b200.so (prefix nplk_).
 *
 * These entry points replace the reference's microkernel / dispatch layer that
 * the NPL operators call into:
 *   mil_sgemm         composite/mkernel_interface/src/mil_gemm.cpp:210-330
 *   k_dispatch_matmul composite/dispatch_kernel/src/k_kernel_dispatch.cpp:229-255
 *   mil_reluf         composite/mkernel_interface/src/mil_vector.cpp:195-197
 * and the per-operator CPU loops in advanced/neural_layer/src/*.cpp (cited per
 * function below).
 *
 * Conventions:
 *   - All tensor pointers are DEVICE pointers (cudaMalloc'd, managed, or a
 *     torch tensor's data_ptr) of fp32 data unless stated otherwise.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *     Calls are asynchronous on that stream; nothing is synchronised.
 *   - `workspace` is caller-provided device scratch of at least the size the
 *     matching *_workspace_size() returns, 256-byte aligned.
 *   - `status` is a device int the tcgen05 kernels set non-zero if one of their
 *     bounded waits expired (the kernel then returns early instead of
 *     hanging). It may be NULL; the library then uses its own per-device word,
 *     read back with nplk_read_status().
 *   - Return value: 0 on success, or a negative NPL_ERR_* code for invalid
 *     arguments or CUDA launch errors.
 */
#ifndef NPL_B200_NPL_KERNELS_H_
#define NPL_B200_NPL_KERNELS_H_

#include <stddef.h>
#include <stdint.h>

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

/* Optional epilogue activation codes (same values as npl_activation_t). */
#define NPLK_ACT_NONE 0
#define NPLK_ACT_RELU 1
#define NPLK_ACT_LEAKY_RELU 7

/* GEMM flags. */
#define NPLK_GEMM_TF32_FAST 1u /* one TF32 pass instead of three (reported separately) */
/* Operand form of nplk_gemm. With a workspace of nplk_gemm_workspace_size()
 * bytes, A and B are first split into tf32 hi/lo copies there (the faster
 * form). Without one (NULL or too small), A and B are read in place (raw form:
 * the tensor core truncates them to tf32, the lo parts are formed in shared
 * memory), which needs A, B 16-byte aligned and lda, ldb multiples of 4.
 * These flags force one form (RAW fails with NPL_ERR_UNSUPPORTED when A or B
 * do not qualify). */
#define NPLK_GEMM_SPLIT_OPERANDS 2u
#define NPLK_GEMM_RAW_OPERANDS 4u
/* nplk_gemm_allgather: store into the destinations through the TMA unit (one
 * tensor store per 32 x 32 piece and destination) instead of with 16-byte
 * stores from the epilogue threads (the default). Taken when the destinations
 * are 16-byte aligned with ldc and col_offset multiples of 4 and the split
 * operand form runs; otherwise the thread stores run. Both give the same C;
 * measured slower on 2 and 8 B200s (8192 x 16384 x 4096 column-sharded:
 * 1.094 vs 1.031 ms at 8 GPUs). */
#define NPLK_GEMM_PEER_TMA_STORES 8u
/* nplk_gemm_allgather: dst[0] (n_dst == 1) is this rank's C as seen through
 * an NVLink multicast object that binds every rank's C (for example the
 * multicast address of a symmetric-memory buffer): the epilogue writes each
 * output element once with a 16-byte multimem store and the NVSwitch delivers
 * it to every rank's C, so a rank's NVLink egress is its own block once
 * instead of once per peer. Requires dst[0] 16-byte aligned, ldc, N_local and
 * col_offset multiples of 4, and not NPLK_GEMM_PEER_TMA_STORES; otherwise the
 * call returns NPL_ERR_INVALID_ARG. */
#define NPLK_GEMM_MULTIMEM_STORES 16u

/* ---- dense contractions (tcgen05, 3xTF32) ---------------------------------- */

/* Scratch bytes nplk_gemm needs for an M x N x K product (hi/lo operand splits;
 * the raw operand form uses none, so the workspace may then be NULL). */
NPL_API size_t nplk_gemm_workspace_size(int64_t M, int64_t N, int64_t K);

/* C[M,N] = act(alpha * A[M,K] @ B[K,N] + beta * C + bias[N]), fp32 row-major
 * with leading dimensions lda/ldb/ldc (elements). bias may be NULL. When
 * beta == 0, C is not read. Replaces mil_sgemm -> cblas_sgemm
 * (mil_gemm.cpp:290-316) on the npl_matmul path (npl_tensor_ops.cpp:217-311). */
NPL_API int nplk_gemm(void *stream, int64_t M, int64_t N, int64_t K, float alpha, const float *A,
              int64_t lda, const float *B, int64_t ldb, float beta, float *C, int64_t ldc,
              const float *bias, int act, float act_alpha, unsigned flags, void *workspace,
              size_t workspace_bytes, int *status);

/* NCHW 2-D convolution geometry. Output is [N, Cout, Ho, Wo]. */
typedef struct {
  int64_t n, c_in, h, w;      /* input */
  int64_t c_out, kh, kw;      /* weights [c_out, c_in, kh, kw] */
  int64_t stride_h, stride_w; /* >= 1 */
  int64_t pad_top, pad_left;  /* zero padding before the first row/column */
  int64_t dil_h, dil_w;       /* >= 1 */
  int64_t h_out, w_out;
} nplk_conv_geom_t;

/* Scratch bytes for nplk_conv2d_fused with this geometry: split weights,
 * per-channel epilogue constants and, when c_in is a multiple of 32 and the
 * geometry suits the TMA im2col mode, two NHWC copies of the input (tf32 hi
 * and lo parts) that the fastest kernel reads. */
NPL_API size_t nplk_conv_workspace_size(const nplk_conv_geom_t *g);

/* Conv kernels (all compute the same products in the same order, so their
 * results are identical bit for bit):
 *   DIRECT         gathers x (NCHW) per k-block into shared memory; any geometry;
 *   IM2COL         NHWC tf32 hi/lo planes of x, one im2col TMA load per k-block;
 *                  C_in % 32 == 0;
 *   WINDOW         raw NHWC plane of x, one im2col TMA window per (tile, channel
 *                  block, filter row) shared by the filter columns (stride_w 1);
 *   WINDOW_GATHER  the same windows gathered from NCHW x inside the conv kernel
 *                  (no planes, one launch). AUTO picks the fastest that applies. */
enum {
  NPLK_CONV_ALGO_AUTO = 0,
  NPLK_CONV_ALGO_DIRECT = 1,
  NPLK_CONV_ALGO_IM2COL = 2,
  NPLK_CONV_ALGO_WINDOW = 3,
  NPLK_CONV_ALGO_WINDOW_GATHER = 4,
  NPLK_CONV_ALGO_WINDOW_PAIR = 5 /* the gather windows on CTA pairs (M = 256 MMAs over two SMs) */
};

/* Workspace bytes of nplk_conv2d_run_algo with `algo`; 0 when the geometry
 * does not suit that kernel. */
NPL_API size_t nplk_conv_workspace_size_algo(const nplk_conv_geom_t *g, int algo);

/* Smallest workspace the conv entry points accept (split weights and
 * epilogue constants only). With less than nplk_conv_workspace_size bytes
 * the conv runs on the direct-gather kernel, which reads NCHW x itself; the
 * results are the same bit for bit. */
NPL_API size_t nplk_conv_workspace_min_size(const nplk_conv_geom_t *g);

/* out = act(BN(conv(x, w) + bias)) as one implicit-GEMM kernel: no im2col is
 * materialised, BN (inference form gamma*(t-mean)/sqrt(var+eps)+beta, the
 * formula of npl_activation_norm.cpp:389-398) and the activation run in the
 * epilogue before the single HBM write. bias, and each of the BN arrays, may
 * be NULL; with mean == NULL the BN step is skipped. act is an
 * npl_activation_t value; act_alpha is the LeakyReLU slope. Replaces
 * ExecuteConvDirect (npl_convolution.cpp:248-378) plus the BN / activation
 * passes the reference leaves out (npl_convolution.cpp:116-126). */
NPL_API int nplk_conv2d_fused(void *stream, const nplk_conv_geom_t *g, const float *x, const float *w,
                      const float *bias, const float *bn_mean, const float *bn_var,
                      const float *bn_gamma, const float *bn_beta, float bn_eps, int act,
                      float act_alpha, float *out, void *workspace, size_t workspace_bytes,
                      int *status);

/* The two halves of nplk_conv2d_fused, for callers that reuse one set of
 * weights across many inputs (inference): prepare writes the tap-major tf32
 * hi/lo split of w and the per-channel epilogue constants (bias, BN) into the
 * workspace; run executes the implicit-GEMM kernel against a prepared
 * workspace (and, given the full workspace size, first rewrites x into the
 * NHWC planes after the prepared part). Without BN parameters the constants
 * are the identity. */
NPL_API int nplk_conv2d_prepare(void *stream, const nplk_conv_geom_t *g, const float *w,
                                const float *bias, const float *bn_mean, const float *bn_var,
                                const float *bn_gamma, const float *bn_beta, float bn_eps,
                                void *workspace, size_t workspace_bytes);
NPL_API int nplk_conv2d_run(void *stream, const nplk_conv_geom_t *g, const float *x, int act,
                            float act_alpha, float *out, void *workspace,
                            size_t workspace_bytes, int *status);

/* nplk_conv2d_run with a given kernel (NPLK_CONV_ALGO_*), for tests and
 * tuning: NPL_ERR_UNSUPPORTED when the geometry does not suit it,
 * NPL_ERR_INVALID_ARG when the workspace is below
 * nplk_conv_workspace_size_algo. */
NPL_API int nplk_conv2d_run_algo(void *stream, const nplk_conv_geom_t *g, const float *x, int act,
                                 float act_alpha, float *out, void *workspace,
                                 size_t workspace_bytes, int *status, int algo);

/* nplk_conv2d_run in two steps, for the kernels that read NHWC planes (the
 * AUTO choice is IM2COL or WINDOW, with the full workspace): stage_input rewrites x as the NHWC tf32 hi/lo planes
 * in the workspace, run_staged runs the conv kernel on them. One staged input
 * serves any number of run_staged calls of the same geometry (for example
 * two convolutions of one input). Both return NPL_ERR_UNSUPPORTED where the
 * path does not apply. */
NPL_API int nplk_conv2d_stage_input(void *stream, const nplk_conv_geom_t *g, const float *x,
                                    void *workspace, size_t workspace_bytes);
NPL_API int nplk_conv2d_run_staged(void *stream, const nplk_conv_geom_t *g, int act,
                                   float act_alpha, float *out, void *workspace,
                                   size_t workspace_bytes, int *status);

/* nplk_conv2d_fused for callers that cannot allocate device memory (hosts
 * that reserve their whole device budget up front, code running inside an
 * allocator callback, foreign-language callers that must not trigger the
 * device-wide synchronisation cudaMalloc/cudaFree can cause). No counterpart
 * in the reference: it has no device memory at all. The weight split and
 * epilogue constants live in an 8 MiB array inside the library that every
 * GPU loading the library keeps until exit; larger geometries are rejected
 * with NPL_ERR_UNSUPPORTED. The first call on a device looks up that array's
 * address, so it should precede any stream capture. All calls on a device
 * share the array: calls that overlap on the GPU race. status may be NULL:
 * a word beside the array is then cleared by each call and receives any
 * timeout code; nplk_read_status() reads and clears it (and allocates
 * nothing), so read it after each call whose outcome matters. Allocates
 * nothing. */
NPL_API int nplk_conv2d_fused_noalloc(void *stream, const nplk_conv_geom_t *g, const float *x,
                                      const float *w, const float *bias, const float *bn_mean,
                                      const float *bn_var, const float *bn_gamma,
                                      const float *bn_beta, float bn_eps, int act,
                                      float act_alpha, float *out, int *status);

/* Fused stem block: conv (+bias) (+inference BN) (+activation) followed by a
 * 3x3 / stride 2 / pad 1 max pool (floor mode), the reference's
 * npl_conv2d_bn_activation (npl_convolution.cpp:92-137) then npl_pooling
 * max (npl_pooling.cpp:129-219). The conv epilogue writes only the
 * horizontal maxima (half the conv output's bytes) and a vertical pass
 * finishes the pool; the result is bit-identical to the two calls (same
 * scan order, NaN skipped, first of equal values kept). `out` is
 * [N][C_out][(H_out-1)/2+1][W_out/2]. Applies when the conv runs on the
 * direct kernel's row order (C_in not a multiple of 32, filter rows of 3..8
 * columns), C_out <= 64 and W_out is even and >= 32; otherwise the size query returns
 * 0 and the call NPL_ERR_UNSUPPORTED. The workspace holds the conv's
 * weights and constants plus the horizontal maxima. */
NPL_API size_t nplk_conv2d_maxpool_workspace_size(const nplk_conv_geom_t *g);
NPL_API int nplk_conv2d_maxpool_fused(void *stream, const nplk_conv_geom_t *g, const float *x,
                                      const float *w, const float *bias, const float *bn_mean,
                                      const float *bn_var, const float *bn_gamma,
                                      const float *bn_beta, float bn_eps, int act,
                                      float act_alpha, float *out, void *workspace,
                                      size_t workspace_bytes, int *status);

/* ---- bandwidth-bound primitives -------------------------------------------- */

/* Depthwise conv, weights [C,1,kh,kw]; g->c_out must equal g->c_in. Dilation
 * is ignored as in ExecuteDepthwiseConv (npl_convolution.cpp:904-991). */
NPL_API int nplk_depthwise_conv2d(void *stream, const nplk_conv_geom_t *g, const float *x,
                          const float *w, const float *bias, float *out);

/* npl_depthwise_conv2d -> npl_batch_norm (inference) -> npl_activation ->
 * npl_global_avg_pool in one pass (npl_convolution.cpp:60-90,
 * npl_activation_norm.cpp:118-153 and :51-54, npl_pooling.cpp:63-87):
 * gap[n*C + c] = mean over the output plane of
 * act(gamma*((dw(x) + bias) - mean)*rsd + beta), rsd = 1/sqrt(var+eps), with
 * the activation codes of nplk_activation (0..10). y, when not NULL, also
 * receives the activated map [N,C,Ho,Wo]; the depthwise and BN maps are never
 * written. Every value equals what nplk_depthwise_conv2d, nplk_batch_norm_infer,
 * nplk_activation and nplk_global_avg_pool give run one after another, bit for
 * bit. Weights [C,1,kh,kw], g->c_out == g->c_in; gamma, beta, bias may be
 * NULL (1, 0, none). NPL_ERR_UNSUPPORTED unless H*W <= 1024 and Ho*Wo <= 512
 * are multiples of 4 and x (and y) are 16-byte aligned: callers then run the
 * four calls. */
NPL_API int nplk_depthwise_bn_act_gap(void *stream, const nplk_conv_geom_t *g, const float *x,
                                      const float *w, const float *bias, const float *mean,
                                      const float *var, const float *gamma, const float *beta,
                                      float eps, int act, float act_alpha, float *y, float *gap);

/* Inference batch norm over NCHW planes: y = gamma*(x-mean)*rsd + beta with
 * rsd = 1/sqrt(var+eps) (npl_activation_norm.cpp:362-407). */
NPL_API int nplk_batch_norm_infer(void *stream, int64_t n, int64_t c, int64_t hw, const float *x,
                          float *y, const float *mean, const float *var, const float *gamma,
                          const float *beta, float eps);

/* Batch statistics for training-mode batch norm: per channel, the mean over
 * N*HW and the biased variance (ComputeBatchStatistics,
 * npl_activation_norm.cpp:524-552). mean/var are device arrays [c]. */
NPL_API int nplk_batch_norm_stats(void *stream, int64_t n, int64_t c, int64_t hw, const float *x,
                          float *mean, float *var);

/* run = momentum*run + (1-momentum)*batch for mean and variance
 * (npl_activation_norm.cpp:431-436). */
NPL_API int nplk_bn_update_running(void *stream, int64_t c, float *run_mean, float *run_var,
                           const float *mean, const float *var, float momentum);

/* Elementwise activation of n elements (in place allowed). `scalar_semantics`
 * selects the reference's scalar formulas (ExecuteActivationScalar,
 * npl_activation_norm.cpp:186-230) instead of its vectorised path
 * (ExecuteActivationVectorized :232-293); they differ for ReLU on NaN/-0. */
NPL_API int nplk_activation(void *stream, int64_t n, const float *x, float *y, int act, float alpha,
                    int scalar_semantics);

/* Softmax over `axis_len` elements at stride `inner` for each of outer*inner
 * lines (ExecuteSoftmaxAxis, npl_activation_norm.cpp:295-356). */
NPL_API int nplk_softmax(void *stream, int64_t outer, int64_t axis_len, int64_t inner, const float *x,
                 float *y);

/* Layer norm of `rows` rows of `cols` elements, two-moment form
 * (ExecuteLayerNormGeneric, npl_activation_norm.cpp:470-522). */
NPL_API int nplk_layer_norm(void *stream, int64_t rows, int64_t cols, const float *x, float *y,
                    const float *gamma, const float *beta, float eps);

/* Max / average 2-D pooling over NCHW (ExecuteMaxPooling / ExecuteAvgPooling,
 * npl_pooling.cpp:129-315). pool_type: 0 = max, 1 = average. */
NPL_API int nplk_pool2d(void *stream, int64_t n, int64_t c, int64_t h, int64_t w, int64_t kh,
                int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw, int64_t h_out,
                int64_t w_out, int pool_type, int count_include_pad, const float *x, float *y);

/* Mean over each of `planes` contiguous planes of `hw` elements
 * (ExecuteGlobalAvgPooling, npl_pooling.cpp:317-385). */
NPL_API int nplk_global_avg_pool(void *stream, int64_t planes, int64_t hw, const float *x, float *y);

/* Elementwise binary ops over n elements: op 0 = add, 1 = mul (npl_add /
 * npl_mul, npl_tensor_ops.cpp:440-662). b_mode: 0 = same shape, 1 = b is a
 * scalar, 2 = a is a scalar, 3 = b is per-channel [C] over NCHW planes of
 * `inner` elements. */
NPL_API int nplk_binary(void *stream, int op, int64_t n, const float *a, const float *b, float *c,
                int b_mode, int64_t channels, int64_t inner);

/* ---- multi-GPU helpers ------------------------------------------------------ */
/* The reference has no multi-device path: these serve npl_matmul's product
 * (npl_tensor_ops.cpp:115-153 -> ExecuteMatMulDirect :217-311) computed as
 * column blocks on several GPUs, one process per GPU. */

/* Column-shard relayout after an all-gather: src is [g][rows][cols_per_shard]
 * (shard-major, as an all-gather of per-rank C blocks delivers it); dst is
 * row-major [rows][g*cols_per_shard]. */
NPL_API int nplk_colshard_relayout(void *stream, int64_t g, int64_t rows, int64_t cols_per_shard,
                           const float *src, float *dst);

/* ---- multi-GPU: peer buffers and the GEMM that writes into them ------------- */

/* Bytes of an inter-process handle of device memory (CUDA IPC). The nplk_ipc_*
 * calls have no reference counterpart (the reference runs in one process). */
NPL_API size_t nplk_ipc_handle_size(void);

/* Fills `handle` (nplk_ipc_handle_size() bytes) for the allocation holding
 * dev_ptr and *offset with dev_ptr's byte offset inside it. */
NPL_API int nplk_ipc_get_handle(const void *dev_ptr, void *handle, uint64_t *offset);

/* Maps another process's allocation (a handle and offset from
 * nplk_ipc_get_handle) into this process; *dev_ptr receives the address of the
 * byte at `offset`. Peer access over NVLink is enabled as needed. */
NPL_API int nplk_ipc_open_handle(const void *handle, uint64_t offset, void **dev_ptr);

/* Unmaps a pointer returned by nplk_ipc_open_handle with the same offset. */
NPL_API int nplk_ipc_close_handle(void *dev_ptr, uint64_t offset);

/* Column-sharded GEMM fused with its all-gather (replaces nplk_gemm followed by
 * an all-gather of the column blocks and nplk_colshard_relayout). This rank
 * computes its block act(alpha * A[M,K] @ B[K,N_local] + bias[N_local]) and the
 * epilogue stores every output element into each of the n_dst (<= 8) row-major
 * [M][ldc] buffers dst[0..n_dst) -- this GPU's C and the other ranks' C mapped
 * with nplk_ipc_open_handle -- at columns col_offset .. col_offset + N_local, so
 * the exchange crosses NVLink tile by tile while the GEMM runs and every rank
 * ends with the whole row-major C once all ranks' kernels have completed. `dst`
 * is a host array of device addresses valid on the current device. With the
 * usual layout (dst[] in rank order, col_offset = rank * N_local) each rank
 * visits the destinations starting after its own index, so the ranks' stores
 * spread over all peers instead of converging on one; any order gives the
 * same C. The epilogue stages each warp's 32 x 32 piece in shared memory and
 * stores it to every destination with 16-byte stores that cover whole
 * 128-byte row segments (NPLK_GEMM_PEER_TMA_STORES: one TMA tensor store per
 * piece and destination instead; NPLK_GEMM_MULTIMEM_STORES: one multicast
 * store per element into the single destination). beta is 0 (C is not read);
 * other arguments as nplk_gemm. */
NPL_API int nplk_gemm_allgather(void *stream, int64_t M, int64_t N_local, int64_t K,
                                float alpha, const float *A, int64_t lda, const float *B,
                                int64_t ldb, const float *bias, int act, float act_alpha,
                                float *const *dst, int n_dst, int64_t col_offset, int64_t ldc,
                                unsigned flags, void *workspace, size_t workspace_bytes,
                                int *status);

/* ---- status ----------------------------------------------------------------- */

/* Reads (and clears) the library's per-device kernel status word and the
 * status word of nplk_conv2d_fused_noalloc; returns the first non-zero code,
 * 0 = ok. Synchronises `stream`. Allocates nothing: a word that no kernel
 * can have written yet is not created. No reference counterpart: the reference's kernels
 * cannot time out, its errors are the return codes (neural_primitives.h:52-59). */
NPL_API int nplk_read_status(void *stream);

/* Number of library kernels launched on this thread since the last call
 * (resets the counter). */
NPL_API uint64_t nplk_take_launch_count(void);

/* ---- tile-configuration cache ---------------------------------------------- */
/* Replaces the reference's tuning result cache (composite/tuning_rCache/src/
 * tuning_cache.cpp:186-506; cat_* API in include/cached_autotuner.h): the
 * kernel choice measured fastest per (operation, shape, SM count), consulted
 * by the AUTO paths of nplk_conv2d_run / nplk_conv2d_fused (the conv kernel,
 * NPLK_CONV_ALGO_*) and nplk_gemm (the output-tile width BN, 64 or 128), and
 * persisted as a text file with a format version and a hardware signature
 * (device name, compute capability, SM count, L2 size) checked on load.
 * npl_init loads the file named by NPL_TUNING_CACHE (if set and present) and
 * npl_shutdown writes it back; NPL_AUTOTUNE=1 makes npl_conv2d_bn_activation,
 * npl_conv2d and npl_matmul tune a shape on its first call. Thread safe. */
typedef struct {
  uint64_t entries;   /* entries held */
  uint64_t hits;      /* AUTO lookups that found an entry */
  uint64_t misses;    /* AUTO lookups that did not */
  uint64_t tunes;     /* entries written by nplk_*_tune */
  uint64_t evictions; /* entries dropped by the entry limit */
} nplk_tuning_stats_t;

/* Merges a cache file into the cache; returns the entries read, or
 * NPL_ERR_INVALID_ARG (unreadable or malformed file) or NPL_ERR_UNSUPPORTED
 * (another format version or another device: nothing is loaded). */
NPL_API int nplk_tuning_cache_load(const char *path);
/* Writes the cache (atomically, through a temporary file); returns the
 * entries written or NPL_ERR_INTERNAL on an I/O error. */
NPL_API int nplk_tuning_cache_save(const char *path);
/* Drops every entry and zeroes the statistics. */
NPL_API void nplk_tuning_cache_clear(void);
NPL_API int nplk_tuning_cache_stats(nplk_tuning_stats_t *out);
/* Keeps at most n entries, evicting the oldest inserted (0 = unlimited). */
NPL_API int nplk_tuning_cache_set_max_entries(size_t n);
/* The cache key of a conv geometry or a GEMM shape on the current device,
 * written NUL-terminated into buf (truncated to len); returns its length. */
NPL_API size_t nplk_tuning_key_conv(const nplk_conv_geom_t *g, char *buf, size_t len);
NPL_API size_t nplk_tuning_key_gemm(int64_t M, int64_t N, int64_t K, char *buf, size_t len);
/* Direct access to entries (import / export tooling, tests): put inserts or
 * replaces; get returns 1 and fills choice / us when present, else 0. */
NPL_API int nplk_tuning_cache_put(const char *key, int choice, float us);
NPL_API int nplk_tuning_cache_get(const char *key, int *choice, float *us);

/* Measures every conv kernel the geometry and the workspace allow (size the
 * workspace with the largest nplk_conv_workspace_size_algo to try them all)
 * on the caller's tensors: `reps` timed runs each after one warm-up, median
 * device time. Caches the fastest, returns it in *best_algo (and its median
 * time in *best_us when non-NULL) and leaves the conv's output in `out` (all
 * kernels give the same bits). Synchronises `stream`. Arguments as
 * nplk_conv2d_fused. */
NPL_API int nplk_conv2d_tune(void *stream, const nplk_conv_geom_t *g, const float *x,
                             const float *w, const float *bias, const float *bn_mean,
                             const float *bn_var, const float *bn_gamma, const float *bn_beta,
                             float bn_eps, int act, float act_alpha, float *out,
                             void *workspace, size_t workspace_bytes, int reps, int *best_algo,
                             float *best_us);
/* The same for the GEMM's tile configuration: C = A @ B (alpha 1, beta 0)
 * with 64-wide tiles, 128-wide tiles, and (K >= 512) 128-wide tiles with K
 * cut in two slices added into a zeroed C; `reps` timed runs each; caches and
 * returns the fastest as 64, 128 or 1128. nplk_gemm uses two K slices only
 * for a plain product (beta 0, no bias, no activation) in the split operand
 * form; otherwise a cached 1128 means 128-wide tiles. The workspace is the
 * split form's (nplk_gemm_workspace_size). */
NPL_API int nplk_gemm_tune(void *stream, int64_t M, int64_t N, int64_t K, const float *A,
                           int64_t lda, const float *B, int64_t ldb, float *C, int64_t ldc,
                           void *workspace, size_t workspace_bytes, int reps, int *best_bn,
                           float *best_us);

/* ---- fault injection (tests of the failure paths) --------------------------- */
/* No reference counterpart: the reference's CPU loops cannot time out or run
 * out of device memory. Both hooks are off unless armed. */

#define NPLK_DEBUG_GEMM 1        /* the tcgen05 GEMM kernels (split and raw forms) */
#define NPLK_DEBUG_CONV_WINDOW 2 /* the window conv kernels (gather and plane forms) */

/* Arms the next launch of one kernel family, from any thread, to exercise its
 * bounded-wait timeout: that launch's MMA issuer waits on a barrier nothing
 * arrives on, with a limit of stall_us microseconds (<= 60 s) instead of the
 * kernels' 4 s. On expiry the kernel records 102 (MMA wait expired) in its
 * status word, every role leaves on the CTA's abort flag, copies in flight
 * land, TMEM is freed and the kernel returns; its outputs are undefined.
 * stall_us = 0 disarms. Returns 0 or NPL_ERR_INVALID_ARG. */
NPL_API int nplk_debug_arm_wait_timeout(int which, uint32_t stall_us);

/* The next `count` device allocations made by npl_* calls (staging of host
 * tensors and per-call scratch) fail as if the device were out of memory;
 * count = 0 disarms. Returns the number still armed before this call. */
NPL_API int nplk_debug_fail_next_allocations(int count);

#ifdef __cplusplus
}
#endif

#endif /* NPL_B200_NPL_KERNELS_H_ */
