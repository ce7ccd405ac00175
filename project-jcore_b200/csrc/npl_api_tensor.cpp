// Tensor management and tensor ops of the npl_* API
// (reference: advanced/neural_layer/src/npl_tensor_ops.cpp:16-662).
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>
#include <unordered_set>

#include "npl_runtime.h"

using npl::element_count;
using npl::state;
using npl::validate_tensor;

namespace {

std::mutex g_alloc_mu;
std::unordered_set<void *> g_allocations;

size_t element_size(npl_dtype_t dt) {
  switch (dt) {
    case NPL_DTYPE_FP32:
    case NPL_DTYPE_INT32:
      return 4;
    case NPL_DTYPE_FP16:
    case NPL_DTYPE_BF16:
      return 2;
    case NPL_DTYPE_INT8:
      return 1;
    default:
      return 0;
  }
}

void row_major_strides(npl_tensor_t *t) {
  t->strides[t->ndim - 1] = 1;
  for (int i = static_cast<int>(t->ndim) - 2; i >= 0; --i)
    t->strides[i] = t->strides[i + 1] * t->shape[i + 1];
}

}  // namespace

extern "C" int npl_create_tensor(void *data, size_t ndim, const size_t *shape,
                                 npl_dtype_t dtype, npl_data_layout_t layout,
                                 npl_tensor_t *out) {
  if (!out || !shape || ndim == 0 || ndim > NPL_MAX_DIMS) return NPL_ERR_INVALID_ARG;
  out->data = data;
  out->ndim = ndim;
  out->dtype = dtype;
  out->layout = layout;
  size_t total = 1;
  for (size_t i = 0; i < ndim; ++i) {
    out->shape[i] = shape[i];
    total *= shape[i];
  }
  row_major_strides(out);
  out->size_bytes = total * element_size(dtype);
  out->is_contiguous = 1;
  return NPL_OK;
}

// Allocates CUDA managed memory, so host code may fill tensor->data directly
// as with the CPU library (npl_tensor_ops.cpp:49-69 used 64-byte aligned host
// memory; managed allocations are at least 256-byte aligned).
extern "C" int npl_allocate_tensor(npl_tensor_t *t) {
  if (!t) return NPL_ERR_INVALID_ARG;
  if (t->data) return NPL_OK;
  if (t->size_bytes == 0) return NPL_ERR_INVALID_ARG;
  if (state().initialized) cudaSetDevice(state().device);
  void *p = nullptr;
  if (cudaMallocManaged(&p, t->size_bytes, cudaMemAttachGlobal) != cudaSuccess) {
    cudaGetLastError();
    return NPL_ERR_NO_MEMORY;
  }
  {
    std::lock_guard<std::mutex> lock(g_alloc_mu);
    g_allocations.insert(p);
  }
  t->data = p;
  return NPL_OK;
}

// Frees memory this library allocated and clears the pointer. Memory the
// caller attached with npl_create_tensor is not owned by the library and is
// left alone.
extern "C" void npl_free_tensor(npl_tensor_t *t) {
  if (!t || !t->data) return;
  bool ours = false;
  {
    std::lock_guard<std::mutex> lock(g_alloc_mu);
    ours = g_allocations.erase(t->data) > 0;
  }
  if (ours) cudaFree(t->data);
  t->data = nullptr;
}

extern "C" int npl_reshape_tensor(const npl_tensor_t *t, size_t new_ndim,
                                  const size_t *new_shape, npl_tensor_t *out) {
  if (!t || !new_shape || !out || new_ndim > NPL_MAX_DIMS) return NPL_ERR_INVALID_ARG;
  if (new_ndim == 0) return NPL_ERR_INVALID_ARG;
  size_t n = 1;
  for (size_t i = 0; i < new_ndim; ++i) n *= new_shape[i];
  if (n != element_count(t)) return NPL_ERR_SHAPE_MISMATCH;
  *out = *t;
  out->ndim = new_ndim;
  for (size_t i = 0; i < new_ndim; ++i) out->shape[i] = new_shape[i];
  row_major_strides(out);
  return NPL_OK;
}

// ---------------------------------------------------------------------------
// matmul
// ---------------------------------------------------------------------------
extern "C" int npl_matmul(const npl_tensor_t *A, const npl_tensor_t *B, npl_tensor_t *C,
                          float alpha, float beta, npl_perf_stats_t *stats) {
  if (!state().initialized) return NPL_ERR_NOT_INITIALIZED;
  int rc = validate_tensor(A, "A");
  if (rc) return rc;
  rc = validate_tensor(B, "B");
  if (rc) return rc;
  rc = validate_tensor(C, "C");
  if (rc) return rc;
  if (A->dtype != NPL_DTYPE_FP32 || B->dtype != NPL_DTYPE_FP32 || C->dtype != NPL_DTYPE_FP32)
    return NPL_ERR_UNSUPPORTED;
  if (A->ndim < 2 || B->ndim < 2 || C->ndim < 2) return NPL_ERR_SHAPE_MISMATCH;
  const size_t M = A->shape[A->ndim - 2], K = A->shape[A->ndim - 1];
  const size_t N = B->shape[B->ndim - 1];
  if (B->shape[B->ndim - 2] != K || C->shape[C->ndim - 2] != M || C->shape[C->ndim - 1] != N)
    return NPL_ERR_SHAPE_MISMATCH;
  // Batched form (A or B with >= 3 dims): batch = product of A's leading dims
  // (npl_tensor_ops.cpp:313-330); B is shared when it is 2-D.
  size_t batch = 1;
  for (size_t i = 0; i + 2 < A->ndim; ++i) batch *= A->shape[i];
  const bool b_batched = B->ndim >= 3;
  if (element_count(C) < batch * M * N || (b_batched && element_count(B) < batch * K * N))
    return NPL_ERR_SHAPE_MISMATCH;

  npl::Call call;
  const size_t b_elems = (b_batched ? batch : 1) * K * N;
  const float *a = call.input(A->data, batch * M * K * 4);
  const float *b = call.input(B->data, b_elems * 4);
  float *c = call.output(C->data, batch * M * N * 4, beta != 0.0f);
  // The hi/lo operand workspace (805 MB for 8192x4096x16384); when the device
  // cannot spare it, nplk_gemm reads A and B in place (raw operand form).
  size_t ws = nplk_gemm_workspace_size(M, N, K);
  void *w = call.try_scratch(ws);
  if (!w) ws = 0;
  if (call.status()) return call.finish(nullptr, 0, 0, nullptr);
  const unsigned flags = npl::tf32_fast_mode() ? NPLK_GEMM_TF32_FAST : 0u;
  call.start_timer();
  // NPL_AUTOTUNE=1: an untuned shape has its tile width measured once (into
  // C, which the call then overwrites) and cached; beta == 0 only, since the
  // measurement does not keep C.
  if (w && batch == 1 && beta == 0.0f && flags == 0u && npl::autotune_mode() &&
      !npl::gemm_tuned(M, N, K)) {
    int bn = 0;
    call.fail(nplk_gemm_tune(call.stream(), M, N, K, a, K, b, N, c, N, w, ws, 3, &bn, nullptr));
  }
  for (size_t i = 0; i < batch && !call.status(); ++i) {
    const int rc = nplk_gemm(call.stream(), M, N, K, alpha, a + i * M * K, K,
                             b + (b_batched ? i * K * N : 0), N, beta, c + i * M * N, N,
                             nullptr, NPLK_ACT_NONE, 0.0f, flags, w, ws, nullptr);
    // No workspace and operands the raw form cannot read in place: out of memory.
    call.fail(!w && rc == NPL_ERR_INVALID_ARG ? NPL_ERR_OOM : rc);
  }
  call.stop_timer();
  return call.finish(stats, 2.0 * batch * M * N * K,
                     4.0 * batch * (M * K + K * N + (beta != 0.0f ? 2 : 1) * M * N),
                     flags ? "B200-tcgen05-TF32" : "B200-tcgen05-3xTF32");
}

// ---------------------------------------------------------------------------
// add / mul (npl_tensor_ops.cpp:440-662)
// ---------------------------------------------------------------------------
extern "C" int npl_add(const npl_tensor_t *A, const npl_tensor_t *B, npl_tensor_t *C,
                       npl_perf_stats_t *stats) {
  if (!state().initialized) return NPL_ERR_NOT_INITIALIZED;
  int rc = validate_tensor(A, "A");
  if (rc) return rc;
  rc = validate_tensor(B, "B");
  if (rc) return rc;
  rc = validate_tensor(C, "C");
  if (rc) return rc;
  const size_t n = element_count(C);
  // Same-shape contiguous tensors only; broadcasting is unsupported
  // (npl_tensor_ops.cpp:453-467).
  if (!(A->is_contiguous && B->is_contiguous && C->is_contiguous && element_count(A) == n &&
        element_count(B) == n))
    return NPL_ERR_UNSUPPORTED;
  npl::Call call;
  const float *a = call.input(A->data, n * 4);
  const float *b = call.input(B->data, n * 4);
  float *c = call.output(C->data, n * 4);
  if (call.status()) return call.finish(nullptr, 0, 0, nullptr);
  call.start_timer();
  call.fail(nplk_binary(call.stream(), 0, n, a, b, c, 0, 0, 0));
  call.stop_timer();
  return call.finish(stats, 0.0, 12.0 * n, "B200-elementwise");
}

extern "C" int npl_mul(const npl_tensor_t *A, const npl_tensor_t *B, npl_tensor_t *C,
                       npl_perf_stats_t *stats) {
  if (!state().initialized) return NPL_ERR_NOT_INITIALIZED;
  int rc = validate_tensor(A, "A");
  if (rc) return rc;
  rc = validate_tensor(B, "B");
  if (rc) return rc;
  rc = validate_tensor(C, "C");
  if (rc) return rc;
  const size_t n = element_count(C), na = element_count(A), nb = element_count(B);
  int mode = -1;
  int64_t channels = 0, inner = 0;
  size_t work = n;
  bool same_shape = A->is_contiguous && B->is_contiguous && C->is_contiguous && na == n &&
                    nb == n && A->ndim == B->ndim && A->ndim == C->ndim;
  for (size_t i = 0; same_shape && i < A->ndim; ++i)
    same_shape = A->shape[i] == B->shape[i] && A->shape[i] == C->shape[i];
  if (same_shape) {
    mode = 0;  // case 1 (npl_tensor_ops.cpp:546-581)
  } else if (nb == 1) {
    mode = 1;  // B scalar (:583-608)
  } else if (na == 1) {
    mode = 2;  // A scalar (:610-632)
  } else if (A->ndim == 4 && B->ndim == 4 && C->ndim == 4 && A->shape[0] == C->shape[0] &&
             A->shape[1] == B->shape[1] && B->shape[0] == 1 && B->shape[2] == 1 &&
             B->shape[3] == 1) {
    mode = 3;  // per-channel broadcast (:634-666)
    channels = static_cast<int64_t>(A->shape[1]);
    inner = static_cast<int64_t>(A->shape[2] * A->shape[3]);
    work = A->shape[0] * A->shape[1] * A->shape[2] * A->shape[3];
  } else {
    // Strided generic (:668-700) and other broadcasts are not implemented.
    return NPL_ERR_UNSUPPORTED;
  }
  const size_t a_need = mode == 2 ? 1 : work;
  const size_t b_need = mode == 1 ? 1 : (mode == 3 ? static_cast<size_t>(channels) : work);
  if (na < a_need || nb < b_need || n < work) return NPL_ERR_SHAPE_MISMATCH;
  npl::Call call;
  const float *a = call.input(A->data, a_need * 4);
  const float *b = call.input(B->data, b_need * 4);
  float *c = call.output(C->data, work * 4);
  if (call.status()) return call.finish(nullptr, 0, 0, nullptr);
  call.start_timer();
  call.fail(nplk_binary(call.stream(), 1, work, a, b, c, mode, channels, inner));
  call.stop_timer();
  return call.finish(stats, 0.0, 4.0 * (a_need + b_need + work), "B200-elementwise");
}
