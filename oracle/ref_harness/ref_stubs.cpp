// Harness-owned link stubs for building the reference NPL sources as a CPU
// oracle. TEST INFRASTRUCTURE ONLY: nothing in the product links this file.
//
// The reference's NPL sources (advanced/neural_layer/src/npl_convolution.cpp,
// npl_activation_norm.cpp, npl_pooling.cpp, npl_tensor_ops.cpp) compile here
// unchanged, but they reference tiers that cannot be built in this container
// (LLVM-20 JIT, EVE, the operator graph / AGEE engine, SLEEF, libnuma). This
// file supplies those symbols with the behaviour the reference exhibits on the
// hot path when those tiers are absent or unused:
//   * AGEE / operator-graph calls fail. The reference's im2col path fails the
//     same way, because og_add_node rejects its tensor-less GEMM node
//     (advanced/operator_graph/src/operator_graph_construction.cpp:169-178).
//   * jkg_is_initialized() == 0, so npl_matmul takes the mil_sgemm path
//     (npl_tensor_ops.cpp:236-240). That path honours beta; the reference's
//     JIT path for dims <= 512 would ignore it.
//   * kfe_eve_is_available() == 1 and kfe_eve_simd_width() == 8, the width of
//     eve::wide<float> on AVX2 (advanced/kFusion_engine/src/kernel_fusion_eve.cpp:431-438).
//   * mil_is_initialized() == 1, backend OpenBLAS, and k_dispatch_matmul fails.
//     mil_sgemm then calls cblas_sgemm directly
//     (composite/mkernel_interface/src/mil_gemm.cpp:261-316). That is the same
//     BLAS routine the dispatcher would have picked.
//   * npl_init is replaced by a harness version that marks the state
//     initialised. It sets config.num_threads and a non-null scheduler
//     sentinel, so that ParallelFor (neural_primitives_internal.h:412-441)
//     runs its OpenMP split. ParallelFor only null-checks the scheduler.
#include <omp.h>
#include <cstdint>
#include <cstdlib>

#include "neural_primitives_internal.h"

namespace npl_internal {
NPLState g_npl_state;
}  // namespace npl_internal

using namespace npl_internal;

extern "C" {

// ---- OpenBLAS thread control (defined in ref_cblas_shim.c) -----------------
void npl_ref_blas_set_threads(int n);

// ---- harness replacements for npl_core.cpp entry points ---------------------
int npl_get_default_config(npl_config_t *c) {
  if (!c) return NPL_ERR_INVALID_ARG;
  // Same defaults as advanced/neural_layer/src/npl_core.cpp:172-189.
  c->num_threads = 0;
  c->enable_fusion = 1;
  c->enable_graph_optimization = 1;
  c->enable_jit = 1;
  c->enable_poly = 1;
  c->enable_vectorization = 1;
  c->enable_numa = 1;
  c->enable_memory_pooling = 1;
  c->workspace_size_mb = DEFAULT_WORKSPACE_SIZE_MB;
  c->verbose = 0;
  return NPL_OK;
}

static int g_scheduler_sentinel;

int npl_init(const npl_config_t *config) {
  std::lock_guard<std::mutex> lock(g_npl_state.state_mutex);
  if (g_npl_state.initialized) return NPL_OK;
  if (config) {
    g_npl_state.config = *config;
  } else {
    npl_get_default_config(&g_npl_state.config);
  }
  size_t n = g_npl_state.config.num_threads;
  if (n == 0) n = 1;
  g_npl_state.num_threads = n;
  omp_set_num_threads(static_cast<int>(n));
  npl_ref_blas_set_threads(static_cast<int>(n));
  // The reference reaches vmath_init through npl_init -> agee_init -> ... ->
  // mil_init (composite/mkernel_interface/src/mil_core.cpp:284-299); the
  // transcendental activations fail without it.
  if (vmath_init() != VMATH_OK) return NPL_ERR_INTERNAL;
  // Non-null so ParallelFor splits work; it is never dereferenced on the path.
  g_npl_state.scheduler =
      reinterpret_cast<jcore::global_thread::GlobalThreadScheduler *>(&g_scheduler_sentinel);
  g_npl_state.agee_session = nullptr;
  g_npl_state.initialized = true;
  return NPL_OK;
}

void npl_shutdown(void) {
  std::lock_guard<std::mutex> lock(g_npl_state.state_mutex);
  g_npl_state.initialized = false;
  g_npl_state.scheduler = nullptr;
  g_npl_state.total_ops_executed = 0;
}

int npl_is_initialized(void) { return g_npl_state.initialized ? 1 : 0; }

// ---- AGEE / operator graph: unavailable, calls fail --------------------------
int agee_is_initialized(void) { return 0; }
int agee_create_session(agee_session_t *) { return AGEE_ERR_NOT_INITIALIZED; }
void agee_destroy_session(agee_session_t) {}
int agee_create_plan_from_graph(agee_session_t, void *, agee_graph_plan_t *) {
  return AGEE_ERR_NOT_INITIALIZED;
}
void agee_destroy_plan(agee_graph_plan_t) {}
int agee_execute_plan(agee_session_t, agee_graph_plan_t, agee_exec_stats_t *) {
  return AGEE_ERR_NOT_INITIALIZED;
}
int agee_execute_plan_with_tensors(agee_session_t, agee_graph_plan_t, void **, size_t,
                                   void **, size_t, agee_exec_stats_t *) {
  return AGEE_ERR_NOT_INITIALIZED;
}
int og_create_graph(og_graph_t *g) {
  if (g) *g = nullptr;
  return OG_ERR_INTERNAL;
}
void og_destroy_graph(og_graph_t) {}
int og_add_tensor(og_graph_t, const og_tensor_t *, uint64_t *) { return OG_ERR_INTERNAL; }
int og_add_node(og_graph_t, const og_node_t *, uint64_t *) { return OG_ERR_INTERNAL; }
int og_add_edge(og_graph_t, uint64_t, uint64_t) { return OG_ERR_INTERNAL; }
int og_finalize_graph(og_graph_t) { return OG_ERR_INTERNAL; }
int og_optimize_graph(og_graph_t) { return OG_ERR_INTERNAL; }

// ---- LLVM JIT: not initialised ------------------------------------------------
int jkg_is_initialized(void) { return 0; }
int jkg_generate_gemm_tile(size_t, size_t, size_t, jkg_kernel_internal_t **h) {
  if (h) *h = nullptr;
  return JKG_ERR_NOT_INITIALIZED;
}
int jkg_generate_fused_gemm(size_t, size_t, size_t, jkg_activation_t, float,
                            jkg_kernel_internal_t **h) {
  if (h) *h = nullptr;
  return JKG_ERR_NOT_INITIALIZED;
}
void *jkg_get_kernel_function(jkg_kernel_internal_t *) { return nullptr; }
void jkg_release_kernel(jkg_kernel_internal_t *) {}

// ---- EVE width ----------------------------------------------------------------
int kfe_eve_is_available(void) { return 1; }
size_t kfe_eve_simd_width(void) { return 8; }

// ---- MIL backend state and kernel dispatch --------------------------------------
int mil_is_initialized(void) { return 1; }
mil_backend_t mil_get_backend(void) { return MIL_BACKEND_OPENBLAS; }
const char *mil_backend_name(mil_backend_t) { return "OpenBLAS"; }
int k_dispatch_matmul(const float *, const float *, float *, size_t, size_t, size_t) {
  return JCORE_ERR_NOT_FOUND;
}
const char *k_dispatch_get_last_selected_kernel() { return "cblas_sgemm"; }

// ---- libnuma helper used by mem_wrapper.c ----------------------------------------
int numa_helper_set_node(int) { return -1; }

// ---- ISA dispatch registry (vmath_init only); never initialised by the oracle -----
int jcore_init_dispatch(void) { return JCORE_OK; }

}  // extern "C"

// ---- SLEEF AVX2 kernels (vmath_sleef_isolated.cpp needs SLEEF, absent) -------------
// vmath_sleef_wrapper.cpp only calls these after sleef initialisation has found
// AVX2. The oracle never initialises SLEEF, so every vector op takes the
// wrapper's scalar fallback (for ReLU: fallback_maxf = std::max(x, 0),
// composite/vmath_engine/src/vmath_fallback.cpp:188). Each stub reports zero
// elements processed, which would also route any stray call to the scalar tail.
#define NPL_SLEEF_UNARY(name, T) \
  extern "C" size_t name(const T *, T *, size_t) { return 0; }
#define NPL_SLEEF_BINARY(name, T) \
  extern "C" size_t name(const T *, const T *, T *, size_t) { return 0; }
NPL_SLEEF_UNARY(sleef_avx2_expf_process, float)
NPL_SLEEF_UNARY(sleef_avx2_logf_process, float)
NPL_SLEEF_UNARY(sleef_avx2_log10f_process, float)
NPL_SLEEF_UNARY(sleef_avx2_sinf_process, float)
NPL_SLEEF_UNARY(sleef_avx2_cosf_process, float)
NPL_SLEEF_UNARY(sleef_avx2_tanf_process, float)
NPL_SLEEF_UNARY(sleef_avx2_sqrtf_process, float)
NPL_SLEEF_UNARY(sleef_avx2_cbrtf_process, float)
NPL_SLEEF_UNARY(sleef_avx2_sinhf_process, float)
NPL_SLEEF_UNARY(sleef_avx2_coshf_process, float)
NPL_SLEEF_UNARY(sleef_avx2_tanhf_process, float)
NPL_SLEEF_UNARY(sleef_avx2_asinf_process, float)
NPL_SLEEF_UNARY(sleef_avx2_acosf_process, float)
NPL_SLEEF_UNARY(sleef_avx2_atanf_process, float)
NPL_SLEEF_UNARY(sleef_avx2_erff_process, float)
NPL_SLEEF_UNARY(sleef_avx2_erfcf_process, float)
NPL_SLEEF_UNARY(sleef_avx2_log1pf_process, float)
NPL_SLEEF_BINARY(sleef_avx2_powf_process, float)
NPL_SLEEF_BINARY(sleef_avx2_atan2f_process, float)
NPL_SLEEF_BINARY(sleef_avx2_maxf_process, float)
NPL_SLEEF_BINARY(sleef_avx2_minf_process, float)
NPL_SLEEF_UNARY(sleef_avx2_exp_process, double)
NPL_SLEEF_UNARY(sleef_avx2_log_process, double)
NPL_SLEEF_UNARY(sleef_avx2_log10_process, double)
NPL_SLEEF_UNARY(sleef_avx2_sin_process, double)
NPL_SLEEF_UNARY(sleef_avx2_cos_process, double)
NPL_SLEEF_UNARY(sleef_avx2_tan_process, double)
NPL_SLEEF_UNARY(sleef_avx2_sqrt_process, double)
NPL_SLEEF_UNARY(sleef_avx2_cbrt_process, double)
NPL_SLEEF_UNARY(sleef_avx2_sinh_process, double)
NPL_SLEEF_UNARY(sleef_avx2_cosh_process, double)
NPL_SLEEF_UNARY(sleef_avx2_tanh_process, double)
NPL_SLEEF_UNARY(sleef_avx2_asin_process, double)
NPL_SLEEF_UNARY(sleef_avx2_acos_process, double)
NPL_SLEEF_UNARY(sleef_avx2_atan_process, double)
NPL_SLEEF_UNARY(sleef_avx2_erf_process, double)
NPL_SLEEF_UNARY(sleef_avx2_erfc_process, double)
NPL_SLEEF_UNARY(sleef_avx2_log1p_process, double)
NPL_SLEEF_BINARY(sleef_avx2_pow_process, double)
NPL_SLEEF_BINARY(sleef_avx2_atan2_process, double)
NPL_SLEEF_BINARY(sleef_avx2_max_process, double)
NPL_SLEEF_BINARY(sleef_avx2_min_process, double)
