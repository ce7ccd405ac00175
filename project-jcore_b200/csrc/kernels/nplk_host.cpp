// Host-side helpers for the kernel launchers (see nplk_host.h).
#include "nplk_host.h"

#include <cudaTypedefs.h>

#include <atomic>
#include <map>
#include <mutex>
#include <utility>

namespace nplk {

int map_cuda_error(cudaError_t e) {
  switch (e) {
    case cudaSuccess:
      return kOk;
    case cudaErrorMemoryAllocation:
      return kErrOom;
    case cudaErrorInvalidValue:
    case cudaErrorInvalidDevicePointer:
      return kErrInvalidArg;
    default:
      return kErrInternal;
  }
}

namespace {
constexpr int kMaxDevices = 64;
std::once_flag g_sm_once[kMaxDevices];
int g_sm_count[kMaxDevices];
std::mutex g_status_mu;
int *g_status[kMaxDevices];
thread_local uint64_t t_launches = 0;
constexpr int kDebugFamilies = 3;  // index = NPLK_DEBUG_* code
std::atomic<uint32_t> g_armed_stall[kDebugFamilies];

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      p = nullptr;
    }
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

PFN_cuTensorMapEncodeIm2col_v12000 encode_im2col_fn() {
  static PFN_cuTensorMapEncodeIm2col_v12000 fn = [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeIm2col", &p, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess) {
      p = nullptr;
    }
    return reinterpret_cast<PFN_cuTensorMapEncodeIm2col_v12000>(p);
  }();
  return fn;
}
}  // namespace

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  std::call_once(g_sm_once[dev], [dev] {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_sm_count[dev] = n > 0 ? n : 148;
  });
  return g_sm_count[dev];
}

int *device_status_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_status_mu);
  if (!g_status[dev]) {
    int *p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, sizeof(int)) != cudaSuccess) {
      cudaFree(p);
      return nullptr;
    }
    g_status[dev] = p;
  }
  return g_status[dev];
}

int *device_status_word_if_allocated() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_status_mu);
  return g_status[dev];
}

uint32_t take_armed_stall(int which) {
  if (which <= 0 || which >= kDebugFamilies) return 0u;
  // Cheap when nothing is armed: a load, no read-modify-write.
  if (g_armed_stall[which].load(std::memory_order_relaxed) == 0u) return 0u;
  return g_armed_stall[which].exchange(0u);
}

void count_launch(uint64_t n) { t_launches += n; }

int launch_result() { return map_cuda_error(cudaGetLastError()); }

int ensure_dynamic_smem(const void *func, int bytes) {
  // The attribute is raised, never lowered: a kernel launched with several
  // shared-memory sizes keeps the largest one set so far.
  static std::mutex mu;
  static std::map<std::pair<int, const void *>, int> set_bytes;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kErrInternal;
  std::lock_guard<std::mutex> lock(mu);
  auto it = set_bytes.find({dev, func});
  if (it != set_bytes.end() && it->second >= bytes) return kOk;
  cudaError_t e =
      cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return map_cuda_error(e);
  set_bytes[{dev, func}] = bytes;
  return kOk;
}

namespace {
int encode_2d_f32(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer,
                  uint64_t row_pitch_bytes, uint32_t box_inner, uint32_t box_outer,
                  CUtensorMapSwizzle swizzle);
}  // namespace

int encode_tmap_2d_f32_sw128(CUtensorMap *map, const void *base, uint64_t inner,
                             uint64_t outer, uint64_t row_pitch_bytes, uint32_t box_inner,
                             uint32_t box_outer) {
  return encode_2d_f32(map, base, inner, outer, row_pitch_bytes, box_inner, box_outer,
                       CU_TENSOR_MAP_SWIZZLE_128B);
}

int encode_tmap_2d_f32_sw128_atom32(CUtensorMap *map, const void *base, uint64_t inner,
                                    uint64_t outer, uint64_t row_pitch_bytes,
                                    uint32_t box_inner, uint32_t box_outer) {
  return encode_2d_f32(map, base, inner, outer, row_pitch_bytes, box_inner, box_outer,
                       CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
}

namespace {
int encode_2d_f32(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer,
                  uint64_t row_pitch_bytes, uint32_t box_inner, uint32_t box_outer,
                  CUtensorMapSwizzle swizzle) {
  auto fn = encode_fn();
  if (!fn) return kErrInternal;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (row_pitch_bytes & 15u) != 0)
    return kErrInvalidArg;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_pitch_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void *>(base), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kOk : kErrInternal;
}
}  // namespace

int encode_tmap_im2col_nhwc_f32_sw128(CUtensorMap *map, const void *base, uint64_t c,
                                     uint64_t w, uint64_t h, uint64_t n, int lower_w,
                                     int lower_h, int upper_w, int upper_h, uint32_t stride_w,
                                     uint32_t stride_h, uint32_t channels, uint32_t pixels) {
  auto fn = encode_im2col_fn();
  if (!fn) return kErrInternal;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (c * 4) % 16 != 0) return kErrInvalidArg;
  cuuint64_t dims[4] = {c, w, h, n};
  cuuint64_t strides[3] = {c * 4, c * w * 4, c * w * h * 4};
  int lower[2] = {lower_w, lower_h};
  int upper[2] = {upper_w, upper_h};
  cuuint32_t estr[4] = {1, stride_w, stride_h, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void *>(base), dims,
                  strides, lower, upper, channels, pixels, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? kOk : kErrInternal;
}

}  // namespace nplk

extern "C" int nplk_read_status(void *stream) {
  // Two words can hold a report: the library's per-device word (kernels
  // launched with status == NULL) and the word of the no-allocation conv
  // entry point. Each is read and cleared only if it exists, so reading the
  // status allocates nothing. The first non-zero code is returned.
  int *words[2] = {nplk::device_status_word_if_allocated(),
                   nplk::noalloc_status_word_if_set_up()};
  int vals[2] = {0, 0};
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int i = 0; i < 2; ++i) {
    if (!words[i]) continue;
    if (cudaMemcpyAsync(&vals[i], words[i], sizeof(int), cudaMemcpyDeviceToHost, s) !=
        cudaSuccess)
      return nplk::kErrInternal;
    if (cudaMemsetAsync(words[i], 0, sizeof(int), s) != cudaSuccess) return nplk::kErrInternal;
  }
  if (cudaStreamSynchronize(s) != cudaSuccess) return nplk::kErrInternal;
  return vals[0] ? vals[0] : vals[1];
}

extern "C" int nplk_debug_arm_wait_timeout(int which, uint32_t stall_us) {
  if (which != NPLK_DEBUG_GEMM && which != NPLK_DEBUG_CONV_WINDOW) return nplk::kErrInvalidArg;
  if (stall_us > 60000000u) return nplk::kErrInvalidArg;  // at most one minute
  nplk::g_armed_stall[which].store(stall_us);
  return nplk::kOk;
}

extern "C" uint64_t nplk_take_launch_count(void) {
  uint64_t n = nplk::t_launches;
  nplk::t_launches = 0;
  return n;
}
