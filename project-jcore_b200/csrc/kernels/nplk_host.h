// Host-side helpers shared by the kernel launchers: CUDA error mapping,
// per-device properties, TMA descriptor encoding, the library status word and
// the launch counter.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

#include "npl_kernels.h"

namespace nplk {

// NPL error codes (mirrors include/neural_primitives.h).
constexpr int kOk = 0;
constexpr int kErrInvalidArg = -2;
constexpr int kErrNoMemory = -3;
constexpr int kErrInternal = -4;
constexpr int kErrUnsupported = -5;
constexpr int kErrOom = -7;

int map_cuda_error(cudaError_t e);

// Number of SMs of the current device (cached per device).
int sm_count();

// Device status word of the current device (allocated on first use).
int *device_status_word();

// The same word if it has been allocated on the current device, else NULL
// (nothing has reported to it yet). Never allocates.
int *device_status_word_if_allocated();

// Status word of the no-allocation conv entry point on the current device if
// that entry point has been set up there, else NULL. Never allocates.
int *noalloc_status_word_if_set_up();

// Fault injection (nplk_debug_arm_wait_timeout): the stall, in microseconds,
// armed for the next launch of kernel family `which` (NPLK_DEBUG_*), which
// this call consumes; 0 when nothing is armed.
uint32_t take_armed_stall(int which);

// Counts one library kernel launch on the calling thread.
void count_launch(uint64_t n = 1);

// Checks the last launch and maps the error.
int launch_result();

// Raises a kernel's dynamic shared-memory limit on the current device (once
// per device and function).
int ensure_dynamic_smem(const void *func, int bytes);

// 2-D fp32 tensor map: dims {inner, outer} elements, row pitch in bytes,
// box {box_inner, box_outer}, 128-byte swizzle, zero fill out of bounds.
int encode_tmap_2d_f32_sw128(CUtensorMap *map, const void *base, uint64_t inner,
                             uint64_t outer, uint64_t row_pitch_bytes, uint32_t box_inner,
                             uint32_t box_outer);
// The same with the 128-byte swizzle of 32-byte atoms (MN-major tf32 operands).
int encode_tmap_2d_f32_sw128_atom32(CUtensorMap *map, const void *base, uint64_t inner,
                                    uint64_t outer, uint64_t row_pitch_bytes,
                                    uint32_t box_inner, uint32_t box_outer);

// 4-D NHWC fp32 im2col tensor map (dims {c, w, h, n}, densely packed): each
// load gathers `pixels` output pixels x `channels` channels, walking the
// bounding box [lower, dim-1+upper] of every image with the given traversal
// strides (W then H then N); corners are in [-128, 127]. 128-byte swizzle,
// zero fill outside the image.
int encode_tmap_im2col_nhwc_f32_sw128(CUtensorMap *map, const void *base, uint64_t c,
                                     uint64_t w, uint64_t h, uint64_t n, int lower_w,
                                     int lower_h, int upper_w, int upper_h, uint32_t stride_w,
                                     uint32_t stride_h, uint32_t channels, uint32_t pixels);

// Launches `kernel` with programmatic stream serialization: it may start
// while the previous kernel in the stream is still running and must call
// griddep_wait() before reading what that kernel writes. Counts the launch.
template <typename... KArgs, typename... Args>
int launch_programmatic(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                        cudaStream_t stream, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  count_launch();
  return map_cuda_error(cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...));
}

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

}  // namespace nplk
