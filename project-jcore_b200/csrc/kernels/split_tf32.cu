// TF32 hi/lo operand splitting for the 3xTF32 tensor-core kernels.
//
// Both kernels write the blocked, zero-padded, K-major layout the GEMM's TMA
// descriptors expect:  dst[block][part][row_in_block][kp]  with part 0 = hi,
// part 1 = lo, rows grouped in blocks of `row_block`, and kp a multiple of 32
// (one 128-byte swizzle row). Elements outside the logical matrix are zero,
// so the MMA pipeline never needs edge handling in K or in the block rows.
// Both kernels are HBM-bound streaming passes: 4 bytes read, 8 bytes written
// per element.
#include <cuda_runtime.h>

#include "nplk_host.h"
#include "ptx_sm100.cuh"

namespace nplk {

// Row-major source (K contiguous) -> blocked hi/lo. Each thread produces 4
// consecutive k of one row (one 16-byte store per part). grid.y strides rows.
__global__ void split_rows_kernel(const float *__restrict__ src, int64_t rows, int64_t cols,
                                  int64_t ld, int64_t col_offset, float *__restrict__ dst,
                                  int row_block_shift, int64_t kp, int64_t rows_pad) {
  griddep_launch_dependents();  // the B split and the GEMM may start meanwhile
  const int64_t k = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  if (k >= kp) return;
  const int64_t row_block = int64_t(1) << row_block_shift;
  for (int64_t r = blockIdx.y; r < rows_pad; r += gridDim.y) {
    float x[4];
    const float *s = src + r * ld + col_offset + k;
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = (r < rows && k + j < cols) ? __ldg(s + j) : 0.0f;
    float4 hi, lo;
    tf32_split(x[0], hi.x, lo.x);
    tf32_split(x[1], hi.y, lo.y);
    tf32_split(x[2], hi.z, lo.z);
    tf32_split(x[3], hi.w, lo.w);
    const int64_t blk = r >> row_block_shift;
    const int64_t rr = r & (row_block - 1);
    float *d = dst + ((blk * 2) * row_block + rr) * kp + k;
    *reinterpret_cast<float4 *>(d) = hi;
    *reinterpret_cast<float4 *>(d + row_block * kp) = lo;
  }
}

// Row-major [krows][ncols] source -> transposed blocked hi/lo (rows of the
// destination are source columns). 32x32 tiles through shared memory so that
// both the read (along n) and the write (along k) are coalesced.
__global__ void split_transpose_kernel(const float *__restrict__ src, int64_t krows,
                                       int64_t ncols, int64_t ld, float *__restrict__ dst,
                                       int row_block_shift, int64_t kp, int64_t npad) {
  __shared__ float tile[32][33];
  griddep_launch_dependents();
  const int64_t k0 = static_cast<int64_t>(blockIdx.x) * 32;
  const int64_t row_block = int64_t(1) << row_block_shift;
  for (int64_t n0 = static_cast<int64_t>(blockIdx.y) * 32; n0 < npad;
       n0 += static_cast<int64_t>(gridDim.y) * 32) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t k = k0 + threadIdx.y + 8 * i;
      const int64_t n = n0 + threadIdx.x;
      tile[threadIdx.y + 8 * i][threadIdx.x] =
          (k < krows && n < ncols) ? __ldg(src + k * ld + n) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t n = n0 + threadIdx.y + 8 * i;
      const int64_t k = k0 + threadIdx.x;
      float hi, lo;
      tf32_split(tile[threadIdx.x][threadIdx.y + 8 * i], hi, lo);
      const int64_t blk = n >> row_block_shift;
      const int64_t rr = n & (row_block - 1);
      float *d = dst + ((blk * 2) * row_block + rr) * kp + k;
      d[0] = hi;
      d[row_block * kp] = lo;
    }
    __syncthreads();
  }
  // When launched to overlap the A split before it, finish only after it:
  // the GEMM behind waits for this grid, and so for both splits.
  griddep_wait();
}

static int log2_exact(int v) {
  int s = 0;
  while ((1 << s) < v) ++s;
  return (1 << s) == v ? s : -1;
}

int launch_split_rows(cudaStream_t s, const float *src, int64_t rows, int64_t cols, int64_t ld,
                      int64_t col_offset, float *dst, int row_block, int64_t kp,
                      int64_t rows_pad) {
  const int shift = log2_exact(row_block);
  if (shift < 0 || kp % 32 != 0 || rows_pad % row_block != 0) return kErrInvalidArg;
  const int threads = 128;
  const int64_t gx = ceil_div(kp / 4, threads);
  const int64_t gy = rows_pad < 65535 ? rows_pad : 65535;
  split_rows_kernel<<<dim3(static_cast<unsigned>(gx), static_cast<unsigned>(gy)), threads, 0,
                      s>>>(src, rows, cols, ld, col_offset, dst, shift, kp, rows_pad);
  count_launch();
  return launch_result();
}

int launch_split_transpose(cudaStream_t s, const float *src, int64_t krows, int64_t ncols,
                           int64_t ld, float *dst, int row_block, int64_t kp, int64_t npad,
                           bool overlap_previous) {
  const int shift = log2_exact(row_block);
  if (shift < 0 || kp % 32 != 0 || npad % 32 != 0 || npad % row_block != 0)
    return kErrInvalidArg;
  const int64_t gx = kp / 32;
  int64_t gy = npad / 32;
  if (gy > 65535) gy = 65535;
  if (gx > 2147483647) return kErrUnsupported;
  const dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(gy));
  if (overlap_previous)
    return launch_programmatic(split_transpose_kernel, grid, dim3(32, 8), 0, s, src, krows, ncols,
                               ld, dst, shift, kp, npad);
  split_transpose_kernel<<<grid, dim3(32, 8), 0, s>>>(src, krows, ncols, ld, dst, shift, kp, npad);
  count_launch();
  return launch_result();
}

}  // namespace nplk
