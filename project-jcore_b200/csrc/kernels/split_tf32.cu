// TF32 hi/lo operand splitting for the 3xTF32 tensor-core kernels.
//
// The kernel writes the blocked, zero-padded, K-major layout the GEMM's TMA
// descriptors expect:  dst[block][part][row_in_block][kp]  with part 0 = hi,
// part 1 = lo, rows grouped in blocks of `row_block`, and kp a multiple of 32
// (one 128-byte swizzle row). Elements outside the logical matrix are zero,
// so the MMA pipeline never needs edge handling in K or in the block rows.
// It is a streaming pass: 4 bytes read, 8 bytes written per element.
#include <cuda_runtime.h>

#include "nplk_host.h"
#include "ptx_sm100.cuh"

namespace nplk {

// One launch does the whole preparation of a GEMM call; its 256-thread blocks
// take one of three jobs by block index:
//   [0, a_blocks)                 A split: 32 rows x 128 k of row-major A
//                                 (K contiguous), each thread 4 consecutive k
//                                 of 4 rows (16-byte stores per part);
//   [a_blocks, +b_blocks)         B split-transpose: 32 k x 128 n of row-major
//                                 B ([K][N]) through shared memory, so that
//                                 both the read (along n) and the write (along
//                                 k) are whole 128-byte rows;
//   [a_blocks+b_blocks, +c_blocks) C zeroing (8 rows a block), for the split-K
//                                 GEMM whose K slices add into C.
struct SplitJobs {
  const float *a;
  int64_t a_rows, a_cols, a_ld, a_rows_pad;
  float *a_dst;
  int a_shift;
  const float *b;
  int64_t b_krows, b_ncols, b_ld, b_npad;
  float *b_dst;
  int b_shift;
  int64_t kp;
  float *c;
  int64_t c_rows, c_cols, c_ld;
  int64_t a_blocks, b_blocks, c_blocks;
  int64_t a_kchunks, b_kchunks;  // 128-k chunks of A, 32-k chunks of B
  int a_vec, c_vec;              // 16-byte loads of A / stores into C allowed
};

__global__ void __launch_bounds__(256)
    split_operands_kernel(const __grid_constant__ SplitJobs j) {
  __shared__ float tile[32][129];
  griddep_launch_dependents();  // the GEMM's CTAs may set up meanwhile
  const int w = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int64_t i = blockIdx.x;
  if (i < j.a_blocks) {
    const int64_t k = (i % j.a_kchunks) * 128 + 4 * lane;
    if (k >= j.kp) return;
    const int64_t row_block = int64_t(1) << j.a_shift;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int64_t r = (i / j.a_kchunks) * 32 + w + 8 * q;
      if (r >= j.a_rows_pad) break;
      float x[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      if (r < j.a_rows) {
        const float *s = j.a + r * j.a_ld + k;
        if (j.a_vec && k + 4 <= j.a_cols) {
          const float4 v = __ldg(reinterpret_cast<const float4 *>(s));
          x[0] = v.x;
          x[1] = v.y;
          x[2] = v.z;
          x[3] = v.w;
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (k + e < j.a_cols) x[e] = __ldg(s + e);
        }
      }
      float4 hi, lo;
      tf32_split(x[0], hi.x, lo.x);
      tf32_split(x[1], hi.y, lo.y);
      tf32_split(x[2], hi.z, lo.z);
      tf32_split(x[3], hi.w, lo.w);
      const int64_t blk = r >> j.a_shift;
      float *d = j.a_dst + ((blk * 2) * row_block + (r & (row_block - 1))) * j.kp + k;
      *reinterpret_cast<float4 *>(d) = hi;
      *reinterpret_cast<float4 *>(d + row_block * j.kp) = lo;
    }
    return;
  }
  i -= j.a_blocks;
  if (i < j.b_blocks) {
    const int64_t k0 = (i % j.b_kchunks) * 32;
    const int64_t n0 = (i / j.b_kchunks) * 128;
    // Read: warp w takes k rows w, w+8, w+16, w+24; lane + 32 q along n, so
    // each load instruction reads 128 contiguous bytes and each shared store
    // hits 32 distinct banks.
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int kk = w + 8 * r;
      const int64_t k = k0 + kk;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int64_t n = n0 + lane + 32 * q;
        tile[kk][lane + 32 * q] =
            (k < j.b_krows && n < j.b_ncols) ? __ldg(j.b + k * j.b_ld + n) : 0.0f;
      }
    }
    __syncthreads();
    // Write: warp w takes output rows (source columns) w, w+8, ..., w+120;
    // lane = k, so each part's store is one 128-byte row segment.
    const int64_t row_block = int64_t(1) << j.b_shift;
#pragma unroll 4
    for (int r = 0; r < 16; ++r) {
      const int nn = w + 8 * r;
      const int64_t n = n0 + nn;
      if (n >= j.b_npad) break;
      float hi, lo;
      tf32_split(tile[lane][nn], hi, lo);
      const int64_t blk = n >> j.b_shift;
      float *d = j.b_dst + ((blk * 2) * row_block + (n & (row_block - 1))) * j.kp + k0 + lane;
      d[0] = hi;
      d[row_block * j.kp] = lo;
    }
    return;
  }
  i -= j.b_blocks;
  if (i < j.c_blocks) {
    const int64_t r = i * 8 + w;
    if (r >= j.c_rows) return;
    float *crow = j.c + r * j.c_ld;
    if (j.c_vec) {
      for (int64_t c = 4 * lane; c < j.c_cols; c += 128)
        *reinterpret_cast<float4 *>(crow + c) = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    } else {
      for (int64_t c = lane; c < j.c_cols; c += 32) crow[c] = 0.0f;
    }
  }
}

static int log2_exact(int v) {
  int s = 0;
  while ((1 << s) < v) ++s;
  return (1 << s) == v ? s : -1;
}

int launch_split_operands(cudaStream_t s, const float *a, int64_t rows, int64_t cols,
                          int64_t lda, float *a_dst, int a_row_block, int64_t rows_pad,
                          const float *b, int64_t krows, int64_t ncols, int64_t ldb,
                          float *b_dst, int b_row_block, int64_t npad, int64_t kp, float *c,
                          int64_t ldc) {
  SplitJobs j{};
  j.a_shift = log2_exact(a_row_block);
  j.b_shift = log2_exact(b_row_block);
  if (j.a_shift < 0 || j.b_shift < 0 || kp % 32 != 0 || rows_pad % a_row_block != 0 ||
      npad % b_row_block != 0 || a_row_block % 32 != 0)
    return kErrInvalidArg;
  j.a = a;
  j.a_rows = rows;
  j.a_cols = cols;
  j.a_ld = lda;
  j.a_rows_pad = rows_pad;
  j.a_dst = a_dst;
  j.b = b;
  j.b_krows = krows;
  j.b_ncols = ncols;
  j.b_ld = ldb;
  j.b_npad = npad;
  j.b_dst = b_dst;
  j.kp = kp;
  j.a_kchunks = ceil_div(kp, 128);
  j.b_kchunks = kp / 32;
  j.a_blocks = (rows_pad / 32) * j.a_kchunks;
  j.b_blocks = ceil_div(npad, 128) * j.b_kchunks;
  j.a_vec = (lda % 4 == 0) && ((reinterpret_cast<uintptr_t>(a) & 15u) == 0);
  if (c) {
    j.c = c;
    j.c_rows = rows;
    j.c_cols = ncols;
    j.c_ld = ldc;
    j.c_blocks = ceil_div(rows, 8);
    j.c_vec = (ldc % 4 == 0) && (ncols % 4 == 0) && ((reinterpret_cast<uintptr_t>(c) & 15u) == 0);
  }
  const int64_t blocks = j.a_blocks + j.b_blocks + j.c_blocks;
  if (blocks > 2147483647) return kErrUnsupported;
  split_operands_kernel<<<static_cast<unsigned>(blocks), 256, 0, s>>>(j);
  count_launch();
  return launch_result();
}

}  // namespace nplk
