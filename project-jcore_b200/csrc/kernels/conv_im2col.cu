// Fused conv2d + bias + BN + activation for C_in % 32 == 0, with the A
// operand (the implicit im2col matrix) fetched by the Tensor Memory
// Accelerator in im2col mode.
//
// Same GEMM view, k order (channel-block-major: each 32-wide k-block is one
// filter tap over 32 consecutive channels), 3xTF32 MMA sequence and epilogue
// as the direct-gather kernel in conv_igemm.cu, and therefore the same
// results bit for bit; only the way A reaches shared memory differs:
//
//   1. nchw_to_nhwc_split_kernel rewrites the NCHW input once as two NHWC
//      planes, hi = tf32 truncation of x and lo = x - hi (exact), so that the
//      32 channels of a pixel are one contiguous 128-byte row;
//   2. conv_im2col_3xtf32_kernel: one producer thread issues, per k-block
//      (tile, channel block cb, tap (kh, kw)), two im2col TMA loads (hi, lo)
//      of 128 output pixels x 32 channels, walking the output pixels of the
//      tile in (n, oh, ow) order with the input position shifted by the tap
//      (kw*dw, kh*dh); padding is the TMA's zero fill outside the image. It
//      also loads the [W'_hi; W'_lo] slab of the k-block (2-D tiled TMA).
//      The MMA warp and the four epilogue warps are those of the direct
//      kernel.
//
// Roles: per pipeline one TMA producer thread and one MMA-issuing warp, then
// four epilogue warps (see ConvTmaTraits).
// Reference semantics: as conv_igemm.cu (ExecuteConvDirect,
// advanced/neural_layer/src/npl_convolution.cpp:248-378, plus the fused
// bias / inference BN / activation epilogue).
#include <cuda_runtime.h>

#include "conv_common.cuh"
#include "nplk_host.h"

namespace nplk {

// ---------------------------------------------------------------------------
// NCHW -> NHWC hi/lo planes
// ---------------------------------------------------------------------------
constexpr int kTrC = 32;  // channels per block
constexpr int kTrP = 64;  // pixels per block

// Block (256 threads) = 32 channels x 64 pixels of one image: coalesced
// reads along the pixels of each channel, coalesced 16-byte writes along
// the channels of each pixel. The shared tile is padded to 65 columns, which
// makes the transposed reads conflict-free.
// kSplit: write hi = trunc(x) and lo = x - hi; otherwise write x itself to
// hi (lo unused).
template <bool kSplit>
__global__ void __launch_bounds__(256) nchw_to_nhwc_split_kernel(const float *__restrict__ x,
                                                                 float *__restrict__ hi,
                                                                 float *__restrict__ lo, int C,
                                                                 int64_t HW, int vec) {
  __shared__ float tile[kTrC][kTrP + 1];
  const int n = blockIdx.z;
  const int c0 = blockIdx.y * kTrC;
  const int64_t p0 = static_cast<int64_t>(blockIdx.x) * kTrP;
  const float *xb = x + (static_cast<int64_t>(n) * C + c0) * HW + p0;
  const int t = threadIdx.x;
  if (vec && p0 + kTrP <= HW) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int q = t + i * 256;
      const int c = q >> 4;
      const int p = (q & 15) * 4;
      const float4 v = __ldg(reinterpret_cast<const float4 *>(xb + c * HW + p));
      tile[c][p + 0] = v.x;
      tile[c][p + 1] = v.y;
      tile[c][p + 2] = v.z;
      tile[c][p + 3] = v.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int q = t + i * 256;
      const int c = q >> 6;
      const int p = q & 63;
      tile[c][p] = (p0 + p < HW) ? __ldg(xb + c * HW + p) : 0.0f;
    }
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int q = t + i * 256;
    const int p = q >> 3;
    const int c = (q & 7) * 4;
    if (p0 + p < HW) {
      const int64_t off = (static_cast<int64_t>(n) * HW + p0 + p) * C + c0 + c;
      if (kSplit) {
        float4 h, l;
        tf32_split_trunc(tile[c + 0][p], h.x, l.x);
        tf32_split_trunc(tile[c + 1][p], h.y, l.y);
        tf32_split_trunc(tile[c + 2][p], h.z, l.z);
        tf32_split_trunc(tile[c + 3][p], h.w, l.w);
        *reinterpret_cast<float4 *>(hi + off) = h;
        *reinterpret_cast<float4 *>(lo + off) = l;
      } else {
        *reinterpret_cast<float4 *>(hi + off) =
            make_float4(tile[c + 0][p], tile[c + 1][p], tile[c + 2][p], tile[c + 3][p]);
      }
    }
  }
}

int launch_nchw_to_nhwc_split(cudaStream_t s, const float *x, float *hi, float *lo, int n, int c,
                              int64_t hw) {
  if (c % kTrC != 0 || n <= 0 || n > 65535 || c / kTrC > 65535 || hw <= 0) return kErrInvalidArg;
  const int64_t px_blocks = ceil_div(hw, kTrP);
  if (px_blocks > 0x7fffffff) return kErrUnsupported;
  const int vec = (hw % 4 == 0) && ((reinterpret_cast<uintptr_t>(x) & 15u) == 0);
  dim3 grid(static_cast<unsigned>(px_blocks), static_cast<unsigned>(c / kTrC),
            static_cast<unsigned>(n));
  if (lo)
    nchw_to_nhwc_split_kernel<true><<<grid, 256, 0, s>>>(x, hi, lo, c, hw, vec);
  else
    nchw_to_nhwc_split_kernel<false><<<grid, 256, 0, s>>>(x, hi, nullptr, c, hw, vec);
  count_launch();
  return launch_result();
}

// ---------------------------------------------------------------------------
// TMA-im2col implicit-GEMM conv
// ---------------------------------------------------------------------------
// Pipelines: the tensor core accepts roughly one tcgen05.mma ahead of the one
// it is executing, so every cycle the issuing thread spends elsewhere (an
// mbarrier wait costs ~200 cycles even on a completed phase, since the
// tensor core's operand reads keep the shared-memory pipe busy) idles the
// tensor pipe. With C_out <= 64 the per-k-block MMA work (~470 cycles) is
// short enough for that to cost ~40%, so the CTA runs two independent
// pipelines (producer thread, stage ring, MMA warp, accumulators), each on
// alternate tiles: while one MMA warp waits for its next stage, the other's
// MMAs keep the tensor pipe busy. Wider tiles (C_out > 64) do twice the MMA
// work per k-block and run one pipeline with a deeper ring.
template <int BNC>
struct ConvTmaTraits {
  static constexpr int kPipes = BNC == 64 ? 2 : 1;
  static constexpr int kStages = BNC == 64 ? 2 : 3;  // per pipeline
  static constexpr int kAHalfBytes = kConvBM * kConvBK * 4;  // 16 KB: hi or lo
  static constexpr int kBBytes = 2 * BNC * kConvBK * 4;       // [W'_hi; W'_lo]
  static constexpr int kStageBytes = 2 * kAHalfBytes + kBBytes;
  static constexpr int kFirstMmaWarp = kPipes;        // warps [0, kPipes): producers
  static constexpr int kFirstEpiWarp = 2 * kPipes;    // 4 epilogue warps after the MMA warps
  static constexpr int kThreads = (2 * kPipes + 4) * 32;
  static constexpr int kAccCols = 2 * BNC;            // one accumulator: [hi*W | hi*W_lo]
  static constexpr int kAccPerPipe = 2;               // double buffered
  static constexpr int kTmemCols = kPipes * kAccPerPipe * kAccCols;  // 512 in both cases
  static constexpr int kBarrierBytes = 256;
  static constexpr int kSmemBytes =
      1024 + kPipes * kStages * kStageBytes + kBarrierBytes + BNC * 20;
  static_assert(kTmemCols == 512, "TMEM budget");
};

template <int BNC, int kAct>
__global__ void __launch_bounds__(ConvTmaTraits<BNC>::kThreads, 1)
    conv_im2col_3xtf32_kernel(const __grid_constant__ CUtensorMap map_hi,
                              const __grid_constant__ CUtensorMap map_lo,
                              const __grid_constant__ CUtensorMap map_w, const ConvParams p) {
  using T = ConvTmaTraits<BNC>;
  constexpr int P = T::kPipes;
  constexpr int S = T::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align_smem_1024(smem_raw);
  uint8_t *bars = smem + P * S * T::kStageBytes;
  uint64_t *full = reinterpret_cast<uint64_t *>(bars);  // [P][S]
  uint64_t *empty = full + P * S;                        // [P][S]
  uint64_t *acc_full = empty + P * S;                    // [P * kAccPerPipe]
  uint64_t *acc_empty = acc_full + P * T::kAccPerPipe;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + P * T::kAccPerPipe);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  float4 *ep_s = reinterpret_cast<float4 *>(bars + T::kBarrierBytes);
  float *ep_beta_s = reinterpret_cast<float *>(ep_s + BNC);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P * S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < P * T::kAccPerPipe; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&map_hi);
    tma_prefetch_desc(&map_lo);
    tma_prefetch_desc(&map_w);
  }
  if (warp == T::kFirstMmaWarp) {
    tmem_alloc(tmem_slot, T::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  const int num_tiles = p.m_blocks * p.n_blocks;
  // Local tile j of this CTA is tile blockIdx.x + j*gridDim.x; pipeline
  // j % P runs it as its (j / P)-th tile.

  if (warp < P) {
    // ---------------- TMA producer of pipeline `pipe` ----------------
    const int pipe = warp;
    if (lane == 0) {
      const int taps = p.KH * p.KW;
      uint64_t *pf = full + pipe * S;
      uint64_t *pe = empty + pipe * S;
      uint8_t *pst = smem + pipe * S * T::kStageBytes;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0, issued_phase = 0;  // per-stage bits: loads in flight, their phase
      for (int tile = blockIdx.x + pipe * gridDim.x; tile < num_tiles; tile += P * gridDim.x) {
        const int mb = tile / p.n_blocks;
        const int nb = tile - mb * p.n_blocks;
        const int m0 = mb * kConvBM;
        const int n0 = m0 / static_cast<int>(p.HoWo);
        const int pix = m0 - n0 * static_cast<int>(p.HoWo);
        const int oh0 = pix / p.Wo;
        const int ow0 = pix - oh0 * p.Wo;
        const int w0 = ow0 * p.sw - p.pl;
        const int h0 = oh0 * p.sh - p.pt;
        int cb = 0, tap = 0;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          const int kh = tap / p.KW;
          const int kw = tap - kh * p.KW;
          if (!mbar_wait(&pe[stage], phase ^ 1u, abort_flag, p.status, kStatusTimeoutProducer))
            goto producer_done;
          uint8_t *st = pst + stage * T::kStageBytes;
          mbar_arrive_expect_tx(&pf[stage], T::kStageBytes);
          const uint16_t ow_off = static_cast<uint16_t>(kw * p.dw);
          const uint16_t oh_off = static_cast<uint16_t>(kh * p.dh);
          tma_load_im2col_4d(&map_hi, &pf[stage], st, cb * kConvBK, w0, h0, n0, ow_off, oh_off);
          tma_load_im2col_4d(&map_lo, &pf[stage], st + T::kAHalfBytes, cb * kConvBK, w0, h0, n0,
                             ow_off, oh_off);
          tma_load_2d(&map_w, &pf[stage], st + 2 * T::kAHalfBytes, kb * kConvBK, nb * 2 * BNC);
          issued |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          if (++tap == taps) {
            tap = 0;
            ++cb;
          }
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    producer_done:
      // Let every issued copy land before the CTA can exit (all of them
      // already have unless the CTA aborted).
      for (int s = 0; s < S; ++s)
        if (issued & (1u << s)) mbar_drain(&pf[s], (issued_phase >> s) & 1u);
    }
  } else if (warp < T::kFirstEpiWarp) {
    // ---------------- MMA issuer of pipeline `pipe` ----------------
    const int pipe = warp - T::kFirstMmaWarp;
    if (lane == 0) {
      const uint32_t idesc_2n = umma_idesc_tf32(kConvBM, 2 * BNC);
      const uint32_t idesc_n = umma_idesc_tf32(kConvBM, BNC);
      const uint64_t desc0 =
          umma_desc_sw128(smem_u32(smem + pipe * S * T::kStageBytes));
      constexpr uint64_t kLoOff = T::kAHalfBytes >> 4;
      constexpr uint64_t kBOff = (2 * T::kAHalfBytes) >> 4;
      uint64_t *pf = full + pipe * S;
      uint64_t *pe = empty + pipe * S;
      int stage = 0;
      uint32_t phase = 0;
      int jj = 0;
      for (int tile = blockIdx.x + pipe * gridDim.x; tile < num_tiles;
           tile += P * gridDim.x, ++jj) {
        const int acc = pipe * T::kAccPerPipe + (jj & 1);
        const uint32_t acc_phase = (jj >> 1) & 1;
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, abort_flag, p.status,
                       kStatusTimeoutAccFree))
          break;
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * T::kAccCols;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&pf[stage], phase, abort_flag, p.status, kStatusTimeoutMma))
            goto mma_done;
          tc_fence_after_sync();
          const uint64_t a_desc = desc0 + static_cast<uint64_t>(stage * (T::kStageBytes >> 4));
          const uint64_t b_desc = a_desc + kBOff;
#pragma unroll
          for (int kk = 0; kk < kConvBK / 8; ++kk) {
            mma_tf32_ss(d_tmem, a_desc + 2 * kk, b_desc + 2 * kk, idesc_2n,
                        (kb > 0 || kk > 0) ? 1u : 0u);
            mma_tf32_ss(d_tmem, a_desc + kLoOff + 2 * kk, b_desc + 2 * kk, idesc_n, 1u);
          }
          mma_commit(&pe[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        mma_commit(&acc_full[acc]);
      }
    mma_done:;
    }
  } else {
    // ---------------- epilogue (4 warps, one per TMEM lane quadrant) ----------------
    const int quad = warp & 3;
    const int et = threadIdx.x - T::kFirstEpiWarp * 32;  // 0..127
    int j = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++j) {
      const int pipe = j % P;
      const int jj = j / P;
      const int acc = pipe * T::kAccPerPipe + (jj & 1);
      const uint32_t acc_phase = (jj >> 1) & 1;
      const int mb = tile / p.n_blocks;
      const int nb = tile - mb * p.n_blocks;
      if (!conv_epilogue_tile<BNC, kAct>(p, tmem_base + acc * T::kAccCols, quad, lane, et, mb, nb,
                                         ep_s, ep_beta_s, &acc_full[acc], acc_phase, abort_flag))
        break;
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
    }
  }

  __syncthreads();
  if (warp == T::kFirstMmaWarp) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, T::kTmemCols);
  }
}

namespace {

struct Im2colCorners {
  int lower_w, lower_h, upper_w, upper_h;
};

// Bounding box of the traversal in each image: output column ow starts at
// input column ow*sw - pl, so the box spans [-pl, (Wo-1)*sw - pl], i.e.
// lower = -pl and upper = (Wo-1)*sw - pl - (W-1) relative to the far edge.
Im2colCorners corners(const ConvParams &p) {
  Im2colCorners c;
  c.lower_w = -p.pl;
  c.lower_h = -p.pt;
  c.upper_w = (p.Wo - 1) * p.sw - p.pl - (p.W - 1);
  c.upper_h = (p.Ho - 1) * p.sh - p.pt - (p.H - 1);
  return c;
}

bool in_corner_range(int v) { return v >= -128 && v <= 127; }

template <int BNC, int kAct>
int launch_tma(cudaStream_t s, const CUtensorMap &mh, const CUtensorMap &ml, const CUtensorMap &mw,
               const ConvParams &prm) {
  using T = ConvTmaTraits<BNC>;
  int rc = ensure_dynamic_smem(reinterpret_cast<const void *>(conv_im2col_3xtf32_kernel<BNC, kAct>),
                               T::kSmemBytes);
  if (rc) return rc;
  const int64_t tiles = static_cast<int64_t>(prm.m_blocks) * prm.n_blocks;
  const int grid = static_cast<int>(tiles < sm_count() ? tiles : sm_count());
  conv_im2col_3xtf32_kernel<BNC, kAct><<<grid, T::kThreads, T::kSmemBytes, s>>>(mh, ml, mw, prm);
  count_launch();
  return launch_result();
}

template <int BNC>
int dispatch_tma(cudaStream_t s, const CUtensorMap &mh, const CUtensorMap &ml,
                 const CUtensorMap &mw, const ConvParams &prm) {
  if (prm.act == 0) return launch_tma<BNC, kEpiActNone>(s, mh, ml, mw, prm);
  if (prm.act == 1) return launch_tma<BNC, kEpiActRelu>(s, mh, ml, mw, prm);
  return launch_tma<BNC, kEpiActAny>(s, mh, ml, mw, prm);
}

}  // namespace

bool conv_im2col_supported(const ConvParams &p, int n_img) {
  if (p.C % kConvBK != 0 || n_img <= 0 || n_img > 65535) return false;
  if (p.sw > 8 || p.sh > 8) return false;  // TMA traversal stride limit
  if ((p.KW - 1) * p.dw > 65535 || (p.KH - 1) * p.dh > 65535) return false;  // 16-bit offsets
  const Im2colCorners c = corners(p);
  if (!in_corner_range(c.lower_w) || !in_corner_range(c.lower_h) ||
      !in_corner_range(c.upper_w) || !in_corner_range(c.upper_h))
    return false;
  // Small planes stay on the direct-gather kernel.
  const int64_t plane_bytes = static_cast<int64_t>(n_img) * p.H * p.W * p.C * 4;
  return plane_bytes >= (int64_t(128) << 10);
}

int launch_conv_im2col(cudaStream_t s, int bnc, const float *wsplit, int64_t kp,
                       int64_t n_blocks, const float *x_hi, const float *x_lo,
                       const ConvParams &prm, int n_img) {
  if (!conv_im2col_supported(prm, n_img)) return kErrUnsupported;
  const Im2colCorners c = corners(prm);
  CUtensorMap mh, ml, mw;
  int rc = encode_tmap_im2col_nhwc_f32_sw128(&mh, x_hi, prm.C, prm.W, prm.H, n_img, c.lower_w,
                                             c.lower_h, c.upper_w, c.upper_h, prm.sw, prm.sh,
                                             kConvBK, kConvBM);
  if (rc) return rc;
  rc = encode_tmap_im2col_nhwc_f32_sw128(&ml, x_lo, prm.C, prm.W, prm.H, n_img, c.lower_w,
                                         c.lower_h, c.upper_w, c.upper_h, prm.sw, prm.sh, kConvBK,
                                         kConvBM);
  if (rc) return rc;
  rc = encode_tmap_2d_f32_sw128(&mw, wsplit, kp, n_blocks * 2 * bnc, kp * 4, kConvBK, 2 * bnc);
  if (rc) return rc;
  return bnc == 64 ? dispatch_tma<64>(s, mh, ml, mw, prm) : dispatch_tma<128>(s, mh, ml, mw, prm);
}

}  // namespace nplk
