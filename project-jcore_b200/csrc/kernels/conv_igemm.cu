// K2: NCHW 2-D convolution as an implicit GEMM on the sm_100a tensor cores
// (3xTF32), with bias, inference batch norm and activation in the epilogue.
//
// GEMM view: D[m][co] = sum_k A[m][k] * W'[co][k]
//   m  = (n, oh, ow)           output pixel, M = N*Ho*Wo
//   k  = (ci, kh, kw) in one of three orders, K = KH*KW*Cin:
//        Cin % 32 == 0: channel-block-major, k = ((cb*KH*KW) + tap)*32 + ci%32,
//                       so each 32-wide k-block is one tap over 32 channels;
//        filter rows of 3..8 columns (no column dilation): row order,
//                       k = (ci*KH + kh)*S + kw with S = 4 or 8 slots per
//                       filter row (slots past KW hold zero), so a thread
//                       reads S contiguous input columns per filter row;
//        otherwise:     tap-major, k = tap*Cin + ci
//   A[m][k] = x[n][ci][oh*sh - pt + kh*dh][ow*sw - pl + kw*dw]  (0 outside)
//   W'[co][k] = w[co][ci][kh][kw]
// Reference semantics: ExecuteConvDirect (advanced/neural_layer/src/
// npl_convolution.cpp:248-378) accumulates the same products in fp32; the
// epilogue then applies bias (:344-367), batch norm in the inference form of
// ExecuteBatchNormInference (npl_activation_norm.cpp:389-398) and the
// activation, i.e. what npl_conv2d_bn_activation is specified to compute
// (the reference itself stops after the conv, npl_convolution.cpp:116-126).
//
// No im2col matrix is materialised. Per persistent CTA:
//   producer warps, in groups of two (one group per shared-memory stage),
//               gather A: each thread owns two pixel rows and the 32
//               k-columns of a stage, loads them straight from NCHW global
//               memory (coalesced along ow), splits each value into tf32
//               hi/lo and writes both into 128-byte-swizzled shared memory;
//               the group's first thread also TMA-loads the matching
//               [W'_hi; W'_lo] slab;
//   MMA warp    issues tcgen05.mma: MMA(A_hi, [W_hi; W_lo]) with N = 2*BNC and
//               MMA(A_lo, W_hi) with N = BNC into a TMEM accumulator;
//   4 epilogue warps: out = act(BN(D[:, :BNC] + D[:, BNC:] + bias)), one
//               coalesced HBM write per output element.
// The weights are prepared by conv_prep_kernel (permute to the k order,
// split, zero-pad) together with the per-channel epilogue constants.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <type_traits>
#include <vector>

#include "conv_common.cuh"
#include "nplk_host.h"
#include "tuning_cache.h"

namespace nplk {

// Producer warps work in groups of two; group g fills shared-memory stage g
// for every work item (tile, k-block) whose index is g modulo the number of
// stages, so as many stages are being gathered concurrently as there are
// stages, each with 64 independent loads per thread in flight.
constexpr int kConvGroupWarps = 2;

template <int BNC>
struct ConvTraits {
  static constexpr int kStages = BNC == 64 ? 4 : 3;
  static constexpr int kProducerWarps = kStages * kConvGroupWarps;
  static constexpr int kMmaWarp = kProducerWarps;  // the 4 warps after it: epilogue
  static constexpr int kThreads = (kProducerWarps + 1 + 4) * 32;
  static constexpr int kAStageBytes = 2 * kConvBM * kConvBK * 4;  // hi + lo: 32 KB
  static constexpr int kBStageBytes = 2 * BNC * kConvBK * 4;
  static constexpr int kAccCols = 2 * BNC;
  static constexpr int kTmemCols = 2 * kAccCols;
  static constexpr int kSmemBytes =
      1024 + kStages * (kAStageBytes + kBStageBytes) + 256 + BNC * 20;  // + epilogue constants
};

// k orders of the direct kernel (4 and 8 are the row order's slot counts).
constexpr int kModeTaps = 0;
constexpr int kModeChannelBlocks = 1;

// Row-order slots per filter row for a geometry, 0 when the row order does not
// apply: channels not a multiple of 32 (channel blocks take those), filter
// rows of 3..8 columns, no column dilation.
inline int conv_row_slots(int64_t C, int64_t KW, int64_t dw) {
  if (C % kConvBK == 0 || dw != 1 || KW < 3 || KW > 8) return 0;
  return KW <= 4 ? 4 : 8;
}

// kMode (the k order, see conv_prep_kernel): kModeChannelBlocks -- C is a
// multiple of 32, so every 32-wide k-block is one filter tap across 32
// consecutive channels and the gather needs no per-element tap bookkeeping;
// 4 or 8 -- row order with that many slots per filter row; kModeTaps --
// tap-major, any geometry.
// Fuse: NoHmax (the conv output y) or HmaxOut (the fused max pool's
// horizontal maxima instead, conv_epilogue_tile_hmax).
template <int BNC, int kMode, int kAct, class Fuse>
__global__ void __launch_bounds__(ConvTraits<BNC>::kThreads, 1)
    conv_igemm_3xtf32_kernel(const __grid_constant__ CUtensorMap map_w, const ConvParams p,
                             const __grid_constant__ Fuse fz) {
  using T = ConvTraits<BNC>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align_smem_1024(smem_raw);
  uint8_t *smem_a = smem;
  uint8_t *smem_b = smem + T::kStages * T::kAStageBytes;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem_b + T::kStages * T::kBStageBytes);
  uint64_t *empty = full + T::kStages;
  uint64_t *acc_full = empty + T::kStages;
  uint64_t *acc_empty = acc_full + 2;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 2);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  float4 *ep_s = reinterpret_cast<float4 *>(smem_b + T::kStages * T::kBStageBytes + 256);
  float *ep_beta_s = reinterpret_cast<float *>(ep_s + BNC);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < T::kStages; ++s) {
      mbar_init(&full[s], kConvGroupWarps + 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&map_w);
  }
  if (warp == T::kMmaWarp) {
    tmem_alloc(tmem_slot, T::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  const int num_tiles = p.m_blocks * p.n_blocks;

  if (warp < T::kProducerWarps) {
    // ---------------- A gather + weight TMA (group = stage) ----------------
    const int group = warp / kConvGroupWarps;
    const int gt = threadIdx.x - group * kConvGroupWarps * 32;  // 0..63 within the group
    const int stage = group;
    uint32_t phase = 0;
    const int my_tiles = num_tiles > static_cast<int>(blockIdx.x)
                             ? (num_tiles - 1 - static_cast<int>(blockIdx.x)) / gridDim.x + 1
                             : 0;
    const int items = my_tiles * p.k_blocks;
    int cur_tile = -1;
    int ih0[2] = {0, 0}, iw0[2] = {0, 0};
    uint32_t cmask[2] = {0u, 0u};  // row order: filter columns inside the image
    bool valid[2] = {false, false};
    const float *xb[2] = {p.x, p.x};
    int nb = 0;
    bool issued = false;  // a weight copy was issued into this group's stage
    uint32_t issued_phase = 0;
    for (int it = group; it < items; it += T::kStages) {
      const int lt = it / p.k_blocks;
      const int kb = it - lt * p.k_blocks;
      const int tile = blockIdx.x + lt * gridDim.x;
      if (tile != cur_tile) {
        cur_tile = tile;
        const int mb = tile / p.n_blocks;
        nb = tile - mb * p.n_blocks;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          int n, oh, ow;
          valid[r] = conv_tile_pixel(p, mb, gt + 64 * r, n, oh, ow);
          ih0[r] = oh * p.sh - p.pt;
          iw0[r] = ow * p.sw - p.pl;
          xb[r] = p.x + static_cast<int64_t>(n) * p.CHW;
          if (kMode == 4 || kMode == 8) {
            cmask[r] = 0u;
            for (int kw = 0; kw < p.KW; ++kw)
              if (static_cast<unsigned>(iw0[r] + kw) < static_cast<unsigned>(p.W))
                cmask[r] |= 1u << kw;
          }
        }
      }
      // Gather 2 rows x 32 k into registers before waiting for the stage.
      float v[2][32];
      if (kMode == 4 || kMode == 8) {
        // Row order: the k-block holds 32 / S (channel, filter row) pairs of
        // S filter columns; each pair is S contiguous input columns.
        constexpr int S = kMode == 8 ? 8 : 4;
        constexpr int kPairs = kConvBK / S;
        const int q0 = kb * kPairs;
        int ci = q0 / p.KH;
        int kh = q0 - ci * p.KH;
#pragma unroll
        for (int i = 0; i < kPairs; ++i) {
#pragma unroll
          for (int r = 0; r < 2; ++r) {
            const int ih = ih0[r] + kh * p.dh;
            const uint32_t m = (ci < p.C && valid[r] &&
                                static_cast<unsigned>(ih) < static_cast<unsigned>(p.H))
                                   ? cmask[r]
                                   : 0u;
            const float *base = xb[r] + static_cast<int64_t>(ci) * p.HW +
                                static_cast<int64_t>(ih) * p.W + iw0[r];
#pragma unroll
            for (int kw = 0; kw < S; ++kw) v[r][i * S + kw] = ((m >> kw) & 1u) ? __ldg(base + kw) : 0.0f;
          }
          if (++kh == p.KH) {
            kh = 0;
            ++ci;
          }
        }
      } else if (kMode == kModeChannelBlocks) {
        const int taps = p.KH * p.KW;
        const int cb = kb / taps;
        const int tap = kb - cb * taps;
        const int kh = tap / p.KW;
        const int kw = tap - kh * p.KW;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int ih = ih0[r] + kh * p.dh, iw = iw0[r] + kw * p.dw;
          const bool ok = valid[r] && static_cast<unsigned>(ih) < static_cast<unsigned>(p.H) &&
                          static_cast<unsigned>(iw) < static_cast<unsigned>(p.W);
          const float *base =
              xb[r] + static_cast<int64_t>(cb * kConvBK) * p.HW + static_cast<int64_t>(ih) * p.W + iw;
          if (ok) {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[r][j] = __ldg(base + static_cast<int64_t>(j) * p.HW);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[r][j] = 0.0f;
          }
        }
      } else {
        int k = kb * kConvBK;
        int tap = k / p.C;
        int ci = k - tap * p.C;
        int kh = tap / p.KW;
        int kw = tap - kh * p.KW;
        bool ok[2];
        const float *ptr[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const int ih = ih0[r] + kh * p.dh, iw = iw0[r] + kw * p.dw;
          ok[r] = valid[r] && kh < p.KH &&
                  static_cast<unsigned>(ih) < static_cast<unsigned>(p.H) &&
                  static_cast<unsigned>(iw) < static_cast<unsigned>(p.W);
          ptr[r] = xb[r] + static_cast<int64_t>(ci) * p.HW + static_cast<int64_t>(ih) * p.W + iw;
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          v[0][j] = ok[0] ? __ldg(ptr[0]) : 0.0f;
          v[1][j] = ok[1] ? __ldg(ptr[1]) : 0.0f;
          ptr[0] += p.HW;
          ptr[1] += p.HW;
          if (++ci == p.C) {
            ci = 0;
            if (++kw == p.KW) {
              kw = 0;
              ++kh;
            }
#pragma unroll
            for (int r = 0; r < 2; ++r) {
              const int ih = ih0[r] + kh * p.dh, iw = iw0[r] + kw * p.dw;
              ok[r] = valid[r] && kh < p.KH &&
                      static_cast<unsigned>(ih) < static_cast<unsigned>(p.H) &&
                      static_cast<unsigned>(iw) < static_cast<unsigned>(p.W);
              ptr[r] = xb[r] + static_cast<int64_t>(ih) * p.W + iw;
            }
          }
        }
      }
      if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.status, kStatusTimeoutProducer))
        break;
      if (gt == 0) {
        mbar_arrive_expect_tx(&full[stage], T::kBStageBytes);
        tma_load_2d(&map_w, &full[stage], smem_b + stage * T::kBStageBytes, kb * kConvBK,
                    nb * 2 * BNC);
        issued = true;
        issued_phase = phase;
      }
      uint8_t *a_hi = smem_a + stage * T::kAStageBytes;
      uint8_t *a_lo = a_hi + kConvBM * 128;
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int row = gt + 64 * r;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          // The hi part is stored as the raw value: the tensor core reads a
          // tf32 operand as the truncation of its fp32 bits, which is
          // exactly tf32_split_trunc's hi.
          const float4 hi = make_float4(v[r][4 * c + 0], v[r][4 * c + 1], v[r][4 * c + 2],
                                        v[r][4 * c + 3]);
          float4 lo;
          float t;
          tf32_split_trunc(hi.x, t, lo.x);
          tf32_split_trunc(hi.y, t, lo.y);
          tf32_split_trunc(hi.z, t, lo.z);
          tf32_split_trunc(hi.w, t, lo.w);
          const uint32_t off = sw128_offset(row, c);
          *reinterpret_cast<float4 *>(a_hi + off) = hi;
          *reinterpret_cast<float4 *>(a_lo + off) = lo;
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[stage]);
      phase ^= 1u;
    }
    // Let the last weight copy land before the CTA can exit (it already has
    // unless the CTA aborted).
    if (gt == 0 && issued) mbar_drain(&full[stage], issued_phase);
  } else if (warp == T::kMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc_2n = umma_idesc_tf32(kConvBM, 2 * BNC);
      const uint32_t idesc_n = umma_idesc_tf32(kConvBM, BNC);
      const uint64_t a_desc0 = umma_desc_sw128(smem_u32(smem_a));
      const uint64_t b_desc0 = umma_desc_sw128(smem_u32(smem_b));
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, abort_flag, p.status,
                       kStatusTimeoutAccFree))
          break;
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * T::kAccCols;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.status, kStatusTimeoutMma))
            goto mma_done;
          tc_fence_after_sync();
          const uint64_t a_desc = a_desc0 + static_cast<uint64_t>(stage * (T::kAStageBytes >> 4));
          const uint64_t b_desc = b_desc0 + static_cast<uint64_t>(stage * (T::kBStageBytes >> 4));
          constexpr uint64_t kLoOff = (kConvBM * 128) >> 4;
#pragma unroll
          for (int kk = 0; kk < kConvBK / 8; ++kk) {
            mma_tf32_ss(d_tmem, a_desc + 2 * kk, b_desc + 2 * kk, idesc_2n,
                        (kb > 0 || kk > 0) ? 1u : 0u);
            mma_tf32_ss(d_tmem, a_desc + kLoOff + 2 * kk, b_desc + 2 * kk, idesc_n, 1u);
          }
          mma_commit(&empty[stage]);
          if (++stage == T::kStages) {
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
    const int et = threadIdx.x - (T::kMmaWarp + 1) * 32;  // 0..127
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      const int mb = tile / p.n_blocks;
      const int nb = tile - mb * p.n_blocks;
      bool ok;
      if constexpr (std::is_same<Fuse, HmaxOut>::value)
        ok = conv_epilogue_tile_hmax<BNC, kAct>(
            p, tmem_base + acc * T::kAccCols, quad, lane, et, mb, nb, ep_s, ep_beta_s,
            &acc_full[acc], acc_phase, abort_flag, fz,
            reinterpret_cast<float *>(ep_beta_s + BNC) + quad * 32 * kHmaxPitch);
      else
        ok = conv_epilogue_tile<BNC, kAct>(p, tmem_base + acc * T::kAccCols, quad, lane, et, mb,
                                           nb, ep_s, ep_beta_s, &acc_full[acc], acc_phase,
                                           abort_flag);
      if (!ok) break;
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
    }
  }

  __syncthreads();
  if (warp == T::kMmaWarp) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, T::kTmemCols);
  }
}

// Weight preparation: w[co][ci][kh][kw] -> the k order of the geometry
// (channel blocks, row order with row_slots > 0, else tap-major), tf32-split,
// blocked [n_blocks][2][BNC][kp] (zero padded), plus the epilogue constants.
__global__ void conv_prep_kernel(const float *__restrict__ w, int Cout, int C, int KH, int KW,
                                 int row_slots, int kp, int bnc, float *__restrict__ wsplit,
                                 int64_t wsplit_elems, const float *bias, const float *mean,
                                 const float *var, const float *gamma, const float *beta,
                                 float eps, float *__restrict__ ep, int cout_pad) {
  // The conv kernel that follows in nplk_conv2d_fused may be scheduled now
  // and start gathering x; its weight and constant readers wait
  // (griddep_wait) for this grid to complete and its writes to be visible.
  griddep_launch_dependents();
  const int64_t tid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int K = C * KH * KW;
  // One thread per (row, k) of the hi part; it also writes the lo part.
  const int64_t half_elems = wsplit_elems / 2;
  for (int64_t i = tid; i < half_elems; i += stride) {
    const int64_t rowg = i / kp;  // global padded output-channel row
    const int k = static_cast<int>(i - rowg * kp);
    const int co = static_cast<int>(rowg);
    float x = 0.0f;
    if (row_slots > 0) {
      // row order: k = (ci*KH + kh)*row_slots + kw, slots past KW zero
      const int q = k / row_slots;
      const int kw = k - q * row_slots;
      const int ci = q / KH;
      const int kh = q - ci * KH;
      if (co < Cout && ci < C && kw < KW)
        x = w[((static_cast<int64_t>(co) * C + ci) * KH + kh) * KW + kw];
    } else if (co < Cout && k < K) {
      int ci, tap;
      if (C % kConvBK == 0) {
        // channel-block-major: k = ((cb * KH*KW) + tap) * 32 + ci_in
        const int kb = k / kConvBK;
        const int cb = kb / (KH * KW);
        tap = kb - cb * (KH * KW);
        ci = cb * kConvBK + (k - kb * kConvBK);
      } else {
        // tap-major: k = tap * C + ci
        tap = k / C;
        ci = k - tap * C;
      }
      const int kh = tap / KW;
      const int kw = tap - kh * KW;
      x = w[((static_cast<int64_t>(co) * C + ci) * KH + kh) * KW + kw];
    }
    float hi, lo;
    tf32_split(x, hi, lo);
    const int blk = co / bnc;
    const int rr = co - blk * bnc;
    float *d = wsplit + ((static_cast<int64_t>(blk) * 2) * bnc + rr) * kp + k;
    d[0] = hi;
    d[static_cast<int64_t>(bnc) * kp] = lo;
  }
  for (int64_t c = tid; c < cout_pad; c += stride) {
    const bool in = c < Cout;
    ep[kEpBias * cout_pad + c] = (in && bias) ? bias[c] : 0.0f;
    ep[kEpMean * cout_pad + c] = (in && mean) ? mean[c] : 0.0f;
    ep[kEpGamma * cout_pad + c] = (in && gamma) ? gamma[c] : 1.0f;
    ep[kEpBeta * cout_pad + c] = (in && beta) ? beta[c] : 0.0f;
    ep[kEpInvStd * cout_pad + c] = (in && var) ? 1.0f / sqrtf(var[c] + eps) : 1.0f;
  }
}

namespace {

// Kernel that runs a geometry given the full workspace.
enum ConvPath {
  kPathDirect = 0,  // direct NCHW gather (conv_igemm_3xtf32_kernel)
  kPathIm2col = 1,  // NHWC hi/lo planes + im2col TMA per k-block (conv_im2col.cu)
  kPathWindow = 2,  // raw NHWC plane + im2col TMA windows shared by the KW taps (conv_window.cu)
  kPathWindowGather = 3,  // the same windows gathered from NCHW x by the kernel itself
  kPathWindowPair = 4,    // the gather windows on CTA pairs (conv_window_pair.cu)
};

// Workspace layout: [W' split: w_bytes][epilogue constants: ep_bytes], then
// the NHWC input planes: x_hi and x_lo (im2col path) or raw x (window path).
struct ConvPlan {
  int bnc;
  int mode;  // k order of the direct kernel: kModeTaps, kModeChannelBlocks, 4 or 8
  int64_t kp, n_blocks, cout_pad;
  size_t w_bytes, ep_bytes;
  int path;
  int planes;          // NHWC planes the path stages (0, 1 or 2)
  size_t plane_bytes;  // bytes of one plane
  size_t min_bytes() const { return w_bytes + ep_bytes; }
  size_t full_bytes() const { return w_bytes + ep_bytes + planes * plane_bytes; }
};

// Kernel parameters that depend on the geometry only.
ConvParams conv_params(const nplk_conv_geom_t *g, const ConvPlan &c) {
  ConvParams prm{};
  prm.C = static_cast<int>(g->c_in);
  prm.H = static_cast<int>(g->h);
  prm.W = static_cast<int>(g->w);
  prm.Cout = static_cast<int>(g->c_out);
  prm.KH = static_cast<int>(g->kh);
  prm.KW = static_cast<int>(g->kw);
  prm.sh = static_cast<int>(g->stride_h);
  prm.sw = static_cast<int>(g->stride_w);
  prm.pt = static_cast<int>(g->pad_top);
  prm.pl = static_cast<int>(g->pad_left);
  prm.dh = static_cast<int>(g->dil_h);
  prm.dw = static_cast<int>(g->dil_w);
  prm.Ho = static_cast<int>(g->h_out);
  prm.Wo = static_cast<int>(g->w_out);
  prm.HW = g->h * g->w;
  prm.HoWo = g->h_out * g->w_out;
  prm.CHW = g->c_in * g->h * g->w;
  prm.M = static_cast<int>(g->n * g->h_out * g->w_out);
  prm.Wv = prm.Wo;
  prm.Mv = prm.M;
  prm.K = static_cast<int>(g->c_in * g->kh * g->kw);
  prm.k_blocks = static_cast<int>(c.kp / kConvBK);
  prm.m_blocks = static_cast<int>(ceil_div(prm.M, kConvBM));
  prm.n_blocks = static_cast<int>(c.n_blocks);
  prm.cout_pad = static_cast<int>(c.cout_pad);
  return prm;
}

// Plan for algorithm `algo` (NPLK_CONV_ALGO_*); path -1 when the geometry
// does not suit it. AUTO picks the shared-window gather kernel for stride-1
// filters wider than one column, the per-k-block im2col kernel for the
// other TMA-eligible geometries and the direct kernel otherwise.
ConvPlan plan_conv(const nplk_conv_geom_t *g, int algo = NPLK_CONV_ALGO_AUTO,
                   bool use_cache = true) {
  ConvPlan c{};
  c.bnc = g->c_out <= 64 ? 64 : 128;
  const int slots = conv_row_slots(g->c_in, g->kw, g->dil_w);
  c.mode = g->c_in % kConvBK == 0 ? kModeChannelBlocks : slots > 0 ? slots : kModeTaps;
  const int64_t K = slots > 0 ? g->c_in * g->kh * slots : g->c_in * g->kh * g->kw;
  c.kp = ceil_div(K, kConvBK) * kConvBK;
  c.n_blocks = ceil_div(g->c_out, c.bnc);
  c.cout_pad = c.n_blocks * c.bnc;
  c.w_bytes = align_up(static_cast<size_t>(c.cout_pad) * 2 * c.kp * 4, 256);
  c.ep_bytes = align_up(static_cast<size_t>(kEpCount) * c.cout_pad * 4, 256);
  c.plane_bytes = align_up(static_cast<size_t>(g->n * g->h * g->w * g->c_in) * 4, 256);
  const ConvParams prm = conv_params(g, c);
  const int n = static_cast<int>(g->n);
  const bool window_ok = conv_window_supported(prm, n);
  const bool gather_ok = conv_window_gather_supported(prm, n);
  const bool im2col_ok = conv_im2col_supported(prm, n);
  const bool pair_ok = conv_window_pair_supported(prm, n, c.bnc, c.n_blocks);
  const bool shared_taps = g->stride_w == 1 && g->kw > 1;
  switch (algo) {
    case NPLK_CONV_ALGO_AUTO:
      c.path = (gather_ok && shared_taps)   ? kPathWindowGather
               : (window_ok && shared_taps) ? kPathWindow
               : im2col_ok                  ? kPathIm2col
                                            : kPathDirect;
      break;
    case NPLK_CONV_ALGO_DIRECT:
      c.path = kPathDirect;
      break;
    case NPLK_CONV_ALGO_IM2COL:
      c.path = im2col_ok ? kPathIm2col : -1;
      break;
    case NPLK_CONV_ALGO_WINDOW:
      c.path = window_ok ? kPathWindow : -1;
      break;
    case NPLK_CONV_ALGO_WINDOW_GATHER:
      c.path = gather_ok ? kPathWindowGather : -1;
      break;
    case NPLK_CONV_ALGO_WINDOW_PAIR:
      c.path = pair_ok ? kPathWindowPair : -1;
      break;
    default:
      c.path = -1;
  }
  c.planes = c.path == kPathIm2col ? 2 : c.path == kPathWindow ? 1 : 0;
  // AUTO takes the kernel the tile-configuration cache measured fastest for
  // this geometry on this device (nplk_conv2d_tune), when there is one.
  int cached = 0;
  if (algo == NPLK_CONV_ALGO_AUTO && use_cache && !tuning_cache_empty() &&
      tuning_lookup(tuning_key_conv(g), &cached) && cached != NPLK_CONV_ALGO_AUTO) {
    const ConvPlan t = plan_conv(g, cached, false);
    if (t.path >= 0) return t;
  }
  return c;
}

template <int BNC, int kMode, int kAct, class Fuse = NoHmax>
int launch_conv(cudaStream_t s, const ConvPlan &c, const float *wsplit, ConvParams prm,
                const Fuse &fz = Fuse{}) {
  using T = ConvTraits<BNC>;
  CUtensorMap map_w;
  int rc = encode_tmap_2d_f32_sw128(&map_w, wsplit, c.kp, c.n_blocks * 2 * BNC, c.kp * 4,
                                    kConvBK, 2 * BNC);
  if (rc) return rc;
  // The fused max pool's epilogue stages 32 x 32 blocks after the epilogue
  // constants.
  const int smem = T::kSmemBytes + (std::is_same<Fuse, HmaxOut>::value ? kHmaxStageBytes : 0);
  rc = ensure_dynamic_smem(
      reinterpret_cast<const void *>(conv_igemm_3xtf32_kernel<BNC, kMode, kAct, Fuse>), smem);
  if (rc) return rc;
  const int64_t tiles = static_cast<int64_t>(prm.m_blocks) * prm.n_blocks;
  const int grid = static_cast<int>(tiles < sm_count() ? tiles : sm_count());
  conv_igemm_3xtf32_kernel<BNC, kMode, kAct, Fuse><<<grid, T::kThreads, smem, s>>>(map_w, prm, fz);
  count_launch();
  return launch_result();
}

template <int BNC, int kMode>
int dispatch_act(cudaStream_t s, const ConvPlan &c, const float *wsplit, const ConvParams &prm) {
  if (prm.act == 0) return launch_conv<BNC, kMode, kEpiActNone>(s, c, wsplit, prm);
  if (prm.act == 1) return launch_conv<BNC, kMode, kEpiActRelu>(s, c, wsplit, prm);
  return launch_conv<BNC, kMode, kEpiActAny>(s, c, wsplit, prm);
}

template <int BNC>
int dispatch_mode(cudaStream_t s, const ConvPlan &c, const float *wsplit, const ConvParams &prm) {
  switch (c.mode) {
    case kModeChannelBlocks:
      return dispatch_act<BNC, kModeChannelBlocks>(s, c, wsplit, prm);
    case 4:
      return dispatch_act<BNC, 4>(s, c, wsplit, prm);
    case 8:
      return dispatch_act<BNC, 8>(s, c, wsplit, prm);
    default:
      return dispatch_act<BNC, kModeTaps>(s, c, wsplit, prm);
  }
}

int dispatch_conv(cudaStream_t s, const ConvPlan &c, const float *wsplit, ConvParams prm) {
  // Row order (C_in not a multiple of 32: the stem's 3 channels) with output
  // planes of whole 16 x 8 blocks: 2-D tiles. A 1-D tile spans ~1.1 output
  // rows and gathers 7-9 whole input rows per channel, whose vertical reuse
  // falls in other tiles; a 16 x 8 tile of a 7x7 stride-2 filter gathers a
  // 21 x 37 patch per channel (a third of the lines), reused inside the tile.
  if ((c.mode == 4 || c.mode == 8) && prm.Wo % 16 == 0 && prm.Ho % 8 == 0) {
    prm.t2d_w = 16;
    prm.t2d_cols = prm.Wo / 16;
    prm.t2d_tiles = (prm.Ho / 8) * prm.t2d_cols;
    prm.m_blocks = static_cast<int>(static_cast<int64_t>(prm.M) / kConvBM);
  }
  return c.bnc == 64 ? dispatch_mode<64>(s, c, wsplit, prm) : dispatch_mode<128>(s, c, wsplit, prm);
}

}  // namespace

int validate_conv_geom(const nplk_conv_geom_t *g) {
  if (!g) return kErrInvalidArg;
  if (g->n <= 0 || g->c_in <= 0 || g->h <= 0 || g->w <= 0 || g->c_out <= 0 || g->kh <= 0 ||
      g->kw <= 0 || g->stride_h <= 0 || g->stride_w <= 0 || g->dil_h <= 0 || g->dil_w <= 0 ||
      g->h_out <= 0 || g->w_out <= 0 || g->pad_top < 0 || g->pad_left < 0)
    return kErrInvalidArg;
  // 32-bit index arithmetic inside the kernels.
  const int64_t lim = int64_t(1) << 31;
  if (g->n * g->h_out * g->w_out >= lim || g->n * g->c_in * g->h * g->w >= (int64_t(1) << 40) ||
      g->c_in * g->kh * g->kw >= lim / 64 || g->h >= lim || g->w >= lim ||
      g->h_out * g->w_out >= lim)
    return kErrUnsupported;
  return kOk;
}

}  // namespace nplk

using namespace nplk;

extern "C" size_t nplk_conv_workspace_size(const nplk_conv_geom_t *g) {
  if (validate_conv_geom(g) != kOk) return 0;
  return plan_conv(g).full_bytes();
}

extern "C" size_t nplk_conv_workspace_size_algo(const nplk_conv_geom_t *g, int algo) {
  if (validate_conv_geom(g) != kOk) return 0;
  const ConvPlan c = plan_conv(g, algo);
  return c.path < 0 ? 0 : c.full_bytes();
}

extern "C" size_t nplk_conv_workspace_min_size(const nplk_conv_geom_t *g) {
  if (validate_conv_geom(g) != kOk) return 0;
  return plan_conv(g).min_bytes();
}

namespace {

// Checks geometry and workspace shared by prepare and run.
int check_conv_call(const nplk_conv_geom_t *g, void *workspace, size_t workspace_bytes,
                    ConvPlan *c) {
  int rc = validate_conv_geom(g);
  if (rc) return rc;
  *c = plan_conv(g);
  if (!workspace || workspace_bytes < c->min_bytes() ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return kErrInvalidArg;
  return kOk;
}

}  // namespace

extern "C" int nplk_conv2d_prepare(void *stream, const nplk_conv_geom_t *g, const float *w,
                                   const float *bias, const float *bn_mean,
                                   const float *bn_var, const float *bn_gamma,
                                   const float *bn_beta, float bn_eps, void *workspace,
                                   size_t workspace_bytes) {
  ConvPlan c;
  int rc = check_conv_call(g, workspace, workspace_bytes, &c);
  if (rc) return rc;
  if (!w) return kErrInvalidArg;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float *wsplit = static_cast<float *>(workspace);
  float *ep = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + c.w_bytes);
  const int64_t wsplit_elems = c.cout_pad * 2 * c.kp;
  const int threads = 256;
  int64_t blocks = ceil_div(wsplit_elems / 2, threads);
  if (blocks > 4096) blocks = 4096;
  conv_prep_kernel<<<static_cast<unsigned>(blocks), threads, 0, s>>>(
      w, static_cast<int>(g->c_out), static_cast<int>(g->c_in), static_cast<int>(g->kh),
      static_cast<int>(g->kw), c.mode == 4 || c.mode == 8 ? c.mode : 0, static_cast<int>(c.kp),
      c.bnc, wsplit, wsplit_elems, bias,
      bn_mean, bn_var, bn_gamma, bn_beta, bn_eps, ep, static_cast<int>(c.cout_pad));
  count_launch();
  return launch_result();
}

namespace {

// Everything run needs besides x: validated plan, status word and the
// geometry-dependent kernel parameters.
int begin_run(const nplk_conv_geom_t *g, void *workspace, size_t workspace_bytes, int act,
              float act_alpha, float *out, int *status, ConvPlan *c, ConvParams *prm) {
  int rc = check_conv_call(g, workspace, workspace_bytes, c);
  if (rc) return rc;
  if (!out) return kErrInvalidArg;
  if (!status) status = device_status_word();
  if (!status) return kErrInternal;
  *prm = conv_params(g, *c);
  prm->y = out;
  prm->ep = reinterpret_cast<const float *>(static_cast<const uint8_t *>(workspace) + c->w_bytes);
  prm->act = act;
  prm->act_alpha = act_alpha;
  prm->status = status;
  return kOk;
}

float *plane_hi(void *workspace, const ConvPlan &c) {
  return reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + c.min_bytes());
}

float *plane_lo(void *workspace, const ConvPlan &c) {
  return reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + c.min_bytes() +
                                   c.plane_bytes);
}

bool has_planes(const ConvPlan &c, size_t workspace_bytes) {
  return c.planes > 0 && workspace_bytes >= c.full_bytes();
}

}  // namespace

namespace {

// Runs plan `c` (workspace already checked against c.full_bytes()).
// after_prep: the previous kernel in the stream is this call's
// conv_prep_kernel (nplk_conv2d_fused), which the gather kernel may overlap.
int run_plan(cudaStream_t s, const nplk_conv_geom_t *g, const float *x, const ConvPlan &c,
             ConvParams prm, void *workspace, bool stage, bool after_prep = false) {
  const float *wsplit = static_cast<const float *>(workspace);
  const int n = static_cast<int>(g->n);
  switch (c.path) {
    case kPathWindowGather:
      prm.x = x;
      return launch_conv_window(s, c.bnc, wsplit, c.kp, c.n_blocks, nullptr, prm, n, after_prep);
    case kPathWindowPair:
      prm.x = x;
      return launch_conv_window_pair(s, wsplit, c.kp, prm, n, after_prep);
    case kPathWindow:
    case kPathIm2col: {
      if (stage) {
        int rc = launch_nchw_to_nhwc_split(s, x, plane_hi(workspace, c),
                                           c.planes == 2 ? plane_lo(workspace, c) : nullptr, n,
                                           static_cast<int>(g->c_in), g->h * g->w);
        if (rc) return rc;
      }
      if (c.path == kPathWindow)
        return launch_conv_window(s, c.bnc, wsplit, c.kp, c.n_blocks, plane_hi(workspace, c), prm,
                                  n);
      return launch_conv_im2col(s, c.bnc, wsplit, c.kp, c.n_blocks, plane_hi(workspace, c),
                                plane_lo(workspace, c), prm, n);
    }
    case kPathDirect:
      prm.x = x;
      return dispatch_conv(s, c, wsplit, prm);
    default:
      return kErrUnsupported;
  }
}

}  // namespace

extern "C" int nplk_conv2d_stage_input(void *stream, const nplk_conv_geom_t *g, const float *x,
                                       void *workspace, size_t workspace_bytes) {
  ConvPlan c;
  int rc = check_conv_call(g, workspace, workspace_bytes, &c);
  if (rc) return rc;
  if (!x) return kErrInvalidArg;
  if (!has_planes(c, workspace_bytes)) return kErrUnsupported;
  return launch_nchw_to_nhwc_split(static_cast<cudaStream_t>(stream), x, plane_hi(workspace, c),
                                   c.planes == 2 ? plane_lo(workspace, c) : nullptr,
                                   static_cast<int>(g->n), static_cast<int>(g->c_in), g->h * g->w);
}

extern "C" int nplk_conv2d_run_staged(void *stream, const nplk_conv_geom_t *g, int act,
                                      float act_alpha, float *out, void *workspace,
                                      size_t workspace_bytes, int *status) {
  ConvPlan c;
  ConvParams prm;
  int rc = begin_run(g, workspace, workspace_bytes, act, act_alpha, out, status, &c, &prm);
  if (rc) return rc;
  if (!has_planes(c, workspace_bytes)) return kErrUnsupported;
  return run_plan(static_cast<cudaStream_t>(stream), g, nullptr, c, prm, workspace, false);
}

namespace {

int run_auto(void *stream, const nplk_conv_geom_t *g, const float *x, int act, float act_alpha,
             float *out, void *workspace, size_t workspace_bytes, int *status, bool after_prep) {
  ConvPlan c;
  ConvParams prm;
  int rc = begin_run(g, workspace, workspace_bytes, act, act_alpha, out, status, &c, &prm);
  if (rc) return rc;
  if (!x) return kErrInvalidArg;
  // A workspace too small for the planes of the chosen kernel selects the
  // kernel AUTO picks without the tile-configuration cache if that fits, else
  // the direct kernel (same results either way).
  if (workspace_bytes < c.full_bytes()) {
    const ConvPlan h = plan_conv(g, NPLK_CONV_ALGO_AUTO, false);
    if (workspace_bytes >= h.full_bytes())
      c = h;
    else
      c.path = kPathDirect;
  }
  return run_plan(static_cast<cudaStream_t>(stream), g, x, c, prm, workspace, true, after_prep);
}

}  // namespace

extern "C" int nplk_conv2d_run(void *stream, const nplk_conv_geom_t *g, const float *x,
                               int act, float act_alpha, float *out, void *workspace,
                               size_t workspace_bytes, int *status) {
  return run_auto(stream, g, x, act, act_alpha, out, workspace, workspace_bytes, status, false);
}

extern "C" int nplk_conv2d_run_algo(void *stream, const nplk_conv_geom_t *g, const float *x,
                                    int act, float act_alpha, float *out, void *workspace,
                                    size_t workspace_bytes, int *status, int algo) {
  ConvPlan c;
  ConvParams prm;
  int rc = begin_run(g, workspace, workspace_bytes, act, act_alpha, out, status, &c, &prm);
  if (rc) return rc;
  if (!x) return kErrInvalidArg;
  c = plan_conv(g, algo);
  if (c.path < 0) return kErrUnsupported;
  if (workspace_bytes < c.full_bytes()) return kErrInvalidArg;
  return run_plan(static_cast<cudaStream_t>(stream), g, x, c, prm, workspace, true);
}

extern "C" int nplk_conv2d_fused(void *stream, const nplk_conv_geom_t *g, const float *x,
                                 const float *w, const float *bias, const float *bn_mean,
                                 const float *bn_var, const float *bn_gamma,
                                 const float *bn_beta, float bn_eps, int act, float act_alpha,
                                 float *out, void *workspace, size_t workspace_bytes,
                                 int *status) {
  if (!x || !w || !out) return kErrInvalidArg;
  int rc = nplk_conv2d_prepare(stream, g, w, bias, bn_mean, bn_var, bn_gamma, bn_beta, bn_eps,
                               workspace, workspace_bytes);
  if (rc) return rc;
  return run_auto(stream, g, x, act, act_alpha, out, workspace, workspace_bytes, status, true);
}

extern "C" int nplk_conv2d_tune(void *stream, const nplk_conv_geom_t *g, const float *x,
                                const float *w, const float *bias, const float *bn_mean,
                                const float *bn_var, const float *bn_gamma,
                                const float *bn_beta, float bn_eps, int act, float act_alpha,
                                float *out, void *workspace, size_t workspace_bytes, int reps,
                                int *best_algo, float *best_us) {
  if (!x || !w || !out || !best_algo || reps < 1 || reps > 1000) return kErrInvalidArg;
  int rc = nplk_conv2d_prepare(stream, g, w, bias, bn_mean, bn_var, bn_gamma, bn_beta, bn_eps,
                               workspace, workspace_bytes);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  if (cudaEventCreate(&e0) != cudaSuccess || cudaEventCreate(&e1) != cudaSuccess) {
    if (e0) cudaEventDestroy(e0);
    return kErrInternal;
  }
  int best = 0;
  float best_ms = 0.0f;
  for (int algo : {NPLK_CONV_ALGO_DIRECT, NPLK_CONV_ALGO_IM2COL, NPLK_CONV_ALGO_WINDOW,
                   NPLK_CONV_ALGO_WINDOW_GATHER, NPLK_CONV_ALGO_WINDOW_PAIR}) {
    const ConvPlan c = plan_conv(g, algo, false);
    if (c.path < 0 || workspace_bytes < c.full_bytes()) continue;  // not a candidate here
    std::vector<float> ms;
    for (int r = 0; r <= reps && rc == kOk; ++r) {
      if (cudaEventRecord(e0, s) != cudaSuccess) rc = kErrInternal;
      if (rc == kOk)
        rc = nplk_conv2d_run_algo(stream, g, x, act, act_alpha, out, workspace, workspace_bytes,
                                  nullptr, algo);
      if (rc == kOk && (cudaEventRecord(e1, s) != cudaSuccess ||
                        cudaEventSynchronize(e1) != cudaSuccess))
        rc = kErrInternal;
      float t = 0.0f;
      if (rc == kOk && r > 0) {  // the first run is the warm-up
        cudaEventElapsedTime(&t, e0, e1);
        ms.push_back(t);
      }
    }
    if (rc != kOk) break;
    std::nth_element(ms.begin(), ms.begin() + ms.size() / 2, ms.end());
    const float med = ms[ms.size() / 2];
    if (best == 0 || med < best_ms) {
      best = algo;
      best_ms = med;
    }
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (rc != kOk) return rc;
  if (best == 0) return kErrUnsupported;
  if (nplk_read_status(stream) != 0) return kErrInternal;
  // The last candidate run left its output in `out`; every kernel writes
  // the same bits, so it is the conv's result.
  tuning_insert(tuning_key_conv(g), best, best_ms * 1000.0);
  *best_algo = best;
  if (best_us) *best_us = best_ms * 1000.0f;
  return kOk;
}

// ---------------------------------------------------------------------------
// conv -> 3x3/s2/p1 max pool, fused through the horizontal-max epilogue
// (conv_epilogue_tile_hmax) and a vertical pass. Replaces the reference's
// stem sequence of npl_conv2d_bn_activation (npl_convolution.cpp:92-137) and
// npl_pooling max 3x3/s2/p1 (npl_pooling.cpp:129-219) for geometries the
// direct kernel's row order serves (C_in not a multiple of 32, filter rows of
// 3..8 columns), C_out <= 64 and an even output width.
// ---------------------------------------------------------------------------
namespace nplk {
namespace {

// out[n][c][ph][pw] = max over rows {2ph-1, 2ph, 2ph+1} of h[n][c][row][pw]
// in the reference's scan order; where h lacks its left neighbour (the
// centre is the first pixel of a 32-pixel group) the previous group's last
// pixel e[group-1][c] is folded in first. Grid: y over (n, c) planes, x over the
// plane's outputs, kV consecutive columns per thread (float4 when wp % 4 == 0).
template <int kV>
__global__ void pool_vmax_kernel(const float *__restrict__ h, const float *__restrict__ e,
                                 float *__restrict__ out, int64_t planes, int C, int Ho, int Wo,
                                 int wp, int po) {
  const float ninf = -__int_as_float(0x7f800000);
  const int wq = wp / kV;
  const int items = po * wq;
  for (int64_t pl = blockIdx.y; pl < planes; pl += gridDim.y) {
    const int c = static_cast<int>(static_cast<uint32_t>(pl) % static_cast<uint32_t>(C));
    const int64_t n = static_cast<int64_t>(static_cast<uint32_t>(pl) / static_cast<uint32_t>(C));
    const float *hp = h + pl * Ho * wp;
    float *op = out + pl * po * wp;
    for (int it = blockIdx.x * blockDim.x + threadIdx.x; it < items; it += gridDim.x * blockDim.x) {
      const int ph = it / wq;
      const int pw0 = (it - ph * wq) * kV;
      float mx[kV];
#pragma unroll
      for (int k = 0; k < kV; ++k) mx[k] = ninf;
#pragma unroll
      for (int dr = -1; dr <= 1; ++dr) {
        const int row = 2 * ph + dr;
        if (row < 0 || row >= Ho) continue;
        float v[kV];
        if constexpr (kV == 4) {
          const float4 t = *reinterpret_cast<const float4 *>(hp + row * wp + pw0);
          v[0] = t.x;
          v[1] = t.y;
          v[2] = t.z;
          v[3] = t.w;
        } else {
          v[0] = hp[row * wp + pw0];
        }
        const int64_t base = (n * Ho + row) * Wo;  // GEMM row of the row's first pixel
#pragma unroll
        for (int k = 0; k < kV; ++k) {
          const int pw = pw0 + k;
          const int64_t pix = base + 2 * pw;  // GEMM row of the centre
          if (pw > 0 && (pix & (kHmaxGroup - 1)) == 0)
            v[k] = pool_max_step(pool_max_step(ninf, e[(pix / kHmaxGroup - 1) * C + c]), v[k]);
          mx[k] = pool_max_step(mx[k], v[k]);
        }
      }
      if constexpr (kV == 4)
        *reinterpret_cast<float4 *>(op + ph * wp + pw0) = make_float4(mx[0], mx[1], mx[2], mx[3]);
      else
        op[ph * wp + pw0] = mx[0];
    }
  }
}

struct PoolFusePlan {
  ConvPlan c;
  int64_t wp, po, m_blocks;
  size_t h_bytes, e_bytes;
  bool ok;
};

PoolFusePlan plan_pool_fuse(const nplk_conv_geom_t *g) {
  PoolFusePlan f{};
  if (validate_conv_geom(g) != kOk) return f;
  f.c = plan_conv(g, NPLK_CONV_ALGO_DIRECT, false);
  f.ok = f.c.bnc == 64 && f.c.n_blocks == 1 && (f.c.mode == 4 || f.c.mode == 8) &&
         g->w_out % 2 == 0 && g->w_out >= 32 && g->h_out >= 1;  // a warp's 32 pixels span <= 2 rows
  f.wp = g->w_out / 2;                // floor((Wo + 2 - 3) / 2) + 1 for even Wo
  f.po = (g->h_out - 1) / 2 + 1;     // floor((Ho + 2 - 3) / 2) + 1
  f.m_blocks = ceil_div(g->n * g->h_out * g->w_out, kConvBM);
  f.h_bytes = align_up(static_cast<size_t>(g->n * g->c_out * g->h_out * f.wp) * 4, 256);
  const int64_t groups = ceil_div(g->n * g->h_out * g->w_out, kHmaxGroup);
  f.e_bytes = align_up(static_cast<size_t>(groups * g->c_out) * 4, 256);
  return f;
}

template <int kMode>
int launch_hmax(cudaStream_t s, const ConvPlan &c, const float *wsplit, const ConvParams &prm,
                const HmaxOut &fz) {
  if (prm.act == 1) return launch_conv<64, kMode, kEpiActRelu>(s, c, wsplit, prm, fz);
  return launch_conv<64, kMode, kEpiActAny>(s, c, wsplit, prm, fz);
}

}  // namespace
}  // namespace nplk

extern "C" size_t nplk_conv2d_maxpool_workspace_size(const nplk_conv_geom_t *g) {
  const PoolFusePlan f = plan_pool_fuse(g);
  if (!f.ok) return 0;
  return f.c.min_bytes() + f.h_bytes + f.e_bytes;
}

extern "C" int nplk_conv2d_maxpool_fused(void *stream, const nplk_conv_geom_t *g,
                                         const float *x, const float *w, const float *bias,
                                         const float *bn_mean, const float *bn_var,
                                         const float *bn_gamma, const float *bn_beta,
                                         float bn_eps, int act, float act_alpha, float *out,
                                         void *workspace, size_t workspace_bytes, int *status) {
  if (!g || !x || !w || !out) return kErrInvalidArg;
  const PoolFusePlan f = plan_pool_fuse(g);
  if (!f.ok) return kErrUnsupported;
  const size_t need = f.c.min_bytes() + f.h_bytes + f.e_bytes;
  if (!workspace || workspace_bytes < need ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return kErrInvalidArg;
  int rc = nplk_conv2d_prepare(stream, g, w, bias, bn_mean, bn_var, bn_gamma, bn_beta, bn_eps,
                               workspace, workspace_bytes);
  if (rc) return rc;
  if (!status) status = device_status_word();
  if (!status) return kErrInternal;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  ConvParams prm = conv_params(g, f.c);
  prm.x = x;
  prm.y = nullptr;  // the epilogue writes the horizontal maxima instead
  prm.ep = reinterpret_cast<const float *>(static_cast<const uint8_t *>(workspace) + f.c.w_bytes);
  prm.act = act;
  prm.act_alpha = act_alpha;
  prm.status = status;
  uint8_t *base = static_cast<uint8_t *>(workspace) + f.c.min_bytes();
  HmaxOut fz;
  fz.h = reinterpret_cast<float *>(base);
  fz.e = reinterpret_cast<float *>(base + f.h_bytes);
  fz.wp = static_cast<int>(f.wp);
  const float *wsplit = static_cast<const float *>(workspace);
  rc = f.c.mode == 8 ? launch_hmax<8>(s, f.c, wsplit, prm, fz)
                     : launch_hmax<4>(s, f.c, wsplit, prm, fz);
  if (rc) return rc;
  // < 2^32: n * h_out * w_out < 2^31 (validate_conv_geom) with w_out >= 32 and c_out <= 64
  const int64_t planes = g->n * g->c_out;
  const bool vec = f.wp % 4 == 0 && (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
  const int threads = 128;
  const int64_t items = f.po * (vec ? f.wp / 4 : f.wp);
  const dim3 grid(static_cast<unsigned>(ceil_div(items, threads)),
                  static_cast<unsigned>(planes < 65535 ? planes : 65535));
  const int C = static_cast<int>(g->c_out), Ho = static_cast<int>(g->h_out),
            Wo = static_cast<int>(g->w_out), po = static_cast<int>(f.po);
  if (vec)
    pool_vmax_kernel<4><<<grid, threads, 0, s>>>(fz.h, fz.e, out, planes, C, Ho, Wo, fz.wp, po);
  else
    pool_vmax_kernel<1><<<grid, threads, 0, s>>>(fz.h, fz.e, out, planes, C, Ho, Wo, fz.wp, po);
  count_launch();
  return launch_result();
}

