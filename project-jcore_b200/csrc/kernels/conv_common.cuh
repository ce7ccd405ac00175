// Pieces shared by the fused conv kernels (direct NCHW gather in
// conv_igemm.cu, TMA im2col over NHWC split planes in conv_im2col.cu, shared
// TMA windows over a raw NHWC plane in conv_window.cu): the
// GEMM tile shape, kernel parameters, per-channel epilogue constants and the
// accumulator-drain epilogue.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "nplk_device.cuh"
#include "ptx_sm100.cuh"

namespace nplk {

constexpr int kConvBM = 128;  // output pixels per tile (TMEM lanes)
constexpr int kConvBK = 32;   // k per stage (one 128-byte swizzle row of fp32)

// Per-channel epilogue constants, [5][cout_pad]: bias, mean, gamma, beta,
// 1/sqrt(var+eps).
enum { kEpBias = 0, kEpMean = 1, kEpGamma = 2, kEpBeta = 3, kEpInvStd = 4, kEpCount = 5 };

struct ConvParams {
  const float *x;
  float *y;
  int C, H, W, Cout, KH, KW, sh, sw, pt, pl, dh, dw, Ho, Wo;
  int64_t HW, HoWo, CHW;
  int M;
  // GEMM rows: "virtual" output pixels (n, oh, ow') with ow' < Wv, Mv of them.
  // Wv = Wo except for the window kernel, whose traversal also visits the
  // (KW-1)*dw columns right of each output row (computed, never stored).
  int Wv, Mv;
  int K, k_blocks, m_blocks, n_blocks;
  const float *ep;
  int cout_pad;
  int act;
  float act_alpha;
  uint32_t stall_us;  // fault injection: 0 except on an armed launch (injected_stall)
  int *status;
  // 2-D tiles (direct kernel, row order): t2d_w > 0 makes each GEMM tile
  // t2d_w output columns x (128 / t2d_w) output rows of one image (t2d_cols
  // tiles across an output row, t2d_tiles per image) instead of 128
  // consecutive pixels, so one tile's input rows stay few and L1-resident.
  int t2d_w, t2d_cols, t2d_tiles;
};

// GEMM row r (0..127) of tile mb as an output pixel (n, oh, ow): 1-D tiles
// take 128 consecutive pixels in (n, oh, ow) order (GEMM rows are real
// pixels: Wv == Wo), 2-D tiles their block of one image. False past the last
// pixel (n, oh, ow are then 0).
__device__ __forceinline__ bool conv_tile_pixel(const ConvParams &p, int mb, int r, int &n,
                                                int &oh, int &ow) {
  if (p.t2d_w == 0) {
    const int m = mb * kConvBM + r;
    n = oh = ow = 0;
    if (m >= p.M) return false;
    n = m / static_cast<int>(p.HoWo);
    const int pix = m - n * static_cast<int>(p.HoWo);
    oh = pix / p.Wo;
    ow = pix - oh * p.Wo;
    return true;
  }
  n = mb / p.t2d_tiles;
  const int t = mb - n * p.t2d_tiles;
  const int tr = t / p.t2d_cols;
  const int tc = t - tr * p.t2d_cols;
  const int dy = r / p.t2d_w;
  oh = tr * (kConvBM / p.t2d_w) + dy;
  ow = tc * p.t2d_w + (r - dy * p.t2d_w);
  return true;
}

// Epilogue activation selected at compile time for the common cases.
enum { kEpiActNone = 0, kEpiActRelu = 1, kEpiActAny = 2 };

template <int kAct>
__device__ __forceinline__ float epilogue_act(float t, int act, float alpha) {
  if (kAct == kEpiActNone) return t;
  if (kAct == kEpiActRelu) return t < 0.0f ? 0.0f : t;  // std::max(t, 0)
  return apply_act(t, act, alpha);
}

__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// One lane's 32 outputs of an accumulator chunk: channel j of the chunk goes
// to y[j * plane]. The constants come from shared memory through pointers the
// compiler knows to be shared (align_smem_1024), and the restrict qualifiers
// tell it that the stores to y do not touch them, so it may load later
// channels' constants before storing earlier outputs.
template <int kAct, bool kFull>
__device__ __forceinline__ void conv_store_chunk(float *__restrict__ y, int64_t plane,
                                                 const float4 *__restrict__ q,
                                                 const float *__restrict__ beta,
                                                 const uint32_t (&v)[32], const uint32_t (&w)[32],
                                                 int nco, int act, float act_alpha) {
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (!kFull && j >= nco) continue;
    const float4 c = q[j];
    float t = (__uint_as_float(v[j]) + __uint_as_float(w[j])) + c.x;
    // Without BN the constants are mean 0, gamma 1, inv_std 1, beta 0.
    t = c.z * (t - c.y) * c.w + beta[j];
    y[j * plane] = epilogue_act<kAct>(t, act, act_alpha);
  }
}

// Drains one finished accumulator tile (GEMM rows mb*128.., channels
// nb*BNC..) to NCHW, skipping rows that are not output pixels:
// out = act(gamma*((D[:, :BNC] + D[:, BNC:] + bias) - mean)*inv_std + beta).
// Called by the 4 epilogue warps (warp quad = TMEM lane quadrant, et = 0..127
// across them); `acc_tmem` is the accumulator's first column. The tile's
// constants are staged in shared memory (every lane reads the same channel,
// so each read is a broadcast). Returns false when the CTA aborted.
// kPair: the accumulator belongs to a CTA pair (conv_window_pair.cu); the
// wait acquires at cluster scope and a timeout also raises the peer's abort
// flag (`peer_abort`, its shared::cluster address).
// `bar_id` names the 128-thread barrier of the draining warpgroup (a kernel
// with several draining warpgroups gives each its own id and constants area).
template <int BNC, int kAct, bool kPair = false>
__device__ __forceinline__ bool conv_epilogue_tile(const ConvParams &p, uint32_t acc_tmem,
                                                   int quad, int lane, int et, int mb, int nb,
                                                   float4 *ep_s, float *ep_beta_s,
                                                   uint64_t *acc_full, uint32_t acc_phase,
                                                   volatile int *abort_flag,
                                                   uint32_t peer_abort = 0u, int bar_id = 1) {
  // The tile's constants are staged before the accumulator wait, so their
  // loads overlap the MMAs still accumulating the tile (for a CTA's last tile
  // they would otherwise follow its last MMA). All four warps pass the first
  // barrier before anyone rewrites the constants of the previous tile.
  named_barrier_sync(bar_id, 128);
  for (int i = et; i < BNC; i += 128) {
    const int co = nb * BNC + i;
    ep_s[i] = make_float4(p.ep[kEpBias * p.cout_pad + co], p.ep[kEpMean * p.cout_pad + co],
                          p.ep[kEpGamma * p.cout_pad + co], p.ep[kEpInvStd * p.cout_pad + co]);
    ep_beta_s[i] = p.ep[kEpBeta * p.cout_pad + co];
  }
  if constexpr (kPair)
    mbar_wait_pair(acc_full, acc_phase, abort_flag, peer_abort, p.status, kStatusTimeoutEpilogue);
  else
    mbar_wait(acc_full, acc_phase, abort_flag, p.status, kStatusTimeoutEpilogue);
  // The four warps leave together if the CTA aborted, and the constants are
  // visible to all of them past this barrier.
  named_barrier_sync(bar_id, 128);
  if (*abort_flag) return false;
  tc_fence_after_sync();
  const int m = mb * kConvBM + quad * 32 + lane;  // GEMM row (virtual pixel)
  bool valid = m < p.Mv;
  int n = 0, pix = 0;
  if (p.t2d_w) {
    int oh, ow;
    valid = conv_tile_pixel(p, mb, quad * 32 + lane, n, oh, ow);
    pix = oh * p.Wo + ow;
  } else if (valid) {
    const int howv = p.Ho * p.Wv;
    n = m / howv;
    const int rem = m - n * howv;
    const int oh = rem / p.Wv;
    const int ow = rem - oh * p.Wv;
    valid = ow < p.Wo;
    pix = oh * p.Wo + ow;
  }
  float *yb = p.y + static_cast<int64_t>(n) * p.Cout * p.HoWo + pix;
  const uint32_t t_row = acc_tmem + (static_cast<uint32_t>(quad * 32) << 16);
#pragma unroll 1
  for (int c0 = 0; c0 < BNC; c0 += 32) {
    uint32_t v[32], w[32];
    tmem_ld32(t_row + c0, v);
    tmem_ld32(t_row + BNC + c0, w);
    tmem_wait_ld2(v, w);
    const int co0 = nb * BNC + c0;
    if (valid) {
      float *yc = yb + static_cast<int64_t>(co0) * p.HoWo;
      if (co0 + 32 <= p.Cout)
        conv_store_chunk<kAct, true>(yc, p.HoWo, ep_s + c0, ep_beta_s + c0, v, w, 32, p.act,
                                     p.act_alpha);
      else
        conv_store_chunk<kAct, false>(yc, p.HoWo, ep_s + c0, ep_beta_s + c0, v, w,
                                      p.Cout - co0, p.act, p.act_alpha);
    }
  }
  return true;
}

// Conv -> 3x3/s2/p1 max pool fusion (nplk_conv2d_maxpool_fused): instead of
// the conv output y, the epilogue writes the horizontal maxima
//   h[n][co][oh][pw] = max over ow in {2pw-1, 2pw, 2pw+1} of y[n][co][oh][ow]
// (half of y's bytes), and a vertical pass takes the maximum over rows
// {2ph-1, 2ph, 2ph+1}. Both passes scan in the reference's order with
// "replace when greater" from -inf (ExecuteMaxPooling, npl_pooling.cpp:
// 129-219), so NaNs are skipped and the first of equal values (+0 / -0) is
// kept, exactly as the 3x3 scan does. Requires an even Wo (pairs of columns
// never straddle a 32-pixel group) and GEMM rows = output pixels
// (n, oh, ow). Each warp holds 32 consecutive pixels; the left neighbour
// (2pw-1) of a group's first pixel belongs to the previous group, so that h
// is written without it and every group's last pixel is saved in
// e[group][co] for the vertical pass to fold in (no exchange between warps).
constexpr int kHmaxGroup = 32;  // pixels per warp
struct HmaxOut {
  float *h;  // [N][Cout][Ho][wp]
  float *e;  // [ceil(M / 32)][Cout]: each 32-pixel group's last pixel
  int wp;    // Wo / 2
};
struct NoHmax {};

// Folds value `v` into a running maximum the reference's way.
__device__ __forceinline__ float pool_max_step(float m, float v) { return v > m ? v : m; }

// Per-warp staging block of the fused max pool's epilogue: 32 pixels x 32
// channels, row pitch 36 floats (16-byte aligned rows, conflict-free float4
// stores and column reads).
constexpr int kHmaxPitch = 36;
constexpr int kHmaxStageBytes = 4 * 32 * kHmaxPitch * 4;

// conv_epilogue_tile for the fused max pool: same accumulator drain, BN and
// activation; each warp then stages its 32 pixels x 32 channels in shared
// memory (`stg`, this warp's block) and reads it back transposed, so that
// lane l scans channel l along the 32 pixels and writes that channel's 16
// horizontal maxima (float4 stores where the row segment allows).
template <int BNC, int kAct>
__device__ __forceinline__ bool conv_epilogue_tile_hmax(const ConvParams &p, uint32_t acc_tmem,
                                                        int quad, int lane, int et, int mb,
                                                        int nb, float4 *ep_s, float *ep_beta_s,
                                                        uint64_t *acc_full, uint32_t acc_phase,
                                                        volatile int *abort_flag,
                                                        const HmaxOut &f, float *stg) {
  mbar_wait(acc_full, acc_phase, abort_flag, p.status, kStatusTimeoutEpilogue);
  named_barrier_sync(1, 128);
  if (*abort_flag) return false;
  for (int i = et; i < BNC; i += 128) {
    const int co = nb * BNC + i;
    ep_s[i] = make_float4(p.ep[kEpBias * p.cout_pad + co], p.ep[kEpMean * p.cout_pad + co],
                          p.ep[kEpGamma * p.cout_pad + co], p.ep[kEpInvStd * p.cout_pad + co]);
    ep_beta_s[i] = p.ep[kEpBeta * p.cout_pad + co];
  }
  named_barrier_sync(1, 128);
  tc_fence_after_sync();
  // The warp's 32 pixels g0 .. g0+31 (warp-uniform): first pixel (n0, oh0,
  // ow0); pixel b (even, since g0 and Wo are even) starts the next output
  // row when b < 32; pixels from `nvalid` on lie past the last one.
  const int g0 = mb * kConvBM + quad * 32;
  const int n0 = g0 / static_cast<int>(p.HoWo);
  const int r0 = g0 - n0 * static_cast<int>(p.HoWo);
  const int oh0 = r0 / p.Wo;
  const int ow0 = r0 - oh0 * p.Wo;
  const int b = p.Wo - ow0;  // >= 32: one row
  const int n1 = oh0 + 1 == p.Ho ? n0 + 1 : n0;
  const int oh1 = oh0 + 1 == p.Ho ? 0 : oh0 + 1;
  const int nvalid = p.M - g0 < 32 ? p.M - g0 : 32;
  const bool vec = b >= 32 && nvalid == 32 && ((ow0 >> 1) & 3) == 0 && (f.wp & 3) == 0;
  const uint32_t t_row = acc_tmem + (static_cast<uint32_t>(quad * 32) << 16);
  const float ninf = -__int_as_float(0x7f800000);
#pragma unroll 1
  for (int c0 = 0; c0 < BNC; c0 += 32) {
    uint32_t v[32], w[32];
    tmem_ld32(t_row + c0, v);
    tmem_ld32(t_row + BNC + c0, w);
    tmem_wait_ld2(v, w);
    float out[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float4 c = ep_s[c0 + j];
      float t = (__uint_as_float(v[j]) + __uint_as_float(w[j])) + c.x;
      t = c.z * (t - c.y) * c.w + ep_beta_s[c0 + j];
      out[j] = epilogue_act<kAct>(t, p.act, p.act_alpha);
    }
    float4 *s4 = reinterpret_cast<float4 *>(stg + lane * kHmaxPitch);
#pragma unroll
    for (int q = 0; q < 8; ++q)
      s4[q] = make_float4(out[4 * q], out[4 * q + 1], out[4 * q + 2], out[4 * q + 3]);
    __syncwarp();
    float col[32];  // channel co0 + lane along the 32 pixels
#pragma unroll
    for (int q = 0; q < 32; ++q) col[q] = stg[q * kHmaxPitch + lane];
    __syncwarp();  // the next chunk rewrites the block
    float hm[16];
#pragma unroll
    for (int q = 0; q < 16; ++q) {
      const int pc = 2 * q;  // centre pixel within the group
      float mx = ninf;
      // left neighbour in the group unless the centre starts a row (the
      // group's first pixel takes it from e in the vertical pass)
      if (pc > 0 && pc != b) mx = pool_max_step(mx, col[pc - 1]);
      mx = pool_max_step(mx, col[pc]);
      mx = pool_max_step(mx, col[pc + 1]);
      hm[q] = mx;
    }
    const int co = nb * BNC + c0 + lane;
    if (co < p.Cout) {
      float *ha = f.h + ((static_cast<int64_t>(n0) * p.Cout + co) * p.Ho + oh0) * f.wp + (ow0 >> 1);
      if (vec) {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          reinterpret_cast<float4 *>(ha)[q] =
              make_float4(hm[4 * q], hm[4 * q + 1], hm[4 * q + 2], hm[4 * q + 3]);
      } else {
        float *hb = f.h + ((static_cast<int64_t>(n1) * p.Cout + co) * p.Ho + oh1) * f.wp;
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const int pc = 2 * q;
          if (pc >= nvalid) break;
          if (pc < b)
            ha[q] = hm[q];
          else
            hb[(pc - b) >> 1] = hm[q];
        }
      }
      // The group's last pixel, for the next group's first centre.
      if (nvalid == 32) f.e[static_cast<int64_t>(g0 / kHmaxGroup) * p.Cout + co] = col[31];
    }
  }
  return true;
}

// Launches the TMA-im2col conv (conv_im2col.cu) for channel counts that are a
// multiple of 32: x_hi / x_lo are the input's NHWC tf32 hi/lo planes written
// by launch_nchw_to_nhwc_split. Returns an NPL error code.
int launch_conv_im2col(cudaStream_t s, int bnc, const float *wsplit, int64_t kp,
                       int64_t n_blocks, const float *x_hi, const float *x_lo,
                       const ConvParams &prm, int n_img);

// True when launch_conv_im2col supports the geometry (corner and traversal
// ranges of the im2col tensor map, plane size).
bool conv_im2col_supported(const ConvParams &prm, int n_img);

// x[n][c][hw] -> hi[n][hw][c], lo[n][hw][c] with hi = tf32 truncation of x
// and lo = x - hi (exact); with lo == nullptr, hi[n][hw][c] = x (no split).
// c must be a multiple of 32.
int launch_nchw_to_nhwc_split(cudaStream_t s, const float *x, float *hi, float *lo, int n,
                              int c, int64_t hw);

// Window conv (conv_window.cu) over the raw NHWC plane x_nhwc, or gathering
// from NCHW prm.x when x_nhwc is NULL; its GEMM rows are the virtual pixels
// given by conv_window_rows. after_prep: the previous kernel in the stream
// is this call's conv_prep_kernel (the gather form then overlaps it).
int launch_conv_window(cudaStream_t s, int bnc, const float *wsplit, int64_t kp, int64_t n_blocks,
                       const float *x_nhwc, ConvParams prm, int n_img, bool after_prep = false);
bool conv_window_supported(const ConvParams &prm, int n_img);

// Window-gather conv on CTA pairs (conv_window_pair.cu): every MMA spans two
// SMs (tcgen05 cta_group::2), each SM reading half of the weight operand.
// Needs the gather form's conditions, C_out <= 64 (one output-channel block
// of 64) and taps shared along the row (stride_w 1, KW > 1, (KW-1)*dw <= 8).
bool conv_window_pair_supported(const ConvParams &prm, int n_img, int bnc, int64_t n_blocks);
int launch_conv_window_pair(cudaStream_t s, const float *wsplit, int64_t kp, ConvParams prm,
                            int n_img, bool after_prep);
// The gather variant also needs x to have fewer than 2^31 elements.
bool conv_window_gather_supported(const ConvParams &prm, int n_img);
void conv_window_rows(const ConvParams &p, int *wv, int64_t *mv);

}  // namespace nplk
