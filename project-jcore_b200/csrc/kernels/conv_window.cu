// Fused conv2d + bias + BN + activation for C_in % 32 == 0 and stride_w == 1:
// TMA im2col "windows" shared by the KW taps of a filter row, over the input
// rewritten once as a raw NHWC plane.
//
// GEMM rows are virtual pixels (n, oh, ow') with ow' < Wv = Wo + (KW-1)*dw:
// the im2col traversal walks each output row plus the (KW-1)*dw positions
// to its right. For such a traversal, the A rows of tap (kh, kw) for 128
// consecutive virtual pixels are the A rows of tap (kh, 0) shifted by kw*dw
// rows, for every row with ow' < Wo (ow' + kw*dw stays in the same output
// row). So one TMA load of 128 + (KW-1)*dw rows per (tile, channel block,
// kh) serves all KW taps: the MMA descriptor start moves by kw*dw 128-byte
// rows (the 128-byte swizzle is a function of the absolute shared-memory
// address, so any row offset reads back what the TMA wrote). Rows with
// ow' >= Wo are computed and dropped in the epilogue (2/58 of the work for a
// 3x3 conv on 56-wide maps).
//
// 3xTF32 split without a lo plane: the tensor core reads an fp32 operand as
// its tf32 truncation, so the raw window is A_hi as it stands; a converter
// warpgroup writes A_lo = x - trunc(x) (exact) next to it, once per window.
// Same products, k order and accumulation sequence as the other conv
// kernels (k-block = one tap over 32 channels, MMA(A_hi, [W_hi; W_lo]) then
// MMA(A_lo, W_hi) per 8-wide k step), so the results equal theirs bit for
// bit.
//
// Per CTA (see ConvWinTraits): kPipes independent pipelines on alternate
// tiles, each with two TMA producer threads (windows, weight slabs), a
// converter warpgroup and an MMA warp, plus four epilogue warps. Reference
// semantics: ExecuteConvDirect (advanced/neural_layer/src/
// npl_convolution.cpp:248-378) plus the fused bias / inference BN /
// activation epilogue.
#include <cuda_runtime.h>

#include "conv_common.cuh"
#include "nplk_host.h"

namespace nplk {

constexpr int kWinMaxExtra = 8;                                   // (KW-1)*dw limit
constexpr int kWinRowsMax = kConvBM + kWinMaxExtra;               // 136
constexpr int kWinBytes = kWinRowsMax * kConvBK * 4;              // 17 KB, 1024-aligned

// Shared memory: per pipeline kWinSlots window slots (x and lo parts), then
// one ring of weight slabs that all pipelines read. With two pipelines
// (C_out <= 64, a single output-channel block) every tile walks the same
// slab sequence, so both MMA warps consume each slab (one TMA load serves
// both, and the ring is twice as deep as two private rings in the same
// space).
template <int BNC, bool kGather>
struct ConvWinTraits {
  static constexpr int kPipes = BNC == 64 ? 2 : 1;
  static constexpr int kWinSlots = BNC == 64 ? 2 : 3;  // per pipeline
  static constexpr int kBSlots = BNC == 64 ? 4 : 3;    // shared
  static constexpr int kBBytes = 2 * BNC * kConvBK * 4;
  static constexpr int kWinSlotBytes = 2 * kWinBytes;  // x + lo
  static constexpr int kWinAreaBytes = kPipes * kWinSlots * kWinSlotBytes;
  static constexpr int kPipeBytes = kWinAreaBytes + kBSlots * kBBytes;  // all stage memory
  // warp 0: weight-slab producer; warps 1..kPipes (TMA windows only): window
  // producers; then one MMA warp per pipeline, 4 window warps per pipeline
  // (converter or gather), 4 epilogue warps.
  static constexpr int kProdWarps = kGather ? 1 : 1 + kPipes;
  static constexpr int kFirstMmaWarp = kProdWarps;
  static constexpr int kFirstCvtWarp = kProdWarps + kPipes;
  static constexpr int kFirstEpiWarp = kFirstCvtWarp + 4 * kPipes;
  static constexpr int kThreads = (kFirstEpiWarp + 4) * 32;
  static constexpr int kAccCols = 2 * BNC;
  static constexpr int kAccPerPipe = 2;
  static constexpr int kTmemCols = kPipes * kAccPerPipe * kAccCols;
  static constexpr int kBarrierBytes = 512;
  // Per-channel epilogue constants (float4 + beta per channel) for each
  // draining warpgroup: the epilogue warps, then each pipeline's window
  // warpgroup, which drains its pipeline's last tile.
  static constexpr int kEpConstBytes = BNC * 20;
  static constexpr int kSmemBytes = 1024 + kPipeBytes + kBarrierBytes + (1 + kPipes) * kEpConstBytes;
  static_assert(kTmemCols == 512, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

struct WinGeom {
  int taps_per_win;  // KW (shared windows) or 1
  int win_rows;      // 128 + (taps_per_win - 1) * dw
  int wins_per_row;  // KW / taps_per_win
};

// kGather: the window warpgroups load the window straight from NCHW x
// (coalesced along w), writing x and lo = x - trunc(x) into the window slot;
// no NHWC plane, no window TMA. Otherwise the window comes from the raw NHWC
// plane by im2col TMA and the warpgroups only add the lo part.
template <int BNC, int kAct, bool kGather>
__global__ void __launch_bounds__(ConvWinTraits<BNC, kGather>::kThreads, 1)
    conv_window_3xtf32_kernel(const __grid_constant__ CUtensorMap map_x,
                              const __grid_constant__ CUtensorMap map_w, const ConvParams p,
                              const WinGeom wg) {
  using T = ConvWinTraits<BNC, kGather>;
  constexpr int P = T::kPipes;
  constexpr int WS = T::kWinSlots;
  constexpr int BS = T::kBSlots;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align_smem_1024(smem_raw);
  uint8_t *bslots = smem + T::kWinAreaBytes;
  uint8_t *bars = smem + T::kPipeBytes;
  uint64_t *win_full = reinterpret_cast<uint64_t *>(bars);  // [P][WS] raw window landed
  uint64_t *win_ready = win_full + P * WS;                   // [P][WS] lo part written
  uint64_t *win_empty = win_ready + P * WS;                  // [P][WS] MMAs done with it
  uint64_t *b_full = win_empty + P * WS;                     // [BS]
  uint64_t *b_empty = b_full + BS;                           // [BS], one arrival per pipeline
  uint64_t *acc_full = b_empty + BS;                         // [P * kAccPerPipe]
  uint64_t *acc_empty = acc_full + P * T::kAccPerPipe;
  uint64_t *never = acc_empty + P * T::kAccPerPipe;  // never arrived on (injected_stall)
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(never + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  // Epilogue constants of draining warpgroup g (0: the epilogue warps, 1 + p:
  // the window warpgroup of pipeline p).
  auto ep_area = [&](int g) {
    return reinterpret_cast<float4 *>(bars + T::kBarrierBytes + g * T::kEpConstBytes);
  };

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < P * WS; ++s) {
      mbar_init(&win_full[s], 1);
      mbar_init(&win_ready[s], 4);
      mbar_init(&win_empty[s], 1);
    }
    for (int s = 0; s < BS; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], P);
    }
    for (int a = 0; a < P * T::kAccPerPipe; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    mbar_init(never, 1);
    *abort_flag = 0;
    fence_mbar_init();
    if (!kGather) tma_prefetch_desc(&map_x);
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
  const int cblocks = p.C / kConvBK;
  const int win_bytes = wg.win_rows * kConvBK * 4;
  // Drains this CTA's local tile j (tile blockIdx.x + j * gridDim.x, run by
  // pipeline j % P) with a warpgroup of four warps (quad = TMEM lane quadrant,
  // et = 0..127): draining warpgroup g, named barrier bar_id. False when the
  // CTA aborted.
  auto drain_tile = [&](int j, int quad, int et, int g, int bar_id) -> bool {
    const int tile = blockIdx.x + j * static_cast<int>(gridDim.x);
    const int jj = j / P;
    const int acc = (j % P) * T::kAccPerPipe + (jj & 1);
    const uint32_t acc_phase = (jj >> 1) & 1;
    const int mb = tile / p.n_blocks;
    const int nb = tile - mb * p.n_blocks;
    float4 *ep_s = ep_area(g);
    if (!conv_epilogue_tile<BNC, kAct>(p, tmem_base + acc * T::kAccCols, quad, lane, et, mb, nb,
                                       ep_s, reinterpret_cast<float *>(ep_s + BNC),
                                       &acc_full[acc], acc_phase, abort_flag, 0u, bar_id))
      return false;
    tc_fence_before_sync();
    __syncwarp();
    if (lane == 0) mbar_arrive(&acc_empty[acc]);
    return true;
  };
  // Window warpgroup of pipeline `pipe`, after its last window: drains the
  // pipeline's last tile, so that the CTA's final tiles drain in parallel
  // rather than one after another in the epilogue warps.
  auto drain_last_tile = [&](int pipe) -> bool {
    const int first = blockIdx.x + pipe * static_cast<int>(gridDim.x);
    if (first >= num_tiles) return true;
    const int step = P * static_cast<int>(gridDim.x);
    const int jj_last = (num_tiles - 1 - first) / step;
    const int et = threadIdx.x - (T::kFirstCvtWarp + 4 * pipe) * 32;
    griddep_wait();  // the epilogue constants may come from the preparation just before
    return drain_tile(pipe + P * jj_last, warp & 3, et, 1 + pipe, 2 + pipe);
  };
  // Local tile j of this CTA is tile blockIdx.x + j*gridDim.x; pipeline j % P
  // runs it. Per tile: windows (cb, kh, kw group) in that order, each
  // followed by its taps_per_win weight slabs.

  if (warp == 0) {
    // ---------------- weight-slab producer (all pipelines) ----------------
    // Round r carries the slabs of each pipeline's r-th tile; with two
    // pipelines those tiles share one output-channel block, so one sequence
    // serves both. A pipeline without an r-th tile is stood in for by an
    // extra arrival on the slab's empty barrier.
    if (lane == 0) {
      griddep_wait();  // the slabs may come from the weight preparation just before
      int bs = 0;
      uint32_t bph = 0;
      uint32_t b_issued = 0, b_issued_ph = 0;
      for (int r = 0;; ++r) {
        const int tile = blockIdx.x + P * r * gridDim.x;  // pipeline 0's r-th tile
        if (tile >= num_tiles) break;
        int missing = 0;
        for (int q = 1; q < P; ++q)
          if (tile + q * static_cast<int>(gridDim.x) >= num_tiles) ++missing;
        const int nb = tile - (tile / p.n_blocks) * p.n_blocks;  // 0 when P > 1
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&b_empty[bs], bph ^ 1u, abort_flag, p.status, kStatusTimeoutProducer))
            goto producer_done;
          mbar_arrive_expect_tx(&b_full[bs], T::kBBytes);
          tma_load_2d(&map_w, &b_full[bs], bslots + bs * T::kBBytes, kb * kConvBK, nb * 2 * BNC);
          for (int q = 0; q < missing; ++q) mbar_arrive(&b_empty[bs]);
          b_issued |= 1u << bs;
          b_issued_ph = (b_issued_ph & ~(1u << bs)) | (bph << bs);
          if (++bs == BS) {
            bs = 0;
            bph ^= 1u;
          }
        }
      }
    producer_done:
      // Let every issued copy land before the CTA can exit (all of them
      // already have unless the CTA aborted).
      for (int s = 0; s < BS; ++s)
        if (b_issued & (1u << s)) mbar_drain(&b_full[s], (b_issued_ph >> s) & 1u);
    }
  } else if (warp < T::kProdWarps) {
    // ---------------- window TMA producer of pipeline `pipe` (raw NHWC plane) ----------------
    const int pipe = warp - 1;
    if (lane == 0) {
      uint8_t *wbase = smem + pipe * WS * T::kWinSlotBytes;
      uint64_t *wf = win_full + pipe * WS, *we = win_empty + pipe * WS;
      int ws = 0;
      uint32_t wph = 0;
      uint32_t w_issued = 0, w_issued_ph = 0;
      for (int tile = blockIdx.x + pipe * gridDim.x; tile < num_tiles; tile += P * gridDim.x) {
        const int mb = tile / p.n_blocks;
        const int v0 = mb * kConvBM;
        const int howv = p.Ho * p.Wv;
        const int n0 = v0 / howv;
        const int rem = v0 - n0 * howv;
        const int oh0 = rem / p.Wv;
        const int ow0 = rem - oh0 * p.Wv;
        const int w0 = ow0 * p.sw - p.pl;
        const int h0 = oh0 * p.sh - p.pt;
        for (int cb = 0; cb < cblocks; ++cb) {
          for (int kh = 0; kh < p.KH; ++kh) {
            for (int kg = 0; kg < wg.wins_per_row; ++kg) {
              if (!mbar_wait(&we[ws], wph ^ 1u, abort_flag, p.status, kStatusTimeoutProducer))
                goto window_done;
              mbar_arrive_expect_tx(&wf[ws], win_bytes);
              tma_load_im2col_4d(&map_x, &wf[ws], wbase + ws * T::kWinSlotBytes, cb * kConvBK, w0,
                                 h0, n0, static_cast<uint16_t>(kg * p.dw),
                                 static_cast<uint16_t>(kh * p.dh));
              w_issued |= 1u << ws;
              w_issued_ph = (w_issued_ph & ~(1u << ws)) | (wph << ws);
              if (++ws == WS) {
                ws = 0;
                wph ^= 1u;
              }
            }
          }
        }
      }
    window_done:
      for (int s = 0; s < WS; ++s)
        if (w_issued & (1u << s)) mbar_drain(&wf[s], (w_issued_ph >> s) & 1u);
    }
  } else if (warp < T::kFirstCvtWarp) {
    // ---------------- MMA issuer of pipeline `pipe` ----------------
    const int pipe = warp - T::kFirstMmaWarp;
    if (lane == 0) {
      const uint32_t idesc_2n = umma_idesc_tf32(kConvBM, 2 * BNC);
      const uint32_t idesc_n = umma_idesc_tf32(kConvBM, BNC);
      const uint64_t win_desc0 = umma_desc_sw128(smem_u32(smem + pipe * WS * T::kWinSlotBytes));
      const uint64_t b_desc0 = umma_desc_sw128(smem_u32(bslots));
      constexpr uint64_t kLoOff = kWinBytes >> 4;
      uint64_t *wr = win_ready + pipe * WS, *we = win_empty + pipe * WS;
      uint64_t *bf = b_full, *be = b_empty;
      int ws = 0, bs = 0;
      uint32_t wph = 0, bph = 0;
      int jj = 0;
      const bool go = injected_stall(never, p.stall_us, abort_flag, p.status);
      for (int tile = blockIdx.x + pipe * gridDim.x; go && tile < num_tiles;
           tile += P * gridDim.x, ++jj) {
        const int acc = pipe * T::kAccPerPipe + (jj & 1);
        const uint32_t acc_phase = (jj >> 1) & 1;
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, abort_flag, p.status,
                       kStatusTimeoutAccFree))
          break;
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * T::kAccCols;
        bool first = true;
        for (int cb = 0; cb < cblocks; ++cb) {
          for (int kh = 0; kh < p.KH; ++kh) {
            for (int kg = 0; kg < wg.wins_per_row; ++kg) {
              if (!mbar_wait(&wr[ws], wph, abort_flag, p.status, kStatusTimeoutMma))
                goto mma_done;
              const uint64_t wdesc = win_desc0 + static_cast<uint64_t>(ws * (T::kWinSlotBytes >> 4));
              for (int t = 0; t < wg.taps_per_win; ++t) {
                if (!mbar_wait(&bf[bs], bph, abort_flag, p.status, kStatusTimeoutMma))
                  goto mma_done;
                tc_fence_after_sync();
                // tap t reads the window from row t*dw (128 bytes per row)
                const uint64_t a_desc = wdesc + static_cast<uint64_t>(t * p.dw * 8);
                const uint64_t b_desc = b_desc0 + static_cast<uint64_t>(bs * (T::kBBytes >> 4));
#pragma unroll
                for (int kk = 0; kk < kConvBK / 8; ++kk) {
                  mma_tf32_ss(d_tmem, a_desc + 2 * kk, b_desc + 2 * kk, idesc_2n,
                              (first && kk == 0) ? 0u : 1u);
                  mma_tf32_ss(d_tmem, a_desc + kLoOff + 2 * kk, b_desc + 2 * kk, idesc_n, 1u);
                }
                first = false;
                mma_commit(&be[bs]);
                if (++bs == BS) {
                  bs = 0;
                  bph ^= 1u;
                }
              }
              mma_commit(&we[ws]);
              if (++ws == WS) {
                ws = 0;
                wph ^= 1u;
              }
            }
          }
        }
        mma_commit(&acc_full[acc]);
      }
    mma_done:;
    }
  } else if (warp < T::kFirstEpiWarp && kGather) {
    // ---------------- gather warpgroup of pipeline `pipe`: window from NCHW x ----------------
    // Warp gw of the group loads channel quads gw and gw + 4 of the window's
    // 32 channels; lane l loads rows l, l + 32, ... (consecutive virtual
    // pixels, so each load instruction reads consecutive input columns).
    const int pipe = (warp - T::kFirstCvtWarp) >> 2;
    const int gw = (warp - T::kFirstCvtWarp) & 3;
    uint8_t *base = smem + pipe * WS * T::kWinSlotBytes;
    uint64_t *we = win_empty + pipe * WS, *wr = win_ready + pipe * WS;
    constexpr int kRowsPerLane = (kWinRowsMax + 31) / 32;  // 5
    int ws = 0;
    uint32_t wph = 0;
    const int howv = p.Ho * p.Wv;
    // x has fewer than 2^31 elements on this path: 32-bit element offsets.
    const int hw = static_cast<int>(p.HW);
    int choff[8];  // offsets of this warp's 8 channels within a 32-channel block
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int e = 0; e < 4; ++e) choff[4 * h + e] = (4 * gw + 16 * h + e) * hw;
    for (int tile = blockIdx.x + pipe * gridDim.x; tile < num_tiles; tile += P * gridDim.x) {
      const int mb = tile / p.n_blocks;
      const int v0 = mb * kConvBM;
      int rbase[kRowsPerLane];  // x offset of (n, ih0, iw0) of the row
      int rih[kRowsPerLane], riw[kRowsPerLane];
      bool rvalid[kRowsPerLane];
#pragma unroll
      for (int i = 0; i < kRowsPerLane; ++i) {
        const int r = lane + 32 * i;
        const int v = v0 + r;
        rvalid[i] = r < wg.win_rows && v < p.Mv;
        int n = 0, oh = 0, ow = 0;
        if (rvalid[i]) {
          n = v / howv;
          const int rem = v - n * howv;
          oh = rem / p.Wv;
          ow = rem - oh * p.Wv;
        }
        rih[i] = oh * p.sh - p.pt;
        riw[i] = ow * p.sw - p.pl;
        rbase[i] = n * static_cast<int>(p.CHW) + rih[i] * p.W + riw[i];
      }
      for (int cb = 0; cb < cblocks; ++cb) {
        for (int kh = 0; kh < p.KH; ++kh) {
          for (int kg = 0; kg < wg.wins_per_row; ++kg) {
            // Load before waiting for the slot, so the load latency overlaps
            // the MMAs still reading it.
            float vals[kRowsPerLane][2][4];
            const int dh = kh * p.dh, dwo = kg * p.dw;
            const int woff = cb * kConvBK * hw + dh * p.W + dwo;
#pragma unroll
            for (int i = 0; i < kRowsPerLane; ++i) {
              const int ih = rih[i] + dh, iw = riw[i] + dwo;
              const bool ok = rvalid[i] && static_cast<unsigned>(ih) < static_cast<unsigned>(p.H) &&
                              static_cast<unsigned>(iw) < static_cast<unsigned>(p.W);
              const int off = rbase[i] + woff;
#pragma unroll
              for (int h = 0; h < 2; ++h)
#pragma unroll
                for (int e = 0; e < 4; ++e)
                  vals[i][h][e] = ok ? __ldg(p.x + (off + choff[4 * h + e])) : 0.0f;
            }
            if (!mbar_wait(&we[ws], wph ^ 1u, abort_flag, p.status, kStatusTimeoutProducer))
              goto role_done;
            uint8_t *slot = base + ws * T::kWinSlotBytes;
#pragma unroll
            for (int i = 0; i < kRowsPerLane; ++i) {
              const int r = lane + 32 * i;
              if (r >= wg.win_rows) continue;
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const uint32_t off = sw128_offset(r, gw + 4 * h);
                float4 hi4 = make_float4(vals[i][h][0], vals[i][h][1], vals[i][h][2], vals[i][h][3]);
                float4 lo4;
                float t;
                tf32_split_trunc(hi4.x, t, lo4.x);
                tf32_split_trunc(hi4.y, t, lo4.y);
                tf32_split_trunc(hi4.z, t, lo4.z);
                tf32_split_trunc(hi4.w, t, lo4.w);
                *reinterpret_cast<float4 *>(slot + off) = hi4;
                *reinterpret_cast<float4 *>(slot + kWinBytes + off) = lo4;
              }
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&wr[ws]);
            if (++ws == WS) {
              ws = 0;
              wph ^= 1u;
            }
          }
        }
      }
    }
    if (!drain_last_tile(pipe)) goto role_done;
  } else if (warp < T::kFirstEpiWarp) {
    // ---------------- converter warpgroup of pipeline `pipe`: lo = x - trunc(x) ----------------
    const int pipe = (warp - T::kFirstCvtWarp) >> 2;
    const int ct = threadIdx.x - (T::kFirstCvtWarp + pipe * 4) * 32;  // 0..127
    uint8_t *base = smem + pipe * WS * T::kWinSlotBytes;
    uint64_t *wf = win_full + pipe * WS, *wr = win_ready + pipe * WS;
    const int chunks = win_bytes >> 4;  // 16-byte chunks of the window
    int ws = 0;
    uint32_t wph = 0;
    const int wins_per_tile = cblocks * p.KH * wg.wins_per_row;
    for (int tile = blockIdx.x + pipe * gridDim.x; tile < num_tiles; tile += P * gridDim.x) {
      for (int wi = 0; wi < wins_per_tile; ++wi) {
        if (!mbar_wait(&wf[ws], wph, abort_flag, p.status, kStatusTimeoutProducer)) goto cvt_done;
        {
          // The split is elementwise, so it works on the swizzled bytes as
          // they lie: chunk i of the lo part is computed from chunk i of x.
          const float4 *src = reinterpret_cast<const float4 *>(base + ws * T::kWinSlotBytes);
          float4 *dst = reinterpret_cast<float4 *>(base + ws * T::kWinSlotBytes + kWinBytes);
          for (int i = ct; i < chunks; i += 128) {
            const float4 v = src[i];
            float4 l;
            float h;
            tf32_split_trunc(v.x, h, l.x);
            tf32_split_trunc(v.y, h, l.y);
            tf32_split_trunc(v.z, h, l.z);
            tf32_split_trunc(v.w, h, l.w);
            dst[i] = l;
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&wr[ws]);
        if (++ws == WS) {
          ws = 0;
          wph ^= 1u;
        }
      }
    }
    drain_last_tile(pipe);
  cvt_done:;
  } else {
    // ---------------- epilogue (4 warps, one per TMEM lane quadrant) ----------------
    const int quad = warp & 3;
    const int et = threadIdx.x - T::kFirstEpiWarp * 32;  // 0..127
    griddep_wait();  // the epilogue constants, likewise
    int j = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++j) {
      // A pipeline's last tile is drained by its window warpgroup.
      if (tile + P * static_cast<int>(gridDim.x) >= num_tiles) continue;
      if (!drain_tile(j, quad, et, 0, 1)) break;
    }
  }

role_done:
  __syncthreads();
  if (warp == T::kFirstMmaWarp) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, T::kTmemCols);
  }
}

namespace {

// Window geometry: KW taps share a window when the traversal steps one input
// column per output column.
WinGeom win_geom(const ConvParams &p) {
  WinGeom g;
  const bool share = p.sw == 1 && p.KW > 1 && (p.KW - 1) * p.dw <= kWinMaxExtra;
  g.taps_per_win = share ? p.KW : 1;
  g.win_rows = kConvBM + (g.taps_per_win - 1) * p.dw;
  g.wins_per_row = p.KW / g.taps_per_win;
  return g;
}

template <int BNC, int kAct, bool kGather>
int launch_win(cudaStream_t s, const CUtensorMap &mx, const CUtensorMap &mw,
               const ConvParams &prm, const WinGeom &wg, bool after_prep) {
  using T = ConvWinTraits<BNC, kGather>;
  auto kernel = conv_window_3xtf32_kernel<BNC, kAct, kGather>;
  int rc = ensure_dynamic_smem(reinterpret_cast<const void *>(kernel), T::kSmemBytes);
  if (rc) return rc;
  const int64_t tiles = static_cast<int64_t>(prm.m_blocks) * prm.n_blocks;
  const int grid = static_cast<int>(tiles < sm_count() ? tiles : sm_count());
  if (after_prep)
    // Overlap with the weight preparation launched just before: the gather
    // warps only read x (complete before the preparation started); the slab
    // producer and the epilogue wait for the preparation's writes.
    return launch_programmatic(kernel, dim3(grid), dim3(T::kThreads), T::kSmemBytes, s, mx, mw,
                               prm, wg);
  kernel<<<grid, T::kThreads, T::kSmemBytes, s>>>(mx, mw, prm, wg);
  count_launch();
  return launch_result();
}

template <int BNC, bool kGather>
int dispatch_win(cudaStream_t s, const CUtensorMap &mx, const CUtensorMap &mw,
                 const ConvParams &prm, const WinGeom &wg, bool after_prep) {
  if (prm.act == 0) return launch_win<BNC, kEpiActNone, kGather>(s, mx, mw, prm, wg, after_prep);
  if (prm.act == 1) return launch_win<BNC, kEpiActRelu, kGather>(s, mx, mw, prm, wg, after_prep);
  return launch_win<BNC, kEpiActAny, kGather>(s, mx, mw, prm, wg, after_prep);
}

}  // namespace

void conv_window_rows(const ConvParams &p, int *wv, int64_t *mv) {
  const WinGeom g = win_geom(p);
  *wv = p.Wo + (g.taps_per_win - 1) * p.dw;
  *mv = static_cast<int64_t>(p.M / p.Wo) * *wv;
}

bool conv_window_gather_supported(const ConvParams &p, int n_img) {
  return conv_window_supported(p, n_img) &&
         static_cast<int64_t>(n_img) * p.CHW < (int64_t(1) << 31);
}

bool conv_window_supported(const ConvParams &p, int n_img) {
  if (p.C % kConvBK != 0 || n_img <= 0 || n_img > 65535) return false;
  if (p.sw > 8 || p.sh > 8) return false;  // TMA traversal stride limit
  if ((p.KW - 1) * p.dw > 65535 || (p.KH - 1) * p.dh > 65535) return false;
  int wv;
  int64_t mv;
  conv_window_rows(p, &wv, &mv);
  if (mv >= (int64_t(1) << 31)) return false;
  const int lower_w = -p.pl, lower_h = -p.pt;
  const int upper_w = (wv - 1) * p.sw - p.pl - (p.W - 1);
  const int upper_h = (p.Ho - 1) * p.sh - p.pt - (p.H - 1);
  for (int v : {lower_w, lower_h, upper_w, upper_h})
    if (v < -128 || v > 127) return false;
  // Small inputs stay on the direct-gather kernel.
  const int64_t plane_bytes = static_cast<int64_t>(n_img) * p.H * p.W * p.C * 4;
  return plane_bytes >= (int64_t(128) << 10);
}

int launch_conv_window(cudaStream_t s, int bnc, const float *wsplit, int64_t kp, int64_t n_blocks,
                       const float *x_nhwc, ConvParams prm, int n_img, bool after_prep) {
  if (!conv_window_supported(prm, n_img)) return kErrUnsupported;
  const bool gather = x_nhwc == nullptr;  // read NCHW prm.x directly
  if (bnc == 64 && n_blocks != 1) return kErrUnsupported;  // pipelines share one slab sequence
  if (gather && !prm.x) return kErrInvalidArg;
  const WinGeom wg = win_geom(prm);
  int wv;
  int64_t mv;
  conv_window_rows(prm, &wv, &mv);
  prm.Wv = wv;
  prm.Mv = static_cast<int>(mv);
  prm.m_blocks = static_cast<int>(ceil_div(mv, kConvBM));
  prm.stall_us = take_armed_stall(NPLK_DEBUG_CONV_WINDOW);
  CUtensorMap mx, mw;
  int rc = kOk;
  if (gather) {
    mx = CUtensorMap{};  // unused
  } else {
    rc = encode_tmap_im2col_nhwc_f32_sw128(
        &mx, x_nhwc, prm.C, prm.W, prm.H, n_img, -prm.pl, -prm.pt,
        (wv - 1) * prm.sw - prm.pl - (prm.W - 1), (prm.Ho - 1) * prm.sh - prm.pt - (prm.H - 1),
        prm.sw, prm.sh, kConvBK, wg.win_rows);
    if (rc) return rc;
  }
  rc = encode_tmap_2d_f32_sw128(&mw, wsplit, kp, n_blocks * 2 * bnc, kp * 4, kConvBK, 2 * bnc);
  if (rc) return rc;
  // Only the gather form may overlap the preparation: the plane-based form
  // reads an NHWC plane written by the kernel right before it.
  if (gather)
    return bnc == 64 ? dispatch_win<64, true>(s, mx, mw, prm, wg, after_prep)
                     : dispatch_win<128, true>(s, mx, mw, prm, wg, after_prep);
  return bnc == 64 ? dispatch_win<64, false>(s, mx, mw, prm, wg, false)
                   : dispatch_win<128, false>(s, mx, mw, prm, wg, false);
}

}  // namespace nplk
