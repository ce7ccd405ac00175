// Fused conv2d + bias + BN + activation on CTA pairs for C_in % 32 == 0,
// stride_w == 1, KW > 1 and C_out <= 64: the window-gather conv of
// conv_window.cu with every MMA spanning two SMs (tcgen05 cta_group::2).
//
// Why pairs: the one-SM kernel is bound by shared-memory bandwidth. Each
// 8-wide k step reads A (128 rows x 32 B) and B ([W_hi; W_lo], 128 rows x
// 32 B) for MMA(A_hi, [W_hi; W_lo]), and A_lo plus W_hi (64 rows) for
// MMA(A_lo, W_hi): 14 KB per step, 128 B/clk at the full tf32 MMA rate of
// the first and above it for the second (N = 64), before the window stores
// and weight slabs are counted. A pair MMA has M = 256 (128 rows of A in
// each SM) and takes half of B from each SM, so each SM reads 11 KB per
// step and stores half as many weight-slab bytes.
//
// Operand split: for MMA(A_hi, [W_hi; W_lo]) (N = 128) the leader (cluster
// rank 0) holds W_hi and the other CTA W_lo; for MMA(A_lo, W_hi) (N = 64) the
// leader holds W_hi rows 0..31 and the other CTA rows 32..63. Each CTA's
// weight slab is therefore 96 rows: its 64-row half of [W_hi; W_lo] (rows
// 64*rank of the split weights) and its 32-row half of W_hi (rows 32*rank),
// loaded by two TMA boxes at the same shared-memory offsets in both CTAs.
// The accumulator columns come out as in the one-SM kernel (x*W_hi + x_lo*W_hi
// in columns 0..63, x*W_lo in 64..127), so the epilogue, the products, the k
// order and the accumulation sequence are those of the other conv kernels.
//
// Tiles: a pair tile is two consecutive 128-row GEMM tiles, CTA rank r taking
// m-block 2*pt + r. Per CTA two pipelines run alternate pair tiles, as in the
// one-SM kernel; the leader's two MMA warps issue for both CTAs, the other
// CTA's MMA warps idle.
//
// Synchronisation (all waits bounded; a timeout raises both CTAs' abort
// flags):
//   win_ready (leader)   8 arrivals: 4 gather warps of each CTA, after their
//                        window stores (remote arrival from the other CTA)
//   b_full (leader)      the leader producer's expect_tx for both CTAs'
//                        slab bytes; both CTAs' TMA loads complete on it
//   win_empty, b_empty,  in each CTA, arrived on by the leader's MMA commit
//   acc_full             (one tcgen05.commit addressed to both CTAs)
//   acc_empty (leader)   8 arrivals: 4 epilogue warps of each CTA
// Reference semantics: ExecuteConvDirect (advanced/neural_layer/src/
// npl_convolution.cpp:248-378) plus the fused bias / inference BN /
// activation epilogue.
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <utility>

#include "conv_common.cuh"
#include "nplk_host.h"

namespace nplk {

namespace {

constexpr int kPairBNC = 64;
constexpr int kPairPipes = 2;
constexpr int kPairWinSlots = 2;                                   // per pipeline
constexpr int kPairMaxExtra = 8;                                   // (KW-1)*dw limit
constexpr int kPairWinBytes = (kConvBM + kPairMaxExtra) * kConvBK * 4;  // 17 KB
constexpr int kPairWinSlotBytes = 2 * kPairWinBytes;               // x + lo
constexpr int kPairWinArea = kPairPipes * kPairWinSlots * kPairWinSlotBytes;
constexpr int kPairSlabRowsA = kPairBNC;      // this CTA's half of [W_hi; W_lo]
constexpr int kPairSlabRowsB = kPairBNC / 2;  // this CTA's half of W_hi
constexpr int kPairSlabBOff = kPairSlabRowsA * kConvBK * 4;                      // 8 KB
constexpr int kPairSlabBytes = (kPairSlabRowsA + kPairSlabRowsB) * kConvBK * 4;  // 12 KB
constexpr int kPairBSlots = 6;
constexpr int kPairStageBytes = kPairWinArea + kPairBSlots * kPairSlabBytes;
constexpr int kPairBarrierBytes = 512;
constexpr int kPairSmemBytes = 1024 + kPairStageBytes + kPairBarrierBytes + kPairBNC * 20;
// warp 0: weight-slab producer; warps 1..2: MMA (one per pipeline; the
// leader's issue); warps 3..10: gather (4 per pipeline); warps 11..14:
// epilogue (one per TMEM lane quadrant).
constexpr int kPairFirstMma = 1;
constexpr int kPairFirstGather = kPairFirstMma + kPairPipes;
constexpr int kPairFirstEpi = kPairFirstGather + 4 * kPairPipes;
constexpr int kPairThreads = (kPairFirstEpi + 4) * 32;
constexpr int kPairAccCols = 2 * kPairBNC;
constexpr int kPairTmemCols = kPairPipes * 2 * kPairAccCols;
static_assert(kPairTmemCols == 512, "TMEM budget");
static_assert(kPairSmemBytes <= 232448, "shared memory budget");
static_assert(kPairSlabBOff % 1024 == 0 && kPairSlabBytes % 1024 == 0 &&
                  kPairWinBytes % 1024 == 0,
              "128-byte-swizzle atoms stay 1024-byte aligned");

// Shared::cluster address of a barrier of the pair's leader (same offset).
__device__ __forceinline__ uint32_t leader_bar(const uint64_t *bar) {
  return mapa_shared(smem_u32(bar), 0u);
}

// Commits the leader's MMAs so far to `bar` in both CTAs.
__device__ __forceinline__ void commit_both(uint64_t *bar) { mma_commit_pair_both(bar); }

}  // namespace

template <int kAct>
__global__ void __launch_bounds__(kPairThreads, 1)
    conv_window_pair_kernel(const __grid_constant__ CUtensorMap map_wa,
                            const __grid_constant__ CUtensorMap map_wb, const ConvParams p,
                            const int win_rows) {
  constexpr int P = kPairPipes;
  constexpr int WS = kPairWinSlots;
  constexpr int BS = kPairBSlots;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align_smem_1024(smem_raw);
  uint8_t *bslots = smem + kPairWinArea;
  uint8_t *bars = smem + kPairStageBytes;
  uint64_t *win_ready = reinterpret_cast<uint64_t *>(bars);  // [P][WS] (leader)
  uint64_t *win_empty = win_ready + P * WS;                   // [P][WS]
  uint64_t *b_full = win_empty + P * WS;                      // [BS] (leader)
  uint64_t *b_empty = b_full + BS;                            // [BS], one arrival per pipeline
  uint64_t *acc_full = b_empty + BS;                          // [P * 2]
  uint64_t *acc_empty = acc_full + P * 2;                     // [P * 2] (leader)
  uint64_t *never = acc_empty + P * 2;                        // never arrived on (injected_stall)
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(never + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  float4 *ep_s = reinterpret_cast<float4 *>(bars + kPairBarrierBytes);
  float *ep_beta_s = reinterpret_cast<float *>(ep_s + kPairBNC);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t peer_abort =
      mapa_shared(smem_u32(const_cast<int *>(abort_flag)), rank ^ 1u);

  if (threadIdx.x == 0) {
    for (int s = 0; s < P * WS; ++s) {
      mbar_init(&win_ready[s], 8);
      mbar_init(&win_empty[s], 1);
    }
    for (int s = 0; s < BS; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], P);
    }
    for (int a = 0; a < P * 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 8);
    }
    mbar_init(never, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&map_wa);
    tma_prefetch_desc(&map_wb);
  }
  if (warp == kPairFirstMma) {
    tmem_alloc_pair(tmem_slot, kPairTmemCols);
    tmem_relinquish_pair();
  }
  tc_fence_before_sync();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers exist before any remote arrival
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;

  const int num_clusters = static_cast<int>(gridDim.x >> 1);
  const int cid = static_cast<int>(blockIdx.x >> 1);
  const int num_pt = (p.m_blocks + 1) >> 1;
  const int cblocks = p.C / kConvBK;
  // Local pair tile j of this cluster is pt = cid + j*num_clusters, run by
  // pipeline j % P. Per pair tile: windows (cb, kh) in that order, each
  // followed by its KW weight slabs.

  if (warp == 0) {
    // ---------------- weight-slab producer (both CTAs) ----------------
    if (lane == 0) {
      griddep_wait();  // the slabs may come from the weight preparation just before
      int bs = 0;
      uint32_t bph = 0;
      uint32_t issued = 0, issued_ph = 0;
      bool aborted = false;
      for (int r = 0;; ++r) {
        const int pt = cid + P * r * num_clusters;  // pipeline 0's r-th pair tile
        if (pt >= num_pt) break;
        const int missing = pt + num_clusters >= num_pt ? 1 : 0;  // no pipeline-1 tile
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait_pair(&b_empty[bs], bph ^ 1u, abort_flag, peer_abort, p.status,
                              kStatusTimeoutProducer)) {
            aborted = true;
            goto producer_done;
          }
          if (rank == 0) mbar_arrive_expect_tx(&b_full[bs], 2 * kPairSlabBytes);
          const uint32_t lb = leader_bar(&b_full[bs]);
          uint8_t *dst = bslots + bs * kPairSlabBytes;
          tma_load_2d_pair(&map_wa, lb, dst, kb * kConvBK, static_cast<int>(rank) * kPairSlabRowsA);
          tma_load_2d_pair(&map_wb, lb, dst + kPairSlabBOff, kb * kConvBK,
                           static_cast<int>(rank) * kPairSlabRowsB);
          for (int q = 0; q < missing; ++q) mbar_arrive(&b_empty[bs]);
          issued |= 1u << bs;
          issued_ph = (issued_ph & ~(1u << bs)) | (bph << bs);
          if (++bs == BS) {
            bs = 0;
            bph ^= 1u;
          }
        }
      }
    producer_done:
      if (rank == 0) {
        // Both CTAs' copies complete on the leader's barriers: let every
        // issued phase land before the pair can exit (they all have unless
        // the pair aborted).
        for (int s = 0; s < BS; ++s)
          if (issued & (1u << s)) mbar_drain(&b_full[s], (issued_ph >> s) & 1u);
      } else if (aborted && issued) {
        // This CTA cannot observe its own copies (they signal the leader):
        // give any still in flight time to land before leaving.
        const uint64_t t0 = global_timer_ns();
        while (global_timer_ns() - t0 < 2000000ull) __nanosleep(1000);
      }
    }
  } else if (warp < kPairFirstGather) {
    // ---------------- MMA issuer of pipeline `pipe` (leader only) ----------------
    const int pipe = warp - kPairFirstMma;
    if (rank == 0 && lane == 0) {
      const uint32_t idesc_2n = umma_idesc_tf32(2 * kConvBM, 2 * kPairBNC);
      const uint32_t idesc_n = umma_idesc_tf32(2 * kConvBM, kPairBNC);
      const uint64_t win_desc0 =
          umma_desc_sw128(smem_u32(smem + pipe * WS * kPairWinSlotBytes));
      const uint64_t b_desc0 = umma_desc_sw128(smem_u32(bslots));
      constexpr uint64_t kLoOff = kPairWinBytes >> 4;
      constexpr uint64_t kBOff = kPairSlabBOff >> 4;
      uint64_t *wr = win_ready + pipe * WS, *we = win_empty + pipe * WS;
      int ws = 0, bs = 0;
      uint32_t wph = 0, bph = 0;
      int jj = 0;
      const bool go = injected_stall(never, p.stall_us, abort_flag, p.status);
      if (!go) pair_raise_abort(peer_abort);
      for (int pt = cid + pipe * num_clusters; go && pt < num_pt;
           pt += P * num_clusters, ++jj) {
        const int acc = pipe * 2 + (jj & 1);
        const uint32_t acc_phase = (jj >> 1) & 1;
        if (!mbar_wait_pair(&acc_empty[acc], acc_phase ^ 1u, abort_flag, peer_abort, p.status,
                            kStatusTimeoutAccFree))
          break;
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * kPairAccCols;
        bool first = true;
        for (int cb = 0; cb < cblocks; ++cb) {
          for (int kh = 0; kh < p.KH; ++kh) {
            if (!mbar_wait_pair(&wr[ws], wph, abort_flag, peer_abort, p.status,
                                kStatusTimeoutMma))
              goto mma_done;
            const uint64_t wdesc = win_desc0 + static_cast<uint64_t>(ws * (kPairWinSlotBytes >> 4));
            for (int t = 0; t < p.KW; ++t) {
              if (!mbar_wait_pair(&b_full[bs], bph, abort_flag, peer_abort, p.status,
                                  kStatusTimeoutMma))
                goto mma_done;
              tc_fence_after_sync();
              // tap t reads the window from row t*dw (128 bytes per row)
              const uint64_t a_desc = wdesc + static_cast<uint64_t>(t * p.dw * 8);
              const uint64_t b_desc = b_desc0 + static_cast<uint64_t>(bs * (kPairSlabBytes >> 4));
#pragma unroll
              for (int kk = 0; kk < kConvBK / 8; ++kk) {
                mma_tf32_ss_pair(d_tmem, a_desc + 2 * kk, b_desc + 2 * kk, idesc_2n,
                                 (first && kk == 0) ? 0u : 1u);
                mma_tf32_ss_pair(d_tmem, a_desc + kLoOff + 2 * kk, b_desc + kBOff + 2 * kk,
                                 idesc_n, 1u);
              }
              first = false;
              commit_both(&b_empty[bs]);
              if (++bs == BS) {
                bs = 0;
                bph ^= 1u;
              }
            }
            commit_both(&we[ws]);
            if (++ws == WS) {
              ws = 0;
              wph ^= 1u;
            }
          }
        }
        commit_both(&acc_full[acc]);
      }
    mma_done:;
    }
  } else if (warp < kPairFirstEpi) {
    // ---------------- gather warpgroup of pipeline `pipe`: this CTA's window ----------------
    // As in conv_window.cu: warp gw loads channel quads gw and gw + 4 of the
    // window's 32 channels, lane l rows l, l + 32, ... (consecutive virtual
    // pixels, so each load instruction reads consecutive input columns).
    const int pipe = (warp - kPairFirstGather) >> 2;
    const int gw = (warp - kPairFirstGather) & 3;
    uint8_t *base = smem + pipe * WS * kPairWinSlotBytes;
    uint64_t *we = win_empty + pipe * WS, *wr = win_ready + pipe * WS;
    constexpr int kRowsPerLane = (kConvBM + kPairMaxExtra + 31) / 32;  // 5
    int ws = 0;
    uint32_t wph = 0;
    const int howv = p.Ho * p.Wv;
    const int hw = static_cast<int>(p.HW);  // x has fewer than 2^31 elements here
    int choff[8];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int e = 0; e < 4; ++e) choff[4 * h + e] = (4 * gw + 16 * h + e) * hw;
    for (int pt = cid + pipe * num_clusters; pt < num_pt; pt += P * num_clusters) {
      // m-block 2*pt + rank; past the last m-block every row is invalid and
      // the window is zeros (the leader's MMA still reads it).
      const int v0 = (2 * pt + static_cast<int>(rank)) * kConvBM;
      int rbase[kRowsPerLane];
      int rih[kRowsPerLane], riw[kRowsPerLane];
      bool rvalid[kRowsPerLane];
#pragma unroll
      for (int i = 0; i < kRowsPerLane; ++i) {
        const int r = lane + 32 * i;
        const int v = v0 + r;
        rvalid[i] = r < win_rows && v < p.Mv;
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
          float vals[kRowsPerLane][2][4];
          const int dh = kh * p.dh;
          const int woff = cb * kConvBK * hw + dh * p.W;
#pragma unroll
          for (int i = 0; i < kRowsPerLane; ++i) {
            const int ih = rih[i] + dh, iw = riw[i];
            const bool ok = rvalid[i] && static_cast<unsigned>(ih) < static_cast<unsigned>(p.H) &&
                            static_cast<unsigned>(iw) < static_cast<unsigned>(p.W);
            const int off = rbase[i] + woff;
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
              for (int e = 0; e < 4; ++e)
                vals[i][h][e] = ok ? __ldg(p.x + (off + choff[4 * h + e])) : 0.0f;
          }
          if (!mbar_wait_pair(&we[ws], wph ^ 1u, abort_flag, peer_abort, p.status,
                              kStatusTimeoutProducer))
            goto role_done;
          uint8_t *slot = base + ws * kPairWinSlotBytes;
#pragma unroll
          for (int i = 0; i < kRowsPerLane; ++i) {
            const int r = lane + 32 * i;
            if (r >= win_rows) continue;
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
              *reinterpret_cast<float4 *>(slot + kPairWinBytes + off) = lo4;
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(leader_bar(&wr[ws]));
          if (++ws == WS) {
            ws = 0;
            wph ^= 1u;
          }
        }
      }
    }
  } else {
    // ---------------- epilogue (4 warps, one per TMEM lane quadrant) ----------------
    const int quad = warp & 3;
    const int et = threadIdx.x - kPairFirstEpi * 32;  // 0..127
    griddep_wait();  // the epilogue constants come from the preparation kernel
    int j = 0;
    for (int pt = cid; pt < num_pt; pt += num_clusters, ++j) {
      const int pipe = j % P;
      const int jj = j / P;
      const int acc = pipe * 2 + (jj & 1);
      const uint32_t acc_phase = (jj >> 1) & 1;
      const int mb = 2 * pt + static_cast<int>(rank);
      if (!conv_epilogue_tile<kPairBNC, kAct, true>(p, tmem_base + acc * kPairAccCols, quad,
                                                    lane, et, mb, 0, ep_s, ep_beta_s,
                                                    &acc_full[acc], acc_phase, abort_flag,
                                                    peer_abort))
        break;
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(leader_bar(&acc_empty[acc]));
    }
  }

role_done:
  __syncthreads();
  cluster_sync();  // no remote arrival, copy or MMA into either CTA is left
  if (warp == kPairFirstMma) {
    tc_fence_after_sync();
    tmem_dealloc_pair(tmem_base, kPairTmemCols);
  }
}

namespace {

// Clusters of two that fit on the device at once (cached per device and
// kernel): the grid of this persistent kernel never exceeds them.
int max_pair_clusters(const void *kernel, cudaLaunchConfig_t cfg) {
  static std::mutex mu;
  static std::map<std::pair<int, const void *>, int> cache;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find({dev, kernel});
  if (it != cache.end()) return it->second;
  int n = 0;
  cfg.gridDim = dim3(static_cast<unsigned>(sm_count() & ~1));
  if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  cache[{dev, kernel}] = n;
  return n;
}

template <int kAct>
int launch_pair(cudaStream_t s, const CUtensorMap &mwa, const CUtensorMap &mwb,
                const ConvParams &prm, int win_rows, bool after_prep) {
  auto kernel = conv_window_pair_kernel<kAct>;
  const void *fn = reinterpret_cast<const void *>(kernel);
  int rc = ensure_dynamic_smem(fn, kPairSmemBytes);
  if (rc) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kPairThreads);
  cfg.dynamicSmemBytes = kPairSmemBytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int fit = max_pair_clusters(fn, cfg);
  if (fit <= 0) return kErrUnsupported;
  const int num_pt = (prm.m_blocks + 1) / 2;
  const int clusters = num_pt < fit ? num_pt : fit;
  cfg.gridDim = dim3(static_cast<unsigned>(2 * clusters));
  // Overlap with the weight preparation launched just before: the gather
  // warps only read x; the slab producer and the epilogue wait for it.
  cfg.numAttrs = after_prep ? 2 : 1;
  count_launch();
  return map_cuda_error(cudaLaunchKernelEx(&cfg, kernel, mwa, mwb, prm, win_rows));
}

}  // namespace

bool conv_window_pair_supported(const ConvParams &p, int n_img, int bnc, int64_t n_blocks) {
  return bnc == kPairBNC && n_blocks == 1 && p.sw == 1 && p.KW > 1 &&
         (p.KW - 1) * p.dw <= kPairMaxExtra && conv_window_gather_supported(p, n_img);
}

int launch_conv_window_pair(cudaStream_t s, const float *wsplit, int64_t kp, ConvParams prm,
                            int n_img, bool after_prep) {
  if (!conv_window_pair_supported(prm, n_img, kPairBNC, 1) || !prm.x) return kErrUnsupported;
  int wv;
  int64_t mv;
  conv_window_rows(prm, &wv, &mv);
  prm.Wv = wv;
  prm.Mv = static_cast<int>(mv);
  prm.m_blocks = static_cast<int>(ceil_div(mv, kConvBM));
  prm.stall_us = take_armed_stall(NPLK_DEBUG_CONV_WINDOW);
  const int win_rows = kConvBM + (prm.KW - 1) * prm.dw;
  // Split weights: rows [W_hi (64); W_lo (64)] of one output-channel block,
  // kp columns. Box A: a CTA's 64-row half of [W_hi; W_lo]; box B: its 32
  // rows of W_hi.
  CUtensorMap mwa, mwb;
  int rc = encode_tmap_2d_f32_sw128(&mwa, wsplit, kp, 2 * kPairBNC, kp * 4, kConvBK,
                                    kPairSlabRowsA);
  if (rc) return rc;
  rc = encode_tmap_2d_f32_sw128(&mwb, wsplit, kp, 2 * kPairBNC, kp * 4, kConvBK, kPairSlabRowsB);
  if (rc) return rc;
  if (prm.act == 0) return launch_pair<kEpiActNone>(s, mwa, mwb, prm, win_rows, after_prep);
  if (prm.act == 1) return launch_pair<kEpiActRelu>(s, mwa, mwb, prm, win_rows, after_prep);
  return launch_pair<kEpiActAny>(s, mwa, mwb, prm, win_rows, after_prep);
}

}  // namespace nplk
