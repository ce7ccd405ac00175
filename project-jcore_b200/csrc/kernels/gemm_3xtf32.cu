// K1: fp32 GEMM on the sm_100a tensor cores with 3xTF32 split precision.
//
// C = act(alpha * A @ B + beta * C + bias), the arithmetic the reference
// obtains from cblas_sgemm behind npl_matmul (advanced/neural_layer/src/
// npl_tensor_ops.cpp:217-311 -> composite/mkernel_interface/src/
// mil_gemm.cpp:290-316).
//
// Pipeline (one persistent CTA per SM, 192 threads):
//   1. split kernels (split_tf32.cu) write A and B^T as tf32 hi/lo pairs in a
//      blocked, zero-padded, K-major layout:
//        A': [m_blocks][2][128][Kp]   (hi rows, then lo rows, per 128-row block)
//        B': [n_blocks][2][BN][Kp]    (B transposed: rows are output columns)
//   2. warp 0 streams 32-wide K slabs of A' and B' into a ring of shared-memory
//      stages with TMA (128-byte swizzle, no multicast);
//   3. warp 1 issues tcgen05.mma kind::tf32 into a TMEM accumulator of 2*BN
//      columns: MMA(A_hi, [B_hi;B_lo]) with N = 2*BN gives A_hi*B_hi in the
//      first BN columns and A_hi*B_lo in the second; MMA(A_lo, B_hi) with
//      N = BN adds A_lo*B_hi into the first BN columns;
//   4. warps 2-5 drain the (double-buffered) accumulator: C = alpha*(D[:, :BN]
//      + D[:, BN:]) + beta*C + bias, activation, store.
#include <cuda_runtime.h>
#include <math_constants.h>

#include <algorithm>
#include <type_traits>
#include <vector>

#include "nplk_device.cuh"
#include "nplk_host.h"
#include "ptx_sm100.cuh"
#include "tuning_cache.h"

namespace nplk {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 32;
constexpr int kGemmThreads = 192;
// Fused-exchange staging per epilogue warp: 32 rows x 32 columns, row pitch 36
// floats (16-byte aligned rows, conflict-free float4 access); four warps.
constexpr int kEpiStagePitch = 36;
constexpr int kEpiStageBytes = 4 * 32 * kEpiStagePitch * 4;

template <int BN>
struct GemmTraits {
  static constexpr int kStages = BN == 128 ? 3 : 4;
  static constexpr int kAStageBytes = 2 * kGemmBM * kGemmBK * 4;  // hi + lo, 32 KB
  static constexpr int kBStageBytes = 2 * BN * kGemmBK * 4;       // hi + lo
  static constexpr int kStageBytes = kAStageBytes + kBStageBytes;
  static constexpr int kAccCols = 2 * BN;
  static constexpr int kTmemCols = 2 * kAccCols;  // two accumulators
  static constexpr int kBarrierBytes = 256;
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kBarrierBytes + kEpiStageBytes;
  // The TMA-store exchange: barriers in a 1 KB slot, then the 1024-byte
  // aligned staging boxes (4 epilogue warps x 2 boxes x 4 KB).
  static constexpr int kSmemBytesTma = 1024 + kStages * kStageBytes + 1024 + 32768;
};

struct GemmParams {
  int M, N, K;
  int m_blocks, n_blocks, k_blocks;
  float alpha, beta;
  float *C;
  int64_t ldc;
  const float *bias;
  int act;
  float act_alpha;
  int one_pass;       // bit 0: one TF32 pass; bits 8..15: K slices per tile (gemm_k_slices)
  uint32_t stall_us;  // fault injection: 0 except on an armed launch (injected_stall)
  int *status;
};

__device__ __forceinline__ bool gemm_one_pass(const GemmParams &p) { return (p.one_pass & 1) != 0; }

// Split-K: each tile's K range is cut into this many slices, each a separate
// work unit whose epilogue adds alpha * (its partial product) into C, which
// the host zeroed (beta 0, no bias, no activation). Two slices added to zero
// give the same sum in either order, so the result stays deterministic.
__device__ __forceinline__ int gemm_k_slices(const GemmParams &p) {
  const int s = (p.one_pass >> 8) & 255;
  return s > 1 ? s : 1;
}

// nplk_gemm_allgather: every output is stored to each of dst[0..n_dst) at
// column dst_col + col (row pitch GemmParams::ldc). A kernel parameter of the
// fused instantiation only: the plain GEMM's parameter block keeps its size
// (with these 88 bytes in it the 1024^3 GEMM kernel ran 45 us against 37).
struct GemmDst {
  float *dst[8];
  int n_dst;
  int dst_vec;  // 16-byte stores allowed into every dst
  int rot;      // first destination this rank visits (then in turn, each warp offset by one)
  int multimem; // dst[0] is a multicast address: one multimem.st reaches every rank's C
  int64_t dst_col;
};
struct GemmNoDst {};

// nplk_gemm_allgather, TMA-store form: map[d] is destination d's block of
// columns [dst_col, dst_col + N_local) as a [M][N_local] fp32 tensor (row pitch
// ldc, 32 x 32 boxes, 128-byte swizzle). Each epilogue warp stages its 32 x 32
// piece of the accumulator in shared memory and one lane hands it to the TMA
// unit once per destination, so the NVLink writes drain asynchronously while
// the warp goes on to the next piece (two staging boxes per warp).
struct alignas(64) GemmDstTma {
  CUtensorMap map[8];
  int n_dst;
  int rot;
};

// Tile order: groups of 8 M-blocks sweep all N-blocks, so the CTAs resident at
// one time share A row-blocks and B column-blocks in L2.
__device__ __forceinline__ void gemm_tile_coords(int tile, int m_blocks, int n_blocks, int &mb,
                                                 int &nb) {
  constexpr int kGroup = 8;
  const int per_group = kGroup * n_blocks;
  const int group = tile / per_group;
  const int first_m = group * kGroup;
  const int gsize = min(m_blocks - first_m, kGroup);
  const int local = tile - group * per_group;
  mb = first_m + local % gsize;
  nb = local / gsize;
}

// Drains one accumulator tile row (this thread's row r of the tile) from
// TMEM: C = alpha*(D[:, :BN] + D[:, BN:]) + beta*C + bias, activation, store.
template <int BN, bool kFused, class Dst>
__device__ __forceinline__ void gemm_epilogue_tile(const GemmParams &p, const Dst &pd,
                                                   uint32_t t_row, int r, int nb, bool vec_ok,
                                                   float *stg, int &box_seq) {
#pragma unroll 1
  for (int c0 = 0; c0 < BN; c0 += 32) {
    const int col0 = nb * BN + c0;
    // The row's C values for beta, loaded before the accumulator is read so
    // that their latency overlaps the TMEM load, and all eight in flight at
    // once (loads placed after a store to C would each wait for it).
    const bool vec_chunk = !kFused && vec_ok && r < p.M && col0 + 32 <= p.N;
    float4 cv[8];
    if (vec_chunk && p.beta != 0.0f) {
      const float4 *src = reinterpret_cast<const float4 *>(p.C + static_cast<int64_t>(r) * p.ldc +
                                                           col0);
#pragma unroll
      for (int q = 0; q < 8; ++q) cv[q] = src[q];
    }
    uint32_t v[32], w[32];
    tmem_ld32(t_row + c0, v);
    if (!gemm_one_pass(p)) {
      tmem_ld32(t_row + BN + c0, w);
      tmem_wait_ld2(v, w);
    } else {
      tmem_wait_ld(v);
#pragma unroll
      for (int j = 0; j < 32; ++j) w[j] = 0u;
    }
    if constexpr (std::is_same<Dst, GemmDstTma>::value) {
      // Fused exchange through the TMA unit: bias and activation, the warp's
      // 32 x 32 piece into a staging box (rows of 128 bytes, 16-byte chunk j
      // of row i at chunk j ^ (i mod 8): the map's 128-byte swizzle, and
      // conflict-free for each quarter-warp's stores), then one tensor store
      // per destination. Rows and columns past the block are clipped by TMA.
      const int lane = threadIdx.x & 31;
      if (col0 < p.N) {
        float *box = stg + (box_seq & 1) * 1024;
        if (lane == 0) bulk_wait_group_read<1>();  // this box's previous stores have read it
        __syncwarp();
        float out[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          float o = p.alpha * (__uint_as_float(v[j]) + __uint_as_float(w[j]));
          if (p.bias && col0 + j < p.N) o += p.bias[col0 + j];
          out[j] = apply_act(o, p.act, p.act_alpha);
        }
        uint8_t *row = reinterpret_cast<uint8_t *>(box) + lane * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q)
          *reinterpret_cast<float4 *>(row + ((q ^ (lane & 7)) << 4)) =
              make_float4(out[4 * q], out[4 * q + 1], out[4 * q + 2], out[4 * q + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          int d = pd.rot + (threadIdx.x >> 5);
          while (d >= pd.n_dst) d -= pd.n_dst;
          for (int i = 0; i < pd.n_dst; ++i) {
            tma_store_2d(&pd.map[d], box, col0, r - lane);
            if (++d == pd.n_dst) d = 0;
          }
          bulk_commit_group();
        }
        ++box_seq;
      }
    } else if constexpr (kFused) {
      // Fused exchange: bias and activation, then the same values to every
      // destination buffer (this GPU's and the peers' over NVLink). The warp's
      // 32 x 32 block goes through shared memory so that each store
      // instruction writes four whole 128-byte row segments instead of 32
      // scattered 16-byte pieces (one row per lane).
      const int lane = threadIdx.x & 31;
      if (col0 < p.N) {
        float out[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          float o = p.alpha * (__uint_as_float(v[j]) + __uint_as_float(w[j]));
          if (p.bias && col0 + j < p.N) o += p.bias[col0 + j];
          out[j] = apply_act(o, p.act, p.act_alpha);
        }
        float4 *s4 = reinterpret_cast<float4 *>(stg + lane * kEpiStagePitch);
#pragma unroll
        for (int q = 0; q < 8; ++q)
          s4[q] = make_float4(out[4 * q], out[4 * q + 1], out[4 * q + 2], out[4 * q + 3]);
      }
      __syncwarp();
      if (col0 < p.N) {
        const int r0 = r - lane;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int rr = 4 * i + (lane >> 3);
          const int col = col0 + 4 * (lane & 7);
          const int row = r0 + rr;
          const float4 val = *reinterpret_cast<const float4 *>(stg + rr * kEpiStagePitch +
                                                               4 * (lane & 7));
          if (row < p.M && col < p.N) {
            const int64_t off = static_cast<int64_t>(row) * p.ldc + pd.dst_col + col;
            // Destinations in turn from a start that differs per rank and per
            // warp, so the ranks' stores spread over all peers' links instead
            // of all converging on the same peer at the same time.
            int d = pd.rot + (threadIdx.x >> 5);
            while (d >= pd.n_dst) d -= pd.n_dst;
            if (pd.multimem) {
              // Written once; NVSwitch delivers it to every rank's C (the
              // host admits this form only with 16-byte aligned whole rows).
              multimem_st_v4(pd.dst[0] + off, val);
            } else if (pd.dst_vec && col + 4 <= p.N) {
              for (int i = 0; i < pd.n_dst; ++i) {
                *reinterpret_cast<float4 *>(pd.dst[d] + off) = val;
                if (++d == pd.n_dst) d = 0;
              }
            } else {
              const float e[4] = {val.x, val.y, val.z, val.w};
              for (int i = 0; i < pd.n_dst; ++i) {
                for (int k = 0; k < 4 && col + k < p.N; ++k) pd.dst[d][off + k] = e[k];
                if (++d == pd.n_dst) d = 0;
              }
            }
          }
        }
      }
      __syncwarp();  // the next chunk rewrites the staging block
    } else if (r < p.M && col0 < p.N) {
      float *crow = p.C + static_cast<int64_t>(r) * p.ldc;
      float out[32];
#pragma unroll
      for (int j = 0; j < 32; ++j)
        out[j] = p.alpha * (__uint_as_float(v[j]) + __uint_as_float(w[j]));
      if (gemm_k_slices(p) > 1) {
        // a K slice's partial product, added into the zeroed C
        if (vec_ok && col0 + 32 <= p.N) {
          float4 *dst = reinterpret_cast<float4 *>(crow + col0);
#pragma unroll
          for (int q = 0; q < 8; ++q)
            atomicAdd(dst + q, make_float4(out[4 * q], out[4 * q + 1], out[4 * q + 2],
                                           out[4 * q + 3]));
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (col0 + j < p.N) atomicAdd(crow + col0 + j, out[j]);
        }
      } else if (vec_chunk) {
        // every load (C, bias) before the first store
        if (p.beta != 0.0f) {
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            out[4 * q] += p.beta * cv[q].x;
            out[4 * q + 1] += p.beta * cv[q].y;
            out[4 * q + 2] += p.beta * cv[q].z;
            out[4 * q + 3] += p.beta * cv[q].w;
          }
        }
        if (p.bias) {
#pragma unroll
          for (int j = 0; j < 32; ++j) out[j] += p.bias[col0 + j];
        }
        float4 *dst = reinterpret_cast<float4 *>(crow + col0);
#pragma unroll
        for (int q = 0; q < 8; ++q)
          dst[q] = make_float4(apply_act(out[4 * q], p.act, p.act_alpha),
                               apply_act(out[4 * q + 1], p.act, p.act_alpha),
                               apply_act(out[4 * q + 2], p.act, p.act_alpha),
                               apply_act(out[4 * q + 3], p.act, p.act_alpha));
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int col = col0 + j;
          if (col < p.N) {
            float o = out[j];
            if (p.beta != 0.0f) o += p.beta * crow[col];
            if (p.bias) o += p.bias[col];
            crow[col] = apply_act(o, p.act, p.act_alpha);
          }
        }
      }
    }
  }
}

// kFused: the fused-exchange epilogue (nplk_gemm_allgather); a separate
// instantiation keeps the plain GEMM's code as it was.
template <int BN, bool kFused, class Dst>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_3xtf32_kernel(const __grid_constant__ CUtensorMap map_a,
                       const __grid_constant__ CUtensorMap map_b, const GemmParams p,
                       const __grid_constant__ Dst pd) {
  using T = GemmTraits<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align_smem_1024(smem_raw);
  uint8_t *smem_a = smem;
  uint8_t *smem_b = smem + T::kStages * T::kAStageBytes;
  uint64_t *full = reinterpret_cast<uint64_t *>(smem_b + T::kStages * T::kBStageBytes);
  uint64_t *empty = full + T::kStages;
  uint64_t *acc_full = empty + T::kStages;
  uint64_t *acc_empty = acc_full + 2;
  uint64_t *never = acc_empty + 2;  // never arrived on (injected_stall)
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(never + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < T::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    mbar_init(never, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, T::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;

  const int num_tiles = p.m_blocks * p.n_blocks;
  // Work unit u: tile u / KS, K slice u % KS (k-blocks [ks * kbp, (ks + 1) * kbp)).
  const int KS = gemm_k_slices(p);
  const int kbp = (p.k_blocks + KS - 1) / KS;
  const int num_units = num_tiles * KS;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      griddep_wait();  // the split operands come from the kernels just before
      int stage = 0;
      uint32_t phase = 0;
      uint32_t pending = 0;  // stages that received a copy, with its phase
      uint32_t pending_phase = 0;
      for (int unit = blockIdx.x; unit < num_units; unit += gridDim.x) {
        const int tile = unit / KS;
        const int kb0 = (unit - tile * KS) * kbp;
        const int kb1 = kb0 + kbp < p.k_blocks ? kb0 + kbp : p.k_blocks;
        int mb, nb;
        gemm_tile_coords(tile, p.m_blocks, p.n_blocks, mb, nb);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.status,
                         kStatusTimeoutProducer))
            goto producer_done;
          mbar_arrive_expect_tx(&full[stage], T::kStageBytes);
          tma_load_2d(&map_a, &full[stage], smem_a + stage * T::kAStageBytes, kb * kGemmBK,
                      mb * 2 * kGemmBM);
          tma_load_2d(&map_b, &full[stage], smem_b + stage * T::kBStageBytes, kb * kGemmBK,
                      nb * 2 * BN);
          pending |= 1u << stage;
          pending_phase = (pending_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == T::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    producer_done:
      // Let the last copy into each stage land before the CTA can exit (they
      // already have unless the CTA aborted).
      for (int s2 = 0; s2 < T::kStages; ++s2)
        if ((pending >> s2) & 1u) mbar_drain(&full[s2], (pending_phase >> s2) & 1u);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc_2n = umma_idesc_tf32(kGemmBM, 2 * BN);
      const uint32_t idesc_n = umma_idesc_tf32(kGemmBM, BN);
      const uint64_t a_desc0 = umma_desc_sw128(smem_u32(smem_a));
      const uint64_t b_desc0 = umma_desc_sw128(smem_u32(smem_b));
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      const bool go = injected_stall(never, p.stall_us, abort_flag, p.status);
      for (int unit = blockIdx.x; go && unit < num_units; unit += gridDim.x, ++local) {
        const int tile = unit / KS;
        const int kb0 = (unit - tile * KS) * kbp;
        const int kb1 = kb0 + kbp < p.k_blocks ? kb0 + kbp : p.k_blocks;
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, abort_flag, p.status,
                       kStatusTimeoutAccFree))
          break;
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * T::kAccCols;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.status, kStatusTimeoutMma))
            goto mma_done;
          tc_fence_after_sync();
          // Descriptors of the stage; a 32-byte step along K adds 2 to the
          // start-address field (address >> 4).
          const uint64_t a_desc = a_desc0 + static_cast<uint64_t>(stage * (T::kAStageBytes >> 4));
          const uint64_t b_desc = b_desc0 + static_cast<uint64_t>(stage * (T::kBStageBytes >> 4));
          constexpr uint64_t kLoOff = (kGemmBM * 128) >> 4;
          if (gemm_one_pass(p)) {
#pragma unroll
            for (int kk = 0; kk < kGemmBK / 8; ++kk)
              mma_tf32_ss(d_tmem, a_desc + 2 * kk, b_desc + 2 * kk, idesc_n,
                          (kb > kb0 || kk > 0) ? 1u : 0u);
          } else {
#pragma unroll
            for (int kk = 0; kk < kGemmBK / 8; ++kk) {
              mma_tf32_ss(d_tmem, a_desc + 2 * kk, b_desc + 2 * kk, idesc_2n,
                          (kb > kb0 || kk > 0) ? 1u : 0u);
              mma_tf32_ss(d_tmem, a_desc + kLoOff + 2 * kk, b_desc + 2 * kk, idesc_n, 1u);
            }
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
    // ---------------- epilogue (warps 2..5) ----------------
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int row_in_tile = quad * 32 + lane;
    constexpr bool kTmaDst = std::is_same<Dst, GemmDstTma>::value;
    float *stg = kTmaDst ? reinterpret_cast<float *>(smem_b + T::kStages * T::kBStageBytes + 1024) +
                               (warp - 2) * 2 * 1024
                         : reinterpret_cast<float *>(smem_b + T::kStages * T::kBStageBytes +
                                                     T::kBarrierBytes) +
                               (warp - 2) * 32 * kEpiStagePitch;
    const bool vec_ok = (p.N % 4 == 0) && (p.ldc % 4 == 0) &&
                        ((reinterpret_cast<uintptr_t>(p.C) & 15u) == 0);
    int local = 0;
    int box_seq = 0;
    for (int unit = blockIdx.x; unit < num_units; unit += gridDim.x, ++local) {
      const int tile = unit / KS;
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&acc_full[acc], acc_phase, abort_flag, p.status, kStatusTimeoutEpilogue))
        break;
      tc_fence_after_sync();
      int mb, nb;
      gemm_tile_coords(tile, p.m_blocks, p.n_blocks, mb, nb);
      const int r = mb * kGemmBM + row_in_tile;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                             static_cast<uint32_t>(acc * T::kAccCols);
      gemm_epilogue_tile<BN, kFused>(p, pd, t_row, r, nb, vec_ok, stg, box_seq);
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
    }
    // Every tensor store of this warp complete before the CTA exits.
    if (kTmaDst && lane == 0) bulk_wait_group<0>();
    if constexpr (std::is_same<Dst, GemmDst>::value) {
      if (pd.multimem) fence_multimem_release();
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, T::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// Raw-operand form: A (row-major [M][K], a K-major operand) and B (row-major
// [K][N], read as an MN-major operand) are loaded as they are by TMA; the
// tensor core truncates them to tf32 for the hi parts, and converter warps
// form the lo parts (x - trunc(x), 0 for +-inf) in shared memory next to
// them. No split kernels and no workspace; half the operand bytes of the
// split form cross L2 per tile, but forming lo costs shared-memory bandwidth,
// which bounds this GEMM, so the split form stays the default when a
// workspace is given.
//   warp 0      TMA producer: A box [128 rows][32 K] (128-byte swizzle), B
//               boxes [32 K][32 N] (128-byte swizzle of 32-byte atoms, the
//               layout MN-major tf32 operands need);
//   warp 1      MMA issuer:   MMA(A_raw, [B_raw | B_lo]) N = 2*BN, then
//                             MMA(A_lo, B_raw) N = BN;
//   warps 2-5   epilogue (gemm_epilogue_tile);
//   warps 6-9   converters: A_lo and B_lo, elementwise over the swizzled tiles
//               (raw and lo tiles share one layout, so no swizzle arithmetic).
// ---------------------------------------------------------------------------
constexpr int kRawConvWarps = 4;
constexpr int kRawThreads = kGemmThreads + kRawConvWarps * 32;

template <int BN>
struct RawGemmTraits {
  static constexpr int kStages = BN == 128 ? 3 : 4;
  static constexpr int kAHalf = kGemmBM * kGemmBK * 4;  // one A tile, 16 KB
  static constexpr int kBAtom = 32 * kGemmBK * 4;       // [32 K][32 N] B atom, 4 KB
  static constexpr int kBHalf = (BN / 32) * kBAtom;     // one B tile
  // Stage: A_raw, A_lo, B_raw atoms, B_lo atoms (1024-byte aligned pieces).
  static constexpr int kStageBytes = 2 * kAHalf + 2 * kBHalf;
  static constexpr int kTxBytes = kAHalf + kBHalf;  // what TMA writes per stage
  static constexpr int kAccCols = 2 * BN;
  static constexpr int kTmemCols = 2 * kAccCols;
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + 256 + kEpiStageBytes;
};

__device__ __forceinline__ float tf32_lo_trunc(float x) {
  const float hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
  return fabsf(x) == CUDART_INF_F ? 0.0f : x - hi;
}

template <int BN, bool kFused, class Dst>
__global__ void __launch_bounds__(kRawThreads, 1)
    gemm_3xtf32_raw_kernel(const __grid_constant__ CUtensorMap map_a,
                           const __grid_constant__ CUtensorMap map_b, const GemmParams p,
                           const __grid_constant__ Dst pd) {
  using T = RawGemmTraits<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align_smem_1024(smem_raw);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + T::kStages * T::kStageBytes);
  uint64_t *lo_ready = full + T::kStages;
  uint64_t *empty = lo_ready + T::kStages;
  uint64_t *acc_full = empty + T::kStages;
  uint64_t *acc_empty = acc_full + 2;
  uint64_t *never = acc_empty + 2;  // never arrived on (injected_stall)
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(never + 1);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < T::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&lo_ready[s], kRawConvWarps);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    mbar_init(never, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, T::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem_base = *tmem_slot;
  const int num_tiles = p.m_blocks * p.n_blocks;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t pending = 0;  // stages that received a copy, with its phase
      uint32_t pending_phase = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
        int mb, nb;
        gemm_tile_coords(tile, p.m_blocks, p.n_blocks, mb, nb);
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, abort_flag, p.status,
                         kStatusTimeoutProducer))
            goto producer_done;
          uint8_t *st = smem + stage * T::kStageBytes;
          mbar_arrive_expect_tx(&full[stage], T::kTxBytes);
          tma_load_2d(&map_a, &full[stage], st, kb * kGemmBK, mb * kGemmBM);
#pragma unroll
          for (int j = 0; j < BN / 32; ++j)
            tma_load_2d(&map_b, &full[stage], st + 2 * T::kAHalf + j * T::kBAtom,
                        nb * BN + 32 * j, kb * kGemmBK);
          pending |= 1u << stage;
          pending_phase = (pending_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == T::kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    producer_done:
      // Let the last copy into each stage land before the CTA can exit (they
      // already have unless the CTA aborted).
      for (int s2 = 0; s2 < T::kStages; ++s2)
        if ((pending >> s2) & 1u) mbar_drain(&full[s2], (pending_phase >> s2) & 1u);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc_2n = umma_idesc_tf32(kGemmBM, 2 * BN) | kUmmaIdescBMajorMN;
      const uint32_t idesc_n = umma_idesc_tf32(kGemmBM, BN) | kUmmaIdescBMajorMN;
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      const bool go = injected_stall(never, p.stall_us, abort_flag, p.status);
      for (int tile = blockIdx.x; go && tile < num_tiles; tile += gridDim.x, ++local) {
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, abort_flag, p.status,
                       kStatusTimeoutAccFree))
          break;
        tc_fence_after_sync();
        const uint32_t d_tmem = tmem_base + acc * T::kAccCols;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&lo_ready[stage], phase, abort_flag, p.status, kStatusTimeoutMma))
            goto mma_done;
          tc_fence_after_sync();
          const uint32_t st = smem_u32(smem + stage * T::kStageBytes);
          // A (K-major): a K = 8 step is 32 bytes (+2 in the address field).
          // B (MN-major, 32-byte-atom swizzle): a K = 8 step is 8 rows of
          // 128 bytes (+64); the B_lo atoms follow the B_raw atoms at the same
          // 4 KB stride, so one descriptor with N = 2*BN covers [B_raw | B_lo].
          const uint64_t a_raw = umma_desc_sw128(st);
          const uint64_t a_lo = umma_desc_sw128(st + T::kAHalf);
          const uint64_t b = umma_desc_mn_sw128_32b(st + 2 * T::kAHalf, T::kBAtom);
          if (gemm_one_pass(p)) {
#pragma unroll
            for (int kk = 0; kk < kGemmBK / 8; ++kk)
              mma_tf32_ss(d_tmem, a_raw + 2 * kk, b + 64 * kk, idesc_n,
                          (kb > 0 || kk > 0) ? 1u : 0u);
          } else {
#pragma unroll
            for (int kk = 0; kk < kGemmBK / 8; ++kk) {
              mma_tf32_ss(d_tmem, a_raw + 2 * kk, b + 64 * kk, idesc_2n,
                          (kb > 0 || kk > 0) ? 1u : 0u);
              mma_tf32_ss(d_tmem, a_lo + 2 * kk, b + 64 * kk, idesc_n, 1u);
            }
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
  } else if (warp < 6) {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quad = warp & 3;
    const int row_in_tile = quad * 32 + lane;
    float *stg = reinterpret_cast<float *>(smem + T::kStages * T::kStageBytes + 256) +
                 (warp - 2) * 32 * kEpiStagePitch;
    const bool vec_ok = (p.N % 4 == 0) && (p.ldc % 4 == 0) &&
                        ((reinterpret_cast<uintptr_t>(p.C) & 15u) == 0);
    int local = 0;
    int box_seq = 0;  // (TMA-store boxes; unused by this form)
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      if (!mbar_wait(&acc_full[acc], acc_phase, abort_flag, p.status, kStatusTimeoutEpilogue))
        break;
      tc_fence_after_sync();
      int mb, nb;
      gemm_tile_coords(tile, p.m_blocks, p.n_blocks, mb, nb);
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quad * 32) << 16) +
                             static_cast<uint32_t>(acc * T::kAccCols);
      gemm_epilogue_tile<BN, kFused>(p, pd, t_row, mb * kGemmBM + row_in_tile, nb, vec_ok,
                                     stg, box_seq);
      tc_fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
    }
    if constexpr (std::is_same<Dst, GemmDst>::value) {
      if (pd.multimem) fence_multimem_release();
    }
  } else {
    // ---------------- converters (warps 6..9) ----------------
    const int ct = threadIdx.x - 6 * 32;  // 0..127
    int stage = 0;
    uint32_t phase = 0;
    const int items = (num_tiles > static_cast<int>(blockIdx.x)
                           ? (num_tiles - 1 - static_cast<int>(blockIdx.x)) / gridDim.x + 1
                           : 0) *
                      p.k_blocks;
    for (int it = 0; it < items; ++it) {
      if (!mbar_wait(&full[stage], phase, abort_flag, p.status, kStatusTimeoutStage)) break;
      uint8_t *st = smem + stage * T::kStageBytes;
      if (!gemm_one_pass(p)) {
        const float4 *a4 = reinterpret_cast<const float4 *>(st);
        float4 *al4 = reinterpret_cast<float4 *>(st + T::kAHalf);
#pragma unroll 4
        for (int i = ct; i < T::kAHalf / 16; i += kRawConvWarps * 32) {
          const float4 v = a4[i];
          al4[i] = make_float4(tf32_lo_trunc(v.x), tf32_lo_trunc(v.y), tf32_lo_trunc(v.z),
                               tf32_lo_trunc(v.w));
        }
        const float4 *b4 = reinterpret_cast<const float4 *>(st + 2 * T::kAHalf);
        float4 *bl4 = reinterpret_cast<float4 *>(st + 2 * T::kAHalf + T::kBHalf);
#pragma unroll 4
        for (int i = ct; i < T::kBHalf / 16; i += kRawConvWarps * 32) {
          const float4 v = b4[i];
          bl4[i] = make_float4(tf32_lo_trunc(v.x), tf32_lo_trunc(v.y), tf32_lo_trunc(v.z),
                               tf32_lo_trunc(v.w));
        }
        fence_proxy_async_smem();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&lo_ready[stage]);
      if (++stage == T::kStages) {
        stage = 0;
        phase ^= 1u;
      }
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after_sync();
    tmem_dealloc(tmem_base, T::kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// host launcher
// ---------------------------------------------------------------------------
namespace {

struct GemmPlan {
  int bn;
  int ks;  // K slices per tile (split-K; only for calls gemm_run finds eligible)
  int64_t m_blocks, n_blocks, kp;
  size_t a_bytes, b_bytes;
  size_t b_bytes_max;  // B' for either tile width (the workspace size covers both)
};

// Tile configurations as the tile-configuration cache stores them: the tile
// width BN, plus 1000 per extra K slice (1128 = 128 wide, K in two slices).
constexpr int kGemmCfgSplitK = 1128;
bool valid_gemm_cfg(int c) { return c == 64 || c == 128 || c == kGemmCfgSplitK; }

// Configuration: force_cfg when valid, else the tile-configuration cache's
// entry for the shape, else 128-wide tiles when they fill the SMs, else, when
// two K slices of 128-wide tiles still fit on the SMs and K has at least 16
// k-blocks, those (split-K), else 64-wide tiles.
GemmPlan plan_gemm(int64_t M, int64_t N, int64_t K, int force_cfg = 0) {
  GemmPlan g{};
  g.m_blocks = ceil_div(M, kGemmBM);
  g.kp = ceil_div(K, kGemmBK) * kGemmBK;
  const int64_t tiles128 = g.m_blocks * ceil_div(N, 128);
  int cfg = tiles128 >= sm_count() ? 128
            : (2 * tiles128 <= sm_count() && g.kp / kGemmBK >= 16) ? kGemmCfgSplitK
                                                                  : 64;
  int cached = 0;
  if (valid_gemm_cfg(force_cfg))
    cfg = force_cfg;
  else if (!tuning_cache_empty() && tuning_lookup(tuning_key_gemm(M, N, K), &cached) &&
           valid_gemm_cfg(cached))
    cfg = cached;
  g.bn = cfg % 1000;
  g.ks = cfg / 1000 + 1;
  if (g.ks > 1 && g.kp / kGemmBK < 2 * g.ks) g.ks = 1;  // every slice keeps >= 2 k-blocks
  g.n_blocks = ceil_div(N, g.bn);
  g.a_bytes = align_up(static_cast<size_t>(g.m_blocks) * 2 * kGemmBM * g.kp * 4, 256);
  g.b_bytes = align_up(static_cast<size_t>(g.n_blocks) * 2 * g.bn * g.kp * 4, 256);
  g.b_bytes_max = align_up(static_cast<size_t>(ceil_div(N, 128)) * 2 * 128 * g.kp * 4, 256);
  return g;
}

template <int BN>
int launch_gemm(cudaStream_t stream, const GemmPlan &g, const float *a_split,
                const float *b_split, const GemmParams &prm, const GemmDst *pd,
                const GemmDstTma *pt) {
  using T = GemmTraits<BN>;
  CUtensorMap map_a, map_b;
  int rc = encode_tmap_2d_f32_sw128(&map_a, a_split, g.kp, g.m_blocks * 2 * kGemmBM, g.kp * 4,
                                    kGemmBK, 2 * kGemmBM);
  if (rc) return rc;
  rc = encode_tmap_2d_f32_sw128(&map_b, b_split, g.kp, g.n_blocks * 2 * BN, g.kp * 4, kGemmBK,
                                2 * BN);
  if (rc) return rc;
  const int64_t tiles = g.m_blocks * g.n_blocks * g.ks;  // work units
  const int grid = static_cast<int>(tiles < sm_count() ? tiles : sm_count());
  // The epilogue staging block only for the fused exchange: with programmatic
  // dependent launch the GEMM's CTAs become resident while the split kernels
  // still run, and 18 KB less shared memory leaves those room on the SM.
  if (pt) {
    auto *fn = gemm_3xtf32_kernel<BN, true, GemmDstTma>;
    rc = ensure_dynamic_smem(reinterpret_cast<const void *>(fn), T::kSmemBytesTma);
    if (rc) return rc;
    return launch_programmatic(fn, dim3(grid), dim3(kGemmThreads), T::kSmemBytesTma, stream,
                               map_a, map_b, prm, *pt);
  }
  if (pd) {
    auto *fn = gemm_3xtf32_kernel<BN, true, GemmDst>;
    rc = ensure_dynamic_smem(reinterpret_cast<const void *>(fn), T::kSmemBytes);
    if (rc) return rc;
    return launch_programmatic(fn, dim3(grid), dim3(kGemmThreads), T::kSmemBytes, stream, map_a,
                               map_b, prm, *pd);
  }
  auto *fn = gemm_3xtf32_kernel<BN, false, GemmNoDst>;
  const int smem = T::kSmemBytes - kEpiStageBytes;
  rc = ensure_dynamic_smem(reinterpret_cast<const void *>(fn), smem);
  if (rc) return rc;
  return launch_programmatic(fn, dim3(grid), dim3(kGemmThreads), smem, stream, map_a, map_b, prm,
                             GemmNoDst{});
}

// The raw-operand form applies when TMA can read A and B in place: 16-byte
// aligned bases and row pitches, and rows of at least 16 bytes.
bool gemm_raw_ok(const float *A, int64_t lda, const float *B, int64_t ldb, int64_t N,
                 int64_t K) {
  return (reinterpret_cast<uintptr_t>(A) & 15u) == 0 && (reinterpret_cast<uintptr_t>(B) & 15u) == 0 &&
         lda % 4 == 0 && ldb % 4 == 0 && K >= 4 && N >= 4;
}

template <int BN>
int launch_gemm_raw(cudaStream_t stream, const GemmPlan &g, const float *A, int64_t lda,
                    const float *B, int64_t ldb, const GemmParams &prm, const GemmDst *pd) {
  using T = RawGemmTraits<BN>;
  CUtensorMap map_a, map_b;
  int rc = encode_tmap_2d_f32_sw128(&map_a, A, prm.K, prm.M, lda * 4, kGemmBK, kGemmBM);
  if (rc) return rc;
  rc = encode_tmap_2d_f32_sw128_atom32(&map_b, B, prm.N, prm.K, ldb * 4, 32, kGemmBK);
  if (rc) return rc;
  const int64_t tiles = g.m_blocks * g.n_blocks;
  const int grid = static_cast<int>(tiles < sm_count() ? tiles : sm_count());
  const bool fused = pd != nullptr;  // staging block only then, as launch_gemm
  const int smem = T::kSmemBytes - (fused ? 0 : kEpiStageBytes);
  const void *fn =
      fused ? reinterpret_cast<const void *>(gemm_3xtf32_raw_kernel<BN, true, GemmDst>)
            : reinterpret_cast<const void *>(gemm_3xtf32_raw_kernel<BN, false, GemmNoDst>);
  rc = ensure_dynamic_smem(fn, smem);
  if (rc) return rc;
  if (fused)
    gemm_3xtf32_raw_kernel<BN, true, GemmDst>
        <<<grid, kRawThreads, smem, stream>>>(map_a, map_b, prm, *pd);
  else
    gemm_3xtf32_raw_kernel<BN, false, GemmNoDst>
        <<<grid, kRawThreads, smem, stream>>>(map_a, map_b, prm, GemmNoDst{});
  count_launch();
  return launch_result();
}

}  // namespace

// Split launcher (split_tf32.cu): A -> A' and B -> B' (hi/lo, blocked,
// zero-padded), and C zeroed when `c` is non-null, in one launch.
int launch_split_operands(cudaStream_t s, const float *a, int64_t rows, int64_t cols,
                          int64_t lda, float *a_dst, int a_row_block, int64_t rows_pad,
                          const float *b, int64_t krows, int64_t ncols, int64_t ldb,
                          float *b_dst, int b_row_block, int64_t npad, int64_t kp, float *c,
                          int64_t ldc);

}  // namespace nplk

using namespace nplk;

extern "C" size_t nplk_gemm_workspace_size(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  const GemmPlan g = plan_gemm(M, N, K);
  return g.a_bytes + g.b_bytes_max;
}

namespace nplk {
namespace {

// Validates the common arguments and runs the GEMM with `prm` (whose epilogue
// fields the caller has set) in the operand form the flags and workspace
// select; `pd` non-null selects the fused exchange epilogue.
int gemm_run(cudaStream_t s, int64_t M, int64_t N, int64_t K, const float *A, int64_t lda,
             const float *B, int64_t ldb, GemmParams prm, const GemmDst *pd, unsigned flags,
             void *workspace, size_t workspace_bytes, int *status, int force_bn = 0,
             const GemmDstTma *pt = nullptr) {
  if (M <= 0 || N <= 0 || K <= 0 || !A || !B) return kErrInvalidArg;
  if (lda < K || ldb < N) return kErrInvalidArg;
  if (M > (int64_t(1) << 30) || N > (int64_t(1) << 30) || K > (int64_t(1) << 30))
    return kErrUnsupported;
  GemmPlan g = plan_gemm(M, N, K, force_bn);
  // Split-K only where its epilogue applies: a plain product written to C
  // (no C read, bias, activation or fused exchange) in the split operand form.
  if (g.ks > 1 && (pd || pt || prm.beta != 0.0f || prm.bias || prm.act != 0 ||
                   (flags & NPLK_GEMM_RAW_OPERANDS) || !workspace ||
                   workspace_bytes < g.a_bytes + g.b_bytes))
    g = plan_gemm(M, N, K, g.bn);
  if (!status) status = device_status_word();
  if (!status) return kErrInternal;
  prm.M = static_cast<int>(M);
  prm.N = static_cast<int>(N);
  prm.K = static_cast<int>(K);
  prm.m_blocks = static_cast<int>(g.m_blocks);
  prm.n_blocks = static_cast<int>(g.n_blocks);
  prm.k_blocks = static_cast<int>(g.kp / kGemmBK);
  prm.one_pass = ((flags & NPLK_GEMM_TF32_FAST) ? 1 : 0) | (g.ks > 1 ? g.ks << 8 : 0);
  prm.stall_us = take_armed_stall(NPLK_DEBUG_GEMM);
  prm.status = status;

  // Operand form: split (hi/lo copies in the workspace, then the GEMM) when
  // the workspace suffices -- it is the faster form: the GEMM is bound by
  // shared-memory bandwidth, and forming the lo parts in shared memory adds
  // ~22% to it (8192x4096x16384: 236.7 vs 194.8 TFLOP/s; 1024^3: 37.3 vs
  // 36.5 us with the split kernels included) -- else raw (A and B read in
  // place, no workspace) when TMA can read them. Callers may force either.
  const bool raw_ok = gemm_raw_ok(A, lda, B, ldb, N, K);
  const bool have_ws = workspace && workspace_bytes >= g.a_bytes + g.b_bytes;
  if ((flags & NPLK_GEMM_RAW_OPERANDS) && !raw_ok) return kErrUnsupported;
  const bool raw = (flags & NPLK_GEMM_RAW_OPERANDS) ||
                   (!have_ws && raw_ok && !(flags & NPLK_GEMM_SPLIT_OPERANDS));
  if (raw && pt) return kErrUnsupported;  // the TMA-store exchange has the split form only
  if (raw) {
    if (g.bn == 128) return launch_gemm_raw<128>(s, g, A, lda, B, ldb, prm, pd);
    return launch_gemm_raw<64>(s, g, A, lda, B, ldb, prm, pd);
  }

  if (!have_ws) return kErrInvalidArg;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255u) != 0) return kErrInvalidArg;
  float *a_split = static_cast<float *>(workspace);
  float *b_split = reinterpret_cast<float *>(static_cast<uint8_t *>(workspace) + g.a_bytes);

  // One launch splits A and B (and zeroes C for the K slices to add into);
  // the GEMM kernel's set-up overlaps it (programmatic dependent launch) and
  // its TMA producer waits for it before the first load.
  const int rc = launch_split_operands(s, A, M, K, lda, a_split, kGemmBM, g.m_blocks * kGemmBM,
                                       B, K, N, ldb, b_split, g.bn, g.n_blocks * g.bn, g.kp,
                                       g.ks > 1 ? prm.C : nullptr, prm.ldc);
  if (rc) return rc;
  if (g.bn == 128) return launch_gemm<128>(s, g, a_split, b_split, prm, pd, pt);
  return launch_gemm<64>(s, g, a_split, b_split, prm, pd, pt);
}

}  // namespace
}  // namespace nplk

extern "C" int nplk_gemm(void *stream, int64_t M, int64_t N, int64_t K, float alpha,
                         const float *A, int64_t lda, const float *B, int64_t ldb, float beta,
                         float *C, int64_t ldc, const float *bias, int act, float act_alpha,
                         unsigned flags, void *workspace, size_t workspace_bytes,
                         int *status) {
  if (!C || ldc < N) return kErrInvalidArg;
  GemmParams prm{};
  prm.alpha = alpha;
  prm.beta = beta;
  prm.C = C;
  prm.ldc = ldc;
  prm.bias = bias;
  prm.act = act;
  prm.act_alpha = act_alpha;
  return gemm_run(static_cast<cudaStream_t>(stream), M, N, K, A, lda, B, ldb, prm, nullptr,
                  flags, workspace, workspace_bytes, status);
}

extern "C" int nplk_gemm_allgather(void *stream, int64_t M, int64_t N_local, int64_t K,
                                   float alpha, const float *A, int64_t lda, const float *B,
                                   int64_t ldb, const float *bias, int act, float act_alpha,
                                   float *const *dst, int n_dst, int64_t col_offset, int64_t ldc,
                                   unsigned flags, void *workspace, size_t workspace_bytes,
                                   int *status) {
  if (!dst || n_dst < 1 || n_dst > 8 || col_offset < 0 || ldc < col_offset + N_local)
    return kErrInvalidArg;
  GemmParams prm{};
  prm.alpha = alpha;
  prm.beta = 0.0f;
  prm.C = nullptr;
  prm.ldc = ldc;
  prm.bias = bias;
  prm.act = act;
  prm.act_alpha = act_alpha;
  GemmDst pd{};
  pd.n_dst = n_dst;
  pd.dst_col = col_offset;
  // This rank's index when the blocks are laid out by rank (col_offset =
  // rank * N_local, dst[] in rank order): it starts with the next rank.
  pd.rot = static_cast<int>((col_offset / N_local + 1) % n_dst);
  bool vec = N_local % 4 == 0 && ldc % 4 == 0 && col_offset % 4 == 0;
  for (int d = 0; d < n_dst; ++d) {
    if (!dst[d]) return kErrInvalidArg;
    pd.dst[d] = dst[d];
    vec = vec && (reinterpret_cast<uintptr_t>(dst[d]) & 15u) == 0;
  }
  pd.dst_vec = vec ? 1 : 0;
  if (flags & NPLK_GEMM_MULTIMEM_STORES) {
    // One multicast destination, written with 16-byte multimem stores only.
    if (n_dst != 1 || !vec || (flags & NPLK_GEMM_PEER_TMA_STORES)) return kErrInvalidArg;
    pd.multimem = 1;
    pd.rot = 0;
    return gemm_run(static_cast<cudaStream_t>(stream), M, N_local, K, A, lda, B, ldb, prm, &pd,
                    flags, workspace, workspace_bytes, status);
  }
  // TMA-store form on request, when the destinations allow 16-byte aligned
  // tensor maps and the split operand form runs (a workspace, not forced raw).
  const bool tma = vec && (flags & NPLK_GEMM_PEER_TMA_STORES) &&
                   !(flags & NPLK_GEMM_RAW_OPERANDS) &&
                   workspace && workspace_bytes >= nplk_gemm_workspace_size(M, N_local, K) &&
                   M >= 32 && N_local >= 32 && M <= (int64_t(1) << 30) &&
                   N_local <= (int64_t(1) << 30);
  if (tma) {
    GemmDstTma pt{};
    pt.n_dst = n_dst;
    pt.rot = pd.rot;
    for (int d = 0; d < n_dst; ++d) {
      const int rc = encode_tmap_2d_f32_sw128(&pt.map[d], dst[d] + col_offset, N_local, M,
                                              ldc * 4, 32, 32);
      if (rc) return rc;
    }
    return gemm_run(static_cast<cudaStream_t>(stream), M, N_local, K, A, lda, B, ldb, prm,
                    nullptr, flags, workspace, workspace_bytes, status, 0, &pt);
  }
  return gemm_run(static_cast<cudaStream_t>(stream), M, N_local, K, A, lda, B, ldb, prm, &pd,
                  flags, workspace, workspace_bytes, status);
}

extern "C" int nplk_gemm_tune(void *stream, int64_t M, int64_t N, int64_t K, const float *A,
                              int64_t lda, const float *B, int64_t ldb, float *C, int64_t ldc,
                              void *workspace, size_t workspace_bytes, int reps, int *best_bn,
                              float *best_us) {
  if (!C || ldc < N || !best_bn || reps < 1 || reps > 1000) return kErrInvalidArg;
  if (M <= 0 || N <= 0 || K <= 0) return kErrInvalidArg;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  GemmParams prm{};
  prm.alpha = 1.0f;
  prm.beta = 0.0f;
  prm.C = C;
  prm.ldc = ldc;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  if (cudaEventCreate(&e0) != cudaSuccess || cudaEventCreate(&e1) != cudaSuccess) {
    if (e0) cudaEventDestroy(e0);
    return kErrInternal;
  }
  int best = 0, rc = kOk;
  float best_ms = 0.0f;
  for (int bn : {64, 128, kGemmCfgSplitK}) {
    if (bn == kGemmCfgSplitK && ceil_div(K, kGemmBK) < 16) continue;
    std::vector<float> ms;
    for (int r = 0; r <= reps && rc == kOk; ++r) {
      if (cudaEventRecord(e0, s) != cudaSuccess) rc = kErrInternal;
      if (rc == kOk)
        rc = gemm_run(s, M, N, K, A, lda, B, ldb, prm, nullptr, 0u, workspace, workspace_bytes,
                      nullptr, bn);
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
      best = bn;
      best_ms = med;
    }
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (rc != kOk) return rc;
  if (nplk_read_status(stream) != 0) return kErrInternal;
  tuning_insert(tuning_key_gemm(M, N, K), best, best_ms * 1000.0);
  *best_bn = best;
  if (best_us) *best_us = best_ms * 1000.0f;
  return kOk;
}

