// Sliding-window kernels over NCHW planes: depthwise convolution and max /
// average pooling.
//
// band_window_kernel (rows of up to 2 K elements): a CTA stages a batch of
// input in shared memory with 16-byte cp.async copies -- several whole planes
// when a plane is small (consecutive planes are contiguous in NCHW), else a
// band of rows of one plane -- while it computes the previous batch; each
// thread computes a column of outputs and consecutive lanes store consecutive
// columns. window_kernel
// (wider rows): one thread per output, consecutive threads on consecutive
// output columns, so the window reads of a warp hit a few cache lines and are
// served from L1 after the first touch. Every output takes the reference's
// order (kh outer, kw inner, padded cells skipped -- the 3x3 path combines
// the operation's identity there instead, which leaves each result bit for
// bit the same), so all paths agree exactly; each input element crosses HBM
// about once.
#include <cuda_runtime.h>
#include <math_constants.h>

#include <numeric>

#include "nplk_device.cuh"
#include "nplk_host.h"
#include "ptx_sm100.cuh"

namespace nplk {

namespace {
int window_grid(int64_t items) {
  const int64_t max_blocks = static_cast<int64_t>(sm_count()) * 16;
  int64_t b = ceil_div(items, 256);
  if (b > max_blocks) b = max_blocks;
  return static_cast<int>(b < 1 ? 1 : b);
}
}  // namespace

struct WindowGeom {
  int C, H, W, KH, KW, sh, sw, ph, pw, Ho, Wo;
  FastDiv div_wo, div_ho, div_c;
};

// Depthwise: out[n][c][oh][ow] = sum_{kh,kw} x[n][c][oh*sh+kh-ph][ow*sw+kw-pw]
// * w[c][kh][kw] (+ bias[c]) with the reference's summation order (kh outer,
// kw inner) and no dilation (npl_convolution.cpp:921-951).
__global__ void dwconv_kernel(const float *__restrict__ x, const float *__restrict__ w,
                              const float *__restrict__ bias, float *__restrict__ y,
                              uint32_t total, WindowGeom g) {
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const uint32_t q1 = fdiv(i, g.div_wo);
    const int ow = static_cast<int>(i - q1 * g.Wo);
    const uint32_t plane = fdiv(q1, g.div_ho);
    const int oh = static_cast<int>(q1 - plane * g.Ho);
    const int c = static_cast<int>(plane - fdiv(plane, g.div_c) * g.C);
    const float *xp = x + static_cast<int64_t>(plane) * g.H * g.W;
    const float *wp = w + static_cast<int64_t>(c) * g.KH * g.KW;
    float sum = 0.0f;
    for (int kh = 0; kh < g.KH; ++kh) {
      const int ih = oh * g.sh + kh - g.ph;
      if (static_cast<unsigned>(ih) >= static_cast<unsigned>(g.H)) continue;
      for (int kw = 0; kw < g.KW; ++kw) {
        const int iw = ow * g.sw + kw - g.pw;
        if (static_cast<unsigned>(iw) < static_cast<unsigned>(g.W))
          sum += __ldg(xp + ih * g.W + iw) * __ldg(wp + kh * g.KW + kw);
      }
    }
    if (bias) sum += bias[c];
    y[i] = sum;
  }
}

// Max pooling (-inf start, padded cells skipped, npl_pooling.cpp:129-219) and
// average pooling (padded cells counted only with count_include_pad,
// npl_pooling.cpp:221-315).
template <int kType>
__global__ void pool_kernel(const float *__restrict__ x, float *__restrict__ y, uint32_t total,
                            WindowGeom g, int count_include_pad) {
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const uint32_t q1 = fdiv(i, g.div_wo);
    const int ow = static_cast<int>(i - q1 * g.Wo);
    const uint32_t plane = fdiv(q1, g.div_ho);
    const int oh = static_cast<int>(q1 - plane * g.Ho);
    const float *xp = x + static_cast<int64_t>(plane) * g.H * g.W;
    if (kType == 0) {
      float m = -CUDART_INF_F;
      for (int kh = 0; kh < g.KH; ++kh) {
        const int ih = oh * g.sh + kh - g.ph;
        if (static_cast<unsigned>(ih) >= static_cast<unsigned>(g.H)) continue;
        for (int kw = 0; kw < g.KW; ++kw) {
          const int iw = ow * g.sw + kw - g.pw;
          if (static_cast<unsigned>(iw) < static_cast<unsigned>(g.W)) {
            const float v = __ldg(xp + ih * g.W + iw);
            m = (m < v) ? v : m;  // std::max(m, v)
          }
        }
      }
      y[i] = m;
    } else {
      float s = 0.0f;
      int cnt = 0;
      for (int kh = 0; kh < g.KH; ++kh) {
        const int ih = oh * g.sh + kh - g.ph;
        const bool row_in = static_cast<unsigned>(ih) < static_cast<unsigned>(g.H);
        for (int kw = 0; kw < g.KW; ++kw) {
          const int iw = ow * g.sw + kw - g.pw;
          if (row_in && static_cast<unsigned>(iw) < static_cast<unsigned>(g.W)) {
            s += __ldg(xp + ih * g.W + iw);
            ++cnt;
          } else if (count_include_pad) {
            ++cnt;
          }
        }
      }
      y[i] = cnt > 0 ? s / static_cast<float>(cnt) : 0.0f;
    }
  }
}

// One output of window operation kOp (0 depthwise, 1 max pool, 2 average
// pool) at (oh, ow) of a plane staged in shared memory from input row ih_lo
// on (row pitch g.W); wp: the plane's filter (depthwise). Same expression and
// order as dwconv_kernel / pool_kernel.
template <int kOp>
__device__ __forceinline__ float window_out(const float *xp, const float *wp, int oh, int ow,
                                            const WindowGeom &g, int count_include_pad,
                                            int ih_lo) {
  if (kOp == 0) {
    float sum = 0.0f;
    for (int kh = 0; kh < g.KH; ++kh) {
      const int ih = oh * g.sh + kh - g.ph;
      if (static_cast<unsigned>(ih) >= static_cast<unsigned>(g.H)) continue;
      for (int kw = 0; kw < g.KW; ++kw) {
        const int iw = ow * g.sw + kw - g.pw;
        if (static_cast<unsigned>(iw) < static_cast<unsigned>(g.W))
          sum += xp[(ih - ih_lo) * g.W + iw] * wp[kh * g.KW + kw];
      }
    }
    return sum;
  } else if (kOp == 1) {
    float m = -CUDART_INF_F;
    for (int kh = 0; kh < g.KH; ++kh) {
      const int ih = oh * g.sh + kh - g.ph;
      if (static_cast<unsigned>(ih) >= static_cast<unsigned>(g.H)) continue;
      for (int kw = 0; kw < g.KW; ++kw) {
        const int iw = ow * g.sw + kw - g.pw;
        if (static_cast<unsigned>(iw) < static_cast<unsigned>(g.W)) {
          const float v = xp[(ih - ih_lo) * g.W + iw];
          m = (m < v) ? v : m;  // std::max(m, v)
        }
      }
    }
    return m;
  } else {
    float s = 0.0f;
    int cnt = 0;
    for (int kh = 0; kh < g.KH; ++kh) {
      const int ih = oh * g.sh + kh - g.ph;
      const bool row_in = static_cast<unsigned>(ih) < static_cast<unsigned>(g.H);
      for (int kw = 0; kw < g.KW; ++kw) {
        const int iw = ow * g.sw + kw - g.pw;
        if (row_in && static_cast<unsigned>(iw) < static_cast<unsigned>(g.W)) {
          s += xp[(ih - ih_lo) * g.W + iw];
          ++cnt;
        } else if (count_include_pad) {
          ++cnt;
        }
      }
    }
    return cnt > 0 ? s / static_cast<float>(cnt) : 0.0f;
  }
}

constexpr int kBandWarps = 4;                      // consumer warps per CTA
constexpr int kBandThreads = (kBandWarps + 1) * 32;  // + one producer warp
constexpr int kBandStages = 8;                     // staged batches per CTA
constexpr int kBandStageBytes = 7136;              // per stage: 4 CTAs (57 KB) per SM
constexpr int kBandItemsMax = 64;                  // items per batch: two per lane

// Output rows per item of the 3x3 path: 14 at vertical stride 1, 7 at 2 (they
// divide the usual plane heights 7, 14, 28, 56, 112); an item covers two
// adjacent output columns.
template <int SH_>
struct StripRows {
  static constexpr int value = SH_ == 1 ? 14 : 7;
};

// Work plan of band_window_kernel. A batch is either np whole planes (whole:
// consecutive NCHW planes are one contiguous range) or one band of R output
// rows of one plane (its input rows are one contiguous range too).
struct BandPlan {
  int whole, np, R, bands;
  int strips;          // strips per plane (whole planes)
  int stage_floats;    // one stage (multiple of 4 floats)
  FastDiv div_pairs;   // by the output column pairs of a row
  FastDiv div_strips;  // by strips
  int64_t batches;
};

struct BandBatch {
  int64_t q0;  // first plane
  int cnt;     // planes
  int oh0, oh1, ih_lo, ih_hi;
};

__device__ __forceinline__ BandBatch band_batch(int64_t b, int64_t planes, const BandPlan &bp,
                                                const WindowGeom &g, int KH) {
  BandBatch r;
  if (bp.whole) {
    r.q0 = b * bp.np;
    r.cnt = static_cast<int>(planes - r.q0 < bp.np ? planes - r.q0 : bp.np);
    r.oh0 = 0;
    r.oh1 = g.Ho;
    r.ih_lo = 0;
    r.ih_hi = g.H;
  } else {
    r.q0 = b / bp.bands;
    const int band = static_cast<int>(b - r.q0 * bp.bands);
    r.cnt = 1;
    r.oh0 = band * bp.R;
    r.oh1 = min(g.Ho, r.oh0 + bp.R);
    r.ih_lo = max(0, r.oh0 * g.sh - g.ph);
    r.ih_hi = min(g.H, (r.oh1 - 1) * g.sh - g.ph + KH);
    if (r.ih_hi < r.ih_lo) r.ih_hi = r.ih_lo;
  }
  return r;
}

// First input element of a batch and how many follow it contiguously.
__device__ __forceinline__ const float *band_src(const float *x, const BandBatch &bb, int HW,
                                                 int W, int &n_in) {
  n_in = (bb.cnt - 1) * HW + (bb.ih_hi - bb.ih_lo) * W;
  return x + bb.q0 * HW + static_cast<int64_t>(bb.ih_lo) * W;
}

// Sliding-window operation kOp over NCHW planes. Warp-specialised: one lane of
// the last warp stages batches (whole planes or row bands, each one
// contiguous range of x) into a ring of kBandStages shared-memory stages with
// one bulk copy each -- the 16-byte-aligned superset of the range, which lies
// on the same mapped pages -- completing on the stage's mbarrier; each of the
// kBandWarps consumer warps computes whole batches (every kBandWarps-th of
// the CTA's) and releases the stage. No CTA-wide barrier: a warp waits only
// for its own batch, and up to kBandStages batches are in flight per CTA.
// SH_, SW_ > 0: 3x3 window with those strides; an item is two adjacent output
// columns over a strip of StripRows<SH_> output rows, so every input row
// under the strip is read from shared memory once, consecutive lanes read
// consecutive columns and each tap is one unconditional combine. SH_ = SW_ =
// 0: any window, one output per item. Outputs are stored straight from
// registers (consecutive lanes on consecutive columns). Bounded waits record
// kStatusTimeoutProducer / kStatusTimeoutStage in *status.
template <int kOp, int SH_, int SW_>
__global__ void __launch_bounds__(kBandThreads, 4) band_window_kernel(
    const float *__restrict__ x, const float *__restrict__ w, const float *__restrict__ bias,
    float *__restrict__ y, int64_t planes, BandPlan bp, WindowGeom g, int count_include_pad,
    int *status) {
  extern __shared__ __align__(128) uint8_t smem_band[];
  float *stages = reinterpret_cast<float *>(smem_band);
  uint64_t *full = reinterpret_cast<uint64_t *>(stages + kBandStages * bp.stage_floats);
  uint64_t *empty = full + kBandStages;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(empty + kBandStages);
  constexpr bool kFast = SH_ > 0;
  const int KH = kFast ? 3 : g.KH;
  const int taps = kFast ? 9 : g.KH * g.KW;
  const int HW = g.H * g.W;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kBandStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  // This CTA's batches: blockIdx.x + k * gridDim.x, k < nk.
  const int64_t nk = bp.batches > blockIdx.x
                         ? (bp.batches - 1 - blockIdx.x) / gridDim.x + 1
                         : 0;

  if (warp == kBandWarps) {
    // ---------------- producer ----------------
    if (lane == 0) {
      int64_t k = 0;
      for (; k < nk; ++k) {
        const int s = static_cast<int>(k % kBandStages);
        const uint32_t ph = static_cast<uint32_t>(k / kBandStages) & 1u;
        if (!mbar_wait(&empty[s], ph ^ 1u, abort_flag, status, kStatusTimeoutProducer)) break;
        const BandBatch bb = band_batch(blockIdx.x + k * gridDim.x, planes, bp, g, KH);
        int n_in;
        const float *src = band_src(x, bb, HW, g.W, n_in);
        const uintptr_t lo = reinterpret_cast<uintptr_t>(src) & ~uintptr_t(15);
        const uintptr_t hi = (reinterpret_cast<uintptr_t>(src + n_in) + 15) & ~uintptr_t(15);
        // A batch with no input rows (a band inside the padding) copies
        // nothing: its src may lie past the end of x.
        const uint32_t bytes = n_in > 0 ? static_cast<uint32_t>(hi - lo) : 0u;
        if (bytes > 0) {
          mbar_arrive_expect_tx(&full[s], bytes);
          bulk_load_g2s(stages + s * bp.stage_floats, reinterpret_cast<const void *>(lo), bytes,
                        &full[s]);
        } else {
          mbar_arrive(&full[s]);
        }
      }
      // Let the last copies land before the CTA can exit (they already have
      // unless the CTA aborted).
      for (int64_t j = k > kBandStages ? k - kBandStages : 0; j < k; ++j)
        mbar_drain(&full[j % kBandStages], static_cast<uint32_t>(j / kBandStages) & 1u);
    }
    return;
  }

  // ---------------- consumers ----------------
  for (int64_t k = warp; k < nk; k += kBandWarps) {
    const int s = static_cast<int>(k % kBandStages);
    const uint32_t ph = static_cast<uint32_t>(k / kBandStages) & 1u;
    const BandBatch bb = band_batch(blockIdx.x + k * gridDim.x, planes, bp, g, KH);
    const int rows = bb.oh1 - bb.oh0;
    const int c0 = kOp == 0 ? static_cast<int>(bb.q0 % g.C) : 0;  // channel of the first plane
    // The 3x3 path: this lane's first item and its filter, loaded from global
    // memory before the wait for the staged input so that the two overlap.
    constexpr int Vf = kFast ? StripRows<SH_ ? SH_ : 1>::value : 1;
    const int strips = bp.whole ? bp.strips : (rows + Vf - 1) / Vf;
    const int pairs = (g.Wo + 1) >> 1;
    int rest0 = 0, pl0 = 0;
    float wnext[9];
    if (kFast) {
      rest0 = static_cast<int>(fdiv(static_cast<uint32_t>(lane), bp.div_pairs));
      pl0 = bp.whole ? static_cast<int>(fdiv(static_cast<uint32_t>(rest0), bp.div_strips)) : 0;
      if (kOp == 0 && pl0 < bb.cnt) {
        const float *wp = w + ((c0 + pl0) % g.C) * 9;
#pragma unroll
        for (int k9 = 0; k9 < 9; ++k9) wnext[k9] = __ldg(wp + k9);
      }
    }
    if (!mbar_wait(&full[s], ph, abort_flag, status, kStatusTimeoutStage)) break;
    int n_in;
    const float *src = band_src(x, bb, HW, g.W, n_in);
    const float *data = stages + s * bp.stage_floats +
                        static_cast<int>((reinterpret_cast<uintptr_t>(src) >> 2) & 3);
    float *out = y + bb.q0 * (static_cast<int64_t>(g.Ho) * g.Wo) +
                 static_cast<int64_t>(bb.oh0) * g.Wo;
    if constexpr (kFast) {
      constexpr int V = StripRows<SH_>::value;
      constexpr int kCols = SW_ + 3;            // input columns under two outputs
      constexpr int kRows = (V - 1) * SH_ + 3;  // input rows under a strip
      const int items = bb.cnt * strips * pairs;
      for (int it = lane; it < items; it += 32) {
        const bool first = it == lane;
        const int rest =
            first ? rest0 : static_cast<int>(fdiv(static_cast<uint32_t>(it), bp.div_pairs));
        const int ow0 = (it - rest * pairs) * 2;
        const int pl = first ? pl0
                     : bp.whole ? static_cast<int>(fdiv(static_cast<uint32_t>(rest), bp.div_strips))
                                : 0;
        const int st = rest - pl * strips;
        const int ohs = bb.oh0 + st * V;
        const int nv = min(V, bb.oh1 - ohs);
        const bool two = ow0 + 1 < g.Wo;
        const float *xp = data + pl * HW;
        const int iw0 = ow0 * SW_ - g.pw;
        const int ih_s = ohs * SH_ - g.ph;
        const int last_r = (nv - 1) * SH_ + 2;  // later rows only feed outputs past nv
        bool cok[kCols];
#pragma unroll
        for (int j = 0; j < kCols; ++j)
          cok[j] = static_cast<unsigned>(iw0 + j) < static_cast<unsigned>(g.W);
        const int c = kOp == 0 ? (c0 + pl) % g.C : 0;
        float wr[9];
        bool finite = true;
        if (kOp == 0) {
#pragma unroll
          for (int k9 = 0; k9 < 9; ++k9) {
            wr[k9] = first ? wnext[k9] : __ldg(w + c * 9 + k9);
            finite = finite && isfinite(wr[k9]);
          }
        }
        float *op = out + (pl * rows + st * V) * g.Wo + ow0;
        if (kOp == 0 && !finite) {
          // 0 * inf would differ from skipping the padded cell: exact path.
          const float bv = bias ? __ldg(bias + c) : 0.0f;
          for (int v = 0; v < nv; ++v) {
            for (int cc = 0; cc < (two ? 2 : 1); ++cc) {
              float o = window_out<0>(xp, w + c * 9, ohs + v, ow0 + cc, g, 0, bb.ih_lo);
              if (bias) o += bv;
              op[v * g.Wo + cc] = o;
            }
          }
          continue;
        }
        // Cells outside the plane (or past the strip's last row) read as the
        // operation's identity -- 0 for sums (a running sum is never -0, and
        // the weights are finite, so adding 0 * w changes nothing), -inf for
        // the running max -- so every tap is combined unconditionally.
        const float kPad = kOp == 1 ? -CUDART_INF_F : 0.0f;
        float acc[V][2];
#pragma unroll
        for (int v = 0; v < V; ++v) acc[v][0] = acc[v][1] = kOp == 1 ? -CUDART_INF_F : 0.0f;
        const float *xrow = xp + (ih_s - bb.ih_lo) * g.W + iw0;
#pragma unroll
        for (int r = 0; r < kRows; ++r) {
          const bool rok =
              r <= last_r && static_cast<unsigned>(ih_s + r) < static_cast<unsigned>(g.H);
          float xv[kCols];
#pragma unroll
          for (int j = 0; j < kCols; ++j) xv[j] = (rok && cok[j]) ? xrow[j] : kPad;
          xrow += g.W;
#pragma unroll
          for (int v = 0; v < V; ++v) {
            const int kh = r - v * SH_;
            if (kh < 0 || kh > 2) continue;
#pragma unroll
            for (int cc = 0; cc < 2; ++cc) {
#pragma unroll
              for (int kw = 0; kw < 3; ++kw) {
                const float xin = xv[cc * SW_ + kw];
                if (kOp == 0)
                  acc[v][cc] += xin * wr[kh * 3 + kw];
                else if (kOp == 1)
                  acc[v][cc] = (acc[v][cc] < xin) ? xin : acc[v][cc];  // std::max(m, v)
                else
                  acc[v][cc] += xin;
              }
            }
          }
        }
        const float bv = (kOp == 0 && bias) ? __ldg(bias + c) : 0.0f;
        int ncols[2] = {0, 0};
        if (kOp == 2) {
#pragma unroll
          for (int cc = 0; cc < 2; ++cc)
#pragma unroll
            for (int kw = 0; kw < 3; ++kw) ncols[cc] += cok[cc * SW_ + kw] ? 1 : 0;
        }
#pragma unroll
        for (int v = 0; v < V; ++v) {
          if (v >= nv) break;
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            if (cc == 1 && !two) break;
            float o = acc[v][cc];
            if (kOp == 0 && bias) o += bv;
            if (kOp == 2) {
              const int ih0 = ih_s + v * SH_;
              const int nrows = max(0, min(g.H, ih0 + 3) - max(0, ih0));
              const int cnt = count_include_pad ? 9 : nrows * ncols[cc];
              o = cnt > 0 ? o / static_cast<float>(cnt) : 0.0f;
            }
            op[v * g.Wo + cc] = o;
          }
        }
      }
    } else {
      const int items = bb.cnt * rows * g.Wo;
      for (int it = lane; it < items; it += 32) {
        const int rest = static_cast<int>(fdiv(static_cast<uint32_t>(it), g.div_wo));
        const int ow = it - rest * g.Wo;
        const int pl = rest / rows;
        const int r = rest - pl * rows;
        const int c = kOp == 0 ? (c0 + pl) % g.C : 0;
        float v = window_out<kOp>(data + pl * HW, w + static_cast<int64_t>(c) * taps, bb.oh0 + r,
                                  ow, g, count_include_pad, bb.ih_lo);
        if (kOp == 0 && bias) v += __ldg(bias + c);
        out[(pl * rows + r) * g.Wo + ow] = v;
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }
}

namespace {

int64_t round4(int64_t v) { return (v + 3) & ~int64_t(3); }

// Fraction of lane slots a batch of `items` fills when 32 lanes loop over it.
double lane_fill(int64_t items) {
  return static_cast<double>(items) / (32.0 * static_cast<double>(ceil_div(items, int64_t(32))));
}

// Batches for band_window_kernel; false when the input rows under one output
// row exceed a stage (the window_kernel family handles those).
bool band_plan(const WindowGeom &g, int64_t planes, bool fast, BandPlan &bp) {
  const int64_t HW = static_cast<int64_t>(g.H) * g.W;
  const int V = !fast ? 1 : g.sh == 1 ? StripRows<1>::value : StripRows<2>::value;
  const int64_t cols = fast ? (g.Wo + 1) / 2 : g.Wo;  // the 3x3 path pairs columns
  const int64_t items_pp = static_cast<int64_t>((g.Ho + V - 1) / V) * cols;
  const int64_t cap = (kBandStageBytes - 32) / 4;  // floats of input per stage
  bp = BandPlan{};
  if (HW <= cap) {
    // As many planes as fit a stage and keep the batch at <= kBandItemsMax
    // items, preferring a batch that fills the lanes.
    int64_t np_max = cap / HW;
    if (np_max > 64) np_max = 64;
    int64_t np = 1;
    double best = -1.0;
    for (int64_t n = 1; n <= np_max; ++n) {
      if (n > 1 && n * items_pp > kBandItemsMax) break;
      const double f = lane_fill(n * items_pp);
      if (f >= best - 1e-9) {
        best = f;
        np = n;
      }
    }
    bp.whole = 1;
    bp.np = static_cast<int>(np);
    bp.R = g.Ho;
    bp.bands = 1;
    bp.batches = ceil_div(planes, np);
    bp.strips = (g.Ho + V - 1) / V;
  } else {
    auto rows_in = [&](int64_t R) {
      const int64_t r = (R - 1) * g.sh + g.KH;
      return r < g.H ? r : static_cast<int64_t>(g.H);
    };
    if (rows_in(1) * g.W > cap) return false;
    int64_t R = 1;
    while (R < g.Ho && rows_in(R + 1) * g.W <= cap &&
           ceil_div(R + 1, static_cast<int64_t>(V)) * cols <= kBandItemsMax)
      ++R;
    if (fast && R > V) R -= R % V;
    bp.whole = 0;
    bp.np = 1;
    bp.R = static_cast<int>(R);
    bp.bands = static_cast<int>(ceil_div(static_cast<int64_t>(g.Ho), R));
    bp.batches = planes * bp.bands;
  }
  bp.stage_floats = static_cast<int>(round4(cap + 8));
  bp.div_pairs = make_fastdiv(static_cast<uint32_t>((g.Wo + 1) / 2));
  bp.div_strips = make_fastdiv(static_cast<uint32_t>(bp.strips > 0 ? bp.strips : 1));
  return true;
}

template <int kOp, int SH_, int SW_>
int launch_band_kernel(cudaStream_t s, const float *x, const float *w, const float *bias,
                       float *y, int64_t planes, const BandPlan &bp, const WindowGeom &g,
                       int count_include_pad) {
  auto kernel = band_window_kernel<kOp, SH_, SW_>;
  const size_t smem =
      static_cast<size_t>(kBandStages) * bp.stage_floats * 4 + 2 * kBandStages * 8 + 16;
  if (int rc = ensure_dynamic_smem(reinterpret_cast<const void *>(kernel), static_cast<int>(smem)))
    return rc;
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kBandThreads, smem) !=
          cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  int64_t blocks = static_cast<int64_t>(sm_count()) * per_sm;
  if (blocks > bp.batches) blocks = bp.batches;
  kernel<<<static_cast<unsigned>(blocks), kBandThreads, smem, s>>>(
      x, w, bias, y, planes, bp, g, count_include_pad, device_status_word());
  count_launch();
  return launch_result();
}

// Runs window operation kOp through band_window_kernel; returns 1 when the
// geometry has no staging plan (the caller then uses the window_kernel
// family).
template <int kOp>
int launch_band(cudaStream_t s, const float *x, const float *w, const float *bias, float *y,
                int64_t planes, const WindowGeom &g, int count_include_pad) {
  if ((reinterpret_cast<uintptr_t>(x) & 3u) || (reinterpret_cast<uintptr_t>(y) & 3u)) return 1;
  const bool fast = g.KH == 3 && g.KW == 3 && g.sh == g.sw && (g.sh == 1 || g.sh == 2);
  BandPlan bp;
  if (!band_plan(g, planes, fast, bp)) return 1;
  if (fast && g.sh == 1)
    return launch_band_kernel<kOp, 1, 1>(s, x, w, bias, y, planes, bp, g, count_include_pad);
  if (fast)
    return launch_band_kernel<kOp, 2, 2>(s, x, w, bias, y, planes, bp, g, count_include_pad);
  return launch_band_kernel<kOp, 0, 0>(s, x, w, bias, y, planes, bp, g, count_include_pad);
}

}  // namespace

}  // namespace nplk

using namespace nplk;

namespace nplk {

// ---------------------------------------------------------------------------
// Depthwise conv -> inference batch norm -> activation -> global average pool
// in one pass (nplk_depthwise_bn_act_gap): the reference's
// npl_depthwise_conv2d (npl_convolution.cpp:60-90, ExecuteDepthwiseConv
// :904-991), npl_batch_norm (npl_activation_norm.cpp:118-153, the inference
// form :389-398), npl_relu / npl_activation (:51-54) and npl_global_avg_pool
// (npl_pooling.cpp:63-87) applied back to back, with the intermediate maps
// never written to HBM unless asked for.
//
// One warp per NCHW plane: the input plane is staged in shared memory (16-byte
// loads, all issued before the first store); lane l computes the outputs at
// flat indices l, l + 32, ... (consecutive lanes read consecutive columns:
// no bank conflicts), each with the depthwise kernel's sum (kh outer, kw
// inner, padding skipped, then the bias), BN's expression and the
// activation; the activated outputs go to a second shared-memory block, and
// lane l then sums its float4 groups l, l + 32, ... in the GAP kernel's order (group by
// group from 0, (a + b) + (c + d) within a group, then the warp butterfly),
// storing them to y when asked. Every value is therefore the one the separate
// kernels produce, bit for bit.
// ---------------------------------------------------------------------------
constexpr int kDwGapWarps = 8;       // planes per 256-thread block

__device__ __forceinline__ float dwgap_warp_sum(float v) {  // the GAP kernel's butterfly
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
inline bool dwgap_aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
constexpr int kDwGapMaxIn = 1024;    // input plane elements staged per warp (4 KB)

// The activated plane, staged in shared memory, to y (when asked) and to its
// average: lane l takes the float4 groups l, l + 32, ... in the GAP kernel's
// order (gap_planes in reduce.cu).
template <int J>
__device__ __forceinline__ void dwgap_finish(const float *xsw, float *__restrict__ y,
                                             float *__restrict__ gap, int64_t plane, int howo,
                                             int lane) {
  float s = 0.0f;
  float4 *y4 = y ? reinterpret_cast<float4 *>(y + plane * howo) : nullptr;
#pragma unroll
  for (int j = 0; j < J; ++j) {
    const int q = lane + 32 * j;
    float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (4 * q < howo) {
      o = reinterpret_cast<const float4 *>(xsw)[q];
      if (y4) y4[q] = o;
    }
    s += (o.x + o.y) + (o.z + o.w);
  }
  s = dwgap_warp_sum(s);
  if (lane == 0) gap[plane] = s / static_cast<float>(howo);
}

// J: output float4 groups per lane (output planes of <= 128 J elements);
// JI: input float4 per lane (input planes of <= 128 JI elements); K3: 3x3
// filter (unrolled taps), else any filter; kRelu: the activation is ReLU
// (code 1), else any code of nplk_activation; SR > 0: 3x3, stride 1, pad 1,
// same-size planes at most 32 wide, whose columns split into 32 / Wo
// segments of SR rows: lane (column, segment) runs down its strip, reads each
// input row's three columns once and folds them into the (up to three)
// output rows they feed, in kh order; padding enters as zero products, which
// leave a sum unchanged when the weights are finite (the depthwise kernel's
// register path does the same), so planes with a non-finite weight take the
// per-output path.
// A channel's filter (3x3 unrolled) and bias, and its BN constants formed
// exactly as bn_infer_kernel forms them.
struct DwGapConsts {
  float wk[9];
  float bv, qg, qm, qi, qb;
};
template <bool K3>
__device__ __forceinline__ void dwgap_consts(DwGapConsts &k, int c, const float *__restrict__ w,
                                             const float *__restrict__ bias,
                                             const float *__restrict__ mean,
                                             const float *__restrict__ var,
                                             const float *__restrict__ gamma,
                                             const float *__restrict__ beta, float eps) {
  if (K3) {
#pragma unroll
    for (int t = 0; t < 9; ++t) k.wk[t] = __ldg(w + c * 9 + t);
  }
  k.bv = bias ? __ldg(bias + c) : 0.0f;
  k.qg = gamma ? __ldg(gamma + c) : 1.0f;
  k.qm = __ldg(mean + c);
  k.qi = 1.0f / sqrtf(__ldg(var + c) + eps);
  k.qb = beta ? __ldg(beta + c) : 0.0f;
}

template <int J, bool K3, bool kRelu, int SR>
__device__ __forceinline__ void dwgap_plane(
    const float *xsw, float *xout, int64_t plane, int lane, const DwGapConsts &kc,
    const float *__restrict__ wc, bool has_bias, int act, float act_alpha,
    float *__restrict__ y, float *__restrict__ gap, const WindowGeom &g) {
  const int howo = g.Ho * g.Wo;
  const float(&wk)[9] = kc.wk;
  const float bv = kc.bv, qg = kc.qg, qm = kc.qm, qi = kc.qi, qb = kc.qb;
  const bool bias = has_bias;
  __syncwarp();
  if constexpr (SR > 0) {
    bool finite = true;
#pragma unroll
    for (int t = 0; t < 9; ++t) finite = finite && isfinite(wk[t]);
    if (finite) {
      const int ow = lane % g.Wo, seg = lane / g.Wo;
      const bool active = seg < 32 / g.Wo;
      const int r0 = seg * SR;
      float acc[SR];
#pragma unroll
      for (int r = 0; r < SR; ++r) acc[r] = 0.0f;
#pragma unroll
      for (int t = 0; t < SR + 2; ++t) {  // input rows r0 - 1 .. r0 + SR
        const int ih = r0 - 1 + t;
        const bool rin = active && static_cast<unsigned>(ih) < static_cast<unsigned>(g.H);
        // indices clamped into the staged plane, so no address leaves it
        const int base = (rin ? ih : 0) * g.W + ow;
        const float v0 = (rin && ow > 0) ? xsw[base - (ow > 0 ? 1 : 0)] : 0.0f;
        const float v1 = rin ? xsw[base] : 0.0f;
        const float v2 = (rin && ow + 1 < g.W) ? xsw[base + (ow + 1 < g.W ? 1 : 0)] : 0.0f;
#pragma unroll
        for (int kh = 0; kh < 3; ++kh) {
          const int r = t - kh;  // output row r0 + r takes input row ih as its tap row kh
          if (r >= 0 && r < SR) {
            acc[r] += v0 * wk[kh * 3 + 0];
            acc[r] += v1 * wk[kh * 3 + 1];
            acc[r] += v2 * wk[kh * 3 + 2];
          }
        }
      }
#pragma unroll
      for (int r = 0; r < SR; ++r) {
        float sum = acc[r];
        if (bias) sum += bv;
        const float t = qg * (sum - qm) * qi + qb;
        acc[r] = kRelu ? (t < 0.0f ? 0.0f : t) : apply_act(t, act, act_alpha);
      }
#pragma unroll
      for (int r = 0; r < SR; ++r)
        if (active && r0 + r < g.Ho) xout[(r0 + r) * g.Wo + ow] = acc[r];
      __syncwarp();
      dwgap_finish<J>(xout, y, gap, plane, howo, lane);
      return;
    }
  }
#pragma unroll 1
  for (int i = 0; i < 4 * J; ++i) {
    const int f = lane + 32 * i;
    if (f < howo) {
      const int oh = static_cast<int>(fdiv(static_cast<uint32_t>(f), g.div_wo));
      const int ow = f - oh * g.Wo;
      float sum = 0.0f;
      if (K3) {
#pragma unroll
        for (int kh = 0; kh < 3; ++kh) {
          const int ih = oh * g.sh + kh - g.ph;
          if (static_cast<unsigned>(ih) >= static_cast<unsigned>(g.H)) continue;
#pragma unroll
          for (int kw = 0; kw < 3; ++kw) {
            const int iw = ow * g.sw + kw - g.pw;
            if (static_cast<unsigned>(iw) < static_cast<unsigned>(g.W))
              sum += xsw[ih * g.W + iw] * wk[kh * 3 + kw];
          }
        }
      } else {
        for (int kh = 0; kh < g.KH; ++kh) {
          const int ih = oh * g.sh + kh - g.ph;
          if (static_cast<unsigned>(ih) >= static_cast<unsigned>(g.H)) continue;
          for (int kw = 0; kw < g.KW; ++kw) {
            const int iw = ow * g.sw + kw - g.pw;
            if (static_cast<unsigned>(iw) < static_cast<unsigned>(g.W))
              sum += xsw[ih * g.W + iw] * __ldg(wc + kh * g.KW + kw);
          }
        }
      }
      if (bias) sum += bv;
      const float t = qg * (sum - qm) * qi + qb;
      xout[f] = kRelu ? (t < 0.0f ? 0.0f : t) : apply_act(t, act, act_alpha);  // apply_act(t, 1)
    }
  }
  __syncwarp();
  dwgap_finish<J>(xout, y, gap, plane, howo, lane);
}


// Input planes staged per warp: 4 for planes of up to 256 elements (several
// HBM round trips in flight per warp), else 2.
template <int J, int JI>
constexpr int kDwGapStages = (J == 2 && JI == 2) ? 4 : 2;

__device__ __forceinline__ void cp_async_16(void *smem_dst, const void *gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)),
               "l"(gmem_src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// The kernel: warps take planes blockIdx.x * kDwGapWarps + warp, then every
// gridDim.x * kDwGapWarps-th; each stages its planes in a ring of
// kDwGapStages shared-memory blocks (plane_floats floats each: the larger of
// the input and output planes) with 16-byte cp.async copies issued
// kDwGapStages - 1 planes ahead, so several HBM round trips per warp overlap
// the arithmetic of the current plane.
template <int J, int JI, bool K3, bool kRelu, int SR = 0>
__global__ void __launch_bounds__(kDwGapWarps * 32) dw_bn_act_gap_kernel(
    const float *__restrict__ x, const float *__restrict__ w, const float *__restrict__ bias,
    const float *__restrict__ mean, const float *__restrict__ var,
    const float *__restrict__ gamma, const float *__restrict__ beta, float eps, int act,
    float act_alpha, float *__restrict__ y, float *__restrict__ gap, int64_t planes,
    WindowGeom g, int plane_floats, bool uniform_channel) {
  extern __shared__ __align__(16) float dwgap_smem[];
  // The softmax that follows in the chain may be scheduled now; it waits for
  // this grid's completion before reading the pooled values.
  griddep_launch_dependents();
  constexpr int NS = kDwGapStages<J, JI>;
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  float *ring = dwgap_smem + wib * (NS + 1) * plane_floats;  // NS staged input planes
  float *xout = ring + NS * plane_floats;                      // activated output
  const int hw4 = (g.H * g.W) >> 2;
  const int64_t step = static_cast<int64_t>(gridDim.x) * kDwGapWarps;
  int64_t plane = static_cast<int64_t>(blockIdx.x) * kDwGapWarps + wib;
  // One commit group per plane and lane (empty past the last plane, so the
  // group count stays the same on every lane and iteration).
  auto issue = [&](int64_t p, int st) {
    if (p < planes) {
      const float4 *x4 = reinterpret_cast<const float4 *>(x) + p * hw4;
      float4 *dst = reinterpret_cast<float4 *>(ring + st * plane_floats);
#pragma unroll
      for (int j = 0; j < JI; ++j)
        if (lane + 32 * j < hw4) cp_async_16(dst + lane + 32 * j, x4 + lane + 32 * j);
    }
    cp_async_commit();
  };
  auto channel = [&](int64_t p) {
    const uint32_t p32 = static_cast<uint32_t>(p);
    return static_cast<int>(p32 - fdiv(p32, g.div_c) * static_cast<uint32_t>(g.C));
  };
#pragma unroll
  for (int k = 0; k < NS - 1; ++k) issue(plane + k * step, k);
  // With step a multiple of C (the launch arranges it when it can) every
  // plane of this warp has the first one's channel: constants loaded once.
  DwGapConsts kc;
  int c = plane < planes ? channel(plane) : 0;
  dwgap_consts<K3>(kc, c, w, bias, mean, var, gamma, beta, eps);
  int st = 0;
  for (; plane < planes; plane += step) {
    __syncwarp();  // every lane is done with the previous plane's stage and output block
    issue(plane + (NS - 1) * step, st == 0 ? NS - 1 : st - 1);  // into the stage just freed
    cp_async_wait<NS - 1>();  // this plane's copies (issued NS - 1 groups ago) have landed
    __syncwarp();             // ... every lane's
    const float *xsw = ring + st * plane_floats;
    st = st + 1 == NS ? 0 : st + 1;
    if (!uniform_channel) {
      c = channel(plane);
      dwgap_consts<K3>(kc, c, w, bias, mean, var, gamma, beta, eps);
    }
    dwgap_plane<J, K3, kRelu, SR>(xsw, xout, plane, lane, kc,
                                  w + static_cast<int64_t>(c) * g.KH * g.KW, bias != nullptr,
                                  act, act_alpha, y, gap, g);
  }
  cp_async_wait<0>();
}

// Same-size 3x3 stride-1 pad-1 planes of R x R (R = 14 or 16): a warp takes
// four planes of one channel at a time (images 4k .. 4k+3), R / 2 lanes per
// plane, each lane two adjacent output columns down the whole plane: every
// input row's four columns are read once and folded into the output rows they
// feed in kh order (kw order within a row), so each output gets the depthwise
// kernel's sum term by term, padding entering as zero products (exact for
// finite weights; a channel with a non-finite weight takes the per-output
// form). About a third of the per-output path's instructions per plane.
constexpr int kDwQuadWarps = 4;   // warps per block
constexpr int kDwQuadStages = 2;  // staged quads per warp

template <int R>
__device__ __forceinline__ void dwquad_plane_slow(const float *xs, float *xo, int lane,
                                                  const DwGapConsts &kc, bool has_bias,
                                                  int act, float act_alpha) {
  constexpr int HW = R * R;
#pragma unroll 1
  for (int f = lane; f < HW; f += 32) {
    const int oh = f / R, ow = f - (f / R) * R;
    float sum = 0.0f;
    for (int kh = 0; kh < 3; ++kh) {
      const int ih = oh + kh - 1;
      if (static_cast<unsigned>(ih) >= static_cast<unsigned>(R)) continue;
      for (int kw = 0; kw < 3; ++kw) {
        const int iw = ow + kw - 1;
        if (static_cast<unsigned>(iw) < static_cast<unsigned>(R))
          sum += xs[ih * R + iw] * kc.wk[kh * 3 + kw];
      }
    }
    if (has_bias) sum += kc.bv;
    xo[f] = apply_act(kc.qg * (sum - kc.qm) * kc.qi + kc.qb, act, act_alpha);
  }
}

template <int R, bool kRelu>
__global__ void __launch_bounds__(kDwQuadWarps * 32) dw_bn_act_gap_quad_kernel(
    const float *__restrict__ x, const float *__restrict__ w, const float *__restrict__ bias,
    const float *__restrict__ mean, const float *__restrict__ var,
    const float *__restrict__ gamma, const float *__restrict__ beta, float eps, int act,
    float act_alpha, float *__restrict__ y, float *__restrict__ gap, int64_t n_img, int C,
    FastDiv div_c, bool uniform_channel) {
  constexpr int HW = R * R, HW4 = HW / 4, QPL = R / 2, NS = kDwQuadStages;
  constexpr int kChunks = 4 * HW4, kChunksPerLane = (kChunks + 31) / 32;
  extern __shared__ __align__(16) float dwquad_smem[];
  griddep_launch_dependents();  // as in dw_bn_act_gap_kernel
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;
  float *ring = dwquad_smem + wib * (NS + 1) * 4 * HW;  // NS stages of four planes
  float *xout = ring + NS * 4 * HW;                     // the four activated planes
  const int64_t groups = (n_img + 3) / 4;
  const int64_t quads = groups * C;
  const int64_t step = static_cast<int64_t>(gridDim.x) * kDwQuadWarps;
  int64_t q = static_cast<int64_t>(blockIdx.x) * kDwQuadWarps + wib;
  // quads < 2^31 (the entry point bounds N * C): 32-bit quotient and remainder
  auto chan = [&](int64_t qq) {
    const uint32_t q32 = static_cast<uint32_t>(qq);
    return static_cast<int>(q32 - fdiv(q32, div_c) * static_cast<uint32_t>(C));
  };
  auto group0 = [&](int64_t qq) {
    return static_cast<int64_t>(fdiv(static_cast<uint32_t>(qq), div_c)) * 4;
  };
  auto issue = [&](int64_t qq, int st) {
    if (qq < quads) {
      const int c = chan(qq);
      const int64_t n0 = group0(qq);
      float *dst = ring + st * 4 * HW;
#pragma unroll
      for (int j = 0; j < kChunksPerLane; ++j) {
        const int k = lane + 32 * j;
        const int i = k / HW4, off = k - (k / HW4) * HW4;
        if (k < kChunks && n0 + i < n_img)
          cp_async_16(dst + i * HW + 4 * off,
                      x + ((n0 + i) * C + c) * static_cast<int64_t>(HW) + 4 * off);
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int k = 0; k < NS - 1; ++k) issue(q + k * step, k);
  DwGapConsts kc;
  int c = q < quads ? chan(q) : 0;
  dwgap_consts<true>(kc, c, w, bias, mean, var, gamma, beta, eps);
  const int pl = lane / QPL, col0 = 2 * (lane - pl * QPL);
  int st = 0;
  for (; q < quads; q += step) {
    __syncwarp();  // every lane is done with the previous quad's stage and output blocks
    issue(q + (NS - 1) * step, st == 0 ? NS - 1 : st - 1);
    cp_async_wait<NS - 1>();
    __syncwarp();
    const float *xs = ring + st * 4 * HW;
    st = st + 1 == NS ? 0 : st + 1;
    if (!uniform_channel) {
      c = chan(q);
      dwgap_consts<true>(kc, c, w, bias, mean, var, gamma, beta, eps);
    }
    const int64_t n0 = group0(q);
    bool finite = true;
#pragma unroll
    for (int t = 0; t < 9; ++t) finite = finite && isfinite(kc.wk[t]);
    if (finite) {
      const bool active = pl < 4 && n0 + pl < n_img;
      const float *xp = xs + (pl < 4 ? pl : 0) * HW;
      float acc[R][2];
#pragma unroll
      for (int r = 0; r < R; ++r) acc[r][0] = acc[r][1] = 0.0f;
#pragma unroll
      for (int t = 0; t < R + 2; ++t) {  // input rows -1 .. R
        const int ih = t - 1;
        const bool rin = active && ih >= 0 && ih < R;
        // indices clamped into the plane, so no address leaves it
        const int base = (rin ? ih : 0) * R + col0;
        const float v0 = (rin && col0 > 0) ? xp[base - (col0 > 0 ? 1 : 0)] : 0.0f;
        const float v1 = rin ? xp[base] : 0.0f;
        const float v2 = rin ? xp[base + 1] : 0.0f;
        const float v3 = (rin && col0 + 2 < R) ? xp[base + (col0 + 2 < R ? 2 : 1)] : 0.0f;
#pragma unroll
        for (int kh = 0; kh < 3; ++kh) {
          const int r = t - kh;  // output row r takes input row ih as its tap row kh
          if (r >= 0 && r < R) {
            acc[r][0] += v0 * kc.wk[kh * 3 + 0];
            acc[r][0] += v1 * kc.wk[kh * 3 + 1];
            acc[r][0] += v2 * kc.wk[kh * 3 + 2];
            acc[r][1] += v1 * kc.wk[kh * 3 + 0];
            acc[r][1] += v2 * kc.wk[kh * 3 + 1];
            acc[r][1] += v3 * kc.wk[kh * 3 + 2];
          }
        }
      }
      if (active) {
        float *xo = xout + pl * HW + col0;
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float o[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            float sum = acc[r][e];
            if (bias) sum += kc.bv;
            const float t = kc.qg * (sum - kc.qm) * kc.qi + kc.qb;
            o[e] = kRelu ? (t < 0.0f ? 0.0f : t) : apply_act(t, act, act_alpha);
          }
          *reinterpret_cast<float2 *>(xo + r * R) = make_float2(o[0], o[1]);
        }
      }
    } else {
      for (int i = 0; i < 4; ++i)
        if (n0 + i < n_img)
          dwquad_plane_slow<R>(xs + i * HW, xout + i * HW, lane, kc, bias != nullptr, act,
                               act_alpha);
    }
    __syncwarp();
#pragma unroll 1
    for (int i = 0; i < 4; ++i) {
      const int64_t n = n0 + i;
      if (n >= n_img) break;
      dwgap_finish<(HW4 + 31) / 32>(xout + i * HW, y, gap, n * C + c, HW, lane);
    }
  }
  cp_async_wait<0>();
}

template <int R, bool kRelu>
int launch_dw_quad(cudaStream_t s, const float *x, const float *w, const float *bias,
                   const float *mean, const float *var, const float *gamma, const float *beta,
                   float eps, int act, float act_alpha, float *y, float *gap, int64_t n_img,
                   int C) {
  auto kernel = dw_bn_act_gap_quad_kernel<R, kRelu>;
  const size_t smem =
      static_cast<size_t>(kDwQuadWarps) * (kDwQuadStages + 1) * 4 * R * R * sizeof(float);
  const int rc = ensure_dynamic_smem(reinterpret_cast<const void *>(kernel), static_cast<int>(smem));
  if (rc) return rc;
  // Up to 6 blocks per SM (shared memory: 37.6 KB per block for 14 x 14); when
  // it fits, a warp count that is a multiple of C
  // (each warp then keeps one channel's constants).
  const int64_t quads = (n_img + 3) / 4 * C;
  const int64_t want = ceil_div(quads, kDwQuadWarps), cap = static_cast<int64_t>(sm_count()) * 6;
  int64_t grid = want < cap ? want : cap;
  const int64_t unit = C / std::gcd(static_cast<int64_t>(C), static_cast<int64_t>(kDwQuadWarps));
  if (grid < want && unit <= cap) grid = cap / unit * unit;
  kernel<<<static_cast<int>(grid), kDwQuadWarps * 32, smem, s>>>(
      x, w, bias, mean, var, gamma, beta, eps, act, act_alpha, y, gap, n_img, C,
      make_fastdiv(static_cast<uint32_t>(C)), (grid * kDwQuadWarps) % C == 0);
  return kOk;
}

template <int J, int JI, bool K3, bool kRelu, int SR = 0>
int launch_dw_gap_one(cudaStream_t s, int grid, size_t smem, const float *x, const float *w,
                      const float *bias, const float *mean, const float *var,
                      const float *gamma, const float *beta, float eps, int act, float act_alpha,
                      float *y, float *gap, int64_t planes, const WindowGeom &g, int pf) {
  auto kernel = dw_bn_act_gap_kernel<J, JI, K3, kRelu, SR>;
  if (smem > 48 * 1024) {
    const int rc = ensure_dynamic_smem(reinterpret_cast<const void *>(kernel), static_cast<int>(smem));
    if (rc) return rc;
  }
  kernel<<<grid, kDwGapWarps * 32, smem, s>>>(x, w, bias, mean, var, gamma, beta, eps, act,
                                               act_alpha, y, gap, planes, g, pf,
                                               (static_cast<int64_t>(grid) * kDwGapWarps) % g.C == 0);
  return kOk;
}

template <int J, int JI>
int launch_dw_gap(cudaStream_t s, bool k3, int grid, const float *x, const float *w,
                  const float *bias, const float *mean, const float *var, const float *gamma,
                  const float *beta, float eps, int act, float act_alpha, float *y, float *gap,
                  int64_t planes, const WindowGeom &g) {
  const int pf = ((g.H * g.W > g.Ho * g.Wo ? g.H * g.W : g.Ho * g.Wo) + 3) & ~3;
  const size_t smem =
      static_cast<size_t>(kDwGapWarps) * (kDwGapStages<J, JI> + 1) * pf * sizeof(float);
#define NPLK_DWGAP_ARGS s, grid, smem, x, w, bias, mean, var, gamma, beta, eps, act, act_alpha, y, gap, planes, g, pf
  if constexpr (J == 2 && JI == 2) {
    // 3x3 stride 1 pad 1 on 14 x 14 / 16 x 16 planes: column strips of 7 / 8 rows
    const bool same = k3 && g.sh == 1 && g.sw == 1 && g.ph == 1 && g.pw == 1 && g.Ho == g.H &&
                      g.Wo == g.W;
    const int strip_rows = same && g.W <= 32 ? (g.Ho + 32 / g.W - 1) / (32 / g.W) : 0;
    if (strip_rows == 7 && act == 1) return launch_dw_gap_one<J, JI, true, true, 7>(NPLK_DWGAP_ARGS);
    if (strip_rows == 8 && act == 1) return launch_dw_gap_one<J, JI, true, true, 8>(NPLK_DWGAP_ARGS);
    if (strip_rows == 7) return launch_dw_gap_one<J, JI, true, false, 7>(NPLK_DWGAP_ARGS);
  }
  if (k3 && act == 1) return launch_dw_gap_one<J, JI, true, true>(NPLK_DWGAP_ARGS);
  if (k3) return launch_dw_gap_one<J, JI, true, false>(NPLK_DWGAP_ARGS);
  return launch_dw_gap_one<J, JI, false, false>(NPLK_DWGAP_ARGS);
#undef NPLK_DWGAP_ARGS
}

}  // namespace nplk

extern "C" int nplk_depthwise_bn_act_gap(void *stream, const nplk_conv_geom_t *g,
                                         const float *x, const float *w, const float *bias,
                                         const float *mean, const float *var, const float *gamma,
                                         const float *beta, float eps, int act, float act_alpha,
                                         float *y, float *gap) {
  if (!g || !x || !w || !mean || !var || !gap) return kErrInvalidArg;
  if (g->n <= 0 || g->c_in <= 0 || g->h <= 0 || g->w <= 0 || g->kh <= 0 || g->kw <= 0 ||
      g->stride_h <= 0 || g->stride_w <= 0 || g->h_out <= 0 || g->w_out <= 0 ||
      g->pad_top < 0 || g->pad_left < 0 || g->c_out != g->c_in)
    return kErrInvalidArg;
  if (act < 0 || act > 10) return kErrInvalidArg;  // nplk_activation's codes
  const int64_t hw = g->h * g->w, howo = g->h_out * g->w_out;
  // One plane per warp in shared memory, float4 groups on both sides.
  if (hw > kDwGapMaxIn || hw % 4 != 0 || howo > 4 * 32 * 4 || howo % 4 != 0 ||
      !dwgap_aligned16(x) || (y && !dwgap_aligned16(y)) ||
      g->n * g->c_in >= (int64_t(1) << 31))
    return kErrUnsupported;
  WindowGeom wg{};
  wg.C = static_cast<int>(g->c_in);
  wg.H = static_cast<int>(g->h);
  wg.W = static_cast<int>(g->w);
  wg.KH = static_cast<int>(g->kh);
  wg.KW = static_cast<int>(g->kw);
  wg.sh = static_cast<int>(g->stride_h);
  wg.sw = static_cast<int>(g->stride_w);
  wg.ph = static_cast<int>(g->pad_top);
  wg.pw = static_cast<int>(g->pad_left);
  wg.Ho = static_cast<int>(g->h_out);
  wg.Wo = static_cast<int>(g->w_out);
  wg.div_wo = make_fastdiv(static_cast<uint32_t>(wg.Wo));
  wg.div_c = make_fastdiv(static_cast<uint32_t>(wg.C));
  const int64_t planes = g->n * g->c_in;
  // up to 8 blocks (2048 threads) per SM; warps loop over the remaining
  // planes. When it fits, the warp count is a multiple of C, so that each
  // warp's planes share one channel (its constants are loaded once).
  const int64_t want = ceil_div(planes, kDwGapWarps), cap = static_cast<int64_t>(sm_count()) * 8;
  int64_t grid64 = want < cap ? want : cap;
  const int64_t unit = g->c_in / std::gcd(g->c_in, static_cast<int64_t>(kDwGapWarps));
  if (grid64 < want && unit <= cap) grid64 = cap / unit * unit;
  const int grid = static_cast<int>(grid64);
  const bool k3 = g->kh == 3 && g->kw == 3;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int j = howo <= 256 ? 2 : 4;
  const int ji = hw <= 256 ? 2 : (hw <= 512 ? 4 : 8);
  int rc;
  const bool quad = k3 && g->stride_h == 1 && g->stride_w == 1 && g->pad_top == 1 &&
                    g->pad_left == 1 && g->h == g->w && g->h_out == g->h && g->w_out == g->w &&
                    (g->h == 14 || g->h == 16) && wg.C < (1 << 20);
  if (quad && g->h == 14)
    rc = act == 1 ? launch_dw_quad<14, true>(s, x, w, bias, mean, var, gamma, beta, eps, act,
                                             act_alpha, y, gap, g->n, wg.C)
                  : launch_dw_quad<14, false>(s, x, w, bias, mean, var, gamma, beta, eps, act,
                                              act_alpha, y, gap, g->n, wg.C);
  else if (quad)
    rc = act == 1 ? launch_dw_quad<16, true>(s, x, w, bias, mean, var, gamma, beta, eps, act,
                                             act_alpha, y, gap, g->n, wg.C)
                  : launch_dw_quad<16, false>(s, x, w, bias, mean, var, gamma, beta, eps, act,
                                              act_alpha, y, gap, g->n, wg.C);
  else if (j == 2 && ji == 2)
    rc = launch_dw_gap<2, 2>(s, k3, grid, x, w, bias, mean, var, gamma, beta, eps, act, act_alpha,
                             y, gap, planes, wg);
  else if (j == 2 && ji == 4)
    rc = launch_dw_gap<2, 4>(s, k3, grid, x, w, bias, mean, var, gamma, beta, eps, act, act_alpha,
                             y, gap, planes, wg);
  else if (j == 2)
    rc = launch_dw_gap<2, 8>(s, k3, grid, x, w, bias, mean, var, gamma, beta, eps, act, act_alpha,
                             y, gap, planes, wg);
  else if (ji <= 4)
    rc = launch_dw_gap<4, 4>(s, k3, grid, x, w, bias, mean, var, gamma, beta, eps, act, act_alpha,
                             y, gap, planes, wg);
  else
    rc = launch_dw_gap<4, 8>(s, k3, grid, x, w, bias, mean, var, gamma, beta, eps, act, act_alpha,
                             y, gap, planes, wg);
  if (rc) return rc;
  count_launch();
  return launch_result();
}

extern "C" int nplk_depthwise_conv2d(void *stream, const nplk_conv_geom_t *g, const float *x,
                                     const float *w, const float *bias, float *out) {
  if (!g || !x || !w || !out) return kErrInvalidArg;
  if (g->n <= 0 || g->c_in <= 0 || g->h <= 0 || g->w <= 0 || g->kh <= 0 || g->kw <= 0 ||
      g->stride_h <= 0 || g->stride_w <= 0 || g->h_out <= 0 || g->w_out <= 0 ||
      g->pad_top < 0 || g->pad_left < 0)
    return kErrInvalidArg;
  const int64_t total = g->n * g->c_in * g->h_out * g->w_out;
  if (total >= (int64_t(1) << 31) || g->h * g->w >= (int64_t(1) << 31)) return kErrUnsupported;
  WindowGeom wg{};
  wg.C = static_cast<int>(g->c_in);
  wg.H = static_cast<int>(g->h);
  wg.W = static_cast<int>(g->w);
  wg.KH = static_cast<int>(g->kh);
  wg.KW = static_cast<int>(g->kw);
  wg.sh = static_cast<int>(g->stride_h);
  wg.sw = static_cast<int>(g->stride_w);
  wg.ph = static_cast<int>(g->pad_top);
  wg.pw = static_cast<int>(g->pad_left);
  wg.Ho = static_cast<int>(g->h_out);
  wg.Wo = static_cast<int>(g->w_out);
  wg.div_wo = make_fastdiv(static_cast<uint32_t>(wg.Wo));
  wg.div_ho = make_fastdiv(static_cast<uint32_t>(wg.Ho));
  wg.div_c = make_fastdiv(static_cast<uint32_t>(wg.C));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int rc = launch_band<0>(s, x, w, bias, out, g->n * g->c_in, wg, 0);
  if (rc != 1) return rc;
  dwconv_kernel<<<window_grid(total), 256, 0, s>>>(x, w, bias, out,
                                                   static_cast<uint32_t>(total), wg);
  count_launch();
  return launch_result();
}

extern "C" int nplk_pool2d(void *stream, int64_t n, int64_t c, int64_t h, int64_t w,
                           int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph,
                           int64_t pw, int64_t h_out, int64_t w_out, int pool_type,
                           int count_include_pad, const float *x, float *y) {
  if (n <= 0 || c <= 0 || h <= 0 || w <= 0 || kh <= 0 || kw <= 0 || sh <= 0 || sw <= 0 ||
      ph < 0 || pw < 0 || h_out <= 0 || w_out <= 0 || !x || !y)
    return kErrInvalidArg;
  if (pool_type != 0 && pool_type != 1) return kErrInvalidArg;
  const int64_t total = n * c * h_out * w_out;
  if (total >= (int64_t(1) << 31) || h * w >= (int64_t(1) << 31)) return kErrUnsupported;
  WindowGeom wg{};
  wg.C = static_cast<int>(c);
  wg.H = static_cast<int>(h);
  wg.W = static_cast<int>(w);
  wg.KH = static_cast<int>(kh);
  wg.KW = static_cast<int>(kw);
  wg.sh = static_cast<int>(sh);
  wg.sw = static_cast<int>(sw);
  wg.ph = static_cast<int>(ph);
  wg.pw = static_cast<int>(pw);
  wg.Ho = static_cast<int>(h_out);
  wg.Wo = static_cast<int>(w_out);
  wg.div_wo = make_fastdiv(static_cast<uint32_t>(wg.Wo));
  wg.div_ho = make_fastdiv(static_cast<uint32_t>(wg.Ho));
  wg.div_c = make_fastdiv(static_cast<uint32_t>(wg.C));
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int rc = pool_type == 0
                     ? launch_band<1>(s, x, nullptr, nullptr, y, n * c, wg, count_include_pad)
                     : launch_band<2>(s, x, nullptr, nullptr, y, n * c, wg, count_include_pad);
  if (rc != 1) return rc;
  if (pool_type == 0)
    pool_kernel<0><<<window_grid(total), 256, 0, s>>>(x, y, static_cast<uint32_t>(total), wg,
                                                      count_include_pad);
  else
    pool_kernel<1><<<window_grid(total), 256, 0, s>>>(x, y, static_cast<uint32_t>(total), wg,
                                                      count_include_pad);
  count_launch();
  return launch_result();
}
