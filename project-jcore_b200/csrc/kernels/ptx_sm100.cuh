// Thin inline-PTX wrappers for the sm_100a features the NPL kernels use:
// mbarriers, TMA tile loads, tcgen05 MMA / commit / TMEM load, TMEM allocation,
// and the UMMA shared-memory and instruction descriptors.
//
// Every wait on an mbarrier is bounded: after kWaitLimitNs of device time it
// records an error code in a status word in global memory, raises a CTA-wide
// abort flag in shared memory, and returns false. The caller then leaves its
// loop, so a broken pipeline ends the kernel instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cstdint>

namespace nplk {

// Status codes a kernel can record in its device status word.
enum : int {
  kStatusOk = 0,
  kStatusTimeoutProducer = 101,  // producer waited too long for a free stage
  kStatusTimeoutMma = 102,       // MMA warp waited too long for a filled stage
  kStatusTimeoutEpilogue = 103,  // epilogue waited too long for an accumulator
  kStatusTimeoutAccFree = 104,   // MMA warp waited too long for a drained accumulator
  kStatusTimeoutStage = 105,     // a consumer warp waited too long for a staged batch
};

// 4 s of device time: orders of magnitude above any legitimate stage wait.
constexpr uint64_t kWaitLimitNs = 4000000000ull;

// Upper bound on how long one try_wait may suspend the thread when the phase
// is not complete yet (the thread resumes as soon as the phase completes).
// Keeps waiting warps off the issue slots instead of spinning.
constexpr uint32_t kSuspendHintNs = 20000u;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// The first 1024-byte boundary at or after `raw` (the dynamic shared-memory
// array), reached by offsetting `raw` itself: the compiler then keeps the
// result and every pointer derived from it in the shared address space, so
// accesses through them are ld/st.shared. Aligning the address as an integer
// instead makes them generic accesses; in the conv epilogue those constant
// loads could not be scheduled ahead of its global stores, one load round
// trip per output channel (3.5 vs 1.3 kcycles per 32 channels measured).
__device__ __forceinline__ uint8_t *align_smem_1024(uint8_t *raw) {
  return raw + ((1024u - (smem_u32(raw) & 1023u)) & 1023u);
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ uint32_t mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return done;
}

// Waits until the phase with the given parity has completed. Returns false if
// the CTA was told to abort or if the wait exceeded limit_ns, in which case
// `code` is recorded in *status (first error wins) and *abort is raised.
__device__ __forceinline__ bool mbar_wait_for(uint64_t *bar, uint32_t parity,
                                              volatile int *abort, int *status, int code,
                                              uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0 = global_timer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 31u) == 0u) {
      if (*abort) return false;
      if (global_timer_ns() - t0 > limit_ns) {
        *abort = 1;
        atomicCAS(status, 0, code);
        return false;
      }
    }
  }
}

// mbar_wait_for with the kernels' standard limit, kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort,
                                          int *status, int code) {
  return mbar_wait_for(bar, parity, abort, status, code, kWaitLimitNs);
}

// Fault injection (nplk_debug_arm_wait_timeout): the MMA issuer of an armed
// launch first waits, with a limit of `stall_us` microseconds, on `never`, a
// barrier of the CTA that is initialised and never arrived on. The wait
// expires through the ordinary timeout path (status code, abort flag), and
// every other role of the CTA leaves its loop on the abort flag. Returns
// false when the CTA is aborting; true (at once) when stall_us is 0.
__device__ __forceinline__ bool injected_stall(uint64_t *never, uint32_t stall_us,
                                               volatile int *abort, int *status) {
  if (stall_us == 0u) return true;
  return mbar_wait_for(never, 0u, abort, status, kStatusTimeoutMma,
                       static_cast<uint64_t>(stall_us) * 1000ull);
}

// Bounded wait that ignores the abort flag: on the way out of an aborted CTA
// the TMA producer waits here for the copies it issued into shared memory, so
// that none lands after the CTA has exited. Returns false after
// kDrainLimitNs.
constexpr uint64_t kDrainLimitNs = 100000000ull;
__device__ __forceinline__ bool mbar_drain(uint64_t *bar, uint32_t parity) {
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_timer_ns() - t0 > kDrainLimitNs) return false;
  }
  return true;
}

// Bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) from
// global to shared memory on the async proxy; completion is counted on `bar`
// (transaction bytes). No multicast.
__device__ __forceinline__ void bulk_load_g2s(void *dst, const void *src, uint32_t bytes,
                                              uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// TMA tensor store of the 2-D box at (x, y) of `map` from shared memory
// (bulk-group completion; no multicast). The box's shared-memory image must be
// laid out as the map's swizzle mode expects.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *smem_src, int x,
                                             int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   map),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Waits until at most N committed bulk groups of this thread still read their
// shared-memory source (their global writes may still be in flight).
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Waits until at most N committed bulk groups of this thread are incomplete.
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Makes this thread's generic-proxy shared-memory writes visible to the async
// proxy (tensor-core operand reads, TMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// NVLink multicast (NVSwitch fan-out). `mc` is an address inside a multicast
// object's mapping; one store reaches the same offset of every GPU's memory
// bound to the object. 16-byte aligned.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void multimem_st_v4(float *mc, float4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc),
               "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}
// Orders this thread's accesses made through different virtual addresses of
// the same memory (a multicast address and the unicast one), then makes its
// writes visible system-wide (other GPUs, the host).
__device__ __forceinline__ void fence_multimem_release() {
  asm volatile("fence.proxy.alias;" ::: "memory");
  asm volatile("fence.acq_rel.sys;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch: a kernel launched with programmatic stream
// serialization may start while the previous kernel in the stream still
// runs; griddep_wait() blocks until that kernel has completed and its
// writes are visible (a no-op for a normally launched kernel), and
// griddep_launch_dependents() lets the next kernel start early.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// TMA (no multicast anywhere in this library)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tile load into this CTA's shared memory; completion is signalled on `bar`
// as transaction bytes. c0 is the innermost coordinate (elements).
__device__ __forceinline__ void tma_load_2d(const CUtensorMap *map, uint64_t *bar, void *dst,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// 4-D im2col load (NHWC tensor map from cuTensorMapEncodeIm2col): gathers the
// map's pixels-per-column output pixels starting at input position (w, h) of
// image n, each shifted by the filter offset (off_w, off_h), channels
// [c, c + channels-per-pixel). Positions outside the image read as zero.
__device__ __forceinline__ void tma_load_im2col_4d(const CUtensorMap *map, uint64_t *bar,
                                                   void *dst, int c, int w, int h, int n,
                                                   uint16_t off_w, uint16_t off_h) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], {%7, %8};" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c), "r"(w), "r"(h), "r"(n),
      "h"(off_w), "h"(off_h)
      : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, commit, load
// ---------------------------------------------------------------------------
// Executed by one full warp. Writes the TMEM base address to *dst_smem.
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::tf32, one CTA. Issued by one thread.
__device__ __forceinline__ void mma_tf32_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::tf32, one CTA. A occupies 128 TMEM
// lanes (one row of A per lane) and 8 consecutive 32-bit columns per K=8 step.
__device__ __forceinline__ void mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Stores 32 consecutive 32-bit TMEM columns of this thread's lane (32x32b
// shape, warp-collective). Completion is awaited with tmem_wait_st().
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Arrives once on `bar` when every tcgen05.mma issued so far by this thread
// has completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Loads 32 consecutive 32-bit TMEM columns of this thread's lane (32x32b
// shape: lane i of the warp reads TMEM lane (warp quadrant * 32 + i)). The
// values are only valid after tmem_wait_ld(), which takes them as operands
// so that no use can be scheduled before the wait.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]),
                 "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]),
                 "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// 16-column variant of tmem_ld32 (32x32b.x16).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// Waits for outstanding TMEM loads; both arrays are tied to the wait.
__device__ __forceinline__ void tmem_wait_ld16x2(uint32_t (&r)[16], uint32_t (&s)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(s[0]), "+r"(s[1]),
                 "+r"(s[2]), "+r"(s[3]), "+r"(s[4]), "+r"(s[5]), "+r"(s[6]), "+r"(s[7]),
                 "+r"(s[8]), "+r"(s[9]), "+r"(s[10]), "+r"(s[11]), "+r"(s[12]), "+r"(s[13]),
                 "+r"(s[14]), "+r"(s[15])
               :
               : "memory");
}

__device__ __forceinline__ void tmem_wait_ld2(uint32_t (&r)[32], uint32_t (&s)[32]) {
  tmem_wait_ld(r);
  // The first wait already covers both loads; this one only pins `s` after it.
  asm volatile(""
               : "+r"(s[0]), "+r"(s[1]), "+r"(s[2]), "+r"(s[3]), "+r"(s[4]), "+r"(s[5]),
                 "+r"(s[6]), "+r"(s[7]), "+r"(s[8]), "+r"(s[9]), "+r"(s[10]), "+r"(s[11]),
                 "+r"(s[12]), "+r"(s[13]), "+r"(s[14]), "+r"(s[15]), "+r"(s[16]),
                 "+r"(s[17]), "+r"(s[18]), "+r"(s[19]), "+r"(s[20]), "+r"(s[21]),
                 "+r"(s[22]), "+r"(s[23]), "+r"(s[24]), "+r"(s[25]), "+r"(s[26]),
                 "+r"(s[27]), "+r"(s[28]), "+r"(s[29]), "+r"(s[30]), "+r"(s[31])
               :
               : "memory");
}

// ---------------------------------------------------------------------------
// CTA pairs (cluster of two CTAs on neighbouring SMs, tcgen05 cta_group::2).
// The pair's leader (cluster rank 0) issues the MMAs; each MMA reads A rows
// and half of B from each CTA's shared memory at the same offsets and writes
// each CTA's own TMEM. No multicast loads: each CTA loads its own operands.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address in the shared::cluster window of the variable at local shared
// address `local` in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}

// Arrives once on an mbarrier given by its shared::cluster address (this
// CTA's or the peer's), releasing this thread's prior writes at cluster scope.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

__device__ __forceinline__ uint32_t mbar_try_wait_cluster(uint64_t *bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return done;
}

// mbar_wait with acquire at cluster scope (the barrier also receives arrivals
// from the peer CTA or the pair's MMA commits). On failure the local abort
// flag is raised and so is the peer's (`peer_abort`: its shared::cluster
// address), so both CTAs of the pair leave their loops.
__device__ __forceinline__ bool mbar_wait_pair(uint64_t *bar, uint32_t parity,
                                               volatile int *abort, uint32_t peer_abort,
                                               int *status, int code) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((it & 31u) == 0u) {
      if (*abort) return false;
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        *abort = 1;
        asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(peer_abort), "r"(1) : "memory");
        atomicCAS(status, 0, code);
        return false;
      }
    }
  }
}

// Raises the peer CTA's abort flag (shared::cluster address).
__device__ __forceinline__ void pair_raise_abort(uint32_t peer_abort) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(peer_abort), "r"(1) : "memory");
}

// Cluster-wide barrier of all threads of both CTAs (release / acquire).
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}

// TMEM allocation for a CTA pair: the same warp of both CTAs executes it and
// both receive the same base address.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// D (+)= A * B^T for the pair, kind::tf32, M = 256 (128 rows of A from each
// CTA), N given by idesc (N/2 rows of B from each CTA). Issued by one thread
// of the leader.
__device__ __forceinline__ void mma_tf32_ss_pair(uint32_t d_tmem, uint64_t a_desc,
                                                 uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// When the pair MMAs issued so far by this thread complete, arrives once on
// the mbarrier at the same shared-memory offset as `bar` in both CTAs of the
// pair (CTA mask 0b11). This is the completion signal of tcgen05, not a data
// copy: nothing is loaded or stored.
__device__ __forceinline__ void mma_commit_pair_both(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}

// 2-D tile load into this CTA's shared memory whose completion (transaction
// bytes) is signalled on the pair leader's mbarrier `leader_bar` (a
// shared::cluster address). No multicast.
__device__ __forceinline__ void tma_load_2d_pair(const CUtensorMap *map, uint32_t leader_bar,
                                                 void *dst, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(leader_bar), "r"(c0), "r"(c1)
      : "memory");
}

// ---------------------------------------------------------------------------
// UMMA descriptors
// ---------------------------------------------------------------------------
// Shared-memory matrix descriptor for a K-major operand stored in the
// 128-byte-swizzle canonical layout: rows of 128 B (32 fp32/tf32 elements of
// K), groups of 8 rows 1024 B apart, tile base 1024-byte aligned. Fields:
// start address>>4 [0,14), leading byte offset>>4 [16,30) (unused for
// swizzled K-major), stride byte offset>>4 [32,46), version=1 [46,48),
// swizzle mode [61,64) = 2 (128B).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_byte_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_byte_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(1u) << 16;
  d |= static_cast<uint64_t>(1024u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(2u) << 61;
  return d;
}

// Instruction descriptor for kind::tf32 with fp32 accumulation, both operands
// K-major: D format F32 at [4,6), A/B format TF32 (=2) at [7,10)/[10,13),
// N>>3 at [17,23), M>>4 at [24,29).
// MN-major fp32 (tf32) operand. The only MN-major shared-memory layout the
// tensor core takes for 32-bit types is the 128-byte swizzle with 32-byte
// atoms (descriptor layout type 1; TMA CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B):
// 32 values along M/N per 128-byte row, rows along K, the swizzle repeating
// every 4 rows. `lbo_bytes` between 32-wide M/N atoms, 512 bytes between
// 4-row K groups; a K = 8 step adds 1024 bytes (+64 in the address field).
// (Measured on this part: the plain 128-byte swizzle reads as zeros.)
__device__ __forceinline__ uint64_t umma_desc_mn_sw128_32b(uint32_t smem_byte_addr,
                                                           uint32_t lbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_byte_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>(512u >> 4) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(1u) << 61;
  return d;
}
// Instruction descriptor bit of an MN-major B operand.
constexpr uint32_t kUmmaIdescBMajorMN = 1u << 16;

__host__ __device__ constexpr uint32_t umma_idesc_tf32(int m, int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

// ---------------------------------------------------------------------------
// TF32 splitting for 3xTF32: x = hi + lo with hi = rna_tf32(x) and
// lo = rna_tf32(x - hi). hi*hi + hi*lo + lo*hi recovers the fp32 product to
// about 2^-22 relative error.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// x = hi + lo with hi = rna_tf32(x). +-inf splits into (x, 0) -- not
// (inf, inf - inf = NaN) -- and a finite x that rounds up to inf is truncated
// instead, so that hi + lo keeps x's value class.
__device__ __forceinline__ void tf32_split(float x, float &hi, float &lo) {
  hi = tf32_rna(x);
  if (fabsf(hi) == __int_as_float(0x7f800000)) {
    if (fabsf(x) != __int_as_float(0x7f800000)) hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
    else {
      lo = 0.0f;
      return;
    }
  }
  lo = tf32_rna(x - hi);
}

// Cheaper split for operands produced inside a kernel's hot loop: hi keeps the
// top 10 mantissa bits (truncation, exactly representable in tf32) and
// lo = x - hi is exact in fp32; the tensor core then uses lo's top 10 mantissa
// bits. Per-product error stays below 2^-20 relative (vs 2^-22 with rounding),
// far under the fp32 accumulation error of the dot products.
__device__ __forceinline__ void tf32_split_trunc(float x, float &hi, float &lo) {
  hi = __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
  lo = x - hi;
}

// Byte offset of 16-byte chunk `chunk` (0..7) of row `row` inside a tile laid
// out in the 128-byte-swizzle pattern (chunk index XOR row mod 8).
__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

}  // namespace nplk
