// sm100.cuh -- thin inline-PTX layer over the Blackwell (sm_100a) features the
// attention kernels use: mbarriers with bounded waits, TMA tensor copies,
// TMEM allocation, tcgen05.mma (UMMA) and tcgen05.ld/st, plus the shared
// memory and instruction descriptor encodings of UMMA.
//
// Shared-memory operand layout used throughout: "K-major, 128-byte swizzle".
// A tile of R rows x 64 bf16 columns (128 bytes per row) is stored row after
// row; the 16-byte chunk j of row r lands at chunk j ^ (r % 8).  The tile base
// is 1024-byte aligned, so the swizzle is a function of the address bits and
// TMA (CU_TENSOR_MAP_SWIZZLE_128B) and UMMA (layout type SWIZZLE_128B) agree
// on it.  Wider tiles are stored as consecutive 64-column blocks.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace ma {
namespace sm100 {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------- register split
// setmaxnreg: a whole warpgroup (4 aligned warps) lowers or raises its
// per-thread register budget.  Increases draw only on what other warpgroups
// of the same CTA released, so a split must sum to the CTA's launch
// allocation (threads x registers at launch); launchers check the compiled
// register count before relying on a split.
template <uint32_t N>
__device__ __forceinline__ void reg_dealloc() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void reg_alloc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

// ------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for phase `parity` of the barrier for at most `limit_ns` of wall time
// (checked every 256 failed polls).  On time-out it sets `*abort` (a shared
// flag all roles poll) and returns false; the caller must then wind down.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort,
                                          uint64_t limit_ns = 2000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (*abort) return false;
      if (globaltimer_ns() - t0 > limit_ns) {
        *abort = 1;
        return false;
      }
    }
  }
}

// Waits for phase `parity` for at most `limit_ns`, without looking at the
// abort flag: the wind-down after a time-out uses it to let the copies and
// tensor-core work it issued itself complete before the CTA frees its TMEM
// and exits.  Returns whether the phase completed.
__device__ __forceinline__ bool mbar_wait_for(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 0 && globaltimer_ns() - t0 > limit_ns) return false;
  }
}

// Limit of the wind-down waits above (in-flight copies and UMMAs finish in
// microseconds).
constexpr uint64_t kDrainLimitNs = 100000000ull;

// After a time-out: waits for the last armed phase of every slot of a ring of
// `nslots` full barriers (bar(s) for slot s), of which `armed` phases were
// armed in total in slot order, i.e. for the TMA loads still in flight into
// the ring.  Called by the thread that armed them.
template <typename BarFn>
__device__ __forceinline__ void drain_ring(BarFn bar, uint32_t nslots, uint32_t armed) {
  for (uint32_t s = 0; s < nslots && s < armed; ++s) {
    const uint32_t last = s + nslots * ((armed - 1 - s) / nslots);  // last arming of slot s
    mbar_wait_for(bar(s), (last / nslots) & 1u, kDrainLimitNs);
  }
}

// mbar_wait for roles that run whole warps: the result is made warp-uniform
// (all lanes fail if any lane failed), so warp-collective instructions that
// follow (tcgen05.ld/st, shuffles, votes) always see a converged warp.
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, volatile int* abort) {
  const bool ok = mbar_wait(bar, parity, abort);
  return __all_sync(0xffffffffu, ok);
}

// Named barrier `id` over `nthreads` threads that also returns the AND of
// every participant's `v` (bar.red.and.pred), so a group can agree on a flag.
__device__ __forceinline__ bool bar_red_and(uint32_t id, uint32_t nthreads, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void bar_sync_named(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ------------------------------------------------- cluster launch control
// A persistent-style kernel launched with one CTA per work unit: a running
// CTA asks the hardware to cancel the launch of a CTA that has not started
// yet and takes over its unit, so fast SMs take more units and the grid ends
// when the work does.  The 16-byte response lands in shared memory at `resp`
// (16-byte aligned) and completes `bar`, which the caller armed for 16 bytes.
__device__ __forceinline__ void clc_try_cancel(uint32_t resp, uint32_t bar) {
  asm volatile(
      "clusterlaunchcontrol.try_cancel.async.shared::cta.mbarrier::complete_tx::bytes.b128 [%0], [%1];" ::"r"(resp),
      "r"(bar)
      : "memory");
}

// The x index of the CTA a completed response cancelled, or -1 when it
// cancelled none (no CTA was left to launch: the grid's work is all taken).
__device__ __forceinline__ int clc_cancelled_x(uint32_t resp) {
  uint64_t lo, hi;
  asm volatile("ld.shared.v2.u64 {%0, %1}, [%2];" : "=l"(lo), "=l"(hi) : "r"(resp) : "memory");
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .b128 rr;\n\t.reg .pred p;\n\t"
      "mov.b128 rr, {%1, %2};\n\t"
      "clusterlaunchcontrol.query_cancel.is_canceled.pred.b128 p, rr;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "l"(lo), "l"(hi));
  if (!ok) return -1;
  uint32_t x;
  asm volatile(
      "{\n\t.reg .b128 rr;\n\t"
      "mov.b128 rr, {%1, %2};\n\t"
      "clusterlaunchcontrol.query_cancel.get_first_ctaid::x.b32.b128 %0, rr;\n\t}"
      : "=r"(x)
      : "l"(lo), "l"(hi));
  return (int)x;
}

// The unit sequence of a CTA scheduled by launch control: unit 0 is its own
// (blockIdx.x); unit g >= 1 is the one response g-1 names, in slot
// (g-1) % kSchedSlots of a ring of 16-byte responses with a full barrier (the
// requester's) and an empty barrier (one arrival per reader) per slot.
constexpr uint32_t kSchedSlots = 4;

struct Sched {
  uint32_t resp;         // slot 0's response; slot u at resp + 16u
  uint32_t full, empty;  // slot 0's barriers; slot u at + 8u
  volatile int* abort;
};

// Unit g of the sequence, or -1 when there is none (or a wait timed out:
// the abort flag is then set).  Every reader calls it once per g, in order;
// WARP: a whole warp reads (lane 0 releases the slot), else one thread.
template <bool WARP>
__device__ __forceinline__ int sched_unit(const Sched& sc, uint32_t g) {
  if (g == 0) return (int)blockIdx.x;
  const uint32_t u = (g - 1) % kSchedSlots, ph = ((g - 1) / kSchedSlots) & 1u;
  if (!(WARP ? mbar_wait_warp(sc.full + 8u * u, ph, sc.abort) : mbar_wait(sc.full + 8u * u, ph, sc.abort)))
    return -1;
  const int k = clc_cancelled_x(sc.resp + 16u * u);
  if (WARP) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(sc.empty + 8u * u);
  } else {
    mbar_arrive(sc.empty + 8u * u);
  }
  return k;
}

// The requester's side: request r (naming unit r+1) into slot r % kSchedSlots,
// once every reader has released the slot's previous response.
__device__ __forceinline__ bool sched_request(const Sched& sc, uint32_t r) {
  const uint32_t u = r % kSchedSlots;
  if (r >= kSchedSlots && !mbar_wait(sc.empty + 8u * u, ((r / kSchedSlots) - 1) & 1u, sc.abort)) return false;
  mbar_arrive_expect_tx(sc.full + 8u * u, 16);
  clc_try_cancel(sc.resp + 16u * u, sc.full + 8u * u);
  return true;
}

// After a time-out: lets the last request still in flight land.
__device__ __forceinline__ void sched_drain(const Sched& sc, uint32_t nreq) {
  if (nreq > 0)
    mbar_wait_for(sc.full + 8u * ((nreq - 1) % kSchedSlots), ((nreq - 1) / kSchedSlots) & 1u, kDrainLimitNs);
}

// ------------------------------------------------------------------ TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Bulk tensor reduction (add) of a shared-memory tile into global memory.
__device__ __forceinline__ void tma_reduce_add_3d(const CUtensorMap* map, uint32_t src, int c0,
                                                  int c1, int c2) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.3d.global.shared::cta.add.tile.bulk_group "
      "[%0, {%2, %3, %4}], [%1];" ::"l"(reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, uint32_t src, int c0, int c1) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group "
      "[%0, {%2, %3}], [%1];" ::"l"(reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, uint32_t src, int c0, int c1,
                                             int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, uint32_t src, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(src), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// ------------------------------------------------------------ TMEM / UMMA
// Allocates `ncols` TMEM columns (power of two >= 32); one full warp calls it.
// The TMEM base address is written to shared memory at `dst`.
__device__ __forceinline__ void tmem_alloc(uint32_t dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst),
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

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, bf16 inputs, fp32 accumulate.
// Issued by one thread.
__device__ __forceinline__ void umma_bf16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]^T, bf16 inputs, fp32 accumulate.  A is
// K-major in TMEM: row m in lane m, two bf16 per 32-bit column (the even K
// index in the low half), so K=16 spans 8 columns.  Issued by one thread.
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on the mbarrier once every tcgen05 operation this thread issued
// before it has completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

// UMMA shared-memory descriptor, 128-byte swizzle (layout type 2), version 1.
//   addr: byte address of the operand start (16-byte aligned)
//   lbo:  leading-dimension byte offset, sbo: stride-dimension byte offset
// For K-major operands sbo is the distance between 8-row groups (1024 B) and
// lbo is unused (16).  For MN-major operands sbo is the distance between
// 8-row groups along K (1024 B) and lbo the distance between 64-element
// blocks along M/N.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// Instruction descriptor of tcgen05.mma kind::f16: bf16 A/B, fp32 D.
// a_mn / b_mn select MN-major (1) instead of K-major (0) operands.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, int a_mn, int b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// 32 lanes x 32 bits, 16 consecutive columns: thread t of the warp gets TMEM
// lane (taddr.lane + t), columns taddr.col .. +15.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// tcgen05.wait::ld that also names the destination registers of the loads it
// waits for, so no use of them can be scheduled above the wait.
__device__ __forceinline__ void tmem_wait_ld_dep(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}

__device__ __forceinline__ void tmem_wait_ld_dep(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]),
                 "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                 "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                 "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// Waits for two batches of 32-column loads issued back to back.
__device__ __forceinline__ void tmem_wait_ld_dep(uint32_t (&a)[32], uint32_t (&b)[32]) {
  tmem_wait_ld_dep(a);
  asm volatile(""
               : "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]),
                 "+r"(b[6]), "+r"(b[7]), "+r"(b[8]), "+r"(b[9]), "+r"(b[10]), "+r"(b[11]),
                 "+r"(b[12]), "+r"(b[13]), "+r"(b[14]), "+r"(b[15]), "+r"(b[16]), "+r"(b[17]),
                 "+r"(b[18]), "+r"(b[19]), "+r"(b[20]), "+r"(b[21]), "+r"(b[22]), "+r"(b[23]),
                 "+r"(b[24]), "+r"(b[25]), "+r"(b[26]), "+r"(b[27]), "+r"(b[28]), "+r"(b[29]),
                 "+r"(b[30]), "+r"(b[31]));
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
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

// Byte offset of bf16 element (row, col) inside a K-major SW128 tile made of
// 64-column blocks of `rows` rows each.
__device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t col, uint32_t rows) {
  const uint32_t blk = col >> 6, c = col & 63u;
  const uint32_t chunk = (c >> 3) ^ (row & 7u);
  return blk * rows * 128u + row * 128u + chunk * 16u + (c & 7u) * 2u;
}

// 2^x with the MUFU.EX2 hardware approximation (PTX ex2.approx.ftz.f32).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max(a, b, c) in one instruction (three-source max.f32, sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

}  // namespace sm100
}  // namespace ma
