// ptx.cuh - thin inline-PTX wrappers for the sm_100a primitives the kernels use:
// mbarriers (with bounded waits), TMA tiled loads, tcgen05 TMEM allocation, MMA,
// commit and TMEM loads, plus the shared-memory / instruction descriptors.
//
// Every wait here is bounded: a wait that has not completed after kWaitLimitNs of
// %globaltimer time records an error code in the kernel's device error word, sets the
// CTA's abort flag and returns false, so that all roles of the CTA leave their loops,
// drain what they issued and free TMEM. The host turns the error word into an error
// status on the next check (see runtime.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sdb {

// Wall-clock bound on any single wait inside a kernel (2 s). A correct wait in these
// kernels lasts at most a few tens of microseconds.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// Error codes written into the device error word (bit flags, OR-ed together).
enum : int {
  kErrWaitFull = 1,       // MMA issuer waited too long for a TMA stage
  kErrWaitEmpty = 2,      // TMA producer waited too long for a free stage
  kErrWaitAccFull = 4,    // epilogue waited too long for an accumulator
  kErrWaitAccEmpty = 8,   // MMA issuer waited too long for a drained accumulator
  kErrWaitDrain = 16,     // teardown waited too long for in-flight copies
  kErrAttnWait = 32,      // attention pipeline wait timed out
  kErrTpBarrier = 64,     // tensor-parallel flag barrier: a peer did not arrive in time
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits until the phase with the given parity has completed. Returns false (after
// recording `code` in *err and raising the CTA abort flag) if the wait exceeds
// kWaitLimitNs, or if another role of the CTA has already aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int* err,
                                          int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        *abort_flag = 1;
        if (err) atomicOr(err, code);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------------------
// TMA (tiled, no multicast)
// ---------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// Loads box {x: inner, y: outer} of a 2-D tensor map into shared memory; completion
// is signalled on `bar` as transaction bytes.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
// Same with an L2 eviction-priority hint (policy from createpolicy).
__device__ __forceinline__ void tma_load_2d_hint(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, "
      "%4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
// 4-D box {x, y, z, w}: x is the innermost (contiguous) coordinate and must be a
// multiple of 16 bytes; the others may be negative or past the extent (zero fill).
__device__ __forceinline__ void tma_load_4d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z,
                                            int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---------------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, commit, loads, fences
// ---------------------------------------------------------------------------------
// Executed by one full warp. Writes the TMEM base address to *slot (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// ---- pairs of CTAs (cluster of 2) sharing one MMA: tcgen05 .cta_group::2 -------------
// Rank of this CTA in its cluster.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Shared::cluster address of the variable at `p` (this CTA's shared memory) in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
// Arrive (release, cluster scope) on an mbarrier given by its shared::cluster address.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// All threads of both CTAs of the cluster.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// TMA 2-D tile load into this CTA's shared memory that completes its bytes on an mbarrier
// of either CTA of the pair (shared::cluster address), without multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}
// 4-D form of tma_load_2d_pair (x innermost, 16-byte aligned; no multicast).
__device__ __forceinline__ void tma_load_4d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster, int x,
                                                 int y, int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, "
      "%5, %6}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}
// TMEM allocation shared by the pair: the same warp of both CTAs executes it with the
// same slot address, and both get the same columns.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// One M=256 MMA over the pair (issued by the leader CTA): A rows 0..127 from the leader's
// shared memory and 128..255 from the peer's (same offsets), B columns split in halves
// the same way; each CTA's TMEM receives its 128 rows of D.
__device__ __forceinline__ void umma_f16_ss_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_tf32_ss_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                  uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrives once on the mbarrier at `bar`'s offset in every CTA of `cta_mask` when the pair
// MMAs issued so far by this thread have completed.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 / fp16 operands, fp32 accumulate).
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// kind::tf32 (fp32 operands read as tf32, fp32 accumulate).
__device__ __forceinline__ void umma_tf32_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// A operand from TMEM (kind::f16): D[tmem] (+)= A[tmem] * B[smem]^T.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Eight back-to-back kind::f16 MMAs (K = 8 x 16) into one accumulator from a single asm
// block, with every descriptor computed beforehand: one issued instruction per MMA, so a
// warp that shares its scheduler with busy warps still keeps the tensor pipe fed. The
// first MMA accumulates iff acc_first != 0, the other seven always do.
__device__ __forceinline__ void umma8_f16_ss(uint32_t d_tmem, const uint64_t (&a)[8], const uint64_t (&b)[8],
                                             uint32_t idesc, uint32_t acc_first) {
  asm volatile(
      "{\n\t.reg .pred p0, p1;\n\t"
      "setp.ne.b32 p0, %17, 0;\n\t"
      "setp.eq.b32 p1, %17, %17;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %9, %18, p0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %10, %18, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %11, %18, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %4, %12, %18, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %5, %13, %18, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %6, %14, %18, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %7, %15, %18, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %8, %16, %18, p1;\n\t"
      "}\n" ::"r"(d_tmem),
      "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(a[4]), "l"(a[5]), "l"(a[6]), "l"(a[7]), "l"(b[0]), "l"(b[1]),
      "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5]), "l"(b[6]), "l"(b[7]), "r"(acc_first), "r"(idesc)
      : "memory");
}

// Four back-to-back kind::f16 MMAs (K = 4 x 16), as umma8_f16_ss.
__device__ __forceinline__ void umma4_f16_ss(uint32_t d_tmem, const uint64_t (&a)[4], const uint64_t (&b)[4],
                                             uint32_t idesc, uint32_t acc_first) {
  asm volatile(
      "{\n\t.reg .pred p0, p1;\n\t"
      "setp.ne.b32 p0, %9, 0;\n\t"
      "setp.eq.b32 p1, %9, %9;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %5, %10, p0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %2, %6, %10, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %3, %7, %10, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %4, %8, %10, p1;\n\t"
      "}\n" ::"r"(d_tmem),
      "l"(a[0]), "l"(a[1]), "l"(a[2]), "l"(a[3]), "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "r"(acc_first),
      "r"(idesc)
      : "memory");
}

// Four back-to-back kind::f16 MMAs with the A operand in tensor memory, as umma8_f16_ts.
__device__ __forceinline__ void umma4_f16_ts(uint32_t d_tmem, const uint32_t (&a)[4], const uint64_t (&b)[4],
                                             uint32_t idesc, uint32_t acc_first) {
  asm volatile(
      "{\n\t.reg .pred p0, p1;\n\t"
      "setp.ne.b32 p0, %9, 0;\n\t"
      "setp.eq.b32 p1, %9, %9;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %5, %10, p0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%2], %6, %10, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%3], %7, %10, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%4], %8, %10, p1;\n\t"
      "}\n" ::"r"(d_tmem),
      "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "l"(b[0]), "l"(b[1]), "l"(b[2]), "l"(b[3]), "r"(acc_first),
      "r"(idesc)
      : "memory");
}

// As umma8_f16_ss with the A operand in tensor memory: a[i] is the TMEM address of the
// i-th 16-wide K slice (8 columns of 16-bit pairs further on per slice).
__device__ __forceinline__ void umma8_f16_ts(uint32_t d_tmem, const uint32_t (&a)[8], const uint64_t (&b)[8],
                                             uint32_t idesc, uint32_t acc_first) {
  asm volatile(
      "{\n\t.reg .pred p0, p1;\n\t"
      "setp.ne.b32 p0, %17, 0;\n\t"
      "setp.eq.b32 p1, %17, %17;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %9, %18, p0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%2], %10, %18, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%3], %11, %18, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%4], %12, %18, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%5], %13, %18, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%6], %14, %18, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%7], %15, %18, p1;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%8], %16, %18, p1;\n\t"
      "}\n" ::"r"(d_tmem),
      "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(a[4]), "r"(a[5]), "r"(a[6]), "r"(a[7]), "l"(b[0]), "l"(b[1]),
      "l"(b[2]), "l"(b[3]), "l"(b[4]), "l"(b[5]), "l"(b[6]), "l"(b[7]), "r"(acc_first), "r"(idesc)
      : "memory");
}

// Arrives once on `bar` when all previously issued tcgen05 async ops of this thread
// have completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 columns of 32-bit: thread i receives columns [col, col+32) of lane (base+i).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// 32 lanes x 16 columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
// 32 lanes x 16 columns store (thread i writes lane base+i).
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// 32 lanes x 32 columns store (thread i writes columns [col, col+32) of lane base+i).
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// Makes this thread's generic-proxy shared-memory writes visible to the async proxy
// (tensor-core operand reads, TMA stores).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------------
// Descriptors
// ---------------------------------------------------------------------------------
// Shared-memory matrix descriptor for a K-major operand stored in the 128-byte
// swizzle layout that TMA writes with CU_TENSOR_MAP_SWIZZLE_128B: rows of 128 bytes,
// groups of 8 rows 1024 bytes apart (stride byte offset), descriptor version 1,
// layout code 2 (SWIZZLE_128B). The leading byte offset is unused for this layout.
__device__ __forceinline__ uint64_t sdesc_k_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;                  // LBO (ignored for swizzled K-major)
  d |= (uint64_t)(1024u >> 4) << 32;        // SBO: 8 rows x 128 B
  d |= (uint64_t)1u << 46;                  // version
  d |= (uint64_t)2u << 61;                  // SWIZZLE_128B
  return d;
}
// Descriptor for an MN-major operand in 128-byte swizzle: 64 bf16 (128 B) contiguous
// along MN per row, one row per K index; rows 128 B apart, 8-row groups `sbo` bytes apart
// along K, and 64-element MN blocks `lbo` bytes apart.
__device__ __forceinline__ uint64_t sdesc_mn_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// Instruction descriptor: fp32 accumulator, A/B format code (1 = bf16 for kind::f16,
// 2 = tf32 for kind::tf32), K-major A (a_mn=0) or MN-major (1), same for B, M x N.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t ab_format, uint32_t a_mn, uint32_t b_mn, uint32_t M,
                                                  uint32_t N) {
  return (1u << 4) | (ab_format << 7) | (ab_format << 10) | (a_mn << 15) | (b_mn << 16) | ((N >> 3) << 17) |
         ((M >> 4) << 24);
}

// ---------------------------------------------------------------------------------
// Numeric helpers
// ---------------------------------------------------------------------------------
// fp32 -> bf16 bit pattern: round to nearest even, inf/NaN truncated. This is the
// rounding the reference backend applies to the A operand (backend_cuda.cu:183-188,
// tensor.cpp:114-121), restated so the packed operand is bit-identical to it.
__device__ __forceinline__ uint16_t f32_to_bf16_rne(float f) {
  uint32_t b = __float_as_uint(f);
  if ((b & 0x7F800000u) == 0x7F800000u) return (uint16_t)(b >> 16);
  b += 0x7FFFu + ((b >> 16) & 1u);
  return (uint16_t)(b >> 16);
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  return (uint32_t)f32_to_bf16_rne(lo) | ((uint32_t)f32_to_bf16_rne(hi) << 16);
}
__device__ __forceinline__ float bf16_to_f32(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }

// Packed fp32 pairs (sm_100 fma.rn.f32x2 / add.rn.f32x2): one instruction for two
// independent round-to-nearest operations, the same results as two fmaf / two adds.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

}  // namespace sdb
