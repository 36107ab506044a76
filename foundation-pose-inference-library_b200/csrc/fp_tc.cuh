// tcgen05 / mbarrier / bulk-copy building blocks shared by the tensor-core
// kernels (fp_gemm.cu, fp_attention.cu). Inline PTX for sm_100a.
//
// Every mbarrier wait is bounded: waitBar gives up after ~2 s (or as soon as
// another role of the kernel has reported an error) and records an error code
// in a device flag the host checks, so no kernel can spin forever.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

namespace fpb {
namespace tc {

constexpr long long kTimeoutCycles = 4000000000LL;  // ~2 s at 1.9 GHz

// Programmatic dependent launch (see fp_launch.hpp): allow the next kernel in
// the stream to be scheduled / wait for the previous one to complete.
__device__ __forceinline__ void pdlTrigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdlWait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ uint32_t smemU32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbarInit(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smemU32(bar)), "r"(count));
}

__device__ __forceinline__ void mbarExpectTx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smemU32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbarArrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smemU32(bar)) : "memory");
}

__device__ __forceinline__ bool mbarTryWait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smemU32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and records `code`) after ~2 s or when another
// role already reported an error.
static __device__ __noinline__ bool waitBar(uint64_t* bar, uint32_t parity, int* err, int code) {
  const long long start = clock64();
  for (uint32_t i = 0;; ++i) {
    if (mbarTryWait(bar, parity)) return true;
    if ((i & 255u) == 255u) {
      if (*reinterpret_cast<volatile int*>(err) != 0) return false;
      if (clock64() - start > kTimeoutCycles) {
        atomicCAS(err, 0, code);
        return false;
      }
    }
  }
}

// Drain wait used on exit paths: bounded, ignores the error flag.
static __device__ __noinline__ void drainBar(uint64_t* bar, uint32_t parity) {
  const long long start = clock64();
  while (!mbarTryWait(bar, parity)) {
    if (clock64() - start > kTimeoutCycles) return;
  }
}

__device__ __forceinline__ void bulkCopy(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smemU32(dst)),
      "l"(src), "r"(bytes), "r"(smemU32(bar))
      : "memory");
}

__device__ __forceinline__ void tmaLoad2d(void* dst, const CUtensorMap* map, int c0, int c1,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, "
      "{%3, %4}], [%2];" ::"r"(smemU32(dst)),
      "l"(map), "r"(smemU32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

// ---- CTA pairs (clusters of two CTAs driving one cta_group::2 MMA) ----

__device__ __forceinline__ uint32_t clusterCtaRank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapaShared(uint32_t addr, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(addr), "r"(rank));
  return out;
}

// Every thread of both CTAs: release this CTA's prior writes, wait for the peer.
__device__ __forceinline__ void clusterSync() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive on an mbarrier given by its shared::cluster address (possibly the peer CTA's).
__device__ __forceinline__ void mbarArriveCluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

// Tiled loads for a CTA pair: the data lands in this CTA's shared memory, the
// transaction bytes are counted on the mbarrier at `bar_cluster` (the pair
// leader's), so one barrier tracks both halves of an MMA operand.
__device__ __forceinline__ void tmaLoad2dPair(void* dst, const CUtensorMap* map, int c0, int c1,
                                              uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, "
      "{%3, %4}], [%2];" ::"r"(smemU32(dst)),
      "l"(map), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}

// ---- Warp-wide issue: the whole issuing warp runs the MMA loop (its
// descriptors and loop state stay warp-uniform) and one lane, chosen by
// elect.sync, issues each tcgen05 instruction. The warp must be converged.

__device__ __forceinline__ void tcMmaElect(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tcMmaTf32Elect(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tcMmaTmemAElect(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tcMmaTf32TmemAElect(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                                    uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tcCommitElect(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smemU32(bar))
      : "memory");
}

__device__ __forceinline__ void tcMmaPairF16Elect(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                  uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tcMmaPairTf32Elect(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                   uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tcCommitPairBothElect(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n\t}" ::"r"(
          smemU32(bar)),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}

__device__ __forceinline__ void tcCommitPairOwnElect(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t"
      "elect.sync _|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smemU32(bar))
      : "memory");
}

// Bounded wait by a whole warp; lane 0's outcome is the warp's.
__device__ __forceinline__ bool warpWaitBar(uint64_t* bar, uint32_t parity, int* err, int code) {
  const bool ok = mbarTryWait(bar, parity) || waitBar(bar, parity, err, code);
  return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

__device__ __forceinline__ void tcFenceBefore() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tcFenceAfter() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

#define FPB_TMEM_LD32(taddr, r)                                                                  \
  asm volatile(                                                                                  \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "    \
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "    \
      "%28, %29, %30, %31}, [%32];"                                                              \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),      \
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),  \
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),            \
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),            \
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])             \
      : "r"(taddr))

__device__ __forceinline__ void tmemWaitLd() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor (tcgen05): start, leading (K-direction) and
// stride (M/N-direction) byte offsets, descriptor version 1, layout type.
__device__ __forceinline__ uint64_t smemDesc(uint32_t addr, uint32_t lbo, uint32_t sbo,
                                             uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(layout & 7u) << 61;
  return d;
}

constexpr uint32_t kLayoutNone = 0;
constexpr uint32_t kLayoutSw128 = 2;

__device__ __forceinline__ void tmemStoreWait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

#define FPB_TMEM_ST32(taddr, r)                                                                  \
  asm volatile(                                                                                  \
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "   \
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "    \
      "%28, %29, %30, %31, %32};" ::"r"(taddr),                                                 \
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),     \
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),          \
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),        \
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),        \
      "r"(r[29]), "r"(r[30]), "r"(r[31])                                                         \
      : "memory")

// fp32 -> TF32 with round-to-nearest (ties away), returned as an fp32 whose
// low 13 mantissa bits are zero. The tensor core reads fp32 operands of a
// kind::tf32 MMA by dropping those bits (truncation, biased toward zero), so
// every fp32 operand is rounded once when it is produced instead.
__device__ __forceinline__ float tf32Round(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Makes this thread's generic-proxy shared-memory writes visible to the async
// proxy (tensor-core operand reads through matrix descriptors).
__device__ __forceinline__ void fenceProxyAsyncSmem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Bulk tensor store of a shared-memory tile to global memory (this GPU's own
// memory, no multicast), tracked in the issuing thread's bulk groups. c0 is
// the innermost coordinate: c0 x element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tmaStore2d(const CUtensorMap* map, int c0, int c1, const void* src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map), "r"(c0),
               "r"(c1), "r"(smemU32(src))
               : "memory");
}
__device__ __forceinline__ void bulkCommit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Waits until at most N committed groups still read their shared-memory source.
template <int N>
__device__ __forceinline__ void bulkWaitRead() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Waits until every committed group has completed (its writes performed).
__device__ __forceinline__ void bulkWaitAll() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

}  // namespace tc
}  // namespace fpb
