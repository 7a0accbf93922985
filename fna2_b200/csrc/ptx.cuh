// Thin inline-PTX wrappers for the sm_100a features the FNA2 kernels use:
// mbarriers (with a bounded, abortable wait), TMA tiled loads, tcgen05 TMEM
// allocation / MMA / load / store, and the hardware ex2 / lg2 instructions.
//
// Every wrapper is a single PTX instruction (or a short fixed sequence) taken
// from the public PTX ISA for sm_100a; nothing here is derived from compiled
// NVIDIA code.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace fna2 {

// ---------------------------------------------------------------------------
// error reporting shared by all kernels of the library
// ---------------------------------------------------------------------------
// Set (first writer wins) to a non-zero site code when a bounded wait gives up.
// Read and cleared by the host through fna2_device_status().  The library is
// built as a single translation unit, so the definition lives here.
__device__ int g_device_error = 0;

// Wait budget of one mbarrier wait before the kernel gives up (nanoseconds).
constexpr uint64_t kWaitTimeoutNs = 4000000000ull;

// Test hooks, set only through fna2_debug_watchdog(): the wait budget in use
// (kWaitTimeoutNs unless a test shortens it) and the site code of one
// mbarrier arrival that a kernel withholds so that the matching wait runs out
// (0 = none; the forward kernel supports kSiteFwdPFull).
__device__ uint64_t g_wait_limit_ns = kWaitTimeoutNs;
__device__ int g_debug_withhold = 0;
constexpr int kSiteFwdPFull = 204;  // the forward MMA thread's wait for P of query tile 0

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
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

// Slow path of a bounded wait: spins on try_wait until the phase completes,
// the CTA-wide abort flag is raised by another role, or the wait budget
// (g_wait_limit_ns, 4 s) passes.  A wait gives up only long after every copy
// and MMA that the CTA issued before it has completed, so the teardown that
// follows (TMEM deallocation, exit) has nothing in flight.
// On timeout it raises the abort flag and records `site` in g_device_error.
// The abort flag and the timer are checked once per 32 suspending try_waits,
// so a phase that completes is noticed with the hardware's wake-up latency.
__device__ __noinline__ static bool mbar_wait_slow(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                                   int site) {
  const uint64_t t0 = globaltimer_ns();
  const uint64_t limit = *reinterpret_cast<volatile uint64_t*>(&g_wait_limit_ns);
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > limit) {
      *abort_flag = 1;
      atomicCAS(&g_device_error, 0, site);
      return false;
    }
  }
}

// Bounded wait for the phase with the given parity. Returns false if the CTA
// is aborting (the caller must stop its role loop and go to the teardown).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int site) {
  if (mbar_try_wait(bar, parity)) return true;
  return mbar_wait_slow(bar, parity, abort_flag, site);
}

// Non-suspending variant for the MMA-issuing thread: polls with test_wait so
// that a completed phase is seen within a few cycles (a suspended try_wait can
// sleep for hundreds of cycles past the phase completion while the tensor
// pipe drains). Same bound and abort semantics as mbar_wait.
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __noinline__ static bool mbar_spin_slow(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                                   int site) {
  const uint64_t t0 = globaltimer_ns();
  const uint64_t limit = *reinterpret_cast<volatile uint64_t*>(&g_wait_limit_ns);
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 256; ++i)
      if (mbar_test_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > limit) {
      *abort_flag = 1;
      atomicCAS(&g_device_error, 0, site);
      return false;
    }
  }
}

__device__ __forceinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int site) {
  if (mbar_test_wait(bar, parity)) return true;
  return mbar_spin_slow(bar, parity, abort_flag, site);
}

// True in exactly one lane of the calling warp, which must be converged.  The
// MMA-issuing warps run their loops with all 32 lanes and issue each group of
// tcgen05 instructions from the lane this selects: measured on B200 with busy
// warps on the same scheduler, a group issued from an `if (lane == 0)` branch
// kept the tensor pipe at about a third of the rate of the same group issued
// under elect.sync from a converged warp (the operands stay warp-uniform).
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .b32 rx;\n\t.reg .pred px;\n\t"
      "elect.sync rx|px, 0xffffffff;\n\t"
      "@px mov.s32 %0, 1;\n\t}\n"
      : "+r"(pred));
  return pred != 0;
}

// Rendezvous of two whole warps on hardware named barrier `id` (64 threads);
// returns the AND of the `ok` values both warps pass.  This is how an
// MMA-issuing warp learns that its operands are ready from a waiter warp that
// does the mbarrier waits for it: a barrier instruction does not queue behind
// the calling warp's own outstanding tcgen05.mma instructions, whereas a
// shared- or global-memory access from that warp does (measured on B200: an
// mbarrier test on an already completed phase, issued behind queued MMAs,
// leaves the tensor pipe idle for 80-180 cycles; this rendezvous costs about
// 20).  Both warps must execute the same sequence of rendezvous; the AND
// carries an abort from the waiter to the issuer at the same point.
__device__ __forceinline__ bool pair_rendezvous(uint32_t id, bool ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "barrier.cta.red.and.aligned.pred q, %2, 64, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"(ok ? 1u : 0u), "r"(id)
      : "memory");
  return r != 0;
}

// ---------------------------------------------------------------------------
// TMA (bulk tensor copies, global -> shared, no multicast)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}

// Make generic-proxy writes to shared memory visible to the async proxy
// (tensor core operand reads, TMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: descriptors
// ---------------------------------------------------------------------------
// Shared-memory matrix descriptor (sm_100 layout): start address, leading and
// stride byte offsets (all >> 4), version 1 at bit 46, layout/swizzle at 61..63.
enum : uint32_t { kSwizzleNone = 0, kSwizzle128B = 2, kSwizzle64B = 4, kSwizzle32B = 6 };

__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                               uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(layout & 0x7u) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with BF16 A/B and FP32 accumulation.
// a_mn / b_mn: 0 = K-major, 1 = MN-major.
__host__ __device__ constexpr uint32_t make_idesc_bf16(int M, int N, int a_mn, int b_mn) {
  return (1u << 4)                                  // D format: F32
         | (1u << 7)                                // A format: BF16
         | (1u << 10)                               // B format: BF16
         | (static_cast<uint32_t>(a_mn) << 15)      // A major
         | (static_cast<uint32_t>(b_mn) << 16)      // B major
         | (static_cast<uint32_t>(N >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);   // M / 16
}

// ---------------------------------------------------------------------------
// tcgen05: MMA (single CTA), commit
// ---------------------------------------------------------------------------
// D[tmem] (+)= A[smem desc] * B[smem desc]
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]; A is M lanes x K (two bf16 per column).
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive (once) on `bar` when all previously issued tcgen05 async ops of this
// thread have completed.
// Shared memory -> tensor memory copy of a 128-row x 32-byte slice described
// by a shared-memory matrix descriptor (same layout rules as an MMA operand):
// row i lands in lane i, 8 consecutive 32-bit columns. Asynchronous; ordered
// before later tcgen05.mma of the same thread and tracked by tcgen05.commit.
__device__ __forceinline__ void tmem_cp_128x256b(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.128x256b [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ---------------------------------------------------------------------------
// CTA pairs (cluster of 2, tcgen05 cta_group::2).  The even-ranked CTA of a
// pair issues the MMAs; each operand half and each accumulator half lives at
// the same shared-memory / TMEM address in both CTAs.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Shared::cluster address of the same shared-memory location in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
// All threads of both CTAs (release / acquire at cluster scope).
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx_cluster(uint32_t cluster_addr, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cluster.shared::cluster.b64 _, [%0], %1;" ::"r"(cluster_addr),
               "r"(bytes)
               : "memory");
}
// TMA load into this CTA's shared memory (a single destination) whose
// completion is counted on an mbarrier of either CTA of the pair.
__device__ __forceinline__ void tma_load_4d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int c0,
                                                 int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, "
      "%4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar_cluster)
      : "memory");
}
// TMEM allocation of a CTA pair: executed by one warp (same warp index) in each CTA.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem, both CTAs] (+)= A * B with M = 256 over the pair (A rows and B columns
// split between the CTAs; each CTA's TMEM holds its 128 rows x N).
__device__ __forceinline__ void mma_pair_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_pair_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive (once) on `bar` -- the same shared-memory offset in both CTAs of the
// pair -- when all previously issued tcgen05 operations of this thread are done.
__device__ __forceinline__ void mma_pair_commit_both(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM <-> registers (32 lanes x 32-bit columns per warp)
// ---------------------------------------------------------------------------
#define FNA2_R8(i) "=r"(r[i]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), "=r"(r[i + 4]), "=r"(r[i + 5]), \
                   "=r"(r[i + 6]), "=r"(r[i + 7])
#define FNA2_W8(i) "+r"(r[i]), "+r"(r[i + 1]), "+r"(r[i + 2]), "+r"(r[i + 3]), "+r"(r[i + 4]), "+r"(r[i + 5]), \
                   "+r"(r[i + 6]), "+r"(r[i + 7])
#define FNA2_S8(i) "r"(r[i]), "r"(r[i + 1]), "r"(r[i + 2]), "r"(r[i + 3]), "r"(r[i + 4]), "r"(r[i + 5]), \
                   "r"(r[i + 6]), "r"(r[i + 7])

// Load 32 consecutive columns of this warp's 32 lanes (thread i <- lane base+i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : FNA2_R8(0), FNA2_R8(8), FNA2_R8(16), FNA2_R8(24)
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : FNA2_R8(0), FNA2_R8(8)
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];" : FNA2_R8(0) : "r"(taddr));
}
// Wait for outstanding tcgen05.ld; the registers are tied in so that no use
// of them can be scheduled before the wait.
__device__ __forceinline__ void tmem_ld_wait32(uint32_t* r) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : FNA2_W8(0), FNA2_W8(8), FNA2_W8(16), FNA2_W8(24)::"memory");
}
__device__ __forceinline__ void tmem_ld_wait8(uint32_t* r) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : FNA2_W8(0)::"memory");
}
__device__ __forceinline__ void tmem_ld_wait16(uint32_t* r) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : FNA2_W8(0), FNA2_W8(8)::"memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      FNA2_S8(0), FNA2_S8(8)
      : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t* r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), FNA2_S8(0)
               : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      FNA2_S8(0), FNA2_S8(8), FNA2_S8(16), FNA2_S8(24)
      : "memory");
}
__device__ __forceinline__ void tmem_st4(uint32_t taddr, const uint32_t* r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr), "r"(r[0]), "r"(r[1]),
               "r"(r[2]), "r"(r[3])
               : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

#undef FNA2_R8
#undef FNA2_W8
#undef FNA2_S8

// ---------------------------------------------------------------------------
// math: hardware MUFU instructions
// ---------------------------------------------------------------------------
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Two raw 32-bit words as the fp32 pair of a packed instruction (__ffma2_rn,
// __fadd2_rn, __fmul2_rn: two fp32 lanes per instruction on sm_100, each lane
// rounded exactly as the scalar operation).
__device__ __forceinline__ float2 f32x2(uint32_t lo, uint32_t hi) {
  return make_float2(__uint_as_float(lo), __uint_as_float(hi));
}
// Round two floats to bf16 (round-to-nearest-even) and pack them, lo in bits 0..15.
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ uint32_t lane_id() { return threadIdx.x & 31u; }
__device__ __forceinline__ uint32_t warp_id() { return threadIdx.x >> 5; }

// Store this warp's 32 rows (thread t holds row t's NU32 packed bf16 pairs) with
// coalesced writes: each thread puts its row into a shared-memory staging buffer
// (32 x 4*NU32 bytes, 16-byte granules XOR-swizzled by row), then each store
// instruction writes whole row segments of 4*NU32 bytes.  Rows r >= nvalid are
// not written.  row0 points at row 0's first element; rows are row_stride
// elements apart.
template <int NU32>
__device__ __forceinline__ void warp_store_rows(uint8_t* stage, const uint32_t* v, __nv_bfloat16* row0,
                                                int64_t row_stride, int nvalid) {
  constexpr int G = NU32 / 4;        // 16-byte granules per row
  constexpr int RPI = 32 / G;        // rows per store instruction
  const int lane = lane_id();
#pragma unroll
  for (int g = 0; g < G; ++g)
    *reinterpret_cast<uint4*>(stage + lane * (16 * G) + ((g ^ (lane % G)) * 16)) =
        make_uint4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
  __syncwarp();
#pragma unroll
  for (int i = 0; i < G; ++i) {
    const int r = RPI * i + lane / G, g = lane % G;
    const uint4 w = *reinterpret_cast<const uint4*>(stage + r * (16 * G) + ((g ^ (r % G)) * 16));
    if (r < nvalid) *reinterpret_cast<uint4*>(row0 + r * row_stride + g * 8) = w;
  }
  __syncwarp();
}

}  // namespace fna2
