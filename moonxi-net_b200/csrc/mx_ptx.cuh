// mx_ptx.cuh -- inline-PTX helpers for sm_100a: mbarriers, TMA tile loads,
// tcgen05 (TMEM allocation, MMA, commit, TMEM loads) and a bounded-wait
// primitive.  Every wait in this library goes through mx::wait_bar(), which
// gives up after a time limit, raises a kernel-wide abort flag and records an
// error code in a device status word; no wait can spin forever.
#pragma once
#include <cstdint>
#include <cuda.h>

namespace mx {

// Status codes written to the device status word (and returned by the ABI).
enum : int {
  kOk = 0,
  kErrInvalid = 1,
  kErrUnsupported = 2,
  kErrCuda = 3,
  kErrTimeout = 4,
  kErrNoMem = 5,
  kErrNoDevice = 6,
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void bar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void bar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool bar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on the phase with the given parity.  Returns false when the
// kernel-wide abort flag is raised (by this or another thread) or when the
// time limit passes; in the latter case it raises the abort flag and writes
// kErrTimeout (plus the call site `where`) to the status word.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity,
                                         volatile int* abort_flag, int* status,
                                         uint64_t limit_ns, int where) {
  if (bar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (bar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > limit_ns) {
      *abort_flag = 1;
      if (status) {
        atomicCAS(status, kOk, kErrTimeout);
        atomicCAS(status + 1, 0, where);
      }
      return false;
    }
  }
}

// Bound on the waits of the abort path (in-flight TMA copies landing, issued
// MMAs completing before TMEM is freed).  It is separate from the caller's
// wait limit: a caller may shorten that limit to microseconds, but work that
// was already issued always gets this long to finish before the CTA exits.
constexpr uint64_t kDrainNs = 1000000000ull;

// Bounded wait of the abort path for a phase that work already in flight
// will complete.  Returns false (and records kErrTimeout with `where` unless
// a status is already recorded) if it did not complete within kDrainNs.
__device__ __forceinline__ bool drain_wait(uint64_t* bar, uint32_t parity, int* status,
                                           int where) {
  if (bar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!bar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kDrainNs) {
      if (status) {
        atomicCAS(status, kOk, kErrTimeout);
        atomicCAS(status + 1, 0, where);
      }
      return false;
    }
  }
  return true;
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled bulk tensor load global -> shared, completion counted on `bar`.
// (x is the innermost coordinate.)  No cluster multicast anywhere.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// 3-D tiled bulk tensor load (x innermost).  No cluster multicast.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// ---------------------------------------------------------------- cp.async
// 4-byte async copy with zero fill: copies `src_bytes` (0 or 4) bytes.
__device__ __forceinline__ void cp_async_4(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
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
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Arrives (once) on `bar` when every tcgen05 op issued so far by this thread
// has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc], kind::tf32, one CTA.
__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Each thread of the warp reads 32 consecutive 32-bit columns of its TMEM lane.
__device__ __forceinline__ void tmem_ld_32cols(uint32_t taddr, uint32_t (&r)[32]) {
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
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// UMMA shared-memory descriptor for a K-major operand tile in the canonical
// swizzled layout written by TMA: rows of `row_bytes` (the swizzle span),
// 8-row groups `sbo_bytes` apart.  layout: 2 = 128B swizzle, 4 = 64B, 6 = 32B.
__device__ __forceinline__ uint64_t sdesc_kmajor(uint32_t saddr, uint32_t sbo_bytes,
                                                 uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);             // start address
  d |= static_cast<uint64_t>(1u) << 16;                             // LBO (unused here)
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;     // SBO
  d |= static_cast<uint64_t>(1u) << 46;                             // sm100 descriptor
  d |= static_cast<uint64_t>(layout & 7u) << 61;                    // swizzle mode
  return d;
}

// UMMA shared-memory descriptor for an MN-major operand tile: 16-byte groups
// contiguous along MN, swizzle-span-wide MN chunks `lbo_bytes` apart, 8-deep
// K groups `sbo_bytes` apart.
__device__ __forceinline__ uint64_t sdesc_mnmajor(uint32_t saddr, uint32_t lbo_bytes,
                                                  uint32_t sbo_bytes, uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);             // start address
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;     // LBO: next MN chunk
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;     // SBO: next K group
  d |= static_cast<uint64_t>(1u) << 46;                             // sm100 descriptor
  d |= static_cast<uint64_t>(layout & 7u) << 61;                    // swizzle mode
  return d;
}

// Instruction descriptor for kind::tf32 with fp32 accumulation, dense;
// a_mn / b_mn select MN-major (transposed) operands.
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n, bool a_mn = false,
                                                  bool b_mn = false) {
  return (1u << 4)                                   // D format: f32
         | (2u << 7)                                 // A format: tf32
         | (2u << 10)                                // B format: tf32
         | ((a_mn ? 1u : 0u) << 15)                  // A major: 0 K, 1 MN
         | ((b_mn ? 1u : 0u) << 16)                  // B major: 0 K, 1 MN
         | (static_cast<uint32_t>(n >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);    // M / 16
}

__device__ __forceinline__ uint32_t f32_to_tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return r;
}

}  // namespace mx
