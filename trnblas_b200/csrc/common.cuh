// Shared sm_100a building blocks for every trnblas_b200 kernel.
//
// Inline-PTX wrappers for mbarriers, TMA tile loads, tcgen05 (MMA, TMEM
// allocation, TMEM loads, commits and fences), shared-memory matrix
// descriptors and instruction descriptors, plus the bounded-wait policy: every
// spin on an mbarrier gives up after a time limit, records a status code in a
// device word the host can read, and lets the kernel drain and exit instead of
// hanging the GPU.
//
// Layout conventions (all kernels):
//   * operand tiles are staged by TMA with the 128-byte swizzle, so one smem
//     "row" is 128 bytes (64 bf16 / 32 fp32 / 128 int8 elements) and an
//     8-row group is one 1024-byte swizzle atom; tiles start 1024-aligned;
//   * K-major tile (rows x 128 B): descriptor SBO = 1024 (8-row group stride),
//     LBO unused; one MMA k-step advances the start address by 32 bytes;
//   * MN-major tile (16-bit types only here): TMA boxes of 64 MN-elements x BK
//     K-rows placed back to back; LBO = box bytes (stride between 64-element MN
//     atoms), SBO = 1024 (8 K-row group stride); one bf16 MMA k-step (K = 16)
//     advances the start address by 16 rows = 2048 bytes.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <type_traits>

namespace tb {

// ---------------------------------------------------------------------------
// Kernel status codes (written to the per-device status word on failure).
// ---------------------------------------------------------------------------
enum Status : int {
  kOk = 0,
  kTimeoutFull = 1,     // MMA issuer waited too long for a TMA stage
  kTimeoutEmpty = 2,    // producer waited too long for a free stage
  kTimeoutAccFull = 3,  // epilogue waited too long for an accumulator
  kTimeoutAccEmpty = 4, // MMA issuer waited too long for a drained accumulator
  kTimeoutDrain = 5,    // exit path could not drain in-flight copies
  kTimeoutTest = 6,     // the deliberate short wait of the status self-test
  kTimeoutAux = 7,      // converter / auxiliary warp wait
};

// Default bound for one wait: 4 s. A healthy wait lasts microseconds; the bound
// only has to be far above the longest legitimate wait (one output tile's
// whole K loop) and short enough that a broken pipeline returns promptly.
constexpr unsigned long long kDefaultTimeoutNs = 4000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t elect_lane0() {
  return (threadIdx.x & 31u) == 0u;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
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
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Per-CTA failure flag in shared memory: once any role times out, every other
// role stops waiting at its next check and the CTA winds down.
struct Abort {
  volatile int* flag;  // shared memory
  int* status;         // global per-device status word
  unsigned long long timeout_ns;

  __device__ __forceinline__ bool raised() const { return *flag != 0; }
  __device__ __forceinline__ void raise(int code) const {
    *flag = 1;
    atomicCAS(status, 0, code);
  }
};

// Wait for the phase of `bar` with parity `parity` to complete. Returns false
// (after recording `code`) when the bound runs out or another role aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, const Abort& ab,
                                          int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (ab.raised()) return false;
    if (globaltimer_ns() - t0 > ab.timeout_ns) {
      ab.raise(code);
      return false;
    }
  }
}

// Warp-uniform wait for code paths that go on to warp-collective
// (.sync.aligned) tcgen05 instructions: lane 0 waits, every lane gets the
// same answer, so the warp never splits between "proceed" and "give up".
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, const Abort& ab,
                                               int code) {
  int ok = 0;
  if ((threadIdx.x & 31u) == 0u) ok = mbar_wait(bar, parity, ab, code) ? 1 : 0;
  ok = __shfl_sync(0xffffffffu, ok, 0);
  return ok != 0;
}

// Soft wave barrier of a persistent work walk: the producer waits until
// every CTA has issued the loads of its previous work item (`target`
// arrivals on the launch's counter), so the CTAs start their items together
// and read the operand slabs they share while those are still in L2 (left
// alone, CTAs drift apart over a long K loop and each re-reads from DRAM what
// the others loaded). Only a performance hint: after `limit_ns` the producer goes
// on regardless, so a CTA that is not resident cannot hold the others up.
__device__ __forceinline__ void soft_wave_wait(const int* ctr, int target,
                                               unsigned long long limit_ns) {
  const unsigned long long t0 = globaltimer_ns();
  while (*reinterpret_cast<const volatile int*>(ctr) < target) {
    if (globaltimer_ns() - t0 > limit_ns) break;
    __nanosleep(128);
  }
}

// ---------------------------------------------------------------------------
// TMA (no multicast anywhere in this library)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_load_5d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2, int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2),
      "r"(c3), "r"(c4)
      : "memory");
}

// Contiguous bulk copy global -> shared (no tensor map, no multicast):
// 16-byte aligned addresses, size a multiple of 16, completion counted on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Make generic-proxy shared-memory writes visible to the async proxy
// (tcgen05.mma / TMA store reads of data written by ordinary stores).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, commit, fences, loads
// ---------------------------------------------------------------------------
// Whole warp. Writes the TMEM base address to *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

// Whole warp (the same warp that allocated).
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

// Arrive once on `bar` when every tcgen05.mma issued so far by this thread
// has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, one instruction; accumulate != 0 keeps D.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem), "l"(adesc),
      "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives
// row (lane base + t), columns col .. col+31 of the accumulator.
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
      : "r"(taddr));
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------
// CTA pairs (clusters of 2, tcgen05 cta_group::2). The pair shares one MMA:
// the even CTA (cluster rank 0, the "leader") issues it, each CTA holds its
// half of the operands and of the accumulator at the same shared-memory and
// TMEM offsets. Loads carry no multicast: each CTA loads its own half.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// The shared::cluster address of shared-memory address `saddr` (this CTA's
// layout) in the CTA of cluster rank `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

// All threads of both CTAs of the cluster (a hardware barrier: every thread
// of the cluster reaches it on every path, after bounded role loops).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// Arrive on an mbarrier given by its shared::cluster address (possibly in the
// peer CTA), release at cluster scope.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

// TMA tile load into this CTA's shared memory whose completion is counted on
// an mbarrier that may live in the peer CTA (cluster address): the
// .cta_group::2 form, without multicast.
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map,
                                                 uint32_t bar_cluster_addr, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// Pair TMEM allocation: the same warp of both CTAs executes it; both get the
// same columns.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// Arrive once on the mbarrier at `bar`'s offset in every CTA of `cta_mask`
// when all pair MMAs issued so far by this thread have completed.
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// Pair MMA: D (both CTAs' TMEM, 128 lanes each) (+)= A (M = 256: 128 rows in
// each CTA) * B^T (N columns: N / 2 in each CTA).
__device__ __forceinline__ void mma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_tf32_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// ---------------------------------------------------------------------------
// Descriptors
// ---------------------------------------------------------------------------
// Shared-memory matrix descriptor, 128-byte swizzle, sm_100 version field.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100
  d |= static_cast<uint64_t>(2) << 61;  // SWIZZLE_128B
  return d;
}

// MN-major 32-bit (tf32) descriptor: the 128-byte swizzle of 32-byte atoms
// (UMMA layout type 1, staged by TMA with CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B):
// rows of 128 bytes (32 MN elements) along K, `lbo` between 32-element MN
// atoms, `sbo` between 4-row K groups (512 for contiguous 128-byte rows).
// Checked with a standalone MMA against fp64 products before use.
__device__ __forceinline__ uint64_t sdesc_sw128_atom32(uint32_t saddr, uint32_t lbo_bytes,
                                                       uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100
  d |= static_cast<uint64_t>(1) << 61;  // SWIZZLE_128B with 32-byte atoms
  return d;
}

// K-major descriptor without swizzle: core matrices of 8 rows x 16 bytes
// (128 contiguous bytes), the two 16-byte K halves of a 32-byte MMA K step
// `lbo` apart, consecutive 8-row groups `sbo` apart.
__device__ __forceinline__ uint64_t sdesc_kmajor_noswz(uint32_t saddr, uint32_t lbo_bytes,
                                                       uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // sm_100 descriptor version; layout 0 = no swizzle
  return d;
}

// Calls f(std::integral_constant<int, I>{}) for I = 0 .. N-1, unrolled, so the
// body sees I as a compile-time constant.
template <int I, int N, typename F>
__device__ __forceinline__ void static_for(F&& f) {
  if constexpr (I < N) {
    f(std::integral_constant<int, I>{});
    static_for<I + 1, N>(f);
  }
}

// A descriptor moved `bytes` further into shared memory (bytes a multiple of
// 16). The start-address field holds addr >> 4 in 14 bits and shared-memory
// addresses stay below 256 KB, so the add never carries out of the field.
__host__ __device__ __forceinline__ constexpr uint64_t sdesc_add(uint64_t d, uint32_t bytes) {
  return d + static_cast<uint64_t>(bytes >> 4);
}

// Generic K-major swizzled descriptor: layout 2 = 128B, 4 = 64B, 6 = 32B.
__device__ __forceinline__ uint64_t sdesc_kmajor(uint32_t saddr, uint32_t sbo_bytes,
                                                 uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>(1) << 16;  // LBO unused for swizzled K-major
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(layout & 7u) << 61;
  return d;
}
enum : uint32_t { kSwz128 = 2, kSwz64 = 4, kSwz32 = 6 };

// Instruction descriptor fields (kind::f16 / kind::tf32 / kind::i8).
enum : uint32_t { kFmtF16 = 0, kFmtBF16 = 1, kFmtTF32 = 2, kFmtS8 = 1 };
enum : uint32_t { kAccF32 = 1, kAccS32 = 2 };

__host__ __device__ constexpr uint32_t idesc(uint32_t acc_fmt, uint32_t a_fmt, uint32_t b_fmt,
                                             uint32_t a_mn, uint32_t b_mn, uint32_t M,
                                             uint32_t N) {
  return (acc_fmt << 4) | (a_fmt << 7) | (b_fmt << 10) | (a_mn << 15) | (b_mn << 16) |
         ((N >> 3) << 17) | ((M >> 4) << 24);
}

// ---------------------------------------------------------------------------
// Small numeric helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float u2f(uint32_t u) { return __uint_as_float(u); }

// 2^n as a double, exact, for n in [-1022, 1023].
// int32 -> fp64 on the integer and fp64 pipes instead of the conversion
// unit: the double with high word 0x43300000 and low word v + 2^31 (as
// unsigned) is 2^52 + 2^31 + v exactly, and subtracting 2^52 + 2^31 is exact.
__device__ __forceinline__ double i32_to_f64(int v) {
  return __hiloint2double(0x43300000, v ^ static_cast<int>(0x80000000u)) - 4503601774854144.0;
}

// 1 / d to within an ulp or two: the hardware's approximate fp64 reciprocal
// refined by three Newton-Raphson steps r <- r + r (1 - d r) (each squares
// the relative error). For finite normal d.
__device__ __forceinline__ double recip_f64(double d) {
  double r;
  asm("rcp.approx.ftz.f64 %0, %1;" : "=d"(r) : "d"(d));
  r = fma(r, fma(-d, r, 1.0), r);
  r = fma(r, fma(-d, r, 1.0), r);
  r = fma(r, fma(-d, r, 1.0), r);
  return r;
}

__device__ __forceinline__ double pow2d(int n) {
  return __longlong_as_double(static_cast<long long>(n + 1023) << 52);
}

// v * 2^ex in two exact power-of-two steps (floor(ex/2), then the rest), so no
// intermediate over/underflows for |ex| up to ~2000.
__device__ __forceinline__ double scale2(double v, int ex) {
  const int h = (ex >= 0) ? ex / 2 : -((-ex + 1) / 2);  // floor(ex / 2)
  return (v * pow2d(h)) * pow2d(ex - h);
}

}  // namespace tb
