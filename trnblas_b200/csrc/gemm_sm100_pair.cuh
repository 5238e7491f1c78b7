// GEMM on CTA pairs: tcgen05.mma.cta_group::2, 256 x 256 output tiles over
// two SMs. bf16 / fp16 (kF16) from the operands' own layout, and fp32 as
// 3xTF32 (kTF32x3) from the split pass's K-major hi / lo planes.
//
// A cluster of two CTAs computes one 256 x 256 tile per step of a persistent
// tile walk. CTA r (cluster rank r = 0, 1) loads rows 128 r .. 128 r + 127 of
// the tile's A block and columns 128 r .. 128 r + 127 of its B block, each
// with its own TMA loads (no multicast), into the same shared-memory offsets.
// The even CTA (the leader) issues M = 256, N = 256 MMAs that read both CTAs'
// halves and accumulate rows 128 r .. of the tile in CTA r's TMEM. Compared
// with one CTA computing a 128 x 256 tile, each SM stages half the B bytes
// per MMA cycle (32 KB of operands per 64-wide K step instead of 48 KB) and
// the pair reads a third less from L2. For 3xTF32 the saving is what makes
// the pair worth it: the three MMAs of a one-CTA 128 x 128 tile read 8 KB of
// shared memory per 64-cycle K step, all of the SM's shared-memory bandwidth
// before the TMA writes of the next stages; each CTA of a pair reads 8 KB
// per 128-cycle K step (its 128 rows of A and 128 of the 256 columns of B).
// fp32 accumulates 4-stage K chunks (K = 128) per TMEM buffer, whose partial
// sums the epilogue adds in fp32 with round-to-nearest (tensor-core
// accumulation truncates), 8 epilogue warps per CTA holding 128 columns each.
//
// Synchronisation (all waits bounded, as in the one-CTA engine):
//   full[s]   leader only: the leader's producer arms it with both CTAs'
//             bytes, both producers' loads complete on it (.cta_group::2);
//   empty[s]  each CTA: the leader's MMA commit multicasts to both;
//   accf[b]   each CTA: MMA commit multicast, the accumulator buffer b of the
//             tile is complete in both CTAs' TMEM;
//   acce[b]   leader only: 2 x EPI_WARPS arrivals, the epilogue warps of
//             each CTA (the peer's arrive remotely) have drained buffer b.
// Both CTAs allocate the same 512 TMEM columns (two 256-column buffers) with
// the pair allocator, and both free them after a cluster barrier that every
// thread of the pair reaches once its role has finished.
#pragma once

#include "gemm_sm100.cuh"

namespace tb {

template <int KIND, int STAGES>
struct PairGemmCfg {
  static constexpr bool TF32 = (KIND == kTF32x3);
  static_assert(KIND == kF16 || KIND == kTF32x3, "pair kernel: 16-bit or split 3xTF32");
  static constexpr int BM = 256, BN = 256;  // pair tile
  static constexpr int HM = 128, HN = 128;  // per-CTA halves of A rows / B columns
  static constexpr int BK = TF32 ? 32 : 64; // one 128-byte swizzle row of K
  static constexpr int NPARTS = TF32 ? 2 : 1;  // hi / lo
  static constexpr int A_TILE = HM * 128;      // bytes of one A part
  static constexpr int B_TILE = HN * 128;
  static constexpr int STAGE_BYTES = NPARTS * (A_TILE + B_TILE);  // per CTA
  static constexpr int NBUF = 2;
  static constexpr int TMEM_COLS = 512;
  // epilogue warps per CTA: 16-bit 4 (one per TMEM lane quarter, all 256
  // columns); fp32 8 (two per quarter, 128 columns of partial sums each)
  static constexpr int EPI_WARPS = TF32 ? 8 : 4;
  static constexpr int THREADS = 32 * (2 + EPI_WARPS);
  static constexpr int CHUNK_KB = TF32 ? 4 : (1 << 30);  // K blocks per TMEM accumulation
  static constexpr int BAR_BYTES = 256;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + BAR_BYTES;
  static_assert(NBUF * BN <= TMEM_COLS, "accumulators fit TMEM");
  static_assert((2 * STAGES + 2 * NBUF + 1) * 8 + 8 <= BAR_BYTES, "barrier block");
};

// Leader's MMA issue loop over the pair's stream of K blocks (tiles x num_kb),
// unrolled over the stages like the one-CTA engine's; an accumulation chunk
// ends at CHUNK_KB K blocks or at the tile's end.
template <int KIND, int STAGES>
__device__ __forceinline__ void gemm_pair_mma_role(const GemmParams& p, uint8_t* smem,
                                                   uint64_t* full_bar, uint64_t* empty_bar,
                                                   uint64_t* accf_bar, uint64_t* acce_bar,
                                                   uint32_t tmem_base, int num_kb,
                                                   long long total, const Abort& ab) {
  using Cfg = PairGemmCfg<KIND, STAGES>;
  constexpr int SB = Cfg::STAGE_BYTES;
  const uint32_t idesc_v = idesc(kAccF32, p.in_fmt, p.in_fmt, p.a_mn, p.b_mn, Cfg::BM, Cfg::BN);
  const uint32_t sa0 = smem_u32(smem);
  const uint32_t sb0 = sa0 + Cfg::NPARTS * Cfg::A_TILE;
  uint64_t ad[4], bd[4];
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    // K-major: a k step (16 bf16 / 8 tf32) advances 32 bytes in the swizzled
    // row; MN-major (16-bit only): 16 K rows = 2048 bytes
    ad[kk] = p.a_mn ? sdesc_sw128(sa0 + kk * 2048, 64 * 128, 1024) : sdesc_sw128(sa0 + kk * 32, 16, 1024);
    bd[kk] = p.b_mn ? sdesc_sw128(sb0 + kk * 2048, 64 * 128, 1024) : sdesc_sw128(sb0 + kk * 32, 16, 1024);
  }
  const int pair = static_cast<int>(blockIdx.x >> 1), npairs = static_cast<int>(gridDim.x >> 1);
  auto tile_kb = [&](int ti) -> int {  // K blocks of the pair's ti-th tile
    if (!p.tri) return num_kb;
    int bz, mb, nb, lo, hi;
    decode_tile(p, pair + ti * npairs, bz, mb, nb);
    tile_k_range(p, mb * Cfg::BM, Cfg::BM, nb * Cfg::BN, Cfg::BN, Cfg::BK, num_kb, lo, hi);
    return hi - lo;
  };
  int ti = 0;
  int cnt = total > 0 ? tile_kb(0) : 0;
  uint32_t phase = 0;
  int gc = 0;
  int kbt = 0;  // K block within the tile
  int kc = 0;   // K block within the accumulation chunk
  uint32_t d_tmem = tmem_base;
  bool stop = false;
  for (long long g = 0; g < total && !stop; g += STAGES) {
    static_for<0, STAGES>([&](auto sc) {
      constexpr int S = decltype(sc)::value;
      constexpr uint32_t OFF = static_cast<uint32_t>(S) * SB;
      if (stop || g + S >= total) return;
      if (kc == 0) {
        const int buf = gc & 1;
        const uint32_t bph = (gc >> 1) & 1;
        if (!mbar_wait(&acce_bar[buf], bph ^ 1u, ab, kTimeoutAccEmpty)) {
          stop = true;
          return;
        }
        tc_fence_after();
        d_tmem = tmem_base + buf * Cfg::BN;
      }
      if (!mbar_wait(&full_bar[S], phase, ab, kTimeoutFull)) {
        stop = true;
        return;
      }
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t acc_in = (kc == 0 && kk == 0) ? 0u : 1u;
        if constexpr (Cfg::TF32) {
          const uint64_t ah = sdesc_add(ad[kk], OFF), al = sdesc_add(ad[kk], OFF + Cfg::A_TILE);
          const uint64_t bh = sdesc_add(bd[kk], OFF), bl = sdesc_add(bd[kk], OFF + Cfg::B_TILE);
          mma_tf32_pair(d_tmem, al, bh, idesc_v, acc_in);  // small terms first
          mma_tf32_pair(d_tmem, ah, bl, idesc_v, 1u);
          mma_tf32_pair(d_tmem, ah, bh, idesc_v, 1u);
        } else {
          mma_f16_pair(d_tmem, sdesc_add(ad[kk], OFF), sdesc_add(bd[kk], OFF), idesc_v, acc_in);
        }
      }
      tc_commit_pair(&empty_bar[S], 0x3);
      ++kbt;
      if (++kc == Cfg::CHUNK_KB || kbt == cnt) {
        tc_commit_pair(&accf_bar[gc & 1], 0x3);
        ++gc;
        kc = 0;
      }
      if (kbt == cnt) {
        kbt = 0;
        cnt = tile_kb(++ti);
      }
    });
    phase ^= 1u;
  }
}

// map_a1 / map_b1: the lo planes for kTF32x3 (unused for kF16).
template <int KIND, int STAGES>
__global__ void __launch_bounds__(PairGemmCfg<KIND, STAGES>::THREADS, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap map_a,
                     const __grid_constant__ CUtensorMap map_a1,
                     const __grid_constant__ CUtensorMap map_b,
                     const __grid_constant__ CUtensorMap map_b1, const GemmParams p) {
  using Cfg = PairGemmCfg<KIND, STAGES>;
  constexpr uint32_t SB = Cfg::STAGE_BYTES;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * SB);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* accf_bar = empty_bar + STAGES;   // [NBUF]
  uint64_t* acce_bar = accf_bar + Cfg::NBUF;  // [NBUF], the leader's
  uint64_t* drain_bar = acce_bar + Cfg::NBUF;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = static_cast<int>(blockIdx.x >> 1);
  const int npairs = static_cast<int>(gridDim.x >> 1);
  const Abort ab{abort_flag, p.status, p.timeout_ns};

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < Cfg::NBUF; ++a) {
      mbar_init(&accf_bar[a], 1);
      mbar_init(&acce_bar[a], 2 * Cfg::EPI_WARPS);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
    if (Cfg::TF32) {
      tma_prefetch_desc(&map_a1);
      tma_prefetch_desc(&map_b1);
    }
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, Cfg::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  __syncwarp();
  cluster_sync_all();  // the peer's barriers are initialised before any remote arrive
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_kb = (p.K + Cfg::BK - 1) / Cfg::BK;
  const int my_tiles = p.num_tiles > pair ? (p.num_tiles - 1 - pair) / npairs + 1 : 0;
  long long my_total = static_cast<long long>(my_tiles) * num_kb;  // K blocks of the pair's walk
  if (p.tri) {
    my_total = 0;
    for (int t = pair; t < p.num_tiles; t += npairs) {
      int bz, mb, nb, lo, hi;
      decode_tile(p, t, bz, mb, nb);
      tile_k_range(p, mb * Cfg::BM, Cfg::BM, nb * Cfg::BN, Cfg::BN, Cfg::BK, num_kb, lo, hi);
      my_total += hi - lo;
    }
  }

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    const uint32_t full_leader = mapa_shared(smem_u32(full_bar), 0);
    int stage = 0;
    uint32_t phase = 0;
    bool aborted = false;
    int wave = 0;
    for (int t = pair; t < p.num_tiles && !aborted; t += npairs, ++wave) {
      if (p.wave_ctr && wave > 0)
        soft_wave_wait(p.wave_ctr, wave * static_cast<int>(gridDim.x), 100000ull);
      int bz, mb, nb;
      decode_tile(p, t, bz, mb, nb);
      if (p.ready && (!wait_ready(p.ready + mb / p.shard_tiles_m, p.ready_epoch, ab) ||
                      !wait_ready(p.ready + p.ready_b0 + bz, p.ready_epoch, ab))) {
        aborted = true;
        break;
      }
      const int m0 = mb * Cfg::BM + Cfg::HM * static_cast<int>(rank);
      const int n0 = nb * Cfg::BN + Cfg::HN * static_cast<int>(rank);
      const int za = p.a_batched ? bz : 0;
      const int zb = p.b_batched ? bz : 0;
      int kb_lo, kb_hi;
      tile_k_range(p, mb * Cfg::BM, Cfg::BM, nb * Cfg::BN, Cfg::BN, Cfg::BK, num_kb, kb_lo, kb_hi);
      for (int kb = kb_lo; kb < kb_hi; ++kb) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, ab, kTimeoutEmpty)) {
          aborted = true;
          break;
        }
        if (rank == 0) mbar_arrive_expect_tx(&full_bar[stage], 2 * SB);
        const uint32_t fb = full_leader + static_cast<uint32_t>(stage) * 8u;
        uint8_t* sa = smem + stage * SB;
        uint8_t* sb = sa + Cfg::NPARTS * Cfg::A_TILE;
        const int k0 = kb * Cfg::BK;
        if (Cfg::TF32) {
          // K-major hi / lo planes of the split pass
          tma_load_3d_pair(sa, &map_a, fb, k0, m0, za);
          tma_load_3d_pair(sa + Cfg::A_TILE, &map_a1, fb, k0, m0, za);
          tma_load_3d_pair(sb, &map_b, fb, k0, n0, zb);
          tma_load_3d_pair(sb + Cfg::B_TILE, &map_b1, fb, k0, n0, zb);
        } else {
          if (!p.a_mn) {
            tma_load_3d_pair(sa, &map_a, fb, k0, m0, za);
          } else {
#pragma unroll
            for (int j = 0; j < Cfg::HM / 64; ++j)
              tma_load_3d_pair(sa + j * (64 * 128), &map_a, fb, m0 + 64 * j, k0, za);
          }
          if (!p.b_mn) {
            tma_load_3d_pair(sb, &map_b, fb, k0, n0, zb);
          } else {
#pragma unroll
            for (int j = 0; j < Cfg::HN / 64; ++j)
              tma_load_3d_pair(sb + j * (64 * 128), &map_b, fb, n0 + 64 * j, k0, zb);
          }
        }
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (p.wave_ctr) atomicAdd(p.wave_ctr, 1);
    }
    if (aborted || ab.raised()) {
      // Copies already issued complete on the leader's barriers, which this
      // CTA cannot observe: give them time to land (bounded) before the exit
      // barrier.
      const unsigned long long t0 = globaltimer_ns();
      while (globaltimer_ns() - t0 < 20000000ull) {
      }
    } else {
      // Producer tail: wait until the MMA has released every stage (its
      // commits arrive on this CTA's empty barriers), so no commit is still
      // in flight towards this CTA when it passes the exit barrier.
      for (int i = 0; i < STAGES; ++i) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, ab, kTimeoutEmpty)) break;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ------------------------------------------------------------ MMA issuer (leader)
    gemm_pair_mma_role<KIND, STAGES>(p, smem, full_bar, empty_bar, accf_bar, acce_bar, tmem_base, num_kb,
                               my_total, ab);
    tc_commit_pair(drain_bar, 0x1);
    const unsigned long long t0 = globaltimer_ns();
    while (!mbar_try_wait(drain_bar, 0)) {
      if (globaltimer_ns() - t0 > 100000000ull) {  // 100 ms
        ab.raise(kTimeoutDrain);
        break;
      }
    }
  } else if (warp >= 2 && Cfg::TF32) {
    // ------------------------------------------------------------ epilogue, fp32 (both CTAs)
    // warp w: TMEM lane quarter w % 4, columns 128 * ((w - 2) / 4) .. + 127
    const int q = warp & 3;
    const int c0 = 128 * ((warp - 2) >> 2);
    const int row_in_tile = Cfg::HM * static_cast<int>(rank) + 32 * q + lane;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(32 * q) << 16) + c0;
    const uint32_t acce_leader = mapa_shared(smem_u32(acce_bar), 0);
    const int num_kb = (p.K + Cfg::BK - 1) / Cfg::BK;
    int gc = 0;
    bool aborted = false;
    for (int t = pair; t < p.num_tiles && !aborted; t += npairs) {
      int bz, mb, nb;
      decode_tile(p, t, bz, mb, nb);
      const int r = mb * Cfg::BM + row_in_tile;
      const int n0 = nb * Cfg::BN + c0;
      // K chunks: partial sums added here with round-to-nearest
      float sum[128];
#pragma unroll
      for (int j = 0; j < 128; ++j) sum[j] = 0.0f;
      int kb_lo, kb_hi;
      tile_k_range(p, mb * Cfg::BM, Cfg::BM, nb * Cfg::BN, Cfg::BN, Cfg::BK, num_kb, kb_lo, kb_hi);
      for (int kb0 = kb_lo; kb0 < kb_hi; kb0 += Cfg::CHUNK_KB, ++gc) {
        const int buf = gc & 1;
        const uint32_t bph = (gc >> 1) & 1;
        if (!mbar_wait_warp(&accf_bar[buf], bph, ab, kTimeoutAccFull)) {
          aborted = true;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 8; ++c) {  // 16 columns a load: fewer live registers
          uint32_t v[16];
          tmem_ld16(lane_base + buf * Cfg::BN + c * 16, v);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) sum[c * 16 + j] += u2f(v[j]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(acce_leader + static_cast<uint32_t>(buf) * 8u);
      }
      if (aborted) break;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        if (n0 + c * 32 < p.N) epilogue_row32(p, bz, r, n0 + c * 32, sum + c * 32);
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue, 16-bit (both CTAs)
    const int q = warp & 3;
    const int row_in_tile = Cfg::HM * static_cast<int>(rank) + 32 * q + lane;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(32 * q) << 16);
    const uint32_t acce_leader = mapa_shared(smem_u32(acce_bar), 0);
    int gc = 0;
    for (int t = pair; t < p.num_tiles; t += npairs) {
      int bz, mb, nb;
      decode_tile(p, t, bz, mb, nb);
      const int r = mb * Cfg::BM + row_in_tile;
      const int n0 = nb * Cfg::BN;
      const int buf = gc & 1;
      const uint32_t bph = (gc >> 1) & 1;
      ++gc;
      if (!mbar_wait_warp(&accf_bar[buf], bph, ab, kTimeoutAccFull)) break;
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < Cfg::BN / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(lane_base + buf * Cfg::BN + c * 32, v);
        tmem_ld_wait();
        if (n0 + c * 32 < p.N) {
          float f[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) f[j] = u2f(v[j]);
          epilogue_row32(p, bz, r, n0 + c * 32, f);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acce_leader + static_cast<uint32_t>(buf) * 8u);
    }
  }

  // Every role has finished (all waits are bounded): after this barrier no
  // MMA reads either CTA's shared memory and no remote arrive is pending.
  tc_fence_before();
  __syncthreads();
  __syncwarp();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace tb
