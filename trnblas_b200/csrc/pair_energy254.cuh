// Fused DF-MP2 pair energy, base-254 digit form: 10 int8 slice products.
//
// The pair walk and work units are those of pair_energy.cu (units of one
// pair (i, j), a 128-row block R of a and a 64-column block C >= 2R of b;
// X = B_i[R] B_j[C]^T and Y = B_j[R] B_i[C]^T in the same TMEM lanes and
// columns).
//
// Digits. B is split per row (i, a) into KS = 4 balanced base-254 digits:
// with e the frexp exponent of the row's max |B| and u = B * 127 * 2^-e
// (exact in fp64, |u| < 127), d_0 = rint(u), then repeatedly
// u = 254 (u - d_s), d_{s+1} = rint(u) (every step is exact in fp64 for fp32
// B: each one drops a fractional bit); |d| <= 127 and
//     B = 2^e / 127 (d_0 + d_1 / 254 + d_2 / 254^2 + d_3 / 254^3) + r,
// |r| <= 2^e * 2.4e-10. T keeps the diagonals s + t <= 3 of the slice
// products (10 products, 4 int32 accumulators per column):
//     T_ab = 2^(e_ia + e_jb) / 127^2 * sum_{d <= 3} 254^-d S_d,
// every S_d exact in int32 while 4 * 127^2 * naux < 2^31 (naux <= 33280).
// Longer naux runs each X and Y pass as chunks of at most 33280 (520 stages)
// of K, each a TMEM accumulation of its own whose fold the epilogue adds in
// fp64.
//
// The truncation errors of different rows are independent, so they average
// out in E, except on the diagonal elements T_aa = sum_P B_ia^2 of the pairs
// i == j, where a digit multiplies itself and the dropped d_s d_t (s + t >= 4)
// are squares: a positive bias of ~1e-9 relative on those elements (measured
// on the GPU: 1.5e-9 on E for the single pair (0, 0) at nvir / naux =
// 300 / 200). Those elements are taken instead from exact fp64 row sums of
// squares, computed in the row-max pass. An fp64 emulation of the whole
// arithmetic then puts E within 4e-12 .. 2e-11 (relative) of the fp64 energy
// on that pair, at 5 / 37 / 45 and at 48 / 432 / 1152 (3 digits with
// diagonals <= 2, 6 products, reach 1.1e-8 at 5 / 37 / 45: too few terms
// average the truncation errors there).
//
// Epilogue in fp64. The diagonals are folded (smallest first), scaled by the
// exact power of two and multiplied into the numerators in fp64; the common
// factor 1 / 127^4 is applied once per thread.
//
// Pipeline. One stage holds a 64-wide K superslab of all 4 planes of the
// 128-row A block (32 KB) and of the 64-row B block (16 KB), each ONE TMA
// tensor copy out of the single digit layout (pe_digit_offset), whose boxes
// land in shared memory as the MMA's no-swizzle images. (An earlier layout
// stored the digits twice, in 128-row and in 64-row blocks, so that each
// operand was one contiguous bulk copy: twice the digit bytes in HBM and in
// L2.) TMEM holds two pass buffers of 4 x 64 columns (X in buffer 0, Y in
// buffer 1: all 512 columns), so the MMA runs the next pass while the
// epilogue folds the last.
#pragma once

#include "ozaki_split.cuh"

namespace tb {

struct Pe254 {
  static constexpr int KS = 4;    // digit planes
  static constexpr int DMAX = 3;  // diagonals s + t <= DMAX are kept
  static constexpr int BM = 128, BN = 64;
  static constexpr int SW = 64;   // K per stage (one superslab of the digit layout)
  static constexpr int A_PLANE = BM * SW, B_PLANE = BN * SW;
  static constexpr int A_OFF = 0, B_OFF = KS * A_PLANE;
  static constexpr int STAGE_BYTES = KS * (A_PLANE + B_PLANE);
  static constexpr int STAGES = 4;
  static constexpr int ACC_COLS = (DMAX + 1) * BN;  // one pass buffer
  static constexpr int EPI_WARPS = 16;              // 4 per TMEM lane quarter, 16 columns each
  static constexpr int THREADS = 32 * (2 + EPI_WARPS);
  static constexpr int BAR_BYTES = 512;
  static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + BAR_BYTES;
  static constexpr long long CHUNK_NAUX = 33280;  // 4 * 127^2 * naux < 2^31, a multiple of SW
  static constexpr int CH_KB = CHUNK_NAUX / SW;     // stages of one exact int32 chunk
  static_assert(2 * ACC_COLS <= 512, "two pass buffers in TMEM");
};

// Digit layout, one copy serving both MMA operands: [K superslab of 64]
// [plane][64-row block][8-row group][16-byte K chunk (4)][row in group (8)]
// [16 bytes]. One plane of one row block is 4 KB; inside it the K-major
// no-swizzle core matrices sit LBO = 128 bytes apart along K and SBO = 512
// bytes apart along the rows. The kernel reads it through a 5-D tensor map
// (bytes of a 256-byte row, the 16 such rows of a plane block, row blocks,
// planes, superslabs): the A operand (128 rows) as the box {256, 16, 2, 4, 1},
// which lands in shared memory as [plane][2 row blocks][4 KB], i.e. 8 KB
// planes whose 16 row groups are SBO apart; the B operand (64 rows) as
// {256, 16, 1, 4, 1}, i.e. [plane][4 KB], the planes stacked along N with the
// same SBO. Offset of plane 0 of padded row p at K index k (plane s adds
// s * nblk * 4096; nblk = padded rows / 64):
__host__ __device__ __forceinline__ long long pe_digit_offset(long long p, int k, long long nblk) {
  const long long ss = k >> 6;
  const int kk = k & 63;
  return ((ss * Pe254::KS * nblk + (p >> 6)) << 12) + (((((p >> 3) & 7) << 2) + (kk >> 4)) << 7) +
         ((p & 7) << 4) + (kk & 15);
}

// Soft wave synchronisation of the pair walk. Every CTA's stream of stages
// (its units x 2 passes x num_kb) is cut into groups of sync_kb stages; after
// issuing a group the producer adds 1 to the launch's counter, and before
// issuing group g it waits (a hint, at most 100 us) until every CTA has
// issued its groups before g - sync_lag. The CTAs then stream the same K range of the
// concurrently processed units together, so an operand block shared by many
// CTAs (one A block feeds ~30 units of a pair, one B block ~5) is read once
// from DRAM while it sits in L2: measured at config 5b (96 / 2208 / 6912),
// the free-running CTAs drifted apart and read 9.34 TB from DRAM per launch
// (60 % of the 15.7 TB the SMs load), most of the kernel's power under the
// 1 kW cap. Counter value once every CTA has issued groups 0 .. g - 1: CTAs
// hold (units of CTA b) = q + (b < r) units for q, r = num_units / grid,
// num_units % grid, and so ceil(units * 2 * num_kb / sync_kb) groups.
__device__ __forceinline__ int pe254_group_target(long long num_units, int grid, int num_kb,
                                                  int sync_kb, int g) {
  const long long q = num_units / grid, r = num_units % grid;
  const long long per_unit = 2ll * num_kb;
  const long long g_hi = ((q + 1) * per_unit + sync_kb - 1) / sync_kb;
  const long long g_lo = (q * per_unit + sync_kb - 1) / sync_kb;
  const long long t = r * (g < g_hi ? g : g_hi) + (grid - r) * (g < g_lo ? g : g_lo);
  return static_cast<int>(t < 0x7fffffffll ? t : 0x7fffffffll);
}

// Per-row statistics of B (R rows of naux fp32, contiguous): max |x| as IEEE
// bits (for the exponent) and the fp64 sum of squares, one warp per row,
// reduced in a fixed order (deterministic).
__global__ void __launch_bounds__(256)
    pe254_rowstats_kernel(const float* __restrict__ B, int naux, long long R,
                          unsigned long long* __restrict__ maxbits, double* __restrict__ rowsq) {
  const long long r = static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= R) return;
  const float* row = B + r * naux;
  unsigned long long mb = 0;
  double sq = 0.0;
  int k = lane;
  for (; k + 96 < naux; k += 128) {
    const float x0 = __ldg(row + k), x1 = __ldg(row + k + 32), x2 = __ldg(row + k + 64),
                x3 = __ldg(row + k + 96);
    mb = umax64(umax64(mb, abs_bits(x0)), umax64(abs_bits(x1), umax64(abs_bits(x2), abs_bits(x3))));
    sq = fma(static_cast<double>(x0), static_cast<double>(x0), sq);
    sq = fma(static_cast<double>(x1), static_cast<double>(x1), sq);
    sq = fma(static_cast<double>(x2), static_cast<double>(x2), sq);
    sq = fma(static_cast<double>(x3), static_cast<double>(x3), sq);
  }
  for (; k < naux; k += 32) {
    const float x = __ldg(row + k);
    mb = umax64(mb, abs_bits(x));
    sq = fma(static_cast<double>(x), static_cast<double>(x), sq);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mb = umax64(mb, __shfl_xor_sync(0xffffffffu, mb, o));
    sq += __shfl_xor_sync(0xffffffffu, sq, o);
  }
  if (lane == 0) {
    maxbits[r] = mb;
    rowsq[r] = sq;
  }
}

// Base-254 digits of B (nocc * nvir rows of naux fp32, row (i, a) at
// i * nvir + a) into the digit layout (pe_digit_offset); padded row
// p = i * nv_pad + a, zero for a >= nvir and k >= naux. 32 x 32 tiles through
// a cp.async ring (persistent grid), each thread 4 consecutive K of one row,
// one 32-bit store per plane.
__global__ void __launch_bounds__(256)
    pe254_digits_kernel(const float* __restrict__ B, int naux, int nvir, int nv_pad,
                        long long rows_pad, int naux_p, const int* __restrict__ exps,
                        int8_t* __restrict__ dig) {
  __shared__ __align__(16) float tile[kOzBuf][32][33];
  const int tx = threadIdx.x, ty = threadIdx.y, t = ty * 32 + tx;
  const int nslab = naux_p / 32;
  const long long nrb = rows_pad / 32;
  const long long total = nrb * nslab;
  auto src_row = [&](long long p) -> long long {
    const long long q = p / nv_pad, a = p - q * nv_pad;
    return a < nvir ? q * nvir + a : -1;
  };
  auto issue = [&](long long tile_id, int buf) {
    if (tile_id < total) {
      const long long rb = tile_id / nslab;
      const int k0 = static_cast<int>(tile_id - rb * nslab) * 32;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int i = ty + 8 * j;
        const long long r = src_row(rb * 32 + i);
        const int k = k0 + tx;
        const bool ok = r >= 0 && k < naux;
        cp_async_zfill<4>(&tile[buf][i][tx], ok ? B + r * naux + k : B, ok);
      }
    }
    cp_async_commit();
  };
  const int crow = t >> 3, kq = (t & 7) * 4;
  const long long G = gridDim.x;
  long long tc = blockIdx.x, tl = blockIdx.x;
#pragma unroll
  for (int b = 0; b < kOzBuf - 1; ++b, tl += G) issue(tl, b);
  const double M = 6755399441055744.0;  // 1.5 * 2^52: adding it rounds |u| < 2^51 to an integer
  for (int it = 0; tc < total; tc += G, ++it) {
    cp_async_wait<kOzBuf - 2>();
    __syncthreads();
    issue(tl, (it + kOzBuf - 1) % kOzBuf);
    tl += G;
    const int buf = it % kOzBuf;
    const long long rb = tc / nslab;
    const int k0 = static_cast<int>(tc - rb * nslab) * 32;
    const long long p = rb * 32 + crow;
    const long long r = src_row(p);
    const double f = 127.0 * pow2d(r >= 0 ? -__ldg(exps + r) : 0);  // exact: |e| <= 149
    double u[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) u[e] = static_cast<double>(tile[buf][crow][kq + e]) * f;  // exact
    const long long nblk = rows_pad >> 6;
    int8_t* out = dig + pe_digit_offset(p, k0 + kq, nblk);
#pragma unroll
    for (int s = 0; s < Pe254::KS; ++s) {
      int d[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const double tt = __dadd_rn(u[e], M);
        d[e] = __double2loint(tt);
        // remainder times 254, both exact (the remainder of an fp32 input
        // keeps fewer than 32 significant bits)
        u[e] = __dmul_rn(__dsub_rn(u[e], __dsub_rn(tt, M)), 254.0);
      }
      const uint32_t w = __byte_perm(__byte_perm(d[0], d[1], 0x0040), __byte_perm(d[2], d[3], 0x0040),
                                     0x5410);
      *reinterpret_cast<uint32_t*>(out + s * (nblk << 12)) = w;
    }
  }
  cp_async_wait<0>();
}

// MMA issue for one stage: SW / 32 K steps of 32; at each, A-plane s against
// the B planes 0 .. DMAX - s stacked along N, into diagonal columns s * BN ...
// of the pass buffer (s = 0 initialises all of them on the pass's first step).
template <int OFF>
__device__ __forceinline__ void pe254_issue(uint64_t dA, uint64_t dB, uint32_t d_tmem, bool first) {
  using C = Pe254;
#pragma unroll
  for (int kk = 0; kk < C::SW / 32; ++kk) {
#pragma unroll
    for (int s = 0; s <= C::DMAX; ++s) {
      const int N = (C::DMAX + 1 - s) * C::BN;
      mma_i8(d_tmem + s * C::BN, sdesc_add(dA, OFF + s * C::A_PLANE + kk * 256),
             sdesc_add(dB, OFF + kk * 256), idesc(kAccS32, kFmtS8, kFmtS8, 0, 0, 128, N),
             (first && kk == 0 && s == 0) ? 0u : 1u);
    }
  }
}

// MMA issuer over this CTA's stream of stages (units x 2 passes x num_kb),
// unrolled over the pipeline stages (compile-time shared-memory offsets). A
// pass is cut into accumulations of at most CH_KB stages (chunks, nch per
// pass); accumulation `it` uses TMEM buffer it & 1.
__device__ __forceinline__ void pe254_mma_role(uint8_t* smem, uint64_t* full_bar, uint64_t* empty_bar,
                                               uint64_t* accf_bar, uint64_t* acce_bar,
                                               uint32_t tmem_base, int num_kb, long long total,
                                               const Abort& ab) {
  using C = Pe254;
  constexpr int STAGES = C::STAGES;
  const uint32_t base = smem_u32(smem);
  const uint64_t dA = sdesc_kmajor_noswz(base + C::A_OFF, 128, C::SW * 8);
  const uint64_t dB = sdesc_kmajor_noswz(base + C::B_OFF, 128, C::SW * 8);
  const int nch = (num_kb + C::CH_KB - 1) / C::CH_KB;
  uint32_t phase = 0;
  int it = 0;   // accumulations started
  int kbp = 0;  // stage within the accumulation
  int ci = 0;   // chunk of the current pass
  int len = num_kb < C::CH_KB ? num_kb : C::CH_KB;
  uint32_t d_tmem = tmem_base;
  bool stop = false;
  for (long long g = 0; g < total && !stop; g += STAGES) {
    static_for<0, STAGES>([&](auto sc) {
      constexpr int S = decltype(sc)::value;
      if (stop || g + S >= total) return;
      if (kbp == 0) {
        const int buf = it & 1;
        if (!mbar_wait(&acce_bar[buf], ((it >> 1) & 1) ^ 1u, ab, kTimeoutAccEmpty)) {
          stop = true;
          return;
        }
        tc_fence_after();
        d_tmem = tmem_base + buf * C::ACC_COLS;
      }
      if (!mbar_wait(&full_bar[S], phase, ab, kTimeoutFull)) {
        stop = true;
        return;
      }
      tc_fence_after();
      pe254_issue<S * C::STAGE_BYTES>(dA, dB, d_tmem, kbp == 0);
      tc_commit(&empty_bar[S]);
      if (++kbp == len) {
        tc_commit(&accf_bar[it & 1]);
        kbp = 0;
        ++it;
        ci = (ci + 1 == nch) ? 0 : ci + 1;
        const int rest = num_kb - ci * C::CH_KB;
        len = rest < C::CH_KB ? rest : C::CH_KB;
      }
    });
    phase ^= 1u;
  }
}

// Block: warp 0 producer, warp 1 MMA issuer and TMEM owner, warps 2..17
// epilogue (four per TMEM lane quarter, 16 columns of the 64 each).
__global__ void __launch_bounds__(Pe254::THREADS, 1)
    pair_energy254_kernel(const PairParams p, const __grid_constant__ CUtensorMap map_a,
                          const __grid_constant__ CUtensorMap map_b) {
  using C = Pe254;
  constexpr int STAGES = C::STAGES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * C::STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* accf_bar = empty_bar + STAGES;  // [2]
  uint64_t* acce_bar = accf_bar + 2;        // [2]
  uint64_t* drain_bar = acce_bar + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  double* red = reinterpret_cast<double*>(smem + STAGES * C::STAGE_BYTES + 256);  // [EPI_WARPS]
  static_assert((2 * STAGES + 5) * 8 + 8 <= 256, "barrier block");
  static_assert(256 + 8 * C::EPI_WARPS <= C::BAR_BYTES, "reduction slots");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Abort ab{abort_flag, p.status, p.timeout_ns};

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&accf_bar[b], 1);
      mbar_init(&acce_bar[b], C::EPI_WARPS);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    for (int w = 0; w < C::EPI_WARPS; ++w) red[w] = 0.0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_kb = p.naux_p / C::SW;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    bool aborted = false;
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
    long long gs = 0;  // stages issued (position in this CTA's stream)
    // the pair (i, j) of the next unit is loaded one unit ahead, so that its
    // latency never holds up the stage ring at a unit boundary
    int2 ij = p.num_units > blockIdx.x ? p.order[blockIdx.x / p.units_per_pair] : make_int2(0, 0);
    for (long long u = blockIdx.x; u < p.num_units && !aborted; u += gridDim.x) {
      const long long un = u + gridDim.x;
      const int2 ij_next = un < p.num_units ? p.order[un / p.units_per_pair] : ij;
      const int i = ij.x, j = ij.y;
      int R, Cb;
      unit_rc(p, u, R, Cb);
      const long long ri = static_cast<long long>(i) * p.nv_pad;
      const long long rj = static_cast<long long>(j) * p.nv_pad;
      for (int pass = 0; pass < 2 && !aborted; ++pass) {
        const long long ra = (pass == 0 ? ri : rj) + 128 * R;  // A rows: B_i[R] then B_j[R]
        const long long rb = (pass == 0 ? rj : ri) + 64 * Cb;  // B rows: B_j[C] then B_i[C]
        for (int kb = 0; kb < num_kb; ++kb, ++gs) {
          if (p.wave_ctr && gs % p.sync_kb == 0 && gs / p.sync_kb > p.sync_lag)
            soft_wave_wait(p.wave_ctr,
                           pe254_group_target(p.num_units, gridDim.x, num_kb, p.sync_kb,
                                              static_cast<int>(gs / p.sync_kb) - p.sync_lag),
                           100000ull);
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, ab, kTimeoutEmpty)) {
            aborted = true;
            break;
          }
          uint8_t* st = smem + stage * C::STAGE_BYTES;
          mbar_arrive_expect_tx(&full_bar[stage], C::STAGE_BYTES);
          // row blocks of 64: A rows ra .. ra + 127 (two blocks), B rows rb .. rb + 63
          tma_load_5d(st + C::A_OFF, &map_a, &full_bar[stage], 0, 0, static_cast<int>(ra >> 6), 0, kb);
          tma_load_5d(st + C::B_OFF, &map_b, &full_bar[stage], 0, 0, static_cast<int>(rb >> 6), 0, kb);
          if (p.wave_ctr && ((gs + 1) % p.sync_kb == 0 ||
                             (u + gridDim.x >= p.num_units && pass == 1 && kb + 1 == num_kb)))
            atomicAdd(p.wave_ctr, 1);  // group complete (or this CTA's last, partial one)
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      ij = ij_next;
    }
    if (aborted || ab.raised()) {
      int s = stage;
      uint32_t ph = phase;
      for (int k = 0; k < STAGES; ++k) {
        if (s == 0) {
          s = STAGES - 1;
          ph ^= 1u;
        } else {
          --s;
        }
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(&full_bar[s], ph))
          if (globaltimer_ns() - t0 > 50000000ull) break;
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    const long long my_units =
        p.num_units > blockIdx.x ? (p.num_units - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    pe254_mma_role(smem, full_bar, empty_bar, accf_bar, acce_bar, tmem_base, num_kb,
                   my_units * 2 * num_kb, ab);
    tc_commit(drain_bar);
    const unsigned long long t0 = globaltimer_ns();
    while (!mbar_try_wait(drain_bar, 0)) {
      if (globaltimer_ns() - t0 > 100000000ull) {
        ab.raise(kTimeoutDrain);
        break;
      }
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------ epilogue
    constexpr int NCOL = C::BN / (C::EPI_WARPS / 4);  // 16 columns per warp
    static_assert(NCOL == 16, "one 16-column TMEM load per diagonal");
    const int q = warp & 3;
    const int col0 = NCOL * ((warp - 2) / 4);
    const int aloc = 32 * q + lane;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(32 * q) << 16) + col0;
    const double c1 = 1.0 / 254.0, c2 = 1.0 / 64516.0, c3 = 1.0 / 16387064.0;
    const int nch = (num_kb + C::CH_KB - 1) / C::CH_KB;
    double acc = 0.0;
    int it = 0;
    bool aborted = false;
    for (long long u = blockIdx.x; u < p.num_units && !aborted; u += gridDim.x) {
      // The unit's row and column data, loaded before the passes so that
      // their latency hides behind the MMAs: lane l < 16 holds exps[j][b] and
      // lane 16 + l exps[i][b] of this warp's column b = b0 + l, lanes < 16
      // also eps_vir[b] (broadcast to the warp by shuffles in the energy
      // loop); every lane its own row a's values.
      int i, j, R, Cb;
      unit_of(p, u, i, j, R, Cb);
      const int a = 128 * R + aloc;
      const int b0 = 64 * Cb + col0;
      const int bl = b0 + (lane & 15);
      int e_col = 0;
      float ev_colf = 0.0f;
      if (bl < p.nvir) {
        e_col = p.exps[(lane < 16 ? j : i) * p.nvir + bl];
        ev_colf = p.eps_vir[bl];
      }
      int eia = 0, eja = 0;
      float eva = 0.0f;
      if (a < p.nvir) {
        eia = p.exps[i * p.nvir + a];
        eja = p.exps[j * p.nvir + a];
        eva = p.eps_vir[a];
      }
      const float eoi = p.eps_occ[i], eoj = p.eps_occ[j];
      double xt[NCOL], yt[NCOL];
#pragma unroll
      for (int jj = 0; jj < NCOL; ++jj) xt[jj] = yt[jj] = 0.0;
#pragma unroll
      for (int pass = 0; pass < 2 && !aborted; ++pass) {
        for (int c = 0; c < nch; ++c, ++it) {
          const int buf = it & 1;
          if (!mbar_wait_warp(&accf_bar[buf], (it >> 1) & 1, ab, kTimeoutAccFull)) {
            aborted = true;
            break;
          }
          tc_fence_after();
          const uint32_t col = lane_base + buf * C::ACC_COLS;
          // one diagonal at a time, smallest first (S_3 / 254^3 + S_2 / 254^2
          // + S_1 / 254 + S_0), 8 columns a load, so that only 8 loaded words
          // are live beside the 32 folds
#pragma unroll
          for (int h = 0; h < NCOL / 8; ++h) {
#pragma unroll
            for (int d = C::DMAX; d >= 0; --d) {
              uint32_t v[8];
              tmem_ld8(col + d * C::BN + 8 * h, v);
              tmem_ld_wait();
              const double cd = d == 3 ? c3 : d == 2 ? c2 : d == 1 ? c1 : 1.0;
#pragma unroll
              for (int jj = 0; jj < 8; ++jj) {
                const double sv = i32_to_f64(static_cast<int>(v[jj]));
                if (pass == 0)
                  xt[8 * h + jj] = fma(sv, cd, xt[8 * h + jj]);
                else
                  yt[8 * h + jj] = fma(sv, cd, yt[8 * h + jj]);
              }
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acce_bar[buf]);  // free for the accumulation after next
        }
      }
      if (aborted) break;
      // lane mode: 2 = both ordered pairs, 1 = (a, b) once, 0 = skip
      int mode = 2;
      if (Cb == 2 * R + 1) mode = (aloc < 64) ? 2 : 1;
      if (Cb == 2 * R) mode = (aloc < 64) ? 1 : 0;
      if (a >= p.nvir) mode = 0;
      double usum = 0.0;
      const double da = (static_cast<double>(eoi) + static_cast<double>(eoj)) - static_cast<double>(eva);
      const double ev_col = static_cast<double>(ev_colf);  // one conversion a lane, shuffled below
#pragma unroll
      for (int jj = 0; jj < NCOL; ++jj) {
        // every lane takes part in the shuffles; the arithmetic is per lane
        const int ejb = __shfl_sync(0xffffffffu, e_col, jj);
        const int eib = __shfl_sync(0xffffffffu, e_col, 16 + jj);
        const double evb = __shfl_sync(0xffffffffu, ev_col, jj);
        const int b = b0 + jj;
        if (mode && b < p.nvir) {
          double X = xt[jj] * pow2d(eia + ejb);
          double Y = yt[jj] * pow2d(eja + eib);
          if (i == j && b == a) X = Y = p.rowsq[i * p.nvir + a] * 16129.0;  // exact T_aa * 127^2
          const double den = da - evb;
          double f = X * (2.0 * X - Y);
          if (mode == 2) f = fma(Y, 2.0 * Y - X, f);
          // f / den as f * (1 / den) (den: an orbital-energy difference,
          // finite and normal); no conversion-unit work but the seed
          usum = fma(f, recip_f64(den), usum);
        }
      }
      acc += ((i == j) ? 1.0 : 2.0) * usum;
    }
    acc *= 1.0 / 260144641.0;  // 127^-4: T = 2^(e + e') / 127^2 * fold
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) red[warp - 2] = acc;
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    double part = 0.0;
    for (int w = 0; w < C::EPI_WARPS; ++w) part += red[w];  // fixed order
    p.partials[blockIdx.x] = part;
  }
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace tb
