// Fused DF-MP2 pair energy on the int8 tensor cores.
//
// Two digit forms share the pair walk, the work units and the host entry
// point below: the base-254 form of pair_energy254.cuh (10 int8 products,
// fp64 epilogue) for naux <= 33280, and the 7-bit form described here (15
// products) for larger naux, up to 104857.
//
// E = sum over occupied pairs i <= j (weight 1 if i == j, else 2) of
//     sum_{a,b} T_ab (2 T_ab - T_ba) / (e_i + e_j - e_a - e_b),  T = B_i B_j^T,
// following the reference's symmetric pair walk (trnblas/nki/dispatch.py:
// 2648-2677: e_ij = e_ji, so off-diagonal pairs count twice).
//
// Numerics. Tensor-core fp32 accumulation truncates, a bias that grows with
// naux and would put E off by ~1e-5 relative; the 1e-9 target needs T free of
// systematic error. So B is split per row (i, a) into KS = 5 balanced 7-bit
// int8 digit planes with a power-of-two exponent (the Ozaki split of
// trnblas/ozaki.py:123-219), and
//     T_ab = 2^(e_ia + e_jb - 12) * sum_{d <= 4} 2^(-7 d) S_d,
//     S_d  = sum_{s+t=d} D_s[i,a,:] . D_t[j,b,:]
// with every S_d exact in int32 TMEM accumulators. Fewer digits leave a
// measurable bias in E (3 slices: ~7e-8 relative at nocc/nvir/naux =
// 48/432/1152, 4 slices with diagonals <= 3: ~2e-9); 5 slices with diagonals
// <= 4 are at ~1e-12. The epilogue folds the diagonals in fp32 with
// round-to-nearest and forms each numerator T_ab (2 T_ab - T_ba) in fp32
// (independent rounding per term, which averages out); the denominators
// e_i + e_j - e_a - e_b are exact in fp64 and the quotient is taken and
// accumulated per thread in fp64. Partial sums are reduced in a fixed
// order, so the result is deterministic.
//
// Work unit: pair (i, j), a 128-row block R of a and a 64-column block C of b
// with C >= 2R (64-blocks 2R and 2R+1 lie inside R). Two passes over naux
// into the same TMEM accumulators (5 diagonals x 64 columns):
//   X = B_i[R] . B_j[C]^T  ->  X[a, b] = T_ab
//   Y = B_j[R] . B_i[C]^T  ->  Y[a, b] = T_ba
// so T_ab and T_ba land in the same TMEM lane and column: no transpose. The
// epilogue (8 warps, 32 columns each) folds X into registers and releases
// TMEM before the Y pass, then Y, then computes the terms from registers
// while the next unit's X pass runs. Per (a, b): if the 64-blocks of a and b differ, the
// unit accounts for both ordered pairs, [X(2X-Y) + Y(2Y-X)] / D; if they are
// the same block, X(2X-Y) / D once; a in block 2R+1 with b in block 2R is
// skipped (unit (R, 2R+1) counted it). The nvir x nvir T never reaches HBM.
#include <algorithm>
#include <cmath>
#include <string>

#include "ozaki_split.cuh"
#include "runtime.hpp"

namespace tb {

struct PairParams {
  const int8_t* digA;      // digits in 128-row blocks (A operand), rows (i, a) at i * nv_pad + a
  const int8_t* digB;      // the same digits in 64-row blocks (B operand)
  long long rows_pad;      // nocc * nv_pad
  int nv_pad;              // nvir rounded up to 128 (zero rows beyond nvir)
  int nocc, nvir, naux_p;  // naux_p: K columns of the digit planes (multiple of 32)
  long long pair_begin;
  const int2* order;       // (i, j) of the range's pairs in processing order
  long long num_units;     // pairs * units_per_pair
  int units_per_pair;
  int nR, nC;              // 128-blocks and 64-blocks of nvir
  const int* exps;         // nocc * nvir
  const double* rowsq;     // nocc * nvir fp64 row sums of squares (base-254 form)
  const float* eps_occ;
  const float* eps_vir;
  double* partials;        // gridDim.x
  int* status;
  unsigned long long timeout_ns;
};

template <int KS>
struct PairCfg {
  static constexpr int BM = 128, BN = 64, BK = 32;
  static constexpr int A_PLANE = BM * BK, B_PLANE = BN * BK;
  static constexpr int A_OFF = 0;
  static constexpr int B_OFF = KS * A_PLANE;
  static constexpr int STAGE_BYTES = KS * (A_PLANE + B_PLANE);
  static_assert(KS * BN <= 512, "the diagonals of one pass must fit TMEM");
};

__device__ __forceinline__ void pair_of(long long p, int& i, int& j) {
  long long jj = static_cast<long long>((sqrt(8.0 * static_cast<double>(p) + 1.0) - 1.0) * 0.5);
  while (jj * (jj + 1) / 2 > p) --jj;
  while ((jj + 1) * (jj + 2) / 2 <= p) ++jj;
  j = static_cast<int>(jj);
  i = static_cast<int>(p - jj * (jj + 1) / 2);
}

// Pairs of [begin, end) (linear index tri(j) + i, i <= j) in an L2-friendly
// order: rows j in chunks of g, and inside a chunk the pairs grouped by
// g-wide blocks of i, so that consecutive units (which run at the same time on
// different SMs) share the digits of at most 2g occupied orbitals. One thread
// per chunk; a chunk's pairs are contiguous in the linear order, so its first
// output position is known in closed form.
__global__ void pair_order_kernel(long long begin, long long end, int g, int2* __restrict__ order) {
  int i0, j0, i1, j1;
  pair_of(begin, i0, j0);
  pair_of(end - 1, i1, j1);
  const long long c = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long rs = j0 + c * g;
  if (rs > j1) return;
  const long long re = (rs + g < j1 + 1) ? rs + g : j1 + 1;
  const long long first = rs * (rs + 1) / 2;
  long long pos = first > begin ? first - begin : 0;
  for (long long ib = 0; ib * g < re; ++ib) {
    for (long long r = rs; r < re; ++r) {
      const long long ihi = (ib * g + g < r + 1) ? ib * g + g : r + 1;
      for (long long i = ib * g; i < ihi; ++i) {
        const long long q = r * (r + 1) / 2 + i;
        if (q < begin || q >= end) continue;
        order[pos++] = make_int2(static_cast<int>(i), static_cast<int>(r));
      }
    }
  }
}

__device__ __forceinline__ void unit_of(const PairParams& p, long long u, int& i, int& j, int& R,
                                        int& C) {
  const long long pr = u / p.units_per_pair;
  int loc = static_cast<int>(u - pr * p.units_per_pair);
  const int2 ij = p.order[pr];
  i = ij.x;
  j = ij.y;
  R = 0;
  while (R < p.nR) {
    const int cnt = p.nC - 2 * R;
    if (loc < cnt) break;
    loc -= cnt;
    ++R;
  }
  C = 2 * R + loc;
}

__device__ __forceinline__ float pow2f(int n) {
  n = n < -126 ? -126 : (n > 127 ? 127 : n);
  return __int_as_float((n + 127) << 23);
}

// The K slab products of one stage: A-plane s against B-planes t0 .. t0+np-1
// (stacked along N) into TMEM columns (s + t0) * BN, diagonal by diagonal.
// Descriptors are the stage-0 ones plus compile-time offsets.
template <int KS, int OFF>
__device__ __forceinline__ void pair_issue(uint64_t dA, uint64_t dB, uint32_t tmem_base,
                                           uint32_t acc) {
  using Cfg = PairCfg<KS>;
#pragma unroll
  for (int s = 0; s < KS; ++s) {
    const uint64_t ad = sdesc_add(dA, OFF + s * Cfg::A_PLANE);
#pragma unroll
    for (int t0 = 0; t0 < KS - s; t0 += 4) {
      const int np = (KS - s - t0 < 4) ? KS - s - t0 : 4;
      mma_i8(tmem_base + (s + t0) * Cfg::BN, ad, sdesc_add(dB, OFF + t0 * Cfg::B_PLANE),
             idesc(kAccS32, kFmtS8, kFmtS8, 0, 0, 128, np * Cfg::BN), (acc || s) ? 1u : 0u);
    }
  }
}

// MMA issuer role over this CTA's stream of `total` K slabs (units x 2
// passes x num_kb). The loop is unrolled over the pipeline stages so that
// every shared-memory offset and barrier address is a compile-time constant:
// a tcgen05.mma issue blocks the issuing thread until the tensor pipe is
// nearly ready for it, so scalar work between the MMAs of consecutive K slabs
// (stage index arithmetic, descriptor rebuilds) leaves the pipe idle. Measured
// with the pair schedule on B200: 646 cycles per K slab with a runtime stage
// index, 525 with this loop, 504 with no barrier ring at all.
template <int KS, int STAGES>
__device__ __forceinline__ void pair_mma_role(uint8_t* smem, uint64_t* full_bar, uint64_t* empty_bar,
                                              uint64_t* accf_bar, uint64_t* acce_bar,
                                              uint32_t tmem_base, int num_kb, long long total,
                                              const Abort& ab) {
  using Cfg = PairCfg<KS>;
  const uint32_t base = smem_u32(smem);
  const uint64_t dA = sdesc_kmajor_noswz(base + Cfg::A_OFF, 128, 256);
  const uint64_t dB = sdesc_kmajor_noswz(base + Cfg::B_OFF, 128, 256);
  uint32_t phase = 0;
  int it = 0;   // passes started
  int kbp = 0;  // K slab within the current pass
  bool stop = false;
  for (long long g = 0; g < total && !stop; g += STAGES) {
    static_for<0, STAGES>([&](auto sc) {
      constexpr int S = decltype(sc)::value;
      if (stop || g + S >= total) return;
      if (kbp == 0) {
        if (!mbar_wait(acce_bar, (it & 1) ^ 1u, ab, kTimeoutAccEmpty)) {
          stop = true;
          return;
        }
        tc_fence_after();
      }
      if (!mbar_wait(&full_bar[S], phase, ab, kTimeoutFull)) {
        stop = true;
        return;
      }
      tc_fence_after();
      pair_issue<KS, S * Cfg::STAGE_BYTES>(dA, dB, tmem_base, kbp > 0 ? 1u : 0u);
      tc_commit(&empty_bar[S]);
      if (++kbp == num_kb) {
        kbp = 0;
        ++it;
        tc_commit(accf_bar);
      }
    });
    phase ^= 1u;
  }
}

// Block: warp 0 producer, warp 1 MMA issuer and TMEM owner, warps 2..9
// epilogue. Two epilogue warps share each TMEM lane quarter (warp w reads
// lanes 32 (w % 4) .. +31), one taking columns 0..31 of the 64-column block,
// the other 32..63, so each warp's energy loop (fp64 quotients and sums,
// latency bound with one warp per scheduler) is half as long.
constexpr int kPairEpiWarps = 8;
constexpr int kPairThreads = 32 * (2 + kPairEpiWarps);

template <int KS, int STAGES>
__global__ void __launch_bounds__(kPairThreads, 1)
    pair_energy_kernel(const PairParams p) {
  using Cfg = PairCfg<KS>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* accf_bar = empty_bar + STAGES;
  uint64_t* acce_bar = accf_bar + 1;
  uint64_t* drain_bar = acce_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  double* red = reinterpret_cast<double*>(smem + STAGES * Cfg::STAGE_BYTES + 128);  // [kPairEpiWarps]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Abort ab{abort_flag, p.status, p.timeout_ns};

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(accf_bar, 1);
    mbar_init(acce_bar, kPairEpiWarps);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    for (int w = 0; w < kPairEpiWarps; ++w) red[w] = 0.0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_kb = p.naux_p / Cfg::BK;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    bool aborted = false;
    for (long long u = blockIdx.x; u < p.num_units && !aborted; u += gridDim.x) {
      int i, j, R, C;
      unit_of(p, u, i, j, R, C);
      const long long ri = static_cast<long long>(i) * p.nv_pad;
      const long long rj = static_cast<long long>(j) * p.nv_pad;
      for (int pass = 0; pass < 2 && !aborted; ++pass) {
        const long long ra = (pass == 0 ? ri : rj) + 128 * R;  // A rows: B_i[R] then B_j[R]
        const long long rb = (pass == 0 ? rj : ri) + 64 * C;   // B rows: B_j[C] then B_i[C]
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1u, ab, kTimeoutEmpty)) {
            aborted = true;
            break;
          }
          uint8_t* st = smem + stage * Cfg::STAGE_BYTES;
          mbar_arrive_expect_tx(&full_bar[stage], Cfg::STAGE_BYTES);
          // all KS planes of the 128-row A block and of the 64-row B block:
          // one contiguous chunk each
          bulk_load(st + Cfg::A_OFF, p.digA + blocked_chunk(kb, ra >> 7, KS, p.rows_pad, 7),
                    KS * Cfg::A_PLANE, &full_bar[stage]);
          bulk_load(st + Cfg::B_OFF, p.digB + blocked_chunk(kb, rb >> 6, KS, p.rows_pad, 6),
                    KS * Cfg::B_PLANE, &full_bar[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
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
    pair_mma_role<KS, STAGES>(smem, full_bar, empty_bar, accf_bar, acce_bar, tmem_base, num_kb,
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
    constexpr int NCOL = 64 / (kPairEpiWarps / 4);  // columns per epilogue warp
    const int q = warp & 3;
    const int col0 = NCOL * ((warp - 2) / 4);
    const int aloc = 32 * q + lane;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(32 * q) << 16) + col0;
    double acc = 0.0;  // this thread's fp64 partial sum
    int it = 0;
    bool aborted = false;
    for (long long u = blockIdx.x; u < p.num_units && !aborted; u += gridDim.x) {
      // fold the KS diagonals of one pass into NCOL fp32 values (unscaled T)
      float xt[NCOL], yt[NCOL];
#pragma unroll
      for (int pass = 0; pass < 2; ++pass, ++it) {
        if (!mbar_wait_warp(accf_bar, it & 1, ab, kTimeoutAccFull)) {
          aborted = true;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < NCOL / 16; ++c) {
          uint32_t v[KS][16];
#pragma unroll
          for (int d = 0; d < KS; ++d) tmem_ld16(lane_base + d * Cfg::BN + 16 * c, v[d]);
          tmem_ld_wait();
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            float t = static_cast<float>(static_cast<int>(v[KS - 1][jj]));
#pragma unroll
            for (int d = KS - 2; d >= 0; --d)
              t = fmaf(t, 0.0078125f, static_cast<float>(static_cast<int>(v[d][jj])));
            if (pass == 0)
              xt[16 * c + jj] = t;
            else
              yt[16 * c + jj] = t;
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acce_bar);  // TMEM free for the next pass
      }
      if (aborted) break;
      int i, j, R, C;
      unit_of(p, u, i, j, R, C);
      const int a = 128 * R + aloc;
      // lane mode: 2 = both ordered pairs, 1 = (a, b) once, 0 = skip
      int mode = 2;
      if (C == 2 * R + 1) mode = (aloc < 64) ? 2 : 1;
      if (C == 2 * R) mode = (aloc < 64) ? 1 : 0;
      if (a >= p.nvir) mode = 0;
      double usum = 0.0;
      if (mode) {
        const int eia = p.exps[i * p.nvir + a], eja = p.exps[j * p.nvir + a];
        // Denominators in fp64, where these sums and differences of fp32
        // values are exact: an fp32 e_i + e_j would carry one rounding error
        // shared by every term of the pair, which does not average out.
        const double da = (static_cast<double>(p.eps_occ[i]) + static_cast<double>(p.eps_occ[j])) -
                          static_cast<double>(p.eps_vir[a]);
        const int b0 = 64 * C + col0;
#pragma unroll
        for (int jj = 0; jj < NCOL; ++jj) {
          const int b = b0 + jj;
          if (b < p.nvir) {
            const float X = xt[jj] * pow2f(eia + p.exps[j * p.nvir + b] - 12);
            const float Y = yt[jj] * pow2f(eja + p.exps[i * p.nvir + b] - 12);
            const double den = da - static_cast<double>(p.eps_vir[b]);
            float f = X * (2.0f * X - Y);
            if (mode == 2) f += Y * (2.0f * Y - X);
            usum += static_cast<double>(f) / den;
          }
        }
      }
      acc += ((i == j) ? 1.0 : 2.0) * usum;
    }
    // warp reduction (fixed tree) then per-CTA partial
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) red[warp - 2] = acc;
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    double part = 0.0;
    for (int w = 0; w < kPairEpiWarps; ++w) part += red[w];  // fixed order
    p.partials[blockIdx.x] = part;
  }
  if (warp == 1) {
    __syncwarp();  // lane 0 arrives from the MMA role, 1..31 straight here
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace tb

#include "pair_energy254.cuh"

namespace tb {

// Sum the per-CTA partials in index order (deterministic).
__global__ void pair_energy_finish(const double* partials, int n, double* energy) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    double s = 0.0;
    for (int k = 0; k < n; ++k) s += partials[k];
    *energy = s;
  }
}

namespace {

constexpr int kPairSlices = 5;
constexpr int kPairStages = 6;
constexpr int kMaxGrid = 1024;

// naux up to Pe254::MAX_NAUX runs the base-254 form (10 int8 products per
// 64-column block); larger naux the 7-bit form (15 products, exact int32 up
// to 104857).
bool use_pe254(long long naux) { return naux <= Pe254::MAX_NAUX; }

struct PairLayout {
  long long naux_p, R, nv_pad, rows_pad;
  int slices;
  size_t off_digb, off_exps, off_max, off_range, off_rowsq, off_part, off_order, total;
};

PairLayout pair_layout(long long nocc, long long nvir, long long naux, long long npairs) {
  PairLayout L{};
  const bool b254 = use_pe254(naux);
  L.slices = b254 ? Pe254::KS : kPairSlices;
  L.naux_p = round_up(std::max<long long>(naux, 1), b254 ? Pe254::SW : 32);
  L.R = nocc * nvir;
  L.nv_pad = round_up(std::max<long long>(nvir, 1), 128);
  L.rows_pad = nocc * L.nv_pad;
  // the digits twice: in 128-row blocks (A operand) and in 64-row blocks (B)
  const size_t dig = static_cast<size_t>(round_up(L.slices * L.rows_pad * L.naux_p, 256));
  L.off_digb = dig;
  L.off_exps = 2 * dig;
  L.off_max = L.off_exps + round_up(4 * L.R, 256);
  L.off_range = L.off_max + round_up(8 * L.R, 256);
  L.off_rowsq = L.off_range + 256;
  L.off_part = L.off_rowsq + round_up(8 * L.R, 256);
  L.off_order = L.off_part + round_up(8 * kMaxGrid, 256);
  L.total = L.off_order + round_up(8 * std::max<long long>(npairs, 1), 256);
  return L;
}

// Pair-block width g of the processing order: the digits of 2g occupied
// orbitals (both layouts) should fit in half of L2.
int pair_block(const PairLayout& L, long long nocc) {
  int l2 = 0;
  if (cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, current_device()) != cudaSuccess || l2 <= 0)
    l2 = 96 << 20;
  const double per_orb = 2.0 * L.slices * static_cast<double>(L.nv_pad) * L.naux_p;
  const long long g = static_cast<long long>(0.5 * l2 / (2.0 * per_orb));
  return static_cast<int>(std::max<long long>(1, std::min<long long>(g, std::max<long long>(nocc, 1))));
}

void host_pair_of(long long p, int& i, int& j) {
  long long jj = static_cast<long long>((std::sqrt(8.0 * static_cast<double>(p) + 1.0) - 1.0) * 0.5);
  while (jj * (jj + 1) / 2 > p) --jj;
  while ((jj + 1) * (jj + 2) / 2 <= p) ++jj;
  j = static_cast<int>(jj);
  i = static_cast<int>(p - jj * (jj + 1) / 2);
}

int units_per_pair(long long nvir) {
  const int nR = static_cast<int>(ceil_div(nvir, 128)), nC = static_cast<int>(ceil_div(nvir, 64));
  int u = 0;
  for (int R = 0; R < nR; ++R) u += std::max(0, nC - 2 * R);
  return u;
}

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" {

size_t trnblas_pair_energy_workspace_size(int64_t nocc, int64_t nvir, int64_t naux,
                                          int64_t pair_begin, int64_t pair_end) {
  if (nocc <= 0 || nvir <= 0 || naux <= 0) return 256;
  return pair_layout(nocc, nvir, naux, std::max<int64_t>(pair_end - pair_begin, 0)).total;
}

int trnblas_pair_energy(int64_t nocc, int64_t nvir, int64_t naux, const float* B,
                        const float* eps_occ, const float* eps_vir, int64_t pair_begin,
                        int64_t pair_end, double* energy, void* workspace,
                        size_t workspace_bytes, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const long long npairs_total = nocc * (nocc + 1) / 2;
  if (nocc < 0 || nvir < 0 || naux < 0 || pair_begin < 0 || pair_end < pair_begin ||
      pair_end > npairs_total) {
    set_error("trnblas_pair_energy: bad sizes or pair range");
    return TRNBLAS_ERR_ARG;
  }
  if (!energy) {
    set_error("trnblas_pair_energy: NULL energy pointer");
    return TRNBLAS_ERR_ARG;
  }
  if (nocc * round_up(std::max<int64_t>(nvir, 1), 128) > 65535ll * 32) {
    set_error("trnblas_pair_energy: nocc * round_up(nvir, 128) must stay below 2097120");
    return TRNBLAS_ERR_ARG;
  }
  if (naux > ((1ll << 31) - 1) / (kPairSlices * 4096ll)) {
    set_error("trnblas_pair_energy: naux too large for exact int32 diagonal sums");
    return TRNBLAS_ERR_ARG;
  }
  if (pair_end == pair_begin || nvir == 0 || naux == 0) {
    cudaError_t e = cudaMemsetAsync(energy, 0, sizeof(double), stream);
    return e == cudaSuccess ? TRNBLAS_OK : cuda_fail(e, "cudaMemsetAsync(energy)");
  }
  if (!B || !eps_occ || !eps_vir) {
    set_error("trnblas_pair_energy: NULL operand");
    return TRNBLAS_ERR_ARG;
  }
  int* status = status_word();
  if (!status) return TRNBLAS_ERR_CUDA;
  const int upp = units_per_pair(nvir);
  const long long num_units = (pair_end - pair_begin) * static_cast<long long>(upp);
  const int grid = static_cast<int>(
      std::min<long long>(std::min<long long>(num_units, num_sms()), kMaxGrid));
  const PairLayout L = pair_layout(nocc, nvir, naux, pair_end - pair_begin);
  if (!workspace || workspace_bytes < L.total) {
    set_error("trnblas_pair_energy needs " + std::to_string(L.total) + " workspace bytes");
    return TRNBLAS_ERR_WORKSPACE;
  }
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int8_t* dig = reinterpret_cast<int8_t*>(ws);
  int8_t* digb = reinterpret_cast<int8_t*>(ws + L.off_digb);
  int* exps = reinterpret_cast<int*>(ws + L.off_exps);
  SplitScratch sc{reinterpret_cast<unsigned long long*>(ws + L.off_max),
                  reinterpret_cast<int*>(ws + L.off_range)};
  double* partials = reinterpret_cast<double*>(ws + L.off_part);
  int2* order = reinterpret_cast<int2*>(ws + L.off_order);
  double* rowsq = reinterpret_cast<double*>(ws + L.off_rowsq);
  const bool b254 = use_pe254(naux);
  cudaError_t e = cudaSuccess;
  if (b254) {
    // per-row exponents and sums of squares, then the base-254 digits in both layouts
    const int R = static_cast<int>(L.R);
    ozk_init_kernel<<<(R + 255) / 256 + 1, 256, 0, stream>>>(sc.maxbits, R, sc.shift_range);
    pe254_rowstats_kernel<<<static_cast<unsigned>((L.R + 7) / 8), 256, 0, stream>>>(
        B, static_cast<int>(naux), L.R, sc.maxbits, rowsq);
    ozk_exps_kernel<<<(R + 255) / 256, 256, 0, stream>>>(sc.maxbits, R, exps, sc.shift_range);
    const long long tiles = (L.rows_pad / 32) * (L.naux_p / 32);
    static int per_sm = 0;
    if (per_sm == 0 &&
        (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, pe254_digits_kernel, 256, 0) != cudaSuccess ||
         per_sm < 1))
      per_sm = 1;
    const long long g3 = std::min<long long>(tiles, static_cast<long long>(num_sms()) * per_sm);
    pe254_digits_kernel<<<static_cast<unsigned>(g3), dim3(32, 8), 0, stream>>>(
        B, static_cast<int>(naux), static_cast<int>(nvir), static_cast<int>(L.nv_pad), L.rows_pad,
        static_cast<int>(L.naux_p), exps, dig, digb);
    e = cudaGetLastError();
  } else {
    e = launch_split_tiled(B, naux, 1, static_cast<int>(L.R), static_cast<int>(naux), nvir, L.nv_pad,
                           L.rows_pad, static_cast<int>(L.naux_p), kPairSlices, dig, 7, digb, 6,
                           exps, sc, stream);
  }
  if (e != cudaSuccess) return cuda_fail(e, "pair energy split launch");
  {
    const int g = pair_block(L, nocc);
    int i0, j0, i1, j1;
    host_pair_of(pair_begin, i0, j0);
    host_pair_of(pair_end - 1, i1, j1);
    const long long chunks = (j1 - j0) / g + 1;
    pair_order_kernel<<<static_cast<unsigned>((chunks + 127) / 128), 128, 0, stream>>>(
        pair_begin, pair_end, g, order);
  }

  PairParams p{};
  p.digA = dig;
  p.digB = digb;
  p.rows_pad = L.rows_pad;
  p.nv_pad = static_cast<int>(L.nv_pad);
  p.nocc = static_cast<int>(nocc);
  p.nvir = static_cast<int>(nvir);
  p.naux_p = static_cast<int>(L.naux_p);
  p.pair_begin = pair_begin;
  p.order = order;
  p.num_units = num_units;
  p.units_per_pair = upp;
  p.nR = static_cast<int>(ceil_div(nvir, 128));
  p.nC = static_cast<int>(ceil_div(nvir, 64));
  p.exps = exps;
  p.rowsq = rowsq;
  p.eps_occ = eps_occ;
  p.eps_vir = eps_vir;
  p.partials = partials;
  p.status = status;
  p.timeout_ns = wait_timeout_ns();

  const int dev = current_device();
  if (b254) {
    static bool attr_set[64] = {};
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
      e = cudaFuncSetAttribute(pair_energy254_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               Pe254::SMEM);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(pair energy smem)");
      if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    pair_energy254_kernel<<<grid, Pe254::THREADS, Pe254::SMEM, stream>>>(p);
  } else {
    constexpr int smem = kPairStages * PairCfg<kPairSlices>::STAGE_BYTES + 1024 + 256;
    auto kern = pair_energy_kernel<kPairSlices, kPairStages>;
    static bool attr_set[64] = {};
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(pair energy smem)");
      if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    kern<<<grid, kPairThreads, smem, stream>>>(p);
  }
  pair_energy_finish<<<1, 32, 0, stream>>>(partials, grid, energy);
  e = cudaGetLastError();
  return e == cudaSuccess ? TRNBLAS_OK : cuda_fail(e, "pair energy launch");
}

}  // extern "C"
