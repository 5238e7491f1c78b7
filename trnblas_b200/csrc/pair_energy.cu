// Fused DF-MP2 pair energy on the int8 tensor cores.
//
// E = sum over occupied pairs i <= j (weight 1 if i == j, else 2) of
//     sum_{a,b} T_ab (2 T_ab - T_ba) / (e_i + e_j - e_a - e_b),  T = B_i B_j^T,
// following the reference's symmetric pair walk (trnblas/nki/dispatch.py:
// 2648-2677: e_ij = e_ji, so off-diagonal pairs count twice).
//
// Numerics. Tensor-core fp32 accumulation truncates, a bias that grows with
// naux and would put E off by ~1e-5 relative; the 1e-9 target needs T free
// of systematic error. So B is split per row (i, a) into int8 digit planes
// with a power-of-two exponent and T is formed from exact int32 sums of
// slice products (pair_energy254.cuh: 4 base-254 digits, 10 products; naux
// longer than one int32-exact chunk runs in chunks folded in fp64).
// Denominators e_i + e_j - e_a - e_b are exact in fp64, quotients and sums
// are fp64 and partial sums are reduced in a fixed order, so the result is
// deterministic.
//
// Work unit: pair (i, j), a 128-row block R of a and a 64-column block C of b
// with C >= 2R (64-blocks 2R and 2R+1 lie inside R). Two passes over naux:
//   X = B_i[R] . B_j[C]^T  ->  X[a, b] = T_ab
//   Y = B_j[R] . B_i[C]^T  ->  Y[a, b] = T_ba
// so T_ab and T_ba land in the same TMEM lane and column: no transpose. Per
// (a, b): if the 64-blocks of a and b differ, the unit accounts for both
// ordered pairs, [X(2X-Y) + Y(2Y-X)] / D; if they are the same block,
// X(2X-Y) / D once; a in block 2R+1 with b in block 2R is skipped (unit
// (R, 2R+1) counted it). The nvir x nvir T never reaches HBM.
#include <algorithm>
#include <cstdlib>
#include <cmath>
#include <string>

#include "ozaki_split.cuh"
#include "runtime.hpp"

namespace tb {

struct PairParams {
  long long rows_pad;      // nocc * nv_pad (digit rows (i, a) at i * nv_pad + a)
  int nv_pad;              // nvir rounded up to 128 (zero rows beyond nvir)
  int nocc, nvir, naux_p;  // naux_p: K columns of the digit planes (multiple of the stage K)
  long long pair_begin;
  const int2* order;       // (i, j) of the range's pairs in processing order
  long long num_units;     // pairs * units_per_pair
  int units_per_pair;
  int nR, nC;              // 128-blocks and 64-blocks of nvir
  const int* exps;         // nocc * nvir
  const double* rowsq;     // nocc * nvir fp64 row sums of squares
  const float* eps_occ;
  const float* eps_vir;
  double* partials;        // gridDim.x
  int* wave_ctr;           // soft wave synchronisation counter (nullptr: none)
  int sync_kb, sync_lag;   // its group length (stages) and lag (groups)
  int* status;
  unsigned long long timeout_ns;
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

// Row block R and column block C of unit u inside its pair (no memory access).
__device__ __forceinline__ void unit_rc(const PairParams& p, long long u, int& R, int& C) {
  const long long pr = u / p.units_per_pair;
  int loc = static_cast<int>(u - pr * p.units_per_pair);
  R = 0;
  while (R < p.nR) {
    const int cnt = p.nC - 2 * R;
    if (loc < cnt) break;
    loc -= cnt;
    ++R;
  }
  C = 2 * R + loc;
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

constexpr int kMaxGrid = 1024;

struct PairLayout {
  long long naux_p, R, nv_pad, rows_pad;
  int slices;
  size_t off_exps, off_max, off_range, off_rowsq, off_part, off_order, total;
};

PairLayout pair_layout(long long nocc, long long nvir, long long naux, long long npairs) {
  PairLayout L{};
  L.slices = Pe254::KS;
  L.naux_p = round_up(std::max<long long>(naux, 1), Pe254::SW);
  L.R = nocc * nvir;
  L.nv_pad = round_up(std::max<long long>(nvir, 1), 128);
  L.rows_pad = nocc * L.nv_pad;
  // the digits (pe_digit_offset), read by both MMA operands
  const size_t dig = static_cast<size_t>(round_up(L.slices * L.rows_pad * L.naux_p, 256));
  L.off_exps = dig;
  L.off_max = L.off_exps + round_up(4 * L.R, 256);
  L.off_range = L.off_max + round_up(8 * L.R, 256);
  L.off_rowsq = L.off_range + 256;
  L.off_part = L.off_rowsq + round_up(8 * L.R, 256);
  L.off_order = L.off_part + round_up(8 * kMaxGrid, 256);
  L.total = L.off_order + round_up(8 * std::max<long long>(npairs, 1), 256);
  return L;
}

double l2_bytes() {
  int l2 = 0;
  if (cudaDeviceGetAttribute(&l2, cudaDevAttrL2CacheSize, current_device()) != cudaSuccess || l2 <= 0)
    l2 = 96 << 20;
  return static_cast<double>(l2);
}

// Pair-block width g of the processing order: the digits of 2g occupied
// orbitals should fit in half of L2.
int pair_block(const PairLayout& L, long long nocc) {
  const double l2 = l2_bytes();
  const double per_orb = static_cast<double>(L.slices) * static_cast<double>(L.nv_pad) * L.naux_p;
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

// Soft wave synchronisation of the pair walk (pe254_group_target): group
// length in stages (TRNBLAS_B200_PAIR_SYNC, 0 = off) and lag in groups
// (TRNBLAS_B200_PAIR_SYNC_LAG). Measured at config 5b (96 / 2208 / 6912) on
// one box: group length 8 / 16 / 32 / 64 stages 1745 / 1646 / 1600 / 1601 ms
// a launch (lags 1 and 2 no better than 0); without it 2.29-2.35 s on
// another box that took 1.48 s with 16-stage groups. In lock-step the MMA
// waits for its stages ~35-40 % of the time (the CTAs' loads arrive in
// bursts); neither L2 prefetches of later stages nor per-CTA rotations of
// the K order changed that (measured, then removed). Used only when the
// digits outgrow L2 (below that they stay resident whatever the order;
// config 3's 113 MB: no change either way).
int env_int(const char* name, int dflt) {
  const char* s = std::getenv(name);
  return (s && *s) ? std::atoi(s) : dflt;
}
int pair_sync_kb() {
  static const int v = env_int("TRNBLAS_B200_PAIR_SYNC", 32);
  return v > 0 ? v : 0;
}
int pair_sync_lag() {
  static const int v = env_int("TRNBLAS_B200_PAIR_SYNC_LAG", 0);
  return v > 0 ? v : 0;
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
  if (naux > (1ll << 30)) {
    set_error("trnblas_pair_energy: naux above 2^30");
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
  int* exps = reinterpret_cast<int*>(ws + L.off_exps);
  SplitScratch sc{reinterpret_cast<unsigned long long*>(ws + L.off_max),
                  reinterpret_cast<int*>(ws + L.off_range)};
  double* partials = reinterpret_cast<double*>(ws + L.off_part);
  int2* order = reinterpret_cast<int2*>(ws + L.off_order);
  double* rowsq = reinterpret_cast<double*>(ws + L.off_rowsq);
  // per-row exponents and sums of squares, then the base-254 digits
  cudaError_t e = cudaSuccess;
  {
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
        static_cast<int>(L.naux_p), exps, dig);
    e = cudaGetLastError();
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

  // The digits as a 5-D tensor: bytes of a 256-byte row, the 16 rows of one
  // plane of a 64-row block, row blocks, planes, K superslabs; the A operand
  // reads two row blocks at a time, the B operand one.
  CUtensorMap map_a, map_b;
  {
    const uint64_t nblk = static_cast<uint64_t>(L.rows_pad / 64);
    const uint64_t dims[5] = {256, 16, nblk, static_cast<uint64_t>(Pe254::KS),
                              static_cast<uint64_t>(L.naux_p / Pe254::SW)};
    const uint64_t strides[4] = {256, 4096, nblk * 4096, Pe254::KS * nblk * 4096};
    const uint32_t box_a[5] = {256, 16, 2, Pe254::KS, 1};
    const uint32_t box_b[5] = {256, 16, 1, Pe254::KS, 1};
    if (!encode_map(&map_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, dig, 5, dims, strides, box_a,
                    CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode_map(&map_b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, dig, 5, dims, strides, box_b,
                    CU_TENSOR_MAP_SWIZZLE_NONE))
      return TRNBLAS_ERR_ALIGN;
  }

  PairParams p{};
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
  p.sync_kb = pair_sync_kb();
  p.sync_lag = pair_sync_lag();
  p.wave_ctr = (p.sync_kb > 0 && static_cast<double>(L.off_exps) > l2_bytes()) ? wave_counter(stream)
                                                                                 : nullptr;
  if (!p.wave_ctr) p.sync_kb = 1;  // unused; keeps the producer's modulo defined
  p.status = status;
  p.timeout_ns = wait_timeout_ns();

  const int dev = current_device();
  {
    static bool attr_set[64] = {};
    if (dev < 0 || dev >= 64 || !attr_set[dev]) {
      e = cudaFuncSetAttribute(pair_energy254_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               Pe254::SMEM);
      if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(pair energy smem)");
      if (dev >= 0 && dev < 64) attr_set[dev] = true;
    }
    pair_energy254_kernel<<<grid, Pe254::THREADS, Pe254::SMEM, stream>>>(p, map_a, map_b);
  }
  pair_energy_finish<<<1, 32, 0, stream>>>(partials, grid, energy);
  e = cudaGetLastError();
  return e == cudaSuccess ? TRNBLAS_OK : cuda_fail(e, "pair energy launch");
}

}  // extern "C"
