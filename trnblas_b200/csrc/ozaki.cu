// fp64-class GEMM by Ozaki splitting on the int8 tensor cores (kind::i8).
//
// op(A) (M x K) is split per row and op(B) (K x N) per column into `k`
// balanced 7-bit digit planes (ozaki_split.cuh), written in the blocked layout
// that is the MMA's shared-memory image, so all k planes of one row block of
// one K slab are one contiguous chunk: a pipeline stage is two bulk copies.
// For an output tile the K loop stages all k A-planes (128 rows) and
// all k B-planes (BN rows, stacked along N) of one 32-wide K slab per pipeline
// stage, then issues the slice
// products of every diagonal d = s + t <= k - 1 into int32 TMEM accumulators,
// diagonal d at TMEM columns [d*BN, (d+1)*BN). Because the B-planes are
// contiguous along N, one MMA of A-plane s against B-planes t0 .. t0+n-1
// (N = n*BN <= 256) lands each product in its own diagonal: k = 8 needs 12
// MMAs per K slab for its 36 slice products. Integer accumulation is exact
// (|S_d| <= (d+1) * K * 2^12 < 2^31 for the K block a launch covers), so the
// epilogue sees the exact diagonal sums S_d and forms, in fp64,
//     acc = sum_{d = k-1 .. 0} fl(acc + S_d * 2^(7 (k-1-d)))
//     C   = acc * 2^(eA_i + eB_j - 12 - 7 (k-1))     (+ C when accumulating
//                                                    K blocks)
// in that order; the oracle restates it bit for bit.
#include <algorithm>
#include <string>

#include "ozaki_split.cuh"
#include "runtime.hpp"

namespace tb {

struct OzParams {
  const int8_t* dA;   // tiled digits of op(A): rows_a_pad rows
  const int8_t* dB;   // tiled digits of op(B)^T: rows_b_pad rows
  long long rows_a_pad, rows_b_pad;
  int M, N, Kp;       // Kp: K columns of the digit planes covered by this launch
  int k0;             // first K column of this launch (multiple of 32)
  int slices;
  int tiles_m, tiles_n, num_tiles;
  const int* expA;    // M
  const int* expB;    // N
  double* C;
  long long ldc;
  int accumulate;     // C += result (later K blocks)
  int* status;
  unsigned long long timeout_ns;
};

template <int BN, int KSMAX>
struct OzCfg {
  static constexpr int BM = 128;
  static constexpr int BK = 32;                  // one 32-byte MMA K step of int8
  static constexpr int A_PLANE = BM * BK;        // bytes
  static constexpr int B_PLANE = BN * BK;
  static constexpr int STAGE_BYTES = KSMAX * (A_PLANE + B_PLANE);
  static_assert(KSMAX * BN <= 512, "diagonal accumulators must fit TMEM");
  static constexpr int PLANES_PER_MMA = 256 / BN;
  static constexpr int BN_LOG2 = BN == 64 ? 6 : 5;
  static_assert(BN == 64 || BN == 32, "B row blocks of 32 or 64 rows");
};

// MMA issuer role for exactly KS slices (compile time): every product of
// diagonal d = s + t <= KS - 1 of each K slab, A-plane s against B-planes
// t0 .. t0 + np - 1 stacked along N, into TMEM columns (s + t0) * BN.
template <int BN, int KSMAX, int KS, int OFF>
__device__ __forceinline__ void oz_issue(uint64_t dA, uint64_t dB, uint32_t tmem_base,
                                         uint32_t acc) {
  using Cfg = OzCfg<BN, KSMAX>;
  constexpr int PPM = Cfg::PLANES_PER_MMA;
#pragma unroll
  for (int s = 0; s < KS; ++s) {
    const uint64_t ad = sdesc_add(dA, OFF + s * Cfg::A_PLANE);
#pragma unroll
    for (int t0 = 0; t0 < KS - s; t0 += PPM) {
      const int np = (KS - s - t0 < PPM) ? KS - s - t0 : PPM;
      mma_i8(tmem_base + (s + t0) * BN, ad, sdesc_add(dB, OFF + t0 * Cfg::B_PLANE),
             idesc(kAccS32, kFmtS8, kFmtS8, 0, 0, Cfg::BM, np * BN), (acc || s) ? 1u : 0u);
    }
  }
}

// MMA issuer role for exactly KS slices (compile time): every product of
// diagonal d = s + t <= KS - 1 of each K slab, A-plane s against B-planes
// t0 .. t0 + np - 1 stacked along N, into TMEM columns (s + t0) * BN. The
// loop runs over this CTA's stream of `total` K slabs (tiles x num_kb) and is
// unrolled over the pipeline stages, so every shared-memory offset and
// barrier address is a compile-time constant: a tcgen05.mma issue holds the
// issuing thread until the tensor pipe is nearly ready for it, so scalar work
// between the MMAs of consecutive K slabs would leave the pipe idle.
template <int BN, int KSMAX, int STAGES, int KS>
__device__ __forceinline__ void oz_mma_role(uint8_t* smem, uint64_t* full_bar, uint64_t* empty_bar,
                                            uint64_t* accf_bar, uint64_t* acce_bar,
                                            uint32_t tmem_base, int num_kb, long long total,
                                            const Abort& ab) {
  using Cfg = OzCfg<BN, KSMAX>;
  const uint32_t base = smem_u32(smem);
  const uint64_t dA = sdesc_kmajor_noswz(base, 128, 256);
  const uint64_t dB = sdesc_kmajor_noswz(base + KSMAX * Cfg::A_PLANE, 128, 256);
  uint32_t phase = 0;
  int it = 0;   // tiles started
  int kbt = 0;  // K slab within the current tile
  bool stop = false;
  for (long long g = 0; g < total && !stop; g += STAGES) {
    static_for<0, STAGES>([&](auto sc) {
      constexpr int S = decltype(sc)::value;
      if (stop || g + S >= total) return;
      if (kbt == 0) {
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
      oz_issue<BN, KSMAX, KS, S * Cfg::STAGE_BYTES>(dA, dB, tmem_base, kbt > 0 ? 1u : 0u);
      tc_commit(&empty_bar[S]);
      if (++kbt == num_kb) {
        kbt = 0;
        ++it;
        tc_commit(accf_bar);
      }
    });
    phase ^= 1u;
  }
}

template <int BN, int KSMAX, int STAGES>
__global__ void __launch_bounds__(192, 1)
    ozaki_gemm_kernel(const OzParams p) {
  using Cfg = OzCfg<BN, KSMAX>;
  constexpr int BM = Cfg::BM;
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

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const Abort ab{abort_flag, p.status, p.timeout_ns};
  const int ks = p.slices;
  const uint32_t stage_tx = static_cast<uint32_t>(ks) * (Cfg::A_PLANE + Cfg::B_PLANE);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(accf_bar, 1);
    mbar_init(acce_bar, 4);
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_kb = (p.Kp + Cfg::BK - 1) / Cfg::BK;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    bool aborted = false;
    for (int t = blockIdx.x; t < p.num_tiles && !aborted; t += gridDim.x) {
      const int mb = t % p.tiles_m, nb = t / p.tiles_m;  // M fastest: B planes reused in L2
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, ab, kTimeoutEmpty)) {
          aborted = true;
          break;
        }
        uint8_t* sa = smem + stage * Cfg::STAGE_BYTES;
        uint8_t* sb = sa + KSMAX * Cfg::A_PLANE;
        mbar_arrive_expect_tx(&full_bar[stage], stage_tx);
        const int kc = p.k0 + kb * Cfg::BK;
        // all ks planes of each operand's row block: one contiguous chunk each
        bulk_load(sa, p.dA + blocked_chunk(kc >> 5, mb, ks, p.rows_a_pad, 7),
                  static_cast<uint32_t>(ks) * Cfg::A_PLANE, &full_bar[stage]);
        bulk_load(sb, p.dB + blocked_chunk(kc >> 5, nb, ks, p.rows_b_pad, Cfg::BN_LOG2),
                  static_cast<uint32_t>(ks) * Cfg::B_PLANE, &full_bar[stage]);
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    if (aborted || ab.raised()) {
      int s = stage;
      uint32_t ph = phase;
      for (int i = 0; i < STAGES; ++i) {
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
    // One fully unrolled issue loop per slice count: with compile-time plane
    // offsets and shapes an MMA costs a few instructions to issue, where the
    // runtime-ks loop spent more issue time than the tensor pipe spent on the
    // (often narrow) MMAs themselves.
    const long long my_tiles =
        p.num_tiles > static_cast<int>(blockIdx.x) ? (p.num_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const long long total = my_tiles * num_kb;
    switch (ks) {
#define TB_OZ_CASE(KS_)                                                        \
  case KS_:                                                                    \
    if constexpr (KS_ <= KSMAX && (KS_ > 8) == (BN == 32))                     \
      oz_mma_role<BN, KSMAX, STAGES, KS_>(smem, full_bar, empty_bar, accf_bar,   \
                                          acce_bar, tmem_base, num_kb, total, ab); \
    break;
      TB_OZ_CASE(1) TB_OZ_CASE(2) TB_OZ_CASE(3) TB_OZ_CASE(4) TB_OZ_CASE(5) TB_OZ_CASE(6)
      TB_OZ_CASE(7) TB_OZ_CASE(8) TB_OZ_CASE(9) TB_OZ_CASE(10) TB_OZ_CASE(11) TB_OZ_CASE(12)
#undef TB_OZ_CASE
      default:
        break;
    }
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
    const int q = warp & 3;
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(32 * q) << 16);
    const int off = -12 - 7 * (ks - 1);
    int it = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++it) {
      if (!mbar_wait_warp(accf_bar, it & 1, ab, kTimeoutAccFull)) break;
      tc_fence_after();
      const int mb = t % p.tiles_m, nb = t / p.tiles_m;
      const int r = mb * BM + 32 * q + lane;
      const int ea = (r < p.M) ? p.expA[r] + off : 0;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        double acc[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) acc[j] = 0.0;
#pragma unroll 1
        for (int d = ks - 1; d >= 0; --d) {
          uint32_t v[32];
          tmem_ld32(lane_base + d * BN + c * 32, v);
          tmem_ld_wait();
          const double w = pow2d(7 * (ks - 1 - d));
#pragma unroll
          for (int j = 0; j < 32; ++j)
            acc[j] = acc[j] + static_cast<double>(static_cast<int>(v[j])) * w;
        }
        const int n0 = nb * BN + c * 32;
        if (r < p.M) {
          double* crow = p.C + static_cast<long long>(r) * p.ldc;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int n = n0 + j;
            if (n < p.N) {
              double val = scale2(acc[j], ea + p.expB[n]);
              if (p.accumulate) val = crow[n] + val;
              crow[n] = val;
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acce_bar);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();  // lane 0 arrives from the MMA role, 1..31 straight here
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

namespace {

template <int BN, int KSMAX, int STAGES>
int launch_oz(const OzParams& p, cudaStream_t stream) {
  constexpr int smem = STAGES * OzCfg<BN, KSMAX>::STAGE_BYTES + 1024 + 256;
  auto kern = ozaki_gemm_kernel<BN, KSMAX, STAGES>;
  static bool attr_set[64] = {};
  const int dev = current_device();
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(ozaki smem)");
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const int grid = static_cast<int>(std::min<long long>(p.num_tiles, num_sms()));
  kern<<<grid, 192, smem, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TRNBLAS_OK : cuda_fail(e, "ozaki kernel launch");
}

struct OzLayout {
  long long kp;        // K padded to 32 (digit plane row length)
  long long ma, nb;    // rows of the tiled A (multiple of 128) and B (multiple of 64)
  size_t dig_a, dig_b; // bytes
  size_t off_dig_b, off_exp_a, off_exp_b, off_max, off_range, total;
};

OzLayout oz_layout(long long M, long long N, long long K, int slices) {
  OzLayout L{};
  L.kp = round_up(std::max<long long>(K, 1), 32);
  L.ma = round_up(std::max<long long>(M, 1), 128);
  L.nb = round_up(std::max<long long>(N, 1), 64);
  L.dig_a = static_cast<size_t>(round_up(slices * L.ma * L.kp, 256));
  L.dig_b = static_cast<size_t>(round_up(slices * L.nb * L.kp, 256));
  L.off_dig_b = L.dig_a;
  L.off_exp_a = L.off_dig_b + L.dig_b;
  L.off_exp_b = L.off_exp_a + round_up(4 * M, 256);
  L.off_max = L.off_exp_b + round_up(4 * N, 256);
  L.off_range = L.off_max + round_up(8 * std::max(M, N), 256);
  L.total = L.off_range + 256;
  return L;
}

// Largest K block whose diagonal sums stay below 2^31: (d+1) * Kb * 2^12.
long long k_block(int slices) {
  const long long kb = ((1ll << 31) - 1) / (static_cast<long long>(slices) * 4096);
  return (kb / 32) * 32;
}

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" {

size_t trnblas_gemm_fp64_workspace_size(int64_t M, int64_t N, int64_t K, int slices) {
  if (M <= 0 || N <= 0 || K <= 0 || slices < 1 || slices > 12) return 0;
  return oz_layout(M, N, K, slices).total;
}

int trnblas_ozaki_split(int64_t R, int64_t K, const double* X, int64_t rs, int64_t ks, int slices,
                        int8_t* digits, int64_t ldd, int32_t* exps, void* workspace,
                        size_t workspace_bytes, void* stream) {
  if (R < 0 || K < 0 || slices < 1 || slices > 12 || ldd < K || R > (1ll << 31) - 1 ||
      ldd > (1ll << 31) - 1) {
    set_error("trnblas_ozaki_split: bad size or slices (1..12)");
    return TRNBLAS_ERR_ARG;
  }
  if (R == 0) return TRNBLAS_OK;
  if (!workspace || workspace_bytes < static_cast<size_t>(8 * R + 256)) {
    set_error("trnblas_ozaki_split needs 8 * R + 256 workspace bytes");
    return TRNBLAS_ERR_WORKSPACE;
  }
  if (!digits || !exps || (K > 0 && !X)) {
    set_error("trnblas_ozaki_split: NULL pointer");
    return TRNBLAS_ERR_ARG;
  }
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  SplitScratch sc{reinterpret_cast<unsigned long long*>(ws),
                  reinterpret_cast<int*>(ws + round_up(8 * R, 16))};
  cudaError_t e = launch_split(X, rs, ks, static_cast<int>(R), static_cast<int>(K),
                               static_cast<int>(ldd), slices, digits, exps, sc,
                               static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TRNBLAS_OK : cuda_fail(e, "ozaki split launch");
}

int trnblas_gemm_fp64(int64_t M, int64_t N, int64_t K, const double* A, int64_t lda, int transA,
                      const double* B, int64_t ldb, int transB, int slices, double* C,
                      int64_t ldc, void* workspace, size_t workspace_bytes, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (M < 0 || N < 0 || K < 0 || slices < 1 || slices > 12) {
    set_error("trnblas_gemm_fp64: bad size or slices (1..12)");
    return TRNBLAS_ERR_ARG;
  }
  const long long lim = (1ll << 31) - 1;
  if (M > lim || N > lim || K > lim) {
    set_error("trnblas_gemm_fp64: size exceeds 2^31-1");
    return TRNBLAS_ERR_ARG;
  }
  if (M == 0 || N == 0) return TRNBLAS_OK;
  if (!C || ldc < N) {
    set_error("trnblas_gemm_fp64: NULL C or ldc < N");
    return TRNBLAS_ERR_ARG;
  }
  if (K == 0) {
    cudaError_t e = cudaMemset2DAsync(C, ldc * 8, 0, N * 8, M, stream);
    return e == cudaSuccess ? TRNBLAS_OK : cuda_fail(e, "cudaMemset2DAsync");
  }
  if (!A || !B) {
    set_error("trnblas_gemm_fp64: NULL operand");
    return TRNBLAS_ERR_ARG;
  }
  const OzLayout L = oz_layout(M, N, K, slices);
  if (!workspace || workspace_bytes < L.total) {
    set_error("trnblas_gemm_fp64 needs " + std::to_string(L.total) + " workspace bytes");
    return TRNBLAS_ERR_WORKSPACE;
  }
  int* status = status_word();
  if (!status) return TRNBLAS_ERR_CUDA;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  int8_t* dA = reinterpret_cast<int8_t*>(ws);
  int8_t* dB = reinterpret_cast<int8_t*>(ws + L.off_dig_b);
  int* eA = reinterpret_cast<int*>(ws + L.off_exp_a);
  int* eB = reinterpret_cast<int*>(ws + L.off_exp_b);
  SplitScratch sc{reinterpret_cast<unsigned long long*>(ws + L.off_max),
                  reinterpret_cast<int*>(ws + L.off_range)};
  // op(A)(m, k): strides; op(B)^T(n, k) = op(B)(k, n)
  const long long ars = transA ? 1 : lda, aks = transA ? lda : 1;
  const long long brs = transB ? ldb : 1, bks = transB ? 1 : ldb;
  // one group of M (N) real rows padded to L.ma (L.nb): padding rows are zero
  const bool wide = slices <= 8;  // BN = 64 holds 8 diagonals; 9..12 use BN = 32
  const int BN = wide ? 64 : 32;
  // A in row blocks of 128 (the MMA's M), B in row blocks of BN
  cudaError_t e = launch_split_tiled(A, ars, aks, static_cast<int>(M), static_cast<int>(K), M,
                                     L.ma, L.ma, static_cast<int>(L.kp), slices, dA, 7, nullptr,
                                     0, eA, sc, stream);
  if (e == cudaSuccess)
    e = launch_split_tiled(B, brs, bks, static_cast<int>(N), static_cast<int>(K), N, L.nb, L.nb,
                           static_cast<int>(L.kp), slices, dB, wide ? 6 : 5, nullptr, 0, eB, sc,
                           stream);
  if (e != cudaSuccess) return cuda_fail(e, "ozaki split launch");

  OzParams p{};
  p.dA = dA;
  p.dB = dB;
  p.rows_a_pad = L.ma;
  p.rows_b_pad = L.nb;
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.slices = slices;
  p.tiles_m = static_cast<int>(ceil_div(M, 128));
  p.tiles_n = static_cast<int>(ceil_div(N, BN));
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.expA = eA;
  p.expB = eB;
  p.C = C;
  p.ldc = ldc;
  p.status = status;
  p.timeout_ns = wait_timeout_ns();
  const long long kbmax = k_block(slices);
  for (long long k0 = 0; k0 < L.kp; k0 += kbmax) {
    p.k0 = static_cast<int>(k0);
    p.Kp = static_cast<int>(std::min(kbmax, L.kp - k0));
    p.accumulate = k0 > 0;
    const int rc = wide ? launch_oz<64, 8, 4>(p, stream) : launch_oz<32, 12, 3>(p, stream);
    if (rc) return rc;
  }
  return TRNBLAS_OK;
}

}  // extern "C"
