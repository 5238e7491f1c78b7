// Warp-specialised, persistent tcgen05 GEMM engine for sm_100a.
//
// One CTA per SM walks output tiles with a static stride. Six warps:
//   warp 0      TMA producer (one elected thread) filling a STAGES-deep ring;
//   warp 1      TMEM owner + MMA issuer (one elected thread);
//   warps 2..5  epilogue: tcgen05.ld of the accumulator, alpha/beta and the
//               C operand fused, converted and stored straight to global.
// The accumulator is multi-buffered in TMEM so the epilogue of one tile (or K
// chunk) overlaps the main loop of the next.
//
// Operand kinds:
//   kF16   bf16 / fp16 operands, kind::f16, fp32 accumulate, one product.
//          Each operand is K-major or MN-major (the layout a transposed or
//          row-major B gives) -- no transposed copies are made.
//   kTF32x3 fp32 API: operands pre-split into (hi, lo) with hi = tf32(x) and
//          lo = x - hi; acc += lo*hi + hi*lo + hi*hi on kind::tf32, which holds
//          about 2^-22 relative error per product (fp32-class). K-major only.
//
// Modes:
//   GEMM  tiles of D[b] = alpha * op(A[b]) op(B[b]) + beta * C[b], batched
//         over a grid dimension folded into the tile index;
//   SYRK  lower-triangle tiles only (BM x BM, or BM x 2BM over column-block
//         pairs); each value v(r,c), r >= c, is stored at (r,c) and mirrored
//         to (c,r), so the full symmetric result is exactly symmetric and the
//         upper tiles are never computed.
#pragma once

#include "common.cuh"

namespace tb {

// kTF32x3F: the fp32 API with the split fused into the kernel: TMA loads the
// raw fp32 tiles (K-major: 128-byte swizzle rows of 32 K; MN-major: boxes
// of 32 MN x 32 K with the 128-byte swizzle of 32-byte atoms) into the "hi"
// slots and converter warps write lo = x - trunc19(x) beside them. The tensor core reads only the top
// 19 bits of a kind::tf32 operand (measured: a product of raw fp32 inputs
// equals the product of inputs truncated to tf32 within the fp32 accumulate
// rounding, 6e-8, and differs from rounded inputs by 1.2e-3), so the raw tile
// serves as hi and hi + lo = x exactly; no hi / lo planes in global memory.
enum GemmKind : int { kF16 = 0, kTF32x3 = 1, kTF32x3F = 2 };
enum OutKind : int { kOutF32 = 0, kOutBF16 = 1, kOutF16 = 2 };
// kModeSyrk: lower-triangle BM x BM tiles; kModeSyrkWide: BM x BN tiles
// (BN = 2 BM) over the lower triangle's column-block pairs, row m holding
// pairs 0 .. m / 2 (the last pair of an even row also spans the strictly upper
// block (m, m + 1), which the epilogue skips).
enum GemmMode : int { kModeGemm = 0, kModeSyrk = 1, kModeSyrkWide = 2 };
// How the epilogue reads C: not at all, C[r][c], or (SYRK, upper-triangle
// storage) C[c][r] for the lower element (r, c).
enum CMode : int { kCNone = 0, kCRow = 1, kCTrans = 2 };

struct GemmParams {
  int M, N, K;
  int batch;
  int a_batched, b_batched;  // TMA batch coordinate = batch index, or 0 (broadcast)
  int a_mn, b_mn;            // operand smem layout: 0 = K-major, 1 = MN-major
  int mode;                  // GemmMode
  int out_kind;              // OutKind
  int in_fmt;                // kFmtBF16 / kFmtF16 / kFmtTF32 (instruction descriptor)
  int c_mode;                // CMode
  float alpha, beta;
  const void* C;
  long long ldc, strideC;
  void* D;
  long long ldd, strideD;
  int tiles_m, tiles_n, num_tiles;
  int group_m;
  int* status;
  unsigned long long timeout_ns;
  int* wave_ctr;  // tile-wave synchronisation counter (nullptr: none)
  // Operands that arrive while the kernel runs (the SPMD GEMM's shards, copied
  // in by the copy engines): before loading a tile the producer waits until
  // ready[row tile / shard_tiles_m] and ready[ready_b0 + batch index] reach
  // ready_epoch. The walk is rotated by rot_m row tiles and rot_b batch
  // entries so that the tiles of the shards already in place come first.
  const int* ready;  // nullptr: operands resident
  int ready_epoch;
  int shard_tiles_m, ready_b0;
  int rot_m, rot_b;
  // Triangular operand (trmm): 0 none; op(A) 1 lower / 2 upper; op(B)
  // 3 lower / 4 upper. The operand holds exact zeros outside its triangle,
  // and each tile runs only the K blocks its rows (A) or columns (B) reach.
  int tri;
};

// K blocks [lo, hi) a tile with rows [m0, m0 + bm) and columns [n0, n0 + bn)
// runs (all of them unless an operand is triangular; at least one block).
__device__ __forceinline__ void tile_k_range(const GemmParams& p, int m0, int bm, int n0, int bn,
                                             int bk, int num_kb, int& lo, int& hi) {
  lo = 0;
  hi = num_kb;
  if (p.tri == 1) hi = min(num_kb, (m0 + bm + bk - 1) / bk);  // A[m][k] = 0 for k > m
  if (p.tri == 2) lo = min(num_kb, m0 / bk);                    // A[m][k] = 0 for k < m
  if (p.tri == 3) lo = min(num_kb, n0 / bk);                    // B[k][n] = 0 for k < n
  if (p.tri == 4) hi = min(num_kb, (n0 + bn + bk - 1) / bk);  // B[k][n] = 0 for k > n
  if (hi <= lo) {
    lo = min(lo, num_kb - 1);
    hi = lo + 1;
  }
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Wait (bounded) until *flag has reached `epoch` (wrap-safe comparison); the
// proxy fence orders the TMA loads that follow after the flag's data.
__device__ __forceinline__ bool wait_ready(const int* flag, int epoch, const Abort& ab) {
  if (ld_acquire_gpu(flag) - epoch < 0) {
    const unsigned long long t0 = globaltimer_ns();
    while (ld_acquire_gpu(flag) - epoch < 0) {
      if (ab.raised()) return false;
      if (globaltimer_ns() - t0 > ab.timeout_ns) {
        ab.raise(kTimeoutAux);
        return false;
      }
      __nanosleep(256);
    }
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
  return true;
}

// x - trunc19(x): the part of x below the 19 bits a kind::tf32 operand keeps
// (exact in fp32); 0 for inf / nan.
__device__ __forceinline__ float tf32_lo(float x) {
  const uint32_t u = __float_as_uint(x);
  if ((u & 0x7F800000u) == 0x7F800000u) return 0.0f;
  return x - __uint_as_float(u & 0xFFFFE000u);
}

// Shared memory after the pipeline stages: 256 bytes of barriers, then one
// 4 KB transpose stage per epilogue warp (SYRK mirror stores).
constexpr int kGemmBarBytes = 256;
constexpr int kEpiStageBytes = 4 * 32 * 32 * 4;

template <int KIND, int BN>
struct GemmCfg {
  static constexpr int BM = 128;
  static constexpr bool TF32 = (KIND == kTF32x3 || KIND == kTF32x3F);
  static constexpr int ESIZE = (KIND == kF16) ? 2 : 4;
  static constexpr int BK = 128 / ESIZE;  // one 128-byte swizzle row of K
  static constexpr int NPARTS = TF32 ? 2 : 1;  // hi/lo
  static constexpr int A_TILE = BM * 128;  // bytes of one A part
  static constexpr int B_TILE = BN * 128;
  static constexpr int STAGE_BYTES = NPARTS * (A_TILE + B_TILE);
  // bytes the TMA loads per stage (the fused split computes the lo parts)
  static constexpr int LOAD_BYTES = (KIND == kTF32x3F) ? (A_TILE + B_TILE) : STAGE_BYTES;
  // warps: producer, MMA, 4 epilogue, and 2 converters for the fused split
  static constexpr int CONV_WARPS = 2;
  static constexpr int THREADS = 32 * (6 + ((KIND == kTF32x3F) ? CONV_WARPS : 0));
  // K blocks accumulated in TMEM before the epilogue takes the partial sum.
  // The tensor core accumulates fp32 with truncation, whose bias grows with
  // the number of accumulations; for the fp32 API the partial sums of 128-wide
  // K chunks are added in the epilogue with round-to-nearest instead, which
  // bounds the relative error near 1e-6 at any K. bf16 / fp16 results round
  // their output far above that bias, so they accumulate the whole K in TMEM.
  static constexpr int CHUNK_KB = TF32 ? 4 : (1 << 30);
  static constexpr int NBUF = TF32 ? 4 : 2;  // TMEM accumulator buffers
  static constexpr int TMEM_COLS = (NBUF * BN <= 32) ? 32 : (NBUF * BN <= 64) ? 64 : (NBUF * BN <= 128) ? 128 : (NBUF * BN <= 256) ? 256 : 512;
  static_assert(NBUF * BN <= 512, "TMEM holds 512 columns");
  static_assert(!TF32 || BN == 128, "chunked epilogue keeps 128 columns in registers");
};

// MMA issuer role over this CTA's stream of K blocks (tiles x num_kb), chunked
// into TMEM accumulator buffers as the epilogue expects (one chunk per tile
// for kF16, CHUNK_KB K blocks for kTF32x3). The loop is unrolled over the
// pipeline stages and the per-k-step descriptors are built once, so an MMA's
// operands are a register plus a compile-time stage offset: a tcgen05.mma
// issue holds the issuing thread until the tensor pipe is nearly ready for
// it, and scalar work between the MMAs of consecutive stages (stage index
// arithmetic, layout selects, descriptor rebuilds) shows up as idle tensor
// cycles.
__device__ __forceinline__ void decode_tile(const GemmParams& p, int t, int& bz, int& mb, int& nb);

// K blocks this CTA runs over all its tiles: my_tiles * num_kb, or for a
// triangular operand the sum of the tiles' K ranges (every role that walks
// the stage stream counts the same stages).
__device__ __forceinline__ long long cta_stage_total(const GemmParams& p, int bm, int bn, int bk,
                                                     int num_kb) {
  const int my_tiles =
      p.num_tiles > static_cast<int>(blockIdx.x) ? (p.num_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  if (!p.tri) return static_cast<long long>(my_tiles) * num_kb;
  long long total = 0;
  for (int ti = 0; ti < my_tiles; ++ti) {
    int bz, mb, nb, lo, hi;
    decode_tile(p, static_cast<int>(blockIdx.x) + ti * static_cast<int>(gridDim.x), bz, mb, nb);
    tile_k_range(p, mb * bm, bm, nb * bn, bn, bk, num_kb, lo, hi);
    total += hi - lo;
  }
  return total;
}

template <int KIND, int BN, int STAGES>
__device__ __forceinline__ void gemm_mma_role(const GemmParams& p, uint8_t* smem,
                                              uint64_t* full_bar, uint64_t* empty_bar,
                                              uint64_t* accf_bar, uint64_t* acce_bar,
                                              uint32_t tmem_base, int num_kb, const Abort& ab) {
  // full_bar: the stage's operands are complete (for kTF32x3F the converters'
  // barriers, which follow the TMA loads and the lo parts)
  using Cfg = GemmCfg<KIND, BN>;
  constexpr int SB = Cfg::STAGE_BYTES;
  const uint32_t idesc_v = idesc(kAccF32, p.in_fmt, p.in_fmt, p.a_mn, p.b_mn, Cfg::BM, BN);
  const uint32_t sa0 = smem_u32(smem);
  const uint32_t sb0 = sa0 + Cfg::NPARTS * Cfg::A_TILE;
  // k step kk of a stage: K-major operands advance 32 bytes inside the
  // 128-byte swizzled row, MN-major (16-bit only) 16 K-rows = 2048 bytes
  uint64_t ad[4], bd[4];
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    // MN-major: boxes of one 128-byte swizzle row of MN x BK K-rows, LBO the
    // box bytes, one k step = K rows of the MMA (16 for 16-bit, 8 for tf32)
    if constexpr (KIND == kF16) {
      ad[kk] = p.a_mn ? sdesc_sw128(sa0 + kk * 2048, 64 * 128, 1024) : sdesc_sw128(sa0 + kk * 32, 16, 1024);
      bd[kk] = p.b_mn ? sdesc_sw128(sb0 + kk * 2048, 64 * 128, 1024) : sdesc_sw128(sb0 + kk * 32, 16, 1024);
    } else if constexpr (KIND == kTF32x3F) {
      // MN-major: 4 KB boxes (32 MN x 32 K rows), one k step = 8 K rows
      ad[kk] = p.a_mn ? sdesc_sw128_atom32(sa0 + kk * 1024, 32 * 128, 512) : sdesc_sw128(sa0 + kk * 32, 16, 1024);
      bd[kk] = p.b_mn ? sdesc_sw128_atom32(sb0 + kk * 1024, 32 * 128, 512) : sdesc_sw128(sb0 + kk * 32, 16, 1024);
    } else {
      ad[kk] = sdesc_sw128(sa0 + kk * 32, 16, 1024);
      bd[kk] = sdesc_sw128(sb0 + kk * 32, 16, 1024);
    }
  }
  const int my_tiles =
      p.num_tiles > static_cast<int>(blockIdx.x) ? (p.num_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  // K blocks of this CTA's ti-th tile (fewer than num_kb only for a
  // triangular operand)
  auto tile_kb = [&](int ti) -> int {
    if (!p.tri) return num_kb;
    int bz, mb, nb, lo, hi;
    decode_tile(p, static_cast<int>(blockIdx.x) + ti * static_cast<int>(gridDim.x), bz, mb, nb);
    tile_k_range(p, mb * Cfg::BM, Cfg::BM, nb * BN, BN, Cfg::BK, num_kb, lo, hi);
    return hi - lo;
  };
  const long long total = cta_stage_total(p, Cfg::BM, BN, Cfg::BK, num_kb);
  int ti = 0;
  int cnt = my_tiles > 0 ? tile_kb(0) : 0;  // K blocks of the current tile
  uint32_t phase = 0;
  int gc = 0;   // accumulation chunks started
  int kbt = 0;  // K block within the tile
  int kbc = 0;  // K block within the chunk
  uint32_t d_tmem = tmem_base;
  bool stop = false;
  for (long long g = 0; g < total && !stop; g += STAGES) {
    static_for<0, STAGES>([&](auto sc) {
      constexpr int S = decltype(sc)::value;
      constexpr uint32_t OFF = static_cast<uint32_t>(S) * SB;
      if (stop || g + S >= total) return;
      if (kbc == 0) {
        const int buf = gc % Cfg::NBUF;
        const uint32_t bph = (gc / Cfg::NBUF) & 1;
        if (!mbar_wait(&acce_bar[buf], bph ^ 1u, ab, kTimeoutAccEmpty)) {
          stop = true;
          return;
        }
        tc_fence_after();
        d_tmem = tmem_base + buf * BN;
      }
      if (!mbar_wait(&full_bar[S], phase, ab, kTimeoutFull)) {
        stop = true;
        return;
      }
      tc_fence_after();
      const bool first = kbc == 0;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint32_t acc_in = (first && kk == 0) ? 0u : 1u;
        if constexpr (KIND == kF16) {
          mma_f16(d_tmem, sdesc_add(ad[kk], OFF), sdesc_add(bd[kk], OFF), idesc_v, acc_in);
        } else {
          const uint64_t ah = sdesc_add(ad[kk], OFF), al = sdesc_add(ad[kk], OFF + Cfg::A_TILE);
          const uint64_t bh = sdesc_add(bd[kk], OFF), bl = sdesc_add(bd[kk], OFF + Cfg::B_TILE);
          mma_tf32(d_tmem, al, bh, idesc_v, acc_in);  // small terms first
          mma_tf32(d_tmem, ah, bl, idesc_v, 1u);
          mma_tf32(d_tmem, ah, bh, idesc_v, 1u);
        }
      }
      tc_commit(&empty_bar[S]);
      ++kbt;
      ++kbc;
      if (kbc == Cfg::CHUNK_KB || kbt == cnt) {
        tc_commit(&accf_bar[gc % Cfg::NBUF]);
        ++gc;
        kbc = 0;
        if (kbt == cnt) {
          kbt = 0;
          ++ti;
          cnt = ti < my_tiles ? tile_kb(ti) : 0;
        }
      }
    });
    phase ^= 1u;
  }
}

__device__ __forceinline__ void decode_tile(const GemmParams& p, int t, int& bz, int& mb,
                                            int& nb) {
  if (p.mode == kModeSyrk) {
    // lower triangle, row-major over (mb, nb <= mb)
    int m = static_cast<int>((sqrtf(8.0f * static_cast<float>(t) + 1.0f) - 1.0f) * 0.5f);
    while (m * (m + 1) / 2 > t) --m;
    while ((m + 1) * (m + 2) / 2 <= t) ++m;
    bz = 0;
    mb = m;
    nb = t - m * (m + 1) / 2;
    return;
  }
  if (p.mode == kModeSyrkWide) {
    // rows before m hold S(m) tiles: S(2k) = k (k + 1), S(2k + 1) = (k + 1)^2
    auto S = [](int m) { const int k = m >> 1; return (m & 1) ? (k + 1) * (k + 1) : k * (k + 1); };
    int m = static_cast<int>(2.0f * sqrtf(static_cast<float>(t)));
    while (m > 0 && S(m) > t) --m;
    while (S(m + 1) <= t) ++m;
    bz = 0;
    mb = m;
    nb = t - S(m);
    return;
  }
  const int per_batch = p.tiles_m * p.tiles_n;
  bz = t / per_batch;
  int r = t - bz * per_batch;
  const int band = p.group_m * p.tiles_n;
  const int g = r / band;
  const int first_m = g * p.group_m;
  int gsz = p.tiles_m - first_m;
  if (gsz > p.group_m) gsz = p.group_m;
  const int rr = r - g * band;
  mb = first_m + rr % gsz;
  nb = rr / gsz;
  // triangular operand: the tiles with the longest K ranges first (rows from
  // the bottom for a lower op(A), columns from the right for an op(B) whose
  // range ends at its columns), so that the walk ends on short tiles
  if (p.tri == 1) mb = p.tiles_m - 1 - mb;
  if (p.tri == 4) nb = p.tiles_n - 1 - nb;
  if (p.ready) {
    bz = (bz + p.rot_b) % p.batch;
    mb = (mb + p.rot_m) % p.tiles_m;
  }
}

__device__ __forceinline__ float load_c(const void* C, int out_kind, long long idx) {
  if (out_kind == kOutF32) return __ldg(reinterpret_cast<const float*>(C) + idx);
  if (out_kind == kOutBF16)
    return __bfloat162float(
        __ushort_as_bfloat16(__ldg(reinterpret_cast<const unsigned short*>(C) + idx)));
  return __half2float(__ushort_as_half(__ldg(reinterpret_cast<const unsigned short*>(C) + idx)));
}

__device__ __forceinline__ void store_d(void* D, int out_kind, long long idx, float v) {
  if (out_kind == kOutF32) {
    reinterpret_cast<float*>(D)[idx] = v;
  } else if (out_kind == kOutBF16) {
    reinterpret_cast<__nv_bfloat16*>(D)[idx] = __float2bfloat16_rn(v);
  } else {
    reinterpret_cast<__half*>(D)[idx] = __float2half_rn(v);
  }
}

// Store out[0..31] at D[row offset drow + c0 ..]: 16-byte vector stores when
// all 32 columns exist and the row start is 16-byte aligned, else element by
// element up to column N.
__device__ __forceinline__ void store_row32(const GemmParams& p, long long drow, int c0,
                                            const float* out, bool full) {
  if (p.out_kind == kOutF32) {
    float* dp = reinterpret_cast<float*>(p.D) + drow + c0;
    if (full && (p.ldd % 4 == 0) && ((reinterpret_cast<uintptr_t>(dp) & 15) == 0)) {
      float4* d4 = reinterpret_cast<float4*>(dp);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        d4[j] = make_float4(out[4 * j], out[4 * j + 1], out[4 * j + 2], out[4 * j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (c0 + j < p.N) dp[j] = out[j];
    }
  } else {
    unsigned short* dp = reinterpret_cast<unsigned short*>(p.D) + drow + c0;
    if (full && (p.ldd % 8 == 0) && ((reinterpret_cast<uintptr_t>(dp) & 15) == 0)) {
      uint4* d4 = reinterpret_cast<uint4*>(dp);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint32_t w[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float lo = out[8 * j + 2 * h], hi = out[8 * j + 2 * h + 1];
          if (p.out_kind == kOutBF16) {
            __nv_bfloat162 b2 = __floats2bfloat162_rn(lo, hi);
            w[h] = *reinterpret_cast<uint32_t*>(&b2);
          } else {
            __half2 h2 = __floats2half2_rn(lo, hi);
            w[h] = *reinterpret_cast<uint32_t*>(&h2);
          }
        }
        d4[j] = make_uint4(w[0], w[1], w[2], w[3]);
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (c0 + j < p.N) store_d(p.D, p.out_kind, drow + c0 + j, out[j]);
    }
  }
}

// SYRK mirror of one warp's 32 x 32 block: lane l holds out[j] = value at
// (r0 + l, c0 + j); D(c0 + j, r0 + l) receives it. The block goes through
// this warp's shared-memory stage `tsm` (row j = mirror row c0 + j, lanes
// along it: conflict-free) and leaves as 16-byte stores, each warp store
// covering four whole 128-byte mirror rows, instead of 32 element stores.
// Needs ldd and the row starts 16-byte aligned (checked by the caller).
__device__ __forceinline__ void syrk_mirror_block(const GemmParams& p, long long dbase, int r0,
                                                  int c0, const float* out, void* tsm) {
  const int lane = threadIdx.x & 31;
  if (p.out_kind == kOutF32) {
    float* T = reinterpret_cast<float*>(tsm);
#pragma unroll
    for (int j = 0; j < 32; ++j) T[j * 32 + lane] = out[j];
    __syncwarp();
    float* D = reinterpret_cast<float*>(p.D) + dbase + r0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int row = 4 * k + (lane >> 3), q4 = (lane & 7) * 4;
      *reinterpret_cast<float4*>(D + static_cast<long long>(c0 + row) * p.ldd + q4) =
          *reinterpret_cast<const float4*>(&T[row * 32 + q4]);
    }
  } else {
    unsigned short* T = reinterpret_cast<unsigned short*>(tsm);
#pragma unroll
    for (int j = 0; j < 32; ++j)
      T[j * 32 + lane] = (p.out_kind == kOutBF16) ? __bfloat16_as_ushort(__float2bfloat16_rn(out[j]))
                                                  : __half_as_ushort(__float2half_rn(out[j]));
    __syncwarp();
    unsigned short* D = reinterpret_cast<unsigned short*>(p.D) + dbase + r0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int row = 8 * k + (lane >> 2), q8 = (lane & 3) * 8;
      *reinterpret_cast<uint4*>(D + static_cast<long long>(c0 + row) * p.ldd + q8) =
          *reinterpret_cast<const uint4*>(&T[row * 32 + q8]);
    }
  }
  __syncwarp();  // the stage is rewritten by the next chunk
}

// Epilogue for one 32-column chunk held by this thread: row r (global), columns
// c0 .. c0+31 (global), accumulator values v[0..31]. `tsm`: this warp's 4 KB
// shared-memory stage (SYRK mirror).
// GEMM epilogue of 32 consecutive columns c0 .. of row r: alpha * acc
// (+ beta * C), stored in the output type.
__device__ __forceinline__ void epilogue_row32(const GemmParams& p, int bz, int r, int c0,
                                               const float* v) {
  const long long dbase = static_cast<long long>(bz) * p.strideD;
  const long long cbase = static_cast<long long>(bz) * p.strideC;
  const bool has_c = (p.c_mode != kCNone) && (p.beta != 0.0f);
  if (r >= p.M) return;
  float out[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) out[j] = p.alpha * v[j];
  const bool full = (c0 + 32 <= p.N);
  if (has_c) {
    const long long crow = cbase + static_cast<long long>(r) * p.ldc;
    if (full && p.out_kind == kOutF32 && (p.ldc % 4 == 0) &&
        ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0) && ((cbase & 3) == 0)) {
      const float4* cp = reinterpret_cast<const float4*>(
          reinterpret_cast<const float*>(p.C) + crow + c0);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        float4 c4 = __ldg(cp + j);
        out[4 * j + 0] += p.beta * c4.x;
        out[4 * j + 1] += p.beta * c4.y;
        out[4 * j + 2] += p.beta * c4.z;
        out[4 * j + 3] += p.beta * c4.w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (c0 + j < p.N) out[j] += p.beta * load_c(p.C, p.out_kind, crow + c0 + j);
    }
  }
  store_row32(p, dbase + static_cast<long long>(r) * p.ldd, c0, out, full);
}

__device__ __forceinline__ void epilogue_chunk(const GemmParams& p, int bz, int r, int c0,
                                               const float* v, bool diag_tile, void* tsm) {
  const long long dbase = static_cast<long long>(bz) * p.strideD;
  const long long cbase = static_cast<long long>(bz) * p.strideC;
  const bool has_c = (p.c_mode != kCNone) && (p.beta != 0.0f);
  if (p.mode == kModeGemm) {
    epilogue_row32(p, bz, r, c0, v);
    return;
  }
  // SYRK: lower element (r, c) with r >= c, mirrored to (c, r).
  const int n = p.M;
  const int r0 = r - static_cast<int>(threadIdx.x & 31);  // this warp's first row
  // whole 32 x 32 block below the diagonal and inside the matrix (uniform
  // over the warp): the row part as the GEMM writes it, the mirror through
  // the transpose stage
  const int vec = (p.out_kind == kOutF32) ? 4 : 8;
  if (c0 + 31 <= r0 && r0 + 32 <= n && !has_c && p.ldd % vec == 0 &&
      ((reinterpret_cast<uintptr_t>(p.D) + static_cast<uintptr_t>(dbase) * (p.out_kind == kOutF32 ? 4 : 2)) & 15) == 0) {
    float out[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) out[j] = p.alpha * v[j];
    store_row32(p, dbase + static_cast<long long>(r) * p.ldd, c0, out, true);
    syrk_mirror_block(p, dbase, r0, c0, out, tsm);
    return;
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int c = c0 + j;
    const bool keep = (r < n) && (c < n) && (!diag_tile || c <= r);
    if (keep) {
      float val = p.alpha * v[j];
      if (has_c) {
        const long long ci = (p.c_mode == kCRow)
                                 ? cbase + static_cast<long long>(r) * p.ldc + c
                                 : cbase + static_cast<long long>(c) * p.ldc + r;
        val += p.beta * load_c(p.C, p.out_kind, ci);
      }
      store_d(p.D, p.out_kind, dbase + static_cast<long long>(r) * p.ldd + c, val);
      if (c != r) store_d(p.D, p.out_kind, dbase + static_cast<long long>(c) * p.ldd + r, val);
    }
  }
}

template <int KIND, int BN, int STAGES>
__global__ void __launch_bounds__(GemmCfg<KIND, BN>::THREADS, 1)
    gemm_sm100_kernel(const __grid_constant__ CUtensorMap map_a0,
                      const __grid_constant__ CUtensorMap map_a1,
                      const __grid_constant__ CUtensorMap map_b0,
                      const __grid_constant__ CUtensorMap map_b1, const GemmParams p) {
  using Cfg = GemmCfg<KIND, BN>;
  constexpr int BM = Cfg::BM;
  constexpr int BK = Cfg::BK;
  constexpr uint32_t STAGE_BYTES = Cfg::STAGE_BYTES;

  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  static_assert((3 * STAGES + 2 * Cfg::NBUF + 1) * 8 + 8 <= kGemmBarBytes, "barrier block");
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* accf_bar = empty_bar + STAGES;   // [NBUF]
  uint64_t* acce_bar = accf_bar + Cfg::NBUF;  // [NBUF]
  uint64_t* drain_bar = acce_bar + Cfg::NBUF; // [1]
  uint64_t* conv_bar = drain_bar + 1;         // [STAGES] kTF32x3F: lo parts written
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(conv_bar + STAGES);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const Abort ab{abort_flag, p.status, p.timeout_ns};

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
      mbar_init(&conv_bar[s], Cfg::CONV_WARPS);
    }
    for (int a = 0; a < Cfg::NBUF; ++a) {
      mbar_init(&accf_bar[a], 1);
      mbar_init(&acce_bar[a], 4);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&map_a0);
    tma_prefetch_desc(&map_b0);
    if (KIND == kTF32x3) {
      tma_prefetch_desc(&map_a1);
      tma_prefetch_desc(&map_b1);
    }
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_kb = (p.K + BK - 1) / BK;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    int stage = 0;
    uint32_t phase = 0;
    // armed-but-unobserved stages (for the drain on abort)
    bool aborted = false;
    int wave = 0;
    for (int t = blockIdx.x; t < p.num_tiles && !aborted; t += gridDim.x, ++wave) {
      if (p.wave_ctr && wave > 0)
        soft_wave_wait(p.wave_ctr, wave * static_cast<int>(gridDim.x), 100000ull);
      int bz, mb, nb;
      decode_tile(p, t, bz, mb, nb);
      if (p.ready && (!wait_ready(p.ready + mb / p.shard_tiles_m, p.ready_epoch, ab) ||
                      !wait_ready(p.ready + p.ready_b0 + bz, p.ready_epoch, ab))) {
        aborted = true;
        break;
      }
      const int m0 = mb * BM;
      const int n0 = nb * ((p.mode == kModeSyrk) ? BM : BN);
      const int za = p.a_batched ? bz : 0;
      const int zb = p.b_batched ? bz : 0;
      int kb_lo, kb_hi;
      tile_k_range(p, m0, BM, n0, BN, BK, num_kb, kb_lo, kb_hi);
      for (int kb = kb_lo; kb < kb_hi; ++kb) {
        if (!mbar_wait(&empty_bar[stage], phase ^ 1u, ab, kTimeoutEmpty)) {
          aborted = true;
          break;
        }
        uint8_t* sa = smem + stage * STAGE_BYTES;
        uint8_t* sb = sa + Cfg::NPARTS * Cfg::A_TILE;
        mbar_arrive_expect_tx(&full_bar[stage], Cfg::LOAD_BYTES);
        const int k0 = kb * BK;
        if (KIND == kTF32x3F) {
          // raw fp32 tiles into the hi slots (MN-major: boxes of 32 MN x 32 K)
          if (!p.a_mn) {
            tma_load_3d(sa, &map_a0, &full_bar[stage], k0, m0, za);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 32; ++j)
              tma_load_3d(sa + j * (32 * 128), &map_a0, &full_bar[stage], m0 + 32 * j, k0, za);
          }
          if (!p.b_mn) {
            tma_load_3d(sb, &map_b0, &full_bar[stage], k0, n0, zb);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 32; ++j)
              tma_load_3d(sb + j * (32 * 128), &map_b0, &full_bar[stage], n0 + 32 * j, k0, zb);
          }
        } else if (KIND == kF16) {
          if (!p.a_mn) {
            tma_load_3d(sa, &map_a0, &full_bar[stage], k0, m0, za);
          } else {
#pragma unroll
            for (int j = 0; j < BM / 64; ++j)
              tma_load_3d(sa + j * (64 * 128), &map_a0, &full_bar[stage], m0 + 64 * j, k0, za);
          }
          if (!p.b_mn) {
            tma_load_3d(sb, &map_b0, &full_bar[stage], k0, n0, zb);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j)
              tma_load_3d(sb + j * (64 * 128), &map_b0, &full_bar[stage], n0 + 64 * j, k0, zb);
          }
        } else {
          tma_load_3d(sa, &map_a0, &full_bar[stage], k0, m0, za);
          tma_load_3d(sa + Cfg::A_TILE, &map_a1, &full_bar[stage], k0, m0, za);
          tma_load_3d(sb, &map_b0, &full_bar[stage], k0, n0, zb);
          tma_load_3d(sb + Cfg::B_TILE, &map_b1, &full_bar[stage], k0, n0, zb);
        }
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (p.wave_ctr) atomicAdd(p.wave_ctr, 1);
    }
    if (aborted || ab.raised()) {
      // Let copies already issued land before the CTA exits: wait (bounded)
      // for the most recent STAGES armed phases.
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
        while (!mbar_try_wait(&full_bar[s], ph)) {
          if (globaltimer_ns() - t0 > 50000000ull) break;  // 50 ms
        }
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    gemm_mma_role<KIND, BN, STAGES>(p, smem, KIND == kTF32x3F ? conv_bar : full_bar, empty_bar,
                                    accf_bar, acce_bar, tmem_base, num_kb, ab);
    // Every MMA this thread issued must finish before TMEM is released.
    tc_commit(drain_bar);
    const unsigned long long t0 = globaltimer_ns();
    while (!mbar_try_wait(drain_bar, 0)) {
      if (globaltimer_ns() - t0 > 100000000ull) {  // 100 ms
        ab.raise(kTimeoutDrain);
        break;
      }
    }
  } else if (KIND == kTF32x3F && warp >= 6) {
    // ------------------------------------------------------------ converters
    // For every stage, in the producer's order: lo = x - trunc19(x) of the
    // raw A and B tiles, written beside them (same swizzled offsets; the
    // split is elementwise). inf / nan keep lo = 0.
    constexpr int CT = 32 * Cfg::CONV_WARPS;
    const int ct = threadIdx.x - 192;  // 0 .. CT - 1
    const long long total = cta_stage_total(p, BM, BN, BK, num_kb);
    int stage = 0;
    uint32_t phase = 0;
    for (long long g = 0; g < total; ++g) {
      if (!mbar_wait_warp(&full_bar[stage], phase, ab, kTimeoutAux)) break;
      uint8_t* st = smem + stage * STAGE_BYTES;
#pragma unroll
      for (int part = 0; part < 2; ++part) {
        const int bytes = part == 0 ? Cfg::A_TILE : Cfg::B_TILE;
        const float4* hi = reinterpret_cast<const float4*>(st + (part == 0 ? 0 : 2 * Cfg::A_TILE));
        float4* lo = reinterpret_cast<float4*>(st + (part == 0 ? Cfg::A_TILE : 2 * Cfg::A_TILE + Cfg::B_TILE));
#pragma unroll 4
        for (int i = ct; i < bytes / 16; i += CT) {
          const float4 x = hi[i];
          float4 l;
          l.x = tf32_lo(x.x);
          l.y = tf32_lo(x.y);
          l.z = tf32_lo(x.z);
          l.w = tf32_lo(x.w);
          lo[i] = l;
        }
      }
      fence_proxy_async_smem();  // the MMA (async proxy) reads what these stores wrote
      __syncwarp();
      if (lane == 0) mbar_arrive(&conv_bar[stage]);
      if (++stage == STAGES) {
        stage = 0;
        phase ^= 1u;
      }
    }
  } else if (warp >= 2 && warp < 6) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int row_in_tile = 32 * q + lane;
    void* tsm = smem + STAGES * STAGE_BYTES + kGemmBarBytes + (warp - 2) * (kEpiStageBytes / 4);
    const uint32_t lane_base = tmem_base + (static_cast<uint32_t>(32 * q) << 16);
    int gc = 0;
    bool aborted = false;
    for (int t = blockIdx.x; t < p.num_tiles && !aborted; t += gridDim.x) {
      int bz, mb, nb;
      decode_tile(p, t, bz, mb, nb);
      const int r = mb * BM + row_in_tile;
      const int ncol = (p.mode == kModeSyrk) ? BM : BN;
      const int n0 = nb * ncol;
      const int nlim = (p.mode == kModeSyrk) ? p.M : p.N;
      // a SYRK tile reaching the diagonal takes the masked path per block
      const bool diag = (p.mode == kModeSyrk && mb == nb) ||
                        (p.mode == kModeSyrkWide && n0 + BN - 1 > mb * BM);
      if (KIND == kF16) {
        // whole K in one TMEM accumulator
        const int buf = gc % Cfg::NBUF;
        const uint32_t bph = (gc / Cfg::NBUF) & 1;
        ++gc;
        if (!mbar_wait_warp(&accf_bar[buf], bph, ab, kTimeoutAccFull)) break;
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < ncol / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(lane_base + buf * BN + c * 32, v);
          tmem_ld_wait();
          if (n0 + c * 32 < nlim) {
            float f[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) f[j] = u2f(v[j]);
            epilogue_chunk(p, bz, r, n0 + c * 32, f, diag, tsm);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acce_bar[buf]);
      } else {
        // K chunks: partial sums added here with round-to-nearest
        float sum[BN];
#pragma unroll
        for (int j = 0; j < BN; ++j) sum[j] = 0.0f;
        int kb_lo, kb_hi;
        tile_k_range(p, mb * BM, BM, n0, BN, BK, num_kb, kb_lo, kb_hi);
        for (int kb0 = kb_lo; kb0 < kb_hi; kb0 += Cfg::CHUNK_KB, ++gc) {
          const int buf = gc % Cfg::NBUF;
          const uint32_t bph = (gc / Cfg::NBUF) & 1;
          if (!mbar_wait_warp(&accf_bar[buf], bph, ab, kTimeoutAccFull)) {
            aborted = true;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < BN / 32; ++c) {
            uint32_t v[32];
            tmem_ld32(lane_base + buf * BN + c * 32, v);
            tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 32; ++j) sum[c * 32 + j] += u2f(v[j]);
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&acce_bar[buf]);
        }
        if (aborted) break;
#pragma unroll
        for (int c = 0; c < BN / 32; ++c)
          if (n0 + c * 32 < nlim) epilogue_chunk(p, bz, r, n0 + c * 32, sum + c * 32, diag, tsm);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();  // lane 0 arrives from the MMA role, 1..31 straight here
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace tb
