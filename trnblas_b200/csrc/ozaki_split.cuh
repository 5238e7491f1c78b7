// Ozaki split on the GPU: per-row power-of-two scaling and balanced 7-bit
// integer digits, bit for bit the digits of the reference's host split
// (trnblas/ozaki.py:123-219, `split` with per="row"; a per-column split of B
// is the per-row split of op(B)^T).
//
// For a logical R x K operand X (element (r, k) at X[r * rs + k * ks]):
//   e_r   = frexp exponent of max_k |X[r, k]| (0 for an all-zero row);
//   shift = 6 - e_r; if any row's shift leaves [-1022, 1023], every row is
//           scaled by two factors 2^floor(shift/2) * 2^(shift - floor(shift/2))
//           (the reference makes this choice once per operand);
//   R     = X * scale (exact);  digit_0 = rint(R);  R -= digit_0;
//   digit_s = rint(128 R); R = 128 R - digit_s ...  (fp64, round half even)
// Digits (|d| <= 64) are written as int8 planes (slices, R, ldd), K-major,
// zero beyond K; exponents as int32. Float inputs are widened exactly.
#pragma once

#include <algorithm>

#include "common.cuh"
#include "runtime.hpp"

namespace tb {

struct SplitScratch {
  unsigned long long* maxbits;  // R words: max |x| as IEEE bits (monotone for x >= 0)
  int* shift_range;             // [0] = max shift, [1] = min shift (for the 2-factor rule)
};

// |x| widened to double, as IEEE bits: unsigned order = magnitude order.
template <typename T>
__device__ __forceinline__ unsigned long long abs_bits(T x) {
  return static_cast<unsigned long long>(__double_as_longlong(fabs(static_cast<double>(x))));
}

__device__ __forceinline__ unsigned long long umax64(unsigned long long a, unsigned long long b) {
  return a > b ? a : b;
}

__device__ __forceinline__ unsigned long long vec_abs_bits(double2 v) {
  return umax64(abs_bits(v.x), abs_bits(v.y));
}

__device__ __forceinline__ unsigned long long vec_abs_bits(float4 v) {
  return umax64(umax64(abs_bits(v.x), abs_bits(v.y)), umax64(abs_bits(v.z), abs_bits(v.w)));
}

// Pass 1 for K-contiguous rows (ks == 1): one warp per row. The row's
// 16-byte-aligned body is read with 16-byte loads, four in flight per lane;
// the unaligned head and the tail element by element.
template <typename T>
__global__ void __launch_bounds__(256)
    ozk_rowmax_rows_kernel(const T* __restrict__ X, long long rs, int R, int K,
                           unsigned long long* __restrict__ maxbits) {
  using Vec = typename std::conditional<sizeof(T) == 8, double2, float4>::type;
  constexpr int V = 16 / static_cast<int>(sizeof(T));
  const long long r = static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= R) return;
  const T* row = X + r * rs;
  const int mis = static_cast<int>((reinterpret_cast<uintptr_t>(row) & 15) / sizeof(T));
  int head = mis ? V - mis : 0;
  if (head > K) head = K;
  unsigned long long b = 0;
  if (lane < head) b = abs_bits(__ldg(row + lane));
  const int nv = (K - head) / V;
  const Vec* body = reinterpret_cast<const Vec*>(row + head);
  int i = lane;
  for (; i + 96 < nv; i += 128) {
    const Vec a0 = __ldg(body + i), a1 = __ldg(body + i + 32);
    const Vec a2 = __ldg(body + i + 64), a3 = __ldg(body + i + 96);
    b = umax64(b, umax64(umax64(vec_abs_bits(a0), vec_abs_bits(a1)),
                         umax64(vec_abs_bits(a2), vec_abs_bits(a3))));
  }
  for (; i < nv; i += 32) b = umax64(b, vec_abs_bits(__ldg(body + i)));
  for (int k = head + nv * V + lane; k < K; k += 32) b = umax64(b, abs_bits(__ldg(row + k)));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) b = umax64(b, __shfl_xor_sync(0xffffffffu, b, o));
  if (lane == 0) maxbits[r] = b;
}

// Pass 1 for row-contiguous operands (rs == 1, e.g. op(B)^T of a row-major
// B): one thread per row over a chunk of `kchunk` K values, eight loads in
// flight; chunks meet in an atomic max (maxbits zeroed beforehand).
template <typename T>
__global__ void __launch_bounds__(256)
    ozk_rowmax_cols_kernel(const T* __restrict__ X, long long ks, int R, int K, int kchunk,
                           unsigned long long* __restrict__ maxbits) {
  const long long r = static_cast<long long>(blockIdx.x) * 256 + threadIdx.x;
  if (r >= R) return;
  const int k0 = blockIdx.y * kchunk;
  const int k1 = min(K, k0 + kchunk);
  const T* p = X + r;
  unsigned long long b = 0;
  int k = k0;
  for (; k + 8 <= k1; k += 8) {
    T v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = __ldg(p + static_cast<long long>(k + u) * ks);
#pragma unroll
    for (int u = 0; u < 8; ++u) b = umax64(b, abs_bits(v[u]));
  }
  for (; k < k1; ++k) b = umax64(b, abs_bits(__ldg(p + static_cast<long long>(k) * ks)));
  if (b) atomicMax(maxbits + r, b);
}

// Pass 1, any strides: per-row max |x| (32 x 32 tiles, coalesced for either layout).
template <typename T>
__global__ void ozk_rowmax_kernel(const T* __restrict__ X, long long rs, long long ks, int R,
                                  int K, unsigned long long* __restrict__ maxbits) {
  __shared__ double tile[32][33];
  const int k0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  if (ks == 1) {
    for (int i = ty; i < 32; i += 8) {
      const int r = r0 + i, k = k0 + tx;
      tile[i][tx] = (r < R && k < K) ? fabs(static_cast<double>(__ldg(X + r * rs + k))) : 0.0;
    }
  } else {
    for (int i = ty; i < 32; i += 8) {
      const int k = k0 + i, r = r0 + tx;
      tile[tx][i] =
          (r < R && k < K) ? fabs(static_cast<double>(__ldg(X + r * rs + k * ks))) : 0.0;
    }
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    unsigned long long b = static_cast<unsigned long long>(__double_as_longlong(tile[i][tx]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long ob = __shfl_xor_sync(0xffffffffu, b, o);
      b = ob > b ? ob : b;
    }
    if (tx == 0 && r0 + i < R && b != 0) atomicMax(maxbits + r0 + i, b);
  }
}

// The digits of one scaled value u (|u| < 64, finite): digit s is the
// remainder left by digits 0..s-1, rounded half-to-even to a multiple of
// 2^(-7s), times 2^(7s). The rounding is the classic add-and-subtract of the
// constant 1.5 * 2^(52 - 7s), whose unit in the last place is 2^(-7s): the
// round-to-nearest-even addition rounds u onto that grid, the low 32 bits of
// the sum are the digit in two's complement, and (sum - constant) is the
// rounded value exactly (same binade). Scaling by 128 commutes with the
// rounding and every remainder is exact, so this yields the digits of
// d = rint(v), v = 128 (v - d), ... bit for bit, with three additions a
// digit and no conversion instructions. `put(s, digit)` receives each digit.
template <typename F>
__device__ __forceinline__ void oz_digit_loop(double u, int slices, F&& put) {
#pragma unroll
  for (int s = 0; s < 12; ++s) {
    if (s >= slices) break;
    const double m =
        __longlong_as_double((static_cast<long long>(1075 - 7 * s) << 52) | (1ll << 51));
    const double t = __dadd_rn(u, m);
    put(s, static_cast<int8_t>(__double2loint(t)));
    u = __dsub_rn(u, __dsub_rn(t, m));
  }
}

// frexp exponent of a non-negative finite double given by its bits.
__device__ __forceinline__ int frexp_exp_bits(unsigned long long b) {
  if (b == 0) return 0;
  const int E = static_cast<int>(b >> 52);
  if (E > 0) return E - 1022;
  // subnormal: value = m * 2^-1074 with m = b < 2^52
  return (64 - __clzll(static_cast<long long>(b))) - 1074;
}

static __global__ void ozk_init_kernel(unsigned long long* maxbits, int R, int* shift_range) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < R) maxbits[i] = 0ull;
  if (i == 0) {
    shift_range[0] = -2147483647;
    shift_range[1] = 2147483647;
  }
}

// Pass 2: exponents and the operand-wide shift range.
static __global__ void ozk_exps_kernel(const unsigned long long* __restrict__ maxbits, int R,
                                       int* __restrict__ exps, int* __restrict__ shift_range) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= R) return;
  const int e = frexp_exp_bits(maxbits[r]);
  exps[r] = e;
  const int shift = 6 - e;
  atomicMax(shift_range + 0, shift);
  atomicMin(shift_range + 1, shift);
}

// Pass 3: digits. 32 x 32 tiles through shared memory; each thread produces
// all `slices` digits of one element.
template <typename T>
__global__ void ozk_digits_kernel(const T* __restrict__ X, long long rs, long long ks, int R,
                                  int K, int ldd, long long plane, int slices,
                                  const int* __restrict__ exps,
                                  const int* __restrict__ shift_range,
                                  int8_t* __restrict__ digits) {
  __shared__ double tile[32][33];
  const int k0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;
  if (ks == 1) {
    for (int i = ty; i < 32; i += 8) {
      const int r = r0 + i, k = k0 + tx;
      tile[i][tx] = (r < R && k < K) ? static_cast<double>(__ldg(X + r * rs + k)) : 0.0;
    }
  } else {
    for (int i = ty; i < 32; i += 8) {
      const int k = k0 + i, r = r0 + tx;
      tile[tx][i] = (r < R && k < K) ? static_cast<double>(__ldg(X + r * rs + k * ks)) : 0.0;
    }
  }
  __syncthreads();
  const bool two = shift_range[0] > 1023 || shift_range[1] < -1022;
  for (int i = ty; i < 32; i += 8) {
    const int r = r0 + i, k = k0 + tx;
    if (r >= R || k >= ldd) continue;
    const long long o = static_cast<long long>(r) * ldd + k;
    if (k >= K) {
      for (int s = 0; s < slices; ++s) digits[s * plane + o] = 0;
      continue;
    }
    const int shift = 6 - exps[r];
    double v = tile[i][tx];
    if (!two) {
      v = v * pow2d(shift);
    } else {
      const int h = (shift >= 0) ? shift / 2 : -((-shift + 1) / 2);
      v = v * pow2d(h);
      v = v * pow2d(shift - h);
    }
    oz_digit_loop(v, slices, [&](int s, int8_t d) { digits[s * plane + o] = d; });
  }
}

// Blocked digit layout: the image the int8 MMA reads from shared memory, laid
// out so that all planes of one row block of one 32-wide K slab form a single
// contiguous chunk, fetched with ONE bulk copy per operand and pipeline stage
// (a bulk copy costs a fixed ~80 cycles of the SM's copy engine on top of its
// bytes, so a stage staged as one copy per plane is copy-bound):
//   [K slab (32)][row block (RB rows)][plane][8-row group][K half (16)]
//   [row in group (8)][16 bytes]
// Inside a chunk each plane is RB x 32 bytes of no-swizzle K-major core
// matrices (8 rows x 16 bytes): LBO = 128 bytes between the K halves, SBO =
// 256 bytes between row groups, planes RB * 32 bytes apart. RB = 2^rb_log2
// (32, 64 or 128) is the MMA tile's row count for that operand.
__host__ __device__ __forceinline__ long long blocked_offset(long long p, int k, int s, int slices,
                                                             long long rows_pad, int rb_log2) {
  const long long slab = k >> 5;
  const int kk = k & 31;
  const long long nblk = rows_pad >> rb_log2;
  const long long blk = p >> rb_log2;
  const long long grp = (p & ((1ll << rb_log2) - 1)) >> 3;
  return (((((((slab * nblk + blk) * slices + s) << (rb_log2 - 3)) + grp) * 2 + (kk >> 4))) << 7) +
         ((p & 7) << 4) + (kk & 15);
}

// Start of the chunk of row block `blk` (all `slices` planes) of K slab `slab`.
__host__ __device__ __forceinline__ long long blocked_chunk(long long slab, long long blk,
                                                            int slices, long long rows_pad,
                                                            int rb_log2) {
  return ((slab * (rows_pad >> rb_log2) + blk) * slices) << (rb_log2 + 5);
}

// Digits in the blocked layout (row blocks of 2^rb_log2 rows), optionally a
// second copy with another row block (digits2, rb_log2_2; NULL for none).
// Padded row p maps to logical row (p / gp) * g + p % gp when p % gp < g (else
// the row is zero padding): the pair energy pads each occupied orbital's nvir
// rows to a multiple of 128, the GEMM pads the end. Work unit: a tile of 32
// padded rows x one 32-wide K slab. The grid is persistent (grid-strided over
// the tiles); each block keeps kOzBuf - 1 input tiles in flight with
// element-wise cp.async into a shared-memory ring (zero-fill for padding rows
// and K >= K_logical), so the loads of later tiles overlap the work on the
// current one. Each thread then takes 4 consecutive K of one row, packs their
// 4 digits of each plane into one 32-bit word and stores it straight into the
// blocked layout (planes RB * 32 bytes apart; a warp's store covers two
// contiguous 64-byte runs).
constexpr int kOzBuf = 4;

template <int BYTES>
__device__ __forceinline__ void cp_async_zfill(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], %2, %3;\n" ::"r"(smem_u32(dst)), "l"(src),
               "n"(BYTES), "r"(valid ? BYTES : 0)
               : "memory");
}

__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

template <typename T>
__global__ void __launch_bounds__(256)
    ozk_digits_tiled_kernel(const T* __restrict__ X, long long rs, long long ks, int K,
                            long long g, long long gp, long long rows_pad, int kpad, int slices,
                            const int* __restrict__ exps, const int* __restrict__ shift_range,
                            int8_t* __restrict__ digits, int rb_log2,
                            int8_t* __restrict__ digits2, int rb_log2_2) {
  __shared__ __align__(16) T tile[kOzBuf][32][33];
  const int tx = threadIdx.x, ty = threadIdx.y, t = ty * 32 + tx;
  const int nslab = kpad / 32;
  const long long nrb = rows_pad / 32;
  const bool two = shift_range[0] > 1023 || shift_range[1] < -1022;
  // Tile cursors (row block, K slab) advance by the grid size without a
  // division per tile.
  const long long G = gridDim.x;
  const long long Gq = G / nslab;
  const int Gr = static_cast<int>(G - Gq * nslab);
  struct Cur {
    long long rb;
    int slab;
  };
  auto advance = [&](Cur& c) {
    c.rb += Gq;
    c.slab += Gr;
    if (c.slab >= nslab) {
      c.slab -= nslab;
      ++c.rb;
    }
  };
  // Source row of padded row p0 + i (p0 = 32 * rb; rows_pad < 2^31): one
  // 32-bit division for p0, then a short carry loop (1 <= g <= gp).
  const unsigned ug = static_cast<unsigned>(g), ugp = static_cast<unsigned>(gp);
  auto src_row = [&](unsigned q0, unsigned a0, int i) -> long long {
    unsigned a = a0 + static_cast<unsigned>(i), q = q0;
    while (a >= ugp) {
      a -= ugp;
      ++q;
    }
    return a < ug ? static_cast<long long>(q) * g + a : -1;
  };
  // Start the copies of tile c into ring slot `buf` (one commit group per
  // call, empty past the last tile, so group counting stays uniform).
  auto issue = [&](const Cur& c, int buf) {
    if (c.rb < nrb) {
      const unsigned p0 = static_cast<unsigned>(c.rb * 32);
      const unsigned q0 = p0 / ugp, a0 = p0 - q0 * ugp;
      const int k0 = c.slab * 32;
      if (ks == 1) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int i = ty + 8 * j;
          const long long r = src_row(q0, a0, i);
          const int k = k0 + tx;
          const bool ok = r >= 0 && k < K;
          cp_async_zfill<sizeof(T)>(&tile[buf][i][tx], ok ? X + r * rs + k : X, ok);
        }
      } else {
        const long long r = src_row(q0, a0, tx);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int kk = ty + 8 * j;
          const int k = k0 + kk;
          const bool ok = r >= 0 && k < K;
          cp_async_zfill<sizeof(T)>(&tile[buf][tx][kk],
                                    ok ? X + r * rs + static_cast<long long>(k) * ks : X, ok);
        }
      }
    }
    cp_async_commit();
  };
  // compute role of this thread: row `crow`, K offsets kq .. kq + 3 of the slab
  const int crow = t >> 3, kq = (t & 7) * 4;
  const long long pstride = 32ll << rb_log2, pstride2 = 32ll << rb_log2_2;
  Cur cc{static_cast<long long>(blockIdx.x) / nslab, static_cast<int>(blockIdx.x % nslab)};
  Cur cl = cc;
#pragma unroll
  for (int b = 0; b < kOzBuf - 1; ++b) {
    issue(cl, b);
    advance(cl);
  }
  for (int it = 0; cc.rb < nrb; advance(cc), ++it) {
    cp_async_wait<kOzBuf - 2>();  // this thread's copies of tile `it` have landed
    __syncthreads();              // ... everyone's; and slot (it - 1) % kOzBuf is free
    issue(cl, (it + kOzBuf - 1) % kOzBuf);
    advance(cl);
    const int buf = it % kOzBuf;
    const unsigned p0 = static_cast<unsigned>(cc.rb * 32);
    const unsigned q0 = p0 / ugp, a0 = p0 - q0 * ugp;
    const int k0 = cc.slab * 32;
    const long long r = src_row(q0, a0, crow);
    const int shift = r >= 0 ? 6 - __ldg(exps + r) : 0;
    const int h1 = two ? ((shift >= 0) ? shift / 2 : -((-shift + 1) / 2)) : shift;
    const double f1 = pow2d(h1), f2 = pow2d(shift - h1);
    double u[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) u[e] = (static_cast<double>(tile[buf][crow][kq + e]) * f1) * f2;
    int8_t* out = digits + blocked_offset(p0 + crow, k0 + kq, 0, slices, rows_pad, rb_log2);
    int8_t* out2 = digits2 ? digits2 + blocked_offset(p0 + crow, k0 + kq, 0, slices, rows_pad,
                                                      rb_log2_2)
                           : nullptr;
    // digits of the 4 values, slice by slice (the rounding of oz_digit_loop)
#pragma unroll
    for (int sl = 0; sl < 12; ++sl) {
      if (sl >= slices) break;
      const double m =
          __longlong_as_double((static_cast<long long>(1075 - 7 * sl) << 52) | (1ll << 51));
      int d[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const double s1 = __dadd_rn(u[e], m);
        d[e] = __double2loint(s1);
        u[e] = __dsub_rn(u[e], __dsub_rn(s1, m));
      }
      const uint32_t w = __byte_perm(__byte_perm(d[0], d[1], 0x0040),
                                     __byte_perm(d[2], d[3], 0x0040), 0x5410);
      *reinterpret_cast<uint32_t*>(out + sl * pstride) = w;
      if (out2) *reinterpret_cast<uint32_t*>(out2 + sl * pstride2) = w;
    }
  }
  cp_async_wait<0>();
}

// Resident blocks per SM of the digit kernel (its persistent grid size per
// SM), from the occupancy calculator; cached per element type.
template <typename T>
inline int oz_digit_blocks_per_sm() {
  static int cached = 0;
  if (cached == 0) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, ozk_digits_tiled_kernel<T>, 256, 0) !=
            cudaSuccess ||
        n < 1)
      n = 1;
    cached = n;
  }
  return cached;
}

// Row max |x| of X (R x K, strides rs, ks) into maxbits (zeroed first).
template <typename T>
inline void launch_rowmax(const T* X, long long rs, long long ks, int R, int K,
                          unsigned long long* maxbits, cudaStream_t stream) {
  if (K <= 0 || R <= 0) return;
  if (ks == 1) {
    ozk_rowmax_rows_kernel<T><<<static_cast<unsigned>((R + 7) / 8), 256, 0, stream>>>(
        X, rs, R, K, maxbits);
  } else if (rs == 1 && (K + 63) / 64 <= 65535) {
    dim3 g(static_cast<unsigned>((R + 255) / 256), static_cast<unsigned>((K + 63) / 64));
    ozk_rowmax_cols_kernel<T><<<g, 256, 0, stream>>>(X, ks, R, K, 64, maxbits);
  } else {
    dim3 g1(static_cast<unsigned>((K + 31) / 32), static_cast<unsigned>((R + 31) / 32));
    ozk_rowmax_kernel<T><<<g1, dim3(32, 8), 0, stream>>>(X, rs, ks, R, K, maxbits);
  }
}

// Split into the blocked layout: R logical rows (row r at X[r * rs + k * ks]),
// rows_pad padded rows grouped as described above (a multiple of every row
// block), K padded to kpad (multiple of 32); digits2 (may be NULL) receives a
// second copy with row blocks of 2^rb_log2_2. scratch as for launch_split.
template <typename T>
inline cudaError_t launch_split_tiled(const T* X, long long rs, long long ks, int R, int K,
                                      long long g, long long gp, long long rows_pad, int kpad,
                                      int slices, int8_t* digits, int rb_log2, int8_t* digits2,
                                      int rb_log2_2, int* exps, SplitScratch scratch,
                                      cudaStream_t stream) {
  auto bad_rb = [&](int lg) { return lg < 5 || lg > 7 || (rows_pad & ((1ll << lg) - 1)); };
  if ((R + 31) / 32 > 65535 || rows_pad / 32 > 65535 || (rows_pad & 31) || (kpad & 31) ||
      g < 1 || gp < g ||
      slices > 12 || bad_rb(rb_log2) || (digits2 && bad_rb(rb_log2_2)))
    return cudaErrorInvalidConfiguration;
  ozk_init_kernel<<<(R + 255) / 256 + 1, 256, 0, stream>>>(scratch.maxbits, R,
                                                          scratch.shift_range);
  dim3 blk(32, 8);
  launch_rowmax(X, rs, ks, R, K, scratch.maxbits, stream);
  ozk_exps_kernel<<<(R + 255) / 256, 256, 0, stream>>>(scratch.maxbits, R, exps,
                                                       scratch.shift_range);
  const long long tiles = (rows_pad / 32) * (kpad / 32);
  const long long g3 = std::min<long long>(tiles, static_cast<long long>(num_sms()) *
                                                      oz_digit_blocks_per_sm<T>());
  if (g3 > 0)
    ozk_digits_tiled_kernel<T><<<static_cast<unsigned>(g3), blk, 0, stream>>>(X, rs, ks, K, g, gp, rows_pad, kpad, slices,
                                                     exps, scratch.shift_range, digits, rb_log2,
                                                     digits2, rb_log2_2);
  return cudaGetLastError();
}

// Run the passes on `stream`. scratch.maxbits (R words) and
// scratch.shift_range (2 ints) are initialised here.
template <typename T>
inline cudaError_t launch_split(const T* X, long long rs, long long ks, int R, int K, int ldd,
                                int slices, int8_t* digits, int* exps, SplitScratch scratch,
                                cudaStream_t stream) {
  if ((R + 31) / 32 > 65535 || (ldd + 31) / 32 > 2147483647 / 2) return cudaErrorInvalidConfiguration;
  ozk_init_kernel<<<(R + 255) / 256 + 1, 256, 0, stream>>>(scratch.maxbits, R,
                                                          scratch.shift_range);
  dim3 blk(32, 8);
  launch_rowmax(X, rs, ks, R, K, scratch.maxbits, stream);
  ozk_exps_kernel<<<(R + 255) / 256, 256, 0, stream>>>(scratch.maxbits, R, exps,
                                                       scratch.shift_range);
  dim3 g3(static_cast<unsigned>((ldd + 31) / 32), static_cast<unsigned>((R + 31) / 32));
  ozk_digits_kernel<T><<<g3, blk, 0, stream>>>(X, rs, ks, R, K, ldd,
                                               static_cast<long long>(R) * ldd, slices, exps,
                                               scratch.shift_range, digits);
  return cudaGetLastError();
}

}  // namespace tb
