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

#include "common.cuh"

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
// rows to a multiple of 128, the GEMM pads the end. A block covers 32 padded
// rows and kOzSlabs K slabs of 32: every input value of the block is loaded
// into registers first (sixteen loads in flight a thread), then each slab's
// digits are staged in shared memory and written 16 bytes at a time.
constexpr int kOzSlabs = 4;

template <typename T>
__global__ void __launch_bounds__(256, 3)
    ozk_digits_tiled_kernel(const T* __restrict__ X, long long rs, long long ks, int K,
                            long long g, long long gp, long long rows_pad, int kpad, int slices,
                            const int* __restrict__ exps, const int* __restrict__ shift_range,
                            int8_t* __restrict__ digits, int rb_log2,
                            int8_t* __restrict__ digits2, int rb_log2_2) {
  __shared__ double tile[32][33];
  __shared__ __align__(16) int8_t dg[12][32][32];
  const int kb = blockIdx.x * (32 * kOzSlabs);
  const long long p0 = static_cast<long long>(blockIdx.y) * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;
  auto src_row = [&](long long p) -> long long {
    const long long q = p / gp, a = p - q * gp;
    return (a < g) ? q * g + a : -1;
  };
  // scale exponents of this thread's compute rows ty + 8 j: one power-of-two
  // step (h1 = shift, h2 = 0), or two when the operand needs them
  const bool two = shift_range[0] > 1023 || shift_range[1] < -1022;
  int h1[4], h2[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const long long r = src_row(p0 + ty + 8 * j);
    const int shift = r >= 0 ? 6 - exps[r] : 0;
    h1[j] = two ? ((shift >= 0) ? shift / 2 : -((-shift + 1) / 2)) : shift;
    h2[j] = shift - h1[j];
  }
  T vals[kOzSlabs][4];
  if (ks == 1) {
    // thread (tx, ty) loads and converts (row ty + 8 j, k tx) of each slab
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const long long r = src_row(p0 + ty + 8 * j);
      const T* xr = X + (r >= 0 ? r : 0) * rs;
#pragma unroll
      for (int s = 0; s < kOzSlabs; ++s) {
        const int k = kb + 32 * s + tx;
        vals[s][j] = (r >= 0 && k < K) ? __ldg(xr + k) : T(0);
      }
    }
  } else {
    // thread (tx, ty) loads (row tx, k ty + 8 j): consecutive rows per warp
    const long long r = src_row(p0 + tx);
    const T* xr = X + (r >= 0 ? r : 0) * rs;
#pragma unroll
    for (int s = 0; s < kOzSlabs; ++s)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int k = kb + 32 * s + ty + 8 * j;
        vals[s][j] = (r >= 0 && k < K) ? __ldg(xr + static_cast<long long>(k) * ks) : T(0);
      }
  }
  const int t = ty * 32 + tx;
#pragma unroll
  for (int s = 0; s < kOzSlabs; ++s) {
    const int k0 = kb + 32 * s;
    if (k0 >= kpad) break;  // uniform over the block
    double v[4];
    if (ks == 1) {
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = static_cast<double>(vals[s][j]);
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) tile[tx][ty + 8 * j] = static_cast<double>(vals[s][j]);
      __syncthreads();
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = tile[ty + 8 * j][tx];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int i = ty + 8 * j;
      oz_digit_loop((v[j] * pow2d(h1[j])) * pow2d(h2[j]), slices,
                    [&](int sl, int8_t d) { dg[sl][i][tx] = d; });
    }
    __syncthreads();
    // 16-byte stores: (plane, row, K half) items
    for (int it = t; it < slices * 64; it += 256) {
      const int sl = it >> 6, row = (it >> 1) & 31, half = it & 1;
      const uint4 w = *reinterpret_cast<const uint4*>(&dg[sl][row][16 * half]);
      *reinterpret_cast<uint4*>(digits + blocked_offset(p0 + row, k0 + 16 * half, sl, slices,
                                                        rows_pad, rb_log2)) = w;
      if (digits2)
        *reinterpret_cast<uint4*>(digits2 + blocked_offset(p0 + row, k0 + 16 * half, sl, slices,
                                                           rows_pad, rb_log2_2)) = w;
    }
    __syncthreads();  // dg and tile are rewritten by the next slab
  }
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
      slices > 12 || bad_rb(rb_log2) || (digits2 && bad_rb(rb_log2_2)))
    return cudaErrorInvalidConfiguration;
  ozk_init_kernel<<<(R + 255) / 256 + 1, 256, 0, stream>>>(scratch.maxbits, R,
                                                          scratch.shift_range);
  dim3 blk(32, 8);
  launch_rowmax(X, rs, ks, R, K, scratch.maxbits, stream);
  ozk_exps_kernel<<<(R + 255) / 256, 256, 0, stream>>>(scratch.maxbits, R, exps,
                                                       scratch.shift_range);
  dim3 g3(static_cast<unsigned>((kpad + 32 * kOzSlabs - 1) / (32 * kOzSlabs)),
          static_cast<unsigned>(rows_pad / 32));
  ozk_digits_tiled_kernel<T><<<g3, blk, 0, stream>>>(X, rs, ks, K, g, gp, rows_pad, kpad, slices,
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
