// C-ABI entry points for GEMM, batched GEMM and SYRK, plus the fp32 (3xTF32)
// operand split kernel and the K == 0 scale kernel.
#include <algorithm>
#include <string>

#include <cstdlib>

#include "gemm_sm100.cuh"
#include "gemm_sm100_pair.cuh"
#include "runtime.hpp"

namespace tb {

// ---------------------------------------------------------------------------
// 3xTF32 split: hi = tf32 round-to-nearest-even of x (low 13 mantissa bits
// zero), lo = x - hi (exact in fp32). Reads the logical R x K operand with
// arbitrary strides (rs, ks) and writes K-major hi / lo planes (R x ldo),
// zero in the K padding. 32 x 32 tiles through shared memory so both the
// strided read and the K-contiguous write are coalesced.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float tf32_rne(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7F800000u) == 0x7F800000u) return x;  // inf / nan unchanged
  const uint32_t lsb = (u >> 13) & 1u;
  u = (u + 0xFFFu + lsb) & 0xFFFFE000u;
  return __uint_as_float(u);
}

__global__ void split_tf32_kernel(const float* __restrict__ X, long long rs, long long ks,
                                  long long bs, int R, int K, int ldo, long long obs,
                                  float* __restrict__ hi, float* __restrict__ lo) {
  __shared__ float tile[32][33];
  const int k0 = blockIdx.x * 32;
  const int r0 = blockIdx.y * 32;
  const long long b = blockIdx.z;
  const float* Xb = X + b * bs;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  if (ks == 1) {
    for (int i = ty; i < 32; i += 8) {
      const int r = r0 + i, k = k0 + tx;
      tile[i][tx] = (r < R && k < K) ? __ldg(Xb + r * rs + k) : 0.0f;
    }
  } else {
    for (int i = ty; i < 32; i += 8) {
      const int k = k0 + i, r = r0 + tx;
      tile[tx][i] = (r < R && k < K) ? __ldg(Xb + r * rs + k * ks) : 0.0f;
    }
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int r = r0 + i, k = k0 + tx;
    if (r < R && k < ldo) {
      const float x = tile[i][tx];
      const float h = tf32_rne(x);
      const long long o = b * obs + static_cast<long long>(r) * ldo + k;
      hi[o] = h;
      lo[o] = ((__float_as_uint(x) & 0x7F800000u) == 0x7F800000u) ? 0.0f : x - h;
    }
  }
}

// The same split for a row-major source (K contiguous, ks == 1), where no
// transpose is needed: one thread per 4 consecutive k of a row, float4 loads
// (`vec`: row and batch strides multiples of 4, 16-byte aligned base; else
// guarded scalar loads) and float4 stores of hi / lo.
__device__ __forceinline__ void split1(float x, float& h, float& l) {
  h = tf32_rne(x);
  l = ((__float_as_uint(x) & 0x7F800000u) == 0x7F800000u) ? 0.0f : x - h;
}

__global__ void split_tf32_rows_kernel(const float* __restrict__ X, long long rs, long long bs,
                                       int R, int K, int kp, long long obs, int vec,
                                       float* __restrict__ hi, float* __restrict__ lo) {
  const int kq = kp >> 2;
  const long long b = blockIdx.z;
  for (int r = blockIdx.y * blockDim.y + threadIdx.y; r < R; r += gridDim.y * blockDim.y) {
    const float* row = X + b * bs + static_cast<long long>(r) * rs;
    const long long o0 = b * obs + static_cast<long long>(r) * kp;
    for (int q = blockIdx.x * blockDim.x + threadIdx.x; q < kq; q += gridDim.x * blockDim.x) {
      const int k = q << 2;
      float4 x;
      if (vec && k + 3 < K) {
        x = __ldg(reinterpret_cast<const float4*>(row + k));
      } else {
        x.x = k < K ? __ldg(row + k) : 0.0f;
        x.y = k + 1 < K ? __ldg(row + k + 1) : 0.0f;
        x.z = k + 2 < K ? __ldg(row + k + 2) : 0.0f;
        x.w = k + 3 < K ? __ldg(row + k + 3) : 0.0f;
      }
      float4 h, l;
      split1(x.x, h.x, l.x);
      split1(x.y, h.y, l.y);
      split1(x.z, h.z, l.z);
      split1(x.w, h.w, l.w);
      *reinterpret_cast<float4*>(hi + o0 + k) = h;
      *reinterpret_cast<float4*>(lo + o0 + k) = l;
    }
  }
}

// The transposing split for a source whose rows are contiguous across r
// (rs == 1, e.g. a row-major K x N B operand read as op(B)^T): 64 (k) x 64 (r)
// tiles through shared memory, float4 loads along r and float4 stores of
// hi / lo along k. Needs ks % 4 == 0, bs % 4 == 0 and a 16-byte aligned base;
// edges are guarded element by element.
__global__ void split_tf32_t64_kernel(const float* __restrict__ X, long long ks, long long bs,
                                      int R, int K, int kp, long long obs,
                                      float* __restrict__ hi, float* __restrict__ lo) {
  __shared__ float tile[64][65];  // [k][r]
  const int k0 = blockIdx.x * 64;
  const int r0 = blockIdx.y * 64;
  const long long b = blockIdx.z;
  const float* Xb = X + b * bs;
  const int t = threadIdx.x;  // 256
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int idx = t + 256 * i;  // 1024 float4 slots: 64 k rows x 16 r-quads
    const int kk = idx >> 4, rq = (idx & 15) << 2;
    const int k = k0 + kk, r = r0 + rq;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (k < K) {
      const float* src = Xb + static_cast<long long>(k) * ks + r;
      if (r + 3 < R) {
        v = __ldg(reinterpret_cast<const float4*>(src));
      } else {
        v.x = r < R ? __ldg(src) : 0.f;
        v.y = r + 1 < R ? __ldg(src + 1) : 0.f;
        v.z = r + 2 < R ? __ldg(src + 2) : 0.f;
      }
    }
    tile[kk][rq] = v.x;
    tile[kk][rq + 1] = v.y;
    tile[kk][rq + 2] = v.z;
    tile[kk][rq + 3] = v.w;
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int idx = t + 256 * i;  // 64 r rows x 16 k-quads
    const int rr = idx >> 4, kq = (idx & 15) << 2;
    const int r = r0 + rr, k = k0 + kq;
    if (r < R && k < kp) {
      float4 h, l;
      split1(tile[kq][rr], h.x, l.x);
      split1(tile[kq + 1][rr], h.y, l.y);
      split1(tile[kq + 2][rr], h.z, l.z);
      split1(tile[kq + 3][rr], h.w, l.w);
      const long long o = b * obs + static_cast<long long>(r) * kp + k;
      *reinterpret_cast<float4*>(hi + o) = h;
      *reinterpret_cast<float4*>(lo + o) = l;
    }
  }
}

// The strictly upper triangle of an n x n matrix from its lower triangle,
// D[c][r] = D[r][c] for r > c (the CTA-pair SYRK writes whole lower pair
// tiles, diagonal tiles included): 32 x 32 tiles below or on the diagonal,
// each read row-wise and written transposed through shared memory. (Also
// tried for bf16 with uint16_t bit patterns: 861 against 934 TFLOP/s for the
// one-CTA column-block-pair kernel at n = k = 4096, so 16-bit SYRK keeps that.)
template <typename T>
__global__ void syrk_mirror_kernel(T* __restrict__ D, long long ldd, int n) {
  __shared__ T t[32][33];
  const int bx = blockIdx.x, by = blockIdx.y;  // source tile: row block by, column block bx
  if (by < bx) return;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  for (int i = ty; i < 32; i += 8) {
    const int r = by * 32 + i, c = bx * 32 + tx;
    t[i][tx] = (r < n && c < n) ? D[static_cast<long long>(r) * ldd + c] : T(0);
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int rr = bx * 32 + i, cc = by * 32 + tx;  // destination (rr, cc) = source (cc, rr)
    if (rr < n && cc < n && cc > rr) D[static_cast<long long>(rr) * ldd + cc] = t[tx][i];
  }
}

// D = beta * C (K == 0): an empty sum times alpha is zero.
__global__ void scale_c_kernel(int out_kind, long long batch, int M, int N, float beta,
                               const void* C, long long ldc, long long strideC, void* D,
                               long long ldd, long long strideD) {
  const long long total = batch * static_cast<long long>(M) * N;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long b = i / (static_cast<long long>(M) * N);
    const long long rc = i - b * M * static_cast<long long>(N);
    const int r = static_cast<int>(rc / N), c = static_cast<int>(rc % N);
    float v = 0.0f;
    if (C && beta != 0.0f) v = beta * load_c(C, out_kind, b * strideC + r * ldc + c);
    store_d(D, out_kind, b * strideD + r * ldd + c, v);
  }
}

namespace {

CUtensorMapDataType map_dtype(int dtype) {
  switch (dtype) {
    case TRNBLAS_BF16:
      return CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    case TRNBLAS_F16:
      return CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    default:
      return CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  }
}

// Tile-walk band width (row tiles per band of the grouped order);
// TRNBLAS_B200_GEMM_GROUP_M overrides it (tuning).
int group_m_override() {
  static const int g = [] {
    const char* s = std::getenv("TRNBLAS_B200_GEMM_GROUP_M");
    const int v = (s && *s) ? std::atoi(s) : 0;
    return v > 0 ? v : 0;
  }();
  return g;
}

// Soft tile-wave synchronisation (soft_wave_wait) for long K loops with at
// least two waves of tiles. Measured on a 32768^3 bf16 product under the 1 kW
// power cap (one-CTA kernel, band of 16 row tiles): DRAM reads per launch
// 144 -> 69 GB; the same box went 1145 -> 1209 TFLOP/s (pair kernel:
// 912 -> 1347 TFLOP/s on another box).
// TRNBLAS_B200_GEMM_WAVESYNC = 0 / 1 overrides the default (on). Not used
// for a triangular operand (trmm), whose tiles' K ranges differ: the CTAs of
// a wave would wait for its longest tile.
bool use_wave_sync(long long K, long long tiles, long long grid) {
  static const int mode = [] {
    const char* s = std::getenv("TRNBLAS_B200_GEMM_WAVESYNC");
    return (s && *s) ? std::atoi(s) : 1;
  }();
  return mode != 0 && K >= 4096 && tiles >= 2 * grid;
}

template <int KIND, int BN, int STAGES>
int launch_gemm(const CUtensorMap& a0, const CUtensorMap& a1, const CUtensorMap& b0,
                const CUtensorMap& b1, GemmParams& p, cudaStream_t stream) {
  using Cfg = GemmCfg<KIND, BN>;
  constexpr int smem = STAGES * Cfg::STAGE_BYTES + 1024 + kGemmBarBytes + kEpiStageBytes;
  auto kern = gemm_sm100_kernel<KIND, BN, STAGES>;
  static bool attr_set[64] = {};  // the attribute is set per device
  const int dev = current_device();
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(gemm smem)");
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const int grid = static_cast<int>(std::min<long long>(p.num_tiles, num_sms()));
  if (p.mode == kModeGemm && !p.tri && use_wave_sync(p.K, p.num_tiles, grid)) p.wave_ctr = wave_counter(stream);
  kern<<<grid, Cfg::THREADS, smem, stream>>>(a0, a1, b0, b1, p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "gemm kernel launch");
  return TRNBLAS_OK;
}

// The CTA-pair kernel: clusters of two CTAs, as many pairs as can be
// resident at once (the persistent tile walk needs every pair running).
// a1 / b1: the lo planes of the split pass for kTF32x3 (pass a / b again for kF16).
template <int KIND, int STAGES>
int launch_gemm_pair(const CUtensorMap& a, const CUtensorMap& a1, const CUtensorMap& b,
                     const CUtensorMap& b1, GemmParams& p, cudaStream_t stream) {
  using Cfg = PairGemmCfg<KIND, STAGES>;
  constexpr int smem = Cfg::SMEM;
  auto kern = gemm_pair_kernel<KIND, STAGES>;
  static int max_pairs[64] = {};
  const int dev = current_device();
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(Cfg::THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (dev < 0 || dev >= 64 || !max_pairs[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute(pair gemm smem)");
    cfg.gridDim = dim3(2 * (num_sms() / 2), 1, 1);
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
    if (e != cudaSuccess) return cuda_fail(e, "cudaOccupancyMaxActiveClusters(pair gemm)");
    if (clusters < 1) {
      set_error("pair gemm: no CTA pair fits on this device");
      return TRNBLAS_ERR_CUDA;
    }
    if (dev >= 0 && dev < 64) max_pairs[dev] = clusters;
    else return TRNBLAS_ERR_CUDA;
  }
  const int pairs = static_cast<int>(std::min<long long>(p.num_tiles, max_pairs[dev]));
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  if (!p.tri && use_wave_sync(p.K, p.num_tiles, pairs)) p.wave_ctr = wave_counter(stream);
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a, a1, b, b1, p);
  if (e != cudaSuccess) return cuda_fail(e, "pair gemm kernel launch");
  return TRNBLAS_OK;
}

bool valid_dtype_f16(int dtype) { return dtype == TRNBLAS_BF16 || dtype == TRNBLAS_F16; }

// CTA-pair tiles (256 x 256) when there are at least as many pair tiles as
// SM pairs (one full wave), M, N > 128 and K >= 1024; smaller problems keep
// the one-CTA kernel, whose smaller tiles occupy more SMs (fp32 1024^3: 16
// pair tiles on 32 SMs ran at 33 TFLOP/s against 39 for 64 one-CTA tiles) and
// whose shorter pipeline fills faster on short K loops (bf16 batched 64 x
// 512^3: 449 TFLOP/s on pairs against 499 on one-CTA 128 x 256 tiles).
// TRNBLAS_B200_GEMM_PAIR=0 keeps the one-CTA kernel everywhere.
// Measured at 32768^3 bf16 under the 1 kW power cap, same box: pair kernel
// with the wave synchronisation 1347 TFLOP/s (52.6 J a product), one-CTA
// kernel 1248 TFLOP/s (52.5-58.7 J). Without the wave synchronisation the
// pair kernel's tiles drift apart and re-read 246 GB from DRAM per product,
// and it lost (912 against 1130 TFLOP/s).
// `wave_div`: the pair tiles needed, as a fraction 1 / wave_div of the SMs
// (2: one wave of pairs; fp32 passes 4, since its one-CTA tiles are shared-
// memory bound and a half-empty wave of pairs still wins: fp32 2048^3, 64
// pair tiles, 171 against 140 TFLOP/s; 3072^3 231 against 185).
bool use_pair_gemm(long long batch, long long M, long long N, long long K, int wave_div = 2) {
  static const int mode = [] {
    const char* s = std::getenv("TRNBLAS_B200_GEMM_PAIR");
    return (s && *s) ? std::atoi(s) : 1;
  }();
  return mode != 0 && M > 128 && N > 128 && K >= 1024 &&
         batch * ceil_div(M, 256) * ceil_div(N, 256) >= num_sms() / wave_div;
}

// fp32 (3xTF32) with the split fused into the GEMM kernel (kTF32x3F) instead
// of the split pass. Off unless TRNBLAS_B200_TF32_FUSED=1: the 3xTF32 MMAs of
// 128 x 128 tiles already take about all of the SM's shared-memory read
// bandwidth (8 KB a 64-cycle K step), and the converter warps' reads and
// writes of every stage come on top, where the split pass adds only the TMA
// writes of the lo tiles. Measured at 8192^3: fused 115 TFLOP/s against
// 207 TFLOP/s for the split pass plus GEMM.
bool use_fused_tf32() {
  static const int mode = [] {
    const char* s = std::getenv("TRNBLAS_B200_TF32_FUSED");
    return (s && *s) ? std::atoi(s) : 0;
  }();
  return mode != 0;
}

// Bytes of one fp32 split plane (R x Kp) for `nb` batch entries, 256-aligned.
size_t plane_bytes(long long nb, long long R, long long K) {
  const long long kp = round_up(std::max<long long>(K, 1), 4);
  return static_cast<size_t>(round_up(nb * R * kp * 4, 256));
}

int check_dims(long long batch, long long M, long long N, long long K) {
  if (batch < 0 || M < 0 || N < 0 || K < 0) {
    set_error("negative size");
    return TRNBLAS_ERR_ARG;
  }
  const long long lim = (1ll << 31) - 1;
  // K is padded to a multiple of 4 for the fp32 split planes and the padded
  // length is used as an int (kernel arguments, tensor-map row stride)
  if (M > lim || N > lim || K > (lim & ~3ll) || batch > 65535ll * 65535ll) {
    set_error("size exceeds the element limit per dimension (2^31-1; K: 2^31-4)");
    return TRNBLAS_ERR_ARG;
  }
  return TRNBLAS_OK;
}

int launch_split(const float* X, long long rs, long long ks, long long bs, long long nb,
                 long long R, long long K, float* hi, float* lo, cudaStream_t stream) {
  const long long kp = round_up(std::max<long long>(K, 1), 4);
  if (ks == 1 && R <= (1ll << 31) - 1 && nb <= 65535) {
    const int vec = (rs % 4 == 0) && (bs % 4 == 0) && (reinterpret_cast<uintptr_t>(X) % 16 == 0);
    const long long kq = kp / 4;
    dim3 blk(64, 4);
    dim3 g(static_cast<unsigned>(std::min<long long>(ceil_div(kq, 64), 1024)),
           static_cast<unsigned>(std::min<long long>(ceil_div(R, 4), 65535)), static_cast<unsigned>(nb));
    split_tf32_rows_kernel<<<g, blk, 0, stream>>>(X, rs, bs, static_cast<int>(R), static_cast<int>(K),
                                                  static_cast<int>(kp), R * kp, vec, hi, lo);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "split kernel launch");
    return TRNBLAS_OK;
  }
  if (rs == 1 && ks % 4 == 0 && bs % 4 == 0 && reinterpret_cast<uintptr_t>(X) % 16 == 0 &&
      ceil_div(R, 64) <= 65535 && nb <= 65535) {
    dim3 g(static_cast<unsigned>(ceil_div(kp, 64)), static_cast<unsigned>(ceil_div(R, 64)),
           static_cast<unsigned>(nb));
    split_tf32_t64_kernel<<<g, 256, 0, stream>>>(X, ks, bs, static_cast<int>(R), static_cast<int>(K),
                                                 static_cast<int>(kp), R * kp, hi, lo);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, "split kernel launch");
    return TRNBLAS_OK;
  }
  dim3 grid(static_cast<unsigned>(ceil_div(kp, 32)), static_cast<unsigned>(ceil_div(R, 32)),
            static_cast<unsigned>(nb));
  if (grid.y > 65535 || grid.z > 65535) {
    set_error("split grid too large");
    return TRNBLAS_ERR_ARG;
  }
  split_tf32_kernel<<<grid, dim3(32, 8), 0, stream>>>(X, rs, ks, bs, static_cast<int>(R),
                                                      static_cast<int>(K),
                                                      static_cast<int>(kp), R * kp, hi, lo);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "split kernel launch");
  return TRNBLAS_OK;
}

// The split of a symmetric n x n operand S read from its stored triangle
// (row-major, leading dimension lds; `lower`: S[r][k] = A[r][k] for r >= k,
// else A[k][r]), into K-major planes hi / lo of n rows by kp = round_up(n, 4)
// (the symm path: no materialised full S). 32 x 32 tiles: a tile below the
// stored diagonal is read in place (lanes along k), one above it through the
// transpose (lanes along r, the tile of the mirrored block), a diagonal tile
// both ways, each element taking the one from the stored triangle.
__global__ void split_tf32_sym_kernel(const float* __restrict__ X, long long lds, int n, int lower,
                                      int kp, float* __restrict__ hi, float* __restrict__ lo) {
  __shared__ float direct[32][33], mirror[32][33];
  const int k0 = blockIdx.x * 32;
  const int r0 = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  // in the stored triangle: r >= k (lower) or r <= k (upper)
  const bool all_stored = lower ? (r0 >= k0 + 31) : (r0 + 31 <= k0);
  const bool none_stored = lower ? (r0 + 31 < k0) : (r0 > k0 + 31);
  if (!none_stored) {
    for (int i = ty; i < 32; i += 8) {
      const int r = r0 + i, k = k0 + tx;
      direct[i][tx] = (r < n && k < n) ? __ldg(X + static_cast<long long>(r) * lds + k) : 0.0f;
    }
  }
  if (!all_stored) {
    // S[r][k] = A[k][r]: read rows k of A along r, store transposed
    for (int i = ty; i < 32; i += 8) {
      const int k = k0 + i, r = r0 + tx;
      mirror[tx][i] = (r < n && k < n) ? __ldg(X + static_cast<long long>(k) * lds + r) : 0.0f;
    }
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int r = r0 + i, k = k0 + tx;
    if (r < n && k < kp) {
      const bool stored = lower ? (r >= k) : (r <= k);
      const float x = (k < n) ? (stored ? direct[i][tx] : mirror[i][tx]) : 0.0f;
      float h, l;
      split1(x, h, l);
      const long long o = static_cast<long long>(r) * kp + k;
      hi[o] = h;
      lo[o] = l;
    }
  }
}

// The full symmetric n x n matrix of 16-bit elements (bf16 / fp16 bit
// patterns copied as they are) from the stored triangle of X, into S
// (row-major, leading dimension ldo >= n): the same tile scheme as
// split_tf32_sym_kernel, one pass.
__global__ void sym_fill16_kernel(const uint16_t* __restrict__ X, long long lds, int n, int lower,
                                  long long ldo, uint16_t* __restrict__ S) {
  __shared__ uint16_t direct[32][33], mirror[32][33];
  const int k0 = blockIdx.x * 32;
  const int r0 = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  const bool all_stored = lower ? (r0 >= k0 + 31) : (r0 + 31 <= k0);
  const bool none_stored = lower ? (r0 + 31 < k0) : (r0 > k0 + 31);
  if (!none_stored) {
    for (int i = ty; i < 32; i += 8) {
      const int r = r0 + i, k = k0 + tx;
      direct[i][tx] = (r < n && k < n) ? X[static_cast<long long>(r) * lds + k] : uint16_t(0);
    }
  }
  if (!all_stored) {
    for (int i = ty; i < 32; i += 8) {
      const int k = k0 + i, r = r0 + tx;
      mirror[tx][i] = (r < n && k < n) ? X[static_cast<long long>(k) * lds + r] : uint16_t(0);
    }
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int r = r0 + i, k = k0 + tx;
    if (r < n && k < n) {
      const bool stored = lower ? (r >= k) : (r <= k);
      S[static_cast<long long>(r) * ldo + k] = stored ? direct[i][tx] : mirror[i][tx];
    }
  }
}

int launch_split_sym(const float* X, long long lds, long long n, int lower, float* hi, float* lo,
                     cudaStream_t stream) {
  const long long kp = round_up(std::max<long long>(n, 1), 4);
  dim3 grid(static_cast<unsigned>(ceil_div(kp, 32)), static_cast<unsigned>(ceil_div(n, 32)), 1);
  if (grid.y > 65535) {
    set_error("symmetric split grid too large");
    return TRNBLAS_ERR_ARG;
  }
  split_tf32_sym_kernel<<<grid, dim3(32, 8), 0, stream>>>(X, lds, static_cast<int>(n), lower,
                                                          static_cast<int>(kp), hi, lo);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? TRNBLAS_OK : cuda_fail(e, "symmetric split kernel launch");
}

// Pick BN for the bf16/fp16 GEMM: 256 unless 128 balances the waves better.
int pick_bn(long long batch, long long M, long long N) {
  if (N <= 128) return 128;
  const long long sms = num_sms();
  auto eff = [&](long long bn, double tile_eff) {
    const long long tiles = batch * ceil_div(M, 128) * ceil_div(N, bn);
    const long long waves = ceil_div(tiles, sms);
    const double fill = static_cast<double>(tiles) / static_cast<double>(waves * sms);
    const double ncover = static_cast<double>(N) / static_cast<double>(ceil_div(N, bn) * bn);
    return fill * ncover * tile_eff;
  };
  return eff(256, 1.0) >= eff(128, 0.85) ? 256 : 128;
}

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" {

size_t trnblas_gemm_workspace_size(int dtype, int64_t batch, int64_t M, int64_t N, int64_t K,
                                   int64_t strideA, int64_t strideB) {
  if (dtype != TRNBLAS_F32 || batch <= 0 || M <= 0 || N <= 0 || K <= 0) return 0;
  const long long na = strideA ? batch : 1, nbb = strideB ? batch : 1;
  return 2 * plane_bytes(na, M, K) + 2 * plane_bytes(nbb, N, K);
}

// Operands that arrive while the GEMM runs (trnblas_gemm_ready).
struct ReadySpec {
  const int* flags;
  int epoch;
  long long shard_rows;  // rows of op(A) per flag
  int b0;                // flags[b0 + b]: batch entry b of op(B)
  long long rot_rows;    // the walk starts at this row of op(A) ...
  int rot_b;             // ... and at this batch entry
};

static int gemm_impl(int dtype, int64_t batch, int64_t M, int64_t N, int64_t K, float alpha,
                     const void* A, int64_t lda, int64_t strideA, int transA, const void* B,
                     int64_t ldb, int64_t strideB, int transB, float beta, const void* C,
                     int64_t ldc, int64_t strideC, void* D, int64_t ldd, int64_t strideD,
                     void* workspace, size_t workspace_bytes, void* stream_, const ReadySpec* rs,
                     int tri = 0, int sym = 0) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (int rc = check_dims(batch, M, N, K)) return rc;
  if (dtype != TRNBLAS_F32 && !valid_dtype_f16(dtype)) {
    set_error("trnblas_gemm: dtype must be F32, BF16 or F16");
    return TRNBLAS_ERR_ARG;
  }
  if (batch == 0 || M == 0 || N == 0) return TRNBLAS_OK;
  if (!D || (K > 0 && (!A || !B))) {
    set_error("trnblas_gemm: NULL operand");
    return TRNBLAS_ERR_ARG;
  }
  if (ldd < N || (C && beta != 0.0f && ldc < N)) {
    set_error("trnblas_gemm: ldc/ldd smaller than N");
    return TRNBLAS_ERR_ARG;
  }
  // Stored row lengths: A is M x K (K x M when transposed), B is K x N
  // (N x K when transposed). Every dtype reads rows of that length at stride
  // ld (the fp32 split kernels as well as the TMA maps), so a shorter or
  // negative ld would read outside the operand.
  {
    const long long a_cols = transA ? M : K, b_cols = transB ? K : N;
    if (K > 0 && (lda < a_cols || ldb < b_cols || lda < 1 || ldb < 1)) {
      set_error("trnblas_gemm: lda/ldb smaller than the stored row length");
      return TRNBLAS_ERR_ARG;
    }
  }
  int* status = status_word();
  if (!status) return TRNBLAS_ERR_CUDA;
  const int out_kind = dtype == TRNBLAS_F32 ? kOutF32 : dtype == TRNBLAS_BF16 ? kOutBF16 : kOutF16;
  if (K == 0) {
    const long long total = batch * M * N;
    const int blocks = static_cast<int>(std::min<long long>(ceil_div(total, 256), 4096));
    scale_c_kernel<<<blocks, 256, 0, stream>>>(out_kind, batch, static_cast<int>(M),
                                               static_cast<int>(N), beta, C, ldc, strideC, D,
                                               ldd, strideD);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? TRNBLAS_OK : cuda_fail(e, "scale kernel launch");
  }

  GemmParams p{};
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.batch = static_cast<int>(batch);
  p.mode = kModeGemm;
  p.out_kind = out_kind;
  p.c_mode = (C && beta != 0.0f) ? kCRow : kCNone;
  p.alpha = alpha;
  p.beta = beta;
  p.C = C;
  p.ldc = ldc;
  p.strideC = strideC;
  p.D = D;
  p.ldd = ldd;
  p.strideD = strideD;
  // bands of 12 row tiles: with the wave synchronisation, the lowest energy
  // per flop measured at 32768^3 under the power cap (widths 4 .. 16 swept)
  p.group_m = group_m_override() ? group_m_override() : 12;
  p.tri = tri;
  p.status = status;
  p.timeout_ns = wait_timeout_ns();
  const bool a_b = strideA != 0 && batch > 1;
  const bool b_b = strideB != 0 && batch > 1;
  p.a_batched = a_b;
  p.b_batched = b_b;
  const long long nba = a_b ? batch : 1, nbb = b_b ? batch : 1;

  CUtensorMap ma0, ma1, mb0, mb1;
  if (rs) {
    if (dtype == TRNBLAS_F32 || !rs->flags || rs->shard_rows <= 0 || rs->shard_rows % 256 ||
        rs->rot_rows < 0 || rs->rot_rows % 256 || rs->rot_rows >= M || rs->rot_b < 0 ||
        rs->rot_b >= batch || rs->b0 < 0) {
      set_error("trnblas_gemm_ready: bf16/fp16 only; flags, shard_rows and rot_rows (multiples of "
                "256) and rot_b < batch required");
      return TRNBLAS_ERR_ARG;
    }
    p.ready = rs->flags;
    p.ready_epoch = rs->epoch;
    p.ready_b0 = rs->b0;
    p.rot_b = rs->rot_b;
  }
  // fp32 with operands the TMA can read (16-byte aligned bases, row and batch
  // strides multiples of 4 elements), when use_fused_tf32(): the split fused
  // into the GEMM kernel. K-major operands as 128-byte swizzle rows of 32 K,
  // MN-major ones as boxes of 32 MN x 32 K with the 128-byte swizzle of
  // 32-byte atoms.
  auto tma_f32 = [](const void* X, long long ld, long long bstride, bool batched) {
    return (reinterpret_cast<uintptr_t>(X) & 15) == 0 && ld % 4 == 0 && (!batched || bstride % 4 == 0);
  };
  if (dtype == TRNBLAS_F32 && !sym && use_fused_tf32() && tma_f32(A, lda, strideA, a_b) &&
      tma_f32(B, ldb, strideB, b_b)) {
    const auto dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    p.a_mn = transA ? 1 : 0;  // A stored K x M
    p.b_mn = transB ? 0 : 1;  // B stored K x N
    p.in_fmt = kFmtTF32;
    const long long a_rows = transA ? K : M, b_rows = transB ? N : K;
    const long long sa2 = a_b ? strideA : round_up(lda * a_rows, 4);
    const long long sb2 = b_b ? strideB : round_up(ldb * b_rows, 4);
    auto mn_map = [&](CUtensorMap* m, const void* X, long long mn, long long ld, long long s2,
                      long long nb) {
      const uint64_t dims[3] = {static_cast<uint64_t>(mn), static_cast<uint64_t>(K),
                                static_cast<uint64_t>(nb)};
      const uint64_t strides[2] = {static_cast<uint64_t>(ld), static_cast<uint64_t>(s2)};
      const uint32_t box[3] = {32, 32, 1};
      return encode_map(m, dt, 4, X, 3, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
    };
    const bool ok = (p.a_mn ? mn_map(&ma0, A, M, lda, sa2, nba)
                            : encode_map_3d(&ma0, dt, 4, A, K, M, nba, lda, sa2, 32, 128)) &&
                    (p.b_mn ? mn_map(&mb0, B, N, ldb, sb2, nbb)
                            : encode_map_3d(&mb0, dt, 4, B, K, N, nbb, ldb, sb2, 32, 128));
    if (!ok) return TRNBLAS_ERR_ALIGN;
    p.tiles_m = static_cast<int>(ceil_div(M, 128));
    p.tiles_n = static_cast<int>(ceil_div(N, 128));
    p.num_tiles = static_cast<int>(batch * p.tiles_m * p.tiles_n);
    return launch_gemm<kTF32x3F, 128, 3>(ma0, ma0, mb0, mb0, p, stream);
  }
  if (dtype == TRNBLAS_F32) {
    const size_t need = trnblas_gemm_workspace_size(dtype, batch, M, N, K, strideA, strideB);
    if (!workspace || workspace_bytes < need) {
      set_error("trnblas_gemm: fp32 needs " + std::to_string(need) + " workspace bytes");
      return TRNBLAS_ERR_WORKSPACE;
    }
    const long long kp = round_up(K, 4);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    float* ahi = reinterpret_cast<float*>(ws);
    float* alo = reinterpret_cast<float*>(ws + plane_bytes(nba, M, K));
    float* bhi = reinterpret_cast<float*>(ws + 2 * plane_bytes(nba, M, K));
    float* blo = reinterpret_cast<float*>(ws + 2 * plane_bytes(nba, M, K) + plane_bytes(nbb, N, K));
    const float* Af = static_cast<const float*>(A);
    const float* Bf = static_cast<const float*>(B);
    // op(A)(m, k) and op(B)^T(n, k) strides
    const long long ars = transA ? 1 : lda, aks = transA ? lda : 1;
    const long long brs = transB ? ldb : 1, bks = transB ? 1 : ldb;
    // sym: op(A) (1 / 2) or op(B) (3 / 4) is symmetric, read from its stored
    // lower (1 / 3) or upper (2 / 4) triangle by the symmetric split
    if (int rc = (sym == 1 || sym == 2)
                     ? launch_split_sym(Af, lda, M, sym == 1, ahi, alo, stream)
                     : launch_split(Af, ars, aks, a_b ? strideA : 0, nba, M, K, ahi, alo, stream))
      return rc;
    if (int rc = (sym == 3 || sym == 4)
                     ? launch_split_sym(Bf, ldb, N, sym == 3, bhi, blo, stream)
                     : launch_split(Bf, brs, bks, b_b ? strideB : 0, nbb, N, K, bhi, blo, stream))
      return rc;
    const auto dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    if (!encode_map_3d(&ma0, dt, 4, ahi, K, M, nba, kp, M * kp, 32, 128) ||
        !encode_map_3d(&ma1, dt, 4, alo, K, M, nba, kp, M * kp, 32, 128) ||
        !encode_map_3d(&mb0, dt, 4, bhi, K, N, nbb, kp, N * kp, 32, 128) ||
        !encode_map_3d(&mb1, dt, 4, blo, K, N, nbb, kp, N * kp, 32, 128))
      return TRNBLAS_ERR_ALIGN;
    p.a_mn = 0;
    p.b_mn = 0;
    p.in_fmt = kFmtTF32;
    if (use_pair_gemm(batch, M, N, K, 4)) {
      // 256 x 256 tiles on CTA pairs: each CTA reads half the shared-memory
      // bytes per MMA of a 128 x 128 tile
      p.group_m = group_m_override() ? group_m_override() : 8;
      p.tiles_m = static_cast<int>(ceil_div(M, 256));
      p.tiles_n = static_cast<int>(ceil_div(N, 256));
      p.num_tiles = static_cast<int>(batch * p.tiles_m * p.tiles_n);
      return launch_gemm_pair<kTF32x3, 3>(ma0, ma1, mb0, mb1, p, stream);
    }
    p.tiles_m = static_cast<int>(ceil_div(M, 128));
    p.tiles_n = static_cast<int>(ceil_div(N, 128));
    p.num_tiles = static_cast<int>(batch * p.tiles_m * p.tiles_n);
    return launch_gemm<kTF32x3, 128, 3>(ma0, ma1, mb0, mb1, p, stream);
  }

  // bf16 / fp16: operands straight from their own layout.
  const auto dt = map_dtype(dtype);
  p.a_mn = transA ? 1 : 0;   // A stored K x M: M contiguous
  p.b_mn = transB ? 0 : 1;   // B stored K x N: N contiguous
  p.in_fmt = dtype == TRNBLAS_BF16 ? kFmtBF16 : kFmtF16;
  const long long a_rows = transA ? K : M;
  const long long b_rows = transB ? N : K;
  const long long sa2 = a_b ? strideA : round_up(lda * a_rows, 8);
  const long long sb2 = b_b ? strideB : round_up(ldb * b_rows, 8);
  if (use_pair_gemm(batch, M, N, K)) {
    // 256 x 256 tiles on CTA pairs; each CTA loads 128 rows of A and 128
    // columns of B
    bool ok = p.a_mn ? encode_map_3d(&ma0, dt, 2, A, M, K, nba, lda, sa2, 64, 64)
                     : encode_map_3d(&ma0, dt, 2, A, K, M, nba, lda, sa2, 64, 128);
    ok = ok && (p.b_mn ? encode_map_3d(&mb0, dt, 2, B, N, K, nbb, ldb, sb2, 64, 64)
                       : encode_map_3d(&mb0, dt, 2, B, K, N, nbb, ldb, sb2, 64, 128));
    if (!ok) return TRNBLAS_ERR_ALIGN;
    p.group_m = group_m_override() ? group_m_override() : 8;
    p.tiles_m = static_cast<int>(ceil_div(M, 256));
    p.tiles_n = static_cast<int>(ceil_div(N, 256));
    p.num_tiles = static_cast<int>(batch * p.tiles_m * p.tiles_n);
    if (rs) {
      p.shard_tiles_m = static_cast<int>(rs->shard_rows / 256);
      p.rot_m = static_cast<int>(rs->rot_rows / 256) % p.tiles_m;
    }
    return launch_gemm_pair<kF16, 6>(ma0, ma0, mb0, mb0, p, stream);
  }
  const int bn = pick_bn(batch, M, N);
  bool ok = p.a_mn ? encode_map_3d(&ma0, dt, 2, A, M, K, nba, lda, sa2, 64, 64)
                   : encode_map_3d(&ma0, dt, 2, A, K, M, nba, lda, sa2, 64, 128);
  ok = ok && (p.b_mn ? encode_map_3d(&mb0, dt, 2, B, N, K, nbb, ldb, sb2, 64, 64)
                     : encode_map_3d(&mb0, dt, 2, B, K, N, nbb, ldb, sb2, 64, bn));
  if (!ok) return TRNBLAS_ERR_ALIGN;
  p.tiles_m = static_cast<int>(ceil_div(M, 128));
  p.tiles_n = static_cast<int>(ceil_div(N, bn));
  p.num_tiles = static_cast<int>(batch * p.tiles_m * p.tiles_n);
  if (rs) {
    p.shard_tiles_m = static_cast<int>(rs->shard_rows / 128);
    p.rot_m = static_cast<int>(rs->rot_rows / 128) % p.tiles_m;
  }
  if (bn == 256) return launch_gemm<kF16, 256, 4>(ma0, ma0, mb0, mb0, p, stream);
  return launch_gemm<kF16, 128, 6>(ma0, ma0, mb0, mb0, p, stream);
}

int trnblas_gemm(int dtype, int64_t batch, int64_t M, int64_t N, int64_t K, float alpha,
                 const void* A, int64_t lda, int64_t strideA, int transA, const void* B,
                 int64_t ldb, int64_t strideB, int transB, float beta, const void* C,
                 int64_t ldc, int64_t strideC, void* D, int64_t ldd, int64_t strideD,
                 void* workspace, size_t workspace_bytes, void* stream) {
  return gemm_impl(dtype, batch, M, N, K, alpha, A, lda, strideA, transA, B, ldb, strideB, transB,
                   beta, C, ldc, strideC, D, ldd, strideD, workspace, workspace_bytes, stream,
                   nullptr);
}

int trnblas_gemm_tri(int dtype, int64_t batch, int64_t M, int64_t N, int64_t K, float alpha,
                     const void* A, int64_t lda, int64_t strideA, int transA, const void* B,
                     int64_t ldb, int64_t strideB, int transB, float beta, const void* C,
                     int64_t ldc, int64_t strideC, void* D, int64_t ldd, int64_t strideD, int tri,
                     void* workspace, size_t workspace_bytes, void* stream) {
  if (tri < 0 || tri > 4) {
    set_error("trnblas_gemm_tri: tri must be 0 .. 4");
    return TRNBLAS_ERR_ARG;
  }
  return gemm_impl(dtype, batch, M, N, K, alpha, A, lda, strideA, transA, B, ldb, strideB, transB,
                   beta, C, ldc, strideC, D, ldd, strideD, workspace, workspace_bytes, stream,
                   nullptr, tri);
}

size_t trnblas_symm_workspace_size(int dtype, int side_right, int64_t M, int64_t N) {
  const int64_t n = side_right ? N : M;
  if (dtype == TRNBLAS_F32) return trnblas_gemm_workspace_size(dtype, 1, M, N, n, 0, 0);
  if (n <= 0) return 256;
  // the full symmetric operand, rows padded to 8 elements (16 bytes)
  return static_cast<size_t>(round_up(n * round_up(n, 8) * 2, 256));
}

int trnblas_symm(int dtype, int side_right, int uplo_lower, int64_t M, int64_t N, float alpha,
                 const void* A, int64_t lda, const void* B, int64_t ldb, float beta, const void* C,
                 int64_t ldc, void* D, int64_t ldd, void* workspace, size_t workspace_bytes,
                 void* stream) {
  if (dtype != TRNBLAS_F32 && !valid_dtype_f16(dtype)) {
    set_error("trnblas_symm: dtype must be F32, BF16 or F16");
    return TRNBLAS_ERR_ARG;
  }
  if (valid_dtype_f16(dtype)) {
    // 16-bit: the full symmetric operand formed in the workspace in one pass
    // from the stored triangle, then the GEMM kernel on it
    const long long n = side_right ? N : M;
    if (int rc = check_dims(1, M, N, n)) return rc;
    if (M == 0 || N == 0) return TRNBLAS_OK;
    // every argument the GEMM will check, before the fill pass is queued
    if (!D || ldd < N || (C && beta != 0.0f && ldc < N) ||
        (n > 0 && (!A || !B || lda < n || ldb < N))) {
      set_error("trnblas_symm: NULL operand, or lda/ldb/ldc/ldd smaller than the stored row length");
      return TRNBLAS_ERR_ARG;
    }
    const long long lds = round_up(std::max<long long>(n, 1), 8);
    const size_t need = trnblas_symm_workspace_size(dtype, side_right, M, N);
    if (n > 0) {
      if (!workspace || workspace_bytes < need) {
        set_error("trnblas_symm: 16-bit needs " + std::to_string(need) + " workspace bytes");
        return TRNBLAS_ERR_WORKSPACE;
      }
      if (ceil_div(n, 32) > 65535) {
        set_error("trnblas_symm: n too large for the fill grid");
        return TRNBLAS_ERR_ARG;
      }
      const dim3 grid(static_cast<unsigned>(ceil_div(n, 32)), static_cast<unsigned>(ceil_div(n, 32)), 1);
      sym_fill16_kernel<<<grid, dim3(32, 8), 0, static_cast<cudaStream_t>(stream)>>>(
          static_cast<const uint16_t*>(A), lda, static_cast<int>(n), uplo_lower, lds,
          static_cast<uint16_t*>(workspace));
      cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) return cuda_fail(e, "symmetric fill kernel launch");
    }
    if (!side_right)
      return gemm_impl(dtype, 1, M, N, n, alpha, workspace, lds, 0, 0, B, ldb, 0, 0, beta, C, ldc, 0,
                       D, ldd, 0, nullptr, 0, stream, nullptr);
    return gemm_impl(dtype, 1, M, N, n, alpha, B, ldb, 0, 0, workspace, lds, 0, 0, beta, C, ldc, 0, D,
                     ldd, 0, nullptr, 0, stream, nullptr);
  }
  if (!side_right) {
    // D = alpha S B + beta C: S (M x M) is op(A), read from its stored triangle
    return gemm_impl(dtype, 1, M, N, M, alpha, A, lda, 0, 0, B, ldb, 0, 0, beta, C, ldc, 0, D, ldd,
                     0, workspace, workspace_bytes, stream, nullptr, 0, uplo_lower ? 1 : 2);
  }
  // D = alpha B S + beta C: S (N x N) is op(B)
  return gemm_impl(dtype, 1, M, N, N, alpha, B, ldb, 0, 0, A, lda, 0, 0, beta, C, ldc, 0, D, ldd, 0,
                   workspace, workspace_bytes, stream, nullptr, 0, uplo_lower ? 3 : 4);
}

int trnblas_gemm_ready(int dtype, int64_t batch, int64_t M, int64_t N, int64_t K, float alpha,
                       const void* A, int64_t lda, int64_t strideA, int transA, const void* B,
                       int64_t ldb, int64_t strideB, int transB, float beta, const void* C,
                       int64_t ldc, int64_t strideC, void* D, int64_t ldd, int64_t strideD,
                       const int* ready, int epoch, int64_t shard_rows, int ready_b0,
                       int64_t rot_rows, int rot_b, void* stream) {
  const ReadySpec rs{ready, epoch, shard_rows, ready_b0, rot_rows, rot_b};
  return gemm_impl(dtype, batch, M, N, K, alpha, A, lda, strideA, transA, B, ldb, strideB, transB,
                   beta, C, ldc, strideC, D, ldd, strideD, nullptr, 0, stream, &rs);
}

size_t trnblas_syrk_workspace_size(int dtype, int64_t n, int64_t k) {
  if (dtype != TRNBLAS_F32 || n <= 0 || k <= 0) return 0;
  return 2 * plane_bytes(1, n, k);
}

int trnblas_syrk(int dtype, int64_t n, int64_t k, float alpha, const void* A, int64_t lda,
                 int trans, float beta, const void* C, int64_t ldc, int c_uplo, void* D,
                 int64_t ldd, void* workspace, size_t workspace_bytes, void* stream_) {
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  if (int rc = check_dims(1, n, n, k)) return rc;
  if (dtype != TRNBLAS_F32 && !valid_dtype_f16(dtype)) {
    set_error("trnblas_syrk: dtype must be F32, BF16 or F16");
    return TRNBLAS_ERR_ARG;
  }
  if (c_uplo < 0 || c_uplo > 2) {
    set_error("trnblas_syrk: c_uplo must be 0, 1 (lower) or 2 (upper)");
    return TRNBLAS_ERR_ARG;
  }
  if (n == 0) return TRNBLAS_OK;
  const bool use_c = C && beta != 0.0f && c_uplo != 0;
  if (!D || (k > 0 && !A) || ldd < n || (use_c && ldc < n)) {
    set_error("trnblas_syrk: NULL operand or leading dimension smaller than n");
    return TRNBLAS_ERR_ARG;
  }
  // A is stored n x k (k x n when trans); every dtype reads rows of that
  // length at stride lda
  if (k > 0 && (lda < (trans ? n : k) || lda < 1)) {
    set_error("trnblas_syrk: lda smaller than the stored row length");
    return TRNBLAS_ERR_ARG;
  }
  int* status = status_word();
  if (!status) return TRNBLAS_ERR_CUDA;
  const int out_kind = dtype == TRNBLAS_F32 ? kOutF32 : dtype == TRNBLAS_BF16 ? kOutBF16 : kOutF16;
  GemmParams p{};
  p.M = static_cast<int>(n);
  p.N = static_cast<int>(n);
  p.K = static_cast<int>(k);
  p.batch = 1;
  p.mode = kModeSyrk;
  p.out_kind = out_kind;
  p.c_mode = use_c ? (c_uplo == 1 ? kCRow : kCTrans) : kCNone;
  p.alpha = alpha;
  p.beta = beta;
  p.C = C;
  p.ldc = ldc;
  p.D = D;
  p.ldd = ldd;
  p.group_m = 16;
  p.status = status;
  p.timeout_ns = wait_timeout_ns();
  p.tiles_m = p.tiles_n = static_cast<int>(ceil_div(n, 128));
  p.num_tiles = p.tiles_m * (p.tiles_m + 1) / 2;
  if (k == 0) {
    // beta * sym(C) alone needs no tile walk; the Python layer forms it.
    set_error("trnblas_syrk: k must be positive");
    return TRNBLAS_ERR_ARG;
  }
  CUtensorMap ma0, ma1;
  if (dtype == TRNBLAS_F32 && use_fused_tf32() && !trans && (reinterpret_cast<uintptr_t>(A) & 15) == 0 &&
      lda % 4 == 0) {
    // the split fused into the kernel: raw fp32 K-major tiles of A for both
    // operands
    const auto dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    p.a_mn = p.b_mn = 0;
    p.in_fmt = kFmtTF32;
    if (!encode_map_3d(&ma0, dt, 4, A, k, n, 1, lda, round_up(lda * n, 4), 32, 128))
      return TRNBLAS_ERR_ALIGN;
    return launch_gemm<kTF32x3F, 128, 3>(ma0, ma0, ma0, ma0, p, stream);
  }
  if (dtype == TRNBLAS_F32) {
    const size_t need = trnblas_syrk_workspace_size(dtype, n, k);
    if (!workspace || workspace_bytes < need) {
      set_error("trnblas_syrk: fp32 needs " + std::to_string(need) + " workspace bytes");
      return TRNBLAS_ERR_WORKSPACE;
    }
    const long long kp = round_up(k, 4);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    float* ahi = reinterpret_cast<float*>(ws);
    float* alo = reinterpret_cast<float*>(ws + plane_bytes(1, n, k));
    const long long rs = trans ? 1 : lda, ks = trans ? lda : 1;
    if (int rc = launch_split(static_cast<const float*>(A), rs, ks, 0, 1, n, k, ahi, alo, stream))
      return rc;
    const auto dt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    if (!encode_map_3d(&ma0, dt, 4, ahi, k, n, 1, kp, n * kp, 32, 128) ||
        !encode_map_3d(&ma1, dt, 4, alo, k, n, 1, kp, n * kp, 32, 128))
      return TRNBLAS_ERR_ALIGN;
    p.in_fmt = kFmtTF32;
    const long long T = ceil_div(n, 256);
    if (use_pair_gemm(1, n, n, k) && T * (T + 1) / 2 >= num_sms() / 2 && p.c_mode != kCTrans) {
      // CTA pairs over the lower triangle's 256 x 256 tiles (the 3xTF32 MMAs
      // of a 128 x 128 tile are shared-memory bound); the pair epilogue
      // writes whole tiles (C read in place, lower storage), then the strictly
      // upper triangle is mirrored from the lower one in a second pass
      p.tiles_m = p.tiles_n = static_cast<int>(T);
      p.num_tiles = static_cast<int>(T * (T + 1) / 2);
      if (int rc = launch_gemm_pair<kTF32x3, 3>(ma0, ma1, ma0, ma1, p, stream)) return rc;
      const dim3 grid(static_cast<unsigned>(ceil_div(n, 32)), static_cast<unsigned>(ceil_div(n, 32)), 1);
      syrk_mirror_kernel<float><<<grid, dim3(32, 8), 0, stream>>>(static_cast<float*>(D), ldd, static_cast<int>(n));
      cudaError_t e = cudaGetLastError();
      return e == cudaSuccess ? TRNBLAS_OK : cuda_fail(e, "syrk mirror kernel launch");
    }
    return launch_gemm<kTF32x3, 128, 3>(ma0, ma1, ma0, ma1, p, stream);
  }
  const auto dt = map_dtype(dtype);
  p.a_mn = p.b_mn = trans ? 1 : 0;
  p.in_fmt = dtype == TRNBLAS_BF16 ? kFmtBF16 : kFmtF16;
  const long long rows = trans ? k : n;
  const long long s2 = round_up(lda * rows, 8);
  // 128 x 256 tiles over the lower triangle's column-block pairs: half the
  // operand bytes per MMA of 128 x 128 tiles, and half the tiles
  CUtensorMap mb0;
  const bool ok = trans ? encode_map_3d(&ma0, dt, 2, A, n, k, 1, lda, s2, 64, 64)
                        : (encode_map_3d(&ma0, dt, 2, A, k, n, 1, lda, s2, 64, 128) &&
                           encode_map_3d(&mb0, dt, 2, A, k, n, 1, lda, s2, 64, 256));
  if (!ok) return TRNBLAS_ERR_ALIGN;
  if (trans) mb0 = ma0;  // MN-major: 64 x 64 boxes for either operand
  p.mode = kModeSyrkWide;
  {
    const int T = p.tiles_m, h = T >> 1;
    p.num_tiles = (T & 1) ? (h + 1) * (h + 1) : h * (h + 1);
  }
  return launch_gemm<kF16, 256, 4>(ma0, ma0, mb0, mb0, p, stream);
}

}  // extern "C"
