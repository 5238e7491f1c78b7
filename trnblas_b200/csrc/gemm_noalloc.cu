// An fp32 GEMM entry point that allocates nothing.
//
// Some callers cannot allocate device memory at the point where they need a
// product: a plugin running inside a host application whose memory manager
// owns every device allocation, or a latency-critical loop in which
// cudaMalloc (which can synchronise the device and stall other streams) is
// not allowed. trnblas_gemm's fp32 path needs scratch for its 3xTF32 operand
// split (a pass that writes hi / lo planes before the GEMM kernel reads
// them; only K-major operands the TMA can read, with the split fused into the
// kernel by TRNBLAS_B200_TF32_FUSED=1, go without); this variant takes that
// scratch from a fixed array compiled into the library instead of from the
// caller.
//
// The array lives for as long as the library is loaded, on every GPU that
// loads it: kNoAllocScratchBytes (64 MiB) per device. Problems whose split
// planes do not fit are rejected with TRNBLAS_ERR_WORKSPACE. Every call on a
// device shares the one array and it keeps the contents of the last call; the
// split kernel rewrites every byte the GEMM reads (including the zero K
// padding), so nothing has to start at zero. Calls that can run at the same
// time on one GPU (different streams, or different host threads) race on the
// array: serialise them, e.g. on one stream.
//
// Host code cannot use the array's name as a device address, so the first
// call on each device looks the address up with cudaGetSymbolAddress (with
// that device current) and caches it. Make that first call on a device before
// any stream capture.
#include <mutex>
#include <string>

#include "runtime.hpp"

namespace tb {
namespace {

constexpr size_t kNoAllocScratchBytes = 64ull << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDev = 64;
std::mutex g_na_mu;
void* g_na_ptr[kMaxDev] = {};

// The scratch array's device address on the current device (looked up once).
void* noalloc_scratch() {
  const int d = current_device();
  if (d < 0 || d >= kMaxDev) {
    set_error("trnblas_gemm_f32_noalloc: device index out of range");
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_na_mu);
  if (!g_na_ptr[d]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      cuda_fail(e, "trnblas_gemm_f32_noalloc: cudaGetSymbolAddress(scratch)");
      return nullptr;
    }
    g_na_ptr[d] = p;
  }
  return g_na_ptr[d];
}

}  // namespace
}  // namespace tb

extern "C" {

int trnblas_gemm_f32_noalloc(int64_t M, int64_t N, int64_t K, float alpha, const float* A,
                             int64_t lda, int transA, const float* B, int64_t ldb, int transB,
                             float beta, const float* C, int64_t ldc, float* D, int64_t ldd,
                             void* stream) {
  if (M < 0 || N < 0 || K < 0) {
    tb::set_error("trnblas_gemm_f32_noalloc: negative size");
    return TRNBLAS_ERR_ARG;
  }
  const long long lim = (1ll << 31) - 1;
  if (M > lim || N > lim || K > (lim & ~3ll)) {
    tb::set_error("trnblas_gemm_f32_noalloc: size exceeds the element limit per dimension "
                  "(2^31-1; K: 2^31-4)");
    return TRNBLAS_ERR_ARG;
  }
  // The split planes take 8 * (M + N) * round_up(K, 4) bytes (plus at most
  // 1 KiB of alignment padding). Compared by division first, so that sizes
  // near the dimension limits cannot overflow the product into a small value.
  const long long kp = tb::round_up(K > 0 ? K : 1, 4);
  if (K > 0 && M > 0 && N > 0 &&
      M + N > static_cast<long long>(tb::kNoAllocScratchBytes / 8) / kp) {
    tb::set_error("trnblas_gemm_f32_noalloc: the problem needs more than the built-in " +
                  std::to_string(tb::kNoAllocScratchBytes) +
                  " scratch bytes (8 * (M + N) * round_up(K, 4) must fit); use trnblas_gemm "
                  "with a caller workspace");
    return TRNBLAS_ERR_WORKSPACE;
  }
  // Leading dimensions as trnblas_gemm checks them, before the scratch
  // address lookup (which needs the device) so a bad call fails as ERR_ARG.
  if (M > 0 && N > 0 && K > 0 &&
      (lda < (transA ? M : K) || ldb < (transB ? K : N) || ldd < N ||
       (C && beta != 0.0f && ldc < N))) {
    tb::set_error("trnblas_gemm_f32_noalloc: lda/ldb/ldc/ldd smaller than the stored row length");
    return TRNBLAS_ERR_ARG;
  }
  const size_t need = trnblas_gemm_workspace_size(TRNBLAS_F32, 1, M, N, K, 0, 0);
  if (need > tb::kNoAllocScratchBytes) {
    tb::set_error("trnblas_gemm_f32_noalloc: the problem needs " + std::to_string(need) +
                  " scratch bytes, above the built-in " +
                  std::to_string(tb::kNoAllocScratchBytes) +
                  " (2 * (M + N) * round_up(K, 4) * 4 must fit); use trnblas_gemm with a "
                  "caller workspace");
    return TRNBLAS_ERR_WORKSPACE;
  }
  void* ws = nullptr;
  if (need > 0) {
    ws = tb::noalloc_scratch();
    if (!ws) return TRNBLAS_ERR_CUDA;
  }
  return trnblas_gemm(TRNBLAS_F32, 1, M, N, K, alpha, A, lda, 0, transA, B, ldb, 0, transB, beta,
                      C, ldc, 0, D, ldd, 0, ws, need, stream);
}

}  // extern "C"
