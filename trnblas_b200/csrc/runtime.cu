// Host runtime: errors, per-device status word, SM counts, tensor maps, and
// the bounded-wait self-test kernel.
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstdlib>
#include <atomic>
#include <mutex>
#include <string>

#include "common.cuh"
#include "runtime.hpp"

namespace tb {

namespace {
thread_local std::string g_last_error;

// One status word per device. Device code writes it with atomicCAS on the
// first failure; trnblas_device_status reads and clears it.
__device__ int g_status_word;

// Wave counters of the GEMM's tile-walk synchronisation, one per launch slot
// (slots rotate, so launches in flight on different streams count apart).
constexpr int kWaveSlots = 64;
__device__ int g_wave_ctr[kWaveSlots];
std::atomic<unsigned> g_wave_next{0};

constexpr int kMaxDevices = 64;
std::mutex g_mu;
int* g_status_ptr[kMaxDevices] = {};
int g_sms[kMaxDevices] = {};
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

bool load_encode() {
  if (g_encode) return true;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || fn == nullptr || q != cudaDriverEntryPointSuccess) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return false;
  }
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return true;
}
}  // namespace

void set_error(const std::string& msg) { g_last_error = msg; }
const char* last_error() { return g_last_error.c_str(); }

int cuda_fail(cudaError_t e, const char* what) {
  set_error(std::string(what) + ": " + cudaGetErrorString(e));
  return TRNBLAS_ERR_CUDA;
}

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

int* status_word() {
  const int d = current_device();
  if (d < 0 || d >= kMaxDevices) {
    set_error("device index out of range");
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_status_ptr[d]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_status_word);
    if (e != cudaSuccess) {
      cuda_fail(e, "cudaGetSymbolAddress(status word)");
      return nullptr;
    }
    g_status_ptr[d] = static_cast<int*>(p);
  }
  return g_status_ptr[d];
}

int* wave_counter(cudaStream_t stream) {
  const int d = current_device();
  if (d < 0 || d >= kMaxDevices) return nullptr;
  static int* base[kMaxDevices] = {};
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!base[d]) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_wave_ctr) != cudaSuccess) return nullptr;
      base[d] = static_cast<int*>(p);
    }
  }
  int* c = base[d] + (g_wave_next.fetch_add(1) % kWaveSlots);
  if (cudaMemsetAsync(c, 0, sizeof(int), stream) != cudaSuccess) return nullptr;
  return c;
}

int num_sms() {
  const int d = current_device();
  if (d < 0 || d >= kMaxDevices) return 1;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_sms[d]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
    g_sms[d] = n > 0 ? n : 1;
  }
  return g_sms[d];
}

unsigned long long wait_timeout_ns() {
  static unsigned long long v = [] {
    const char* s = std::getenv("TRNBLAS_B200_WAIT_NS");
    if (s && *s) {
      unsigned long long x = std::strtoull(s, nullptr, 10);
      if (x > 0) return x;
    }
    return kDefaultTimeoutNs;
  }();
  return v;
}

bool encode_map_3d(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* base,
                   uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1, uint64_t s2,
                   uint32_t box0, uint32_t box1) {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!load_encode()) return false;
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) {
    set_error("operand base address is not 16-byte aligned");
    return false;
  }
  const uint64_t s1b = s1 * static_cast<uint64_t>(esize);
  const uint64_t s2b = s2 * static_cast<uint64_t>(esize);
  if ((s1b & 15) != 0 || (s2b & 15) != 0) {
    set_error("operand row / batch stride is not a multiple of 16 bytes");
    return false;
  }
  if (d0 == 0 || d1 == 0 || d2 == 0 || box0 == 0 || box1 == 0 || box0 > 256 || box1 > 256 ||
      box0 * static_cast<uint32_t>(esize) != 128) {
    set_error("bad tensor map geometry");
    return false;
  }
  if (s1b >= (1ull << 40) || s2b >= (1ull << 40)) {
    set_error("operand stride too large for TMA");
    return false;
  }
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1b, s2b};
  cuuint32_t box[3] = {box0, box1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed with code " + std::to_string(static_cast<int>(r)));
    return false;
  }
  return true;
}

bool encode_map(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* base, int rank,
                const uint64_t* dims, const uint64_t* strides_elems, const uint32_t* box,
                CUtensorMapSwizzle swizzle) {
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!load_encode()) return false;
  }
  if (rank < 1 || rank > 5) {
    set_error("bad tensor map rank");
    return false;
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) {
    set_error("operand base address is not 16-byte aligned");
    return false;
  }
  const uint32_t span = swizzle == CU_TENSOR_MAP_SWIZZLE_128B ? 128
                        : swizzle == CU_TENSOR_MAP_SWIZZLE_64B ? 64
                        : swizzle == CU_TENSOR_MAP_SWIZZLE_32B ? 32 : 0;
  if (span ? box[0] * static_cast<uint32_t>(esize) != span
           : (box[0] * static_cast<uint32_t>(esize)) % 16 != 0) {
    set_error("tensor map inner box does not match the swizzle span");
    return false;
  }
  cuuint64_t d[5];
  cuuint64_t st[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    if (dims[i] == 0 || box[i] == 0 || box[i] > 256) {
      set_error("bad tensor map geometry");
      return false;
    }
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) {
    const uint64_t b = strides_elems[i] * static_cast<uint64_t>(esize);
    if ((b & 15) != 0 || b >= (1ull << 40)) {
      set_error("tensor map stride is not a multiple of 16 bytes (or too large)");
      return false;
    }
    st[i] = b;
  }
  CUresult r = g_encode(map, dt, static_cast<cuuint32_t>(rank), const_cast<void*>(base), d, st,
                        bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed with code " + std::to_string(static_cast<int>(r)));
    return false;
  }
  return true;
}

// One CTA waits on an mbarrier whose phase never completes, gives up after
// `timeout_ns`, records kTimeoutTest and returns.
__global__ void wait_selftest_kernel(int* status, unsigned long long timeout_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const Abort ab{&flag, status, timeout_ns};
    mbar_wait(&bar, 0, ab, kTimeoutTest);
  }
  __syncthreads();
}

}  // namespace tb

extern "C" {

int trnblas_version(void) { return 100; }

const char* trnblas_last_error(void) { return tb::last_error(); }

int trnblas_device_status(int device, int* status) {
  if (!status) {
    tb::set_error("status pointer is NULL");
    return TRNBLAS_ERR_ARG;
  }
  int prev = 0;
  cudaGetDevice(&prev);
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return tb::cuda_fail(e, "cudaSetDevice");
  int* w = tb::status_word();
  int rc = TRNBLAS_OK;
  if (!w) {
    rc = TRNBLAS_ERR_CUDA;
  } else {
    e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
      rc = tb::cuda_fail(e, "cudaDeviceSynchronize");
    } else {
      int v = 0;
      e = cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost);
      if (e == cudaSuccess) e = cudaMemset(w, 0, sizeof(int));
      if (e != cudaSuccess) rc = tb::cuda_fail(e, "status word copy");
      *status = v;
    }
  }
  cudaSetDevice(prev);
  return rc;
}

int trnblas_wait_selftest(unsigned long long timeout_ns, void* stream) {
  int* w = tb::status_word();
  if (!w) return TRNBLAS_ERR_CUDA;
  if (timeout_ns == 0 || timeout_ns > 10000000000ull) {
    tb::set_error("selftest timeout must be in (0, 10 s]");
    return TRNBLAS_ERR_ARG;
  }
  tb::wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(w, timeout_ns);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return tb::cuda_fail(e, "wait_selftest launch");
  return TRNBLAS_OK;
}

}  // extern "C"
