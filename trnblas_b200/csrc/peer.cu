// Device memory shared between the processes of one node (one process per
// GPU) and copies over NVLink by the copy engines, for the SPMD GEMM whose
// operand exchange overlaps its tiles (trnblas_b200.parallel.gemm_2d).
//
//   trnblas_ipc_export     the CUDA IPC handle of the allocation holding
//                          `ptr`, and `ptr`'s offset in it (legacy IPC: no
//                          multicast object, no fabric handle);
//   trnblas_ipc_open       map a peer's allocation (cached per device and
//                          handle; at most kMaxMaps mappings, the oldest
//                          closed first) and return the peer's pointer;
//   trnblas_copy_async     one cudaMemcpyAsync, device to device (with a peer
//                          pointer as source the copy engines pull over
//                          NVLink; no SM is used);
//   trnblas_stream_signal  a 32-bit store of `value` to a device flag, ordered
//                          after the stream's earlier work (a stream memory
//                          operation, with the memory barrier that makes that
//                          work visible before the flag).
#include <cudaTypedefs.h>

#include <cstring>
#include <deque>
#include <mutex>
#include <string>

#include "runtime.hpp"

namespace tb {
namespace {

constexpr int kMaxMaps = 64;

struct Mapping {
  int device;
  cudaIpcMemHandle_t handle;
  void* base;
};

std::mutex g_peer_mu;
std::deque<Mapping> g_maps;
PFN_cuMemGetAddressRange_v3020 g_range = nullptr;
PFN_cuStreamWriteValue32_v11070 g_write32 = nullptr;

template <typename F>
bool driver_fn(const char* name, F& fn, int version) {
  if (fn) return true;
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPointByVersion(name, &p, version, cudaEnableDefault, &q) != cudaSuccess ||
      p == nullptr || q != cudaDriverEntryPointSuccess) {
    set_error(std::string(name) + " is not available from the driver");
    return false;
  }
  fn = reinterpret_cast<F>(p);
  return true;
}

}  // namespace
}  // namespace tb

using namespace tb;

extern "C" {

int trnblas_ipc_export(const void* ptr, void* handle, int64_t* offset) {
  if (!ptr || !handle || !offset) {
    set_error("trnblas_ipc_export: NULL argument");
    return TRNBLAS_ERR_ARG;
  }
  {
    std::lock_guard<std::mutex> lk(g_peer_mu);
    if (!driver_fn("cuMemGetAddressRange", g_range, 3020)) return TRNBLAS_ERR_CUDA;
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (g_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) {
    set_error("trnblas_ipc_export: pointer is not device memory of this process");
    return TRNBLAS_ERR_ARG;
  }
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcGetMemHandle");
  std::memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return TRNBLAS_OK;
}

int trnblas_ipc_open(const void* handle, int64_t offset, void** ptr) {
  if (!handle || !ptr || offset < 0) {
    set_error("trnblas_ipc_open: bad argument");
    return TRNBLAS_ERR_ARG;
  }
  const int dev = current_device();
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  std::lock_guard<std::mutex> lk(g_peer_mu);
  for (const Mapping& m : g_maps) {
    if (m.device == dev && std::memcmp(&m.handle, &h, sizeof(h)) == 0) {
      *ptr = static_cast<char*>(m.base) + offset;
      return TRNBLAS_OK;
    }
  }
  void* base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "cudaIpcOpenMemHandle");
  if (static_cast<int>(g_maps.size()) >= kMaxMaps) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(g_maps.front().device);
    cudaIpcCloseMemHandle(g_maps.front().base);
    cudaSetDevice(prev);
    g_maps.pop_front();
  }
  g_maps.push_back(Mapping{dev, h, base});
  *ptr = static_cast<char*>(base) + offset;
  return TRNBLAS_OK;
}

int trnblas_ipc_close_all(void) {
  std::lock_guard<std::mutex> lk(g_peer_mu);
  int prev = 0;
  cudaGetDevice(&prev);
  int rc = TRNBLAS_OK;
  for (const Mapping& m : g_maps) {
    cudaSetDevice(m.device);
    const cudaError_t e = cudaIpcCloseMemHandle(m.base);
    if (e != cudaSuccess) rc = cuda_fail(e, "cudaIpcCloseMemHandle");
  }
  g_maps.clear();
  cudaSetDevice(prev);
  return rc;
}

int trnblas_copy_async(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return TRNBLAS_OK;
  if (!dst || !src) {
    set_error("trnblas_copy_async: NULL pointer");
    return TRNBLAS_ERR_ARG;
  }
  const cudaError_t e =
      cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TRNBLAS_OK : cuda_fail(e, "cudaMemcpyAsync (device to device)");
}

int trnblas_stream_signal(int* flag, int value, void* stream) {
  if (!flag) {
    set_error("trnblas_stream_signal: NULL flag");
    return TRNBLAS_ERR_ARG;
  }
  {
    std::lock_guard<std::mutex> lk(g_peer_mu);
    if (!driver_fn("cuStreamWriteValue32", g_write32, 11070)) return TRNBLAS_ERR_CUDA;
  }
  const CUresult r = g_write32(static_cast<CUstream>(stream), reinterpret_cast<CUdeviceptr>(flag),
                               static_cast<cuuint32_t>(value), CU_STREAM_WRITE_VALUE_DEFAULT);
  if (r != CUDA_SUCCESS) {
    set_error("cuStreamWriteValue32 failed with code " + std::to_string(static_cast<int>(r)));
    return TRNBLAS_ERR_CUDA;
  }
  return TRNBLAS_OK;
}

}  // extern "C"
