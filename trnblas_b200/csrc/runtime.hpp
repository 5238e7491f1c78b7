// Host-side runtime shared by the C-ABI entry points: error reporting,
// per-device status word, SM count cache, and TMA tensor-map encoding through
// the driver entry point (no link-time dependency on libcuda).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/trnblas_b200.h"

namespace tb {

// Thread-local last error message (trnblas_last_error).
void set_error(const std::string& msg);
const char* last_error();

// Record a CUDA runtime failure; returns TRNBLAS_ERR_CUDA.
int cuda_fail(cudaError_t e, const char* what);

// Per-device kernel status word (device memory, zero when healthy).
int* status_word();            // current device; nullptr on failure (error set)
int num_sms();                 // current device
// A zeroed (stream-ordered) counter for one launch's tile-wave
// synchronisation on the current device; nullptr if unavailable.
int* wave_counter(cudaStream_t stream);
int current_device();

// Encode a 3-D tiled tensor map with the 128-byte swizzle. dims/strides are in
// elements (innermost first); strides for dims 1 and 2 are converted to bytes.
// Returns false (error set) when the driver rejects it or an alignment rule
// fails.
bool encode_map_3d(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* base,
                   uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1, uint64_t s2,
                   uint32_t box0, uint32_t box1);

inline long long ceil_div(long long a, long long b) { return (a + b - 1) / b; }
inline long long round_up(long long a, long long b) { return ceil_div(a, b) * b; }

// General tiled map: rank 1..5, given swizzle (CU_TENSOR_MAP_SWIZZLE_*);
// box0 * esize must equal the swizzle span (or be a multiple of 16 bytes
// without swizzle). Strides are in elements for dims 1..rank-1.
bool encode_map(CUtensorMap* map, CUtensorMapDataType dt, int esize, const void* base, int rank,
                const uint64_t* dims, const uint64_t* strides_elems, const uint32_t* box,
                CUtensorMapSwizzle swizzle);

// Kernel wait bound in ns (TRNBLAS_B200_WAIT_NS overrides; tests shorten it).
unsigned long long wait_timeout_ns();

}  // namespace tb
