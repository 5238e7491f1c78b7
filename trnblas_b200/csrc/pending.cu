// Entry points whose kernels are not built yet: they fail loudly.
#include "runtime.hpp"

extern "C" {
size_t trnblas_gemm_fp64_workspace_size(int64_t, int64_t, int64_t, int) { return 0; }
int trnblas_gemm_fp64(int64_t, int64_t, int64_t, const double*, int64_t, int, const double*,
                      int64_t, int, int, double*, int64_t, void*, size_t, void*) {
  tb::set_error("trnblas_gemm_fp64: not built yet");
  return TRNBLAS_ERR_ARG;
}
int trnblas_ozaki_split(int64_t, int64_t, const double*, int64_t, int64_t, int, int8_t*, int64_t,
                        int32_t*, void*) {
  tb::set_error("trnblas_ozaki_split: not built yet");
  return TRNBLAS_ERR_ARG;
}
size_t trnblas_pair_energy_workspace_size(int64_t, int64_t, int64_t, int64_t, int64_t) { return 0; }
int trnblas_pair_energy(int64_t, int64_t, int64_t, const float*, const float*, const float*,
                        int64_t, int64_t, double*, void*, size_t, void*) {
  tb::set_error("trnblas_pair_energy: not built yet");
  return TRNBLAS_ERR_ARG;
}
}
