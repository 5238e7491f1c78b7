/*
 * trnblas_b200 -- C ABI of the B200 (sm_100a) GEMM-family hot path.
 *
 * Plain pointers, sizes and a CUDA stream handle (passed as void*); no torch
 * types. Every entry point is stream-ordered and asynchronous, reads its
 * inputs without modifying them, writes only the output it is given, and
 * returns TRNBLAS_OK or a nonzero status with a message from
 * trnblas_last_error() (thread-local). Device-side failures (a bounded wait
 * that ran out) are recorded in a per-device status word read by
 * trnblas_device_status().
 *
 * Matrix conventions are row-major, BLAS-style: for transX == 0, X is stored
 * rows x cols of op(X) with row stride ldX (elements); for transX != 0 it is
 * stored transposed. Batched operands carry a batch stride in elements; 0
 * broadcasts one matrix over the batch.
 *
 * Each entry point replaces one kernel boundary of the reference trnblas
 * (trnsci/trnblas 0.13.0), cited beside it.
 */
#ifndef TRNBLAS_B200_H_
#define TRNBLAS_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define TRNBLAS_API __attribute__((visibility("default")))
#else
#define TRNBLAS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum trnblas_status {
  TRNBLAS_OK = 0,
  TRNBLAS_ERR_ARG = 1,      /* bad size, stride, dtype or flag */
  TRNBLAS_ERR_ALIGN = 2,    /* pointer / stride breaks the 16-byte TMA rule */
  TRNBLAS_ERR_CUDA = 3,     /* CUDA runtime / driver call failed */
  TRNBLAS_ERR_WORKSPACE = 4 /* workspace missing or too small */
};

enum trnblas_dtype {
  TRNBLAS_F32 = 0,  /* fp32 API, computed as 3xTF32 on the tensor cores */
  TRNBLAS_BF16 = 1, /* bf16 in/out, fp32 accumulate */
  TRNBLAS_F16 = 2,  /* fp16 in/out, fp32 accumulate */
  TRNBLAS_F64 = 3   /* fp64 (Ozaki entry points only) */
};

/* Library version, as 10000*major + 100*minor + patch. */
TRNBLAS_API int trnblas_version(void);

/* Last error message of the calling thread ("" when none). */
TRNBLAS_API const char* trnblas_last_error(void);

/* Synchronise `device`, read its kernel status word into *status (0 when
 * healthy, else the first failure code) and clear it. */
TRNBLAS_API int trnblas_device_status(int device, int* status);

/* Bytes of workspace trnblas_gemm needs (0 for bf16/fp16). */
TRNBLAS_API size_t trnblas_gemm_workspace_size(int dtype, int64_t batch, int64_t M, int64_t N, int64_t K,
                                   int64_t strideA, int64_t strideB);

/*
 * D[b] = alpha * op(A[b]) @ op(B[b]) + beta * C[b],  b = 0 .. batch-1.
 * op(A) is M x K, op(B) is K x N, C and D are M x N (C may be NULL or
 * beta == 0, then C is not read: NaN in C does not propagate).
 * Replaces the GEMM kernel boundary of the reference:
 *   trnblas/level3.py:69-109 (gemm), :112-134 (batched_gemm) and
 *   trnblas/nki/dispatch.py:1527-1551 (nki_gemm), :1385-1427
 *   (nki_batched_gemm), :2441-2511 (_nki_gemm_impl), the NKI kernels
 *   dispatch.py:3324-3561 and 3723-3760.
 * D must not overlap A, B or C.
 */
TRNBLAS_API int trnblas_gemm(int dtype, int64_t batch, int64_t M, int64_t N, int64_t K, float alpha,
                 const void* A, int64_t lda, int64_t strideA, int transA, const void* B,
                 int64_t ldb, int64_t strideB, int transB, float beta, const void* C,
                 int64_t ldc, int64_t strideC, void* D, int64_t ldd, int64_t strideD,
                 void* workspace, size_t workspace_bytes, void* stream);

/*
 * fp32 GEMM (no batch) that allocates nothing: D = alpha * op(A) @ op(B) +
 * beta * C with the argument meanings of trnblas_gemm, for callers that may
 * not allocate device memory when they multiply (plugins whose host owns all
 * device memory, loops where cudaMalloc's device synchronisation is not
 * allowed). Its scratch for the 3xTF32 split planes (written by the split
 * pass before the GEMM kernel) is a 64 MiB array built into the library and held on
 * every GPU that loads it; problems with 2 * (M + N) * round_up(K, 4) * 4
 * bytes of split planes above that are rejected (TRNBLAS_ERR_WORKSPACE).
 * The first call on a device looks up the array's address (make it before any
 * stream capture). All calls on a device share the array: calls that may
 * overlap on the GPU (other streams, other threads) race and must be
 * serialised. No counterpart in the reference.
 */
TRNBLAS_API int trnblas_gemm_f32_noalloc(int64_t M, int64_t N, int64_t K, float alpha, const float* A,
                             int64_t lda, int transA, const float* B, int64_t ldb, int transB,
                             float beta, const float* C, int64_t ldc, float* D, int64_t ldd,
                             void* stream);

/*
 * trnblas_gemm with one triangular operand (trmm): tri = 1 / 2 when op(A) is
 * lower / upper triangular, 3 / 4 when op(B) is, holding exact zeros outside
 * the triangle. Each output tile multiplies only the K blocks its rows (A) or
 * columns (B) reach, about half the products of the dense GEMM; tri = 0 is
 * trnblas_gemm. Replaces the triangular multiply of the reference's trmm
 * (trnblas/level3.py:383-417), which multiplies the masked triangle densely.
 */
TRNBLAS_API int trnblas_gemm_tri(int dtype, int64_t batch, int64_t M, int64_t N, int64_t K, float alpha,
                     const void* A, int64_t lda, int64_t strideA, int transA, const void* B,
                     int64_t ldb, int64_t strideB, int transB, float beta, const void* C,
                     int64_t ldc, int64_t strideC, void* D, int64_t ldd, int64_t strideD, int tri,
                     void* workspace, size_t workspace_bytes, void* stream);

/*
 * Symmetric multiply: D = alpha * S @ B + beta * C (side_right = 0; S is
 * M x M, B is M x N) or alpha * B @ S + beta * C (side_right = 1; S is
 * N x N), S given by the stored triangle of A (row-major, leading dimension
 * lda; uplo_lower = 1: the lower triangle, 0: the upper; the other triangle
 * is never read). B, C, D row-major with their leading dimensions. fp32: the
 * 3xTF32 split pass reads S from the triangle itself (no full S is formed),
 * then the GEMM kernel. bf16 / fp16: one pass writes the full S into the
 * workspace, then the GEMM kernel. Workspace: trnblas_symm_workspace_size.
 * Replaces the reference's symm (trnblas/level3.py:196-240), which forms the
 * full symmetric matrix with three elementwise passes before a dense GEMM.
 */
TRNBLAS_API size_t trnblas_symm_workspace_size(int dtype, int side_right, int64_t M, int64_t N);
TRNBLAS_API int trnblas_symm(int dtype, int side_right, int uplo_lower, int64_t M, int64_t N,
                 float alpha, const void* A, int64_t lda, const void* B, int64_t ldb, float beta,
                 const void* C, int64_t ldc, void* D, int64_t ldd, void* workspace,
                 size_t workspace_bytes, void* stream);

/*
 * bf16 / fp16 trnblas_gemm (no workspace) whose operands arrive while it runs:
 * rows [s * shard_rows, (s + 1) * shard_rows) of op(A) may be read once
 * ready[s] has reached `epoch` (wrap-safe), batch entry b of op(B) once
 * ready[ready_b0 + b] has; the tile walk starts at row rot_rows of op(A) and
 * batch entry rot_b (so tiles whose operands are already in place go
 * first). The flags are device ints written by the caller's copies, e.g.
 * trnblas_copy_async followed by trnblas_stream_signal on a copy stream.
 * Every wait is bounded (the status word records a timeout). shard_rows and
 * rot_rows are multiples of 256. Replaces the gather-then-multiply step of
 * the reference's 2-D SPMD GEMM primitives (trnblas/parallel.py:81-120,
 * all_gather_rows + gemm_row/col_parallel) for trnblas_b200.parallel.gemm_2d.
 */
TRNBLAS_API int trnblas_gemm_ready(int dtype, int64_t batch, int64_t M, int64_t N, int64_t K, float alpha,
                       const void* A, int64_t lda, int64_t strideA, int transA, const void* B,
                       int64_t ldb, int64_t strideB, int transB, float beta, const void* C,
                       int64_t ldc, int64_t strideC, void* D, int64_t ldd, int64_t strideD,
                       const int* ready, int epoch, int64_t shard_rows, int ready_b0,
                       int64_t rot_rows, int rot_b, void* stream);

/*
 * Device memory of another process of this node (one process per GPU):
 * trnblas_ipc_export writes the 64-byte CUDA IPC handle of the allocation
 * holding `ptr` and ptr's offset in it; trnblas_ipc_open maps a peer's
 * allocation (cached per device and handle, at most 64 mappings) and returns
 * the peer pointer; trnblas_ipc_close_all unmaps them. Legacy CUDA IPC (no
 * multicast object). The all-gather step of the reference's SPMD GEMM
 * (trnblas/parallel.py:81-86, all_gather_rows) becomes copies from these
 * pointers.
 */
TRNBLAS_API int trnblas_ipc_export(const void* ptr, void* handle, int64_t* offset);
TRNBLAS_API int trnblas_ipc_open(const void* handle, int64_t offset, void** ptr);
TRNBLAS_API int trnblas_ipc_close_all(void);

/* One device-to-device cudaMemcpyAsync (a peer pointer as source: the copy
 * engines pull over NVLink, no SM is used). */
TRNBLAS_API int trnblas_copy_async(void* dst, const void* src, size_t bytes, void* stream);

/* Store `value` to the device int *flag once the stream's earlier work is
 * done and visible (a stream memory operation). */
TRNBLAS_API int trnblas_stream_signal(int* flag, int value, void* stream);

/* Bytes of workspace trnblas_syrk needs (0 for bf16/fp16). */
TRNBLAS_API size_t trnblas_syrk_workspace_size(int dtype, int64_t n, int64_t k);

/*
 * D = alpha * op(A) @ op(A)^T + beta * sym(C), full symmetric n x n result.
 * op(A) = A (n x k) when trans == 0, A^T (A stored k x n) otherwise.
 * c_uplo: 1 = only the lower triangle of C is referenced, 2 = only the upper;
 * 0 or beta == 0: C is not read. Only lower-triangle tiles are computed; each
 * value is stored at (r, c) and (c, r), so D is exactly symmetric.
 * Replaces trnblas/level3.py:243-295 (syrk), trnblas/nki/dispatch.py:1555-1594
 * (nki_syrk), :3202-3251 (_nki_syrk_impl), :3178-3199 (_symmetrize) and the
 * NKI kernel dispatch.py:4494-4544 (_syrk_kernel).
 */
TRNBLAS_API int trnblas_syrk(int dtype, int64_t n, int64_t k, float alpha, const void* A, int64_t lda,
                 int trans, float beta, const void* C, int64_t ldc, int c_uplo, void* D,
                 int64_t ldd, void* workspace, size_t workspace_bytes, void* stream);

/* Bytes of workspace trnblas_gemm_fp64 needs. */
TRNBLAS_API size_t trnblas_gemm_fp64_workspace_size(int64_t M, int64_t N, int64_t K, int slices);

/*
 * C = op(A) @ op(B) in fp64 by Ozaki splitting on the int8 tensor cores:
 * per-row (A) / per-column (B) power-of-two scaling, `slices` balanced 7-bit
 * integer digits (|d| <= 64) per operand, every diagonal s + t = d <= slices-1
 * of slice products summed exactly in int32, recombined in fp64 with the
 * exponents. A, B, C fp64 row-major (C is M x N, row stride ldc).
 * 1 <= slices <= 12. Operands must be finite (the caller checks).
 * Replaces trnblas/level3.py:137-193 (gemm_fp64), trnblas/nki/dispatch.py:958-980
 * (nki_gemm_fp64), trnblas/ozaki.py:514-565 (run) with :123-219 (split) and
 * :418-455 (combine), and the NKI kernels dispatch.py:3768-3918 (Ozaki GEMM)
 * and 3941-4356 (device split).
 */
TRNBLAS_API int trnblas_gemm_fp64(int64_t M, int64_t N, int64_t K, const double* A, int64_t lda, int transA,
                      const double* B, int64_t ldb, int transB, int slices, double* C,
                      int64_t ldc, void* workspace, size_t workspace_bytes, void* stream);

/*
 * The Ozaki split alone (for parity checks): digits (slices, R, ldd) int8 and
 * exponents (R,) int32 of the R x K operand X (element (r, k) at
 * X[r * rs + k * ks]), scaled per row r. Digit d_s(r, k) is the reference's
 * digit of trnblas/ozaki.py:123-219 (split, per="row"). Needs
 * 8 * R + 256 bytes of workspace.
 */
TRNBLAS_API int trnblas_ozaki_split(int64_t R, int64_t K, const double* X, int64_t rs, int64_t ks,
                        int slices, int8_t* digits, int64_t ldd, int32_t* exps,
                        void* workspace, size_t workspace_bytes, void* stream);

/* Bytes of workspace trnblas_pair_energy needs. */
TRNBLAS_API size_t trnblas_pair_energy_workspace_size(int64_t nocc, int64_t nvir, int64_t naux,
                                          int64_t pair_begin, int64_t pair_end);

/*
 * DF-MP2 pair energy over the occupied pairs i <= j with linear index
 * p = j (j + 1) / 2 + i in [pair_begin, pair_end):
 *   E = sum_p w_p sum_{a,b} T_ab (2 T_ab - T_ba) / (e_i + e_j - e_a - e_b),
 *   T = B_i B_j^T (nvir x nvir, contracted over naux), w_p = 1 (i == j) or 2.
 * B is (nocc, nvir, naux) fp32 contiguous, eps fp32. B is split per row
 * (i, a) into 4 int8 base-254 digit planes with a power-of-two exponent; T
 * keeps the slice products of diagonals <= 3 (10 products), the diagonal
 * elements of the i == j pairs come from exact fp64 row sums of squares. T is
 * formed tile by tile from exact int32 diagonal sums in TMEM (K chunks of at
 * most 33280 naux, whose folds are added in fp64) and reduced in the
 * epilogue in fp64; it never reaches HBM. naux <= 2^30. The fp64 result is
 * written to *energy (device pointer). Deterministic. Workspace holds the
 * digit planes once: about 4 * nocc * round_up(nvir, 128) * round_up(naux,
 * 64) bytes.
 * Replaces trnblas/nki/dispatch.py:2537-2569 (nki_batched_pair_energy),
 * :2768-2795 (_nki_pair_energy_sym_impl), trnblas/nki/multicore.py:212-289
 * (sym_rows / aten_rows) and the NKI kernel dispatch.py:4900-5001
 * (_pair_energy_sym_kernel).
 */
TRNBLAS_API int trnblas_pair_energy(int64_t nocc, int64_t nvir, int64_t naux, const float* B,
                        const float* eps_occ, const float* eps_vir, int64_t pair_begin,
                        int64_t pair_end, double* energy, void* workspace,
                        size_t workspace_bytes, void* stream);

/*
 * Self-test of the bounded-wait machinery: launches one CTA that waits on an
 * mbarrier nothing will complete, with a `timeout_ns` bound, and returns.
 * The status word then holds the test's timeout code (6). No fault, no hang.
 */
TRNBLAS_API int trnblas_wait_selftest(unsigned long long timeout_ns, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TRNBLAS_B200_H_ */
