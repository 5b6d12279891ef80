// GEMMs of the general route: the stem projection, the drive projection and the
// synthesis of every request the fused route does not take.  gemm_rows runs
// them on this library's tcgen05 row GEMMs (rowgemm.cuh: bf16 x bf16 for bf16
// operands, split-bf16 x3 -- fp32-level accuracy -- for fp32 operands):
//   * the warp-specialised TMA pipeline (rowgemm_ws_kernel) when the operands
//     are TMA-addressable, n <= 256 and B fits in shared memory -- every
//     BASELINE configuration;
//   * the one-tile-at-a-time kernel (rowgemm_kernel) for other n, k <= 128
//     (unaligned or odd-pitch operands);
//   * cuBLAS otherwise (fp32 requests in CUBLAS_COMPUTE_32F, bf16 requests on
//     TF32 or bf16 tensor cores), or when lnet_b200_set_gemm_backend(1) asks.
#pragma once

#include <cublas_v2.h>

#include <mutex>
#include <unordered_map>

#include "common.cuh"
#include "rowgemm.cuh"

namespace lnet {

// One handle per (host thread, device), created on first use and kept.
inline int blas_handle(cublasHandle_t *out) {
  thread_local std::unordered_map<int, cublasHandle_t> handles;
  int dev = 0;
  LNET_TRY(cuda_check(cudaGetDevice(&dev), "cudaGetDevice"));
  auto it = handles.find(dev);
  if (it == handles.end()) {
    cublasHandle_t h = nullptr;
    if (cublasCreate(&h) != CUBLAS_STATUS_SUCCESS)
      return fail(LNET_ERR_CUDA, "cublasCreate failed on device %d", dev);
    it = handles.emplace(dev, h).first;
  }
  *out = it->second;
  return LNET_OK;
}

// C[rows, n] (row-major, leading dimension ldc) = A[rows, k] (row-major, lda) * B^T + beta C,
// with element (j, kk) of B at Bm[j * ldbn + kk * ldbk] (one of ldbn, ldbk is 1).
// C of type `tc` (fp32, or bf16 for bf16 A and B); accumulation is fp32.
inline int gemm_rows_t(cudaStream_t st, const void *A, cudaDataType ta, int64_t lda,
                       const void *Bm, cudaDataType tb, int64_t ldbn, int64_t ldbk, void *C,
                       cudaDataType tc, int64_t ldc, int64_t rows, int n, int k, bool tf32,
                       const char *what, float beta = 0.f) {
  if (rows == 0 || n == 0) return LNET_OK;
  if (rows > INT32_MAX) return fail(LNET_ERR_UNSUPPORTED, "%s: %lld rows", what, (long long)rows);
  cublasHandle_t h;
  LNET_TRY(blas_handle(&h));
  if (cublasSetStream(h, st) != CUBLAS_STATUS_SUCCESS)
    return fail(LNET_ERR_CUDA, "cublasSetStream failed");
  // column-major view: C^T (n x rows) = B (n x k) * A^T (k x rows)
  cublasOperation_t op_b;
  int ld_b;
  if (ldbn == 1) {
    op_b = CUBLAS_OP_N;
    ld_b = (int)ldbk;
  } else {
    op_b = CUBLAS_OP_T;
    ld_b = (int)ldbn;
  }
  const float alpha = 1.f;
  const cublasStatus_t s = cublasGemmEx(
      h, op_b, CUBLAS_OP_N, n, (int)rows, k, &alpha, Bm, tb, ld_b, A, ta, (int)lda, &beta, C,
      tc, (int)ldc, tf32 ? CUBLAS_COMPUTE_32F_FAST_TF32 : CUBLAS_COMPUTE_32F,
      CUBLAS_GEMM_DEFAULT);
  if (s != CUBLAS_STATUS_SUCCESS) return fail(LNET_ERR_CUDA, "%s: cublasGemmEx status %d", what, (int)s);
  return after_library(what);
}

// Whether gemm_rows may use rowgemm (process-wide; tests compare both).
inline bool &rowgemm_enabled() {
  static bool on = true;
  return on;
}

inline int gemm_rows(cudaStream_t st, const void *A, cudaDataType ta, int64_t lda, const void *Bm,
                     cudaDataType tb, int64_t ldbn, int64_t ldbk, float *C, int64_t ldc,
                     int64_t rows, int n, int k, bool tf32, const char *what,
                     float beta = 0.f, uint32_t *status = nullptr) {
  if (rowgemm_enabled() && rows > 0 && (beta == 0.f || beta == 1.f) &&
      rowgemm_ws_supported(A, ta, tb, lda, n, k, C, ldc))
    return rowgemm_ws(st, A, ta, lda, Bm, ldbn, ldbk, C, ldc, rows, n, k, beta, status, what);
  if (rowgemm_enabled() && rows > 0 && rowgemm_supported(ta, tb, n, k))
    return rowgemm(st, A, ta, lda, Bm, ldbn, ldbk, C, ldc, rows, n, k, beta, status, what);
  return gemm_rows_t(st, A, ta, lda, Bm, tb, ldbn, ldbk, C, CUDA_R_32F, ldc, rows, n, k, tf32,
                     what, beta);
}

}  // namespace lnet
