// cuBLAS for the plain GEMMs of the library (weight gradients and hoisted products of the grid
// layer, the per-tick projections of the FLB cell path): one handle per host thread and device,
// bound to the caller's stream and to a workspace carved from the caller's buffer.
#pragma once
#include <cublas_v2.h>

#include <string>

#include "common.cuh"

namespace flb {

struct BlasHandle {
  cublasHandle_t h = nullptr;
  int dev = -1;
};
// slot 0: the caller's stream; slot 1: a library side stream running concurrently with it
inline thread_local BlasHandle t_blas_handle[2];

inline int blas(cudaStream_t s, void* ws, size_t ws_bytes, cublasHandle_t* out, int slot = 0) {
  int dev = 0;
  cudaGetDevice(&dev);
  BlasHandle& bh = t_blas_handle[slot];
  if (bh.h == nullptr || bh.dev != dev) {
    if (bh.h != nullptr) cublasDestroy(bh.h);
    bh.h = nullptr;
    if (cublasCreate(&bh.h) != CUBLAS_STATUS_SUCCESS) return fail(FLB_ERR_CUDA, "cublasCreate failed");
    bh.dev = dev;
  }
  if (cublasSetStream(bh.h, s) != CUBLAS_STATUS_SUCCESS)
    return fail(FLB_ERR_CUDA, "cublasSetStream failed");
  if (cublasSetWorkspace(bh.h, ws, ws_bytes) != CUBLAS_STATUS_SUCCESS)
    return fail(FLB_ERR_CUDA, "cublasSetWorkspace failed");
  *out = bh.h;
  return FLB_OK;
}

// Row-major C[M x N] (+)= op(A)[M x K] . op(B)[K x N], bf16 inputs, fp32 accumulation, output
// in `ctype` (fp32 by default), batched with element strides sA, sB, sC.
inline int gemm_rm(cublasHandle_t h, bool ta, bool tb, int M, int N, int K, const void* A, int lda,
                   long long sA, const void* Bm, int ldb, long long sB, void* Cm, int ldc,
                   long long sC, int batch, float beta, cudaDataType ctype = CUDA_R_32F) {
  const float alpha = 1.f;
  cublasStatus_t st = cublasGemmStridedBatchedEx(
      h, tb ? CUBLAS_OP_T : CUBLAS_OP_N, ta ? CUBLAS_OP_T : CUBLAS_OP_N, N, M, K, &alpha, Bm,
      CUDA_R_16BF, ldb, sB, A, CUDA_R_16BF, lda, sA, &beta, Cm, ctype, ldc, sC, batch,
      CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
  if (st != CUBLAS_STATUS_SUCCESS)
    return fail(FLB_ERR_CUDA, "cublasGemmStridedBatchedEx failed (" + std::to_string((int)st) + ")");
  return FLB_OK;
}

}  // namespace flb
