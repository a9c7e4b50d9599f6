/*
 * C ABI of libgemm3_b200_cublaslt.so: the NVFP4 GEMM of nvfp4_gemm.h computed by cuBLASLt on this
 * GPU. A vendor baseline and a second implementation to compare against; not part of the
 * gemm3_b200 compute path. Replaces, for B200, the reference's cuBLASLt benchmark adapter
 * (benchmarks/cublaslt_lib.cu:9-69), which is built for the reference's GPU.
 *
 * Same operand formats as nvfp4_gemm_run (packed E2M1 [rows, K/2] row-major, 128x4 swizzled
 * UE4M3 scales, C [M, N] row-major FP16/BF16).
 */
#ifndef GEMM3_B200_NVFP4_CUBLASLT_H_
#define GEMM3_B200_NVFP4_CUBLASLT_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  NVFP4_CUBLASLT_OK = 0,
  NVFP4_CUBLASLT_ERR_INVALID_VALUE = 1,
  NVFP4_CUBLASLT_ERR_CUDA = 4,
  NVFP4_CUBLASLT_ERR_CUBLAS = 7,   /* see nvfp4_cublaslt_last_status() */
  NVFP4_CUBLASLT_ERR_NO_ALGO = 8   /* cuBLASLt offers no algorithm for this problem */
};
enum { NVFP4_CUBLASLT_F16 = 0, NVFP4_CUBLASLT_BF16 = 1 };

/*
 * C = alpha * dequant(A) . dequant(B)^T with cuBLASLt (FP32 accumulation). alpha is a host value.
 * `workspace` (device, may be NULL with workspace_bytes 0) bounds the algorithms considered.
 * The first call for a shape creates the handle and plan (host allocations inside cuBLASLt);
 * requires N % 64 == 0 and K % 64 == 0.
 */
int nvfp4_cublaslt_gemm(const void* a, const void* b, const void* sfa, const void* sfb, void* c, float alpha,
                        int64_t m, int64_t n, int64_t k, int32_t out_dtype, void* workspace,
                        int64_t workspace_bytes, void* stream);

/* The most recent failing cuBLASLt call on this thread: 100 * (its source line in the adapter)
 * + its cublasStatus_t. */
int32_t nvfp4_cublaslt_last_status(void);

#ifdef __cplusplus
}
#endif

#endif /* GEMM3_B200_NVFP4_CUBLASLT_H_ */
