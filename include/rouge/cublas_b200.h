/*
 * librouge_b200_cublas.so: the cuBLAS-API GEMM subset on the B200 kernels.
 *
 * The reference ships a cuBLAS shim (software/rouge-numerics/include/rouge/
 * cublas_shim.h, src/cublas_shim.cpp) that runs the public cuBLAS GEMM API
 * on its CPU GEMM, so that programs written against cuBLAS run unchanged.
 * This library exports the same API names with the same argument meaning
 * and status codes, computing on the sm_100a tensor-core kernels of
 * librouge_b200.so (through rouge_b200_gemm_colmajor). Device pointers are
 * used in place and calls are asynchronous on the handle's stream, as in
 * cuBLAS. Host pointers (the memory the reference's CPU shim works on) are
 * accepted too: those operands are copied to the device and the result
 * back, and the call returns when done.
 *
 * Covered: handle management, streams, pointer mode, cublasSgemm_v2 and
 * cublasSgemmStridedBatched (f32 on tf32 tensor cores with split operands,
 * f32-accurate), and cublasGemmEx for f16 / bf16 / e4m3 inputs with f32
 * output and int8 inputs with int32 output. Everything else is absent: a
 * program that needs it fails to link instead of computing something else.
 * Enum values are those of the public cuBLAS API.
 */
#pragma once

#include <driver_types.h>  /* cudaStream_t */
#include <library_types.h> /* cudaDataType_t (CUDA_R_32F, CUDA_R_16F, ...) */
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  CUBLAS_STATUS_SUCCESS = 0,
  CUBLAS_STATUS_NOT_INITIALIZED = 1,
  CUBLAS_STATUS_ALLOC_FAILED = 3,
  CUBLAS_STATUS_INVALID_VALUE = 7,
  CUBLAS_STATUS_ARCH_MISMATCH = 8,
  CUBLAS_STATUS_MAPPING_ERROR = 11,
  CUBLAS_STATUS_EXECUTION_FAILED = 13,
  CUBLAS_STATUS_INTERNAL_ERROR = 14,
  CUBLAS_STATUS_NOT_SUPPORTED = 15,
  CUBLAS_STATUS_LICENSE_ERROR = 16
} cublasStatus_t;

typedef enum { CUBLAS_OP_N = 0, CUBLAS_OP_T = 1, CUBLAS_OP_C = 2 } cublasOperation_t;

typedef enum { CUBLAS_POINTER_MODE_HOST = 0, CUBLAS_POINTER_MODE_DEVICE = 1 } cublasPointerMode_t;

typedef enum {
  CUBLAS_COMPUTE_16F = 64,
  CUBLAS_COMPUTE_32F = 68,
  CUBLAS_COMPUTE_32F_PEDANTIC = 69,
  CUBLAS_COMPUTE_32I = 72,
  CUBLAS_COMPUTE_32I_PEDANTIC = 73,
  CUBLAS_COMPUTE_32F_FAST_16F = 74,
  CUBLAS_COMPUTE_32F_FAST_16BF = 75,
  CUBLAS_COMPUTE_32F_FAST_TF32 = 77
} cublasComputeType_t;

typedef enum { CUBLAS_GEMM_DEFAULT = -1 } cublasGemmAlgo_t;

typedef struct rouge_b200_cublas_ctx *cublasHandle_t;

/* cublas_shim.h:44-47 */
const char *cublasGetStatusString(cublasStatus_t status);
cublasStatus_t cublasCreate_v2(cublasHandle_t *handle);
cublasStatus_t cublasDestroy_v2(cublasHandle_t handle);
cublasStatus_t cublasGetVersion_v2(cublasHandle_t handle, int *version);

/* Stream of the handle (cuBLAS API; the reference's shim has none: it runs
 * on the host). NULL = the legacy default stream. */
cublasStatus_t cublasSetStream_v2(cublasHandle_t handle, cudaStream_t stream);
cublasStatus_t cublasGetStream_v2(cublasHandle_t handle, cudaStream_t *stream);

/* cublas_shim.h:85-88 */
cublasStatus_t cublasGetPointerMode_v2(cublasHandle_t handle, cublasPointerMode_t *mode);
cublasStatus_t cublasSetPointerMode_v2(cublasHandle_t handle, cublasPointerMode_t mode);

/* cublas_shim.h:50-53 (cublas_shim.cpp:199-211): C = alpha*op(A)*op(B) + beta*C,
 * column-major; op N, T or C (C == T for real types). */
cublasStatus_t cublasSgemm_v2(cublasHandle_t handle, cublasOperation_t transa,
                              cublasOperation_t transb, int m, int n, int k, const float *alpha,
                              const float *A, int lda, const float *B, int ldb, const float *beta,
                              float *C, int ldc);

/* cublas_shim.h:73-76 (cublas_shim.cpp:314-335): batchCount independent
 * GEMMs at the given element strides. */
cublasStatus_t cublasSgemmStridedBatched(cublasHandle_t handle, cublasOperation_t transa,
                                         cublasOperation_t transb, int m, int n, int k,
                                         const float *alpha, const float *A, int lda,
                                         long long strideA, const float *B, int ldb,
                                         long long strideB, const float *beta, float *C, int ldc,
                                         long long strideC, int batchCount);

/* cuBLAS GemmEx (no reference counterpart: the reference's shim has only the
 * typed gemm entries): Atype == Btype in {CUDA_R_16F,
 * CUDA_R_16BF, CUDA_R_8F_E4M3, CUDA_R_32F} with Ctype CUDA_R_32F and a 32F
 * compute type (alpha, beta: float), or CUDA_R_8I with Ctype CUDA_R_32I and
 * CUBLAS_COMPUTE_32I (alpha, beta: int32_t, 1 and 0 only). Other
 * combinations: CUBLAS_STATUS_NOT_SUPPORTED. algo is ignored. */
cublasStatus_t cublasGemmEx(cublasHandle_t handle, cublasOperation_t transa,
                            cublasOperation_t transb, int m, int n, int k, const void *alpha,
                            const void *A, cudaDataType_t Atype, int lda, const void *B,
                            cudaDataType_t Btype, int ldb, const void *beta, void *C,
                            cudaDataType_t Ctype, int ldc, cublasComputeType_t computeType,
                            cublasGemmAlgo_t algo);

#ifdef __cplusplus
} /* extern "C" */
#endif
