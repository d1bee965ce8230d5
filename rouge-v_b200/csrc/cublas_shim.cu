// librouge_b200_cublas.so: the cuBLAS GEMM API subset of
// include/rouge/cublas_b200.h on rouge_b200_gemm_colmajor (tcgen05 kernels).
// The reference's shim (cublas_shim.cpp) keeps the same entry names and
// statuses on its CPU GEMM; here device pointers are used in place and the
// work is queued on the handle's stream, and host pointers (what the
// reference's callers pass) are staged through device memory, the call
// returning when the result is back. Each handle owns a growable device
// workspace for the packed operands and one for staged host operands.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <mutex>
#include <new>

#include "rouge/cublas_b200.h"
#include "rouge/numerics_b200.h"
#include "shim_stage.h"

struct rouge_b200_cublas_ctx {
  int magic;
  cudaStream_t stream;
  cublasPointerMode_t mode;
  void *ws;
  size_t ws_bytes;
  rb200shim::DevBuf stage;
  std::mutex lock;
};

namespace {

constexpr int kMagic = 0x52423230;  // "RB20"

bool valid(cublasHandle_t h) { return h && h->magic == kMagic; }

cublasStatus_t map_status(int s) {
  switch (s) {
    case ROUGE_B200_OK: return CUBLAS_STATUS_SUCCESS;
    case ROUGE_B200_EINVAL: return CUBLAS_STATUS_INVALID_VALUE;
    case ROUGE_B200_EUNSUPPORTED: return CUBLAS_STATUS_NOT_SUPPORTED;
    case ROUGE_B200_ENODEV: return CUBLAS_STATUS_ARCH_MISMATCH;
    case ROUGE_B200_ENOMEM:
    case ROUGE_B200_ETOOBIG: return CUBLAS_STATUS_ALLOC_FAILED;
    default: return CUBLAS_STATUS_EXECUTION_FAILED;
  }
}

bool valid_op(cublasOperation_t o) {
  return o == CUBLAS_OP_N || o == CUBLAS_OP_T || o == CUBLAS_OP_C;
}

// Reads a scalar argument in the handle's pointer mode.
template <class T>
bool scalar(cublasHandle_t h, const void *p, T *out) {
  if (!p) return false;
  if (h->mode == CUBLAS_POINTER_MODE_HOST) {
    std::memcpy(out, p, sizeof(T));
    return true;
  }
  return cudaMemcpyAsync(out, p, sizeof(T), cudaMemcpyDeviceToHost, h->stream) == cudaSuccess &&
         cudaStreamSynchronize(h->stream) == cudaSuccess;
}

// Grows the handle's workspace to `bytes` (after the stream's queued work,
// which may still use the old one).
bool ensure_ws(cublasHandle_t h, size_t bytes) {
  if (bytes <= h->ws_bytes) return true;
  if (h->ws) {
    cudaStreamSynchronize(h->stream);
    cudaFree(h->ws);
    h->ws = nullptr;
    h->ws_bytes = 0;
  }
  if (cudaMalloc(&h->ws, bytes) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  h->ws_bytes = bytes;
  return true;
}

// Elements spanned by a column-major rows x cols matrix with pitch ld.
size_t extent(int rows, int cols, int ld) {
  return rows <= 0 || cols <= 0 || ld < rows ? 0 : static_cast<size_t>(cols - 1) * ld + rows;
}

size_t esize_of(int t) {
  return t == ROUGE_B200_T_F32 || t == ROUGE_B200_T_I32 ? 4
         : t == ROUGE_B200_T_F16 || t == ROUGE_B200_T_BF16 ? 2 : 1;
}

cublasStatus_t gemm(cublasHandle_t h, cublasOperation_t ta, cublasOperation_t tb, int m, int n,
                    int k, int ab_type, float alpha, const void *A, int lda, const void *B, int ldb,
                    float beta, void *C, int c_type, int ldc) {
  const size_t need = rouge_b200_gemm_colmajor_workspace(ab_type, m, n, k);
  if (need && !ensure_ws(h, need)) return CUBLAS_STATUS_ALLOC_FAILED;
  const bool an = ta == CUBLAS_OP_N, bn = tb == CUBLAS_OP_N;
  rb200shim::Staging sg(h->stage, h->stream);
  sg.add(A, extent(an ? m : k, an ? k : m, lda) * esize_of(ab_type), true, false);
  sg.add(B, extent(bn ? k : n, bn ? n : k, ldb) * esize_of(ab_type), true, false);
  sg.add(C, extent(m, n, ldc) * esize_of(c_type), beta != 0.0f, true);
  if (!sg.begin()) return CUBLAS_STATUS_ALLOC_FAILED;
  const int s = rouge_b200_gemm_colmajor(an ? 0 : 1, bn ? 0 : 1, m, n, k, ab_type, alpha, sg.dev(A),
                                         lda, sg.dev(B), ldb, beta, sg.dev(C), c_type, ldc, h->ws,
                                         h->ws_bytes, h->stream);
  const bool ok = sg.finish();
  if (s != ROUGE_B200_OK) return map_status(s);
  return ok ? CUBLAS_STATUS_SUCCESS : CUBLAS_STATUS_EXECUTION_FAILED;
}

int ab_type_of(cudaDataType_t t) {
  switch (t) {
    case CUDA_R_32F: return ROUGE_B200_T_F32;
    case CUDA_R_16F: return ROUGE_B200_T_F16;
    case CUDA_R_16BF: return ROUGE_B200_T_BF16;
    case CUDA_R_8F_E4M3: return ROUGE_B200_T_E4M3;
    case CUDA_R_8I: return ROUGE_B200_T_I8;
    default: return -1;
  }
}

}  // namespace

extern "C" {

const char *cublasGetStatusString(cublasStatus_t status) {
  switch (status) {
    case CUBLAS_STATUS_SUCCESS: return "CUBLAS_STATUS_SUCCESS";
    case CUBLAS_STATUS_NOT_INITIALIZED: return "CUBLAS_STATUS_NOT_INITIALIZED";
    case CUBLAS_STATUS_ALLOC_FAILED: return "CUBLAS_STATUS_ALLOC_FAILED";
    case CUBLAS_STATUS_INVALID_VALUE: return "CUBLAS_STATUS_INVALID_VALUE";
    case CUBLAS_STATUS_ARCH_MISMATCH: return "CUBLAS_STATUS_ARCH_MISMATCH";
    case CUBLAS_STATUS_MAPPING_ERROR: return "CUBLAS_STATUS_MAPPING_ERROR";
    case CUBLAS_STATUS_EXECUTION_FAILED: return "CUBLAS_STATUS_EXECUTION_FAILED";
    case CUBLAS_STATUS_INTERNAL_ERROR: return "CUBLAS_STATUS_INTERNAL_ERROR";
    case CUBLAS_STATUS_NOT_SUPPORTED: return "CUBLAS_STATUS_NOT_SUPPORTED";
    case CUBLAS_STATUS_LICENSE_ERROR: return "CUBLAS_STATUS_LICENSE_ERROR";
  }
  return "CUBLAS_STATUS_UNKNOWN";
}

cublasStatus_t cublasCreate_v2(cublasHandle_t *handle) {
  if (!handle) return CUBLAS_STATUS_INVALID_VALUE;
  if (!rouge_b200_device_ok()) return CUBLAS_STATUS_NOT_INITIALIZED;
  auto *h = new (std::nothrow) rouge_b200_cublas_ctx();
  if (!h) return CUBLAS_STATUS_ALLOC_FAILED;
  h->magic = kMagic;
  h->stream = nullptr;
  h->mode = CUBLAS_POINTER_MODE_HOST;
  h->ws = nullptr;
  h->ws_bytes = 0;
  *handle = h;
  return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasDestroy_v2(cublasHandle_t handle) {
  if (!valid(handle)) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (handle->ws) {
    cudaStreamSynchronize(handle->stream);
    cudaFree(handle->ws);
  }
  handle->stage.release(handle->stream);
  handle->magic = 0;
  delete handle;
  return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasGetVersion_v2(cublasHandle_t handle, int *version) {
  if (!valid(handle)) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (!version) return CUBLAS_STATUS_INVALID_VALUE;
  *version = 120900;  // the cuBLAS API level of the CUDA 12.9 toolkit this follows
  return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasSetStream_v2(cublasHandle_t handle, cudaStream_t stream) {
  if (!valid(handle)) return CUBLAS_STATUS_NOT_INITIALIZED;
  std::lock_guard<std::mutex> g(handle->lock);
  handle->stream = stream;
  return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasGetStream_v2(cublasHandle_t handle, cudaStream_t *stream) {
  if (!valid(handle)) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (!stream) return CUBLAS_STATUS_INVALID_VALUE;
  *stream = handle->stream;
  return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasGetPointerMode_v2(cublasHandle_t handle, cublasPointerMode_t *mode) {
  if (!valid(handle)) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (!mode) return CUBLAS_STATUS_INVALID_VALUE;
  *mode = handle->mode;
  return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasSetPointerMode_v2(cublasHandle_t handle, cublasPointerMode_t mode) {
  if (!valid(handle)) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (mode != CUBLAS_POINTER_MODE_HOST && mode != CUBLAS_POINTER_MODE_DEVICE)
    return CUBLAS_STATUS_INVALID_VALUE;
  handle->mode = mode;
  return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasSgemm_v2(cublasHandle_t handle, cublasOperation_t transa,
                              cublasOperation_t transb, int m, int n, int k, const float *alpha,
                              const float *A, int lda, const float *B, int ldb, const float *beta,
                              float *C, int ldc) {
  if (!valid(handle)) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (!valid_op(transa) || !valid_op(transb)) return CUBLAS_STATUS_INVALID_VALUE;
  std::lock_guard<std::mutex> g(handle->lock);
  float al, be;
  if (!scalar(handle, alpha, &al) || !scalar(handle, beta, &be)) return CUBLAS_STATUS_INVALID_VALUE;
  return gemm(handle, transa, transb, m, n, k, ROUGE_B200_T_F32, al, A, lda, B, ldb, be, C,
              ROUGE_B200_T_F32, ldc);
}

cublasStatus_t cublasSgemmStridedBatched(cublasHandle_t handle, cublasOperation_t transa,
                                         cublasOperation_t transb, int m, int n, int k,
                                         const float *alpha, const float *A, int lda,
                                         long long strideA, const float *B, int ldb,
                                         long long strideB, const float *beta, float *C, int ldc,
                                         long long strideC, int batchCount) {
  if (!valid(handle)) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (!valid_op(transa) || !valid_op(transb) || batchCount < 0) return CUBLAS_STATUS_INVALID_VALUE;
  std::lock_guard<std::mutex> g(handle->lock);
  float al, be;
  if (!scalar(handle, alpha, &al) || !scalar(handle, beta, &be)) return CUBLAS_STATUS_INVALID_VALUE;
  for (int b = 0; b < batchCount; ++b) {
    const cublasStatus_t s =
        gemm(handle, transa, transb, m, n, k, ROUGE_B200_T_F32, al, A + b * strideA, lda,
             B + b * strideB, ldb, be, C + b * strideC, ROUGE_B200_T_F32, ldc);
    if (s != CUBLAS_STATUS_SUCCESS) return s;
  }
  return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasGemmEx(cublasHandle_t handle, cublasOperation_t transa,
                            cublasOperation_t transb, int m, int n, int k, const void *alpha,
                            const void *A, cudaDataType_t Atype, int lda, const void *B,
                            cudaDataType_t Btype, int ldb, const void *beta, void *C,
                            cudaDataType_t Ctype, int ldc, cublasComputeType_t computeType,
                            cublasGemmAlgo_t algo) {
  (void)algo;
  if (!valid(handle)) return CUBLAS_STATUS_NOT_INITIALIZED;
  if (!valid_op(transa) || !valid_op(transb)) return CUBLAS_STATUS_INVALID_VALUE;
  const int ab = ab_type_of(Atype);
  if (ab < 0 || Btype != Atype) return CUBLAS_STATUS_NOT_SUPPORTED;
  std::lock_guard<std::mutex> g(handle->lock);
  if (ab == ROUGE_B200_T_I8) {
    if (Ctype != CUDA_R_32I ||
        (computeType != CUBLAS_COMPUTE_32I && computeType != CUBLAS_COMPUTE_32I_PEDANTIC))
      return CUBLAS_STATUS_NOT_SUPPORTED;
    int32_t al, be;
    if (!scalar(handle, alpha, &al) || !scalar(handle, beta, &be)) return CUBLAS_STATUS_INVALID_VALUE;
    if (al != 1 || be != 0) return CUBLAS_STATUS_NOT_SUPPORTED;
    return gemm(handle, transa, transb, m, n, k, ab, 1.0f, A, lda, B, ldb, 0.0f, C,
                ROUGE_B200_T_I32, ldc);
  }
  if (Ctype != CUDA_R_32F ||
      (computeType != CUBLAS_COMPUTE_32F && computeType != CUBLAS_COMPUTE_32F_PEDANTIC &&
       computeType != CUBLAS_COMPUTE_32F_FAST_TF32 && computeType != CUBLAS_COMPUTE_32F_FAST_16F &&
       computeType != CUBLAS_COMPUTE_32F_FAST_16BF))
    return CUBLAS_STATUS_NOT_SUPPORTED;
  float al, be;
  if (!scalar(handle, alpha, &al) || !scalar(handle, beta, &be)) return CUBLAS_STATUS_INVALID_VALUE;
  return gemm(handle, transa, transb, m, n, k, ab, al, A, lda, B, ldb, be, C, ROUGE_B200_T_F32, ldc);
}

}  // extern "C"
