// Column-major BLAS GEMM on the tcgen05 kernels (the semantics of
// cublasSgemm / cublasGemmEx, which the reference implements on its CPU
// GEMM in cublas_shim.cpp:36-65,199-211):
//     C (m x n, column-major, ldc) = alpha * op(A) * op(B) + beta * C
// The row-major kernels compute the transposed triple C^T = op(B)^T op(A)^T
// straight into C's memory (a column-major m x n matrix with pitch ldc is a
// row-major n x m matrix with pitch ldc):
//     A' [n][Kp]  row j = column j of op(B)         (the kernel's A, K-major)
//     B' [m][Kp]  row i = row i of op(A)            (the kernel's B, K-major)
// Both are packed into a caller-provided workspace by one transposing copy
// (16-byte aligned, K padded with zeros to the kernel's pitch), whatever the
// transposes and leading dimensions. f32 operands are split for "3xTF32":
// A' = [B_hi | B_hi | B_lo], B' = [A_hi | A_lo | A_hi] along K (hi = tf32
// round-to-nearest of x, lo = x - hi), so one tf32 GEMM over 3 Kp
// accumulates hi*hi + hi*lo + lo*hi, f32-accurate.
#include <cuda_runtime.h>

#include <cstdint>

#include "pack.cuh"
#include "runtime.cuh"

namespace rb200 {

int launch_gemm_blas_tiles(int kind, int M, int N, int K, const void *A, long long lda,
                           const void *B, long long ldb, int b_layout, float alpha, float beta,
                           float *Cp, long long ldc, int tile_hint, cudaStream_t st);
int launch_gemm_i8(int M, int N, int K, const int8_t *A, long long lda, const int8_t *B,
                   long long ldb, int b_layout, const float *sa, int a_rows, const float *sb,
                   int b_cols, void *Cp, long long ldc, int out_type, cudaStream_t st);

namespace {

// C (m x n column-major, ldc) = beta * C, zero when beta == 0 (k == 0 or
// alpha == 0: no product to add).
__global__ void scale_kernel(float *C, int m, int n, long long ldc, float beta) {
  const long long total = static_cast<long long>(m) * n;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    float *c = C + (i / m) * ldc + i % m;
    *c = beta == 0.0f ? 0.0f : beta * *c;
  }
}

template <class T>
int pack(const void *src, long long sr, long long sp, int R, int K, int Kp, int split, void *out,
         long long kp_out, cudaStream_t st) {
  return pack_launch<T>(src, 0, sr, sp, R, K, Kp, split, out, 0, kp_out, 1, st);
}

size_t rup(size_t v, size_t a) { return (v + a - 1) / a * a; }

int esize_of(int type) {
  switch (type) {
    case ROUGE_B200_T_E4M3: case ROUGE_B200_T_I8: return 1;
    case ROUGE_B200_T_F16: case ROUGE_B200_T_BF16: return 2;
    case ROUGE_B200_T_F32: return 4;
    default: return 0;
  }
}

// Padded K (elements): 16-byte rows for every type, and the kernel's
// 128-byte k-block for f32 so that the three split blocks stay aligned.
int padded_k(int type, int k) {
  const int es = esize_of(type);
  return static_cast<int>(rup(k, type == ROUGE_B200_T_F32 ? 32 : 16 / es));
}

}  // namespace
}  // namespace rb200

using namespace rb200;

extern "C" {

size_t rouge_b200_gemm_colmajor_workspace(int ab_type, int m, int n, int k) {
  const int es = esize_of(ab_type);
  if (!es || m <= 0 || n <= 0 || k <= 0) return 0;
  const size_t kp = padded_k(ab_type, k) * (ab_type == ROUGE_B200_T_F32 ? 3 : 1);
  return rup(static_cast<size_t>(n) * kp * es, 256) + rup(static_cast<size_t>(m) * kp * es, 256);
}

int rouge_b200_gemm_colmajor(int transa, int transb, int m, int n, int k, int ab_type, float alpha,
                             const void *A, int lda, const void *B, int ldb, float beta, void *C,
                             int c_type, int ldc, void *workspace, size_t workspace_bytes,
                             void *stream) {
  const int es = esize_of(ab_type);
  if (!es || (transa != 0 && transa != 1) || (transb != 0 && transb != 1))
    return set_status(ROUGE_B200_EINVAL);
  if (m < 0 || n < 0 || k < 0 || ldc < (m > 1 ? m : 1)) return set_status(ROUGE_B200_EINVAL);
  // op(A) is m x k: stored k x m when transposed; op(B) is k x n.
  if (lda < ((transa ? k : m) > 1 ? (transa ? k : m) : 1) ||
      ldb < ((transb ? n : k) > 1 ? (transb ? n : k) : 1))
    return set_status(ROUGE_B200_EINVAL);
  const bool int8 = ab_type == ROUGE_B200_T_I8;
  if (int8 ? c_type != ROUGE_B200_T_I32 : c_type != ROUGE_B200_T_F32)
    return set_status(ROUGE_B200_EUNSUPPORTED);
  if (int8 && (alpha != 1.0f || beta != 0.0f)) return set_status(ROUGE_B200_EUNSUPPORTED);
  if (m == 0 || n == 0) return ROUGE_B200_OK;
  if (!C || (k > 0 && (!A || !B))) return set_status(ROUGE_B200_EINVAL);
  int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  cudaStream_t st = as_stream(stream);
  if (k == 0 || (!int8 && alpha == 0.0f)) {
    if (int8) return cuda_status(cudaMemset2DAsync(C, static_cast<size_t>(ldc) * 4, 0,
                                                   static_cast<size_t>(m) * 4, n, st));
    scale_kernel<<<512, 256, 0, st>>>(static_cast<float *>(C), m, n, ldc, beta);
    return cuda_status(cudaGetLastError());
  }
  if (!workspace || workspace_bytes < rouge_b200_gemm_colmajor_workspace(ab_type, m, n, k) ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return set_status(ROUGE_B200_ETOOBIG);
  const int Kp = padded_k(ab_type, k);
  const bool f32 = ab_type == ROUGE_B200_T_F32;
  const long long kp_row = static_cast<long long>(Kp) * (f32 ? 3 : 1);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  void *Ap = ws;                                                      // A' [n][kp_row]
  void *Bp = ws + rup(static_cast<size_t>(n) * kp_row * es, 256);     // B' [m][kp_row]
  // A'[j][p] = op(B)[p][j]: B[p + j*ldb] (N) or B[j + p*ldb] (T).
  const long long a_sr = transb ? 1 : ldb, a_sp = transb ? ldb : 1;
  // B'[i][p] = op(A)[i][p]: A[i + p*lda] (N) or A[p + i*lda] (T).
  const long long b_sr = transa ? lda : 1, b_sp = transa ? 1 : lda;
  switch (es) {
    case 1:
      s = pack<uint8_t>(B, a_sr, a_sp, n, k, Kp, 0, Ap, kp_row, st);
      if (s == ROUGE_B200_OK) s = pack<uint8_t>(A, b_sr, b_sp, m, k, Kp, 0, Bp, kp_row, st);
      break;
    case 2:
      s = pack<uint16_t>(B, a_sr, a_sp, n, k, Kp, 0, Ap, kp_row, st);
      if (s == ROUGE_B200_OK) s = pack<uint16_t>(A, b_sr, b_sp, m, k, Kp, 0, Bp, kp_row, st);
      break;
    default:
      s = pack<uint32_t>(B, a_sr, a_sp, n, k, Kp, 1, Ap, kp_row, st);
      if (s == ROUGE_B200_OK) s = pack<uint32_t>(A, b_sr, b_sp, m, k, Kp, 2, Bp, kp_row, st);
      break;
  }
  if (s != ROUGE_B200_OK) return s;
  if (int8)
    return launch_gemm_i8(n, m, static_cast<int>(kp_row), static_cast<const int8_t *>(Ap), kp_row,
                          static_cast<const int8_t *>(Bp), kp_row, ROUGE_B200_B_NK, nullptr, 0,
                          nullptr, 0, C, ldc, ROUGE_B200_OUT_I32, st);
  const int kind = ab_type == ROUGE_B200_T_E4M3 ? 0 : ab_type == ROUGE_B200_T_F16 ? 1
                   : ab_type == ROUGE_B200_T_BF16 ? 2 : 3;
  return launch_gemm_blas_tiles(kind, n, m, static_cast<int>(kp_row), Ap, kp_row, Bp, kp_row,
                                ROUGE_B200_B_NK, alpha, beta, static_cast<float *>(C), ldc, 0, st);
}

}  // extern "C"

namespace rb200 {

// Row-major f32 GEMM in K-chunks (the engine of the drop-in
// rouge_gemm_f32): C[M][N] = A[M][K] . B[K][N], device pointers, row
// pitches K, N and N. The tensor cores accumulate each MMA into f32 with a
// rounding that loses up to an ulp of the accumulator per step, so an
// error that grows with the number of steps into one accumulator; here
// every chunk of kF32ChunkK elements of K is one 3xTF32 GEMM of its own
// (at most 3 * 256 / 8 = 96 MMA steps), and the chunks are summed in C by
// the epilogue (C = acc + C, one round-to-nearest add per chunk).
// Operands are packed chunk by chunk, each chunk's [hi | hi | lo] (A) and
// [hi | lo | hi] (B^T) blocks side by side in a row of kp_row floats.
constexpr int kF32ChunkK = 256;

long long f32_chunk_row(int K) {
  const long long full = K / kF32ChunkK, rest = K % kF32ChunkK;
  return 3 * (full * kF32ChunkK + static_cast<long long>(rup(rest, 32)));
}

size_t gemm_f32_rowmajor_workspace(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  const size_t row = static_cast<size_t>(f32_chunk_row(K)) * 4;
  return rup(static_cast<size_t>(M) * row, 256) + rup(static_cast<size_t>(N) * row, 256);
}

int gemm_f32_rowmajor(int M, int N, int K, const float *A, const float *B, float *C,
                      void *workspace, size_t workspace_bytes, int tile_hint, cudaStream_t st) {
  if (M <= 0 || N <= 0 || K <= 0 || !A || !B || !C) return set_status(ROUGE_B200_EINVAL);
  if (!workspace || workspace_bytes < gemm_f32_rowmajor_workspace(M, N, K) ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return set_status(ROUGE_B200_ETOOBIG);
  const long long kp_row = f32_chunk_row(K);
  uint32_t *Ap = static_cast<uint32_t *>(workspace);                        // [M][kp_row]
  uint32_t *Bp = reinterpret_cast<uint32_t *>(static_cast<uint8_t *>(workspace) +
                                              rup(static_cast<size_t>(M) * kp_row * 4, 256));
  const int full = K / kF32ChunkK, rest = K % kF32ChunkK;
  const long long cw = 3LL * kF32ChunkK;  // packed width of a whole chunk
  // A rows are contiguous along K (sr = K, sp = 1); B^T row n = column n of
  // B (sr = 1, sp = N). Whole chunks as one batched pack, then the rest.
  int s = ROUGE_B200_OK;
  if (full > 0) {
    s = pack_launch<uint32_t>(A, kF32ChunkK, K, 1, M, kF32ChunkK, kF32ChunkK, 1, Ap, cw, kp_row,
                              full, st);
    if (s == ROUGE_B200_OK)
      s = pack_launch<uint32_t>(B, static_cast<long long>(kF32ChunkK) * N, 1, N, N, kF32ChunkK,
                                kF32ChunkK, 2, Bp, cw, kp_row, full, st);
  }
  if (s == ROUGE_B200_OK && rest > 0) {
    const int rp = static_cast<int>(rup(rest, 32));
    const long long k0 = static_cast<long long>(full) * kF32ChunkK;
    s = pack_launch<uint32_t>(A + k0, 0, K, 1, M, rest, rp, 1, Ap + full * cw, 0, kp_row, 1, st);
    if (s == ROUGE_B200_OK)
      s = pack_launch<uint32_t>(B + k0 * N, 0, 1, N, N, rest, rp, 2, Bp + full * cw, 0, kp_row, 1,
                                st);
  }
  const int chunks = full + (rest > 0 ? 1 : 0);
  for (int c = 0; s == ROUGE_B200_OK && c < chunks; ++c) {
    const int kc = c < full ? 3 * kF32ChunkK : 3 * static_cast<int>(rup(rest, 32));
    s = launch_gemm_blas_tiles(3, M, N, kc, Ap + c * cw, kp_row, Bp + c * cw, kp_row,
                               ROUGE_B200_B_NK, 1.0f, c == 0 ? 0.0f : 1.0f, C, N, tile_hint, st);
  }
  return s;
}

}  // namespace rb200
