// Transposing pack of a strided 2-D view into a K-major operand, shared by
// the column-major BLAS entry (blas.cu) and the cuDNN-style convolution
// forward (conv_fwd.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "runtime.cuh"

namespace rb200 {
namespace {

constexpr int kPackTile = 32;

__device__ __forceinline__ float tf32_round_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// For batch z = blockIdx.z:
//   out[z*so + r*kp_out + p] = src[z*ss + r*sr + p*sp]   r < R, p < K
//                            = 0                          K <= p < Kp
// split (4-byte T only, f32 bits): 0 plain copy; 1 writes [hi | hi | lo],
// 2 writes [hi | lo | hi] in three blocks of Kp (hi = tf32 round to
// nearest, ties away, lo = x - hi, exact). 32 x 32 tiles through shared
// memory, read along whichever of r / p is contiguous in the source.
template <class T>
__global__ void pack_kernel(const T *__restrict__ src, long long ss, long long sr, long long sp,
                            int R, int K, int Kp, int split, T *__restrict__ out, long long so,
                            long long kp_out) {
  __shared__ T t[kPackTile][kPackTile + 1];
  const int r0 = blockIdx.y * kPackTile, p0 = blockIdx.x * kPackTile;
  src += blockIdx.z * ss;
  out += blockIdx.z * so;
  const bool along_r = sr == 1;  // source contiguous along r: read by r, write by p
  for (int i = threadIdx.y; i < kPackTile; i += blockDim.y) {
    const int r = along_r ? r0 + threadIdx.x : r0 + i;
    const int p = along_r ? p0 + i : p0 + threadIdx.x;
    T v = T(0);
    if (r < R && p < K) v = src[r * sr + p * sp];
    if (along_r)
      t[threadIdx.x][i] = v;
    else
      t[i][threadIdx.x] = v;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < kPackTile; i += blockDim.y) {
    const int r = r0 + i, p = p0 + threadIdx.x;
    if (r >= R || p >= Kp) continue;
    const T v = t[i][threadIdx.x];
    T *row = out + r * kp_out;
    if constexpr (sizeof(T) == 4) {
      if (split) {
        const float x = __uint_as_float(static_cast<uint32_t>(v));
        const float hi = tf32_round_rna(x);
        const float lo = x - hi;
        row[p] = static_cast<T>(__float_as_uint(hi));
        row[Kp + p] = static_cast<T>(__float_as_uint(split == 1 ? hi : lo));
        row[2 * Kp + p] = static_cast<T>(__float_as_uint(split == 1 ? lo : hi));
        continue;
      }
    }
    row[p] = v;
  }
}

// Launches pack_kernel over `batch` slices (grid z; batches above 65535
// are issued in pieces).
template <class T>
int pack_launch(const void *src, long long ss, long long sr, long long sp, int R, int K, int Kp,
                int split, void *out, long long so, long long kp_out, int batch, cudaStream_t st) {
  for (int z0 = 0; z0 < batch; z0 += 65535) {
    const int nz = batch - z0 < 65535 ? batch - z0 : 65535;
    const dim3 grid((Kp + kPackTile - 1) / kPackTile, (R + kPackTile - 1) / kPackTile, nz);
    pack_kernel<T><<<grid, dim3(kPackTile, 8), 0, st>>>(
        static_cast<const T *>(src) + z0 * ss, ss, sr, sp, R, K, Kp, split,
        static_cast<T *>(out) + z0 * so, so, kp_out);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e);
  }
  return ROUGE_B200_OK;
}

}  // namespace
}  // namespace rb200
