// Layout kernel of the N-sharded GEMM.
//
// Rank r of g computes the output columns [r*ns, (r+1)*ns) of C[M][N]. The
// shards are all-gathered band by band (R rows at a time, so the exchange of
// band b overlaps the GEMM of band b+1); an all-gather concatenates the rank
// buffers, which leaves the gathered output as
//   src[band][rank][R][ns]
// This kernel writes it row-major into dst[M][ldd] (columns beyond N of the
// last shard, when N is not a multiple of ns, are dropped). HBM-bound:
// 16-byte loads and stores, grid-stride, grid a multiple of the SM count.
#include <cuda_runtime.h>

#include <cstdint>

#include "runtime.cuh"

namespace rb200 {
namespace {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads) unshard_kernel(const uint4 *__restrict__ src,
                                                           uint4 *__restrict__ dst, int M, int N,
                                                           int g, int ns_vec, int R,
                                                           long long ldd_vec, int vec_elems) {
  // One work item = one 16-byte vector of one row of one rank's shard.
  const long long per_row = static_cast<long long>(g) * ns_vec;
  const long long total = static_cast<long long>(M) * per_row;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += stride) {
    const long long m = i / per_row;
    const int rest = static_cast<int>(i - m * per_row);
    const int r = rest / ns_vec;
    const int j = rest - r * ns_vec;
    const long long col = (static_cast<long long>(r) * ns_vec + j) * vec_elems;
    if (col >= N) continue;
    const long long band = m / R, mr = m - band * R;
    const long long s = ((band * g + r) * R + mr) * ns_vec + j;
    dst[m * ldd_vec + r * static_cast<long long>(ns_vec) + j] = __ldcs(src + s);
  }
}

}  // namespace
}  // namespace rb200

using namespace rb200;

extern "C" {

int rouge_b200_unshard_columns(const void *src, void *dst, int M, int N, int g, int ns, int R,
                               int ldd, int esize, void *stream) {
  if (!src || !dst || M <= 0 || N <= 0 || g <= 0 || ns <= 0 || R <= 0 || M % R ||
      (esize != 1 && esize != 2 && esize != 4) || static_cast<long long>(g) * ns < N || ldd < N)
    return set_status(ROUGE_B200_EINVAL);
  const int vec_elems = 16 / esize;
  if (ns % vec_elems || ldd % vec_elems || N % vec_elems || (reinterpret_cast<uintptr_t>(src) & 15u) ||
      (reinterpret_cast<uintptr_t>(dst) & 15u))
    return set_status(ROUGE_B200_EUNSUPPORTED);
  int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  const int sms = current_sm_count();
  unshard_kernel<<<sms * 8, kThreads, 0, as_stream(stream)>>>(
      static_cast<const uint4 *>(src), static_cast<uint4 *>(dst), M, N, g, ns / vec_elems, R,
      ldd / vec_elems, vec_elems);
  return cuda_status(cudaGetLastError());
}

}  // extern "C"
