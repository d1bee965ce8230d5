// f32 NCHW convolution drop-ins (rouge_conv2d_f32, conv.cpp:26-66, and
// rouge_conv_implicit_f32, conv_implicit.cpp:24-79: the same result by two
// CPU algorithms) on the tcgen05 implicit-GEMM convolution.
//
// f32 precision from tf32 tensor cores ("3xTF32"): every operand x is split
// into hi = tf32(x) (round to nearest, ties away) and lo = x - hi (exact in
// f32), and the convolution runs over three channel blocks
//     X' = [X_hi | X_hi | X_lo],   W' = [W_hi | W_lo | W_hi]
// so one tf32 implicit GEMM with 3 * Cin' channels accumulates
// hi*hi + hi*lo + lo*hi in f32; the dropped lo*lo term and the tf32
// truncation of lo are below 2^-21 of each product. Layout on the device:
//   X' [Np][H][W][3 * Cp]   NHWC, Cp = Cin rounded up to 32 (zero channels),
//                           Np >= N images so that X' spans at least 128 KB
//   W' [Cop][KH][KW][3 * Cp] Cop = Cout rounded up to 4 (zero rows)
//   Y' [Np * OH * OW][Cop]  NHWC f32 (+ bias; the padding images' rows are
//                           computed and dropped), then transposed to NCHW.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "runtime.cuh"

namespace rb200 {

int launch_conv_tf32(int N, int H, int W, int Cin, int Cout, int KH, int KW, int stride, int pad,
                     const float *X, const float *Wt, const float *bias, float *Y, long long ldy,
                     cudaStream_t st);

namespace {

constexpr int kTile = 32;

__device__ __forceinline__ float tf32_hi(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// X[n][c][p] (p = h * W + w) -> X'[n][p][{c, Cp + c, 2 Cp + c}] = {hi, hi, lo}.
// One 32 x 32 (channel x pixel) tile per block, transposed through shared
// memory so that reads run along pixels and writes along channels.
__global__ void split_nchw_to_nhwc(const float *__restrict__ x, int Cin, int P, int Cp,
                                   float *__restrict__ xs) {
  __shared__ float t[kTile][kTile + 1];
  const int n = blockIdx.z;
  const int p0 = blockIdx.x * kTile, c0 = blockIdx.y * kTile;
  const float *xn = x + static_cast<size_t>(n) * Cin * P;
  for (int i = threadIdx.y; i < kTile; i += blockDim.y) {
    const int c = c0 + i, p = p0 + threadIdx.x;
    t[i][threadIdx.x] = (c < Cin && p < P) ? xn[static_cast<size_t>(c) * P + p] : 0.0f;
  }
  __syncthreads();
  float *xsn = xs + static_cast<size_t>(n) * P * 3 * Cp;
  for (int i = threadIdx.y; i < kTile; i += blockDim.y) {
    const int p = p0 + i, c = c0 + threadIdx.x;
    if (p < P && c < Cp) {
      const float v = t[threadIdx.x][i];
      const float hi = tf32_hi(v);
      float *row = xsn + static_cast<size_t>(p) * 3 * Cp;
      row[c] = hi;
      row[Cp + c] = hi;
      row[2 * Cp + c] = v - hi;
    }
  }
}

// Wt[co][c][kr][kc] -> W'[co][kr][kc][{c, Cp + c, 2 Cp + c}] = {hi, lo, hi},
// zero for co >= Cout or c >= Cin.
__global__ void split_weights(const float *__restrict__ w, int Cout, int Cin, int KH, int KW,
                              int Cop, int Cp, float *__restrict__ ws) {
  const size_t total = static_cast<size_t>(Cop) * KH * KW * Cp;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % Cp);
    const size_t r = i / Cp;  // (co, kr, kc)
    const int kc = static_cast<int>(r % KW);
    const int kr = static_cast<int>((r / KW) % KH);
    const int co = static_cast<int>(r / (static_cast<size_t>(KW) * KH));
    float v = 0.0f;
    if (co < Cout && c < Cin) v = w[((static_cast<size_t>(co) * Cin + c) * KH + kr) * KW + kc];
    const float hi = tf32_hi(v);
    float *row = ws + r * 3 * Cp;
    row[c] = hi;
    row[Cp + c] = v - hi;
    row[2 * Cp + c] = hi;
  }
}

// Y'[n][p][co] (row pitch Cop) -> Y[n][co][p], 32 x 32 tiles through shared
// memory.
__global__ void nhwc_to_nchw(const float *__restrict__ yt, int Cout, int Cop, int P,
                             float *__restrict__ y) {
  __shared__ float t[kTile][kTile + 1];
  const int n = blockIdx.z;
  const int p0 = blockIdx.x * kTile, c0 = blockIdx.y * kTile;
  const float *ytn = yt + static_cast<size_t>(n) * P * Cop;
  for (int i = threadIdx.y; i < kTile; i += blockDim.y) {
    const int p = p0 + i, c = c0 + threadIdx.x;
    t[i][threadIdx.x] = (p < P && c < Cout) ? ytn[static_cast<size_t>(p) * Cop + c] : 0.0f;
  }
  __syncthreads();
  float *yn = y + static_cast<size_t>(n) * Cout * P;
  for (int i = threadIdx.y; i < kTile; i += blockDim.y) {
    const int c = c0 + i, p = p0 + threadIdx.x;
    if (c < Cout && p < P) yn[static_cast<size_t>(c) * P + p] = t[threadIdx.x][i];
  }
}

size_t rup(size_t v, size_t a) { return (v + a - 1) / a * a; }

// The drop-in body shared by both entries. Returns without writing Y on
// invalid arguments (reference behaviour) and on parameters the im2col TMA
// cannot express (status ROUGE_B200_EUNSUPPORTED): padding above 128, a
// filter taller or wider than pad + 129 or than 256, stride above 8.
void conv2d_f32_host(int N, int Cin, int H, int W, int Cout, int KH, int KW, int stride, int pad,
                     const float *X, const float *Wt, const float *bias, float *Y) {
  if (!X || !Wt || !Y) return;  // conv.cpp:30-33, conv_implicit.cpp:28-31
  if (N <= 0 || Cin <= 0 || H <= 0 || W <= 0 || Cout <= 0 || KH <= 0 || KW <= 0 || stride <= 0 ||
      pad < 0)
    return;
  const long long OHl = (static_cast<long long>(H) + 2 * pad - KH) / stride + 1;
  const long long OWl = (static_cast<long long>(W) + 2 * pad - KW) / stride + 1;
  if (OHl <= 0 || OWl <= 0) return;  // conv.cpp:36
  if (pad > 128 || KH > pad + 129 || KW > pad + 129 || KH > 256 || KW > 256 || stride > 8 ||
      KH > H + 2 * pad || KW > W + 2 * pad) {
    set_status(ROUGE_B200_EUNSUPPORTED);
    return;
  }
  const int OH = static_cast<int>(OHl), OW = static_cast<int>(OWl);
  const long long Mpix = static_cast<long long>(N) * OH * OW;
  if (Mpix > 0x7fffffffLL || static_cast<long long>(KH) * KW * Cin * 3 > 0x7fffffffLL) {
    set_status(ROUGE_B200_EUNSUPPORTED);
    return;
  }
  HostCallContext *ctx = host_context();
  if (!ctx) return;
  std::lock_guard<std::mutex> g(ctx->lock);
  const int Cp = static_cast<int>(rup(Cin, 32));
  const int Cop = static_cast<int>(rup(Cout, 4));
  const size_t P = static_cast<size_t>(H) * W, Q = static_cast<size_t>(OH) * OW;
  const size_t img_bytes = P * 3 * Cp * 4;
  const size_t Np = (N * img_bytes >= 131072) ? N : (131072 + img_bytes - 1) / img_bytes;
  const size_t nx = static_cast<size_t>(N) * Cin * P, nw = static_cast<size_t>(Cout) * Cin * KH * KW;
  const size_t sz[7] = {nx * 4,  nw * 4, static_cast<size_t>(Cout) * 4, Np * img_bytes,
                        static_cast<size_t>(Cop) * KH * KW * 3 * Cp * 4,
                        Np * Q * Cop * 4, static_cast<size_t>(N) * Cout * Q * 4};
  size_t need = 0;
  for (size_t b : sz) need += rup(b, 256);
  if (ensure_workspace(ctx, need) != ROUGE_B200_OK) return;
  uint8_t *base = static_cast<uint8_t *>(ctx->ws);
  float *buf[7];
  for (int i = 0; i < 7; ++i) {
    buf[i] = reinterpret_cast<float *>(base);
    base += rup(sz[i], 256);
  }
  float *dX = buf[0], *dW = buf[1], *dbias = buf[2], *dXs = buf[3], *dWs = buf[4], *dYt = buf[5],
        *dY = buf[6];
  cudaStream_t st = ctx->stream;
  int s = cuda_status(cudaMemcpyAsync(dX, X, sz[0], cudaMemcpyHostToDevice, st));
  if (s == ROUGE_B200_OK) s = cuda_status(cudaMemcpyAsync(dW, Wt, sz[1], cudaMemcpyHostToDevice, st));
  if (s == ROUGE_B200_OK && bias)
    s = cuda_status(cudaMemcpyAsync(dbias, bias, sz[2], cudaMemcpyHostToDevice, st));
  if (s == ROUGE_B200_OK && Np > static_cast<size_t>(N))  // padding images read as zeros
    s = cuda_status(cudaMemsetAsync(dXs + static_cast<size_t>(N) * P * 3 * Cp, 0,
                                    (Np - N) * img_bytes, st));
  if (s != ROUGE_B200_OK) return;
  const dim3 tb(kTile, 8);
  split_nchw_to_nhwc<<<dim3(static_cast<unsigned>((P + kTile - 1) / kTile), (Cp + kTile - 1) / kTile,
                           N),
                       tb, 0, st>>>(dX, Cin, static_cast<int>(P), Cp, dXs);
  const size_t nws = static_cast<size_t>(Cop) * KH * KW * Cp;
  const unsigned wblocks = static_cast<unsigned>(nws / 256 + 1 < 4096 ? nws / 256 + 1 : 4096);
  split_weights<<<wblocks, 256, 0, st>>>(dW, Cout, Cin, KH, KW, Cop, Cp, dWs);
  if (cuda_status(cudaGetLastError()) != ROUGE_B200_OK) return;
  if (launch_conv_tf32(static_cast<int>(Np), H, W, 3 * Cp, Cop, KH, KW, stride, pad, dXs, dWs,
                       bias ? dbias : nullptr, dYt, Cop, st) != ROUGE_B200_OK)
    return;
  nhwc_to_nchw<<<dim3(static_cast<unsigned>((Q + kTile - 1) / kTile), (Cout + kTile - 1) / kTile, N),
                 tb, 0, st>>>(dYt, Cout, Cop, static_cast<int>(Q), dY);
  if (cuda_status(cudaGetLastError()) != ROUGE_B200_OK) return;
  if (cuda_status(cudaStreamSynchronize(st)) != ROUGE_B200_OK) return;
  if (take_device_error(st) != ROUGE_B200_OK) return;  // no copy of a result a kernel gave up on
  if (cuda_status(cudaMemcpyAsync(Y, dY, sz[6], cudaMemcpyDeviceToHost, st)) != ROUGE_B200_OK) return;
  cuda_status(cudaStreamSynchronize(st));
}

}  // namespace
}  // namespace rb200

using namespace rb200;

extern "C" {

void rouge_conv2d_f32(int N, int Cin, int H, int W, int Cout, int KH, int KW, int stride, int pad,
                      const float *X, const float *Wt, const float *bias, float *Y,
                      const RougeGemmConfig *cfg) {
  (void)cfg;
  conv2d_f32_host(N, Cin, H, W, Cout, KH, KW, stride, pad, X, Wt, bias, Y);
}

void rouge_conv_implicit_f32(int N, int Cin, int H, int W, int Cout, int KH, int KW, int stride,
                             int pad, const float *X, const float *Wt, const float *bias, float *Y,
                             const RougeGemmConfig *cfg) {
  (void)cfg;
  conv2d_f32_host(N, Cin, H, W, Cout, KH, KW, stride, pad, X, Wt, bias, Y);
}

}  // extern "C"
