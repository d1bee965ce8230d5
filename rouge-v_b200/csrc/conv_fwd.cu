// Convolution forward with cuDNN's semantics on the tcgen05 implicit-GEMM
// convolution (the entry the cuDNN-API library calls; the reference's
// cuDNN shim runs this operation on its CPU conv, cudnn_shim.cpp:188-232):
//     Y = alpha * conv(X, Wt) + beta * Y
// cross-correlation, symmetric stride and zero padding, X / Wt / Y of one
// element type (f32, f16 or bf16), each in NCHW or NHWC (a filter in NCHW
// is [Cout][Cin][KH][KW], in NHWC [Cout][KH][KW][Cin]).
//
// Direct path (no workspace): 16-bit X and Wt in NHWC with Cin % 64 == 0,
// X of at least 128 KB, Y in NHWC with Cout % 8 == 0, 16-byte aligned
// pointers. The kernel reads X and Wt as stored and its epilogue writes
// Y = alpha * acc + beta * Y (f16 / bf16, round to nearest even) in place.
//
// Staged path (everything else), in the caller's workspace:
//   X' [Np][H][W][Cs]   NHWC, channels padded with zeros to the kernel's
//                       k-block (64 for 16-bit, 32 for f32), images padded
//                       so that X' spans 128 KB; f32 split for 3xTF32 into
//                       [X_hi | X_hi | X_lo] (Cs = 3 Cp)
//   W' [Cop][KH][KW][Cs] K-major, Cop = Cout rounded up to 4, f32 split
//                       into [W_hi | W_lo | W_hi]
//   Y: written by the epilogue directly when its layout allows (NHWC, no
//      padding images, 16-byte rows), else the kernel writes f32
//      T [Np*OH*OW][Cop] and one pass forms Y = alpha * T + beta * Y in
//      Y's layout and type (the reference's order: two products, one sum).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "pack.cuh"
#include "runtime.cuh"

namespace rb200 {

int launch_conv_blas(int ab_type, int N, int H, int W, int Cin, int Cout, int KH, int KW,
                     int stride, int pad, const void *X, const void *Wt, float alpha, float beta,
                     void *Y, long long ldy, int y_type, cudaStream_t st);

namespace {

size_t rup(size_t v, size_t a) { return (v + a - 1) / a * a; }

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

struct ConvPlan {
  int OH, OW, P;        // output size, input pixels per image
  int Cp, Cs, es;       // padded channels, channels the kernel sees, operand bytes
  int Np, Cop;          // images and filters after padding
  bool pack_x, pack_w, stage_y;
  size_t x_bytes, w_bytes, t_bytes;
  size_t need() const {
    return (pack_x ? rup(x_bytes, 256) : 0) + (pack_w ? rup(w_bytes, 256) : 0) +
           (stage_y ? rup(t_bytes, 256) : 0);
  }
};

// Validates the problem; fills the plan for the given pointers (null
// pointers are taken as 16-byte aligned: the workspace query).
int make_plan(int N, int Cin, int H, int W, int Cout, int KH, int KW, int stride, int pad,
              int type, int x_layout, int w_layout, int y_layout, const void *X, const void *Wt,
              const void *Y, ConvPlan &p) {
  if (N <= 0 || Cin <= 0 || H <= 0 || W <= 0 || Cout <= 0 || KH <= 0 || KW <= 0 || stride <= 0 ||
      pad < 0)
    return ROUGE_B200_EINVAL;
  if (type != ROUGE_B200_T_F32 && type != ROUGE_B200_T_F16 && type != ROUGE_B200_T_BF16)
    return ROUGE_B200_EUNSUPPORTED;
  for (int l : {x_layout, w_layout, y_layout})
    if (l != ROUGE_B200_NCHW && l != ROUGE_B200_NHWC) return ROUGE_B200_EINVAL;
  const long long OH = (static_cast<long long>(H) + 2 * pad - KH) / stride + 1;
  const long long OW = (static_cast<long long>(W) + 2 * pad - KW) / stride + 1;
  if (OH <= 0 || OW <= 0) return ROUGE_B200_EINVAL;
  // im2col TMA limits: corners in [-128, 127], filter offsets below 256,
  // traversal stride up to 8.
  if (pad > 128 || pad - (KW - 1) < -128 || pad - (KH - 1) < -128 || KH > 256 || KW > 256 ||
      stride > 8)
    return ROUGE_B200_EUNSUPPORTED;
  const bool f32 = type == ROUGE_B200_T_F32;
  p.OH = static_cast<int>(OH);
  p.OW = static_cast<int>(OW);
  p.P = H * W;
  p.es = f32 ? 4 : 2;
  p.Cp = static_cast<int>(rup(Cin, f32 ? 32 : 64));
  p.Cs = f32 ? 3 * p.Cp : p.Cp;
  const size_t img = static_cast<size_t>(p.P) * p.Cs * p.es;
  p.Np = static_cast<size_t>(N) * img >= 131072 ? N : static_cast<int>((131072 + img - 1) / img);
  p.Cop = static_cast<int>(rup(Cout, 4));
  if (static_cast<long long>(p.Np) * OH * OW > 0x7fffffffLL ||
      static_cast<long long>(KH) * KW * p.Cs > 0x7fffffffLL)
    return ROUGE_B200_EUNSUPPORTED;
  p.pack_x = f32 || x_layout != ROUGE_B200_NHWC || p.Cs != Cin || p.Np != N || !aligned16(X);
  p.pack_w = f32 || w_layout != ROUGE_B200_NHWC || p.Cs != Cin || p.Cop != Cout || !aligned16(Wt);
  p.stage_y = y_layout != ROUGE_B200_NHWC || p.Np != N || (Cout * p.es) % 16 != 0 || !aligned16(Y);
  p.x_bytes = static_cast<size_t>(p.Np) * img;
  p.w_bytes = static_cast<size_t>(p.Cop) * KH * KW * p.Cs * p.es;
  p.t_bytes = static_cast<size_t>(p.Np) * p.OH * p.OW * p.Cop * 4;
  return ROUGE_B200_OK;
}

__device__ __forceinline__ float load_as_f32(const uint16_t *y, long long i, int half) {
  const uint16_t b = y[i];
  return half ? __half2float(__ushort_as_half(b)) : __uint_as_float(static_cast<uint32_t>(b) << 16);
}

__device__ __forceinline__ uint16_t to_16(float v, int half) {
  return half ? __half_as_ushort(__float2half_rn(v)) : __bfloat16_as_ushort(__float2bfloat16_rn(v));
}

// y = alpha * t + beta * y (y read only when beta != 0), rounded to Y's type.
template <class YT>
__device__ __forceinline__ void finish_one(const float t, float alpha, float beta, YT *Y,
                                           long long i, int half) {
  float r = __fmul_rn(alpha, t);
  if constexpr (sizeof(YT) == 4) {
    if (beta != 0.0f) r = __fadd_rn(r, __fmul_rn(beta, Y[i]));
    Y[i] = r;
  } else {
    if (beta != 0.0f) r = __fadd_rn(r, __fmul_rn(beta, load_as_f32(Y, i, half)));
    Y[i] = to_16(r, half);
  }
}

// T [n*P + p][ldt] (f32) -> Y, P = OH*OW output pixels per image, for
// images n < N. NHWC: straight rows. NCHW: 32 x 32 (pixel x channel) tiles
// transposed through shared memory (grid x: pixels, y: channels, z: image).
template <class YT>
__global__ void finish_nhwc(const float *__restrict__ T, long long ldt, long long rows, int Cout,
                            float alpha, float beta, YT *Y, int half) {
  const long long total = rows * Cout;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long r = i / Cout;
    const int c = static_cast<int>(i - r * Cout);
    finish_one(T[r * ldt + c], alpha, beta, Y, i, half);
  }
}

template <class YT>
__global__ void finish_nchw(const float *__restrict__ T, long long ldt, int P, int Cout,
                            float alpha, float beta, YT *Y, int half) {
  __shared__ float t[kPackTile][kPackTile + 1];
  const int n = blockIdx.z;
  const int p0 = blockIdx.x * kPackTile, c0 = blockIdx.y * kPackTile;
  const float *Tn = T + static_cast<long long>(n) * P * ldt;
  for (int i = threadIdx.y; i < kPackTile; i += blockDim.y) {
    const int p = p0 + i, c = c0 + threadIdx.x;
    t[i][threadIdx.x] = (p < P && c < Cout) ? Tn[static_cast<long long>(p) * ldt + c] : 0.0f;
  }
  __syncthreads();
  YT *Yn = Y + static_cast<long long>(n) * Cout * P;
  for (int i = threadIdx.y; i < kPackTile; i += blockDim.y) {
    const int c = c0 + i, p = p0 + threadIdx.x;
    if (c < Cout && p < P)
      finish_one(t[threadIdx.x][i], alpha, beta, Yn, static_cast<long long>(c) * P + p, half);
  }
}

template <class YT>
int finish(const float *T, long long ldt, int N, int P, int Cout, int y_layout, float alpha,
           float beta, void *Y, int half, cudaStream_t st) {
  YT *y = static_cast<YT *>(Y);
  if (y_layout == ROUGE_B200_NHWC) {
    const long long total = static_cast<long long>(N) * P * Cout;
    const long long blocks = (total + 255) / 256;
    finish_nhwc<YT><<<static_cast<unsigned>(blocks < 148 * 16 ? blocks : 148 * 16), 256, 0, st>>>(
        T, ldt, static_cast<long long>(N) * P, Cout, alpha, beta, y, half);
    return cuda_status(cudaGetLastError());
  }
  for (int n0 = 0; n0 < N; n0 += 65535) {
    const int nz = N - n0 < 65535 ? N - n0 : 65535;
    const dim3 grid((P + kPackTile - 1) / kPackTile, (Cout + kPackTile - 1) / kPackTile, nz);
    finish_nchw<YT><<<grid, dim3(kPackTile, 8), 0, st>>>(
        T + static_cast<long long>(n0) * P * ldt, ldt, P, Cout, alpha, beta,
        y + static_cast<long long>(n0) * Cout * P, half);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e);
  }
  return ROUGE_B200_OK;
}

template <class T>
int pack_operands(const ConvPlan &p, int N, int Cin, int Cout, int KH, int KW, int x_layout,
                  int w_layout, const void *X, const void *Wt, void *Xp, void *Wp, int f32,
                  cudaStream_t st) {
  int s = ROUGE_B200_OK;
  const int taps = KH * KW;
  const long long kp = p.Cs;  // row pitch (elements) of X' and W'
  if (p.pack_x) {
    // image n: X'[n][pix][c] = X(n, c, pix); NCHW: c stride P, NHWC: pix stride Cin
    const long long sr = x_layout == ROUGE_B200_NCHW ? 1 : Cin;
    const long long sp = x_layout == ROUGE_B200_NCHW ? p.P : 1;
    s = pack_launch<T>(X, static_cast<long long>(Cin) * p.P, sr, sp, p.P, Cin, p.Cp, f32 ? 1 : 0,
                       Xp, static_cast<long long>(p.P) * kp, kp, N, st);
    if (s == ROUGE_B200_OK && p.Np > N) {
      const size_t img = static_cast<size_t>(p.P) * kp * sizeof(T);
      s = cuda_status(cudaMemsetAsync(static_cast<uint8_t *>(Xp) + N * img, 0, (p.Np - N) * img, st));
    }
    if (s != ROUGE_B200_OK) return s;
  }
  if (p.pack_w) {
    if (w_layout == ROUGE_B200_NHWC)  // rows (co, tap), channels contiguous
      s = pack_launch<T>(Wt, 0, Cin, 1, Cout * taps, Cin, p.Cp, f32 ? 2 : 0, Wp, 0, kp, 1, st);
    else  // filter co: [c][tap] -> rows tap, channel stride taps
      s = pack_launch<T>(Wt, static_cast<long long>(Cin) * taps, 1, taps, taps, Cin, p.Cp,
                         f32 ? 2 : 0, Wp, taps * kp, kp, Cout, st);
    if (s == ROUGE_B200_OK && p.Cop > Cout) {
      const size_t filt = static_cast<size_t>(taps) * kp * sizeof(T);
      s = cuda_status(cudaMemsetAsync(static_cast<uint8_t *>(Wp) + Cout * filt, 0,
                                      (p.Cop - Cout) * filt, st));
    }
  }
  return s;
}

}  // namespace
}  // namespace rb200

using namespace rb200;

extern "C" {

size_t rouge_b200_conv2d_forward_workspace(int N, int Cin, int H, int W, int Cout, int KH, int KW,
                                           int stride, int pad, int type, int x_layout,
                                           int w_layout, int y_layout) {
  ConvPlan p;
  if (make_plan(N, Cin, H, W, Cout, KH, KW, stride, pad, type, x_layout, w_layout, y_layout,
                nullptr, nullptr, nullptr, p) != ROUGE_B200_OK)
    return 0;
  return p.need();
}

int rouge_b200_conv2d_forward(int N, int Cin, int H, int W, int Cout, int KH, int KW, int stride,
                              int pad, int type, float alpha, const void *X, int x_layout,
                              const void *Wt, int w_layout, float beta, void *Y, int y_layout,
                              void *workspace, size_t workspace_bytes, void *stream) {
  if (!X || !Wt || !Y) return set_status(ROUGE_B200_EINVAL);
  ConvPlan p;
  int s = make_plan(N, Cin, H, W, Cout, KH, KW, stride, pad, type, x_layout, w_layout, y_layout, X,
                    Wt, Y, p);
  if (s != ROUGE_B200_OK) return set_status(s);
  const size_t need = p.need();
  if (need && (!workspace || workspace_bytes < need ||
               (reinterpret_cast<uintptr_t>(workspace) & 255u)))
    return set_status(ROUGE_B200_ETOOBIG);
  s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  cudaStream_t st = as_stream(stream);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  void *Xp = p.pack_x ? ws : const_cast<void *>(X);
  if (p.pack_x) ws += rup(p.x_bytes, 256);
  void *Wp = p.pack_w ? ws : const_cast<void *>(Wt);
  if (p.pack_w) ws += rup(p.w_bytes, 256);
  float *T = p.stage_y ? reinterpret_cast<float *>(ws) : nullptr;
  const bool f32 = type == ROUGE_B200_T_F32;
  s = f32 ? pack_operands<uint32_t>(p, N, Cin, Cout, KH, KW, x_layout, w_layout, X, Wt, Xp, Wp, 1, st)
          : pack_operands<uint16_t>(p, N, Cin, Cout, KH, KW, x_layout, w_layout, X, Wt, Xp, Wp, 0,
                                    st);
  if (s != ROUGE_B200_OK) return set_status(s);
  const int gemm_n = p.pack_w ? p.Cop : Cout;
  if (!p.stage_y)
    return launch_conv_blas(type, p.Np, H, W, p.Cs, Cout, KH, KW, stride, pad, Xp, Wp, alpha, beta,
                            Y, Cout, type, st);
  s = launch_conv_blas(type, p.Np, H, W, p.Cs, gemm_n, KH, KW, stride, pad, Xp, Wp, 1.0f, 0.0f, T,
                       p.Cop, ROUGE_B200_T_F32, st);
  if (s != ROUGE_B200_OK) return s;
  const int opix = p.OH * p.OW;
  s = f32 ? finish<float>(T, p.Cop, N, opix, Cout, y_layout, alpha, beta, Y, 0, st)
          : finish<uint16_t>(T, p.Cop, N, opix, Cout, y_layout, alpha, beta, Y,
                             type == ROUGE_B200_T_F16 ? 1 : 0, st);
  return s == ROUGE_B200_OK ? s : set_status(s);
}

}  // extern "C"
