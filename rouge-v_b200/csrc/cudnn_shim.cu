// librouge_b200_cudnn.so: the cuDNN API subset of include/rouge/cudnn_b200.h.
// Convolution forward runs on rouge_b200_conv2d_forward (the sm_100a
// implicit-GEMM kernel of librouge_b200.so); the element-wise operations
// are the kernels below, with the reference's arithmetic (cudnn_shim.cpp)
// written out operation by operation so that no multiply-add is fused
// where the reference rounds twice.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdint>
#include <mutex>
#include <new>

#include "rouge/cudnn_b200.h"
#include "rouge/numerics_b200.h"
#include "shim_stage.h"

using rb200shim::DevBuf;
using rb200shim::Staging;

struct rouge_b200_cudnn_ctx {
  int magic;
  cudaStream_t stream;
  DevBuf ws;     // convolution workspace when the caller's is too small
  DevBuf stage;  // host operands
  DevBuf scratch;
  std::mutex lock;
};
struct rouge_b200_cudnn_tensor {
  int n, c, h, w;
  cudnnDataType_t type;
  cudnnTensorFormat_t format;
};
struct rouge_b200_cudnn_filter {
  int k, c, h, w;
  cudnnDataType_t type;
  cudnnTensorFormat_t format;
};
struct rouge_b200_cudnn_conv {
  int pad_h, pad_w, stride_h, stride_w;
};
struct rouge_b200_cudnn_act {
  cudnnActivationMode_t mode;
  double coef;
};

namespace {

constexpr int kMagic = 0x52424e4e;  // "RBNN"

bool valid(cudnnHandle_t h) { return h && h->magic == kMagic; }

cudnnStatus_t map_status(int s) {
  switch (s) {
    case ROUGE_B200_OK: return CUDNN_STATUS_SUCCESS;
    case ROUGE_B200_EINVAL: return CUDNN_STATUS_BAD_PARAM;
    case ROUGE_B200_EUNSUPPORTED: return CUDNN_STATUS_NOT_SUPPORTED;
    case ROUGE_B200_ENODEV: return CUDNN_STATUS_ARCH_MISMATCH;
    case ROUGE_B200_ENOMEM:
    case ROUGE_B200_ETOOBIG: return CUDNN_STATUS_ALLOC_FAILED;
    default: return CUDNN_STATUS_EXECUTION_FAILED;
  }
}

int rb_type(cudnnDataType_t t) {
  switch (t) {
    case CUDNN_DATA_FLOAT: return ROUGE_B200_T_F32;
    case CUDNN_DATA_HALF: return ROUGE_B200_T_F16;
    case CUDNN_DATA_BFLOAT16: return ROUGE_B200_T_BF16;
    default: return -1;
  }
}

size_t esize(cudnnDataType_t t) { return t == CUDNN_DATA_FLOAT ? 4 : 2; }

size_t elems(const rouge_b200_cudnn_tensor *d) {
  return static_cast<size_t>(d->n) * d->c * d->h * d->w;
}

bool valid_format(cudnnTensorFormat_t f) { return f == CUDNN_TENSOR_NCHW || f == CUDNN_TENSOR_NHWC; }

// x / y of an element-wise operation: same dims, type and format.
bool same_tensor(const rouge_b200_cudnn_tensor *a, const rouge_b200_cudnn_tensor *b) {
  return a && b && a->type == b->type && a->format == b->format && a->n == b->n &&
         a->c == b->c && a->h == b->h && a->w == b->w && valid_format(a->format);
}

cudnnStatus_t finish_call(Staging &sg, cudaError_t launch) {
  const bool ok = sg.finish();
  if (launch != cudaSuccess) return CUDNN_STATUS_EXECUTION_FAILED;
  return ok ? CUDNN_STATUS_SUCCESS : CUDNN_STATUS_EXECUTION_FAILED;
}

unsigned grid_for(size_t n) {
  const size_t b = (n + 255) / 256;
  return static_cast<unsigned>(b < 148 * 8 ? (b ? b : 1) : 148 * 8);
}

// ------------------------------------------------------------ element I/O

template <class T>
struct Elem;
template <>
struct Elem<float> {
  static __device__ __forceinline__ float ld(const float *p, size_t i, int) { return p[i]; }
  static __device__ __forceinline__ void st(float *p, size_t i, float v, int) { p[i] = v; }
};
template <>
struct Elem<uint16_t> {  // f16 (half != 0) or bf16 bits
  static __device__ __forceinline__ float ld(const uint16_t *p, size_t i, int half) {
    return half ? __half2float(__ushort_as_half(p[i]))
                : __uint_as_float(static_cast<uint32_t>(p[i]) << 16);
  }
  static __device__ __forceinline__ void st(uint16_t *p, size_t i, float v, int half) {
    p[i] = half ? __half_as_ushort(__float2half_rn(v)) : __bfloat16_as_ushort(__float2bfloat16_rn(v));
  }
};

// ------------------------------------------------------------ activation

// cudnn_shim.cpp:271-294: a = act(v); y = alpha * a + beta * y, in f32
// with two rounded products and one rounded sum (y not read when
// beta == 0).
template <class T>
__global__ void activation_kernel(const T *__restrict__ x, T *y, size_t n, int mode, float coef,
                                  int coef_pos, float alpha, float beta, int half) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const float v = Elem<T>::ld(x, i, half);
    float a = 0.0f;
    switch (mode) {
      case CUDNN_ACTIVATION_RELU: a = v > 0.0f ? v : 0.0f; break;
      case CUDNN_ACTIVATION_CLIPPED_RELU: a = v < 0.0f ? 0.0f : (coef_pos && v > coef ? coef : v); break;
      case CUDNN_ACTIVATION_SIGMOID: a = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-v))); break;
      default: a = tanhf(v); break;
    }
    float r = __fmul_rn(alpha, a);
    if (beta != 0.0f) r = __fadd_rn(r, __fmul_rn(beta, Elem<T>::ld(y, i, half)));
    Elem<T>::st(y, i, r, half);
  }
}

// ------------------------------------------------------------ add tensor

// cudnn_shim.cpp:309-312: B = alpha1 * A + alpha2 * B. A's dims are B's
// or 1; (sn, sc, sh, sw) are A's element strides, 0 along broadcast dims.
template <class T>
__global__ void add_kernel(const T *__restrict__ A, T *B, size_t n, int C, int H, int W, int nhwc,
                           long long sn, long long sc, long long sh, long long sw, float a1,
                           float a2, int half) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    int c, h, w;
    size_t r;
    if (nhwc) {
      c = static_cast<int>(i % C);
      r = i / C;
      w = static_cast<int>(r % W);
      r /= W;
      h = static_cast<int>(r % H);
      r /= H;
    } else {
      w = static_cast<int>(i % W);
      r = i / W;
      h = static_cast<int>(r % H);
      r /= H;
      c = static_cast<int>(r % C);
      r /= C;
    }
    const size_t ai = r * sn + c * sc + h * sh + w * sw;
    float v = __fmul_rn(a1, Elem<T>::ld(A, ai, half));
    if (a2 != 0.0f) v = __fadd_rn(v, __fmul_rn(a2, Elem<T>::ld(B, i, half)));
    Elem<T>::st(B, i, v, half);
  }
}

// ------------------------------------------------------------ softmax

// cudnn_shim.cpp:335-348 for one row of `len` values at stride `stride`:
// maximum and sum of exp(x - max) in double, then
//   v = LOG ? x - max - log(sum) : exp(x - max) / sum
//   y = (float)(alpha * v + (float)(beta * y))
__device__ __forceinline__ void softmax_out(const float *x, float *y, size_t k, double mx,
                                            double sum, double lsum, int is_log, float alpha,
                                            float beta) {
  const double d = __dsub_rn(static_cast<double>(x[k]), mx);
  const double v = is_log ? __dsub_rn(d, lsum) : __ddiv_rn(exp(d), sum);
  const float by = beta != 0.0f ? __fmul_rn(beta, y[k]) : 0.0f;
  y[k] = __double2float_rn(__dadd_rn(__dmul_rn(static_cast<double>(alpha), v), static_cast<double>(by)));
}

__device__ __forceinline__ double warp_max(double v) {
  for (int o = 16; o; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ double warp_sum(double v) {
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// One block per row of `len` contiguous values (INSTANCE mode: an image).
constexpr int kSoftmaxThreads = 512;
__global__ void __launch_bounds__(kSoftmaxThreads) softmax_rows_kernel(const float *__restrict__ x, float *y, size_t len, int is_log,
                                    float alpha, float beta) {
  __shared__ double red[32];
  const float *xr = x + blockIdx.x * len;
  float *yr = y + blockIdx.x * len;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  double m = -INFINITY;
  for (size_t k = threadIdx.x; k < len; k += blockDim.x) m = fmax(m, static_cast<double>(xr[k]));
  m = warp_max(m);
  if (lane == 0) red[warp] = m;
  __syncthreads();
  if (warp == 0) {
    double t = lane < nw ? red[lane] : -INFINITY;
    t = warp_max(t);
    if (lane == 0) red[0] = t;
  }
  __syncthreads();
  const double mx = red[0];
  __syncthreads();
  double s = 0.0;
  for (size_t k = threadIdx.x; k < len; k += blockDim.x)
    s += exp(__dsub_rn(static_cast<double>(xr[k]), mx));
  s = warp_sum(s);
  if (lane == 0) red[warp] = s;
  __syncthreads();
  if (warp == 0) {
    double t = lane < nw ? red[lane] : 0.0;
    t = warp_sum(t);
    if (lane == 0) red[0] = t;
  }
  __syncthreads();
  const double sum = red[0];
  const double lsum = log(sum);
  for (size_t k = threadIdx.x; k < len; k += blockDim.x)
    softmax_out(xr, yr, k, mx, sum, lsum, is_log, alpha, beta);
}

// CHANNEL mode: one thread per (n, pixel) over its C values at stride
// `cstride` (NCHW: HW, pixels of a warp adjacent; NHWC: 1).
__global__ void softmax_channel_kernel(const float *__restrict__ x, float *y, int N, int C,
                                       long long HW, int nhwc, int is_log, float alpha, float beta) {
  const long long total = static_cast<long long>(N) * HW;
  for (long long t = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long n = t / HW, p = t - n * HW;
    const size_t base = nhwc ? static_cast<size_t>(t) * C : static_cast<size_t>(n) * C * HW + p;
    const long long cs = nhwc ? 1 : HW;
    const float *xr = x + base;
    float *yr = y + base;
    double mx = -INFINITY;
    for (int c = 0; c < C; ++c) mx = fmax(mx, static_cast<double>(xr[c * cs]));
    double sum = 0.0;
    for (int c = 0; c < C; ++c) sum += exp(__dsub_rn(static_cast<double>(xr[c * cs]), mx));
    const double lsum = log(sum);
    for (int c = 0; c < C; ++c) softmax_out(xr, yr, c * cs, mx, sum, lsum, is_log, alpha, beta);
  }
}

// ------------------------------------------------------------ batch norm

// cudnn_shim.cpp:396-404 per channel: inv = 1 / sqrt(var + eps),
// s = scale * inv, b = bias - (float)(scale * mean) * inv, in double.
__global__ void bn_prep_kernel(const float *S, const float *B, const float *M, const float *V,
                               int C, double eps, double *sb) {
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < C; c += gridDim.x * blockDim.x) {
    const double inv = __ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(static_cast<double>(V[c]), eps)));
    sb[2 * c] = __dmul_rn(static_cast<double>(S[c]), inv);
    sb[2 * c + 1] = __dsub_rn(static_cast<double>(B[c]),
                              __dmul_rn(static_cast<double>(__fmul_rn(S[c], M[c])), inv));
  }
}

// y = (float)(alpha * (s * x + b) + (float)(beta * y)).
__global__ void bn_apply_kernel(const float *__restrict__ x, float *y, size_t n, int C,
                                long long HW, int nhwc, const double *__restrict__ sb, float alpha,
                                float beta) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const int c = nhwc ? static_cast<int>(i % C) : static_cast<int>((i / HW) % C);
    const double v = __dadd_rn(__dmul_rn(sb[2 * c], static_cast<double>(x[i])), sb[2 * c + 1]);
    const float by = beta != 0.0f ? __fmul_rn(beta, y[i]) : 0.0f;
    y[i] = __double2float_rn(
        __dadd_rn(__dmul_rn(static_cast<double>(alpha), v), static_cast<double>(by)));
  }
}

template <class T>
T read_host(const void *p) {
  T v;
  __builtin_memcpy(&v, p, sizeof(T));
  return v;
}

}  // namespace

extern "C" {

const char *cudnnGetErrorString(cudnnStatus_t s) {
  switch (s) {
    case CUDNN_STATUS_SUCCESS: return "CUDNN_STATUS_SUCCESS";
    case CUDNN_STATUS_NOT_INITIALIZED: return "CUDNN_STATUS_NOT_INITIALIZED";
    case CUDNN_STATUS_ALLOC_FAILED: return "CUDNN_STATUS_ALLOC_FAILED";
    case CUDNN_STATUS_BAD_PARAM: return "CUDNN_STATUS_BAD_PARAM";
    case CUDNN_STATUS_INTERNAL_ERROR: return "CUDNN_STATUS_INTERNAL_ERROR";
    case CUDNN_STATUS_INVALID_VALUE: return "CUDNN_STATUS_INVALID_VALUE";
    case CUDNN_STATUS_ARCH_MISMATCH: return "CUDNN_STATUS_ARCH_MISMATCH";
    case CUDNN_STATUS_MAPPING_ERROR: return "CUDNN_STATUS_MAPPING_ERROR";
    case CUDNN_STATUS_EXECUTION_FAILED: return "CUDNN_STATUS_EXECUTION_FAILED";
    case CUDNN_STATUS_NOT_SUPPORTED: return "CUDNN_STATUS_NOT_SUPPORTED";
    case CUDNN_STATUS_LICENSE_ERROR: return "CUDNN_STATUS_LICENSE_ERROR";
  }
  return "CUDNN_STATUS_UNKNOWN";
}

cudnnStatus_t cudnnCreate(cudnnHandle_t *h) {
  if (!h) return CUDNN_STATUS_BAD_PARAM;
  if (!rouge_b200_device_ok()) return CUDNN_STATUS_NOT_INITIALIZED;
  auto *c = new (std::nothrow) rouge_b200_cudnn_ctx();
  if (!c) return CUDNN_STATUS_ALLOC_FAILED;
  c->magic = kMagic;
  c->stream = nullptr;
  *h = c;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnDestroy(cudnnHandle_t h) {
  if (!valid(h)) return CUDNN_STATUS_BAD_PARAM;
  h->ws.release(h->stream);
  h->stage.release(h->stream);
  h->scratch.release(h->stream);
  h->magic = 0;
  delete h;
  return CUDNN_STATUS_SUCCESS;
}

size_t cudnnGetVersion(void) { return 300; }  // cudnn_shim.cpp:81: the shim's own version, 0.3.0

cudnnStatus_t cudnnSetStream(cudnnHandle_t h, cudaStream_t s) {
  if (!valid(h)) return CUDNN_STATUS_BAD_PARAM;
  std::lock_guard<std::mutex> g(h->lock);
  h->stream = s;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnGetStream(cudnnHandle_t h, cudaStream_t *s) {
  if (!valid(h) || !s) return CUDNN_STATUS_BAD_PARAM;
  *s = h->stream;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnCreateTensorDescriptor(cudnnTensorDescriptor_t *d) {
  if (!d) return CUDNN_STATUS_BAD_PARAM;
  auto *t = new (std::nothrow) rouge_b200_cudnn_tensor{0, 0, 0, 0, CUDNN_DATA_FLOAT, CUDNN_TENSOR_NCHW};
  if (!t) return CUDNN_STATUS_ALLOC_FAILED;
  *d = t;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnSetTensor4dDescriptor(cudnnTensorDescriptor_t d, cudnnTensorFormat_t f,
                                         cudnnDataType_t t, int n, int c, int h, int w) {
  if (!d || n <= 0 || c <= 0 || h <= 0 || w <= 0) return CUDNN_STATUS_BAD_PARAM;
  *d = rouge_b200_cudnn_tensor{n, c, h, w, t, f};
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnDestroyTensorDescriptor(cudnnTensorDescriptor_t d) {
  if (!d) return CUDNN_STATUS_BAD_PARAM;
  delete d;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnCreateFilterDescriptor(cudnnFilterDescriptor_t *d) {
  if (!d) return CUDNN_STATUS_BAD_PARAM;
  auto *f = new (std::nothrow) rouge_b200_cudnn_filter{0, 0, 0, 0, CUDNN_DATA_FLOAT, CUDNN_TENSOR_NCHW};
  if (!f) return CUDNN_STATUS_ALLOC_FAILED;
  *d = f;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnSetFilter4dDescriptor(cudnnFilterDescriptor_t d, cudnnDataType_t t,
                                         cudnnTensorFormat_t f, int k, int c, int h, int w) {
  if (!d || k <= 0 || c <= 0 || h <= 0 || w <= 0) return CUDNN_STATUS_BAD_PARAM;
  *d = rouge_b200_cudnn_filter{k, c, h, w, t, f};
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnDestroyFilterDescriptor(cudnnFilterDescriptor_t d) {
  if (!d) return CUDNN_STATUS_BAD_PARAM;
  delete d;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnCreateConvolutionDescriptor(cudnnConvolutionDescriptor_t *d) {
  if (!d) return CUDNN_STATUS_BAD_PARAM;
  auto *c = new (std::nothrow) rouge_b200_cudnn_conv{0, 0, 1, 1};
  if (!c) return CUDNN_STATUS_ALLOC_FAILED;
  *d = c;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnSetConvolution2dDescriptor(cudnnConvolutionDescriptor_t d, int pad_h, int pad_w,
                                              int stride_h, int stride_w, int dil_h, int dil_w,
                                              int mode, cudnnDataType_t) {
  if (!d || pad_h < 0 || pad_w < 0 || stride_h <= 0 || stride_w <= 0) return CUDNN_STATUS_BAD_PARAM;
  if (pad_h != pad_w || stride_h != stride_w || dil_h != 1 || dil_w != 1 || mode != 0)
    return CUDNN_STATUS_NOT_SUPPORTED;
  *d = rouge_b200_cudnn_conv{pad_h, pad_w, stride_h, stride_w};
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnDestroyConvolutionDescriptor(cudnnConvolutionDescriptor_t d) {
  if (!d) return CUDNN_STATUS_BAD_PARAM;
  delete d;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnGetConvolution2dForwardOutputDim(const cudnnConvolutionDescriptor_t conv,
                                                    const cudnnTensorDescriptor_t in,
                                                    const cudnnFilterDescriptor_t f, int *n,
                                                    int *c, int *h, int *w) {
  if (!conv || !in || !f || !n || !c || !h || !w) return CUDNN_STATUS_BAD_PARAM;
  *n = in->n;
  *c = f->k;
  *h = (in->h + 2 * conv->pad_h - f->h) / conv->stride_h + 1;
  *w = (in->w + 2 * conv->pad_w - f->w) / conv->stride_w + 1;
  if (*h <= 0 || *w <= 0) return CUDNN_STATUS_BAD_PARAM;
  return CUDNN_STATUS_SUCCESS;
}

}  // extern "C"

namespace {

// Argument checks of cudnn_shim.cpp:194-216, with FLOAT / HALF / BFLOAT16
// in either format accepted.
cudnnStatus_t check_conv(const cudnnTensorDescriptor_t xD, const cudnnFilterDescriptor_t wD,
                         const cudnnConvolutionDescriptor_t conv, cudnnConvolutionFwdAlgo_t algo,
                         const cudnnTensorDescriptor_t yD) {
  if (xD->type != wD->type || xD->type != yD->type || rb_type(xD->type) < 0)
    return CUDNN_STATUS_NOT_SUPPORTED;
  if (!valid_format(xD->format) || !valid_format(yD->format) || !valid_format(wD->format))
    return CUDNN_STATUS_NOT_SUPPORTED;
  if (xD->c != wD->c || yD->c != wD->k || yD->n != xD->n) return CUDNN_STATUS_BAD_PARAM;
  if (algo != CUDNN_CONVOLUTION_FWD_ALGO_IMPLICIT_GEMM && algo != CUDNN_CONVOLUTION_FWD_ALGO_GEMM &&
      algo != CUDNN_CONVOLUTION_FWD_ALGO_DIRECT && algo != CUDNN_CONVOLUTION_FWD_ALGO_WINOGRAD)
    return CUDNN_STATUS_NOT_SUPPORTED;
  const int OH = (xD->h + 2 * conv->pad_h - wD->h) / conv->stride_h + 1;
  const int OW = (xD->w + 2 * conv->pad_w - wD->w) / conv->stride_w + 1;
  if (yD->h != OH || yD->w != OW) return CUDNN_STATUS_BAD_PARAM;
  return CUDNN_STATUS_SUCCESS;
}

int layout(cudnnTensorFormat_t f) { return f == CUDNN_TENSOR_NHWC ? ROUGE_B200_NHWC : ROUGE_B200_NCHW; }

size_t conv_ws(const cudnnTensorDescriptor_t xD, const cudnnFilterDescriptor_t wD,
               const cudnnConvolutionDescriptor_t conv, const cudnnTensorDescriptor_t yD) {
  return rouge_b200_conv2d_forward_workspace(xD->n, xD->c, xD->h, xD->w, wD->k, wD->h, wD->w,
                                             conv->stride_h, conv->pad_h, rb_type(xD->type),
                                             layout(xD->format), layout(wD->format),
                                             layout(yD->format));
}

}  // namespace

extern "C" {

cudnnStatus_t cudnnGetConvolutionForwardWorkspaceSize(cudnnHandle_t handle,
                                                      const cudnnTensorDescriptor_t xD,
                                                      const cudnnFilterDescriptor_t wD,
                                                      const cudnnConvolutionDescriptor_t conv,
                                                      const cudnnTensorDescriptor_t yD,
                                                      cudnnConvolutionFwdAlgo_t algo,
                                                      size_t *bytes) {
  if (!valid(handle)) return CUDNN_STATUS_NOT_INITIALIZED;
  if (!xD || !wD || !conv || !yD || !bytes) return CUDNN_STATUS_BAD_PARAM;
  const cudnnStatus_t s = check_conv(xD, wD, conv, algo, yD);
  if (s != CUDNN_STATUS_SUCCESS) return s;
  *bytes = conv_ws(xD, wD, conv, yD);
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnConvolutionForward(cudnnHandle_t handle, const void *alpha,
                                      const cudnnTensorDescriptor_t xD, const void *x,
                                      const cudnnFilterDescriptor_t wD, const void *w,
                                      const cudnnConvolutionDescriptor_t conv,
                                      cudnnConvolutionFwdAlgo_t algo, void *workSpace,
                                      size_t workSpaceSizeInBytes, const void *beta,
                                      const cudnnTensorDescriptor_t yD, void *y) {
  if (!valid(handle)) return CUDNN_STATUS_NOT_INITIALIZED;
  if (!alpha || !xD || !x || !wD || !w || !conv || !beta || !yD || !y) return CUDNN_STATUS_BAD_PARAM;
  cudnnStatus_t cs = check_conv(xD, wD, conv, algo, yD);
  if (cs != CUDNN_STATUS_SUCCESS) return cs;
  std::lock_guard<std::mutex> g(handle->lock);
  const float al = read_host<float>(alpha), be = read_host<float>(beta);
  const size_t es = esize(xD->type);
  Staging sg(handle->stage, handle->stream);
  sg.add(x, elems(xD) * es, true, false);
  sg.add(w, static_cast<size_t>(wD->k) * wD->c * wD->h * wD->w * es, true, false);
  sg.add(y, elems(yD) * es, be != 0.0f, true);
  if (!sg.begin()) return CUDNN_STATUS_ALLOC_FAILED;
  const size_t need = conv_ws(xD, wD, conv, yD);
  void *ws = workSpace;
  size_t ws_bytes = workSpaceSizeInBytes;
  if (need && (!ws || ws_bytes < need || (reinterpret_cast<uintptr_t>(ws) & 255u) ||
               rb200shim::is_host_memory(ws))) {
    if (!handle->ws.ensure(need, handle->stream)) return CUDNN_STATUS_ALLOC_FAILED;
    ws = handle->ws.p;
    ws_bytes = handle->ws.bytes;
  }
  const int s = rouge_b200_conv2d_forward(
      xD->n, xD->c, xD->h, xD->w, wD->k, wD->h, wD->w, conv->stride_h, conv->pad_h,
      rb_type(xD->type), al, sg.dev(x), layout(xD->format), sg.dev(w), layout(wD->format), be,
      sg.dev(y), layout(yD->format), ws, ws_bytes, handle->stream);
  if (s != ROUGE_B200_OK) {
    sg.finish();
    return map_status(s);
  }
  return sg.finish() ? CUDNN_STATUS_SUCCESS : CUDNN_STATUS_EXECUTION_FAILED;
}

cudnnStatus_t cudnnCreateActivationDescriptor(cudnnActivationDescriptor_t *d) {
  if (!d) return CUDNN_STATUS_BAD_PARAM;
  auto *a = new (std::nothrow) rouge_b200_cudnn_act{CUDNN_ACTIVATION_RELU, 0.0};
  if (!a) return CUDNN_STATUS_ALLOC_FAILED;
  *d = a;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnSetActivationDescriptor(cudnnActivationDescriptor_t d, cudnnActivationMode_t mode,
                                           cudnnNanPropagation_t, double coef) {
  if (!d) return CUDNN_STATUS_BAD_PARAM;
  if (mode != CUDNN_ACTIVATION_SIGMOID && mode != CUDNN_ACTIVATION_RELU &&
      mode != CUDNN_ACTIVATION_TANH && mode != CUDNN_ACTIVATION_CLIPPED_RELU)
    return CUDNN_STATUS_NOT_SUPPORTED;
  d->mode = mode;
  d->coef = coef;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnDestroyActivationDescriptor(cudnnActivationDescriptor_t d) {
  if (!d) return CUDNN_STATUS_BAD_PARAM;
  delete d;
  return CUDNN_STATUS_SUCCESS;
}

cudnnStatus_t cudnnActivationForward(cudnnHandle_t handle, cudnnActivationDescriptor_t act,
                                     const void *alpha, const cudnnTensorDescriptor_t xD,
                                     const void *x, const void *beta,
                                     const cudnnTensorDescriptor_t yD, void *y) {
  if (!valid(handle)) return CUDNN_STATUS_NOT_INITIALIZED;
  if (!act || !alpha || !xD || !x || !beta || !yD || !y) return CUDNN_STATUS_BAD_PARAM;
  if (!same_tensor(xD, yD) || rb_type(xD->type) < 0) return CUDNN_STATUS_NOT_SUPPORTED;
  std::lock_guard<std::mutex> g(handle->lock);
  const float al = read_host<float>(alpha), be = read_host<float>(beta);
  const size_t n = elems(xD), es = esize(xD->type);
  Staging sg(handle->stage, handle->stream);
  sg.add(x, n * es, true, false);
  sg.add(y, n * es, be != 0.0f || x == y, true);
  if (!sg.begin()) return CUDNN_STATUS_ALLOC_FAILED;
  const float coef = static_cast<float>(act->coef);
  const int coef_pos = act->coef > 0.0 ? 1 : 0;
  if (xD->type == CUDNN_DATA_FLOAT)
    activation_kernel<float><<<grid_for(n), 256, 0, handle->stream>>>(
        static_cast<const float *>(sg.dev(x)), static_cast<float *>(sg.dev(y)), n, act->mode, coef,
        coef_pos, al, be, 0);
  else
    activation_kernel<uint16_t><<<grid_for(n), 256, 0, handle->stream>>>(
        static_cast<const uint16_t *>(sg.dev(x)), static_cast<uint16_t *>(sg.dev(y)), n, act->mode,
        coef, coef_pos, al, be, xD->type == CUDNN_DATA_HALF ? 1 : 0);
  return finish_call(sg, cudaGetLastError());
}

cudnnStatus_t cudnnAddTensor(cudnnHandle_t handle, const void *alpha1,
                             const cudnnTensorDescriptor_t aD, const void *A, const void *alpha2,
                             const cudnnTensorDescriptor_t bD, void *B) {
  if (!valid(handle)) return CUDNN_STATUS_NOT_INITIALIZED;
  if (!alpha1 || !aD || !A || !alpha2 || !bD || !B) return CUDNN_STATUS_BAD_PARAM;
  if (aD->type != bD->type || rb_type(aD->type) < 0 || !valid_format(bD->format))
    return CUDNN_STATUS_NOT_SUPPORTED;
  const int ad[4] = {aD->n, aD->c, aD->h, aD->w}, bd[4] = {bD->n, bD->c, bD->h, bD->w};
  bool bcast = false;
  for (int i = 0; i < 4; ++i) {
    if (ad[i] == bd[i]) continue;
    if (ad[i] != 1) return CUDNN_STATUS_NOT_SUPPORTED;
    bcast = true;
  }
  if (aD->format != bD->format && !(bcast && aD->h == 1 && aD->w == 1))
    return CUDNN_STATUS_NOT_SUPPORTED;
  std::lock_guard<std::mutex> g(handle->lock);
  const float a1 = read_host<float>(alpha1), a2 = read_host<float>(alpha2);
  const size_t n = elems(bD), es = esize(bD->type);
  // A's element strides in its own format, 0 along broadcast dims.
  const bool anhwc = aD->format == CUDNN_TENSOR_NHWC;
  long long sn, sc, sh, sw;
  if (anhwc) {
    sc = 1; sw = aD->c; sh = static_cast<long long>(aD->c) * aD->w; sn = sh * aD->h;
  } else {
    sw = 1; sh = aD->w; sc = static_cast<long long>(aD->w) * aD->h; sn = sc * aD->c;
  }
  if (aD->n == 1) sn = 0;
  if (aD->c == 1) sc = 0;
  if (aD->h == 1) sh = 0;
  if (aD->w == 1) sw = 0;
  Staging sg(handle->stage, handle->stream);
  sg.add(A, elems(aD) * es, true, false);
  sg.add(B, n * es, true, true);
  if (!sg.begin()) return CUDNN_STATUS_ALLOC_FAILED;
  const int nhwc = bD->format == CUDNN_TENSOR_NHWC ? 1 : 0;
  if (bD->type == CUDNN_DATA_FLOAT)
    add_kernel<float><<<grid_for(n), 256, 0, handle->stream>>>(
        static_cast<const float *>(sg.dev(A)), static_cast<float *>(sg.dev(B)), n, bD->c, bD->h,
        bD->w, nhwc, sn, sc, sh, sw, a1, a2, 0);
  else
    add_kernel<uint16_t><<<grid_for(n), 256, 0, handle->stream>>>(
        static_cast<const uint16_t *>(sg.dev(A)), static_cast<uint16_t *>(sg.dev(B)), n, bD->c,
        bD->h, bD->w, nhwc, sn, sc, sh, sw, a1, a2, bD->type == CUDNN_DATA_HALF ? 1 : 0);
  return finish_call(sg, cudaGetLastError());
}

cudnnStatus_t cudnnSoftmaxForward(cudnnHandle_t handle, cudnnSoftmaxAlgorithm_t algo,
                                  cudnnSoftmaxMode_t mode, const void *alpha,
                                  const cudnnTensorDescriptor_t xD, const void *x, const void *beta,
                                  const cudnnTensorDescriptor_t yD, void *y) {
  if (!valid(handle)) return CUDNN_STATUS_NOT_INITIALIZED;
  if (!alpha || !xD || !x || !beta || !yD || !y) return CUDNN_STATUS_BAD_PARAM;
  if (algo != CUDNN_SOFTMAX_FAST && algo != CUDNN_SOFTMAX_ACCURATE && algo != CUDNN_SOFTMAX_LOG)
    return CUDNN_STATUS_NOT_SUPPORTED;
  if (mode != CUDNN_SOFTMAX_MODE_INSTANCE && mode != CUDNN_SOFTMAX_MODE_CHANNEL)
    return CUDNN_STATUS_NOT_SUPPORTED;
  if (!same_tensor(xD, yD) || xD->type != CUDNN_DATA_FLOAT) return CUDNN_STATUS_NOT_SUPPORTED;
  if (x == y) return CUDNN_STATUS_NOT_SUPPORTED;  // every output reads its whole row
  std::lock_guard<std::mutex> g(handle->lock);
  const float al = read_host<float>(alpha), be = read_host<float>(beta);
  const size_t n = elems(xD);
  Staging sg(handle->stage, handle->stream);
  sg.add(x, n * 4, true, false);
  sg.add(y, n * 4, be != 0.0f, true);
  if (!sg.begin()) return CUDNN_STATUS_ALLOC_FAILED;
  const int is_log = algo == CUDNN_SOFTMAX_LOG ? 1 : 0;
  const float *dx = static_cast<const float *>(sg.dev(x));
  float *dy = static_cast<float *>(sg.dev(y));
  const long long HW = static_cast<long long>(xD->h) * xD->w;
  if (mode == CUDNN_SOFTMAX_MODE_INSTANCE)
    softmax_rows_kernel<<<xD->n, kSoftmaxThreads, 0, handle->stream>>>(dx, dy, n / xD->n, is_log, al, be);
  else
    softmax_channel_kernel<<<grid_for(static_cast<size_t>(xD->n) * HW), 256, 0, handle->stream>>>(
        dx, dy, xD->n, xD->c, HW, xD->format == CUDNN_TENSOR_NHWC ? 1 : 0, is_log, al, be);
  return finish_call(sg, cudaGetLastError());
}

cudnnStatus_t cudnnBatchNormalizationForwardInference(
    cudnnHandle_t handle, cudnnBatchNormMode_t mode, const void *alpha, const void *beta,
    const cudnnTensorDescriptor_t xD, const void *x, const cudnnTensorDescriptor_t yD, void *y,
    const cudnnTensorDescriptor_t bnD, const void *scale, const void *bias, const void *estMean,
    const void *estVar, double epsilon) {
  if (!valid(handle)) return CUDNN_STATUS_NOT_INITIALIZED;
  if (!alpha || !beta || !xD || !x || !yD || !y || !bnD || !scale || !bias || !estMean || !estVar)
    return CUDNN_STATUS_BAD_PARAM;
  if (mode != CUDNN_BATCHNORM_SPATIAL && mode != CUDNN_BATCHNORM_PER_ACTIVATION)
    return CUDNN_STATUS_NOT_SUPPORTED;
  if (!same_tensor(xD, yD) || xD->type != CUDNN_DATA_FLOAT) return CUDNN_STATUS_NOT_SUPPORTED;
  if (bnD->type != CUDNN_DATA_FLOAT || bnD->n != 1 || bnD->c != xD->c || bnD->h != 1 || bnD->w != 1)
    return CUDNN_STATUS_BAD_PARAM;
  if (!(epsilon >= 0.0)) return CUDNN_STATUS_BAD_PARAM;
  std::lock_guard<std::mutex> g(handle->lock);
  const float al = read_host<float>(alpha), be = read_host<float>(beta);
  const size_t n = elems(xD);
  const int C = xD->c;
  Staging sg(handle->stage, handle->stream);
  sg.add(x, n * 4, true, false);
  sg.add(y, n * 4, be != 0.0f || x == y, true);
  for (const void *p : {scale, bias, estMean, estVar}) sg.add(p, static_cast<size_t>(C) * 4, true, false);
  if (!sg.begin()) return CUDNN_STATUS_ALLOC_FAILED;
  if (!handle->scratch.ensure(static_cast<size_t>(C) * 16, handle->stream)) {
    sg.finish();
    return CUDNN_STATUS_ALLOC_FAILED;
  }
  double *sb = static_cast<double *>(handle->scratch.p);
  bn_prep_kernel<<<(C + 255) / 256, 256, 0, handle->stream>>>(
      static_cast<const float *>(sg.dev(scale)), static_cast<const float *>(sg.dev(bias)),
      static_cast<const float *>(sg.dev(estMean)), static_cast<const float *>(sg.dev(estVar)), C,
      epsilon, sb);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) {
    bn_apply_kernel<<<grid_for(n), 256, 0, handle->stream>>>(
        static_cast<const float *>(sg.dev(x)), static_cast<float *>(sg.dev(y)), n, C,
        static_cast<long long>(xD->h) * xD->w, xD->format == CUDNN_TENSOR_NHWC ? 1 : 0, sb, al, be);
    e = cudaGetLastError();
  }
  return finish_call(sg, e);
}

}  // extern "C"
