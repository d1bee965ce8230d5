// Bandwidth-bound kernels of the rouge-numerics path on sm_100a:
//   - per-row symmetric int8 quantization   (quant_int8.cpp:72-90)
//   - int8 dequantization                   (quant_int8.cpp:145-160)
//   - per-tensor absolute maximum           (e4m3 per-tensor scale, test_ai.cpp:219-231)
//   - scaled E4M3 encoding                  (fp8.cpp:75-106 applied to x / s)
//   - elementwise f32 <-> f16 / bf16 / e4m3 (fp16.cpp, fp8.cpp)
//
// All use 128-bit coalesced global accesses, grid-stride loops sized to a
// multiple of the SM count, and warp-shuffle reductions.
#include <cuda_runtime.h>

#include <cstdint>

#include "formats.cuh"
#include "x86fp.cuh"
#include "runtime.cuh"

namespace rb200 {
namespace {

constexpr int kThreads = 256;

// ---------------------------------------------------------------- int8

// One int8 code from an f32 value and the row's double reciprocal scale,
// as quant_int8.cpp:38-46,87 computes it on x86-64: nearbyint of the
// double product, then a conversion whose out-of-range / NaN result is
// INT32_MIN, then the clamp to [-127, 127].
__device__ __forceinline__ int code_i8(float x, double inv) {
  const double p = __dmul_rn(static_cast<double>(x), inv);
  if (!(p >= -2147483648.5 && p < 2147483647.5)) return -127;  // NaN, +-Inf, overflow
  const int q = __double2int_rn(p);
  return q < -127 ? -127 : (q > 127 ? 127 : q);
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  return (static_cast<uint32_t>(a) & 0xFFu) | ((static_cast<uint32_t>(b) & 0xFFu) << 8) |
         ((static_cast<uint32_t>(c) & 0xFFu) << 16) | ((static_cast<uint32_t>(d) & 0xFFu) << 24);
}

__device__ __forceinline__ float absmax4(float4 v) {
  return fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
}

__device__ __forceinline__ float block_max(float v, float *red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float m = red[0];
#pragma unroll
  for (int w = 1; w < kThreads / 32; ++w) m = fmaxf(m, red[w]);
  return m;
}

// One CTA per row (grid-stride over rows). The first VPT*256 float4 of the
// row stay in registers between the max pass and the encode pass; longer
// rows re-read the remainder (an L2 hit: the row was just streamed).
template <int VPT>
__global__ void __launch_bounds__(kThreads) quant_i8_rows_kernel(const float *__restrict__ x,
                                                                 int rows, int cols,
                                                                 float *__restrict__ scales,
                                                                 int8_t *__restrict__ out) {
  __shared__ float red[kThreads / 32];
  __shared__ double s_inv;
  const int nvec = cols >> 2;
  for (int r = blockIdx.x; r < rows; r += gridDim.x) {
    const float4 *xr = reinterpret_cast<const float4 *>(x + static_cast<size_t>(r) * cols);
    uint32_t *orow = reinterpret_cast<uint32_t *>(out + static_cast<size_t>(r) * cols);
    float4 v[VPT];
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int i = threadIdx.x + j * kThreads;
      if (i < nvec) {
        v[j] = __ldcs(xr + i);
        amax = fmaxf(amax, absmax4(v[j]));
      }
    }
    for (int i = threadIdx.x + VPT * kThreads; i < nvec; i += kThreads)
      amax = fmaxf(amax, absmax4(__ldg(xr + i)));
    amax = block_max(amax, red);
    if (threadIdx.x == 0) {
      // quant_int8.cpp:82-84: scale and its reciprocal in double.
      const double a = static_cast<double>(amax);
      const float s = a > 0.0 ? __double2float_rn(__ddiv_rn(a, 127.0)) : 1.0f;
      scales[r] = s;
      s_inv = __ddiv_rn(1.0, static_cast<double>(s));
    }
    __syncthreads();
    const double inv = s_inv;
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int i = threadIdx.x + j * kThreads;
      if (i < nvec)
        orow[i] = pack4(code_i8(v[j].x, inv), code_i8(v[j].y, inv), code_i8(v[j].z, inv),
                        code_i8(v[j].w, inv));
    }
    for (int i = threadIdx.x + VPT * kThreads; i < nvec; i += kThreads) {
      const float4 t = __ldcs(xr + i);
      orow[i] = pack4(code_i8(t.x, inv), code_i8(t.y, inv), code_i8(t.z, inv), code_i8(t.w, inv));
    }
    __syncthreads();  // red[] and s_inv are reused by the next row
  }
}

// Per-tensor variant (quant_int8.cpp:54-68): the scale comes from the
// tensor's absolute maximum, already reduced into *amax.
__global__ void __launch_bounds__(kThreads) quant_i8_tensor_kernel(const float *__restrict__ x,
                                                                   size_t n,
                                                                   const float *__restrict__ amax,
                                                                   float *__restrict__ scale_out,
                                                                   int8_t *__restrict__ out) {
  const double a = static_cast<double>(__ldg(amax));
  const float s = a > 0.0 ? __double2float_rn(__ddiv_rn(a, 127.0)) : 1.0f;
  const double inv = __ddiv_rn(1.0, static_cast<double>(s));
  const size_t tid = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  if (tid == 0 && scale_out) *scale_out = s;
  const size_t n4 = n / 4;
  const float4 *x4 = reinterpret_cast<const float4 *>(x);
  uint32_t *o4 = reinterpret_cast<uint32_t *>(out);
  for (size_t i = tid; i < n4; i += stride) {
    const float4 t = __ldcs(x4 + i);
    o4[i] = pack4(code_i8(t.x, inv), code_i8(t.y, inv), code_i8(t.z, inv), code_i8(t.w, inv));
  }
  for (size_t t = n4 * 4 + tid; t < n; t += stride) out[t] = static_cast<int8_t>(code_i8(x[t], inv));
}

// out = (float)q * s per element; s = scales[row] or the single `scale`.
__global__ void __launch_bounds__(kThreads) dequant_i8_kernel(const int8_t *__restrict__ q,
                                                              int rows, int cols,
                                                              const float *__restrict__ scales,
                                                              float scale,
                                                              float *__restrict__ out) {
  const size_t n4 = static_cast<size_t>(rows) * cols / 4;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const uint32_t *q4 = reinterpret_cast<const uint32_t *>(q);
  float4 *o4 = reinterpret_cast<float4 *>(out);
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n4; i += stride) {
    const uint32_t w = __ldcs(q4 + i);
    const float s = scales ? __ldg(scales + (i * 4) / cols) : scale;
    float4 o;
    o.x = x86_mul(static_cast<float>(static_cast<int8_t>(w & 0xFFu)), s);
    o.y = x86_mul(static_cast<float>(static_cast<int8_t>((w >> 8) & 0xFFu)), s);
    o.z = x86_mul(static_cast<float>(static_cast<int8_t>((w >> 16) & 0xFFu)), s);
    o.w = x86_mul(static_cast<float>(static_cast<int8_t>(w >> 24)), s);
    __stcs(o4 + i, o);
  }
}

// ---------------------------------------------------------------- e4m3

// Per-tensor max |x| (NaN ignored) folded into *amax_bits with atomicMax on
// the bit pattern (order-preserving for non-negative floats). *amax_bits
// must be zero on entry.
__global__ void __launch_bounds__(kThreads) absmax_kernel(const float *__restrict__ x, size_t n,
                                                          unsigned int *__restrict__ amax_bits) {
  __shared__ float red[kThreads / 32];
  const size_t n4 = n / 4;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const size_t tid = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  const float4 *x4 = reinterpret_cast<const float4 *>(x);
  float m0 = 0.0f, m1 = 0.0f;
  size_t i = tid;
  for (; i + stride < n4; i += 2 * stride) {  // two independent loads in flight
    const float4 a = __ldcs(x4 + i), b = __ldcs(x4 + i + stride);
    m0 = fmaxf(m0, absmax4(a));
    m1 = fmaxf(m1, absmax4(b));
  }
  if (i < n4) m0 = fmaxf(m0, absmax4(__ldcs(x4 + i)));
  for (size_t t = n4 * 4 + tid; t < n; t += stride) m1 = fmaxf(m1, fabsf(x[t]));
  const float m = block_max(fmaxf(m0, m1), red);
  if (threadIdx.x == 0 && m > 0.0f) atomicMax(amax_bits, __float_as_uint(m));
}

__device__ __forceinline__ uint32_t enc4(float4 v, float s) {
  return static_cast<uint32_t>(encode_e4m3(x86_div(v.x, s))) |
         (static_cast<uint32_t>(encode_e4m3(x86_div(v.y, s))) << 8) |
         (static_cast<uint32_t>(encode_e4m3(x86_div(v.z, s))) << 16) |
         (static_cast<uint32_t>(encode_e4m3(x86_div(v.w, s))) << 24);
}

// out[i] = e4m3(x[i] / s), s = amax / 448 (1 when amax == 0). 16 elements
// per thread per step: four 16-byte loads, one 16-byte store.
__global__ void __launch_bounds__(kThreads) e4m3_scaled_kernel(const float *__restrict__ x,
                                                               size_t n,
                                                               const float *__restrict__ amax,
                                                               float *__restrict__ scale_out,
                                                               uint8_t *__restrict__ out) {
  const float a = __ldg(amax);
  const float s = a > 0.0f ? __fdiv_rn(a, 448.0f) : 1.0f;
  const size_t tid = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  if (tid == 0 && scale_out) *scale_out = s;
  const size_t n16 = n / 16;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const float4 *x4 = reinterpret_cast<const float4 *>(x);
  uint4 *o16 = reinterpret_cast<uint4 *>(out);
  for (size_t i = tid; i < n16; i += stride) {
    const float4 a0 = __ldcs(x4 + 4 * i), a1 = __ldcs(x4 + 4 * i + 1);
    const float4 a2 = __ldcs(x4 + 4 * i + 2), a3 = __ldcs(x4 + 4 * i + 3);
    uint4 o;
    o.x = enc4(a0, s);
    o.y = enc4(a1, s);
    o.z = enc4(a2, s);
    o.w = enc4(a3, s);
    o16[i] = o;
  }
  for (size_t t = n16 * 16 + tid; t < n; t += stride) out[t] = encode_e4m3(x86_div(x[t], s));
}

// ---------------------------------------------------------------- converts

template <int KIND>  // 0: f32 -> f16, 1: f32 -> bf16
__global__ void __launch_bounds__(kThreads) f32_to_half_kernel(const float *__restrict__ x, size_t n,
                                                               uint16_t *__restrict__ out) {
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const size_t tid = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  const size_t n4 = n / 4;
  const float4 *x4 = reinterpret_cast<const float4 *>(x);
  uint2 *o4 = reinterpret_cast<uint2 *>(out);
  for (size_t i = tid; i < n4; i += stride) {
    const float4 v = __ldcs(x4 + i);
    uint2 o;
    if (KIND == 0) {
      o.x = encode_f16(v.x) | (static_cast<uint32_t>(encode_f16(v.y)) << 16);
      o.y = encode_f16(v.z) | (static_cast<uint32_t>(encode_f16(v.w)) << 16);
    } else {
      o.x = encode_bf16(v.x) | (static_cast<uint32_t>(encode_bf16(v.y)) << 16);
      o.y = encode_bf16(v.z) | (static_cast<uint32_t>(encode_bf16(v.w)) << 16);
    }
    o4[i] = o;
  }
  for (size_t t = n4 * 4 + tid; t < n; t += stride)
    out[t] = KIND == 0 ? encode_f16(x[t]) : encode_bf16(x[t]);
}

__global__ void __launch_bounds__(kThreads) e4m3_to_f32_kernel(const uint8_t *__restrict__ x,
                                                               size_t n, float *__restrict__ out) {
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const size_t tid = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  const size_t n4 = n / 4;
  const uint32_t *x4 = reinterpret_cast<const uint32_t *>(x);
  float4 *o4 = reinterpret_cast<float4 *>(out);
  for (size_t i = tid; i < n4; i += stride) {
    const uint32_t w = __ldcs(x4 + i);
    o4[i] = make_float4(decode_e4m3(w & 0xFFu), decode_e4m3((w >> 8) & 0xFFu),
                        decode_e4m3((w >> 16) & 0xFFu), decode_e4m3(w >> 24));
  }
  for (size_t t = n4 * 4 + tid; t < n; t += stride) out[t] = decode_e4m3(x[t]);
}

inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline bool aligned4(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

// Grid for the elementwise kernels: enough CTAs to cover the work, capped
// at a whole number of waves (8 resident 256-thread CTAs per SM).
int stream_grid(size_t work_items) {
  const int sms = current_sm_count();
  const size_t cap = static_cast<size_t>(sms > 0 ? sms : 148) * 8;
  size_t g = (work_items + kThreads - 1) / kThreads;
  if (g > cap) g = cap;
  return static_cast<int>(g < 1 ? 1 : g);
}

}  // namespace

// Launchers used by the host drop-in layer (no validation beyond what the
// callers already did).
int launch_quant_i8_rows(const float *x, int rows, int cols, float *scales, int8_t *out,
                         cudaStream_t st) {
  const int sms = current_sm_count();
  const int grid = rows < sms * 8 ? rows : sms * 8;
  const int nvec = cols / 4;
  if (nvec <= 4 * kThreads)
    quant_i8_rows_kernel<4><<<grid, kThreads, 0, st>>>(x, rows, cols, scales, out);
  else
    quant_i8_rows_kernel<8><<<grid, kThreads, 0, st>>>(x, rows, cols, scales, out);
  return cuda_status(cudaGetLastError());
}

int launch_absmax(const float *x, size_t n, float *amax, cudaStream_t st);

int launch_quant_i8_tensor(const float *x, size_t n, float *amax, float *scale_out, int8_t *out,
                           cudaStream_t st) {
  int s = launch_absmax(x, n, amax, st);
  if (s != ROUGE_B200_OK) return s;
  quant_i8_tensor_kernel<<<stream_grid(n / 4 + 1), kThreads, 0, st>>>(x, n, amax, scale_out, out);
  return cuda_status(cudaGetLastError());
}

int launch_dequant_i8(const int8_t *q, int rows, int cols, const float *scales, float scale,
                      float *out, cudaStream_t st) {
  const size_t n4 = static_cast<size_t>(rows) * cols / 4;
  dequant_i8_kernel<<<stream_grid(n4), kThreads, 0, st>>>(q, rows, cols, scales, scale, out);
  return cuda_status(cudaGetLastError());
}

int launch_absmax(const float *x, size_t n, float *amax, cudaStream_t st) {
  int s = cuda_status(cudaMemsetAsync(amax, 0, sizeof(float), st));
  if (s != ROUGE_B200_OK) return s;
  absmax_kernel<<<stream_grid(n / 8 + 1), kThreads, 0, st>>>(
      x, n, reinterpret_cast<unsigned int *>(amax));
  return cuda_status(cudaGetLastError());
}

int launch_e4m3_scaled(const float *x, size_t n, const float *amax, float *scale_out,
                       uint8_t *out, cudaStream_t st) {
  e4m3_scaled_kernel<<<stream_grid(n / 16 + 1), kThreads, 0, st>>>(x, n, amax, scale_out, out);
  return cuda_status(cudaGetLastError());
}

int launch_f32_to_half(const float *x, size_t n, uint16_t *out, int bf16, cudaStream_t st) {
  if (bf16)
    f32_to_half_kernel<1><<<stream_grid(n / 4 + 1), kThreads, 0, st>>>(x, n, out);
  else
    f32_to_half_kernel<0><<<stream_grid(n / 4 + 1), kThreads, 0, st>>>(x, n, out);
  return cuda_status(cudaGetLastError());
}

int launch_e4m3_to_f32(const uint8_t *x, size_t n, float *out, cudaStream_t st) {
  e4m3_to_f32_kernel<<<stream_grid(n / 4 + 1), kThreads, 0, st>>>(x, n, out);
  return cuda_status(cudaGetLastError());
}

}  // namespace rb200

using namespace rb200;

extern "C" {

int rouge_b200_quantize_i8_rows(const float *x, int rows, int cols, float *scales, int8_t *out,
                                void *stream) {
  if (!x || !scales || !out || rows <= 0 || cols <= 0) return set_status(ROUGE_B200_EINVAL);
  if ((cols & 3) || !aligned16(x) || !aligned4(out)) return set_status(ROUGE_B200_EUNSUPPORTED);
  int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  return launch_quant_i8_rows(x, rows, cols, scales, out, as_stream(stream));
}

int rouge_b200_dequantize_i8_rows(const int8_t *q, int rows, int cols, const float *scales,
                                  float scale, float *out, void *stream) {
  if (!q || !out || rows <= 0 || cols <= 0 || (!scales && scale == 0.0f))
    return set_status(ROUGE_B200_EINVAL);
  if ((cols & 3) || !aligned4(q) || !aligned16(out)) return set_status(ROUGE_B200_EUNSUPPORTED);
  int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  return launch_dequant_i8(q, rows, cols, scales, scale, out, as_stream(stream));
}

int rouge_b200_absmax_f32(const float *x, size_t n, float *amax, void *stream) {
  if (!x || !amax || n == 0) return set_status(ROUGE_B200_EINVAL);
  if (!aligned16(x)) return set_status(ROUGE_B200_EUNSUPPORTED);
  int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  return launch_absmax(x, n, amax, as_stream(stream));
}

int rouge_b200_quantize_e4m3_scaled(const float *x, size_t n, const float *amax,
                                    float *scale_out, uint8_t *out, void *stream) {
  if (!x || !amax || !out || n == 0 || scale_out == amax) return set_status(ROUGE_B200_EINVAL);
  if (!aligned16(x) || !aligned16(out)) return set_status(ROUGE_B200_EUNSUPPORTED);
  int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  return launch_e4m3_scaled(x, n, amax, scale_out, out, as_stream(stream));
}

int rouge_b200_quantize_e4m3_tensor(const float *x, size_t n, float *amax_out, float *scale_out,
                                    uint8_t *out, void *stream) {
  if (!x || !amax_out || !out || n == 0 || scale_out == amax_out)
    return set_status(ROUGE_B200_EINVAL);
  if (!aligned16(x) || !aligned16(out)) return set_status(ROUGE_B200_EUNSUPPORTED);
  int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  s = launch_absmax(x, n, amax_out, as_stream(stream));
  if (s != ROUGE_B200_OK) return s;
  return launch_e4m3_scaled(x, n, amax_out, scale_out, out, as_stream(stream));
}

int rouge_b200_convert_f32_to_f16(const float *x, size_t n, uint16_t *out, void *stream) {
  if (!x || !out || n == 0) return set_status(ROUGE_B200_EINVAL);
  if (!aligned16(x) || (reinterpret_cast<uintptr_t>(out) & 7u))
    return set_status(ROUGE_B200_EUNSUPPORTED);
  int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  return launch_f32_to_half(x, n, out, 0, as_stream(stream));
}

int rouge_b200_convert_f32_to_bf16(const float *x, size_t n, uint16_t *out, void *stream) {
  if (!x || !out || n == 0) return set_status(ROUGE_B200_EINVAL);
  if (!aligned16(x) || (reinterpret_cast<uintptr_t>(out) & 7u))
    return set_status(ROUGE_B200_EUNSUPPORTED);
  int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  return launch_f32_to_half(x, n, out, 1, as_stream(stream));
}

int rouge_b200_convert_e4m3_to_f32(const uint8_t *x, size_t n, float *out, void *stream) {
  if (!x || !out || n == 0) return set_status(ROUGE_B200_EINVAL);
  if (!aligned4(x) || !aligned16(out)) return set_status(ROUGE_B200_EUNSUPPORTED);
  int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  return launch_e4m3_to_f32(x, n, out, as_stream(stream));
}

}  // extern "C"
