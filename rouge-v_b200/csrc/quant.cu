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

#include <algorithm>
#include <atomic>
#include <cstdint>

#include "formats.cuh"
#include "x86fp.cuh"
#include "ptx.cuh"
#include "i8code.cuh"
#include "runtime.cuh"

namespace rb200 {
namespace {

constexpr int kThreads = 256;

// ---------------------------------------------------------------- int8

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

template <int VPT>
__device__ __forceinline__ void load_row(float4 (&v)[VPT], const float4 *xr, int nvec) {
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int i = threadIdx.x + j * kThreads;
    v[j] = i < nvec ? __ldcs(xr + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// Persistent CTAs (grid = resident CTAs), grid-stride over rows. The first
// VPT*256 float4 of a row stay in registers between its max pass and its
// encode pass, and the next row's loads are issued before the current row
// is reduced, so HBM reads stay in flight across the block reduction.
// Longer rows re-read their remainder (an L2 hit). One __syncthreads per
// row: the reduction slots are double-buffered by row parity.
template <int VPT>
__global__ void __launch_bounds__(kThreads) quant_i8_rows_kernel(const float *__restrict__ x,
                                                                 int rows, int cols,
                                                                 float *__restrict__ scales,
                                                                 int8_t *__restrict__ out) {
  __shared__ float red[2][kThreads / 32];
  const int nvec = cols >> 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int r = blockIdx.x;
  float4 cur[VPT];
  if (r < rows) load_row(cur, reinterpret_cast<const float4 *>(x + static_cast<size_t>(r) * cols), nvec);
  for (int parity = 0; r < rows; r += gridDim.x, parity ^= 1) {
    const float4 *xr = reinterpret_cast<const float4 *>(x + static_cast<size_t>(r) * cols);
    uint32_t *orow = reinterpret_cast<uint32_t *>(out + static_cast<size_t>(r) * cols);
    const int rn = r + gridDim.x;
    float4 nxt[VPT];
    if (rn < rows)
      load_row(nxt, reinterpret_cast<const float4 *>(x + static_cast<size_t>(rn) * cols), nvec);
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < VPT; ++j) amax = fmaxf(amax, absmax4(cur[j]));
    for (int i = threadIdx.x + VPT * kThreads; i < nvec; i += kThreads)
      amax = fmaxf(amax, absmax4(__ldg(xr + i)));
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) red[parity][warp] = amax;
    __syncthreads();
    float m = red[parity][0];
#pragma unroll
    for (int w = 1; w < kThreads / 32; ++w) m = fmaxf(m, red[parity][w]);
    // quant_int8.cpp:82-84: scale and its reciprocal in double, one lane per warp.
    float s = 0.0f;
    double inv = 0.0;
    if (lane == 0) {
      const double a = static_cast<double>(m);
      s = a > 0.0 ? __double2float_rn(__ddiv_rn(a, 127.0)) : 1.0f;
      inv = __ddiv_rn(1.0, static_cast<double>(s));
    }
    s = __shfl_sync(0xffffffffu, s, 0);
    inv = __shfl_sync(0xffffffffu, inv, 0);
    if (threadIdx.x == 0) scales[r] = s;
    const float inv_f = __double2float_rn(inv);
    const bool exact_row = isinf(inv_f);
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int i = threadIdx.x + j * kThreads;
      if (i < nvec) orow[i] = encode4_i8(cur[j], inv, inv_f, exact_row);
    }
    for (int i = threadIdx.x + VPT * kThreads; i < nvec; i += kThreads)
      orow[i] = encode4_i8(__ldcs(xr + i), inv, inv_f, exact_row);
#pragma unroll
    for (int j = 0; j < VPT; ++j) cur[j] = nxt[j];
  }
}

// One warp per row with the whole row in registers (VPL float4 per lane,
// rows up to VPL * 128 elements), fed by bulk copies. One CTA per SM owns a
// contiguous range of rows; its 12 warps take the range's rows one at a time
// from a shared-memory counter, so every SM finishes within about one
// row-time of the others. Each warp owns one shared-memory row slot: it
// copies the slot into registers, claims its next row and (lane 0) starts
// that row's cp.async.bulk into the same slot, then reduces (warp
// shuffles), computes the scale in double exactly as the reference, and
// encodes from registers while the copy runs -- so the warp's next row
// streams in during its compute. The encode is branch-free (paired f32x2
// instructions); words near a rounding tie are re-encoded in double
// afterwards from a second read of their inputs. The time-bounded slot
// waits report ROUGE_B200_ETIMEOUT through *err; a warp that gives up waits
// (bounded) for its copy in flight before it exits.
template <int VPL>
__global__ void __launch_bounds__(384, 1)
    quant_i8_rows_tma_kernel(const float *__restrict__ x, int rows, int cols,
                             float *__restrict__ scales, int8_t *__restrict__ out, int *err) {
  static_assert(VPL >= 1 && VPL <= 32, "one bit per word of a lane in the fix-up mask");
  extern __shared__ __align__(128) uint8_t qsm[];
  __shared__ __align__(8) uint64_t bars[12];
  __shared__ int next_row;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int nvec = cols >> 2;
  const uint32_t row_bytes = static_cast<uint32_t>(cols) * 4u;
  const int per = rows / static_cast<int>(gridDim.x);
  const int extra = rows % static_cast<int>(gridDim.x);
  const int b = static_cast<int>(blockIdx.x);
  const int r_beg = b * per + min(b, extra);
  const int r_end = r_beg + per + (b < extra ? 1 : 0);
  uint8_t *slot = qsm + static_cast<size_t>(warp) * row_bytes;
  uint64_t *bar = &bars[warp];
  if (threadIdx.x == 0) {
    next_row = r_beg + static_cast<int>(blockDim.x >> 5);
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) mbar_init(&bars[w], 1);
    mbar_init_fence();
  }
  __syncthreads();
  // Launched with programmatic serialisation: the set-up above overlaps the
  // previous kernel's tail; x (perhaps that kernel's output) is read, and
  // the codes (perhaps still read by it) written, only after it completed.
  grid_dependency_wait();
  // The GEMM that consumes these codes may start its prologue now; it waits
  // for this grid's completion before it reads them.
  grid_launch_dependents();
  int r = r_beg + warp;
  if (lane == 0 && r < r_end) {
    mbar_arrive_expect_tx(bar, row_bytes);
    bulk_load(slot, x + static_cast<size_t>(r) * cols, row_bytes, bar);
  }
  const volatile int never = 0;
  uint32_t phase = 0;
  bool in_flight = r < r_end;
  while (r < r_end) {
    const bool got = mbar_wait(bar, phase, &never);
    if (!__all_sync(0xffffffffu, got)) {
      if (lane == 0 && err) atomicCAS(err, 0, ROUGE_B200_ETIMEOUT);
      break;
    }
    phase ^= 1u;
    in_flight = false;
    const float4 *row = reinterpret_cast<const float4 *>(slot);
    float4 v[VPL];
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int i = j * 32 + lane;
      v[j] = i < nvec ? row[i] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float amax = 0.0f;
#pragma unroll
    for (int j = 0; j < VPL; ++j)
      amax = max3(amax, max3(fabsf(v[j].x), fabsf(v[j].y), fabsf(v[j].z)), fabsf(v[j].w));
    // Every lane's copy of the slot is in registers (the maximum used all of
    // it): the slot takes this warp's next row.
    __syncwarp();
    int rn = 0;
    if (lane == 0) {
      rn = atomicAdd(&next_row, 1);
      if (rn < r_end) {
        mbar_arrive_expect_tx(bar, row_bytes);
        bulk_load(slot, x + static_cast<size_t>(rn) * cols, row_bytes, bar);
      }
    }
    rn = __shfl_sync(0xffffffffu, rn, 0);
    in_flight = rn < r_end;
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    // quant_int8.cpp:82-84: scale and its reciprocal in double.
    const double a = static_cast<double>(amax);
    const float s = a > 0.0 ? __double2float_rn(__ddiv_rn(a, 127.0)) : 1.0f;
    const double inv = __ddiv_rn(1.0, static_cast<double>(s));
    const float inv_f = __double2float_rn(inv);
    const bool exact_row = isinf(inv_f);
    if (lane == 0) scales[r] = s;
    uint32_t *orow = reinterpret_cast<uint32_t *>(out + static_cast<size_t>(r) * cols);
    const float4 *xr = reinterpret_cast<const float4 *>(x + static_cast<size_t>(r) * cols);
    uint32_t redo = 0;
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
      const int i = j * 32 + lane;
      bool tie;
      const uint32_t w = encode4_i8_fast(v[j], inv_f, tie);
      tie |= exact_row;
      if (i < nvec && !tie) orow[i] = w;
      redo |= (tie && i < nvec) ? (1u << j) : 0u;
    }
    while (redo) {
      const int j = __ffs(redo) - 1;
      redo &= redo - 1;
      const int i = j * 32 + lane;
      orow[i] = encode4_i8_exact(__ldg(xr + i), inv);
    }
    r = rn;
  }
  if (in_flight && lane == 0) mbar_wait(bar, phase, &never);  // let the last copy land
}

// Row pipeline through shared memory: thread 0 keeps `stages` rows in
// flight with cp.async.bulk copies (one mbarrier per slot); all 256
// threads reduce and encode the oldest row from shared memory, then free
// its slot for the row `stages` ahead. Persistent CTAs, grid-stride over
// rows; row bytes (cols * 4) up to the slot size. The time-bounded waits
// report ROUGE_B200_ETIMEOUT through *err instead of hanging.
__global__ void __launch_bounds__(kThreads) quant_i8_rows_bulk_kernel(
    const float *__restrict__ x, int rows, int cols, float *__restrict__ scales,
    int8_t *__restrict__ out, int stages, int *err) {
  extern __shared__ __align__(128) uint8_t qsm[];
  __shared__ float red[2][kThreads / 32];
  __shared__ __align__(8) uint64_t full[8];
  const int nvec = cols >> 2;
  const uint32_t row_bytes = static_cast<uint32_t>(cols) * 4u;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const volatile int never = 0;
  bool aborted = false;
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) mbar_init(&full[s], 1);
    mbar_init_fence();
    int r = blockIdx.x;
    for (int s = 0; s < stages && r < rows; ++s, r += gridDim.x) {
      mbar_arrive_expect_tx(&full[s], row_bytes);
      bulk_load(qsm + static_cast<size_t>(s) * row_bytes, x + static_cast<size_t>(r) * cols,
                row_bytes, &full[s]);
    }
  }
  __syncthreads();
  int i = 0;
  for (int r = blockIdx.x; r < rows; r += gridDim.x, ++i) {
    const int s = i % stages;
    const uint32_t phase = static_cast<uint32_t>(i / stages) & 1u;
    const bool ok = mbar_wait(&full[s], phase, &never);
    const float4 *row = reinterpret_cast<const float4 *>(qsm + static_cast<size_t>(s) * row_bytes);
    float amax = 0.0f;
    for (int v = threadIdx.x; v < nvec; v += kThreads) amax = fmaxf(amax, absmax4(row[v]));
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) red[i & 1][warp] = amax;
    // One barrier both publishes the partial maxima and makes the timeout
    // decision collective, so no thread is left waiting at a later barrier.
    if (__syncthreads_or(!ok)) {
      if (threadIdx.x == 0 && err) atomicCAS(err, 0, ROUGE_B200_ETIMEOUT);
      aborted = true;
      break;
    }
    float m = red[i & 1][0];
#pragma unroll
    for (int w = 1; w < kThreads / 32; ++w) m = fmaxf(m, red[i & 1][w]);
    // quant_int8.cpp:82-84: scale and its reciprocal in double, one lane per warp.
    float sc = 0.0f;
    double inv = 0.0;
    if (lane == 0) {
      const double a = static_cast<double>(m);
      sc = a > 0.0 ? __double2float_rn(__ddiv_rn(a, 127.0)) : 1.0f;
      inv = __ddiv_rn(1.0, static_cast<double>(sc));
    }
    sc = __shfl_sync(0xffffffffu, sc, 0);
    inv = __shfl_sync(0xffffffffu, inv, 0);
    if (threadIdx.x == 0) scales[r] = sc;
    const float inv_f = __double2float_rn(inv);
    const bool exact_row = isinf(inv_f);
    uint32_t *orow = reinterpret_cast<uint32_t *>(out + static_cast<size_t>(r) * cols);
#pragma unroll 4
    for (int v = threadIdx.x; v < nvec; v += kThreads)
      orow[v] = encode4_i8(row[v], inv, inv_f, exact_row);
    __syncthreads();  // slot s fully read: refill it with the row `stages` ahead
    if (threadIdx.x == 0) {
      const int rn = r + stages * gridDim.x;
      if (rn < rows) {
        mbar_arrive_expect_tx(&full[s], row_bytes);
        bulk_load(qsm + static_cast<size_t>(s) * row_bytes, x + static_cast<size_t>(rn) * cols,
                  row_bytes, &full[s]);
      }
    }
  }
  if (aborted && threadIdx.x == 0) {
    // Let the copies already issued (rows i .. i+stages-1 of this CTA, as
    // far as they exist) land before the shared memory is released.
    const int n_cta = (rows - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) /
                      static_cast<int>(gridDim.x);
    for (int j = i; j < i + stages && j < n_cta; ++j)
      mbar_wait(&full[j % stages], static_cast<uint32_t>(j / stages) & 1u, &never);
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
  const float inv_f = __double2float_rn(inv);
  const size_t tid = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  if (tid == 0 && scale_out) *scale_out = s;
  const size_t n4 = n / 4;
  const float4 *x4 = reinterpret_cast<const float4 *>(x);
  uint32_t *o4 = reinterpret_cast<uint32_t *>(out);
  const bool exact_row = isinf(inv_f);
  for (size_t i = tid; i < n4; i += stride) o4[i] = encode4_i8(__ldcs(x4 + i), inv, inv_f, exact_row);
  for (size_t t = n4 * 4 + tid; t < n; t += stride)
    out[t] = static_cast<int8_t>(code_i8(x[t], inv, inv_f));
}

// Asymmetric per-group quantization (quant_int8.cpp:94-142), one warp per
// group of gsz = cols / groups consecutive elements of a row. In double, as
// the reference: lo/hi of the group; scale and zero by the three cases of
// :122-131; code = clamp(rne(x * (1.0/scale) + zero), 0, 255) with the
// multiply and the add rounded separately (the reference's translation unit
// is built without FMA instructions).
__global__ void __launch_bounds__(kThreads) quant_i8_group_kernel(
    const float *__restrict__ x, int rows, int cols, int groups, float *__restrict__ scales,
    uint8_t *__restrict__ zeros, uint8_t *__restrict__ out) {
  const int gsz = cols / groups;
  const long long total = static_cast<long long>(rows) * groups;
  const int lane = threadIdx.x & 31;
  const long long warps = static_cast<long long>(gridDim.x) * (blockDim.x >> 5);
  for (long long g = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; g < total;
       g += warps) {
    const float *src = x + (g / groups) * static_cast<long long>(cols) + (g % groups) * gsz;
    uint8_t *dst = out + (g / groups) * static_cast<long long>(cols) + (g % groups) * gsz;
    float lo = src[0], hi = src[0];
    for (int i = lane; i < gsz; i += 32) {
      const float v = src[i];
      lo = v < lo ? v : lo;  // comparisons ignore NaN, as the reference's do
      hi = v > hi ? v : hi;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float l2 = __shfl_xor_sync(0xffffffffu, lo, o), h2 = __shfl_xor_sync(0xffffffffu, hi, o);
      lo = l2 < lo ? l2 : lo;
      hi = h2 > hi ? h2 : hi;
    }
    float scale = 1.0f;
    int zero = 0;
    double inv = 1.0;
    if (lane == 0) {
      const double dlo = lo, dhi = hi;
      if (dlo >= 0.0) {
        zero = 0;
        scale = dhi > 0.0 ? __double2float_rn(__ddiv_rn(dhi, 255.0)) : 1.0f;
      } else if (dhi <= 0.0) {
        zero = 255;
        scale = dlo < 0.0 ? __double2float_rn(__ddiv_rn(-dlo, 255.0)) : 1.0f;
      } else {
        scale = __double2float_rn(__ddiv_rn(__dsub_rn(dhi, dlo), 255.0));
        const double z = __ddiv_rn(-dlo, static_cast<double>(scale));
        int zi = (z >= -2147483648.5 && z < 2147483647.5) ? __double2int_rn(z) : INT_MIN;
        zero = zi < 0 ? 0 : (zi > 255 ? 255 : zi);
      }
      inv = __ddiv_rn(1.0, static_cast<double>(scale));
      scales[g] = scale;
      zeros[g] = static_cast<uint8_t>(zero);
    }
    zero = __shfl_sync(0xffffffffu, zero, 0);
    inv = __shfl_sync(0xffffffffu, inv, 0);
    const double dz = static_cast<double>(zero);
    for (int i = lane; i < gsz; i += 32) {
      const double q = __dadd_rn(__dmul_rn(static_cast<double>(src[i]), inv), dz);
      int qi = (q >= -2147483648.5 && q < 2147483647.5) ? __double2int_rn(q) : INT_MIN;
      dst[i] = static_cast<uint8_t>(qi < 0 ? 0 : (qi > 255 ? 255 : qi));
    }
  }
}

// out = (float)(((double)q - zero) * (double)scale)  (quant_int8.cpp:162-179)
__global__ void __launch_bounds__(kThreads) dequant_i8_group_kernel(
    const uint8_t *__restrict__ q, int rows, int cols, int groups, const float *__restrict__ scales,
    const uint8_t *__restrict__ zeros, float *__restrict__ out) {
  const int gsz = cols / groups;
  const long long n = static_cast<long long>(rows) * cols;
  const long long stride = static_cast<long long>(gridDim.x) * blockDim.x;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
    const long long g = (i / cols) * groups + (i % cols) / gsz;
    const double v = __dmul_rn(__dsub_rn(static_cast<double>(q[i]), static_cast<double>(zeros[g])),
                               static_cast<double>(scales[g]));
    out[i] = __double2float_rn(v);
  }
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
  for (; i + 3 * stride < n4; i += 4 * stride) {  // four independent loads in flight
    const float4 a = __ldcs(x4 + i), b = __ldcs(x4 + i + stride);
    const float4 c = __ldcs(x4 + i + 2 * stride), d = __ldcs(x4 + i + 3 * stride);
    m0 = fmaxf(m0, fmaxf(absmax4(a), absmax4(c)));
    m1 = fmaxf(m1, fmaxf(absmax4(b), absmax4(d)));
  }
  for (; i < n4; i += stride) m0 = fmaxf(m0, absmax4(__ldcs(x4 + i)));
  for (size_t t = n4 * 4 + tid; t < n; t += stride) m1 = fmaxf(m1, fabsf(x[t]));
  const float m = block_max(fmaxf(m0, m1), red);
  if (threadIdx.x == 0 && m > 0.0f) atomicMax(amax_bits, __float_as_uint(m));
}

// Two f32 values to E4M3 codes with the hardware conversion (round to
// nearest even, saturating to +-448): `lo` in bits 0-7, `hi` in bits 8-15.
__device__ __forceinline__ uint32_t cvt_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// Four codes e4m3(x / s) (element 0 in the low byte) without a division:
// q = x * r with r = 1/s correctly rounded lies within 2^-23 of the
// reference quotient fl(x / s) (relative), so when the hardware codes of
// q * (1 - 2^-21) and q * (1 + 2^-21) agree, every value between them,
// fl(x / s) included, has that code (rounding is monotonic). Elements whose
// bracket straddles a code boundary, non-finite quotients, and nonzero
// quotients below 2^-9 (where the reference drops the sign of results that
// underflow to zero and the hardware keeps it) are flagged in `redo` and
// take the exact path (x86 division and the reference encoder).
__device__ __forceinline__ uint32_t enc4_fast(float4 v, float r, uint32_t &redo) {
  const float q[4] = {__fmul_rn(v.x, r), __fmul_rn(v.y, r), __fmul_rn(v.z, r), __fmul_rn(v.w, r)};
  float lo[4], hi[4];
  uint32_t bad = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    lo[k] = __fmul_rn(q[k], 0.99999952316284180f);  // 1 - 2^-21
    hi[k] = __fmul_rn(q[k], 1.00000047683715820f);  // 1 + 2^-21
    const float aq = fabsf(q[k]);
    bad |= ((!(aq <= 3.0e38f)) || (aq < 0.001953125f && aq != 0.0f)) ? (1u << k) : 0u;
  }
  const uint32_t clo = cvt_e4m3x2(lo[0], lo[1]) | (cvt_e4m3x2(lo[2], lo[3]) << 16);
  const uint32_t chi = cvt_e4m3x2(hi[0], hi[1]) | (cvt_e4m3x2(hi[2], hi[3]) << 16);
  const uint32_t diff = clo ^ chi;
#pragma unroll
  for (int k = 0; k < 4; ++k) bad |= ((diff >> (8 * k)) & 0xFFu) ? (1u << k) : 0u;
  redo = bad;
  return clo;
}

// out[i] = e4m3(x[i] / s), s = amax / 448 (1 when amax == 0). 16 elements
// per thread per step: four 16-byte loads, one 16-byte store. When s is not
// a finite normal float, or r = 1/s is not, every element takes the exact
// path.
__global__ void __launch_bounds__(kThreads) e4m3_scaled_kernel(const float *__restrict__ x,
                                                               size_t n,
                                                               const float *__restrict__ amax,
                                                               float *__restrict__ scale_out,
                                                               uint8_t *__restrict__ out) {
  const float a = __ldg(amax);
  const float s = a > 0.0f ? __fdiv_rn(a, 448.0f) : 1.0f;
  const float r = __frcp_rn(s);
  const bool exact_all = !(fabsf(s) >= 1.1754944e-38f && fabsf(s) <= 3.0e38f &&
                           fabsf(r) >= 1.1754944e-38f && fabsf(r) <= 3.0e38f);
  const size_t tid = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  if (tid == 0 && scale_out) *scale_out = s;
  const size_t n16 = n / 16;
  const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
  const float4 *x4 = reinterpret_cast<const float4 *>(x);
  uint4 *o16 = reinterpret_cast<uint4 *>(out);
  for (size_t i = tid; i < n16; i += stride) {
    float4 v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = __ldcs(x4 + 4 * i + k);
    uint32_t w[4], redo[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      w[k] = enc4_fast(v[k], r, redo[k]);
      if (exact_all) redo[k] = 0xFu;
    }
    if (redo[0] | redo[1] | redo[2] | redo[3]) {  // rare: re-encode flagged elements exactly
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float e[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (redo[k] & (1u << j)) {
            const uint32_t c = encode_e4m3(x86_div(e[j], s));
            w[k] = (w[k] & ~(0xFFu << (8 * j))) | (c << (8 * j));
          }
      }
    }
    o16[i] = make_uint4(w[0], w[1], w[2], w[3]);
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
// Resident CTAs per SM of a kernel, from the occupancy calculator (cached
// per kernel; the value is the same on every B200).
template <class K>
int resident_ctas(K kernel, int &cache) {
  if (cache == 0) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, kThreads, 0) != cudaSuccess) {
      cudaGetLastError();
      n = 4;
    }
    cache = n > 0 ? n : 1;
  }
  return cache * current_sm_count();
}

// One CTA of 12 warps per SM (grid), 12 row slots of shared memory; the
// shared-memory opt-in is set once per device and kernel instance.
template <int VPL>
int launch_quant_tma(const float *x, int rows, int cols, float *scales, int8_t *out, int grid,
                     cudaStream_t st) {
  constexpr int kWarps = 12;
  auto kern = quant_i8_rows_tma_kernel<VPL>;
  static std::atomic<unsigned long long> attr_done{0};
  const unsigned long long bit = 1ull << (current_device() & 63);
  if (!(attr_done.load() & bit)) {
    int s = cuda_status(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kWarps * VPL * 128 * 4));
    if (s != ROUGE_B200_OK) return s;
    attr_done.fetch_or(bit);
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(32 * kWarps, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(kWarps) * cols * 4;
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, kern, x, rows, cols, scales, out,
                                        device_error_word()));
}

int launch_quant_i8_rows(const float *x, int rows, int cols, float *scales, int8_t *out,
                         cudaStream_t st) {
  static int occ4 = 0, occ8 = 0;
  const int nvec = cols / 4;
  const size_t row_bytes = static_cast<size_t>(cols) * 4;
  const int sms = current_sm_count();
  if (nvec <= 1024 && rows >= 2 * sms) {
    // Bulk-copy-fed warps: one CTA of 12 warps per SM, one row slot each.
    const int grid = std::min(sms, rows);
    if (nvec <= 256) return launch_quant_tma<8>(x, rows, cols, scales, out, grid, st);
    if (nvec <= 512) return launch_quant_tma<16>(x, rows, cols, scales, out, grid, st);
    return launch_quant_tma<32>(x, rows, cols, scales, out, grid, st);
  }
  if (row_bytes <= 32768) {
    // Shared-memory row pipeline: 64 KB of rows in flight per CTA (96 KB
    // for 32 KB rows), 2-3 CTAs per SM.
    const int stages =
        row_bytes <= 16384 ? static_cast<int>(std::min<size_t>(8, 65536 / row_bytes)) : 3;
    const int smem = static_cast<int>(stages * row_bytes);
    static std::atomic<unsigned long long> attr_done{0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(attr_done.load() & (1ull << (dev & 63)))) {
      int s = cuda_status(cudaFuncSetAttribute(quant_i8_rows_bulk_kernel,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize, 98304));
      if (s != ROUGE_B200_OK) return s;
      attr_done.fetch_or(1ull << (dev & 63));
    }
    int occ = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, quant_i8_rows_bulk_kernel, kThreads,
                                                      smem) != cudaSuccess || occ < 1) {
      cudaGetLastError();
      occ = 1;
    }
    const int cap = occ * current_sm_count();
    quant_i8_rows_bulk_kernel<<<rows < cap ? rows : cap, kThreads, smem, st>>>(
        x, rows, cols, scales, out, stages, device_error_word());
  } else if (nvec <= 4 * kThreads) {
    const int cap = resident_ctas(quant_i8_rows_kernel<4>, occ4);
    quant_i8_rows_kernel<4><<<rows < cap ? rows : cap, kThreads, 0, st>>>(x, rows, cols, scales, out);
  } else {
    const int cap = resident_ctas(quant_i8_rows_kernel<8>, occ8);
    quant_i8_rows_kernel<8><<<rows < cap ? rows : cap, kThreads, 0, st>>>(x, rows, cols, scales, out);
  }
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

int launch_quant_i8_group(const float *x, int rows, int cols, int groups, float *scales,
                          uint8_t *zeros, uint8_t *out, cudaStream_t st) {
  const long long total = static_cast<long long>(rows) * groups;
  quant_i8_group_kernel<<<stream_grid(static_cast<size_t>(total) * 32), kThreads, 0, st>>>(
      x, rows, cols, groups, scales, zeros, out);
  return cuda_status(cudaGetLastError());
}

int launch_dequant_i8_group(const uint8_t *q, int rows, int cols, int groups, const float *scales,
                            const uint8_t *zeros, float *out, cudaStream_t st) {
  dequant_i8_group_kernel<<<stream_grid(static_cast<size_t>(rows) * cols), kThreads, 0, st>>>(
      q, rows, cols, groups, scales, zeros, out);
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

int rouge_b200_quantize_i8_group(const float *x, int rows, int cols, int groups, float *scales,
                                 uint8_t *zeros, uint8_t *out, void *stream) {
  if (!x || !scales || !zeros || !out || rows <= 0 || cols <= 0 || groups <= 0 ||
      cols % groups != 0)
    return set_status(ROUGE_B200_EINVAL);
  int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  return launch_quant_i8_group(x, rows, cols, groups, scales, zeros, out, as_stream(stream));
}

int rouge_b200_dequantize_i8_group(const uint8_t *q, int rows, int cols, int groups,
                                   const float *scales, const uint8_t *zeros, float *out,
                                   void *stream) {
  if (!q || !scales || !zeros || !out || rows <= 0 || cols <= 0 || groups <= 0 ||
      cols % groups != 0)
    return set_status(ROUGE_B200_EINVAL);
  int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  return launch_dequant_i8_group(q, rows, cols, groups, scales, zeros, out, as_stream(stream));
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
