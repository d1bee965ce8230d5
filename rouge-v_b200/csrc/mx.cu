// MX / NVFP4 block quantizers and the narrow-format codecs (narrow.cpp:
// 166-331): the reference's host entries (rouge_mx_quantize_f32, ...,
// rouge_quantize_e5m2, ...) and their device-pointer forms.
//
// Blocks are 32 (MX) or 16 (NVFP4) consecutive elements of a flat array,
// the last block partial, exactly as the reference walks them; for an
// [M][K] matrix with K % 32 == 0 they are the per-row K-blocks a
// block-scaled GEMM consumes. Kernels: 8 (MX) or 4 (NVFP4) lanes per block,
// one float4 per lane, block maximum by shuffles, scale, encode 4 elements
// to one 32-bit store; memory-bound (4 B read, 1 B + 1/32 B written per
// element).
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "narrow.cuh"
#include "runtime.cuh"
#include "x86fp.cuh"

namespace rb200 {
namespace {

constexpr int kMxThreads = 256;

__device__ __forceinline__ float4 load4(const float *__restrict__ x, size_t e0, size_t n,
                                        bool vec) {
  if (vec && e0 + 4 <= n) return __ldg(reinterpret_cast<const float4 *>(x + e0));
  float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
  if (e0 < n) v.x = x[e0];
  if (e0 + 1 < n) v.y = x[e0 + 1];
  if (e0 + 2 < n) v.z = x[e0 + 2];
  if (e0 + 3 < n) v.w = x[e0 + 3];
  return v;
}

__device__ __forceinline__ void store4(uint8_t *__restrict__ q, size_t e0, size_t n, bool vec,
                                       uint32_t w) {
  if (vec && e0 + 4 <= n) {
    *reinterpret_cast<uint32_t *>(q + e0) = w;
    return;
  }
  for (int i = 0; i < 4; ++i)
    if (e0 + i < n) q[e0 + i] = static_cast<uint8_t>(w >> (8 * i));
}

__device__ __forceinline__ float amax4(float4 v) {
  return fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
}

// e4m3 / e5m2 codes of x * inv for an MX block (inv = 2^(127 - scale code),
// so every finite |x * inv| <= emax / 2: the reference's overflow edges are
// out of reach). The hardware conversion equals the reference except for
// NaN (sign kept by the reference) and for nonzero magnitudes below half
// the smallest subnormal, which the hardware rounds to a signed zero and
// the reference to +0. Both show cheaply per group of four: a NaN makes
// the sum NaN, a signed zero is a 0x80 byte; such groups take the exact
// path (x86 products, the reference encoder).
template <int ID>
__device__ __forceinline__ uint32_t mx_encode4_f8(float4 x, float inv) {
  const float sum = (x.x + x.y) + (x.z + x.w);
  const uint32_t lo = ID == kE4M3 ? cvt_pair_e4m3(__fmul_rn(x.x, inv), __fmul_rn(x.y, inv))
                                  : cvt_pair_e5m2(__fmul_rn(x.x, inv), __fmul_rn(x.y, inv));
  const uint32_t hi = ID == kE4M3 ? cvt_pair_e4m3(__fmul_rn(x.z, inv), __fmul_rn(x.w, inv))
                                  : cvt_pair_e5m2(__fmul_rn(x.z, inv), __fmul_rn(x.w, inv));
  const uint32_t w = lo | (hi << 16);
  if (sum == sum && __vcmpeq4(w, 0x80808080u) == 0u) return w;
  return narrow_encode(x86_mul(x.x, inv), ID, false) |
         (narrow_encode(x86_mul(x.y, inv), ID, false) << 8) |
         (narrow_encode(x86_mul(x.z, inv), ID, false) << 16) |
         (narrow_encode(x86_mul(x.w, inv), ID, false) << 24);
}

// MXFP8 (ID e4m3 / e5m2) and MXFP4 (e2m1): narrow.cpp:200-265. The block
// maximum ignores NaN (the reference's strict comparison does);
// scale 2^p with the smallest p >= 0 such that amax <= emax * 2^p, stored
// as E8M0 code p + 128, elements encoded from x * 2^(127 - code).
template <int ID>
__global__ void __launch_bounds__(kMxThreads, 8)
    mx_quant_kernel(const float *__restrict__ x, size_t n, uint8_t *__restrict__ codes,
                    uint8_t *__restrict__ scales, int vec_in, int vec_out) {
  constexpr float kEmax = ID == kE4M3 ? 448.0f : ID == kE5M2 ? 57344.0f : 6.0f;
  constexpr int kU = 4;  // groups of 4 blocks per warp iteration: kU loads in flight per lane
  const size_t nblk = (n + 31) / 32;
  const int lane = threadIdx.x & 31, sub = lane & 7;
  const size_t nwarps = (static_cast<size_t>(gridDim.x) * blockDim.x) >> 5;
  for (size_t b0 = ((static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5) * 4 * kU;
       b0 < nblk; b0 += nwarps * 4 * kU) {
    float4 v[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const size_t blk = b0 + u * 4 + (lane >> 3);
      v[u] = blk < nblk ? load4(x, blk * 32 + sub * 4, n, vec_in) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const size_t blk = b0 + u * 4 + (lane >> 3);
      float a = amax4(v[u]);
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
      a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 4));
      const uint32_t sc = mx_scale_code(a > 0.0f ? block_pow(a, kEmax) : 0);
      const float inv = e8m0_inverse(sc);
      if (blk >= nblk) continue;
      if (sub == 0) scales[blk] = static_cast<uint8_t>(sc);
      uint32_t w;
      if constexpr (ID == kE2M1) {
        // (the sign of a NaN does not matter: e2m1 codes it +MAX)
        w = encode_e2m1(__fmul_rn(v[u].x, inv)) | (encode_e2m1(__fmul_rn(v[u].y, inv)) << 8) |
            (encode_e2m1(__fmul_rn(v[u].z, inv)) << 16) | (encode_e2m1(__fmul_rn(v[u].w, inv)) << 24);
      } else {
        w = mx_encode4_f8<ID>(v[u], inv);
      }
      store4(codes, blk * 32 + sub * 4, n, vec_out, w);
    }
  }
}

// Four e2m1 codes (RNE, satfinite) from the hardware conversion, one per
// nibble, x0 in the low nibble.
__device__ __forceinline__ uint32_t cvt4_e2m1(float x0, float x1, float x2, float x3) {
  uint16_t r;
  asm("{\n\t.reg .b8 t0, t1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t1, %4, %3;\n\t"
      "mov.b16 %0, {t0, t1};\n\t}"
      : "=h"(r)
      : "f"(x0), "f"(x1), "f"(x2), "f"(x3));
  return r;
}

__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// e2m1 input fix: the reference encodes magnitudes in (0, 0.25) as +0, the
// hardware as a signed zero; zeroing the negative ones first makes them
// agree (-0.25 and -0 keep their sign in both).
__device__ __forceinline__ float e2m1_pre(float y) { return (y > -0.25f && y < 0.0f) ? 0.0f : y; }

// MXFP8 / MXFP4 fast kernel (e4m3 / e5m2 / e2m1, whole blocks, 16-byte aligned x and
// codes): two lanes per 32-element block, 16 consecutive elements (four
// float4) per lane, so that the block maximum takes one shuffle and the
// scale work is shared by 16 elements; the codes leave as one 16-byte
// store per lane. The hardware codes equal the reference's (see
// mx_encode4_f8) except for NaN inputs (codes 0x7F / 0xFF, which no finite
// |x * inv| <= emax / 2 produces) and for 0x80 bytes: those are redone per
// element (a 0x80 byte stands for -0, -2^-10 in e4m3 or -2^-17 in e5m2,
// kept by the reference, or a tinier negative value, which it makes +0).
// (MXFP4: e2m1 codes from the hardware conversion of values whose
// (-0.25, 0) part is zeroed first; a block holding a NaN, found by a
// NaN-propagating maximum, takes the exact threshold encoder.)
template <int ID>
__global__ void __launch_bounds__(kMxThreads, 4)
    mx_quant_blocks_kernel(const float4 *__restrict__ x, uint32_t nblk, uint4 *__restrict__ codes,
                           uint8_t *__restrict__ scales) {
  constexpr float kEmax = ID == kE4M3 ? 448.0f : (ID == kE5M2 ? 57344.0f : 6.0f);
  constexpr float kTiny = ID == kE4M3 ? 0.0009765625f : 7.62939453125e-06f;  // 2^-10, 2^-17
  const uint32_t lane = threadIdx.x & 31;
  const uint32_t stride = (gridDim.x * blockDim.x) >> 1;  // blocks per grid step
  for (uint32_t blk = (blockIdx.x * blockDim.x + threadIdx.x) >> 1; ; blk += stride) {
    // (warp-uniform exit: all lanes of a warp cover 16 consecutive blocks)
    if (__shfl_sync(0xffffffffu, blk, 0) >= nblk) break;
    const bool live = blk < nblk;
    const uint32_t q0 = blk * 8u + (lane & 1u) * 4u;  // first float4 of this lane
    float4 v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = live ? __ldg(x + q0 + j) : make_float4(0.f, 0.f, 0.f, 0.f);
    float a = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j) a = fmaxf(a, amax4(v[j]));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
    const uint32_t sc = mx_scale_code(a > kEmax ? block_pow(a, kEmax) : 0);
    const float inv = e8m0_inverse(sc);
    uint32_t w[4];
    if constexpr (ID == kE2M1) {
      float mn = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j)
        mn = max_nan(mn, max_nan(max_nan(fabsf(v[j].x), fabsf(v[j].y)),
                                 max_nan(fabsf(v[j].z), fabsf(v[j].w))));
      const bool nan = mn != mn;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float y0 = __fmul_rn(v[j].x, inv), y1 = __fmul_rn(v[j].y, inv);
        const float y2 = __fmul_rn(v[j].z, inv), y3 = __fmul_rn(v[j].w, inv);
        uint32_t c;
        if (nan) {
          c = encode_e2m1(y0) | (encode_e2m1(y1) << 8) | (encode_e2m1(y2) << 16) |
              (encode_e2m1(y3) << 24);
        } else {
          const uint32_t h = cvt4_e2m1(e2m1_pre(y0), e2m1_pre(y1), e2m1_pre(y2), e2m1_pre(y3));
          c = (h & 0xFu) | ((h & 0xF0u) << 4) | ((h & 0xF00u) << 8) | ((h & 0xF000u) << 12);
        }
        w[j] = c;
      }
    } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t lo = ID == kE4M3 ? cvt_pair_e4m3(__fmul_rn(v[j].x, inv), __fmul_rn(v[j].y, inv))
                                      : cvt_pair_e5m2(__fmul_rn(v[j].x, inv), __fmul_rn(v[j].y, inv));
      const uint32_t hi = ID == kE4M3 ? cvt_pair_e4m3(__fmul_rn(v[j].z, inv), __fmul_rn(v[j].w, inv))
                                      : cvt_pair_e5m2(__fmul_rn(v[j].z, inv), __fmul_rn(v[j].w, inv));
      w[j] = lo | (hi << 16);
    }
    // bytes with (b & 0x7F) == 0x7F (NaN) or b == 0x80
    uint32_t odd = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t t = w[j] ^ 0x80808080u;
      odd |= (((w[j] & 0x7F7F7F7Fu) + 0x01010101u) | ((t - 0x01010101u) & ~t)) & 0x80808080u;
    }
    if (odd) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float e[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t b = (w[j] >> (8 * i)) & 0xFFu;
          if (b == 0x80u || (b & 0x7Fu) == 0x7Fu) {
            const float y = x86_mul(e[i], inv);
            const uint32_t c = (b == 0x80u && y != 0.0f && fabsf(y) < kTiny)
                                   ? 0u
                                   : narrow_encode(y, ID, false);
            w[j] = (w[j] & ~(0xFFu << (8 * i))) | (c << (8 * i));
          }
        }
      }
    }
    }  // (e4m3 / e5m2)
    if (!live) continue;
    if ((lane & 1u) == 0) scales[blk] = static_cast<uint8_t>(sc);
    codes[blk * 2u + (lane & 1u)] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// NVFP4: narrow.cpp:270-300. Blocks of 16 e2m1 codes, 4 lanes per block;
// block maximum of |x| * gs, block scale 2^p coded by the generic e4m3
// encoder (2^9 and above saturate to 448), elements x * (1 / (scale * gs)).
__global__ void __launch_bounds__(kMxThreads)
    nvfp4_quant_kernel(const float *__restrict__ x, size_t n, float gs,
                       uint8_t *__restrict__ codes, uint8_t *__restrict__ scales, int vec_in,
                       int vec_out) {
  const size_t nblk = (n + 15) / 16;
  const int lane = threadIdx.x & 31, sub = lane & 3;
  const size_t nwarps = (static_cast<size_t>(gridDim.x) * blockDim.x) >> 5;
  for (size_t b0 = ((static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5) * 8;
       b0 < nblk; b0 += nwarps * 8) {
    const size_t blk = b0 + (lane >> 2);
    const size_t e0 = blk * 16 + sub * 4;
    const float4 v = blk < nblk ? load4(x, e0, n, vec_in) : make_float4(0.f, 0.f, 0.f, 0.f);
    float a = fmaxf(fmaxf(__fmul_rn(fabsf(v.x), gs), __fmul_rn(fabsf(v.y), gs)),
                    fmaxf(__fmul_rn(fabsf(v.z), gs), __fmul_rn(fabsf(v.w), gs)));
    // elements past n are zeros: 0 * gs = 0 leaves the maximum unchanged
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
    a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
    const int p = a > 0.0f ? block_pow(a, 448.0f) : 0;
    const uint32_t sc = narrow_encode(__uint_as_float(static_cast<uint32_t>(p + 127) << 23), kE4M3,
                                      false);
    const float inv = __fdiv_rn(1.0f, __fmul_rn(narrow_decode(sc, kE4M3), gs));
    if (blk >= nblk) continue;
    if (sub == 0) scales[blk] = static_cast<uint8_t>(sc);
    const uint32_t w = encode_e2m1(__fmul_rn(v.x, inv)) | (encode_e2m1(__fmul_rn(v.y, inv)) << 8) |
                       (encode_e2m1(__fmul_rn(v.z, inv)) << 16) |
                       (encode_e2m1(__fmul_rn(v.w, inv)) << 24);
    store4(codes, e0, n, vec_out, w);
  }
}

// NVFP4 fast kernel (16-byte aligned x, whole blocks): one lane per
// 16-element block (four float4), no shuffles. The block maximum uses a
// NaN-propagating max: a block holding a NaN takes the exact per-element
// encoder instead. max(|x| * gs) == max|x| * gs (rounding is monotonic).
// PACKED: codes leave two per byte (8 bytes per block) for the fp4 GEMM,
// otherwise one per byte (the reference's layout, 16 bytes per block).
template <bool PACKED>
__global__ void __launch_bounds__(kMxThreads)
    nvfp4_quant_blocks_kernel(const float4 *__restrict__ x, uint32_t nblk, float gs,
                              uint8_t *__restrict__ codes, uint8_t *__restrict__ scales) {
  for (uint32_t blk = blockIdx.x * blockDim.x + threadIdx.x; blk < nblk;
       blk += gridDim.x * blockDim.x) {
    float4 v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = __ldg(x + blk * 4u + j);
    float m = 0.0f;
#pragma unroll
    for (int j = 0; j < 4; ++j)
      m = max_nan(m, max_nan(max_nan(fabsf(v[j].x), fabsf(v[j].y)),
                             max_nan(fabsf(v[j].z), fabsf(v[j].w))));
    const bool has_nan = m != m;
    if (has_nan) {  // the reference's maximum skips NaN
      m = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j) m = fmaxf(m, amax4(v[j]));
    }
    const float amax = __fmul_rn(m, gs);
    const int p = amax > 448.0f ? block_pow(amax, 448.0f) : 0;
    const uint32_t sc = p <= 8 ? static_cast<uint32_t>(p + 7) << 3 : 0x7Eu;  // e4m3 of 2^p
    const float inv = __fdiv_rn(1.0f, __fmul_rn(narrow_decode(sc, kE4M3), gs));
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float y0 = __fmul_rn(v[j].x, inv), y1 = __fmul_rn(v[j].y, inv);
      const float y2 = __fmul_rn(v[j].z, inv), y3 = __fmul_rn(v[j].w, inv);
      if (has_nan)
        w[j] = encode_e2m1(y0) | (encode_e2m1(y1) << 4) | (encode_e2m1(y2) << 8) |
               (encode_e2m1(y3) << 12);
      else
        w[j] = cvt4_e2m1(e2m1_pre(y0), e2m1_pre(y1), e2m1_pre(y2), e2m1_pre(y3));
    }
    scales[blk] = static_cast<uint8_t>(sc);
    if constexpr (PACKED) {
      reinterpret_cast<uint2 *>(codes)[blk] = make_uint2(w[0] | (w[1] << 16), w[2] | (w[3] << 16));
    } else {
      uint32_t b[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        b[j] = (w[j] & 0xFu) | ((w[j] & 0xF0u) << 4) | ((w[j] & 0xF00u) << 8) |
               ((w[j] & 0xF000u) << 12);
      reinterpret_cast<uint4 *>(codes)[blk] = make_uint4(b[0], b[1], b[2], b[3]);
    }
  }
}

// narrow.cpp:304-331: out = decode(code) * 2^(scale - 127), the product with
// x86's NaN rules (a NaN code keeps its sign and payload).
template <int ID>
__global__ void __launch_bounds__(kMxThreads)
    mx_dequant_kernel(const uint8_t *__restrict__ codes, const uint8_t *__restrict__ scales,
                      size_t n, float *__restrict__ out, int vec) {
  __shared__ float lut[256];
  for (int c = threadIdx.x; c < 256; c += blockDim.x)
    lut[c] = narrow_decode(ID == kE2M1 ? (c & 0x0F) : c, ID);
  __syncthreads();
  for (size_t e0 = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4; e0 < n;
       e0 += static_cast<size_t>(gridDim.x) * blockDim.x * 4) {
    const float s = e8m0_decode(scales[e0 / 32]);
    if (vec && e0 + 4 <= n) {
      const uint32_t w = __ldg(reinterpret_cast<const uint32_t *>(codes + e0));
      *reinterpret_cast<float4 *>(out + e0) =
          make_float4(x86_mul(lut[w & 0xFF], s), x86_mul(lut[(w >> 8) & 0xFF], s),
                      x86_mul(lut[(w >> 16) & 0xFF], s), x86_mul(lut[w >> 24], s));
    } else {
      for (int i = 0; i < 4 && e0 + i < n; ++i) out[e0 + i] = x86_mul(lut[codes[e0 + i]], s);
    }
  }
}

// Scale re-layout for the block-scaled GEMM: src [rows][K/32] (the block
// quantizer's scales of a row-major [rows][K] matrix) into 512-byte atoms
// [ceil(rows/128)][ceil(K/128)], atom byte 16*(r%32) + 4*(r/32) + j = the
// scale of row 128*rb + r, K-block 4*kb + j (the layout tcgen05.cp
// 32x128b.warpx4 turns into TMEM words: lane r%32, column r/32, byte j).
// Rows or K-blocks past the matrix get 127 (scale 1: their operand bytes
// are zero-filled by the GEMM's loads).
// (generic form: `per_row` scales per row in src, `groups` atoms per 128
// rows in dst, `pad` for positions past the matrix)
__global__ void mx_scale_atoms_kernel(const uint8_t *__restrict__ src, int rows, int per_row,
                                      uint8_t *__restrict__ dst, int groups, size_t atoms,
                                      uint8_t pad) {
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < atoms * 512;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const size_t atom = i >> 9;
    const int off = static_cast<int>(i & 511);
    const int rb = static_cast<int>(atom / groups), kb = static_cast<int>(atom % groups);
    const int r = (off >> 4) + 32 * ((off >> 2) & 3), j = off & 3;
    const int row = rb * 128 + r, col = kb * 4 + j;
    dst[i] = (row < rows && col < per_row) ? src[static_cast<size_t>(row) * per_row + col] : pad;
  }
}

// Two e2m1 codes per byte, the lower-index element in the low nibble
// (the packed operand layout of the fp4 tensor-core kinds).
__global__ void fp4_pack_kernel(const uint32_t *__restrict__ codes, size_t nwords,
                                uint16_t *__restrict__ packed) {
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < nwords;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const uint32_t w = codes[i];
    packed[i] = static_cast<uint16_t>((w & 0xFu) | ((w >> 4) & 0xF0u) | ((w >> 8) & 0xF00u) |
                                      ((w >> 12) & 0xF000u));
  }
}

unsigned grid_for(size_t work_items, int per_block) {
  const size_t need = (work_items + per_block - 1) / per_block;
  const size_t cap = static_cast<size_t>(current_sm_count()) * 8;
  return static_cast<unsigned>(need < 1 ? 1 : (need < cap ? need : cap));
}

bool a16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
bool a4(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }

}  // namespace

int launch_mx_quantize(const float *x, size_t n, int fmt, uint8_t *codes, uint8_t *scales,
                       cudaStream_t st) {
  // MXFP8 with aligned operands: whole blocks by the fast kernel, a partial
  // last block by the general one
  const size_t full = n / 32;
  if (a16(x) && a16(codes) && full > 0 && full < (1u << 28)) {
    const size_t want = (full + kMxThreads / 2 - 1) / (kMxThreads / 2);
    const size_t cap = static_cast<size_t>(current_sm_count()) * 4;  // resident CTAs
    const unsigned g = static_cast<unsigned>(want < cap ? want : cap);
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    uint4 *c4 = reinterpret_cast<uint4 *>(codes);
    const uint32_t nb = static_cast<uint32_t>(full);
    if (fmt == kE4M3)
      mx_quant_blocks_kernel<kE4M3><<<g, kMxThreads, 0, st>>>(x4, nb, c4, scales);
    else if (fmt == kE5M2)
      mx_quant_blocks_kernel<kE5M2><<<g, kMxThreads, 0, st>>>(x4, nb, c4, scales);
    else
      mx_quant_blocks_kernel<kE2M1><<<g, kMxThreads, 0, st>>>(x4, nb, c4, scales);
    const int s = cuda_status(cudaGetLastError());
    if (s != ROUGE_B200_OK || full * 32 == n) return s;
    x += full * 32;
    codes += full * 32;
    scales += full;
    n -= full * 32;
  }
  const unsigned grid = grid_for((n + 31) / 32, kMxThreads / 8 * 4);
  const int vi = a16(x), vo = a4(codes);
  switch (fmt) {
    case kE4M3: mx_quant_kernel<kE4M3><<<grid, kMxThreads, 0, st>>>(x, n, codes, scales, vi, vo); break;
    case kE5M2: mx_quant_kernel<kE5M2><<<grid, kMxThreads, 0, st>>>(x, n, codes, scales, vi, vo); break;
    default: mx_quant_kernel<kE2M1><<<grid, kMxThreads, 0, st>>>(x, n, codes, scales, vi, vo); break;
  }
  return cuda_status(cudaGetLastError());
}

int launch_nvfp4_quantize(const float *x, size_t n, float gs, uint8_t *codes, uint8_t *scales,
                          cudaStream_t st) {
  // whole blocks of aligned operands by the fast kernel, a partial last
  // block by the general one
  const size_t full = n / 16;
  if (a16(x) && a16(codes) && full > 0 && full < (1u << 28)) {
    const size_t want = (full + kMxThreads - 1) / kMxThreads;
    const size_t cap = static_cast<size_t>(current_sm_count()) * 8;
    nvfp4_quant_blocks_kernel<false><<<static_cast<unsigned>(want < cap ? want : cap), kMxThreads,
                                       0, st>>>(reinterpret_cast<const float4 *>(x),
                                                static_cast<uint32_t>(full), gs, codes, scales);
    const int s = cuda_status(cudaGetLastError());
    if (s != ROUGE_B200_OK || full * 16 == n) return s;
    x += full * 16;
    codes += full * 16;
    scales += full;
    n -= full * 16;
  }
  const unsigned grid = grid_for((n + 15) / 16, kMxThreads / 4);
  nvfp4_quant_kernel<<<grid, kMxThreads, 0, st>>>(x, n, gs, codes, scales, a16(x), a4(codes));
  return cuda_status(cudaGetLastError());
}

int launch_mx_dequantize(const uint8_t *codes, const uint8_t *scales, size_t n, int fmt,
                         float *out, cudaStream_t st) {
  const unsigned grid = grid_for((n + 3) / 4, kMxThreads);
  const int v = a4(codes) && a16(out);
  switch (fmt) {
    case kE4M3: mx_dequant_kernel<kE4M3><<<grid, kMxThreads, 0, st>>>(codes, scales, n, out, v); break;
    case kE5M2: mx_dequant_kernel<kE5M2><<<grid, kMxThreads, 0, st>>>(codes, scales, n, out, v); break;
    default: mx_dequant_kernel<kE2M1><<<grid, kMxThreads, 0, st>>>(codes, scales, n, out, v); break;
  }
  return cuda_status(cudaGetLastError());
}

namespace {

bool valid_mx_fmt(int fmt) { return fmt == kE4M3 || fmt == kE5M2 || fmt == kE2M1; }

// Ends a host-pointer call: waits for the stream, folds in device failures.
int call_finish(cudaStream_t st) {
  const int s = cuda_status(cudaStreamSynchronize(st));
  return s != ROUGE_B200_OK ? s : take_device_error(st);
}

// Host-pointer call: x (n floats) in, codes (n bytes) and scales out.
int host_quantize(const float *x, int n, int fmt, float gs, bool nv, uint8_t *out,
                  uint8_t *scale_out) {
  HostCallContext *ctx = host_context();
  if (!ctx) return 0;
  std::lock_guard<std::mutex> g(ctx->lock);
  const size_t nn = static_cast<size_t>(n);
  const size_t nblk = nv ? (nn + 15) / 16 : (nn + 31) / 32;
  const size_t need = round_up(nn * 4, 256) + round_up(nn, 256) + round_up(nblk, 256);
  if (ensure_workspace(ctx, need) != ROUGE_B200_OK) return 0;
  uint8_t *base = static_cast<uint8_t *>(ctx->ws);
  float *dx = reinterpret_cast<float *>(base);
  uint8_t *dq = base + round_up(nn * 4, 256);
  uint8_t *ds = dq + round_up(nn, 256);
  cudaStream_t st = ctx->stream;
  int s = cuda_status(cudaMemcpyAsync(dx, x, nn * 4, cudaMemcpyHostToDevice, st));
  if (s == ROUGE_B200_OK)
    s = nv ? launch_nvfp4_quantize(dx, nn, gs, dq, ds, st) : launch_mx_quantize(dx, nn, fmt, dq, ds, st);
  if (s == ROUGE_B200_OK) s = cuda_status(cudaMemcpyAsync(out, dq, nn, cudaMemcpyDeviceToHost, st));
  if (s == ROUGE_B200_OK)
    s = cuda_status(cudaMemcpyAsync(scale_out, ds, nblk, cudaMemcpyDeviceToHost, st));
  const int f = call_finish(st);
  return s == ROUGE_B200_OK && f == ROUGE_B200_OK ? static_cast<int>(nblk) : 0;
}

void host_dequantize(const uint8_t *in, const uint8_t *scales, int n, int fmt, float *out) {
  HostCallContext *ctx = host_context();
  if (!ctx) return;
  std::lock_guard<std::mutex> g(ctx->lock);
  const size_t nn = static_cast<size_t>(n), nblk = (nn + 31) / 32;
  const size_t need = round_up(nn * 4, 256) + round_up(nn, 256) + round_up(nblk, 256);
  if (ensure_workspace(ctx, need) != ROUGE_B200_OK) return;
  uint8_t *base = static_cast<uint8_t *>(ctx->ws);
  float *dout = reinterpret_cast<float *>(base);
  uint8_t *dq = base + round_up(nn * 4, 256);
  uint8_t *ds = dq + round_up(nn, 256);
  cudaStream_t st = ctx->stream;
  int s = cuda_status(cudaMemcpyAsync(dq, in, nn, cudaMemcpyHostToDevice, st));
  if (s == ROUGE_B200_OK) s = cuda_status(cudaMemcpyAsync(ds, scales, nblk, cudaMemcpyHostToDevice, st));
  if (s == ROUGE_B200_OK) s = launch_mx_dequantize(dq, ds, nn, fmt, dout, st);
  if (s == ROUGE_B200_OK) s = cuda_status(cudaMemcpyAsync(out, dout, nn * 4, cudaMemcpyDeviceToHost, st));
  call_finish(st);
}

}  // namespace
}  // namespace rb200

using namespace rb200;

extern "C" {

// numerics.h:257-264: single-value codecs (host), narrow.cpp:166-198.
uint8_t rouge_quantize_e5m2(float f) { return static_cast<uint8_t>(narrow_encode(f, kE5M2, false)); }
float rouge_dequantize_e5m2(uint8_t u) { return narrow_decode(u, kE5M2); }
uint8_t rouge_quantize_e3m2(float f) { return static_cast<uint8_t>(narrow_encode(f, kE3M2, true) & 0x3Fu); }
float rouge_dequantize_e3m2(uint8_t u) { return narrow_decode(u & 0x3Fu, kE3M2); }
uint8_t rouge_quantize_e2m3(float f) { return static_cast<uint8_t>(narrow_encode(f, kE2M3, true) & 0x3Fu); }
float rouge_dequantize_e2m3(uint8_t u) { return narrow_decode(u & 0x3Fu, kE2M3); }
uint8_t rouge_quantize_e2m1(float f) { return static_cast<uint8_t>(narrow_encode(f, kE2M1, true) & 0x0Fu); }
float rouge_dequantize_e2m1(uint8_t u) { return narrow_decode(u & 0x0Fu, kE2M1); }

// numerics.h:278-289 (narrow.cpp:200-331). Invalid arguments: 0 / no write.
int rouge_mx_quantize_f32(const float *x, int n, int elem_bytes, uint8_t *out, uint8_t *scale_out) {
  if (!x || !out || !scale_out || n <= 0 || (elem_bytes != 1 && elem_bytes != 2)) return 0;
  return host_quantize(x, n, elem_bytes == 1 ? kE4M3 : kE5M2, 1.0f, false, out, scale_out);
}

int rouge_mx_quantize_f32_e2m1(const float *x, int n, uint8_t *out, uint8_t *scale_out) {
  if (!x || !out || !scale_out || n <= 0) return 0;
  return host_quantize(x, n, kE2M1, 1.0f, false, out, scale_out);
}

int rouge_nvfp4_quantize_f32(const float *x, int n, float global_scale, uint8_t *out,
                             uint8_t *scale_out) {
  if (!x || !out || !scale_out || n <= 0) return 0;
  if (!(global_scale > 0.0f)) global_scale = 1.0f;
  return host_quantize(x, n, kE2M1, global_scale, true, out, scale_out);
}

void rouge_mx_dequantize_f32(const uint8_t *in, const uint8_t *scales, int n, int elem_bytes,
                             float *out) {
  if (!in || !scales || !out || n <= 0 || (elem_bytes != 1 && elem_bytes != 2)) return;
  host_dequantize(in, scales, n, elem_bytes == 1 ? kE4M3 : kE5M2, out);
}

void rouge_mx_dequantize_f32_e2m1(const uint8_t *in, const uint8_t *scales, int n, float *out) {
  if (!in || !scales || !out || n <= 0) return;
  host_dequantize(in, scales, n, kE2M1, out);
}

// Device-pointer forms (asynchronous on `stream`).
int rouge_b200_mx_quantize(const float *x, size_t n, int fmt, uint8_t *codes, uint8_t *scales,
                           void *stream) {
  if (!x || !codes || !scales || n == 0 || !valid_mx_fmt(fmt)) return set_status(ROUGE_B200_EINVAL);
  const int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  return launch_mx_quantize(x, n, fmt, codes, scales, as_stream(stream));
}

int rouge_b200_nvfp4_quantize(const float *x, size_t n, float global_scale, uint8_t *codes,
                              uint8_t *scales, void *stream) {
  if (!x || !codes || !scales || n == 0) return set_status(ROUGE_B200_EINVAL);
  const int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  if (!(global_scale > 0.0f)) global_scale = 1.0f;
  return launch_nvfp4_quantize(x, n, global_scale, codes, scales, as_stream(stream));
}

size_t rouge_b200_mx_scale_atoms_bytes(int rows, int K) {
  if (rows <= 0 || K <= 0) return 0;
  return static_cast<size_t>((rows + 127) / 128) * ((K + 127) / 128) * 512;
}

int rouge_b200_mx_scale_atoms(const uint8_t *scales, int rows, int K, uint8_t *atoms,
                              void *stream) {
  if (!scales || !atoms || rows <= 0 || K <= 0 || K % 32) return set_status(ROUGE_B200_EINVAL);
  const int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  const size_t n = rouge_b200_mx_scale_atoms_bytes(rows, K) / 512;
  mx_scale_atoms_kernel<<<grid_for(n * 512, kMxThreads), kMxThreads, 0, as_stream(stream)>>>(
      scales, rows, K / 32, atoms, (K + 127) / 128, n, 127);
  return cuda_status(cudaGetLastError());
}

// NVFP4: K / 16 UE4M3 scales per row; four atoms (256 K) per GEMM stage.
size_t rouge_b200_nvfp4_scale_atoms_bytes(int rows, int K) {
  if (rows <= 0 || K <= 0) return 0;
  return static_cast<size_t>((rows + 127) / 128) * ((K + 255) / 256) * 4 * 512;
}

int rouge_b200_nvfp4_scale_atoms(const uint8_t *scales, int rows, int K, uint8_t *atoms,
                                 void *stream) {
  if (!scales || !atoms || rows <= 0 || K <= 0 || K % 16) return set_status(ROUGE_B200_EINVAL);
  const int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  const size_t n = rouge_b200_nvfp4_scale_atoms_bytes(rows, K) / 512;
  // pad with 0x38 (UE4M3 1.0): the padded K positions of the operands are zero
  mx_scale_atoms_kernel<<<grid_for(n * 512, kMxThreads), kMxThreads, 0, as_stream(stream)>>>(
      scales, rows, K / 16, atoms, (K + 255) / 256 * 4, n, 0x38);
  return cuda_status(cudaGetLastError());
}

// MXFP4 operands of the fp4 GEMM: K / 32 E8M0 scales per row, two atoms
// per 256 K.
size_t rouge_b200_mxfp4_scale_atoms_bytes(int rows, int K) {
  if (rows <= 0 || K <= 0) return 0;
  return static_cast<size_t>((rows + 127) / 128) * ((K + 255) / 256) * 2 * 512;
}

int rouge_b200_mxfp4_scale_atoms(const uint8_t *scales, int rows, int K, uint8_t *atoms,
                                 void *stream) {
  if (!scales || !atoms || rows <= 0 || K <= 0 || K % 32) return set_status(ROUGE_B200_EINVAL);
  const int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  const size_t n = rouge_b200_mxfp4_scale_atoms_bytes(rows, K) / 512;
  mx_scale_atoms_kernel<<<grid_for(n * 512, kMxThreads), kMxThreads, 0, as_stream(stream)>>>(
      scales, rows, K / 32, atoms, (K + 255) / 256 * 2, n, 127);
  return cuda_status(cudaGetLastError());
}

int rouge_b200_fp4_pack(const uint8_t *codes, size_t n, uint8_t *packed, void *stream) {
  if (!codes || !packed || n == 0 || n % 4 || !a4(codes) || (reinterpret_cast<uintptr_t>(packed) & 1u))
    return set_status(ROUGE_B200_EINVAL);
  const int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  fp4_pack_kernel<<<grid_for(n / 4, kMxThreads), kMxThreads, 0, as_stream(stream)>>>(
      reinterpret_cast<const uint32_t *>(codes), n / 4, reinterpret_cast<uint16_t *>(packed));
  return cuda_status(cudaGetLastError());
}

int rouge_b200_nvfp4_quantize_packed(const float *x, size_t n, float global_scale,
                                     uint8_t *packed, uint8_t *scales, void *stream) {
  if (!x || !packed || !scales || n == 0 || n % 16 || (n / 16) >= (1u << 28) ||
      (reinterpret_cast<uintptr_t>(x) & 15u) || (reinterpret_cast<uintptr_t>(packed) & 7u))
    return set_status(ROUGE_B200_EINVAL);
  const int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  if (!(global_scale > 0.0f)) global_scale = 1.0f;
  const size_t full = n / 16;
  const size_t want = (full + kMxThreads - 1) / kMxThreads;
  const size_t cap = static_cast<size_t>(current_sm_count()) * 8;
  nvfp4_quant_blocks_kernel<true><<<static_cast<unsigned>(want < cap ? want : cap), kMxThreads, 0,
                                    as_stream(stream)>>>(reinterpret_cast<const float4 *>(x),
                                                         static_cast<uint32_t>(full), global_scale,
                                                         packed, scales);
  return cuda_status(cudaGetLastError());
}

int rouge_b200_mx_dequantize(const uint8_t *codes, const uint8_t *scales, size_t n, int fmt,
                             float *out, void *stream) {
  if (!codes || !scales || !out || n == 0 || !valid_mx_fmt(fmt)) return set_status(ROUGE_B200_EINVAL);
  const int s = device_ready();
  if (s != ROUGE_B200_OK) return s;
  return launch_mx_dequantize(codes, scales, n, fmt, out, as_stream(stream));
}

}  // extern "C"
