// int8 codes of the per-row symmetric quantizer (quant_int8.cpp:38-46,
// 72-90) on the device, shared by the row quantizer kernels and the fused
// quantize + GEMM kernel: exact x86 semantics through a double path, a
// single-precision fast path that defers to it near rounding ties, and
// quant_row_smem, one warp's quantization of one row held in shared memory.
#pragma once

#include <cstdint>

#include "ptx.cuh"

namespace rb200 {

// One int8 code from an f32 value and the row's double reciprocal scale,
// as quant_int8.cpp:38-46,87 computes it on x86-64: nearbyint of the
// double product, then a conversion whose out-of-range / NaN result is
// INT32_MIN, then the clamp to [-127, 127].
__device__ __forceinline__ int code_i8_exact(float x, double inv) {
  const double p = __dmul_rn(static_cast<double>(x), inv);
  if (!(p >= -2147483648.5 && p < 2147483647.5)) return -127;  // NaN, +-Inf, overflow
  const int q = __double2int_rn(p);
  return q < -127 ? -127 : (q > 127 ? 127 : q);
}

// Same result as code_i8_exact, mostly in single precision. With
// inv_f = (float)inv the f32 product differs from the double product by
// less than 2^-15 whenever |p| < 2^8, so its round-to-nearest-even integer
// agrees unless p lies within 2^-12 of a half-integer; those elements (and
// large or non-finite products) take the double path. The integer is read
// from the bits of p + 1.5 * 2^23, which rounds to nearest even.
__device__ __forceinline__ int code_i8(float x, double inv, float inv_f) {
  const float p = __fmul_rn(x, inv_f);
  const float big = __fadd_rn(p, 12582912.0f);
  const float r = __fsub_rn(big, 12582912.0f);
  const float dist_to_tie = fabsf(fabsf(__fsub_rn(p, r)) - 0.5f);
  if (!(fabsf(p) < 256.0f) || dist_to_tie < 0.000244140625f) return code_i8_exact(x, inv);
  const int q = static_cast<int>(__float_as_uint(big)) - 0x4B400000;
  return q < -127 ? -127 : (q > 127 ? 127 : q);
}

__device__ __forceinline__ uint32_t pack4(int a, int b, int c, int d) {
  return (static_cast<uint32_t>(a) & 0xFFu) | ((static_cast<uint32_t>(b) & 0xFFu) << 8) |
         ((static_cast<uint32_t>(c) & 0xFFu) << 16) | ((static_cast<uint32_t>(d) & 0xFFu) << 24);
}

constexpr float kRoundMagic = 12582912.0f;  // 1.5 * 2^23

// Single-precision code of one element in the low byte of the returned
// word. p + 1.5*2^23 rounds p to the nearest even integer q and, for
// |q| <= 127, has the bit pattern 0x4B400000 + q, whose low byte is q in
// two's complement; clamping that sum to [magic - 127, magic + 127] is the
// clamp of quant_int8.cpp:45 and maps a NaN product to -127 as x86 does.
// `tie` is set when p lies within 2^-12 of a half-integer (see code_i8).
__device__ __forceinline__ uint32_t code_word(float x, float inv_f, bool &tie) {
  const float p = __fmul_rn(x, inv_f);
  const float big = __fadd_rn(p, kRoundMagic);
  const float r = __fsub_rn(big, kRoundMagic);
  tie |= fabsf(fabsf(__fsub_rn(p, r)) - 0.5f) < 0.000244140625f;
  return __float_as_uint(fminf(fmaxf(big, kRoundMagic - 127.0f), kRoundMagic + 127.0f));
}

// Four codes packed into one word (element 0 in the low byte). Rows whose
// reciprocal scale is not a finite float (scale below 2^-128 or zero: the
// products may overflow to +inf, which x86 maps to -127) and elements near
// a rounding tie take the double-precision path of code_i8_exact.
__device__ __forceinline__ uint32_t encode4_i8(float4 t, double inv, float inv_f, bool exact_row) {
  bool tie = exact_row;
  const uint32_t a = code_word(t.x, inv_f, tie), b = code_word(t.y, inv_f, tie);
  const uint32_t c = code_word(t.z, inv_f, tie), d = code_word(t.w, inv_f, tie);
  if (tie)
    return pack4(code_i8_exact(t.x, inv), code_i8_exact(t.y, inv), code_i8_exact(t.z, inv),
                 code_i8_exact(t.w, inv));
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// encode4_i8 with paired arithmetic. Same codes: the product p = x * inv_f,
// its nearest-even integer through the 1.5 * 2^23 constant, and the
// distance d = p - rne(p) (exact: both subtractions are of nearby values)
// are the f32 path of code_i8; |d| within 2^-12 of 0.5 sends the four
// elements to the double path. On the f32 path (inv_f finite, so the scale
// is above 2^-128 and carries a relative error below 2^-21, subnormal or
// not) |p| = |x| * inv_f <= 127 * (1 + 2^-20) < 127.5 because |x| is at
// most the row maximum; so only the lower clamp is needed, and it maps a
// NaN product to -127.
// Branch-free part: the four f32-path codes, and whether any element lies
// near a tie (the caller re-encodes such words with code_i8_exact).
__device__ __forceinline__ uint32_t encode4_i8_fast(float4 t, float inv_f, bool &tie) {
  float p0, p1, p2, p3, b0, b1, b2, b3, r0, r1, r2, r3, d0, d1, d2, d3;
  mul2(p0, p1, t.x, t.y, inv_f);
  mul2(p2, p3, t.z, t.w, inv_f);
  add2(b0, b1, p0, p1, kRoundMagic, kRoundMagic);
  add2(b2, b3, p2, p3, kRoundMagic, kRoundMagic);
  sub2(r0, r1, b0, b1, kRoundMagic, kRoundMagic);
  sub2(r2, r3, b2, b3, kRoundMagic, kRoundMagic);
  sub2(d0, d1, p0, p1, r0, r1);
  sub2(d2, d3, p2, p3, r2, r3);
  tie = fmaxf(max3(fabsf(d0), fabsf(d1), fabsf(d2)), fabsf(d3)) >= 0.499755859375f;  // 0.5 - 2^-12
  constexpr float lo = kRoundMagic - 127.0f;
  const uint32_t a = __float_as_uint(fmaxf(b0, lo)), b = __float_as_uint(fmaxf(b1, lo));
  const uint32_t c = __float_as_uint(fmaxf(b2, lo)), d = __float_as_uint(fmaxf(b3, lo));
  return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

__device__ __forceinline__ uint32_t encode4_i8_exact(float4 t, double inv) {
  return pack4(code_i8_exact(t.x, inv), code_i8_exact(t.y, inv), code_i8_exact(t.z, inv),
               code_i8_exact(t.w, inv));
}

__device__ __forceinline__ uint32_t encode4_i8_x2(float4 t, double inv, float inv_f,
                                                  bool exact_row) {
  bool tie;
  const uint32_t w = encode4_i8_fast(t, inv_f, tie);
  return (exact_row || tie) ? encode4_i8_exact(t, inv) : w;
}

// One warp quantizes the row of nvec float4 held in shared memory at `row`:
// its scale (quant_int8.cpp:82-84, double arithmetic) to *scale (lane 0)
// and its codes to orow (one 32-bit word per float4). Same scale and codes
// as quant_i8_rows_tma_kernel; the maximum ignores NaN as fmaxf does.
__device__ __forceinline__ void quant_row_smem(const float4 *row, int nvec, uint32_t *orow,
                                               float *scale, int lane) {
  float amax = 0.0f;
#pragma unroll 8
  for (int i = lane; i < nvec; i += 32) {
    const float4 v = row[i];
    amax = max3(amax, max3(fabsf(v.x), fabsf(v.y), fabsf(v.z)), fabsf(v.w));
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const double a = static_cast<double>(amax);
  const float s = a > 0.0 ? __double2float_rn(__ddiv_rn(a, 127.0)) : 1.0f;
  const double inv = __ddiv_rn(1.0, static_cast<double>(s));
  const float inv_f = __double2float_rn(inv);
  const bool exact_row = isinf(inv_f);
  if (lane == 0) *scale = s;
#pragma unroll 8
  for (int i = lane; i < nvec; i += 32) {
    const float4 v = row[i];
    bool tie;
    const uint32_t w = encode4_i8_fast(v, inv_f, tie);
    orow[i] = (tie || exact_row) ? encode4_i8_exact(v, inv) : w;
  }
}

}  // namespace rb200
