// OCP narrow formats and MX / NVFP4 block scales, host and device, with the
// rouge-numerics reference semantics bit for bit (narrow.cpp:46-163):
//   e4m3 (bias 7, max 0x7E, NaN 0x7F), e5m2 (bias 15, max 0x7B, Inf 0x7C,
//   NaN 0x7F), e3m2 (bias 3, max 28), e2m3 (bias 1, max 7.5), e2m1 (bias 1,
//   max 6); codes are the format's field in the low bits of a byte.
// Encoding is round to nearest even with saturation to the signed maximum;
// magnitudes below half the smallest subnormal give +0 (the sign dropped);
// NaN gives sign|NaN (e4m3, e5m2) or +MAX (the others). Unlike fp8.cpp's
// e4m3 encoder this generic one keeps a rounded result that lands on the
// NaN pattern (e4m3 values in [464, 512) give sign|0x7F; e5m2 values in
// [61440, 2^17) give the Inf / NaN codes 0x7C-0x7F): the reference does.
// E8M0: value 2^(code - 127), 255 = NaN; the reference's encoder codes a
// power of two 2^p as p + 128 (frexp's exponent), i.e. the stored block
// scale is twice the chosen one.
#pragma once

#include <cstdint>

#include "formats.cuh"

namespace rb200 {

enum NarrowId { kE4M3 = 0, kE5M2 = 1, kE3M2 = 2, kE2M3 = 3, kE2M1 = 4 };

struct NarrowFmt {
  int exp_bits, man_bits, bias;
  uint32_t max_bits, nan_bits;  // field patterns without the sign; nan_bits 0: no NaN
  int width;                    // field width in bits (sign included)
};

// OCP OFP8 Table 1-2 and OCP MX v1.0 Table 7 (the constants of narrow.cpp:61-65).
RB_HD NarrowFmt narrow_fmt(int id) {
  switch (id) {
    case kE4M3: return NarrowFmt{4, 3, 7, 0x7Eu, 0x7Fu, 8};
    case kE5M2: return NarrowFmt{5, 2, 15, 0x7Bu, 0x7Fu, 8};
    case kE3M2: return NarrowFmt{3, 2, 3, 0x1Fu, 0x00u, 6};
    case kE2M3: return NarrowFmt{2, 3, 1, 0x1Fu, 0x00u, 6};
    default: return NarrowFmt{2, 1, 1, 0x07u, 0x00u, 4};
  }
}

// The 6- and 4-bit formats have no NaN: a NaN input encodes as +MAX.
RB_HD bool narrow_nan_to_max(int id) { return id >= kE3M2; }

RB_HD float narrow_decode(uint32_t bits, int id) {
  const NarrowFmt F = narrow_fmt(id);
  const uint32_t sign = ((bits >> (F.width - 1)) & 1u) << 31;
  const uint32_t maxe = (1u << F.exp_bits) - 1u;
  const uint32_t e = (bits >> F.man_bits) & maxe;
  const uint32_t m = bits & ((1u << F.man_bits) - 1u);
  if (e == 0) {
    if (m == 0) return bits_f32(sign);
    const int lz = lead_zeros_small(m, F.man_bits + 1);  // normalise the subnormal
    const uint32_t mm = (m << lz) & ((1u << F.man_bits) - 1u);
    return bits_f32(sign | (static_cast<uint32_t>(128 - F.bias - lz) << 23) |
                    (mm << (23 - F.man_bits)));
  }
  if (e == maxe && F.nan_bits) {
    const bool top_binade_normal = ((F.max_bits >> F.man_bits) & maxe) == maxe;
    if (!top_binade_normal) return bits_f32(sign | (m ? 0x7FC00000u : 0x7F800000u));
    if (m == (1u << F.man_bits) - 1u) return bits_f32(sign | 0x7FC00000u);
  }
  return bits_f32(sign | (static_cast<uint32_t>(static_cast<int>(e) - F.bias + 127) << 23) |
                  (m << (23 - F.man_bits)));
}

// The exact (integer) encoder; nan_to_max as narrow_nan_to_max(id) for the
// reference's public codecs.
RB_HD uint32_t narrow_encode(float f, int id, bool nan_to_max) {
  const NarrowFmt F = narrow_fmt(id);
  const uint32_t x = f32_bits(f);
  const uint32_t bexp = (x >> 23) & 0xFFu, frac = x & 0x7FFFFFu;
  const uint32_t sbit = (x >> 31) << (F.width - 1);
  const int M = F.man_bits;
  const int maxe = (1 << F.exp_bits) - 1;
  const uint32_t field = (1u << F.width) - 1u;
  if (bexp == 0xFFu) {
    if (frac) return nan_to_max ? F.max_bits : (sbit | F.nan_bits);
    return sbit | F.max_bits;
  }
  if ((x & 0x7FFFFFFFu) == 0) return sbit;
  const int te = static_cast<int>(bexp) - 127 + F.bias;
  if (te > maxe) return sbit | F.max_bits;
  if (te <= 0) {
    if (te < -M) return 0;
    return sbit | (shr_rne(frac | 0x800000u, 1 - te + (23 - M)) & field);
  }
  uint32_t q = (static_cast<uint32_t>(te) << M) | (frac >> (23 - M));
  const uint32_t r = frac & ((1u << (23 - M)) - 1u), h = 1u << (22 - M);
  if (r > h || (r == h && (q & 1u))) {
    ++q;
    if (static_cast<int>(q >> M) > maxe) return sbit | F.max_bits;
  }
  return sbit | (q & field);
}

// ------------------------------------------------------------ E8M0 scales

RB_HD float e8m0_decode(uint32_t c) {
  if (c == 255u) return bits_f32(0x7FC00000u);
  return bits_f32(c ? c << 23 : 0x00400000u);
}

// 1 / e8m0_decode(c) for a code the block quantizer produces (128..254):
// 2^(127 - c), exact.
RB_HD float e8m0_inverse(uint32_t c) {
  return bits_f32(c < 254u ? (254u - c) << 23 : 0x00400000u);
}

// Smallest p in [0, 127] with amax <= emax * 2^p (narrow.cpp:213-216; emax
// * 2^p may overflow to +Inf, which ends the search as in the reference).
RB_HD int block_pow(float amax, float emax) {
  if (!(amax > emax)) return 0;
  // start one binade below the estimate, then step as the reference does
  int p = static_cast<int>((f32_bits(amax) >> 23) & 0xFFu) - static_cast<int>((f32_bits(emax) >> 23) & 0xFFu) - 1;
  if (p < 0) p = 0;
  auto scaled = [&](int k) {  // emax * 2^k, exact or +Inf
    const int be = static_cast<int>((f32_bits(emax) >> 23) & 0xFFu) + k;
    return be >= 255 ? bits_f32(0x7F800000u) : bits_f32((f32_bits(emax) & 0x807FFFFFu) | (static_cast<uint32_t>(be) << 23));
  };
  while (p < 127 && amax > scaled(p)) ++p;
  return p;
}

// E8M0 code of the MX block scale 2^p (frexp's exponent: p + 1, clamped).
RB_HD uint32_t mx_scale_code(int p) { return static_cast<uint32_t>((p + 1 > 127 ? 127 : p + 1) + 127); }

#if defined(__CUDACC__)
// ------------------------------------------------ fast device encoders
// Equal to narrow_encode for every input (the hardware conversion covers
// the ordinary range; the reference's edges are patched).

__device__ __forceinline__ uint32_t cvt_pair_e4m3(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t cvt_pair_e5m2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e5m2x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// e4m3 / e5m2 code of v from the hardware code hw (RNE, satfinite): the
// reference differs only for NaN, for magnitudes below 2^-10 (e4m3) /
// 2^-17 (e5m2), which give +0, and for magnitudes from 464 (e4m3) / 61440
// (e5m2) up, where it keeps codes on the NaN / Inf patterns.
template <int ID>
__device__ __forceinline__ uint32_t fix_f8(float v, uint32_t hw) {
  const float a = fabsf(v);
  constexpr float kTiny = ID == kE4M3 ? 0.0009765625f : 7.62939453125e-06f;   // 2^-10, 2^-17
  constexpr float kBig = ID == kE4M3 ? 464.0f : 61440.0f;
  if (a < kTiny) return a == 0.0f ? hw : 0u;  // signed zero kept, tiny values +0
  if (a >= kBig || a != a) return narrow_encode(v, ID, false);
  return hw;
}

template <int ID>
__device__ __forceinline__ uint32_t encode4_f8(float4 v) {
  const uint32_t p0 = ID == kE4M3 ? cvt_pair_e4m3(v.x, v.y) : cvt_pair_e5m2(v.x, v.y);
  const uint32_t p1 = ID == kE4M3 ? cvt_pair_e4m3(v.z, v.w) : cvt_pair_e5m2(v.z, v.w);
  return fix_f8<ID>(v.x, p0 & 0xFFu) | (fix_f8<ID>(v.y, p0 >> 8) << 8) |
         (fix_f8<ID>(v.z, p1 & 0xFFu) << 16) | (fix_f8<ID>(v.w, p1 >> 8) << 24);
}

// e2m1 with NaN -> +MAX: the rounding boundaries of the eight magnitudes
// {0, .5, 1, 1.5, 2, 3, 4, 6}, ties to the even code; magnitudes in
// (0, 0.25) give +0.
__device__ __forceinline__ uint32_t encode_e2m1(float v) {
  const float a = fabsf(v);
  if (a != a) return 0x7u;
  const uint32_t c = (a > 0.25f) + (a >= 0.75f) + (a > 1.25f) + (a >= 1.75f) + (a > 2.5f) +
                     (a >= 3.5f) + (a > 5.0f);
  const uint32_t s = (a >= 0.25f || a == 0.0f) ? (__float_as_uint(v) >> 31) << 3 : 0u;
  return s | c;
}
#endif

}  // namespace rb200
