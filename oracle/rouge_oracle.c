/*
 * TEST INFRASTRUCTURE ONLY -- CPU oracle for the rouge-numerics hot path.
 *
 * A plain-C restatement of the reference algorithms, used by tests/, by
 * __graft_entry__.smoke() and by bench.py's cpu_baseline leg as the checker.
 * The product (rouge-v_b200/) never links, loads or calls this file.
 *
 * Every function names the reference lines it restates
 * (software/rouge-numerics/src/<file>:<line>). Parity of this restatement is
 * pinned two ways: against the golden vectors of the reference's own tests
 * (tests/test_oracle_golden.py) and against the reference library itself,
 * compiled from its sources into oracle/_ref/ (tests/test_oracle_vs_ref.py).
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>

static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ---- IEEE half <-> f32: fp16.cpp:31-58 (decode), :61-92 (encode) ------- */

float or_f16_decode(uint16_t h) {
  uint32_t s = (uint32_t)(h >> 15) << 31, e = (h >> 10) & 31u, m = h & 0x3ffu;
  if (e == 0) {
    if (m == 0) return u2f(s);
    /* subnormal: value = m * 2^-24, exact in f32 */
    int sh = 0;
    while (!(m & 0x400u)) { m <<= 1; ++sh; }
    return u2f(s | ((uint32_t)(113 - sh) << 23) | ((m & 0x3ffu) << 13));
  }
  if (e == 31) return u2f(s | 0x7f800000u | (m << 13));
  return u2f(s | ((e + 112u) << 23) | (m << 13));
}

uint16_t or_f16_encode(float f) {
  uint32_t x = f2u(f), s = (x >> 16) & 0x8000u, e = (x >> 23) & 0xffu, m = x & 0x7fffffu;
  if (e == 0xff) return (uint16_t)(s | (m ? 0x7e00u : 0x7c00u));
  if (e == 0 && m == 0) return (uint16_t)s;
  int te = (int)e - 112; /* biased half exponent */
  if (te >= 31) return (uint16_t)(s | 0x7c00u);
  if (te <= 0) {
    if (te < -10) return (uint16_t)s;
    uint32_t full = m | 0x800000u;
    int sh = 14 - te;
    uint32_t q = full >> sh, r = full & ((1u << sh) - 1u), h = 1u << (sh - 1);
    if (r > h || (r == h && (q & 1u))) ++q;
    /* fp16.cpp:83 keeps only the low 10 bits, so a subnormal that rounds up
     * to 2^-14 (q == 0x400) encodes as signed zero, not 0x0400. */
    return (uint16_t)(s | (q & 0x3ffu));
  }
  uint32_t q = ((uint32_t)te << 10) | (m >> 13), r = m & 0x1fffu;
  if (r > 0x1000u || (r == 0x1000u && (q & 1u))) {
    ++q;
    if ((q >> 10) >= 31) return (uint16_t)(s | 0x7c00u);
  }
  return (uint16_t)(s | q);
}

/* ---- bf16 <-> f32: fp16.cpp:95-112 ------------------------------------- */

float or_bf16_decode(uint16_t b) { return u2f((uint32_t)b << 16); }

uint16_t or_bf16_encode(float f) {
  uint32_t x = f2u(f);
  if ((x & 0x7f800000u) == 0x7f800000u && (x & 0x7fffffu)) return 0x7fc0u;
  if ((x & 0x7f800000u) == 0x7f800000u) return (uint16_t)(x >> 16);
  return (uint16_t)((x + 0x7fffu + ((x >> 16) & 1u)) >> 16);
}

/* ---- OCP E4M3 <-> f32: fp8.cpp:42-71 (decode), :75-106 (encode) -------- */

float or_e4m3_decode(uint8_t c) {
  uint32_t s = (uint32_t)(c >> 7) << 31, e = (c >> 3) & 15u, m = c & 7u;
  if (e == 0) {
    if (m == 0) return u2f(s);
    int sh = 0;
    while (!(m & 8u)) { m <<= 1; ++sh; }
    return u2f(s | ((uint32_t)(121 - sh) << 23) | ((m & 7u) << 20));
  }
  if (e == 15 && m == 7) return u2f(s | 0x7fc00000u);
  return u2f(s | ((e + 120u) << 23) | (m << 20));
}

uint8_t or_e4m3_encode(float f) {
  uint32_t x = f2u(f), s = (x >> 24) & 0x80u, e = (x >> 23) & 0xffu, m = x & 0x7fffffu;
  if (e == 0xff) return (uint8_t)(s | (m ? 0x7fu : 0x7eu));
  if (e == 0 && m == 0) return (uint8_t)s;
  int te = (int)e - 120;
  if (te > 15) return (uint8_t)(s | 0x7eu);
  if (te <= 0) {
    if (te < -3) return 0; /* fp8.cpp:86: magnitude < 2^-10 -> +0, sign dropped */
    uint32_t full = m | 0x800000u;
    int sh = 21 - te;
    uint32_t q = full >> sh, r = full & ((1u << sh) - 1u), h = 1u << (sh - 1);
    if (r > h || (r == h && (q & 1u))) ++q;
    return (uint8_t)(s | q);
  }
  uint32_t q = ((uint32_t)te << 3) | (m >> 20), r = m & 0xfffffu;
  if (r > 0x80000u || (r == 0x80000u && (q & 1u))) ++q;
  if ((q >> 3) > 15 || q == 0x7fu) return (uint8_t)(s | 0x7eu); /* fp8.cpp:102-104 */
  return (uint8_t)(s | q);
}

void or_e4m3_encode_n(const float *x, size_t n, uint8_t *out) {
  for (size_t i = 0; i < n; ++i) out[i] = or_e4m3_encode(x[i]);
}
void or_e4m3_decode_n(const uint8_t *c, size_t n, float *out) {
  for (size_t i = 0; i < n; ++i) out[i] = or_e4m3_decode(c[i]);
}
void or_f16_encode_n(const float *x, size_t n, uint16_t *out) {
  for (size_t i = 0; i < n; ++i) out[i] = or_f16_encode(x[i]);
}
void or_f16_decode_n(const uint16_t *c, size_t n, float *out) {
  for (size_t i = 0; i < n; ++i) out[i] = or_f16_decode(c[i]);
}
void or_bf16_encode_n(const float *x, size_t n, uint16_t *out) {
  for (size_t i = 0; i < n; ++i) out[i] = or_bf16_encode(x[i]);
}

/* ---- int8 symmetric quantization: quant_int8.cpp:38-46, 54-90 ---------- */

static int8_t q_code(double v) {
  /* quant_int8.cpp:38-46: nearbyint then static_cast<int32_t>. On x86-64 an
   * out-of-range or NaN conversion yields INT32_MIN, which the clamp maps to
   * -127; restated explicitly so the result does not depend on the host. */
  double r = nearbyint(v);
  int32_t i = (r != r || r >= 2147483648.0 || r < -2147483648.0) ? INT32_MIN : (int32_t)r;
  return (int8_t)(i < -127 ? -127 : (i > 127 ? 127 : i));
}

static float row_scale(const float *x, size_t n) {
  double amax = 0.0; /* quant_int8.cpp:76-81 */
  for (size_t i = 0; i < n; ++i) {
    double a = fabs((double)x[i]);
    if (a > amax) amax = a;
  }
  return amax > 0.0 ? (float)(amax / 127.0) : 1.0f; /* :82 */
}

int or_quantize_i8_rows(const float *x, int rows, int cols, float *scales, int8_t *out) {
  if (!x || !scales || !out || rows <= 0 || cols <= 0) return 0;
  for (int r = 0; r < rows; ++r) {
    const float *row = x + (size_t)r * cols;
    float s = row_scale(row, (size_t)cols);
    double inv = 1.0 / (double)s; /* :84 */
    scales[r] = s;
    for (int c = 0; c < cols; ++c) out[(size_t)r * cols + c] = q_code((double)row[c] * inv);
  }
  return 1;
}

int or_quantize_i8_tensor(const float *x, int n, float *scale_out, int8_t *out) {
  if (!x || !scale_out || !out || n <= 0) return 0;
  float s = row_scale(x, (size_t)n); /* :57-62 */
  double inv = 1.0 / (double)s;
  *scale_out = s;
  for (int i = 0; i < n; ++i) out[i] = q_code((double)x[i] * inv);
  return 1;
}

/* Asymmetric per-group: quant_int8.cpp:94-142. */
static uint8_t clamp_u8(double v) {
  double r = nearbyint(v);
  int32_t i = (r != r || r >= 2147483648.0 || r < -2147483648.0) ? INT32_MIN : (int32_t)r;
  return (uint8_t)(i < 0 ? 0 : (i > 255 ? 255 : i));
}

int or_quantize_i8_group(const float *x, int rows, int cols, int groups, float *scales,
                         uint8_t *zeros, uint8_t *out) {
  if (!x || !scales || !zeros || !out || rows <= 0 || cols <= 0 || groups <= 0) return 0;
  if (cols % groups) return 0;
  int gsz = cols / groups;
  for (int r = 0; r < rows; ++r)
    for (int g = 0; g < groups; ++g) {
      const float *v = x + (size_t)r * cols + (size_t)g * gsz;
      double lo = v[0], hi = v[0]; /* :107-113 */
      for (int i = 1; i < gsz; ++i) {
        if ((double)v[i] < lo) lo = v[i];
        if ((double)v[i] > hi) hi = v[i];
      }
      float s;
      uint8_t z;
      if (lo >= 0.0) { /* :122-131 */
        z = 0;
        s = hi > 0.0 ? (float)(hi / 255.0) : 1.0f;
      } else if (hi <= 0.0) {
        z = 255;
        s = lo < 0.0 ? (float)(-lo / 255.0) : 1.0f;
      } else {
        s = (float)((hi - lo) / 255.0);
        z = clamp_u8(-lo / (double)s);
      }
      scales[r * groups + g] = s;
      zeros[r * groups + g] = z;
      double inv = 1.0 / (double)s; /* :134-138 */
      for (int i = 0; i < gsz; ++i) {
        double q = (double)v[i] * inv;
        q = q + (double)z;
        out[(size_t)r * cols + (size_t)g * gsz + i] = clamp_u8(q);
      }
    }
  return 1;
}

/* quant_int8.cpp:162-179 */
void or_dequantize_i8_group(const uint8_t *q, int rows, int cols, int groups,
                            const float *scales, const uint8_t *zeros, float *out) {
  int gsz = cols / groups;
  for (int r = 0; r < rows; ++r)
    for (int g = 0; g < groups; ++g) {
      float s = scales[r * groups + g];
      double z = zeros[r * groups + g];
      for (int i = 0; i < gsz; ++i) {
        size_t k = (size_t)r * cols + (size_t)g * gsz + i;
        out[k] = (float)(((double)q[k] - z) * (double)s);
      }
    }
}

void or_dequantize_i8_rows(const int8_t *q, int rows, int cols, const float *scales, float *out) {
  for (int r = 0; r < rows; ++r) /* quant_int8.cpp:151-160 */
    for (int c = 0; c < cols; ++c)
      out[(size_t)r * cols + c] = (float)q[(size_t)r * cols + c] * scales[r];
}

/* ---- exact int8 GEMM: quant_int8.cpp:189-211 -------------------------- */
/* b_nk = 0: B[K][N] (reference layout); b_nk = 1: B[N][K]. Computes only
 * the listed rows (row_ids == NULL: rows 0..nrows-1) so the full-size tests
 * can check sampled row blocks. acc_out[nrows][N] int32 (may be NULL),
 * c_out[nrows][N] f32 = ((float)acc * sa) * sb (may be NULL). */
void or_gemm_i8_rows(int N, int K, const int8_t *A, const int8_t *B, int b_nk,
                     const int *row_ids, int nrows, const float *scales_a, int a_rows,
                     const float *scales_b, int b_cols, int32_t *acc_out, float *c_out) {
  for (int i = 0; i < nrows; ++i) {
    int m = row_ids ? row_ids[i] : i;
    const int8_t *a = A + (size_t)m * K;
    for (int n = 0; n < N; ++n) {
      int32_t acc = 0;
      if (b_nk) {
        const int8_t *b = B + (size_t)n * K;
        for (int k = 0; k < K; ++k) acc += (int32_t)a[k] * (int32_t)b[k];
      } else {
        for (int k = 0; k < K; ++k) acc += (int32_t)a[k] * (int32_t)B[(size_t)k * N + n];
      }
      if (acc_out) acc_out[(size_t)i * N + n] = acc;
      if (c_out) {
        float sa = a_rows ? scales_a[m] : scales_a[0];
        float sb = b_cols ? scales_b[n] : scales_b[0];
        float v = (float)acc * sa; /* :208, left to right, no contraction */
        c_out[(size_t)i * N + n] = v * sb;
      }
    }
  }
}

/* ---- float GEMM used under the f16 / bf16 / e4m3 entries ---------------
 * fp16.cpp:123-141 and fp8.cpp:116-124 decode to f32 and call
 * rouge_gemm_f32 (gemm.cpp:291), C = A*B with f32 accumulation. The oracle
 * accumulates in double: the GPU result is compared under the relative-L2
 * tolerance stated in the tests, against this and against the reference's
 * own f32 result. a[M][K] and b (b_nk ? [N][K] : [K][N]) are f32. */
void or_gemm_f32_rows(int N, int K, const float *A, const float *B, int b_nk,
                      const int *row_ids, int nrows, float *C) {
  for (int i = 0; i < nrows; ++i) {
    int m = row_ids ? row_ids[i] : i;
    const float *a = A + (size_t)m * K;
    for (int n = 0; n < N; ++n) {
      double s = 0.0;
      if (b_nk) {
        const float *b = B + (size_t)n * K;
        for (int k = 0; k < K; ++k) s += (double)a[k] * (double)b[k];
      } else {
        for (int k = 0; k < K; ++k) s += (double)a[k] * (double)B[(size_t)k * N + n];
      }
      C[(size_t)i * N + n] = (float)s;
    }
  }
}

/* ---- per-tensor E4M3 scaling: tests/test_ai.cpp:219-231 convention ----- */

float or_absmax(const float *x, size_t n) {
  float m = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    float a = fabsf(x[i]);
    if (a > m) m = a;
  }
  return m;
}

/* s = amax / 448.0f (1.0f when amax == 0); out[i] = e4m3(x[i] / s). */
float or_quantize_e4m3_scaled(const float *x, size_t n, float amax, uint8_t *out) {
  float s = amax > 0.0f ? amax / 448.0f : 1.0f;
  for (size_t i = 0; i < n; ++i) out[i] = or_e4m3_encode(x[i] / s);
  return s;
}

/* ---- direct convolution, NHWC, double accumulation ---------------------
 * The reference computes NCHW f32 conv by im2col + GEMM (conv.cpp:26-66,
 * OH = (H + 2p - KH)/s + 1, zero padding, bias added after the GEMM). The
 * oracle is the direct sum in NHWC with weights [Cout][KH][KW][Cin];
 * x and w are f32 (already decoded from f16). Computes output pixels
 * [p0, p1) of the flattened (n, oh, ow) index. */
void or_conv2d_nhwc(int N, int H, int W, int Cin, int Cout, int KH, int KW, int stride,
                    int pad, const float *x, const float *w, const float *bias,
                    long p0, long p1, float *y) {
  int OH = (H + 2 * pad - KH) / stride + 1, OW = (W + 2 * pad - KW) / stride + 1;
  (void)N;
  for (long p = p0; p < p1; ++p) {
    int ow = (int)(p % OW), oh = (int)((p / OW) % OH), n = (int)(p / ((long)OW * OH));
    for (int co = 0; co < Cout; ++co) {
      double s = 0.0;
      for (int kr = 0; kr < KH; ++kr) {
        int ih = oh * stride - pad + kr;
        if (ih < 0 || ih >= H) continue;
        for (int kc = 0; kc < KW; ++kc) {
          int iw = ow * stride - pad + kc;
          if (iw < 0 || iw >= W) continue;
          const float *xp = x + (((size_t)n * H + ih) * W + iw) * Cin;
          const float *wp = w + (((size_t)co * KH + kr) * KW + kc) * Cin;
          for (int c = 0; c < Cin; ++c) s += (double)xp[c] * (double)wp[c];
        }
      }
      y[(size_t)(p - p0) * Cout + co] = (float)(s + (bias ? (double)bias[co] : 0.0));
    }
  }
}

/* ---- narrow formats of narrow.cpp (e4m3 / e5m2 / e3m2 / e2m3 / e2m1) ----
 * narrow.cpp:46-65 (format table), :67-106 (decode), :108-144 (encode).
 * Codes are the format's field in the low bits of a byte. This is the
 * generic encoder the MX / NVFP4 quantizers use; it differs from fp8.cpp's
 * e4m3 encoder: a rounded result that lands on 0x7F (values in [464, 512))
 * is kept, i.e. encodes NaN, instead of saturating to 0x7E. */
typedef struct {
  int exp_bits, man_bits, bias;
  uint32_t max_bits, nan_bits;
  int width;
} or_narrow_fmt;

/* fmt: 0 e4m3, 1 e5m2, 2 e3m2, 3 e2m3, 4 e2m1 */
static const or_narrow_fmt OR_NARROW[5] = {
    {4, 3, 7, 0x7Eu, 0x7Fu, 8}, {5, 2, 15, 0x7Bu, 0x7Fu, 8}, {3, 2, 3, 0x1Fu, 0x00u, 6},
    {2, 3, 1, 0x1Fu, 0x00u, 6}, {2, 1, 1, 0x07u, 0x00u, 4}};

float or_narrow_decode(uint32_t bits, int fmt) {
  const or_narrow_fmt *F = &OR_NARROW[fmt];
  const uint32_t fsign = ((bits >> (F->width - 1)) & 1u) << 31;
  const uint32_t maxe = (1u << F->exp_bits) - 1u;
  const uint32_t e = (bits >> F->man_bits) & maxe, m = bits & ((1u << F->man_bits) - 1u);
  if (e == 0) {
    if (m == 0) return u2f(fsign);
    /* subnormal: m * 2^(1 - bias - man_bits), normalised */
    uint32_t mm = m;
    int sh = 0;
    while (!(mm & (1u << F->man_bits))) { mm <<= 1; ++sh; }
    mm &= (1u << F->man_bits) - 1u;
    return u2f(fsign | ((uint32_t)(128 - F->bias - sh) << 23) | (mm << (23 - F->man_bits)));
  }
  if (e == maxe && F->nan_bits) {
    /* a format whose all-ones exponent is not a normal binade (e5m2) has
     * Inf at mantissa 0 and NaN otherwise; e4m3 only NaN at mantissa all-ones */
    const int top_normal = ((F->max_bits >> F->man_bits) & maxe) == maxe;
    if (!top_normal) return u2f(fsign | (m ? 0x7fc00000u : 0x7f800000u));
    if (m == (1u << F->man_bits) - 1u) return u2f(fsign | 0x7fc00000u);
  }
  return u2f(fsign | ((uint32_t)((int)e - F->bias + 127) << 23) | (m << (23 - F->man_bits)));
}

uint32_t or_narrow_encode(float f, int fmt, int nan_to_max) {
  const or_narrow_fmt *F = &OR_NARROW[fmt];
  const uint32_t x = f2u(f), e = (x >> 23) & 0xffu, m = x & 0x7fffffu;
  const uint32_t sbit = ((x >> 31) & 1u) << (F->width - 1);
  const int M = F->man_bits;
  const uint32_t maxe = (1u << F->exp_bits) - 1u, field = (1u << F->width) - 1u;
  if (e == 0xffu && m) return nan_to_max ? F->max_bits : (sbit | F->nan_bits);
  if (e == 0xffu) return sbit | F->max_bits; /* Inf saturates */
  if (e == 0 && m == 0) return sbit;
  const int te = (int)e - 127 + F->bias;
  if (te > (int)maxe) return sbit | F->max_bits;
  if (te <= 0) {
    if (te < -M) return 0; /* narrow.cpp:128: too small -> +0, sign dropped */
    const uint32_t full = 0x800000u | m;
    const int sh = 1 - te + (23 - M);
    uint32_t q = full >> sh;
    const uint32_t r = full & ((1u << sh) - 1u), h = 1u << (sh - 1);
    if (r > h || (r == h && (q & 1u))) ++q;
    return sbit | (q & field);
  }
  uint32_t q = ((uint32_t)te << M) | (m >> (23 - M));
  const uint32_t r = m & ((1u << (23 - M)) - 1u), h = 1u << (22 - M);
  if (r > h || (r == h && (q & 1u))) {
    ++q;
    if ((q >> M) > maxe) return sbit | F->max_bits;
  }
  return sbit | (q & field);
}

void or_narrow_encode_n(const float *x, size_t n, int fmt, int nan_to_max, uint8_t *out) {
  for (size_t i = 0; i < n; ++i) out[i] = (uint8_t)or_narrow_encode(x[i], fmt, nan_to_max);
}
void or_narrow_decode_n(const uint8_t *c, size_t n, int fmt, float *out) {
  for (size_t i = 0; i < n; ++i) out[i] = or_narrow_decode(c[i], fmt);
}

/* ---- E8M0 block scales: narrow.cpp:146-163 ----------------------------- */

float or_e8m0_decode(uint8_t c) {
  if (c == 255) return u2f(0x7fc00000u);
  if (c == 0) return u2f(0x00400000u); /* 2^-127, subnormal */
  return u2f((uint32_t)c << 23);
}

/* frexp's exponent of a positive finite scale, clamped to [-126, 127] and
 * biased by 127. For a power of two 2^p frexp gives p + 1, so the code is
 * p + 128: the stored scale is twice the chosen one (the reference's
 * behaviour, kept). Non-positive or non-finite scales give 127 (1.0). */
uint8_t or_e8m0_encode(float s) {
  if (!(s > 0.0f) || !isfinite(s)) return 127;
  int e = 0;
  frexpf(s, &e);
  if (e < -126) e = -126;
  if (e > 127) e = 127;
  return (uint8_t)(e + 127);
}

/* smallest p >= 0 (at most 127) with amax <= emax * 2^p: narrow.cpp:213-216 */
static int or_block_pow(float amax, float emax) {
  int p = 0;
  while (amax > ldexpf(emax, p) && p < 127) ++p;
  return p;
}

/* MXFP8 / MXFP4: narrow.cpp:200-265. fmt 0 (e4m3), 1 (e5m2) or 4 (e2m1,
 * NaN -> +MAX); blocks of 32, the last one partial. Returns the block count. */
int or_mx_quantize(const float *x, int n, int fmt, uint8_t *out, uint8_t *scales) {
  const int nan_to_max = fmt == 4;
  const float emax = or_narrow_decode(OR_NARROW[fmt].max_bits, fmt);
  for (int base = 0; base < n; base += 32) {
    const int cnt = n - base < 32 ? n - base : 32;
    float amax = 0.0f;
    for (int i = 0; i < cnt; ++i) {
      const float a = fabsf(x[base + i]);
      if (a > amax) amax = a;
    }
    const float scale = amax > 0.0f ? ldexpf(1.0f, or_block_pow(amax, emax)) : 1.0f;
    const uint8_t sc = or_e8m0_encode(scale);
    scales[base / 32] = sc;
    const float inv = 1.0f / or_e8m0_decode(sc);
    for (int i = 0; i < cnt; ++i) {
      const uint32_t q = or_narrow_encode(x[base + i] * inv, fmt, nan_to_max);
      out[base + i] = (uint8_t)(fmt == 4 ? (q & 0x0Fu) : q);
    }
  }
  return (n + 31) / 32;
}

/* NVFP4: narrow.cpp:270-300. Blocks of 16 e2m1 codes; block scale 2^p coded
 * in e4m3 by the generic encoder (2^9 and above saturate to 448); amax over
 * |x| * gs, elements x * (1 / (scale * gs)); gs <= 0 (or NaN) becomes 1. */
int or_nvfp4_quantize(const float *x, int n, float gs, uint8_t *out, uint8_t *scales) {
  if (!(gs > 0.0f)) gs = 1.0f;
  const float emax = or_narrow_decode(OR_NARROW[0].max_bits, 0);
  for (int base = 0; base < n; base += 16) {
    const int cnt = n - base < 16 ? n - base : 16;
    float amax = 0.0f;
    for (int i = 0; i < cnt; ++i) {
      const float a = fabsf(x[base + i]) * gs;
      if (a > amax) amax = a;
    }
    const float bs = amax > 0.0f ? ldexpf(1.0f, or_block_pow(amax, emax)) : 1.0f;
    const uint8_t sc = (uint8_t)or_narrow_encode(bs, 0, 0);
    scales[base / 16] = sc;
    const float inv = 1.0f / (or_narrow_decode(sc, 0) * gs);
    for (int i = 0; i < cnt; ++i)
      out[base + i] = (uint8_t)(or_narrow_encode(x[base + i] * inv, 4, 1) & 0x0Fu);
  }
  return (n + 15) / 16;
}

/* narrow.cpp:304-331: element decode times the block's E8M0 scale. */
void or_mx_dequantize(const uint8_t *in, const uint8_t *scales, int n, int fmt, float *out) {
  for (int i = 0; i < n; ++i) {
    const uint32_t c = fmt == 4 ? (in[i] & 0x0Fu) : in[i];
    out[i] = or_narrow_decode(c, fmt) * or_e8m0_decode(scales[i / 32]);
  }
}
