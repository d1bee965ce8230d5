/*
 * TEST INFRASTRUCTURE ONLY -- thin driver around the reference library.
 *
 * Linked together with the reference's own sources (compiled by
 * oracle/Makefile from software/rouge-numerics/src into oracle/_ref/) so the
 * tests and bench.py's reference arm can call the unmodified reference
 * functions. It adds two things the reference does not have:
 *   - an int32-returning restatement of the exact loop at
 *     quant_int8.cpp:196-203 (rouge_gemm_i8 only returns floats, which are
 *     inexact for |acc| > 2^24);
 *   - a row-sliced std::thread driver. Row slices of rouge_gemm_i8 and of
 *     rouge_quantize_i8_channel are bit-identical to the single-threaded
 *     call, because every output row depends only on its own input row.
 */
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

extern "C" {
int rouge_quantize_i8_channel(const float *x, int rows, int cols, float *scales, int8_t *out);
void rouge_gemm_i8(int M, int N, int K, const int8_t *A, const int8_t *B,
                   const float *scales_a, int a_rows, const float *scales_b, int b_cols,
                   float *C);
uint8_t rouge_quantize_e5m2(float f);
float rouge_dequantize_e5m2(uint8_t u);
uint8_t rouge_quantize_e3m2(float f);
float rouge_dequantize_e3m2(uint8_t u);
uint8_t rouge_quantize_e2m3(float f);
float rouge_dequantize_e2m3(uint8_t u);
uint8_t rouge_quantize_e2m1(float f);
float rouge_dequantize_e2m1(uint8_t u);
}

namespace {

template <class F>
void for_row_slices(int rows, int threads, F f) {
  if (threads < 1) threads = 1;
  if (threads > rows) threads = rows;
  std::vector<std::thread> pool;
  for (int t = 1; t < threads; ++t) {
    int r0 = (int)((long long)rows * t / threads), r1 = (int)((long long)rows * (t + 1) / threads);
    pool.emplace_back([=] { f(r0, r1); });
  }
  f(0, (int)((long long)rows / threads));
  for (auto &th : pool) th.join();
}

}  // namespace

extern "C" {

int ref_hw_threads(void) {
  unsigned n = std::thread::hardware_concurrency();
  return n ? (int)n : 1;
}

/* rouge_quantize_i8_channel over row slices on `threads` threads. */
int ref_quantize_i8_channel_mt(const float *x, int rows, int cols, float *scales, int8_t *out,
                               int threads) {
  if (!x || !scales || !out || rows <= 0 || cols <= 0) return 0;
  for_row_slices(rows, threads, [&](int r0, int r1) {
    if (r1 > r0)
      rouge_quantize_i8_channel(x + (size_t)r0 * cols, r1 - r0, cols, scales + r0,
                                out + (size_t)r0 * cols);
  });
  return 1;
}

/* rouge_gemm_i8 over row slices of A/C on `threads` threads. */
void ref_gemm_i8_mt(int M, int N, int K, const int8_t *A, const int8_t *B, const float *scales_a,
                    int a_rows, const float *scales_b, int b_cols, float *C, int threads) {
  for_row_slices(M, threads, [&](int r0, int r1) {
    if (r1 <= r0) return;
    rouge_gemm_i8(r1 - r0, N, K, A + (size_t)r0 * K, B, a_rows ? scales_a + r0 : scales_a,
                  a_rows, scales_b, b_cols, C + (size_t)r0 * N);
  });
}

/* The reference's scalar converters applied to arrays, for bulk
 * comparisons (fp8.cpp:112, fp16.cpp:118-120). */
uint8_t rouge_quantize_e4m3(float f);
uint16_t rouge_quantize_f16(float f);
uint16_t rouge_quantize_bf16(float f);
void ref_e4m3_encode_n(const float *x, size_t n, uint8_t *out) {
  for (size_t i = 0; i < n; ++i) out[i] = rouge_quantize_e4m3(x[i]);
}
void ref_f16_encode_n(const float *x, size_t n, uint16_t *out) {
  for (size_t i = 0; i < n; ++i) out[i] = rouge_quantize_f16(x[i]);
}
void ref_bf16_encode_n(const float *x, size_t n, uint16_t *out) {
  for (size_t i = 0; i < n; ++i) out[i] = rouge_quantize_bf16(x[i]);
}
float rouge_dequantize_e4m3(uint8_t u);
float rouge_dequantize_f16(uint16_t u);
/* Decoders write through memory, so signalling-NaN payloads survive (a
 * round trip through a double, as a scripting-language call does, would
 * quiet them). */
void ref_e4m3_decode_n(const uint8_t *c, size_t n, float *out) {
  for (size_t i = 0; i < n; ++i) out[i] = rouge_dequantize_e4m3(c[i]);
}
void ref_f16_decode_n(const uint16_t *c, size_t n, float *out) {
  for (size_t i = 0; i < n; ++i) out[i] = rouge_dequantize_f16(c[i]);
}

/* Bulk forms of the narrow-format codecs (numerics.h:257-264);
 * fmt 1 e5m2, 2 e3m2, 3 e2m3, 4 e2m1. */
void ref_narrow_encode_n(const float *x, size_t n, int fmt, uint8_t *out) {
  uint8_t (*enc)(float) = fmt == 1 ? rouge_quantize_e5m2 : fmt == 2 ? rouge_quantize_e3m2
                        : fmt == 3 ? rouge_quantize_e2m3 : rouge_quantize_e2m1;
  for (size_t i = 0; i < n; ++i) out[i] = enc(x[i]);
}
void ref_narrow_decode_n(const uint8_t *c, size_t n, int fmt, float *out) {
  float (*dec)(uint8_t) = fmt == 1 ? rouge_dequantize_e5m2 : fmt == 2 ? rouge_dequantize_e3m2
                        : fmt == 3 ? rouge_dequantize_e2m3 : rouge_dequantize_e2m1;
  for (size_t i = 0; i < n; ++i) out[i] = dec(c[i]);
}

/* Exact int32 accumulators of rows [r0, r1) of A[M][K] x B[K][N]: the loop
 * of quant_int8.cpp:196-203 returning its int32 row accumulator. */
void ref_gemm_i8_acc_rows(int N, int K, const int8_t *A, const int8_t *B, int r0, int r1,
                          int32_t *acc_out) {
  for (int m = r0; m < r1; ++m) {
    int32_t *acc = acc_out + (size_t)(m - r0) * N;
    std::memset(acc, 0, sizeof(int32_t) * (size_t)N);
    const int8_t *arow = A + (size_t)m * K;
    for (int k = 0; k < K; ++k) {
      const int32_t av = arow[k];
      if (av == 0) continue;
      const int8_t *brow = B + (size_t)k * N;
      for (int n = 0; n < N; ++n) acc[n] += av * (int32_t)brow[n];
    }
  }
}

}  // extern "C"
