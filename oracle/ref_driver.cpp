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
#include <atomic>
#include <cmath>
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

/* Seeded benchmark inputs, generated here so that the reference arm of the
 * benchmark never loads the library under test. Counter-based splitmix64
 * (element i of stream `seed` = mix(seed + (i+1) * golden gamma)), uniforms
 * from the top 24 bits, normals by Box-Muller on consecutive pairs in
 * double, outliers by an independent uniform stream (seed ^ a fixed
 * constant): the generator the benchmark's own arm uses, so both arms see
 * the same bits (checked by a CPU test). Any thread count gives the same
 * values, so the fill runs on all hardware threads. */
}  // extern "C"

namespace {
constexpr uint64_t kGamma = 0x9E3779B97F4A7C15ull;
inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
inline uint64_t draw(uint64_t seed, uint64_t i) { return mix64(seed + (i + 1) * kGamma); }
inline double unit24(uint64_t v) { return static_cast<double>(v >> 40) * (1.0 / 16777216.0); }
template <class F>
void fill_ranges(size_t n, F f) {
  unsigned hw = std::thread::hardware_concurrency();
  size_t threads = (n < (1u << 16) || !hw) ? 1 : hw;
  std::vector<std::thread> pool;
  for (size_t t = 1; t < threads; ++t) pool.emplace_back(f, n * t / threads, n * (t + 1) / threads);
  f(size_t(0), n / threads);
  for (auto &th : pool) th.join();
}
}  // namespace

extern "C" {

int ref_synth_uniform(uint64_t seed, size_t n, float lo, float hi, float *out) {
  if (!out) return -1;
  fill_ranges(n, [=](size_t a, size_t b) {
    const double span = static_cast<double>(hi) - static_cast<double>(lo);
    for (size_t i = a; i < b; ++i)
      out[i] = static_cast<float>(static_cast<double>(lo) + span * unit24(draw(seed, i)));
  });
  return 0;
}

int ref_synth_normal_at(uint64_t seed, size_t offset, size_t n, float mean, float stddev,
                        float *out) {
  if (!out || (offset & 1)) return -1;
  const size_t pairs = (n + 1) / 2, p0 = offset / 2;
  fill_ranges(pairs, [=](size_t a, size_t b) {
    for (size_t j = a; j < b; ++j) {
      const size_t g = p0 + j;
      const double u1 = (static_cast<double>(draw(seed, 2 * g) >> 40) + 1.0) * (1.0 / 16777216.0);
      const double u2 = unit24(draw(seed, 2 * g + 1));
      const double r = std::sqrt(-2.0 * std::log(u1));
      const double t = 6.283185307179586476925286766559 * u2;
      out[2 * j] = static_cast<float>(mean + stddev * r * std::cos(t));
      if (2 * j + 1 < n) out[2 * j + 1] = static_cast<float>(mean + stddev * r * std::sin(t));
    }
  });
  return 0;
}

long long ref_synth_outliers_at(uint64_t seed, size_t offset, size_t n, float frac, float mult,
                                float *x) {
  if (!x) return -1;
  const uint64_t s2 = seed ^ 0xD1B54A32D192ED03ull;
  std::atomic<long long> total{0};
  fill_ranges(n, [&](size_t a, size_t b) {
    long long c = 0;
    for (size_t i = a; i < b; ++i)
      if (unit24(draw(s2, offset + i)) < static_cast<double>(frac)) {
        x[i] *= mult;
        ++c;
      }
    total += c;
  });
  return total.load();
}

/* rouge_quantize_bf16 (fp16.cpp:118-121) over n values on `threads`
 * threads: the bf16 output step of the sharded config. */
void ref_bf16_encode_mt(const float *x, size_t n, uint16_t *out, int threads) {
  const int rows = threads < 1 ? 1 : threads;
  for_row_slices(rows, threads, [&](int r0, int r1) {
    const size_t a = n * r0 / rows, b = n * r1 / rows;
    for (size_t i = a; i < b; ++i) out[i] = rouge_quantize_bf16(x[i]);
  });
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
