// Seeded synthetic inputs for benchmarks and tests (host code).
//
// The generator is counter-based splitmix64: element i of the stream for
// `seed` is mix(seed + (i + 1) * 0x9E3779B97F4A7C15), the i-th output of a
// splitmix64 generator started at `seed`. Because every element depends
// only on (seed, i), the fill is split across host threads with identical
// results for any thread count. Uniforms take the top 24 bits; normals use
// the Box-Muller transform on consecutive pairs, computed in double. This
// is the same generator family as the reference's rouge_rng_*
// (splitmix64 + Box-Muller, sparse_random.cpp:47-91); it does not reproduce
// that function's exact stream.
#include <atomic>
#include <cmath>
#include <cstddef>
#include <cstdint>
#include <thread>
#include <vector>

namespace {

constexpr uint64_t kGamma = 0x9E3779B97F4A7C15ull;
constexpr double kTwoPi = 6.283185307179586476925286766559;

inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

inline uint64_t draw(uint64_t seed, uint64_t i) { return mix64(seed + (i + 1) * kGamma); }

inline double unit(uint64_t v) { return static_cast<double>(v >> 40) * (1.0 / 16777216.0); }

template <class F>
void parallel_ranges(size_t n, F f) {
  unsigned hw = std::thread::hardware_concurrency();
  size_t threads = hw ? hw : 1;
  if (n < (1u << 16)) threads = 1;
  std::vector<std::thread> pool;
  for (size_t t = 1; t < threads; ++t)
    pool.emplace_back(f, n * t / threads, n * (t + 1) / threads);
  f(size_t(0), n / threads);
  for (auto &th : pool) th.join();
}

}  // namespace

extern "C" {

/* out[i] = lo + (hi - lo) * u_i, u_i uniform in [0, 1) (24-bit grid). */
int rouge_b200_synth_uniform(uint64_t seed, size_t n, float lo, float hi, float *out) {
  if (!out) return -1;
  parallel_ranges(n, [=](size_t a, size_t b) {
    const double span = static_cast<double>(hi) - static_cast<double>(lo);
    for (size_t i = a; i < b; ++i)
      out[i] = static_cast<float>(static_cast<double>(lo) + span * unit(draw(seed, i)));
  });
  return 0;
}

/* Elements [offset, offset + n) of the N(mean, std^2) stream for `seed`
 * into out[0..n): Box-Muller on draws (2j, 2j+1) gives elements 2j (cosine
 * branch) and 2j+1 (sine branch). offset must be even. */
int rouge_b200_synth_normal_at(uint64_t seed, size_t offset, size_t n, float mean, float stddev,
                               float *out) {
  if (!out || (offset & 1)) return -1;
  const size_t pairs = (n + 1) / 2, p0 = offset / 2;
  parallel_ranges(pairs, [=](size_t a, size_t b) {
    for (size_t j = a; j < b; ++j) {
      const size_t g = p0 + j;
      const double u1 = (static_cast<double>(draw(seed, 2 * g) >> 40) + 1.0) * (1.0 / 16777216.0);
      const double u2 = unit(draw(seed, 2 * g + 1));
      const double r = std::sqrt(-2.0 * std::log(u1));
      const double t = kTwoPi * u2;
      out[2 * j] = static_cast<float>(mean + stddev * r * std::cos(t));
      if (2 * j + 1 < n) out[2 * j + 1] = static_cast<float>(mean + stddev * r * std::sin(t));
    }
  });
  return 0;
}

int rouge_b200_synth_normal(uint64_t seed, size_t n, float mean, float stddev, float *out) {
  return rouge_b200_synth_normal_at(seed, 0, n, mean, stddev, out);
}

/* Multiplies x[i] (element offset + i of the stream) by `mult` where an
 * independent uniform draw (stream seed ^ 0xD1B54A32D192ED03) is below
 * `frac`: the "1% of entries x20 outliers" of the W8A8 activation
 * workload. Returns the count. */
long long rouge_b200_synth_outliers_at(uint64_t seed, size_t offset, size_t n, float frac,
                                       float mult, float *x) {
  if (!x) return -1;
  const uint64_t s2 = seed ^ 0xD1B54A32D192ED03ull;
  std::atomic<long long> total{0};
  parallel_ranges(n, [&](size_t a, size_t b) {
    long long c = 0;
    for (size_t i = a; i < b; ++i)
      if (unit(draw(s2, offset + i)) < static_cast<double>(frac)) {
        x[i] *= mult;
        ++c;
      }
    total += c;
  });
  return total.load();
}

long long rouge_b200_synth_outliers(uint64_t seed, size_t n, float frac, float mult, float *x) {
  return rouge_b200_synth_outliers_at(seed, 0, n, frac, mult, x);
}

}  // extern "C"
