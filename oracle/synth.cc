// synth.cc -- TEST INFRASTRUCTURE ONLY. The seeded synthetic inputs of the
// five configurations, generated on the host for the oracle side: the bench's
// reference arm and CPU baseline draw their inputs here, so they never load
// the product library. tests/test_seeds.py checks that these arrays equal the
// product generator's (libstade_b200 stade_fill_*) bit for bit.
//
// The scheme (stated, not shared code): seed = FNV-1a 64 of "<kernel>:<array>"
// (val_stable_seed, src/STADE.jl:16619-16626). An array is cut into chunks of
// 2^20 elements; chunk c draws from xoshiro256** (Blackman & Vigna 2018)
// seeded by four splitmix64 outputs of seed + c * 0x9E3779B97F4A7C15. A
// uniform is the top 53 bits times 2^-53; a normal is the Box-Muller cosine
// branch of val_normal (src/STADE.jl:16628-16638), u1 = 1 - U, u2 = U,
// sqrt(-2 log u1) cos(2 pi u2); a one-hot row takes class floor(U * n_o).
#include <cmath>
#include <cstdint>

namespace {

constexpr int64_t kSpan = int64_t(1) << 20;   // elements (or rows) per generator
constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;

class Stream {
 public:
  explicit Stream(uint64_t seed) {
    uint64_t x = seed;
    for (int i = 0; i < 4; ++i) {
      x += kGolden;
      uint64_t z = x;
      z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
      z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
      st_[i] = z ^ (z >> 31);
    }
  }
  double uniform() { return double(bits() >> 11) * 0x1.0p-53; }
  double normal() {
    const double u1 = 1.0 - uniform();
    const double u2 = uniform();
    return std::sqrt(-2.0 * std::log(u1)) * std::cos(2.0 * M_PI * u2);
  }

 private:
  static uint64_t rot(uint64_t v, int k) { return (v << k) | (v >> (64 - k)); }
  uint64_t bits() {
    const uint64_t out = rot(st_[1] * 5, 7) * 9;
    const uint64_t sh = st_[1] << 17;
    st_[2] ^= st_[0];
    st_[3] ^= st_[1];
    st_[1] ^= st_[2];
    st_[0] ^= st_[3];
    st_[2] ^= sh;
    st_[3] = rot(st_[3], 45);
    return out;
  }
  uint64_t st_[4];
};

// Calls body(stream, lo, hi) for each span of n items, spans in parallel.
template <class Body>
void spans(int64_t n, uint64_t seed, Body body) {
  if (n <= 0) return;
  const int64_t count = (n + kSpan - 1) / kSpan;
#pragma omp parallel for schedule(static) if (count > 1)
  for (int64_t c = 0; c < count; ++c) {
    Stream g(seed + uint64_t(c) * kGolden);
    const int64_t lo = c * kSpan;
    body(g, lo, lo + kSpan < n ? lo + kSpan : n);
  }
}

}  // namespace

extern "C" {

uint64_t oracle_fnv1a64(const char* s) {
  uint64_t h = 0xcbf29ce484222325ull;
  for (; *s; ++s) h = (h ^ uint64_t((unsigned char)*s)) * 0x00000100000001b3ull;
  return h;
}

void oracle_fill_normal_f64(double* out, int64_t n, uint64_t seed, double mean, double sd) {
  spans(n, seed, [=](Stream& g, int64_t lo, int64_t hi) {
    for (int64_t i = lo; i < hi; ++i) out[i] = mean + sd * g.normal();
  });
}
void oracle_fill_normal_f32(float* out, int64_t n, uint64_t seed, double mean, double sd) {
  spans(n, seed, [=](Stream& g, int64_t lo, int64_t hi) {
    for (int64_t i = lo; i < hi; ++i) out[i] = float(mean + sd * g.normal());
  });
}
void oracle_fill_uniform_f64(double* out, int64_t n, uint64_t seed, double a, double b) {
  spans(n, seed, [=](Stream& g, int64_t lo, int64_t hi) {
    for (int64_t i = lo; i < hi; ++i) out[i] = a + (b - a) * g.uniform();
  });
}
void oracle_fill_uniform_f32(float* out, int64_t n, uint64_t seed, double a, double b) {
  spans(n, seed, [=](Stream& g, int64_t lo, int64_t hi) {
    for (int64_t i = lo; i < hi; ++i) out[i] = float(a + (b - a) * g.uniform());
  });
}
void oracle_fill_onehot_f64(double* out, int64_t rows, int64_t n_o, uint64_t seed) {
  if (n_o <= 0) return;
  spans(rows, seed, [=](Stream& g, int64_t lo, int64_t hi) {
    for (int64_t r = lo; r < hi; ++r) {
      int64_t cls = int64_t(g.uniform() * double(n_o));
      cls = cls < n_o ? cls : n_o - 1;
      for (int64_t j = 0; j < n_o; ++j) out[r * n_o + j] = j == cls ? 1.0 : 0.0;
    }
  });
}
void oracle_fill_onehot_f32(float* out, int64_t rows, int64_t n_o, uint64_t seed) {
  if (n_o <= 0) return;
  spans(rows, seed, [=](Stream& g, int64_t lo, int64_t hi) {
    for (int64_t r = lo; r < hi; ++r) {
      int64_t cls = int64_t(g.uniform() * double(n_o));
      cls = cls < n_o ? cls : n_o - 1;
      for (int64_t j = 0; j < n_o; ++j) out[r * n_o + j] = j == cls ? 1.0f : 0.0f;
    }
  });
}

}  // extern "C"
