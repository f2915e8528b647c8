// Synthetic, seeded inputs for the five benchmark configurations.
//
// Seeds follow the scheme of `val_stable_seed` (src/STADE.jl:16619-16626):
// FNV-1a 64 over the UTF-8 bytes of a name. The uniform stream is our own
// documented generator (xoshiro256**, Blackman & Vigna 2018), because Julia's
// Xoshiro seeding code is not part of the reference. To fill large arrays with
// several host threads, an array is cut into chunks of 2^20 elements and chunk
// c runs its own xoshiro256** whose state comes from splitmix64 applied to
// seed + c * 0x9E3779B97F4A7C15. Normals use the Box-Muller cosine branch of
// `val_normal` (src/STADE.jl:16628-16638): u1 = 1 - U, u2 = U,
// sqrt(-2 log u1) cos(2 pi u2), two uniform draws per normal.
#include <cmath>
#include <cstdint>
#include <cstring>

#include "stade_b200.h"

namespace {

constexpr int64_t kChunk = int64_t(1) << 20;

inline uint64_t splitmix64(uint64_t& x) {
  uint64_t z = (x += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

inline uint64_t rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

struct Xoshiro256ss {
  uint64_t s[4];
  explicit Xoshiro256ss(uint64_t seed) {
    uint64_t x = seed;
    for (auto& v : s) v = splitmix64(x);
  }
  uint64_t next() {
    const uint64_t result = rotl(s[1] * 5, 7) * 9;
    const uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl(s[3], 45);
    return result;
  }
  // uniform in [0, 1) with 53 random bits
  double uniform() { return double(next() >> 11) * 0x1.0p-53; }
  double normal() {
    const double u1 = 1.0 - uniform();
    const double u2 = uniform();
    return std::sqrt(-2.0 * std::log(u1)) * std::cos(2.0 * M_PI * u2);
  }
};

inline uint64_t chunk_seed(uint64_t seed, int64_t c) {
  return seed + uint64_t(c) * 0x9E3779B97F4A7C15ull;
}

template <class T, class F>
void fill_chunked(T* out, int64_t n, uint64_t seed, F draw) {
  if (n <= 0) return;
  const int64_t nchunks = (n + kChunk - 1) / kChunk;
#pragma omp parallel for schedule(static) if (nchunks > 1)
  for (int64_t c = 0; c < nchunks; ++c) {
    Xoshiro256ss g(chunk_seed(seed, c));
    const int64_t lo = c * kChunk;
    const int64_t hi = (lo + kChunk < n) ? lo + kChunk : n;
    for (int64_t i = lo; i < hi; ++i) out[i] = T(draw(g));
  }
}

template <class T>
void fill_onehot(T* out, int64_t n_rows, int64_t n_o, uint64_t seed) {
  if (n_rows <= 0 || n_o <= 0) return;
  const int64_t nchunks = (n_rows + kChunk - 1) / kChunk;
#pragma omp parallel for schedule(static) if (nchunks > 1)
  for (int64_t c = 0; c < nchunks; ++c) {
    Xoshiro256ss g(chunk_seed(seed, c));
    const int64_t lo = c * kChunk;
    const int64_t hi = (lo + kChunk < n_rows) ? lo + kChunk : n_rows;
    for (int64_t r = lo; r < hi; ++r) {
      int64_t cls = int64_t(g.uniform() * double(n_o));
      if (cls >= n_o) cls = n_o - 1;
      for (int64_t j = 0; j < n_o; ++j) out[r * n_o + j] = T(j == cls ? 1.0 : 0.0);
    }
  }
}

}  // namespace

extern "C" {

uint64_t stade_fnv1a64(const char* s) {
  uint64_t h = 0xcbf29ce484222325ull;
  for (const unsigned char* p = reinterpret_cast<const unsigned char*>(s); *p; ++p) {
    h ^= uint64_t(*p);
    h *= 0x00000100000001b3ull;
  }
  return h;
}

void stade_fill_normal_f64(double* out, int64_t n, uint64_t seed, double mean, double std) {
  fill_chunked(out, n, seed, [=](Xoshiro256ss& g) { return mean + std * g.normal(); });
}
void stade_fill_normal_f32(float* out, int64_t n, uint64_t seed, double mean, double std) {
  fill_chunked(out, n, seed, [=](Xoshiro256ss& g) { return mean + std * g.normal(); });
}
void stade_fill_uniform_f64(double* out, int64_t n, uint64_t seed, double lo, double hi) {
  fill_chunked(out, n, seed, [=](Xoshiro256ss& g) { return lo + (hi - lo) * g.uniform(); });
}
void stade_fill_uniform_f32(float* out, int64_t n, uint64_t seed, double lo, double hi) {
  fill_chunked(out, n, seed, [=](Xoshiro256ss& g) { return lo + (hi - lo) * g.uniform(); });
}
void stade_fill_onehot_f32(float* out, int64_t n_rows, int64_t n_o, uint64_t seed) {
  fill_onehot(out, n_rows, n_o, seed);
}
void stade_fill_onehot_f64(double* out, int64_t n_rows, int64_t n_o, uint64_t seed) {
  fill_onehot(out, n_rows, n_o, seed);
}

}  // extern "C"
