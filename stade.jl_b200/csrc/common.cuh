// Shared infrastructure of libstade_b200: status codes, the thread-local
// error text, the launch counter, stream and workspace handling, and the
// deterministic (fixed-order) reduction helpers every kernel uses instead of
// floating-point atomics.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "stade_b200.h"

namespace stade {

// ---- errors -------------------------------------------------------------
void set_error(const char* fmt, ...);
stade_status fail(stade_status code, const char* fmt, ...);
stade_status cuda_fail(cudaError_t e, const char* what, const char* file, int line);

#define STADE_CUDA(call)                                                   \
  do {                                                                     \
    cudaError_t e__ = (call);                                              \
    if (e__ != cudaSuccess) return ::stade::cuda_fail(e__, #call, __FILE__, __LINE__); \
  } while (0)

#define STADE_CHECK_LAUNCH()                                               \
  do {                                                                     \
    ::stade::count_launch();                                               \
    cudaError_t e__ = cudaGetLastError();                                  \
    if (e__ != cudaSuccess) return ::stade::cuda_fail(e__, "kernel launch", __FILE__, __LINE__); \
  } while (0)

#define STADE_REQUIRE(cond, ...)                                           \
  do {                                                                     \
    if (!(cond)) return ::stade::fail(STADE_EINVAL, __VA_ARGS__);          \
  } while (0)

void count_launch();

// ---- phase profiler ---------------------------------------------------------
// When enabled (stade_profile_enable), entry points bracket each phase (one
// or a few kernels) with CUDA events on their stream; stade_profile_read sums
// the elapsed device time per phase name. Off by default: then a PhaseScope
// costs one branch.
bool profile_on();
void phase_begin(const char* name, cudaStream_t s);
void phase_end(cudaStream_t s);
struct PhaseScope {
  bool on;
  cudaStream_t s;
  PhaseScope(const char* name, cudaStream_t st) : on(profile_on()), s(st) {
    if (on) phase_begin(name, s);
  }
  void end() {
    if (on) phase_end(s);
    on = false;
  }
  ~PhaseScope() { end(); }
};

// ---- options --------------------------------------------------------------
inline cudaStream_t stream_of(const stade_opts* o) {
  return o ? static_cast<cudaStream_t>(o->stream) : static_cast<cudaStream_t>(0);
}
inline uint32_t flags_of(const stade_opts* o) { return o ? o->flags : 0u; }

// Workspace: the caller's buffer when given (and large enough), else a
// per-device cached buffer grown on first use. Returns STADE_OK and sets *p.
stade_status get_workspace(const stade_opts* o, size_t bytes, void** p);

inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Carves aligned sub-buffers out of one workspace.
struct Carver {
  char* base;
  size_t off = 0;
  explicit Carver(void* b) : base(static_cast<char*>(b)) {}
  template <class T> T* take(size_t count) {
    off = align_up(off, 256);
    T* p = reinterpret_cast<T*>(base + off);
    off += count * sizeof(T);
    return p;
  }
};
// Size-only twin of Carver, for the *_workspace queries.
struct Sizer {
  size_t off = 0;
  template <class T> void take(size_t count) {
    off = align_up(off, 256);
    off += count * sizeof(T);
  }
  size_t bytes() const { return align_up(off, 256); }
};

// Scalar in/out parameters (a scalar argument's adjoint, returned by value in
// the generated Julia): device pointers by default, host with the flag.
template <class T>
struct ScalarOut {
  T* user;
  bool host;
};

// ---- device helpers ---------------------------------------------------------
template <class T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sum over the block in a fixed tree; every thread gets the result.
// `red` needs blockDim.x / 32 entries of shared memory.
template <class T>
__device__ __forceinline__ T block_sum(T v, T* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nwarps = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  T s = T(0);
  if (warp == 0) {
    s = lane < nwarps ? red[lane] : T(0);
    s = warp_sum(s);
    if (lane == 0) red[0] = s;
  }
  __syncthreads();
  s = red[0];
  return s;
}

// Sums `count` partial vectors of length `len` (partials[p * len + e]) in the
// fixed order p = 0, 1, ..., and adds the result into dst[e] (or stores it
// when `accumulate` is false). One thread per element: deterministic.

// sum over q of v[q * stride] added in the order q = 0, 1, ..., count - 1
// (reverse: count - 1 down to 0); the loads are issued 8 at a time so their
// latencies overlap, the additions stay in that order.
template <class T>
__device__ __forceinline__ T ordered_sum(const T* __restrict__ v, int count, int64_t stride,
                                         bool reverse = false) {
  T acc = T(0);
  int p = 0;
  for (; p + 8 <= count; p += 8) {
    T r[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int q = reverse ? count - 1 - (p + u) : p + u;
      r[u] = v[(int64_t)q * stride];
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) acc = acc + r[u];
  }
  for (; p < count; ++p) {
    const int q = reverse ? count - 1 - p : p;
    acc = acc + v[(int64_t)q * stride];
  }
  return acc;
}
template <class T>
__global__ void reduce_partials_kernel(const T* __restrict__ partials, int64_t len, int count,
                                       T* __restrict__ dst, bool accumulate) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= len) return;
  T acc = T(0);
  int p = 0;
  for (; p + 4 <= count; p += 4) {
    const T a0 = partials[(int64_t)(p + 0) * len + e];
    const T a1 = partials[(int64_t)(p + 1) * len + e];
    const T a2 = partials[(int64_t)(p + 2) * len + e];
    const T a3 = partials[(int64_t)(p + 3) * len + e];
    acc = acc + a0;
    acc = acc + a1;
    acc = acc + a2;
    acc = acc + a3;
  }
  for (; p < count; ++p) acc = acc + partials[(int64_t)p * len + e];
  dst[e] = accumulate ? dst[e] + acc : acc;
}

// Sums a long vector into one scalar in a fixed order with one block:
// thread t sums elements t, t + blockDim, ... then a block tree.
template <class T>
__global__ void sum_to_scalar_kernel(const T* __restrict__ v, int64_t len, T* __restrict__ dst,
                                     bool accumulate) {
  __shared__ T red[32];
  T acc = T(0);
  for (int64_t e = threadIdx.x; e < len; e += blockDim.x) acc = acc + v[e];
  acc = block_sum(acc, red);
  if (threadIdx.x == 0) dst[0] = accumulate ? dst[0] + acc : acc;
}

template <class T>
stade_status launch_reduce_partials(const T* partials, int64_t len, int count, T* dst,
                                    bool accumulate, cudaStream_t s) {
  if (len <= 0) return STADE_OK;
  const int threads = 256;
  const int64_t blocks = (len + threads - 1) / threads;
  reduce_partials_kernel<T><<<(unsigned)blocks, threads, 0, s>>>(partials, len, count, dst, accumulate);
  STADE_CHECK_LAUNCH();
  return STADE_OK;
}

template <class T>
stade_status launch_sum_to_scalar(const T* v, int64_t len, T* dst, bool accumulate, cudaStream_t s) {
  sum_to_scalar_kernel<T><<<1, 1024, 0, s>>>(v, len, dst, accumulate);
  STADE_CHECK_LAUNCH();
  return STADE_OK;
}

inline unsigned ceil_div_u(int64_t a, int64_t b) { return (unsigned)((a + b - 1) / b); }

}  // namespace stade
