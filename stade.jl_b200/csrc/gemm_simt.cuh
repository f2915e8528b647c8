// SIMT (CUDA-core FMA) tiled GEMM with functor operand loaders, functor
// epilogues and a deterministic split-K: C[m, n] = sum_k A(m, k) B(k, n).
//
// Used for the Float64 contractions (tcgen05 has no f64 kind, so DFMA is the
// path to the FP64 peak) and as the reference Float32 path. Each of the
// 16 x 16 threads of a block owns a TM x TN sub-tile made of 4 x 4 groups
// strided by 64 rows / columns (conflict-free 16-byte shared-memory reads);
// operand tiles are double-buffered through registers and shared memory.
// With split-K every slice of K writes its own partial tile and a second pass
// sums the slices in slice order, so results do not depend on scheduling.
#pragma once

#include "common.cuh"

namespace stade {

template <class T> struct Vec4;
template <> struct Vec4<float> {
  float v[4];
  __device__ __forceinline__ void load(const float* p) {
    const float4 q = *reinterpret_cast<const float4*>(p);
    v[0] = q.x; v[1] = q.y; v[2] = q.z; v[3] = q.w;
  }
};
template <> struct Vec4<double> {
  double v[4];
  __device__ __forceinline__ void load(const double* p) {
    const double2 q0 = *reinterpret_cast<const double2*>(p);
    const double2 q1 = *reinterpret_cast<const double2*>(p + 2);
    v[0] = q0.x; v[1] = q0.y; v[2] = q1.x; v[3] = q1.y;
  }
};

// BM = 64 * RM, BN = 64 * RN; TM = 4 * RM, TN = 4 * RN.
template <class T, int RM, int RN, int BK>
struct SimtCfg {
  static constexpr int BM = 64 * RM, BN = 64 * RN;
  static constexpr int TM = 4 * RM, TN = 4 * RN;
  static constexpr int PAD = 4;
  static constexpr int LDA = BM + PAD, LDB = BN + PAD;
  static constexpr int A_PER = BM * BK / 256, B_PER = BN * BK / 256;
  static_assert((BM * BK) % 256 == 0 && (BN * BK) % 256 == 0, "tile / thread mismatch");
};

// A_KC: the loader's cheap direction is k (consecutive threads read
// consecutive k); otherwise m. B_NC: consecutive threads read consecutive n;
// otherwise k. Loaders are called only for in-range (m, k) / (k, n).
template <class T, int RM, int RN, int BK, bool A_KC, bool B_NC, class LA, class LB, class Epi>
__global__ void __launch_bounds__(256)
gemm_simt_kernel(int M, int N, int K, int k_slice, LA la, LB lb, T* __restrict__ partial, Epi epi) {
  using C = SimtCfg<T, RM, RN, BK>;
  __shared__ __align__(16) T As[2][BK][C::LDA];
  __shared__ __align__(16) T Bs[2][BK][C::LDB];

  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;
  const int m0 = blockIdx.y * C::BM, n0 = blockIdx.x * C::BN;
  const int kbeg = blockIdx.z * k_slice;
  const int kend = min(K, kbeg + k_slice);

  T ra[C::A_PER], rb[C::B_PER];
  auto gload = [&](int k0) {
#pragma unroll
    for (int q = 0; q < C::A_PER; ++q) {
      const int e = tid + q * 256;
      const int mm = A_KC ? e / BK : e % C::BM;
      const int kk = A_KC ? e % BK : e / C::BM;
      const int m = m0 + mm, k = k0 + kk;
      ra[q] = (m < M && k < kend) ? la(m, k) : T(0);
    }
#pragma unroll
    for (int q = 0; q < C::B_PER; ++q) {
      const int e = tid + q * 256;
      const int nn = B_NC ? e % C::BN : e / BK;
      const int kk = B_NC ? e / C::BN : e % BK;
      const int n = n0 + nn, k = k0 + kk;
      rb[q] = (n < N && k < kend) ? lb(k, n) : T(0);
    }
  };
  auto sstore = [&](int buf) {
#pragma unroll
    for (int q = 0; q < C::A_PER; ++q) {
      const int e = tid + q * 256;
      const int mm = A_KC ? e / BK : e % C::BM;
      const int kk = A_KC ? e % BK : e / C::BM;
      As[buf][kk][mm] = ra[q];
    }
#pragma unroll
    for (int q = 0; q < C::B_PER; ++q) {
      const int e = tid + q * 256;
      const int nn = B_NC ? e % C::BN : e / BK;
      const int kk = B_NC ? e / C::BN : e % BK;
      Bs[buf][kk][nn] = rb[q];
    }
  };

  T acc[C::TM][C::TN];
#pragma unroll
  for (int i = 0; i < C::TM; ++i)
#pragma unroll
    for (int j = 0; j < C::TN; ++j) acc[i][j] = T(0);

  int buf = 0;
  if (kbeg < kend) {
    gload(kbeg);
    sstore(0);
    __syncthreads();
    for (int k0 = kbeg; k0 < kend; k0 += BK) {
      const bool more = k0 + BK < kend;
      if (more) gload(k0 + BK);
#pragma unroll
      for (int kk = 0; kk < BK; ++kk) {
        T a[C::TM], b[C::TN];
#pragma unroll
        for (int g = 0; g < RM; ++g) {
          Vec4<T> v;
          v.load(&As[buf][kk][g * 64 + ty * 4]);
#pragma unroll
          for (int i = 0; i < 4; ++i) a[g * 4 + i] = v.v[i];
        }
#pragma unroll
        for (int g = 0; g < RN; ++g) {
          Vec4<T> v;
          v.load(&Bs[buf][kk][g * 64 + tx * 4]);
#pragma unroll
          for (int j = 0; j < 4; ++j) b[g * 4 + j] = v.v[j];
        }
#pragma unroll
        for (int i = 0; i < C::TM; ++i)
#pragma unroll
          for (int j = 0; j < C::TN; ++j) acc[i][j] = fma(a[i], b[j], acc[i][j]);
      }
      if (more) {
        sstore(buf ^ 1);
        __syncthreads();
        buf ^= 1;
      }
    }
  }

#pragma unroll
  for (int i = 0; i < C::TM; ++i) {
    const int m = m0 + (i / 4) * 64 + ty * 4 + (i % 4);
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < C::TN; ++j) {
      const int n = n0 + (j / 4) * 64 + tx * 4 + (j % 4);
      if (n >= N) continue;
      if (partial)
        partial[((int64_t)blockIdx.z * M + m) * N + n] = acc[i][j];
      else
        epi(m, n, acc[i][j]);
    }
  }
  // block-level hook of the epilogue (e.g. a per-block loss partial);
  // reached by every thread of the block
  if (!partial) epi.finish((int64_t)blockIdx.y * gridDim.x + blockIdx.x);
}

// Sums split-K partials in slice order and applies the epilogue.
template <class T, class Epi>
__global__ void gemm_splitk_finish_kernel(const T* __restrict__ partial, int splits, int M, int N,
                                          Epi epi) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t MN = (int64_t)M * N;
  if (e < MN) {
    T acc = T(0);
    acc = ordered_sum(partial + e, splits, MN);
    epi((int)(e / N), (int)(e % N), acc);
  }
  epi.finish((int64_t)blockIdx.x);
}

// Epilogues derive from this to get the no-op block hook.
struct EpiBase {
  __device__ __forceinline__ void finish(int64_t) const {}
};

struct SplitPlan {
  int splits;
  int k_slice;
};

// Picks the number of K slices so that the grid covers the GPU about twice.
inline SplitPlan split_plan(int tiles, int K, int BK, int max_splits, int sms = 148) {
  SplitPlan p;
  int want = (2 * sms + tiles - 1) / tiles;
  if (want < 1) want = 1;
  const int kblocks = (K + BK - 1) / BK;
  if (want > kblocks) want = kblocks;
  if (want > max_splits) want = max_splits;
  // each slice gets at least 4 k-blocks
  while (want > 1 && kblocks / want < 4) --want;
  const int per = (kblocks + want - 1) / want;
  p.k_slice = per * BK;
  p.splits = (K + p.k_slice - 1) / p.k_slice;
  if (p.splits < 1) p.splits = 1;
  return p;
}

// Launches C = A B with the epilogue, split over K when the tile grid alone is
// too small for the GPU. `partial` must hold splits * M * N elements when
// splits > 1 (query with gemm_partial_elems).
template <class T, int RM, int RN, int BK, bool A_KC, bool B_NC, class LA, class LB, class Epi>
stade_status gemm_simt(int M, int N, int K, LA la, LB lb, Epi epi, T* partial, int splits,
                       cudaStream_t s) {
  using C = SimtCfg<T, RM, RN, BK>;
  if (M <= 0 || N <= 0) return STADE_OK;
  const int tiles_m = (M + C::BM - 1) / C::BM, tiles_n = (N + C::BN - 1) / C::BN;
  if (tiles_m > 65535) return fail(STADE_ENOTSUP, "gemm: M = %d too large", M);
  int k_slice = K > 0 ? K : 1;
  if (splits > 1) {
    const int kblocks = (K + BK - 1) / BK;
    const int per = (kblocks + splits - 1) / splits;
    k_slice = per * BK;
    splits = (K + k_slice - 1) / k_slice;
    if (splits < 1) splits = 1;
  } else {
    splits = 1;
  }
  dim3 grid(tiles_n, tiles_m, splits);
  gemm_simt_kernel<T, RM, RN, BK, A_KC, B_NC, LA, LB, Epi>
      <<<grid, 256, 0, s>>>(M, N, K, k_slice, la, lb, splits > 1 ? partial : nullptr, epi);
  STADE_CHECK_LAUNCH();
  if (splits > 1) {
    const int64_t MN = (int64_t)M * N;
    gemm_splitk_finish_kernel<T, Epi><<<ceil_div_u(MN, 256), 256, 0, s>>>(partial, splits, M, N, epi);
    STADE_CHECK_LAUNCH();
  }
  return STADE_OK;
}

}  // namespace stade
