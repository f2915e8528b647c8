// Float64 GEMM on the FP64 tensor cores (DMMA, mma.sync m8n8k4 .f64 — the
// only f64 tensor-core instruction: tcgen05 has no f64 kind), with the same
// functor operand loaders, functor epilogues and deterministic split-K as
// gemm_simt: C[m, n] = sum_k A(m, k) B(k, n).
//
// Block tile 128 x 128, K staged 16 at a time through double-buffered
// shared memory (operands pass through registers, so any loader works);
// 8 warps in a 2 x 4 grid, each warp owns a 64 x 32 tile = 8 x 4 DMMA tiles
// (64 accumulators per thread). Fragment reads from shared memory are
// conflict-free with rows padded to 132 doubles. A split-K slice writes its
// own partial tile; gemm_splitk_finish_kernel sums the slices in order.
#pragma once

#include "gemm_simt.cuh"

namespace stade {

namespace dmma {
constexpr int BM = 128, BN = 128, BK = 16;
constexpr int LDA = BM + 4, LDB = BN + 4;
constexpr int A_PER = BM * BK / 256, B_PER = BN * BK / 256;
constexpr size_t kSmemBytes = sizeof(double) * 2 * BK * (LDA + LDB);

__device__ __forceinline__ void mma_m8n8k4(double& d0, double& d1, double a, double b) {
  asm volatile("mma.sync.aligned.m8n8k4.row.col.f64.f64.f64.f64 {%0, %1}, {%2}, {%3}, {%0, %1};"
               : "+d"(d0), "+d"(d1)
               : "d"(a), "d"(b));
}
}  // namespace dmma

template <bool A_KC, bool B_NC, class LA, class LB, class Epi>
__global__ void __launch_bounds__(256, 1)
gemm_dmma_kernel(int M, int N, int K, int k_slice, LA la, LB lb, double* __restrict__ partial,
                 Epi epi) {
  using namespace dmma;
  extern __shared__ __align__(16) double dsm[];
  double* As = dsm;                       // [2][BK][LDA]
  double* Bs = dsm + 2 * BK * LDA;        // [2][BK][LDB]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int wm = (warp >> 2) * 64, wn = (warp & 3) * 32;  // warp tile origin in the block tile
  const int g = lane >> 2, q = lane & 3;                   // fragment coordinates
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int kbeg = blockIdx.z * k_slice;
  const int kend = min(K, kbeg + k_slice);

  double ra[A_PER], rb[B_PER];
  auto gload = [&](int k0) {
#pragma unroll
    for (int p = 0; p < A_PER; ++p) {
      const int e = tid + p * 256;
      const int mm = A_KC ? e / BK : e % BM;
      const int kk = A_KC ? e % BK : e / BM;
      const int m = m0 + mm, k = k0 + kk;
      ra[p] = (m < M && k < kend) ? la(m, k) : 0.0;
    }
#pragma unroll
    for (int p = 0; p < B_PER; ++p) {
      const int e = tid + p * 256;
      const int nn = B_NC ? e % BN : e / BK;
      const int kk = B_NC ? e / BN : e % BK;
      const int n = n0 + nn, k = k0 + kk;
      rb[p] = (n < N && k < kend) ? lb(k, n) : 0.0;
    }
  };
  auto sstore = [&](int buf) {
#pragma unroll
    for (int p = 0; p < A_PER; ++p) {
      const int e = tid + p * 256;
      const int mm = A_KC ? e / BK : e % BM;
      const int kk = A_KC ? e % BK : e / BM;
      As[(buf * BK + kk) * LDA + mm] = ra[p];
    }
#pragma unroll
    for (int p = 0; p < B_PER; ++p) {
      const int e = tid + p * 256;
      const int nn = B_NC ? e % BN : e / BK;
      const int kk = B_NC ? e / BN : e % BK;
      Bs[(buf * BK + kk) * LDB + nn] = rb[p];
    }
  };

  double acc[8][4][2];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j][0] = acc[i][j][1] = 0.0;

  int buf = 0;
  if (kbeg < kend) {
    gload(kbeg);
    sstore(0);
    __syncthreads();
    for (int k0 = kbeg; k0 < kend; k0 += BK) {
      const bool more = k0 + BK < kend;
      if (more) gload(k0 + BK);
      const double* a_s = As + buf * BK * LDA;
      const double* b_s = Bs + buf * BK * LDB;
#pragma unroll
      for (int ks = 0; ks < BK; ks += 4) {
        double af[8], bf[4];
#pragma unroll
        for (int i = 0; i < 8; ++i) af[i] = a_s[(ks + q) * LDA + wm + 8 * i + g];
#pragma unroll
        for (int j = 0; j < 4; ++j) bf[j] = b_s[(ks + q) * LDB + wn + 8 * j + g];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) dmma::mma_m8n8k4(acc[i][j][0], acc[i][j][1], af[i], bf[j]);
      }
      if (more) {
        sstore(buf ^ 1);
        __syncthreads();
        buf ^= 1;
      }
    }
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = m0 + wm + 8 * i + g;
    if (m >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int n = n0 + wn + 8 * j + 2 * q + h;
        if (n >= N) continue;
        if (partial)
          partial[((int64_t)blockIdx.z * M + m) * N + n] = acc[i][j][h];
        else
          epi(m, n, acc[i][j][h]);
      }
    }
  }
  if (!partial) epi.finish((int64_t)blockIdx.y * gridDim.x + blockIdx.x);
}

// Same contract as gemm_simt<double, ...> (splits and partial included).
template <bool A_KC, bool B_NC, class LA, class LB, class Epi>
stade_status gemm_dmma(int M, int N, int K, LA la, LB lb, Epi epi, double* partial, int splits,
                       cudaStream_t s) {
  using namespace dmma;
  if (M <= 0 || N <= 0) return STADE_OK;
  const int tiles_m = (M + BM - 1) / BM, tiles_n = (N + BN - 1) / BN;
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
  auto kern = gemm_dmma_kernel<A_KC, B_NC, LA, LB, Epi>;
  STADE_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  (int)kSmemBytes));
  dim3 grid(tiles_n, tiles_m, splits);
  kern<<<grid, 256, kSmemBytes, s>>>(M, N, K, k_slice, la, lb, splits > 1 ? partial : nullptr, epi);
  STADE_CHECK_LAUNCH();
  if (splits > 1) {
    const int64_t MN = (int64_t)M * N;
    gemm_splitk_finish_kernel<double, Epi>
        <<<ceil_div_u(MN, 256), 256, 0, s>>>(partial, splits, M, N, epi);
    STADE_CHECK_LAUNCH();
  }
  return STADE_OK;
}

}  // namespace stade
