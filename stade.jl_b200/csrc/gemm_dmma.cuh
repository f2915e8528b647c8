// Float64 GEMM on the FP64 tensor cores (DMMA: mma.sync .f64 — tcgen05 has no
// f64 kind), with the same functor operand loaders, functor epilogues and
// deterministic split-K as gemm_simt: C[m, n] = sum_k A(m, k) B(k, n).
//
// Block tile 128 x 128, K staged 16 at a time through double-buffered
// shared memory (operands pass through registers, so any loader works);
// 8 warps in a 2 x 4 grid, each warp owns a 64 x 32 tile = 4 x 4 tiles of
// mma.sync.m16n8k8.f64 (64 accumulators per thread; one instruction is 1024
// multiply-adds, eight times an m8n8k4's). Fragment reads from shared memory
// are conflict-free with rows padded to 132 doubles. A split-K slice writes
// its own partial tile; gemm_splitk_finish_kernel sums the slices in order.
#pragma once

#include "gemm_simt.cuh"

namespace stade {

namespace dmma {
constexpr int BM = 128, BN = 128, BK = 16;
constexpr int LDA = BM + 4, LDB = BN + 4;
constexpr int A_PER = BM * BK / 256, B_PER = BN * BK / 256;
constexpr size_t kSmemBytes = sizeof(double) * 2 * BK * (LDA + LDB);

// D (16 x 8) += A (16 x 8, row) B (8 x 8, col). Fragments, g = lane / 4,
// t = lane % 4: a = {A[g][t], A[g+8][t], A[g][t+4], A[g+8][t+4]};
// b = {B[t][g], B[t+4][g]}; d = {D[g][2t], D[g][2t+1], D[g+8][2t], D[g+8][2t+1]}.
__device__ __forceinline__ void mma_m16n8k8(double (&d)[4], double a0, double a1, double a2,
                                            double a3, double b0, double b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f64.f64.f64.f64 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+d"(d[0]), "+d"(d[1]), "+d"(d[2]), "+d"(d[3])
      : "d"(a0), "d"(a1), "d"(a2), "d"(a3), "d"(b0), "d"(b1));
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

  double acc[4][4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int h = 0; h < 4; ++h) acc[i][j][h] = 0.0;

  // m16 / n8 tiles of the warp's 64 x 32 that hold any row / column of C
  // (warp-uniform): a ragged last tile skips the MMAs of its empty part
  const int mi = min(4, max(0, (M - m0 - wm + 15) / 16));
  const int nj = min(4, max(0, (N - n0 - wn + 7) / 8));
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
      for (int ks = 0; ks < BK; ks += 8) {
        double bf[4][2];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          bf[j][0] = b_s[(ks + q) * LDB + wn + 8 * j + g];
          bf[j][1] = b_s[(ks + q + 4) * LDB + wn + 8 * j + g];
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          if (i >= mi) break;
          const double* ap = a_s + (ks + q) * LDA + wm + 16 * i + g;
          const double a0 = ap[0], a1 = ap[8], a2 = ap[4 * LDA], a3 = ap[4 * LDA + 8];
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (j < nj) dmma::mma_m16n8k8(acc[i][j], a0, a1, a2, a3, bf[j][0], bf[j][1]);
        }
      }
      if (more) {
        sstore(buf ^ 1);
        __syncthreads();
        buf ^= 1;
      }
    }
  }

#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int hm = 0; hm < 2; ++hm) {
      const int m = m0 + wm + 16 * i + 8 * hm + g;
      if (m >= M) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int n = n0 + wn + 8 * j + 2 * q + h;
          if (n >= N) continue;
          if (partial)
            partial[((int64_t)blockIdx.z * M + m) * N + n] = acc[i][j][2 * hm + h];
          else
            epi(m, n, acc[i][j][2 * hm + h]);
        }
      }
    }
  }
  if (!partial) epi.finish((int64_t)blockIdx.y * gridDim.x + blockIdx.x);
}

// Split-K slices for the DMMA kernel (one 128 x 128 block per SM at a time:
// 242-252 registers x 256 threads): the slice count minimising whole waves of
// blocks x K blocks per slice, plus a charge of 4 K blocks per partial tile
// written and summed back; at least 8 K blocks per slice. The weight
// gradients of mlp2_ce_hv (28 tiles, K = 16,384 / 32,768) get 5 slices: 140
// blocks, one wave, where a target of two blocks per SM (11 slices, 308
// blocks) left a third wave 8 % full.
inline int dmma_splits(int tiles, int K, int sms) {
  const int kb = (K + dmma::BK - 1) / dmma::BK;
  int best = 1;
  double best_cost = 0.0;
  for (int sl = 1; sl <= 64; ++sl) {
    const int per = (kb + sl - 1) / sl;
    if (sl > 1 && per < 8) break;
    const int slices = (kb + per - 1) / per;
    const int waves = (tiles * slices + sms - 1) / sms;
    const double cost = (double)waves * per + (slices > 1 ? 4.0 * slices * tiles / sms : 0.0);
    if (sl == 1 || cost < best_cost) {
      best = sl;
      best_cost = cost;
    }
  }
  return best;
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
