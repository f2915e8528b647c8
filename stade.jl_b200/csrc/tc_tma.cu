// TMA-fed tensor-core (tcgen05 / TMEM) Float32 contractions with 3xTF32
// splitting: the mlp2_ce adjoint's three GEMMs.
//
// Every Float32 operand is held in memory as two planes, hi (low 13 mantissa
// bits cleared: exactly representable in TF32) and lo = value - hi (exact).
// kind::tf32 reads only the top 19 bits of each 32-bit operand (measured on
// the B200: products with the raw value and with hi agree bit for bit), so a
// caller's array serves as its own hi plane and one pass writes its lo plane
// (x, W1); s1b is written as planes directly by the pass that produces it. D = A B^T then needs
// hi*hi + hi*lo + lo*hi (lo*lo is below Float32 rounding), three
// tcgen05.mma.kind::tf32 per K step into one TMEM accumulator.
//
// Two kernels share this scheme: tma_gemm_pair_kernel (the default for C2's
// three GEMMs) runs 256 x 256 tiles on CTA pairs with the 2-SM MMA and writes
// its output with TMA stores / reductions; tma_gemm_kernel runs one
// 128 x 128 tile per CTA and stores from registers (where a pair tile does not
// apply: logits partials in the forward epilogue, outputs not 16-byte aligned,
// or STADE_TMA_PAIR=0). The one-CTA form:
// Persistent kernel, one CTA per SM, warp-specialised:
//   warp 0  one thread issues TMA loads (cp.async.bulk.tensor, each copy into its own CTA)
//           of the four 128 x 32 operand tiles of a K block into a 3-stage
//           ring of 128-byte-swizzled shared memory, signalled by
//           mbarrier complete_tx;
//   warp 1  owns TMEM (2 accumulators x 128 columns) and one thread issues
//           the MMAs, releasing each stage with tcgen05.commit;
//   warps 2-9 drain an accumulator with tcgen05.ld while the MMAs fill the
//           other one, and apply the fused epilogue.
// An operand is K-major (K contiguous in memory: one 128 x 32 box) or
// MN-major (M or N contiguous: four 32 x 32 boxes), described to the MMA by
// its shared-memory descriptor, so no operand is ever transposed.
// Every wait is bounded (~2 s of clock); on timeout the kernel sets
// g_tma_error, stops issuing work, waits (bounded) for its own copies and
// tensor-core operations, frees TMEM and returns.
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <vector>

#include "tc_tma.cuh"
#include "tcgen05.cuh"

namespace stade {
namespace tma {

constexpr int BM = 128, BN = 128, BK = 32, STAGES = 3;
constexpr int kEpiWarps = 8;
constexpr int kThreads = (2 + kEpiWarps) * 32;  // 320
constexpr int kTileBytes = 128 * BK * 4;        // 16 KiB
constexpr int kStageBytes = 4 * kTileBytes;     // A hi, A lo, B hi, B lo
// stages + alignment slack + barrier block (256 B); the logits epilogue adds
// kW2SmemBytes right after the barrier block
constexpr int kSmemBytes = STAGES * kStageBytes + 1024 + 256;
// TMEM accumulators the MMAs rotate through: the MMA thread may run up to
// kAccBufs - 1 accumulation chains ahead of the epilogue warps draining them
constexpr int kAccBufs = 4;
constexpr uint32_t kTmemCols = kAccBufs * 128;  // all 512 columns of the SM's TMEM
constexpr int kBarWords = 2 * STAGES + 2 * kAccBufs + 1;  // full, empty, tfull, tempty, done
static_assert(kBarWords * 8 + 4 <= 256, "barrier block must fit in 256 bytes");
// Default K blocks per TMEM accumulation chain. The tensor core's Float32
// accumulation is not round-to-nearest: its error grows linearly with the
// number of accumulations into one TMEM accumulator (measured: 1.4e-5
// relative after 1000 K). Chains of 4 K blocks (128 K, 48 MMAs) are drained
// into round-to-nearest Float32 sums in registers by the epilogue warps,
// while the other TMEM buffer takes the next chain.
constexpr int kChainBlocks = 4;

__device__ int g_tma_error = 0;

// ---- PTX building blocks (tcgen05.cuh) -------------------------------------------
using tc5::smem_u32;
using tc5::mbar_init;
using tc5::mbar_arrive;
using tc5::mbar_arrive_tx;
using tc5::tma_load_2d;
using tc5::mma_tf32;
using tc5::mma_commit;
using tc5::tmem_ld16;
using tc5::desc_sw128;
using tc5::idesc_tf32;
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  return tc5::mbar_wait(bar, parity, &g_tma_error);
}
__device__ __forceinline__ void tc_fence_before() { tc5::fence_before(); }
__device__ __forceinline__ void tc_fence_after() { tc5::fence_after(); }

// ---- epilogues: a thread owns one accumulator row and gets 16 columns at a time
__host__ __device__ __forceinline__ bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

struct EpiTanhLogits {  // h = tanh(acc + b1); zpart[part][m][c] = sum h w2 over the thread's columns
  float* h;
  const float* b1;
  const float* w2;
  float* zpart;
  int ld, M, N, n_o, parts_per_tile;
  int w2_stride;  // > 0: w2 staged in shared memory with this row stride (multiple of 4)
};
constexpr int kW2SmemBytes = 32768;
struct EpiAccumulate {  // out[m, n] += acc
  float* out;
  int ld, M, N;
};
struct EpiPartial {  // part[slice][m][n] = acc
  float* part;
  int M, N;
};

__device__ __forceinline__ void epi_acc_chunk(const EpiAccumulate& e, int m, int n0,
                                              const float (&v)[16]) {
  if (m >= e.M) return;
  float* o = e.out + (int64_t)m * e.ld + n0;
  if (n0 + 16 <= e.N && aligned16(o)) {
#pragma unroll
    for (int i = 0; i < 16; i += 4) {
      float4 q = *reinterpret_cast<float4*>(o + i);
      q.x += v[i]; q.y += v[i + 1]; q.z += v[i + 2]; q.w += v[i + 3];
      *reinterpret_cast<float4*>(o + i) = q;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (n0 + i < e.N) o[i] = o[i] + v[i];
  }
}

__device__ __forceinline__ void epi_part_chunk(const EpiPartial& e, int m, int n0, int slice,
                                               const float (&v)[16]) {
  if (m >= e.M) return;
  float* o = e.part + ((int64_t)slice * e.M + m) * e.N + n0;
  if (n0 + 16 <= e.N && aligned16(o)) {
#pragma unroll
    for (int i = 0; i < 16; i += 4)
      *reinterpret_cast<float4*>(o + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i)
      if (n0 + i < e.N) o[i] = v[i];
  }
}

// The fused epilogue of one tile, from the thread's register sums of its 64
// columns of row m: 16-wide groups g0, g0 + GS, g0 + 2 GS, g0 + 3 GS (GS = 2:
// two column halves of a 128-wide tile; GS = 4: four column quarters of a
// 256-wide one).
template <int EPI_KIND, int NO, int GS>
__device__ __forceinline__ void epi_tile(const float (&sum)[4][16], int m, int n0, int g0,
                                         int slice, const EpiTanhLogits& el,
                                         const EpiAccumulate& ea, const EpiPartial& ep,
                                         const float* w2s) {
  if constexpr (EPI_KIND == 0) {
    float zp[NO];
#pragma unroll
    for (int c = 0; c < NO; ++c) zp[c] = 0.f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int nn = n0 + (g0 + GS * q) * 16;
      if (m < el.M) {
        float* o = el.h + (int64_t)m * el.ld + nn;
        float hv[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          hv[i] = (nn + i < el.N) ? tanhf(sum[q][i] + __ldg(el.b1 + nn + i)) : 0.f;
        if (nn + 16 <= el.N && aligned16(o)) {
#pragma unroll
          for (int i = 0; i < 16; i += 4)
            *reinterpret_cast<float4*>(o + i) =
                make_float4(hv[i], hv[i + 1], hv[i + 2], hv[i + 3]);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (nn + i < el.N) o[i] = hv[i];
        }
        // logits partial (when asked for); w2 rows are the same for the whole
        // warp (broadcast)
        // logits partials only from 128-wide tiles (the host never asks wider ones)
        if (GS != 2 || el.zpart == nullptr) {
        } else if (el.w2_stride > 0) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            if (nn + i < el.N) {
              const float4* wr = reinterpret_cast<const float4*>(w2s + (nn + i) * el.w2_stride);
#pragma unroll
              for (int c4 = 0; c4 < NO / 4; ++c4) {
                if (4 * c4 < el.n_o) {
                  const float4 wv = wr[c4];
                  zp[4 * c4] = fmaf(hv[i], wv.x, zp[4 * c4]);
                  zp[4 * c4 + 1] = fmaf(hv[i], wv.y, zp[4 * c4 + 1]);
                  zp[4 * c4 + 2] = fmaf(hv[i], wv.z, zp[4 * c4 + 2]);
                  zp[4 * c4 + 3] = fmaf(hv[i], wv.w, zp[4 * c4 + 3]);
                }
              }
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            if (nn + i < el.N) {
              const float* wr = el.w2 + (int64_t)(nn + i) * el.n_o;
#pragma unroll
              for (int cc = 0; cc < NO; ++cc)
                if (cc < el.n_o) zp[cc] = fmaf(hv[i], __ldg(wr + cc), zp[cc]);
            }
          }
        }
      }
    }
    if (GS == 2 && m < el.M && el.zpart != nullptr) {
      const int part = (n0 / BN) * 2 + g0;
      float* zr = el.zpart + ((int64_t)part * el.M + m) * el.n_o;
#pragma unroll
      for (int cc = 0; cc < NO; ++cc)
        if (cc < el.n_o) zr[cc] = zp[cc];
    }
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if constexpr (EPI_KIND == 1) epi_acc_chunk(ea, m, n0 + (g0 + GS * q) * 16, sum[q]);
      else epi_part_chunk(ep, m, n0 + (g0 + GS * q) * 16, slice, sum[q]);
    }
  }

}

struct Geometry {
  int M, N, K;
  int m_tiles, n_tiles, slices, k_slice;
  bool a_mn, b_mn;
  int chain;  // K blocks per TMEM accumulation chain
};

// EPI_KIND: 0 logits (NO classes), 1 accumulate, 2 split-K partial
template <int EPI_KIND, int NO>
__global__ void __launch_bounds__(kThreads, 1)
tma_gemm_kernel(const __grid_constant__ CUtensorMap a_hi, const __grid_constant__ CUtensorMap a_lo,
                const __grid_constant__ CUtensorMap b_hi, const __grid_constant__ CUtensorMap b_lo,
                Geometry g, EpiTanhLogits el, EpiAccumulate ea, EpiPartial ep) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw & 1023u)) & 1023u;
  uint8_t* tiles = smem_raw + pad;
  uint64_t* bars = reinterpret_cast<uint64_t*>(tiles + STAGES * kStageBytes);
  // bars: full[STAGES], empty[STAGES], tfull[2], tempty[2], done
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kBarWords);
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES);
  const uint32_t tfull0 = smem_u32(bars + 2 * STAGES);
  const uint32_t tempty0 = smem_u32(bars + 2 * STAGES + kAccBufs);
  const uint32_t done = smem_u32(bars + 2 * STAGES + 2 * kAccBufs);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_per_slice = g.m_tiles * g.n_tiles;
  const int total = tiles_per_slice * g.slices;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < kAccBufs; ++b) {
      mbar_init(tfull0 + 8 * b, 1);
      mbar_init(tempty0 + 8 * b, kEpiWarps);
    }
    mbar_init(done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer ---------------------------------------------------------
      int kb_all = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        const int slice = t / tiles_per_slice, r = t % tiles_per_slice;
        const int m0 = (r / g.n_tiles) * BM, n0 = (r % g.n_tiles) * BN;
        const int kbeg = slice * g.k_slice;
        const int kend = min(g.K, kbeg + g.k_slice);
        const int nkb = kend > kbeg ? (kend - kbeg + BK - 1) / BK : 0;
        for (int kb = 0; kb < nkb; ++kb, ++kb_all) {
          const int s = kb_all % STAGES;
          const uint32_t ph = (uint32_t)(kb_all / STAGES) & 1u;
          if (!mbar_wait(empty0 + 8 * s, ph ^ 1u)) { ok = false; break; }
          const uint32_t st = smem_u32(tiles + s * kStageBytes);
          const uint32_t fb = full0 + 8 * s;
          mbar_arrive_tx(fb, kStageBytes);
          const int k0 = kbeg + kb * BK;
          if (!g.a_mn) {
            tma_load_2d(st, &a_hi, k0, m0, fb);
            tma_load_2d(st + kTileBytes, &a_lo, k0, m0, fb);
          } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              tma_load_2d(st + q * 4096, &a_hi, m0 + 32 * q, k0, fb);
              tma_load_2d(st + kTileBytes + q * 4096, &a_lo, m0 + 32 * q, k0, fb);
            }
          }
          if (!g.b_mn) {
            tma_load_2d(st + 2 * kTileBytes, &b_hi, k0, n0, fb);
            tma_load_2d(st + 3 * kTileBytes, &b_lo, k0, n0, fb);
          } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              tma_load_2d(st + 2 * kTileBytes + q * 4096, &b_hi, n0 + 32 * q, k0, fb);
              tma_load_2d(st + 3 * kTileBytes + q * 4096, &b_lo, n0 + 32 * q, k0, fb);
            }
          }
        }
      }
      // copies still in flight land before the CTA exits: wait for the last
      // phase armed on every stage (bounded)
      for (int i = 0; i < STAGES && i < kb_all; ++i) {
        const int last = kb_all - 1 - i;
        mbar_wait(full0 + 8 * (last % STAGES), (uint32_t)(last / STAGES) & 1u);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer -------------------------------------------------------------
      const uint32_t idesc_full = idesc_tf32(BM, BN, g.a_mn, g.b_mn);
      const uint32_t a_lbo = g.a_mn ? 4096u : 16u, a_sbo = g.a_mn ? 512u : 1024u;
      const uint32_t b_lbo = g.b_mn ? 4096u : 16u, b_sbo = g.b_mn ? 512u : 1024u;
      const uint32_t a_lay = g.a_mn ? 1u : 2u, b_lay = g.b_mn ? 1u : 2u;
      const uint32_t a_step = g.a_mn ? 1024u : 32u, b_step = g.b_mn ? 1024u : 32u;
      int kb_all = 0, chain = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        const int slice = t / tiles_per_slice;
        const int kbeg = slice * g.k_slice;
        const int kend = min(g.K, kbeg + g.k_slice);
        const int nkb = kend > kbeg ? (kend - kbeg + BK - 1) / BK : 0;
        const int nch = nkb > 0 ? (nkb + g.chain - 1) / g.chain : 1;
        // A ragged last N tile of a K-major B runs MMAs only as wide as its
        // columns (rounded up to 16; the rest of the box is zero-filled and
        // the epilogue stores only columns < N): 784 = 6 x 128 + 16 spends
        // 1/8 of a tile there instead of a whole one.
        uint32_t idesc = idesc_full;
        if (!g.b_mn) {
          const int n0 = ((t % tiles_per_slice) % g.n_tiles) * BN;
          const int n_eff = min(BN, (g.N - n0 + 15) / 16 * 16);
          if (n_eff < BN) idesc = idesc_tf32(BM, n_eff, g.a_mn, g.b_mn);
        }
        for (int ch = 0; ch < nch && ok; ++ch, ++chain) {
          const int b = chain % kAccBufs;
          const uint32_t acc = tmem + (uint32_t)(b * BN);
          if (!mbar_wait(tempty0 + 8 * b, ((uint32_t)(chain / kAccBufs) & 1u) ^ 1u)) { ok = false; break; }
          tc_fence_after();
          const int kb0 = ch * g.chain, kb1 = min(nkb, kb0 + g.chain);
          for (int kb = kb0; kb < kb1; ++kb, ++kb_all) {
            const int s = kb_all % STAGES;
            const uint32_t ph = (uint32_t)(kb_all / STAGES) & 1u;
            if (!mbar_wait(full0 + 8 * s, ph)) { ok = false; break; }
            tc_fence_after();
            const uint32_t st = smem_u32(tiles + s * kStageBytes);
#pragma unroll
            for (int j = 0; j < BK / 8; ++j) {
              const uint64_t ahi = desc_sw128(st + a_step * j, a_lbo, a_sbo, a_lay);
              const uint64_t alo = desc_sw128(st + kTileBytes + a_step * j, a_lbo, a_sbo, a_lay);
              const uint64_t bhi = desc_sw128(st + 2 * kTileBytes + b_step * j, b_lbo, b_sbo, b_lay);
              const uint64_t blo = desc_sw128(st + 3 * kTileBytes + b_step * j, b_lbo, b_sbo, b_lay);
              mma_tf32(acc, ahi, blo, idesc, (kb != kb0 || j != 0) ? 1u : 0u);
              mma_tf32(acc, alo, bhi, idesc, 1u);
              mma_tf32(acc, ahi, bhi, idesc, 1u);
            }
            mma_commit(empty0 + 8 * s);
          }
          // an empty chain (K = 0) still hands a buffer over; the epilogue ignores it
          mma_commit(tfull0 + 8 * b);
        }
      }
      // every MMA issued above completes before TMEM is freed
      mma_commit(done);
      mbar_wait(done, 0);
    }
  } else {
    // ---- epilogue warps -------------------------------------------------------------
    const int e = warp - 2;
    const int quad = warp & 3;       // TMEM lanes 32 quad .. 32 quad + 31
    const int half = e >> 2;         // column half of the tile
    // logits epilogue: all of w2 in shared memory, rows padded to w2_stride
    // (16-byte aligned: the barrier block is 1024-aligned and uses < 256 bytes)
    float* w2s = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 256);
    if constexpr (EPI_KIND == 0) {
      if (el.w2_stride > 0) {
        for (int i = threadIdx.x - 64; i < el.N * el.w2_stride; i += kEpiWarps * 32) {
          const int kk = i / el.w2_stride, c = i % el.w2_stride;
          w2s[i] = c < el.n_o ? el.w2[(int64_t)kk * el.n_o + c] : 0.f;
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kEpiWarps * 32) : "memory");
      }
    }
    int chain = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
      const int slice = t / tiles_per_slice, r = t % tiles_per_slice;
      const int m0 = (r / g.n_tiles) * BM, n0 = (r % g.n_tiles) * BN;
      const int kbeg = slice * g.k_slice;
      const int kend = min(g.K, kbeg + g.k_slice);
      const int nkb = kend > kbeg ? (kend - kbeg + BK - 1) / BK : 0;
      const int nch = nkb > 0 ? (nkb + g.chain - 1) / g.chain : 1;
      const int m = m0 + quad * 32 + lane;
      // the thread's 64 columns: 16-wide groups half, half + 2, half + 4, half + 6
      float sum[BN / 32][16];
#pragma unroll
      for (int q = 0; q < BN / 32; ++q)
#pragma unroll
        for (int i = 0; i < 16; ++i) sum[q][i] = 0.f;
      for (int ch = 0; ch < nch; ++ch, ++chain) {
        const int b = chain % kAccBufs;
        ok = mbar_wait(tfull0 + 8 * b, (uint32_t)(chain / kAccBufs) & 1u);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        if (nkb > 0) {
          const uint32_t base = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(b * BN);
#pragma unroll
          for (int q = 0; q < BN / 32; ++q) {
            float v[16];
            tmem_ld16(base + (uint32_t)((half + 2 * q) * 16), v);
#pragma unroll
            for (int i = 0; i < 16; ++i) sum[q][i] += v[i];
          }
        }
        // this warp is done with accumulator b
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty0 + 8 * b);
      }
      if (!ok) break;
      epi_tile<EPI_KIND, NO, 2>(sum, m, n0, half, slice, el, ea, ep, w2s);
    }
  }

  // ---- teardown -----------------------------------------------------------------
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols)
                 : "memory");
  }
}

// ---- CTA pairs ---------------------------------------------------------------------
// The same contraction with a 2-SM MMA (tcgen05.mma.cta_group::2, M = 256 per
// pair, N = TN): the two CTAs of a cluster each load their own 128 rows of A
// and one half (TN / 2 rows or columns) of the tile's B into their shared
// memory, and the leader CTA's single MMA thread computes the 256 x TN tile
// from both; each CTA's TMEM holds its own 128 rows x TN columns. Per SM and K
// block a TN = 256 tile moves 64 KB of operand planes for twice the MMA work
// of a 128 x 128 tile (a TN = 128 pair: 48 KB for the same work). Completion
// of both CTAs' loads counts on the leader's `full` barrier; the leader's
// commits arrive on `empty`, `tfull` and `done` in both CTAs; the epilogue
// warps of both CTAs arrive on the leader's `tempty`. Every wait is bounded.
template <int TN>
struct PairTile {
  static constexpr int kBHalf = TN / 2;                        // B rows (N) per CTA
  static constexpr int kBPlane = kBHalf * BK * 4;              // 8 KB / 16 KB
  static constexpr int kStageBytes = 2 * kTileBytes + 2 * kBPlane;  // 48 KB / 64 KB
  static constexpr int kStages = TN == 128 ? 4 : 3;
  static constexpr int kAcc = 512 / TN;                        // TMEM accumulators
  // epilogue warps: four per TMEM lane quarter, each thread 64 columns of its row
  static constexpr int kEpiW = TN / 16;                        // 8 / 16
  static constexpr int kThreads = (2 + kEpiW) * 32;            // 320 / 576
  // 256-wide tiles write their output with TMA stores from a 2 KB block per
  // epilogue warp (after the barrier block, where 128-wide ones may stage W2)
  static constexpr bool kTmaOut = TN == 256;
  static constexpr int kStageOutBytes = kTmaOut ? kEpiW * 2048 : 0;
  static constexpr int kBars = 2 * kStages + 2 * kAcc + 1;
  static constexpr int kSmem = kStages * kStageBytes + 1024 + 256;
  static_assert(kBars * 8 + 4 <= 256, "barrier block must fit in 256 bytes");
  static_assert(kSmem + kW2SmemBytes <= 232448, "shared memory of a CTA");
  static_assert(kSmem + kStageOutBytes <= 232448, "shared memory of a CTA");
};

// Tile of work unit t: slice, first row of the pair's 256-row tile, first
// column, and the columns the MMAs run (`n_mma`: a ragged last tile runs only
// as wide as its columns, rounded up to 32 for a K-major B, so each CTA holds
// 16 or more rows of it, and to 64 for an MN-major B, so each CTA holds whole
// 32-column swizzle atoms). Full-width tiles come first in the order, the
// ragged column tiles after them, so that the pairs' strided walk over the
// units gives every pair nearly the same mix of both.
struct PairUnit {
  int slice, m0, n0, n_mma;
};
template <int TN>
__device__ __forceinline__ PairUnit pair_unit(int t, const Geometry& g) {
  const int tiles_per_slice = g.m_tiles * g.n_tiles;
  PairUnit u;
  u.slice = t / tiles_per_slice;
  const int r = t % tiles_per_slice;
  const int n_full = g.N / TN;
  int mt, nt;
  if (r < g.m_tiles * n_full) {
    mt = r / n_full;
    nt = r % n_full;
  } else {
    mt = r - g.m_tiles * n_full;
    nt = n_full;
  }
  u.m0 = mt * (2 * BM);
  u.n0 = nt * TN;
  u.n_mma = TN;
  if (g.N - u.n0 < TN)
    u.n_mma = g.b_mn ? min(TN, (g.N - u.n0 + 63) / 64 * 64) : (g.N - u.n0 + 31) / 32 * 32;
  return u;
}

template <int EPI_KIND, int NO, int TN>
__global__ void __launch_bounds__(PairTile<TN>::kThreads, 1)
tma_gemm_pair_kernel(const __grid_constant__ CUtensorMap a_hi,
                     const __grid_constant__ CUtensorMap a_lo,
                     const __grid_constant__ CUtensorMap b_hi,
                     const __grid_constant__ CUtensorMap b_lo,
                     const __grid_constant__ CUtensorMap out, Geometry g, EpiTanhLogits el,
                     EpiAccumulate ea, EpiPartial ep) {
  using P = PairTile<TN>;
  constexpr int ST = P::kStages, NACC = P::kAcc;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw & 1023u)) & 1023u;
  uint8_t* tiles = smem_raw + pad;
  uint64_t* bars = reinterpret_cast<uint64_t*>(tiles + ST * P::kStageBytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + P::kBars);
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + ST);
  const uint32_t tfull0 = smem_u32(bars + 2 * ST);
  const uint32_t tempty0 = smem_u32(bars + 2 * ST + NACC);
  const uint32_t done = smem_u32(bars + 2 * ST + 2 * NACC);
  const uint32_t rank = tc5::cluster_rank();
  const bool leader = rank == 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total = g.m_tiles * g.n_tiles * g.slices;   // m_tiles counts 256-row tiles
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    for (int b = 0; b < NACC; ++b) {
      mbar_init(tfull0 + 8 * b, 1);
      mbar_init(tempty0 + 8 * b, 2 * P::kEpiW);
    }
    mbar_init(done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tc5::tmem_alloc_pair(smem_u32(tmem_slot), kTmemCols);
  tc_fence_before();
  tc5::cluster_sync();   // both CTAs' barriers exist before anything signals them
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer (both CTAs) ---------------------------------------------------
      int kb_all = 0;
      bool ok = true;
      for (int t = pair; t < total && ok; t += npairs) {
        const PairUnit u = pair_unit<TN>(t, g);
        const int m0 = u.m0 + (int)rank * BM;
        const int nb = u.n0 + (int)rank * (u.n_mma / 2);   // this CTA's half of B
        const int kbeg = u.slice * g.k_slice;
        const int kend = min(g.K, kbeg + g.k_slice);
        const int nkb = kend > kbeg ? (kend - kbeg + BK - 1) / BK : 0;
        for (int kb = 0; kb < nkb; ++kb, ++kb_all) {
          const int s = kb_all % ST;
          const uint32_t ph = (uint32_t)(kb_all / ST) & 1u;
          if (!tc5::mbar_wait_cluster(empty0 + 8 * s, ph ^ 1u, &g_tma_error)) { ok = false; break; }
          const uint32_t st = smem_u32(tiles + s * P::kStageBytes);
          const uint32_t fb = full0 + 8 * s;
          if (leader) mbar_arrive_tx(fb, 2 * P::kStageBytes);
          const int k0 = kbeg + kb * BK;
          if (!g.a_mn) {
            tc5::tma_load_2d_pair(st, &a_hi, k0, m0, fb);
            tc5::tma_load_2d_pair(st + kTileBytes, &a_lo, k0, m0, fb);
          } else {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              tc5::tma_load_2d_pair(st + q * 4096, &a_hi, m0 + 32 * q, k0, fb);
              tc5::tma_load_2d_pair(st + kTileBytes + q * 4096, &a_lo, m0 + 32 * q, k0, fb);
            }
          }
          const uint32_t sb = st + 2 * kTileBytes;
          if (!g.b_mn) {
            tc5::tma_load_2d_pair(sb, &b_hi, k0, nb, fb);
            tc5::tma_load_2d_pair(sb + P::kBPlane, &b_lo, k0, nb, fb);
          } else {
#pragma unroll
            for (int q = 0; q < P::kBHalf / 32; ++q) {
              tc5::tma_load_2d_pair(sb + q * 4096, &b_hi, nb + 32 * q, k0, fb);
              tc5::tma_load_2d_pair(sb + P::kBPlane + q * 4096, &b_lo, nb + 32 * q, k0, fb);
            }
          }
        }
      }
      // this CTA's copies in flight land before it exits (bounded): the last
      // phase of every stage completes on the leader's barriers, so the peer
      // waits for the leader's commits on its own `empty` instead
      for (int i = 0; i < ST && i < kb_all; ++i) {
        const int last = kb_all - 1 - i;
        if (leader)
          tc5::mbar_wait_cluster(full0 + 8 * (last % ST), (uint32_t)(last / ST) & 1u,
                                 &g_tma_error);
        else
          tc5::mbar_wait_cluster(empty0 + 8 * (last % ST), (uint32_t)(last / ST) & 1u,
                                 &g_tma_error);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---- MMA issuer (leader CTA) ------------------------------------------------------
      const uint32_t a_lbo = g.a_mn ? 4096u : 16u, a_sbo = g.a_mn ? 512u : 1024u;
      const uint32_t b_lbo = g.b_mn ? 4096u : 16u, b_sbo = g.b_mn ? 512u : 1024u;
      const uint32_t a_lay = g.a_mn ? 1u : 2u, b_lay = g.b_mn ? 1u : 2u;
      const uint32_t a_step = g.a_mn ? 1024u : 32u, b_step = g.b_mn ? 1024u : 32u;
      int kb_all = 0, chain = 0;
      bool ok = true;
      for (int t = pair; t < total && ok; t += npairs) {
        const PairUnit u = pair_unit<TN>(t, g);
        const uint32_t idesc = idesc_tf32(2 * BM, u.n_mma, g.a_mn, g.b_mn);
        const int kbeg = u.slice * g.k_slice;
        const int kend = min(g.K, kbeg + g.k_slice);
        const int nkb = kend > kbeg ? (kend - kbeg + BK - 1) / BK : 0;
        const int nch = nkb > 0 ? (nkb + g.chain - 1) / g.chain : 1;
        for (int ch = 0; ch < nch && ok; ++ch, ++chain) {
          const int b = chain % NACC;
          const uint32_t acc = tmem + (uint32_t)(b * TN);
          if (!tc5::mbar_wait_cluster(tempty0 + 8 * b, ((uint32_t)(chain / NACC) & 1u) ^ 1u,
                                      &g_tma_error)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int kb0 = ch * g.chain, kb1 = min(nkb, kb0 + g.chain);
          for (int kb = kb0; kb < kb1; ++kb, ++kb_all) {
            const int s = kb_all % ST;
            const uint32_t ph = (uint32_t)(kb_all / ST) & 1u;
            if (!tc5::mbar_wait_cluster(full0 + 8 * s, ph, &g_tma_error)) { ok = false; break; }
            tc_fence_after();
            const uint32_t st = smem_u32(tiles + s * P::kStageBytes);
            const uint32_t sb = st + 2 * kTileBytes;
#pragma unroll
            for (int j = 0; j < BK / 8; ++j) {
              const uint64_t ahi = desc_sw128(st + a_step * j, a_lbo, a_sbo, a_lay);
              const uint64_t alo = desc_sw128(st + kTileBytes + a_step * j, a_lbo, a_sbo, a_lay);
              const uint64_t bhi = desc_sw128(sb + b_step * j, b_lbo, b_sbo, b_lay);
              const uint64_t blo = desc_sw128(sb + P::kBPlane + b_step * j, b_lbo, b_sbo, b_lay);
              tc5::mma_tf32_pair(acc, ahi, blo, idesc, (kb != kb0 || j != 0) ? 1u : 0u);
              tc5::mma_tf32_pair(acc, alo, bhi, idesc, 1u);
              tc5::mma_tf32_pair(acc, ahi, bhi, idesc, 1u);
            }
            tc5::mma_commit_pair(empty0 + 8 * s);
          }
          tc5::mma_commit_pair(tfull0 + 8 * b);
        }
      }
      tc5::mma_commit_pair(done);
    }
    if (lane == 0) tc5::mbar_wait_cluster(done, 0, &g_tma_error);
    __syncwarp();
  } else {
    // ---- epilogue warps (both CTAs) -----------------------------------------------------
    const int e = warp - 2;
    const int quad = warp & 3;       // TMEM lanes 32 quad .. 32 quad + 31
    const int cg = e >> 2;           // column group: 16-wide groups cg + (kEpiW / 4) q
    float* w2s = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 256);
    if constexpr (EPI_KIND == 0) {
      if (el.w2_stride > 0) {
        for (int i = threadIdx.x - 64; i < el.N * el.w2_stride; i += P::kEpiW * 32) {
          const int kk = i / el.w2_stride, c = i % el.w2_stride;
          w2s[i] = c < el.n_o ? el.w2[(int64_t)kk * el.n_o + c] : 0.f;
        }
        asm volatile("bar.sync 1, %0;" ::"r"(P::kEpiW * 32) : "memory");
      }
    }
    const uint32_t tempty_leader = tc5::mapa(tempty0, 0);
    // the warp's 2 KB staging block for TMA stores (32 rows x 16 Float32)
    float* stage = w2s + e * 512;
    const uint32_t stage_s = smem_u32(stage);
    int chain = 0;
    bool ok = true;
    for (int t = pair; t < total && ok; t += npairs) {
      const PairUnit u = pair_unit<TN>(t, g);
      const int kbeg = u.slice * g.k_slice;
      const int kend = min(g.K, kbeg + g.k_slice);
      const int nkb = kend > kbeg ? (kend - kbeg + BK - 1) / BK : 0;
      const int nch = nkb > 0 ? (nkb + g.chain - 1) / g.chain : 1;
      const int m = u.m0 + (int)rank * BM + quad * 32 + lane;
      constexpr int GS = P::kEpiW / 4;
      float sum[4][16];
#pragma unroll
      for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int i = 0; i < 16; ++i) sum[q][i] = 0.f;
      for (int ch = 0; ch < nch; ++ch, ++chain) {
        const int b = chain % NACC;
        ok = tc5::mbar_wait_cluster(tfull0 + 8 * b, (uint32_t)(chain / NACC) & 1u, &g_tma_error);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        if (nkb > 0) {
          const uint32_t base = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(b * TN);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            // columns past the MMAs' width hold nothing of this tile (uniform per warp)
            if ((cg + GS * q) * 16 < u.n_mma) {
              float v[16];
              tmem_ld16(base + (uint32_t)((cg + GS * q) * 16), v);
#pragma unroll
              for (int i = 0; i < 16; ++i) sum[q][i] += v[i];
            }
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) tc5::mbar_arrive_remote(tempty_leader + 8 * b);
      }
      if (!ok) break;
      if constexpr (P::kTmaOut) {
        // the warp's 32 rows x 16 columns at a time through its shared-memory
        // block, written (h, W1b slices) or added (xb) by one TMA operation
        const int row0 = u.m0 + (int)rank * BM + quad * 32;
        const int M = EPI_KIND == 0 ? el.M : EPI_KIND == 1 ? ea.M : ep.M;
        const int N = EPI_KIND == 0 ? el.N : EPI_KIND == 1 ? ea.N : ep.N;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int nn = u.n0 + (cg + GS * q) * 16;
          if (nn >= N || row0 >= M) continue;   // nothing of the box is inside (uniform)
          float v[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            if constexpr (EPI_KIND == 0)
              v[i] = (nn + i < N) ? tanhf(sum[q][i] + __ldg(el.b1 + nn + i)) : 0.f;
            else
              v[i] = sum[q][i];
          }
          // the block's previous store has been read out of shared memory
          if (lane == 0) tc5::bulk_wait_read();
          __syncwarp();
          float4* row = reinterpret_cast<float4*>(stage + lane * 16);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            row[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          tc5::fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            if constexpr (EPI_KIND == 0) tc5::tma_store_2d(&out, stage_s, nn, row0);
            else if constexpr (EPI_KIND == 1) tc5::tma_reduce_add_2d(&out, stage_s, nn, row0);
            else tc5::tma_store_3d(&out, stage_s, nn, row0, u.slice);
            tc5::bulk_commit();
          }
        }
      } else {
        epi_tile<EPI_KIND, NO, GS>(sum, m, u.n0, cg, u.slice, el, ea, ep, w2s);
      }
    }
    if constexpr (P::kTmaOut) {
      if (lane == 0) tc5::bulk_wait();   // every store of this warp has landed
      __syncwarp();
    }
  }

  // ---- teardown: neither CTA leaves (or frees TMEM) while the pair still works ----------
  tc_fence_before();
  __syncthreads();
  tc5::cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tc5::tmem_dealloc_pair(tmem, kTmemCols);
  }
}

// ---- host: tensor maps ---------------------------------------------------------------
// Row-major Float32 plane of rows x cols (row pitch `ld` elements), box of
// box_c (inner, along cols) x box_r, 128-byte swizzle with 16-byte chunks
// (K-major operands) or 32-byte chunks (MN-major operands), zero fill outside.
stade_status make_map(CUtensorMap* map, const float* base, int64_t rows, int64_t cols, int64_t ld,
                      uint32_t box_c, uint32_t box_r, bool chunk32) {
  const int64_t dims[2] = {cols, rows}, pitch[1] = {ld};
  const uint32_t box[2] = {box_c, box_r};
  return tc5::make_map_f32(map, base, 2, dims, pitch, box, chunk32);
}

// An operand of the contraction held as hi / lo planes. mn = false: rows are
// M (or N), columns are K (K contiguous). mn = true: rows are K, columns are
// M (or N).
struct Operand {
  const float *hi, *lo;
  int64_t rows, cols, ld;
  bool mn;
};

stade_status operand_maps(const Operand& o, CUtensorMap* hi, CUtensorMap* lo) {
  const uint32_t bc = 32, br = o.mn ? 32u : 128u;
  stade_status st = make_map(hi, o.hi, o.rows, o.cols, o.ld, bc, br, o.mn);
  if (st != STADE_OK) return st;
  return make_map(lo, o.lo, o.rows, o.cols, o.ld, bc, br, o.mn);
}

using tc5::sm_count;

template <int EPI_KIND, int NO>
stade_status run(const Operand& A, const Operand& B, Geometry g, const EpiTanhLogits& el,
                 const EpiAccumulate& ea, const EpiPartial& ep, cudaStream_t s) {
  CUtensorMap ah, al, bh, bl;
  stade_status st = operand_maps(A, &ah, &al);
  if (st != STADE_OK) return st;
  st = operand_maps(B, &bh, &bl);
  if (st != STADE_OK) return st;
  const int smem = kSmemBytes + (EPI_KIND == 0 && el.w2_stride > 0 ? kW2SmemBytes : 0);
  STADE_CUDA(cudaFuncSetAttribute(tma_gemm_kernel<EPI_KIND, NO>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const int total = g.m_tiles * g.n_tiles * g.slices;
  const int grid = total < sm_count() ? total : sm_count();
  tma_gemm_kernel<EPI_KIND, NO><<<grid, kThreads, smem, s>>>(ah, al, bh, bl, g, el, ea, ep);
  STADE_CHECK_LAUNCH();
  return STADE_OK;
}

// Tile choice (STADE_TMA_PAIR): 0 one CTA per 128 x 128 tile; 1 CTA pairs
// with 256 x 128 tiles for the forward and input-gradient contractions; 2 CTA
// pairs with 256 x 256 tiles for those two; 3 (the default) the same and the
// weight gradient on 256 x 256 pairs too (hidden units as rows, inputs as
// columns).
// Why pairs of 256 x 256: one CTA's 128 x 128 tile reads 96 KB of operands
// out of shared memory per K block for its 12 MMAs while TMA writes 64 KB in,
// ~1250 cycles of shared-memory traffic against 768 cycles of TF32 MMA, so
// the tensor pipe idles ~40 % (measured 51-65 % busy). A 2-SM 256 x 256 tile
// has each SM read 144 KB and take 64 KB in per 1536 MMA cycles (~94 %).
// Measured, C2 at 65,536 samples (ms, one CTA per tile -> pairs): forward
// 0.273 -> 0.210, weight gradient 0.281 -> 0.249, input gradient 0.301 ->
// 0.246.
int pair_mode() {
  const char* e = std::getenv("STADE_TMA_PAIR");
  if (e && e[0] >= '0' && e[0] <= '3' && e[1] == 0) return e[0] - '0';
  return 3;
}
int pair_width() {
  const int m = pair_mode();
  return m == 1 ? 128 : m >= 2 ? 256 : 0;
}

template <int EPI_KIND, int NO, int TN>
stade_status run_pair(const Operand& A, const Operand& B, Geometry g, const EpiTanhLogits& el,
                      const EpiAccumulate& ea, const EpiPartial& ep, cudaStream_t s) {
  using P = PairTile<TN>;
  CUtensorMap ah, al, bh, bl;
  stade_status st = operand_maps(A, &ah, &al);
  if (st != STADE_OK) return st;
  if (B.mn) {
    st = operand_maps(B, &bh, &bl);
  } else {
    st = make_map(&bh, B.hi, B.rows, B.cols, B.ld, 32, P::kBHalf, false);
    if (st == STADE_OK) st = make_map(&bl, B.lo, B.rows, B.cols, B.ld, 32, P::kBHalf, false);
  }
  if (st != STADE_OK) return st;
  g.m_tiles = (g.M + 2 * BM - 1) / (2 * BM);
  g.n_tiles = (g.N + TN - 1) / TN;
  // the output as TMA stores see it: boxes of 16 columns x 32 rows (x 1 slice)
  CUtensorMap om = ah;   // unused by 128-wide tiles
  if constexpr (P::kTmaOut) {
    const uint32_t box[3] = {16, 32, 1};
    if constexpr (EPI_KIND == 0) {
      const int64_t d[2] = {el.N, el.M}, pitch[1] = {el.ld};
      st = tc5::make_out_map_f32(&om, el.h, 2, d, pitch, box);
    } else if constexpr (EPI_KIND == 1) {
      const int64_t d[2] = {ea.N, ea.M}, pitch[1] = {ea.ld};
      st = tc5::make_out_map_f32(&om, ea.out, 2, d, pitch, box);
    } else {
      const int64_t d[3] = {ep.N, ep.M, g.slices};
      const int64_t pitch[2] = {ep.N, (int64_t)ep.M * ep.N};
      st = tc5::make_out_map_f32(&om, ep.part, 3, d, pitch, box);
    }
    if (st != STADE_OK) return st;
  }
  const int smem = P::kSmem + P::kStageOutBytes +
                   (EPI_KIND == 0 && el.w2_stride > 0 ? kW2SmemBytes : 0);
  auto kern = tma_gemm_pair_kernel<EPI_KIND, NO, TN>;
  STADE_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  const int total = g.m_tiles * g.n_tiles * g.slices;
  const int pairs = total < sm_count() / 2 ? total : sm_count() / 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(P::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  STADE_CUDA(cudaLaunchKernelEx(&cfg, kern, ah, al, bh, bl, om, g, el, ea, ep));
  count_launch();
  return STADE_OK;
}

Geometry geometry(int M, int N, int K, int slices, bool a_mn, bool b_mn) {
  Geometry g;
  g.M = M; g.N = N; g.K = K;
  g.m_tiles = (M + BM - 1) / BM;
  g.n_tiles = (N + BN - 1) / BN;
  const int kblocks = (K + BK - 1) / BK;
  const int per = slices > 1 ? (kblocks + slices - 1) / slices : kblocks;
  g.k_slice = (per > 0 ? per : 1) * BK;
  g.slices = K > 0 ? (K + g.k_slice - 1) / g.k_slice : 1;
  g.a_mn = a_mn; g.b_mn = b_mn;
  g.chain = tc5::tc_chain_blocks(kChainBlocks);
  return g;
}

// Slices of the W1b contraction (K = samples). Every (tile, slice) unit costs
// the same, and the persistent grid takes them in waves of one per SM, so the
// slice count minimises waves x K blocks per slice (the busiest SM's work),
// plus a small charge per slice for the partial it writes and the finish pass
// reads; at least 16 K blocks per slice. 784 x 512 over 65,536 samples: 28
// tiles x 21 slices = 588 units, 4 waves 99 % full (22 slices left 616 units:
// 5 waves, the last 16 % full).
int w1b_slices(int S, int I, int H) {
  const int tiles = ((I + BM - 1) / BM) * ((H + BN - 1) / BN);
  const int kblocks = (S + BK - 1) / BK;
  const int sms = tc5::sm_count();
  int best = 1;
  double best_cost = 0.0;
  for (int sl = 1; sl <= 64; ++sl) {
    const int per = (kblocks + sl - 1) / sl;
    if (sl > 1 && per < 16) break;
    const int slices = (kblocks + per - 1) / per;
    const int waves = (tiles * slices + sms - 1) / sms;
    // one partial tile (128 x 128 Float32 written and read) ~ the traffic of
    // 2 K blocks of operands
    const double cost = (double)waves * per + (slices > 1 ? 2.0 * slices * tiles / sms : 0.0);
    if (sl == 1 || cost < best_cost) {
      best = sl;
      best_cost = cost;
    }
  }
  return best;
}

// Slices of a split-K contraction on 256 x TN CTA-pair tiles, from the same
// kind of cost model: the pairs walk the (tile, slice) units with a stride of
// the pair count, a ragged column tile costs its MMA width's share of a full
// one, and the busiest pair's K blocks (plus a charge of 4 K blocks per
// partial tile written and read back) is minimised; at least 16 K blocks per
// slice.
template <int TN>
int pair_slices(int M, int N, int K, bool b_mn) {
  const int m_tiles = (M + 2 * BM - 1) / (2 * BM), n_tiles = (N + TN - 1) / TN;
  const int n_full = N / TN, tiles = m_tiles * n_tiles;
  const int kblocks = (K + BK - 1) / BK;
  const int pairs = tc5::sm_count() / 2;
  const int rag = N - n_full * TN;
  const double rag_cost =
      rag == 0 ? 1.0 : (double)(b_mn ? (rag + 63) / 64 * 64 : (rag + 31) / 32 * 32) / TN;
  int best = 1;
  double best_cost = 0.0;
  std::vector<double> load(pairs > 0 ? pairs : 1);
  for (int sl = 1; sl <= 128; ++sl) {
    const int per = (kblocks + sl - 1) / sl;
    if (sl > 1 && per < 16) break;
    const int slices = (kblocks + per - 1) / per;
    std::fill(load.begin(), load.end(), 0.0);
    for (int t = 0; t < tiles * slices; ++t) {
      const int slice = t / tiles, r = t % tiles;
      const int kb = std::min(per, kblocks - slice * per);
      load[t % load.size()] += kb * (r < m_tiles * n_full ? 1.0 : rag_cost);
    }
    const double busiest = *std::max_element(load.begin(), load.end());
    const double cost = busiest + (slices > 1 ? 4.0 * slices * tiles / load.size() : 0.0);
    if (sl == 1 || cost < best_cost) {
      best = sl;
      best_cost = cost;
    }
  }
  return best;
}

// The lo plane of an array that serves as its own hi plane: the tensor core
// reads just the top 19 bits of a Float32 operand (kind::tf32), so the array
// itself is its (truncated) hi plane and lo = rn(a - trunc(a)) completes it.
// Two arrays' lo planes in one launch: blocks [0, nb0) take the first, the
// rest the second (W1's 0.4 M elements ride along with x's 51 M).
__global__ void split_lo2_kernel(const float* __restrict__ a0, float* __restrict__ lo0, int64_t n0,
                                 const float* __restrict__ a1, float* __restrict__ lo1, int64_t n1,
                                 int nb0) {
  const bool second = (int)blockIdx.x >= nb0;
  const float* a = second ? a1 : a0;
  float* lo = second ? lo1 : lo0;
  const int64_t n = second ? n1 : n0;
  const int64_t b = second ? blockIdx.x - nb0 : blockIdx.x;
  const int64_t nb = second ? (int64_t)gridDim.x - nb0 : nb0;
  const int64_t n4 = n / 4;
  for (int64_t i = b * blockDim.x + threadIdx.x; i < n4; i += nb * blockDim.x) {
    const float4 v = reinterpret_cast<const float4*>(a)[i];
    float4 l;
    l.x = tc5::tf32_lo_of_own(v.x);
    l.y = tc5::tf32_lo_of_own(v.y);
    l.z = tc5::tf32_lo_of_own(v.z);
    l.w = tc5::tf32_lo_of_own(v.w);
    reinterpret_cast<float4*>(lo)[i] = l;
  }
  for (int64_t i = n4 * 4 + b * blockDim.x + threadIdx.x; i < n; i += nb * blockDim.x)
    lo[i] = tc5::tf32_lo_of_own(a[i]);
}

__global__ void w1b_finish_kernel(const float* __restrict__ part, int slices, int64_t MN,
                                  float* __restrict__ w1b) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= MN) return;
  float acc = 0.f;
  acc = ordered_sum(part + e, slices, MN);
  w1b[e] += acc;
}

// w1b[i][h] += sum over slices of part[slice][h][i], in slice order: the pair
// form of the weight gradient has hidden units as rows. 32 x 32 tiles through
// shared memory, so both the partial reads and the w1b updates are coalesced.
__global__ void w1b_finish_t_kernel(const float* __restrict__ part, int slices, int H, int I,
                                    float* __restrict__ w1b) {
  __shared__ float tile[32][33];
  const int i0 = blockIdx.x * 32, h0 = blockIdx.y * 32;
  const int64_t plane = (int64_t)H * I;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int h = h0 + r, i = i0 + threadIdx.x;
    tile[r][threadIdx.x] =
        (h < H && i < I) ? ordered_sum(part + (int64_t)h * I + i, slices, plane) : 0.f;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int i = i0 + r, h = h0 + threadIdx.x;
    if (i < I && h < H) w1b[(int64_t)i * H + h] += tile[threadIdx.x][r];
  }
}

}  // namespace tma

// ---- entry points used by mlp2_ce -------------------------------------------------------
stade_status tma_split_lo2(const float* a0, float* lo0, int64_t n0, const float* a1, float* lo1,
                           int64_t n1, cudaStream_t s) {
  auto blocks_for = [](int64_t n) {
    int64_t b = (n / 4 + 255) / 256;
    if (b > 148 * 16) b = 148 * 16;
    return (int)(b < 1 ? 1 : b);
  };
  const int nb0 = blocks_for(n0), nb1 = blocks_for(n1);
  tma::split_lo2_kernel<<<nb0 + nb1, 256, 0, s>>>(a0, lo0, n0, a1, lo1, n1, nb0);
  STADE_CHECK_LAUNCH();
  return STADE_OK;
}

// Slices of the weight gradient in the current tile mode (the pair form runs
// hidden units as rows, inputs as columns).
static int w1b_slice_count(int64_t n_s, int64_t n_i, int64_t n_h) {
  if (tma::pair_mode() == 3) return tma::pair_slices<256>((int)n_h, (int)n_i, (int)n_s, true);
  return tma::w1b_slices((int)n_s, (int)n_i, (int)n_h);
}

size_t tma_w1b_part_floats(int64_t n_s, int64_t n_i, int64_t n_h) {
  return (size_t)w1b_slice_count(n_s, n_i, n_h) * (size_t)n_i * (size_t)n_h;
}

stade_status tma_forward_tanh_logits(const float* x_hi, const float* x_lo, const float* w1_hi,
                                     const float* w1_lo, const float* b1, const float* w2,
                                     float* h, float* zpart, int S, int I, int H, int O,
                                     cudaStream_t s) {
  // A[m = sample, k = input]: x, K-major. B[n = hidden, k = input] = w1[k, n]: MN-major.
  tma::Operand A{x_hi, x_lo, S, I, I, false};
  tma::Operand B{w1_hi, w1_lo, I, H, H, true};
  tma::Geometry g = tma::geometry(S, H, I, 1, false, true);
  const int stride = (O + 3) / 4 * 4;
  const bool smem_w2 = zpart != nullptr && (int64_t)H * stride * 4 <= tma::kW2SmemBytes;
  tma::EpiTanhLogits el{h, b1, w2, zpart, H, S, H, O, 2, smem_w2 ? stride : 0};
  const int pw = tma::pair_width();
  // 256-wide tiles give each thread's logits partial a different column set:
  // they run only where the logits come from a pass of their own (and store
  // h with TMA, which needs it 16-byte aligned)
  if (pw == 256 && zpart == nullptr && tma::aligned16(h)) {
    if (O <= 16) return tma::run_pair<0, 16, 256>(A, B, g, el, {}, {}, s);
    return tma::run_pair<0, 32, 256>(A, B, g, el, {}, {}, s);
  }
  if (pw != 0) {
    if (O <= 16) return tma::run_pair<0, 16, 128>(A, B, g, el, {}, {}, s);
    return tma::run_pair<0, 32, 128>(A, B, g, el, {}, {}, s);
  }
  if (O <= 16) return tma::run<0, 16>(A, B, g, el, {}, {}, s);
  return tma::run<0, 32>(A, B, g, el, {}, {}, s);
}

stade_status tma_weight_grad(const float* x_hi, const float* x_lo, const float* s1b_hi,
                             const float* s1b_lo, float* w1b, float* part, int S, int I, int H,
                             cudaStream_t s) {
  if (tma::pair_mode() == 3) {
    // A[m = hidden, k = sample] = s1b[k, m]: MN-major. B[n = input, k = sample] = x[k, n]:
    // MN-major. part[slice][hidden][input], summed and transposed into w1b.
    tma::Operand A{s1b_hi, s1b_lo, S, H, H, true};
    tma::Operand B{x_hi, x_lo, S, I, I, true};
    tma::Geometry g = tma::geometry(H, I, S, w1b_slice_count(S, I, H), true, true);
    tma::EpiPartial ep{part, H, I};
    stade_status st = tma::run_pair<2, 1, 256>(A, B, g, {}, {}, ep, s);
    if (st != STADE_OK) return st;
    tma::w1b_finish_t_kernel<<<dim3(ceil_div_u(I, 32), ceil_div_u(H, 32)), dim3(32, 8), 0, s>>>(
        part, g.slices, H, I, w1b);
    STADE_CHECK_LAUNCH();
    return STADE_OK;
  }
  // A[m = input, k = sample] = x[k, m]: MN-major. B[n = hidden, k = sample] = s1b[k, n]: MN-major.
  tma::Operand A{x_hi, x_lo, S, I, I, true};
  tma::Operand B{s1b_hi, s1b_lo, S, H, H, true};
  tma::Geometry g = tma::geometry(I, H, S, tma::w1b_slices(S, I, H), true, true);
  tma::EpiPartial ep{part, I, H};
  stade_status st = tma::run<2, 1>(A, B, g, {}, {}, ep, s);
  if (st != STADE_OK) return st;
  const int64_t MN = (int64_t)I * H;
  tma::w1b_finish_kernel<<<ceil_div_u(MN, 256), 256, 0, s>>>(part, g.slices, MN, w1b);
  STADE_CHECK_LAUNCH();
  return STADE_OK;
}

stade_status tma_input_grad(const float* s1b_hi, const float* s1b_lo, const float* w1_hi,
                            const float* w1_lo, float* xb, int S, int I, int H, cudaStream_t s) {
  // A[m = sample, k = hidden] = s1b: K-major. B[n = input, k = hidden] = w1[n, k]: K-major.
  tma::Operand A{s1b_hi, s1b_lo, S, H, H, false};
  tma::Operand B{w1_hi, w1_lo, I, H, H, false};
  tma::Geometry g = tma::geometry(S, I, H, 1, false, false);
  tma::EpiAccumulate ea{xb, I, S, I};
  const int pw = tma::pair_width();
  // 256-wide tiles add into xb with TMA reductions: xb 16-byte aligned
  if (pw == 256 && tma::aligned16(xb)) return tma::run_pair<1, 1, 256>(A, B, g, {}, ea, {}, s);
  if (pw == 128) return tma::run_pair<1, 1, 128>(A, B, g, {}, ea, {}, s);
  return tma::run<1, 1>(A, B, g, {}, ea, {}, s);
}

}  // namespace stade

namespace stade {
bool tma_mlp_supported(int64_t n_s, int64_t n_i, int64_t n_h) {
  return n_s >= 1 && n_i >= 1 && n_h >= 1 && n_i % 4 == 0 && n_h % 4 == 0 &&
         n_s < (int64_t(1) << 30) && n_i < (1 << 20) && n_h < (1 << 20);
}

// two partial sums per 128-wide tile of hidden units (one per epilogue warp group)
int tma_logit_parts(int64_t n_h) { return 2 * (int)((n_h + tma::BN - 1) / tma::BN); }

// Reads and clears the TMA kernel's error word (-1 when it cannot be read).
int tma_take_error() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, tma::g_tma_error, sizeof(int)) != cudaSuccess) return -1;
  if (v) {
    const int zero = 0;
    cudaMemcpyToSymbol(tma::g_tma_error, &zero, sizeof(int));
  }
  return v;
}
}  // namespace stade

namespace stade {
int conv_tc_take_error();
int heat_take_error();

namespace {
__device__ int g_wait_check_out = 0;
// One thread waits on an mbarrier that nothing arrives on, with the wait loop
// of the tensor-core kernels and a limit of `cycles` SM clock cycles; the
// wait gives up, records the timeout in the TMA kernels' error word and the
// kernel returns. g_wait_check_out receives 1 if the wait returned false.
__global__ void bounded_wait_check_kernel(long long cycles) {
  __shared__ __align__(8) uint64_t bar;
  const uint32_t b = tc5::smem_u32(&bar);
  if (threadIdx.x == 0) tc5::mbar_init(b, 1);
  __syncthreads();
  if (threadIdx.x == 0)
    g_wait_check_out = tc5::mbar_wait_for(b, 0, &tma::g_tma_error, cycles) ? 0 : 1;
}
}  // namespace
}  // namespace stade

extern "C" stade_status stade_check_bounded_wait(int64_t wait_cycles, const stade_opts* opts) {
  using namespace stade;
  STADE_REQUIRE(wait_cycles >= 1000 && wait_cycles <= tc5::kWaitCycles,
                "check_bounded_wait: wait_cycles %lld outside [1000, %lld]",
                (long long)wait_cycles, (long long)tc5::kWaitCycles);
  cudaStream_t s = stream_of(opts);
  bounded_wait_check_kernel<<<1, 32, 0, s>>>((long long)wait_cycles);
  STADE_CHECK_LAUNCH();
  int host = 0;
  STADE_CUDA(cudaMemcpyFromSymbolAsync(&host, g_wait_check_out, sizeof(int), 0,
                                       cudaMemcpyDeviceToHost, s));
  STADE_CUDA(cudaStreamSynchronize(s));
  return host == 1 ? STADE_ETIMEDOUT : fail(STADE_ECUDA, "check_bounded_wait: the wait returned");
}

// The library's device error word: set when a bounded wait inside a
// tensor-core kernel ran out (the kernel then skipped its remaining work and
// returned). Reading clears it.
extern "C" int stade_device_error(void) {
  const int t = stade::tma_take_error();
  const int c = stade::conv_tc_take_error();
  const int h = stade::heat_take_error();
  if (t < 0 || c < 0 || h < 0) return -1;
  return t | c | h;
}
