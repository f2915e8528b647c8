// Tensor-core (tcgen05, 3xTF32) path of conv1d_relu_mse_b: the three
// contractions of the valid 1-D convolution adjoint as implicit GEMMs fed by
// TMA, no im2col buffer.
//
// Layouts (x[b][c][l], w[o][c][k], t / z / r and their shadows [b][o][t] are
// the generated signature's): two operand copies are made once per call, as
// TF32 hi / lo planes (hi = low 13 mantissa bits cleared, lo = v - hi exact):
//   xT[b][l][c]  x with channels innermost;
//   Wf[k][o][c]  w with taps outermost;
// and the forward's epilogue writes the reverse seed g = dloss/dz directly as
// planes gT[b][t][o]. A shift of the convolution by tap k then moves a TMA
// box along a row coordinate (l + k, l - k), which has no alignment rule and
// may start outside the tensor (zero fill), never along the 16-byte-aligned
// innermost coordinate.
//
//   forward  D[t][o] = sum_k sum_c xT[b][t+k][c] Wf[k][o][c]      M = t, N = o
//            epilogue: z, r = max(z, 0), loss partial, tb, g (generated
//            statement order and roundings, as the CUDA-core path)
//   wgrad    D[o][(k,c)] = sum_{b,t} gT[b][t][o] xT[b][t+k][c]   split over b
//   xgrad    D[l][c] = sum_k sum_o gT[b][l-k][o] Wf[k][o][c]     xb += D
//
// Persistent kernel, one CTA per SM, warp-specialised as the mlp2_ce GEMMs:
// warp 0 issues the TMA loads into a 3-stage ring, warp 1 owns TMEM (four
// accumulators) and issues the MMAs, warps 2-9 drain the accumulators in
// chains of 4 K blocks into round-to-nearest register sums (the tensor core's
// Float32 accumulation error grows with chain length) and run the epilogue.
// Every wait is bounded; on timeout the kernel sets g_conv_error, stops,
// waits (bounded) for its own copies and MMAs, frees TMEM and returns.
#include "conv_tc.cuh"
#include "tcgen05.cuh"

namespace stade {
namespace convtc {

using namespace tc5;

constexpr int BM = 128, BK = 32, STAGES = 3;
constexpr int kEpiWarps = 8;
constexpr int kThreads = (2 + kEpiWarps) * 32;
constexpr int kPlane = BM * BK * 4;  // 16 KiB: one 128 x 32 plane tile
constexpr int kStageBytes = 4 * kPlane;
constexpr int kSmemBytes = STAGES * kStageBytes + 1024 + 256;
constexpr int kChainBlocks = 4;
// TMEM accumulators the MMAs rotate through (up to kAccBufs - 1 chains ahead
// of the epilogue warps)
constexpr int kAccBufs = 4;
constexpr int kBarWords = 2 * STAGES + 2 * kAccBufs + 1;  // full, empty, tfull, tempty, done
static_assert(kBarWords * 8 + 4 + 4 * kEpiWarps <= 256, "barrier block overflow");

__device__ int g_conv_error = 0;

struct Geo {
  int B, C, L, O, K, Lo;
  int cblk, oblk, tblk, cpad, nw;  // ceil(C/32), ceil(O/32), ceil(Lo/32), C rounded to 32, K cpad
  int m_tiles, n_tiles, slices, bps;
  int chain;  // K blocks per TMEM accumulation chain
};

struct FwdOut {  // the forward epilogue's arrays
  float *z, *r, *zb, *rb, *tb, *g_hi, *g_lo, *loss_part;
  const float *t, *lossb;
  float inv_n;
};

template <int MODE>
struct Cfg;
template <>
struct Cfg<0> {  // forward
  static constexpr int BN = 128;
  static constexpr bool a_mn = false, b_mn = false;
};
template <>
struct Cfg<1> {  // weight gradient
  static constexpr int BN = 128;
  static constexpr bool a_mn = true, b_mn = true;
};
template <>
struct Cfg<2> {  // input gradient
  static constexpr int BN = 64;
  static constexpr bool a_mn = false, b_mn = true;
};

struct Tile {
  int b, m0, n0, slice, nkb, blo;
};

template <int MODE>
__device__ __forceinline__ Tile decode(const Geo& g, int t) {
  Tile x;
  const int per = g.m_tiles * g.n_tiles;
  if (MODE == 1) {
    x.slice = t / per;
    const int r = t % per;
    x.m0 = (r / g.n_tiles) * BM;
    x.n0 = (r % g.n_tiles) * Cfg<MODE>::BN;
    x.blo = x.slice * g.bps;
    const int bhi = min(g.B, x.blo + g.bps);
    x.nkb = bhi > x.blo ? (bhi - x.blo) * g.tblk : 0;
    x.b = x.blo;
  } else {
    x.b = t / per;
    const int r = t % per;
    x.m0 = (r / g.n_tiles) * BM;
    x.n0 = (r % g.n_tiles) * Cfg<MODE>::BN;
    x.slice = 0;
    x.blo = x.b;
    x.nkb = MODE == 0 ? g.K * g.cblk : g.K * g.oblk;
  }
  return x;
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1)
conv_tc_kernel(const __grid_constant__ CUtensorMap a_hi, const __grid_constant__ CUtensorMap a_lo,
               const __grid_constant__ CUtensorMap b_hi, const __grid_constant__ CUtensorMap b_lo,
               Geo g, FwdOut fo, float* __restrict__ wpart, float* __restrict__ xb) {
  constexpr int BN = Cfg<MODE>::BN;
  constexpr bool A_MN = Cfg<MODE>::a_mn, B_MN = Cfg<MODE>::b_mn;
  constexpr int kBPlane = BN * BK * 4;
  constexpr uint32_t kTx = 2 * kPlane + 2 * kBPlane;
  constexpr uint32_t kTmemCols = kAccBufs * BN;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t pad = (1024u - (raw & 1023u)) & 1023u;
  uint8_t* tiles = smem_raw + pad;
  uint64_t* bars = reinterpret_cast<uint64_t*>(tiles + STAGES * kStageBytes);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + kBarWords);
  float* red = reinterpret_cast<float*>(tmem_slot + 1);  // kEpiWarps floats
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES);
  const uint32_t tfull0 = smem_u32(bars + 2 * STAGES);
  const uint32_t tempty0 = smem_u32(bars + 2 * STAGES + kAccBufs);
  const uint32_t done = smem_u32(bars + 2 * STAGES + 2 * kAccBufs);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total = g.m_tiles * g.n_tiles * g.slices;

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
  if (warp == 1) tmem_alloc(smem_u32(tmem_slot), kTmemCols);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer -------------------------------------------------------------
      int kb_all = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        const Tile tl = decode<MODE>(g, t);
        for (int kb = 0; kb < tl.nkb; ++kb, ++kb_all) {
          const int s = kb_all % STAGES;
          const uint32_t ph = (uint32_t)(kb_all / STAGES) & 1u;
          if (!mbar_wait(empty0 + 8 * s, ph ^ 1u, &g_conv_error)) { ok = false; break; }
          const uint32_t st = smem_u32(tiles + s * kStageBytes);
          const uint32_t sb = st + 2 * kPlane;
          const uint32_t fb = full0 + 8 * s;
          mbar_arrive_tx(fb, kTx);
          if (MODE == 0) {
            const int kk = kb / g.cblk, c0 = (kb % g.cblk) * BK;
            tma_load_3d(st, &a_hi, c0, tl.m0 + kk, tl.b, fb);
            tma_load_3d(st + kPlane, &a_lo, c0, tl.m0 + kk, tl.b, fb);
            tma_load_3d(sb, &b_hi, c0, tl.n0, kk, fb);
            tma_load_3d(sb + kBPlane, &b_lo, c0, tl.n0, kk, fb);
          } else if (MODE == 1) {
            const int b = tl.blo + kb / g.tblk, t0 = (kb % g.tblk) * BK;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              tma_load_3d(st + q * 4096, &a_hi, tl.m0 + 32 * q, t0, b, fb);
              tma_load_3d(st + kPlane + q * 4096, &a_lo, tl.m0 + 32 * q, t0, b, fb);
            }
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int n = tl.n0 + 32 * q;
              const int kk = n / g.cpad, c0 = n % g.cpad;
              tma_load_3d(sb + q * 4096, &b_hi, c0, t0 + kk, b, fb);
              tma_load_3d(sb + kBPlane + q * 4096, &b_lo, c0, t0 + kk, b, fb);
            }
          } else {
            const int kk = kb / g.oblk, o0 = (kb % g.oblk) * BK;
            tma_load_3d(st, &a_hi, o0, tl.m0 - kk, tl.b, fb);
            tma_load_3d(st + kPlane, &a_lo, o0, tl.m0 - kk, tl.b, fb);
#pragma unroll
            for (int q = 0; q < BN / 32; ++q) {
              tma_load_3d(sb + q * 4096, &b_hi, tl.n0 + 32 * q, o0, kk, fb);
              tma_load_3d(sb + kBPlane + q * 4096, &b_lo, tl.n0 + 32 * q, o0, kk, fb);
            }
          }
        }
      }
      for (int i = 0; i < STAGES && i < kb_all; ++i) {
        const int last = kb_all - 1 - i;
        mbar_wait(full0 + 8 * (last % STAGES), (uint32_t)(last / STAGES) & 1u, &g_conv_error);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer -----------------------------------------------------------------
      const uint32_t idesc = idesc_tf32(BM, BN, A_MN, B_MN);
      const uint32_t a_lbo = A_MN ? 4096u : 16u, a_sbo = A_MN ? 512u : 1024u;
      const uint32_t b_lbo = B_MN ? 4096u : 16u, b_sbo = B_MN ? 512u : 1024u;
      const uint32_t a_lay = A_MN ? 1u : 2u, b_lay = B_MN ? 1u : 2u;
      const uint32_t a_step = A_MN ? 1024u : 32u, b_step = B_MN ? 1024u : 32u;
      int kb_all = 0, chain = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
        const Tile tl = decode<MODE>(g, t);
        const int nch = tl.nkb > 0 ? (tl.nkb + g.chain - 1) / g.chain : 1;
        for (int ch = 0; ch < nch && ok; ++ch, ++chain) {
          const int b = chain % kAccBufs;
          const uint32_t acc = tmem + (uint32_t)(b * BN);
          if (!mbar_wait(tempty0 + 8 * b, ((uint32_t)(chain / kAccBufs) & 1u) ^ 1u, &g_conv_error)) {
            ok = false;
            break;
          }
          fence_after();
          const int kb0 = ch * g.chain, kb1 = min(tl.nkb, kb0 + g.chain);
          for (int kb = kb0; kb < kb1; ++kb, ++kb_all) {
            const int s = kb_all % STAGES;
            const uint32_t ph = (uint32_t)(kb_all / STAGES) & 1u;
            if (!mbar_wait(full0 + 8 * s, ph, &g_conv_error)) { ok = false; break; }
            fence_after();
            const uint32_t st = smem_u32(tiles + s * kStageBytes);
            const uint32_t sb = st + 2 * kPlane;
#pragma unroll
            for (int j = 0; j < BK / 8; ++j) {
              const uint64_t ahi = desc_sw128(st + a_step * j, a_lbo, a_sbo, a_lay);
              const uint64_t alo = desc_sw128(st + kPlane + a_step * j, a_lbo, a_sbo, a_lay);
              const uint64_t bhi = desc_sw128(sb + b_step * j, b_lbo, b_sbo, b_lay);
              const uint64_t blo = desc_sw128(sb + kBPlane + b_step * j, b_lbo, b_sbo, b_lay);
              mma_tf32(acc, ahi, blo, idesc, (kb != kb0 || j != 0) ? 1u : 0u);
              mma_tf32(acc, alo, bhi, idesc, 1u);
              mma_tf32(acc, ahi, bhi, idesc, 1u);
            }
            mma_commit(empty0 + 8 * s);
          }
          mma_commit(tfull0 + 8 * b);
        }
      }
      mma_commit(done);
      mbar_wait(done, 0, &g_conv_error);
    }
  } else {
    // ---- epilogue warps -------------------------------------------------------------
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    float lsum = 0.f;
    int chain = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total && ok; t += gridDim.x) {
      const Tile tl = decode<MODE>(g, t);
      const int nch = tl.nkb > 0 ? (tl.nkb + g.chain - 1) / g.chain : 1;
      float sum[BN / 32][16];
#pragma unroll
      for (int q = 0; q < BN / 32; ++q)
#pragma unroll
        for (int i = 0; i < 16; ++i) sum[q][i] = 0.f;
      for (int ch = 0; ch < nch; ++ch, ++chain) {
        const int b = chain % kAccBufs;
        ok = mbar_wait(tfull0 + 8 * b, (uint32_t)(chain / kAccBufs) & 1u, &g_conv_error);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        fence_after();
        if (tl.nkb > 0) {
          const uint32_t base = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(b * BN);
#pragma unroll
          for (int q = 0; q < BN / 32; ++q) {
            float v[16];
            tmem_ld16(base + (uint32_t)((half + 2 * q) * 16), v);
#pragma unroll
            for (int i = 0; i < 16; ++i) sum[q][i] += v[i];
          }
        }
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty0 + 8 * b);
      }
      if (!ok) break;
      const int m = tl.m0 + quad * 32 + lane;
      if (MODE == 0) {
        // m = output position t, columns = output channels o
        if (m < g.Lo) {
          const float lb = __ldg(fo.lossb);
#pragma unroll
          for (int q = 0; q < BN / 32; ++q) {
            const int o0 = tl.n0 + (half + 2 * q) * 16;
            const int64_t idx0 = ((int64_t)tl.b * g.O + o0) * g.Lo + m;
            float gv[16];
            // 8 columns at a time: their loads first (nothing here aliases
            // another thread's elements), then the arithmetic and the stores
#pragma unroll
            for (int h8 = 0; h8 < 16; h8 += 8) {
              float tv[8], rbv[8], zbv[8], tbv[8];
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                const int64_t idx = idx0 + (int64_t)(h8 + i) * g.Lo;
                const bool in = o0 + h8 + i < g.O;
                tv[i] = in ? __ldg(fo.t + idx) : 0.f;
                rbv[i] = in ? fo.rb[idx] : 0.f;
                zbv[i] = in ? fo.zb[idx] : 0.f;
                tbv[i] = in ? fo.tb[idx] : 0.f;
              }
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                gv[h8 + i] = 0.f;
                if (o0 + h8 + i < g.O) {
                  const int64_t idx = idx0 + (int64_t)(h8 + i) * g.Lo;
                  const float a = sum[q][h8 + i];
                  const float rv = a > 0.0f ? a : (a < 0.0f ? 0.0f : (a == 0.0f ? 0.0f : a));
                  const float dlt = __fadd_rn(rv, -tv[i]);
                  lsum = __fadd_rn(lsum, __fmul_rn(fo.inv_n, __fmul_rn(dlt, dlt)));
                  const float cse1 = __fmul_rn(__fmul_rn(fo.inv_n, __fmul_rn(2.0f, dlt)), lb);
                  const float rbt = __fadd_rn(rbv[i], cse1);
                  const float sg = a > 0.0f ? 1.0f : (a < 0.0f ? -1.0f : a);
                  gv[h8 + i] = __fadd_rn(__fmul_rn(0.5f * (1.0f + sg), rbt), zbv[i]);
                  fo.z[idx] = a;
                  fo.r[idx] = rv;
                  fo.tb[idx] = __fadd_rn(tbv[i], -cse1);
                  if (rbv[i] != 0.0f) fo.rb[idx] = 0.0f;
                  if (zbv[i] != 0.0f) fo.zb[idx] = 0.0f;
                }
              }
            }
            const int64_t gi = ((int64_t)tl.b * g.Lo + m) * g.O + o0;
            if (o0 + 16 <= g.O) {
#pragma unroll
              for (int i = 0; i < 16; i += 4) {
                float4 h, l;
                tf32_split(gv[i], h.x, l.x);
                tf32_split(gv[i + 1], h.y, l.y);
                tf32_split(gv[i + 2], h.z, l.z);
                tf32_split(gv[i + 3], h.w, l.w);
                *reinterpret_cast<float4*>(fo.g_hi + gi + i) = h;
                *reinterpret_cast<float4*>(fo.g_lo + gi + i) = l;
              }
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                if (o0 + i < g.O) tf32_split(gv[i], fo.g_hi[gi + i], fo.g_lo[gi + i]);
              }
            }
          }
        }
      } else if (MODE == 1) {
        // m = output channel o, columns n = (k, c) of the padded layout
        if (m < g.O) {
#pragma unroll
          for (int q = 0; q < BN / 32; ++q) {
            const int n0 = tl.n0 + (half + 2 * q) * 16;
            if (n0 < g.nw) {
              float* p = wpart + ((int64_t)tl.slice * g.O + m) * g.nw + n0;
#pragma unroll
              for (int i = 0; i < 16; i += 4)
                *reinterpret_cast<float4*>(p + i) =
                    make_float4(sum[q][i], sum[q][i + 1], sum[q][i + 2], sum[q][i + 3]);
            }
          }
        }
      } else {
        // m = input position l, columns = channels c: xb[b][c][l] += D
        if (m < g.L) {
#pragma unroll
          for (int q = 0; q < BN / 32; ++q) {
            const int c0 = tl.n0 + (half + 2 * q) * 16;
            float* p0 = xb + ((int64_t)tl.b * g.C + c0) * g.L + m;
            float old[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) old[i] = c0 + i < g.C ? p0[(int64_t)i * g.L] : 0.f;
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (c0 + i < g.C) p0[(int64_t)i * g.L] = old[i] + sum[q][i];
          }
        }
      }
    }
    if (MODE == 0) {
      // this CTA's loss partial, fixed order: warp sums, then warps 0..7
      float v = lsum;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, off));
      if (lane == 0) red[warp - 2] = v;
      asm volatile("bar.sync 1, %0;" ::"r"(kEpiWarps * 32) : "memory");
      if (warp == 2 && lane == 0) {
        float s = 0.f;
        for (int i = 0; i < kEpiWarps; ++i) s = __fadd_rn(s, red[i]);
        fo.loss_part[blockIdx.x] = s;
      }
    }
  }

  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---- operand preparation -------------------------------------------------------------
// xT[b][l][c] hi / lo from x[b][c][l]: 32 x 32 tiles through shared memory.
__global__ void __launch_bounds__(256)
xt_split_kernel(const float* __restrict__ x, float* __restrict__ hi, float* __restrict__ lo, int C,
                int L) {
  __shared__ float tile[32][33];
  const int l0 = blockIdx.x * 32, c0 = blockIdx.y * 32, b = blockIdx.z;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const float* xb = x + (int64_t)b * C * L;
#pragma unroll
  for (int j = 0; j < 32; j += 8) {
    const int c = c0 + ty + j, l = l0 + tx;
    tile[ty + j][tx] = (c < C && l < L) ? xb[(int64_t)c * L + l] : 0.f;
  }
  __syncthreads();
  const int64_t base = (int64_t)b * L * C;
#pragma unroll
  for (int j = 0; j < 32; j += 8) {
    const int l = l0 + ty + j, c = c0 + tx;
    if (l < L && c < C) {
      tf32_split(tile[tx][ty + j], hi[base + (int64_t)l * C + c], lo[base + (int64_t)l * C + c]);
    }
  }
}

// Wf[k][o][c] hi / lo from w[o][c][k].
__global__ void wf_split_kernel(const float* __restrict__ w, float* __restrict__ hi,
                                float* __restrict__ lo, int O, int C, int K) {
  const int64_t n = (int64_t)O * C * K;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(e % C);
    const int64_t r = e / C;
    const int o = (int)(r % O), k = (int)(r / O);
    tf32_split(w[((int64_t)o * C + c) * K + k], hi[e], lo[e]);
  }
}

// wb[o][c][k] += sum over slices of part[s][o][k cpad + c], slices in order.
__global__ void wgrad_finish_kernel(const float* __restrict__ part, int slices, Geo g,
                                    float* __restrict__ wb) {
  const int64_t n = (int64_t)g.O * g.C * g.K;
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= n) return;
  const int k = (int)(e % g.K);
  const int64_t r = e / g.K;
  const int c = (int)(r % g.C), o = (int)(r / g.C);
  const int64_t col = (int64_t)o * g.nw + (int64_t)k * g.cpad + c;
  const int64_t stride = (int64_t)g.O * g.nw;
  const float acc = ordered_sum(part + col, slices, stride);
  wb[e] += acc;
}

// ---- host ----------------------------------------------------------------------------
Geo base_geo(const ConvShape& sh) {
  Geo g{};
  g.chain = tc5::tc_chain_blocks(kChainBlocks);
  g.B = (int)sh.n_b; g.C = (int)sh.n_c; g.L = (int)sh.n_l; g.O = (int)sh.n_o; g.K = (int)sh.n_k;
  g.Lo = g.L - g.K + 1;
  g.cblk = (g.C + 31) / 32;
  g.oblk = (g.O + 31) / 32;
  g.tblk = (g.Lo + 31) / 32;
  g.cpad = g.cblk * 32;
  g.nw = g.K * g.cpad;
  return g;
}

Geo geo_fwd(const ConvShape& sh) {
  Geo g = base_geo(sh);
  g.m_tiles = (g.Lo + BM - 1) / BM;
  g.n_tiles = (g.O + 127) / 128;
  g.slices = g.B;
  g.bps = 1;
  return g;
}
Geo geo_wgrad(const ConvShape& sh) {
  Geo g = base_geo(sh);
  g.m_tiles = (g.O + BM - 1) / BM;
  g.n_tiles = (g.nw + 127) / 128;
  const int per = g.m_tiles * g.n_tiles;
  // about 5 tiles per SM in total, whole samples per slice
  int slices = (5 * sm_count() + per - 1) / per;
  if (slices > g.B) slices = g.B;
  if (slices < 1) slices = 1;
  g.bps = (g.B + slices - 1) / slices;
  g.slices = (g.B + g.bps - 1) / g.bps;
  return g;
}
Geo geo_xgrad(const ConvShape& sh) {
  Geo g = base_geo(sh);
  g.m_tiles = (g.L + BM - 1) / BM;
  g.n_tiles = (g.C + 63) / 64;
  g.slices = g.B;
  g.bps = 1;
  return g;
}

struct Ws {
  float *xt_hi, *xt_lo, *wf_hi, *wf_lo, *g_hi, *g_lo, *wpart, *loss_part;
};
template <class Alloc>
void layout(Alloc& a, Ws* w, const ConvShape& sh) {
  const int64_t nx = sh.n_b * sh.n_c * sh.n_l;
  const int64_t nw = sh.n_o * sh.n_c * sh.n_k;
  const int64_t ng = sh.n_b * sh.n_o * (sh.n_l - sh.n_k + 1);
  const Geo gw = geo_wgrad(sh);
  float* p[8];
  p[0] = a.template take<float>((size_t)nx);
  p[1] = a.template take<float>((size_t)nx);
  p[2] = a.template take<float>((size_t)nw);
  p[3] = a.template take<float>((size_t)nw);
  p[4] = a.template take<float>((size_t)ng);
  p[5] = a.template take<float>((size_t)ng);
  p[6] = a.template take<float>((size_t)gw.slices * gw.O * gw.nw);
  p[7] = a.template take<float>(1024);
  if (w) *w = Ws{p[0], p[1], p[2], p[3], p[4], p[5], p[6], p[7]};
}
struct SizeA {
  Sizer z;
  template <class T> T* take(size_t n) { z.take<T>(n); return nullptr; }
};
struct CarveA {
  Carver c;
  explicit CarveA(void* b) : c(b) {}
  template <class T> T* take(size_t n) { return c.take<T>(n); }
};

template <int MODE>
stade_status launch(const CUtensorMap& ah, const CUtensorMap& al, const CUtensorMap& bh,
                    const CUtensorMap& bl, const Geo& g, const FwdOut& fo, float* wpart, float* xb,
                    cudaStream_t s, int* grid_out) {
  STADE_CUDA(cudaFuncSetAttribute(conv_tc_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  kSmemBytes));
  const int total = g.m_tiles * g.n_tiles * g.slices;
  const int grid = total < sm_count() ? total : sm_count();
  if (grid_out) *grid_out = grid;
  if (grid <= 0) return STADE_OK;
  conv_tc_kernel<MODE><<<grid, kThreads, kSmemBytes, s>>>(ah, al, bh, bl, g, fo, wpart, xb);
  STADE_CHECK_LAUNCH();
  return STADE_OK;
}

}  // namespace convtc

bool conv_tc_supported(const ConvShape& sh) {
  const int64_t n_lo = sh.n_l - sh.n_k + 1;
  return sh.n_c % 4 == 0 && sh.n_o % 4 == 0 && n_lo >= 1 && sh.n_b <= (1 << 30) &&
         sh.n_l < (1 << 30) && sh.n_k <= 1024 && sh.n_c <= 4096 && sh.n_o <= 4096;
}

size_t conv_tc_workspace(const ConvShape& sh) {
  convtc::SizeA a;
  convtc::layout(a, nullptr, sh);
  return a.z.bytes();
}

stade_status conv_tc_run(const ConvShape& sh, float* loss, const float* lossb, const float* x,
                         float* xb, const float* w, float* wb, const float* t, float* tb, float* z,
                         float* zb, float* r, float* rb, void* ws, cudaStream_t s) {
  using namespace convtc;
  CarveA ca(ws);
  Ws W;
  layout(ca, &W, sh);
  const Geo gf = geo_fwd(sh), gw = geo_wgrad(sh), gx = geo_xgrad(sh);
  const int64_t B = sh.n_b, C = sh.n_c, L = sh.n_l, O = sh.n_o, K = sh.n_k, Lo = gf.Lo;
  // operand planes
  {
    PhaseScope ph("conv_split", s);
    const dim3 grid((unsigned)((L + 31) / 32), (unsigned)((C + 31) / 32), (unsigned)B);
    xt_split_kernel<<<grid, 256, 0, s>>>(x, W.xt_hi, W.xt_lo, (int)C, (int)L);
    STADE_CHECK_LAUNCH();
    wf_split_kernel<<<ceil_div_u(O * C * K, 256), 256, 0, s>>>(w, W.wf_hi, W.wf_lo, (int)O,
                                                                (int)C, (int)K);
    STADE_CHECK_LAUNCH();
  }
  // tensor maps: xT (c, l, b); Wf (c, o, k); gT (o, t, b)
  CUtensorMap xk_hi, xk_lo, xm_hi, xm_lo, wk_hi, wk_lo, wm_hi, wm_lo, gk_hi, gk_lo, gm_hi, gm_lo;
  {
    const int64_t dx[3] = {C, L, B}, px[2] = {C, L * C};
    const int64_t dw[3] = {C, O, K}, pw[2] = {C, O * C};
    const int64_t dg[3] = {O, Lo, B}, pg[2] = {O, Lo * O};
    const uint32_t kbox[3] = {32, 128, 1}, mbox[3] = {32, 32, 1};
    stade_status st = STADE_OK;
    auto mk = [&](CUtensorMap* m, const float* p, const int64_t* d, const int64_t* pt,
                  const uint32_t* bx, bool mn) {
      if (st == STADE_OK) st = make_map_f32(m, p, 3, d, pt, bx, mn);
    };
    mk(&xk_hi, W.xt_hi, dx, px, kbox, false);
    mk(&xk_lo, W.xt_lo, dx, px, kbox, false);
    mk(&xm_hi, W.xt_hi, dx, px, mbox, true);
    mk(&xm_lo, W.xt_lo, dx, px, mbox, true);
    mk(&wk_hi, W.wf_hi, dw, pw, kbox, false);
    mk(&wk_lo, W.wf_lo, dw, pw, kbox, false);
    mk(&wm_hi, W.wf_hi, dw, pw, mbox, true);
    mk(&wm_lo, W.wf_lo, dw, pw, mbox, true);
    mk(&gk_hi, W.g_hi, dg, pg, kbox, false);
    mk(&gk_lo, W.g_lo, dg, pg, kbox, false);
    mk(&gm_hi, W.g_hi, dg, pg, mbox, true);
    mk(&gm_lo, W.g_lo, dg, pg, mbox, true);
    if (st != STADE_OK) return st;
  }
  FwdOut fo{z, r, zb, rb, tb, W.g_hi, W.g_lo, W.loss_part, t, lossb,
            1.0f / (float)(B * O * Lo)};
  stade_status st;
  {
    PhaseScope ph("conv_fwd", s);
    int grid = 0;
    st = launch<0>(xk_hi, xk_lo, wk_hi, wk_lo, gf, fo, nullptr, nullptr, s, &grid);
    if (st == STADE_OK && grid > 0) st = launch_sum_to_scalar(W.loss_part, grid, loss, true, s);
  }
  if (st != STADE_OK) return st;
  {
    PhaseScope ph("conv_wgrad", s);
    st = launch<1>(gm_hi, gm_lo, xm_hi, xm_lo, gw, fo, W.wpart, nullptr, s, nullptr);
    if (st == STADE_OK) {
      wgrad_finish_kernel<<<ceil_div_u(O * C * K, 256), 256, 0, s>>>(W.wpart, gw.slices, gw, wb);
      STADE_CHECK_LAUNCH();
    }
  }
  if (st != STADE_OK) return st;
  {
    PhaseScope ph("conv_xgrad", s);
    st = launch<2>(gk_hi, gk_lo, wm_hi, wm_lo, gx, fo, nullptr, xb, s, nullptr);
  }
  return st;
}

int conv_tc_take_error() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, convtc::g_conv_error, sizeof(int)) != cudaSuccess) return -1;
  if (v) {
    const int zero = 0;
    cudaMemcpyToSymbol(convtc::g_conv_error, &zero, sizeof(int));
  }
  return v;
}

}  // namespace stade
