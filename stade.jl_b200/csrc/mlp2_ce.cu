// C2 mlp2_ce_b (Float32 adjoint) and C5 mlp2_ce_hv (Float64 HVP).
//
// Generated sweeps being replaced (restated in oracle.cc): the adjoint of a
// batch-loop kernel h = tanh(x W1 + b1), z = h W2 + b2, softmax
// cross-entropy, in the pattern of test/val-corpus/mlp1d_b.jl:5-78 (hidden
// and output layers) and transformer_b.jl:615-667 (softmax reverse), and its
// forward-over-reverse HVP as test/val-corpus/mlp1d_hv.jl.
//
// B200 mapping, per sweep:
//   1. s1 = x W1 (GEMM), epilogue h = tanh(s1 + b1)     [HVP: + s1d, hd]
//   2. per-sample head, one warp per sample: z, softmax, the whole reverse of
//      the loss and softmax, then hb = W2 g and s1b = (1 - h^2) hb, all in
//      registers; the generated code's tape of the row-max chain lives in
//      registers too.
//   3. W2b = h^T g, b2b = sum g: per-chunk partials, fixed-order sum.
//   4. W1b = x^T s1b (GEMM, split over samples, fixed-order slice sum) with
//      b1b = sum s1b fused as an extra row of ones in x^T.
//   5. xb += s1b W1^T (GEMM).
// The generated CUDA.jl port does 2-4 with atomics on every weight
// (cgen_device_assign, src/STADE.jl:11941); here nothing is atomic.
#include <cstdlib>
#include <cstring>
#include <type_traits>

#include "common.cuh"
#include "gemm_dmma.cuh"
#include "gemm_simt.cuh"
#include "tc_tma.cuh"
#include "tcgen05.cuh"

namespace stade {
namespace {

constexpr int kHeadWarps = 8;   // samples in flight per block
constexpr int kHvHeadWarps = 16;  // the same for the Float64 HVP head (one block per SM)
// Sum over the 32 lanes of a[0..15] (each lane its own sixteen values): four
// halving exchanges leave each lane pair one class's sum, class
// ((l >> 4) & 1) * 8 + ((l >> 3) & 1) * 4 + ((l >> 2) & 1) * 2 + ((l >> 1) & 1).
__device__ __forceinline__ double halving_sum16(double (&a)[16], int lane) {
#pragma unroll
  for (int w = 8, bit = 16; w >= 1; w >>= 1, bit >>= 1) {
    const bool upper = (lane & bit) != 0;
#pragma unroll
    for (int i = 0; i < w; ++i) {
      const double keep = upper ? a[i + w] : a[i];
      const double send = upper ? a[i] : a[i + w];
      a[i] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
    }
  }
  return a[0] + __shfl_xor_sync(0xffffffffu, a[0], 1);
}
// A lane that holds class c's sum after halving_sum16.
__device__ __forceinline__ int class_lane16(int c) {
  return (((c >> 3) & 1) << 4) | (((c >> 2) & 1) << 3) | (((c >> 1) & 1) << 2) | ((c & 1) << 1);
}
constexpr int kW2Chunk = 256;   // samples per W2b partial
constexpr int kW2ChunkHv = 64;  // samples per W2b / W2bd partial of the Float64 HVP

template <class T> __device__ __forceinline__ T dtanh(T x);
template <> __device__ __forceinline__ float dtanh(float x) { return tanhf(x); }
template <> __device__ __forceinline__ double dtanh(double x) { return tanh(x); }
template <class T> __device__ __forceinline__ T dexp(T x);
template <> __device__ __forceinline__ float dexp(float x) { return expf(x); }
template <> __device__ __forceinline__ double dexp(double x) { return exp(x); }
template <class T> __device__ __forceinline__ T dlog(T x);
template <> __device__ __forceinline__ float dlog(float x) { return logf(x); }
template <> __device__ __forceinline__ double dlog(double x) { return log(x); }
template <class T> __device__ __forceinline__ T dsign(T x) {
  return x > T(0) ? T(1) : (x < T(0) ? T(-1) : x);
}
// Julia's max: NaN wins, then the larger, +0.0 over -0.0
template <class T> __device__ __forceinline__ T jmax(T a, T b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a > b) return a;
  if (b > a) return b;
  return signbit(a) ? b : a;
}
template <class T> __device__ __forceinline__ T radd(T a, T b);
template <> __device__ __forceinline__ float radd(float a, float b) { return __fadd_rn(a, b); }
template <class T> __device__ __forceinline__ T rmul(T a, T b);
template <> __device__ __forceinline__ float rmul(float a, float b) { return __fmul_rn(a, b); }

// ---------------------------------------------------------------------------
// Per-sample head of the adjoint (Float32 or Float64), one warp per sample.
// NO = class capacity (>= n_o). Writes z, p (forward values), adds into yb,
// consumes zb, pb, hb to zero, and writes g = total zb (gbuf, n_s x n_o) and
// s1b = (1 - h^2) hb (s1b, n_s x n_h).
template <class T, int NO>
__global__ void __launch_bounds__(kHeadWarps * 32)
mlp_head_b_kernel(const T* __restrict__ lossb, const T* __restrict__ y, T* __restrict__ yb,
                  const T* __restrict__ w2, const T* __restrict__ b2, const T* __restrict__ h,
                  T* __restrict__ hb, T* __restrict__ z, T* __restrict__ zb, T* __restrict__ p,
                  T* __restrict__ pb, T* __restrict__ gbuf, T* __restrict__ s1b, int n_s,
                  int n_h, int n_o, T* __restrict__ loss_part) {
  extern __shared__ __align__(16) unsigned char smraw[];
  T* w2t = reinterpret_cast<T*>(smraw);  // [n_o][n_h], transposed for conflict-free reads
  __shared__ T red[kHeadWarps];
  for (int e = threadIdx.x; e < n_h * n_o; e += blockDim.x) {
    const int k = e / n_o, c = e % n_o;
    w2t[c * n_h + k] = w2[e];
  }
  __syncthreads();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int s = blockIdx.x * kHeadWarps + warp;
  const T lb = lossb[0];
  T loss_acc = T(0);
  if (s < n_s) {
    const T* hr = h + (int64_t)s * n_h;
    T zp[NO];
#pragma unroll
    for (int c = 0; c < NO; ++c) zp[c] = T(0);
    for (int k = lane; k < n_h; k += 32) {
      const T hv = hr[k];
#pragma unroll
      for (int c = 0; c < NO; ++c)
        if (c < n_o) zp[c] = fma(hv, w2t[c * n_h + k], zp[c]);
    }
    T zv[NO], yv[NO], pbin[NO], zbin[NO], ybin[NO];
#pragma unroll
    for (int c = 0; c < NO; ++c) {
      T v = c < n_o ? warp_sum(zp[c]) : T(0);
      zv[c] = c < n_o ? v + b2[c] : T(0);
    }
    const int64_t row = (int64_t)s * n_o;
    {
      // lane c loads the per-class inputs, then every lane gets all of them
      const T yl = lane < n_o ? y[row + lane] : T(0);
      const T pbl = lane < n_o ? pb[row + lane] : T(0);
      const T zbl = lane < n_o ? zb[row + lane] : T(0);
      const T ybl = lane < n_o ? yb[row + lane] : T(0);
#pragma unroll
      for (int c = 0; c < NO; ++c) {
        yv[c] = __shfl_sync(0xffffffffu, yl, c);
        pbin[c] = __shfl_sync(0xffffffffu, pbl, c);
        zbin[c] = __shfl_sync(0xffffffffu, zbl, c);
        ybin[c] = __shfl_sync(0xffffffffu, ybl, c);
      }
    }
    // forward softmax cross-entropy, in the generated statement order
    T mprev[NO];
    T m = zv[0];
#pragma unroll
    for (int c = 1; c < NO; ++c)
      if (c < n_o) { mprev[c] = m; m = jmax(m, zv[c]); }
    T pv[NO];
#pragma unroll
    for (int c = 0; c < NO; ++c) pv[c] = c < n_o ? dexp(radd(zv[c], -m)) : T(0);
    T rs = T(0);
#pragma unroll
    for (int c = 0; c < NO; ++c)
      if (c < n_o) rs = radd(rs, pv[c]);
#pragma unroll
    for (int c = 0; c < NO; ++c)
      if (c < n_o) loss_acc = radd(loss_acc, -rmul(yv[c], dlog(pv[c] / rs)));
    // reverse: loss statement, i_c = n_o:-1:1
    T ybout[NO], pbv[NO];
    T rsb = T(0);
#pragma unroll
    for (int c = NO - 1; c >= 0; --c) {
      if (c < n_o) {
        const T q = pv[c] / rs;
        ybout[c] = radd(ybin[c], rmul(-(dlog(q)), lb));
        const T qb = rmul(T(1) / q, rmul(-(yv[c]), lb));
        pbv[c] = radd(pbin[c], rmul(T(1) / rs, qb));
        rsb = radd(rsb, rmul(-(pv[c] / rmul(rs, rs)), qb));
      }
    }
    // row_sum loop, then the exp loop
    T g[NO];
    T mb = T(0);
#pragma unroll
    for (int c = NO - 1; c >= 0; --c) {
      if (c < n_o) {
        const T oldb = radd(pbv[c], rsb);
        const T cse = rmul(pv[c], oldb);
        g[c] = radd(zbin[c], cse);
        mb = radd(mb, -cse);
      }
    }
    // row-max chain, i_c = n_o:-1:2, then row_max = z[1]
#pragma unroll
    for (int c = NO - 1; c >= 1; --c) {
      if (c < n_o) {
        const T oldb = mb;
        mb = rmul(T(0.5) * (T(1) + dsign(radd(mprev[c], -zv[c]))), oldb);
        g[c] = radd(g[c], rmul(T(0.5) * (T(1) + dsign(radd(zv[c], -mprev[c]))), oldb));
      }
    }
    g[0] = radd(g[0], mb);
    // outputs of the per-class part; lane c stores class c
#pragma unroll
    for (int c = 0; c < NO; ++c) {
      if (c < n_o && lane == c) {
        z[row + c] = zv[c];
        p[row + c] = pv[c];
        yb[row + c] = ybout[c];
        zb[row + c] = T(0);
        pb[row + c] = T(0);
        gbuf[row + c] = g[c];
      }
    }
    // hidden adjoint: hb[s,k] += w2[k,c] g_c for c = n_o:-1:1, then consumed
    T* hbr = hb + (int64_t)s * n_h;
    T* s1br = s1b + (int64_t)s * n_h;
    for (int k = lane; k < n_h; k += 32) {
      T acc = hbr[k];
#pragma unroll
      for (int c = NO - 1; c >= 0; --c)
        if (c < n_o) acc = radd(acc, rmul(w2t[c * n_h + k], g[c]));
      const T th = hr[k];
      s1br[k] = rmul(radd(T(1), -rmul(th, th)), acc);
      hbr[k] = T(0);
    }
  }
  // fixed-order block sum of the per-warp loss terms
  if (lane == 0) red[warp] = loss_acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    T acc = T(0);
    for (int w = 0; w < kHeadWarps; ++w) acc += red[w];
    loss_part[blockIdx.x] = acc;
  }
}

// The same logits with four sample rows per warp pass (n_o <= 16, n_h a
// multiple of 128): each w2 float4 read from shared memory serves four rows
// (a quarter of the shared-memory traffic), and the 16 per-class partial sums
// of a lane are reduced across the warp by halving exchanges (8 + 4 + 2 + 1
// shuffles, then one to pair up: 16 per row instead of a 5-shuffle sum for
// each class). Lane l ends with class ((l >> 4) & 1) * 8 + ((l >> 3) & 1) * 4
// + ((l >> 2) & 1) * 2 + ((l >> 1) & 1), written by the even lanes.
constexpr int kLogitRows = 4;
__global__ void __launch_bounds__(256)
mlp_logits_rows_kernel(const float* __restrict__ h, const float* __restrict__ w2,
                       float* __restrict__ z0, int n_s, int n_h, int n_o) {
  extern __shared__ __align__(16) float w2t[];   // 16 x n_h, class-major, zero-padded
  for (int e = threadIdx.x; e < n_h * 16; e += blockDim.x) {
    const int c = e / n_h, k = e % n_h;
    w2t[e] = c < n_o ? w2[(int64_t)k * n_o + c] : 0.f;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int n4 = n_h >> 2;
  const float4* w4 = reinterpret_cast<const float4*>(w2t);
  const int warps = gridDim.x * (blockDim.x >> 5);
  const int groups = (n_s + kLogitRows - 1) / kLogitRows;
  for (int gi = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); gi < groups; gi += warps) {
    const int s0 = gi * kLogitRows;
    float acc[kLogitRows][16];
#pragma unroll
    for (int r = 0; r < kLogitRows; ++r)
#pragma unroll
      for (int c = 0; c < 16; ++c) acc[r][c] = 0.f;
    for (int base = 0; base < n4; base += 32) {
      const int k4 = base + lane;
      float4 hv[kLogitRows];
#pragma unroll
      for (int r = 0; r < kLogitRows; ++r)
        hv[r] = s0 + r < n_s ? reinterpret_cast<const float4*>(h + (int64_t)(s0 + r) * n_h)[k4]
                             : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const float4 w = w4[c * n4 + k4];
#pragma unroll
        for (int r = 0; r < kLogitRows; ++r) {
          acc[r][c] = fmaf(hv[r].x, w.x, acc[r][c]);
          acc[r][c] = fmaf(hv[r].y, w.y, acc[r][c]);
          acc[r][c] = fmaf(hv[r].z, w.z, acc[r][c]);
          acc[r][c] = fmaf(hv[r].w, w.w, acc[r][c]);
        }
      }
    }
#pragma unroll
    for (int r = 0; r < kLogitRows; ++r) {
      float* a = acc[r];
      // halving exchanges: keep the half of the classes this lane's bit selects
#pragma unroll
      for (int w = 8, bit = 16; w >= 1; w >>= 1, bit >>= 1) {
        const bool upper = (lane & bit) != 0;
#pragma unroll
        for (int i = 0; i < w; ++i) {
          const float keep = upper ? a[i + w] : a[i];
          const float send = upper ? a[i] : a[i + w];
          a[i] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
        }
      }
      const float v = a[0] + __shfl_xor_sync(0xffffffffu, a[0], 1);
      const int c = ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 +
                    ((lane >> 1) & 1);
      if ((lane & 1) == 0 && c < n_o && s0 + r < n_s) z0[(int64_t)(s0 + r) * n_o + c] = v;
    }
  }
}

// Logits without bias for the TMA path, z0[s][c] = sum_k h[s, k] w2[k, c]
// (the GEMM epilogue then only computes h, which takes the logits off its
// critical path: forward GEMM 374 -> 270 us, this pass ~90 us, at 65,536 x
// 512). One warp per sample row, n_h % 4 == 0: lane l takes the float4 groups
// l, l + 32, ... of the row (coalesced), all loaded before any arithmetic; w2
// is staged in shared memory class-major, so the lanes' float4 reads are
// consecutive; then one warp sum per class. (Measured slower: one thread per
// sample, with w2 read as broadcasts, and the same fused into the head.)
template <int NO>
__global__ void __launch_bounds__(256)
mlp_logits_kernel(const float* __restrict__ h, const float* __restrict__ w2,
                  float* __restrict__ z0, int n_s, int n_h, int n_o) {
  extern __shared__ __align__(16) float w2t[];   // NO x n_h
  for (int e = threadIdx.x; e < n_h * NO; e += blockDim.x) {
    const int c = e / n_h, k = e % n_h;
    w2t[e] = c < n_o ? w2[(int64_t)k * n_o + c] : 0.f;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int n4 = n_h >> 2;
  const float4* w4 = reinterpret_cast<const float4*>(w2t);
  const int warps = gridDim.x * (blockDim.x >> 5);
  for (int s = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); s < n_s; s += warps) {
    const float4* hr = reinterpret_cast<const float4*>(h + (int64_t)s * n_h);
    float acc[NO];
#pragma unroll
    for (int c = 0; c < NO; ++c) acc[c] = 0.f;
    for (int base = 0; base < n4; base += 128) {
      float4 hv[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int k4 = base + lane + 32 * t;
        hv[t] = k4 < n4 ? hr[k4] : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const int k4 = base + lane + 32 * t;
        if (k4 < n4) {
#pragma unroll
          for (int c = 0; c < NO; ++c) {
            if (c < n_o) {
              const float4 w = w4[c * n4 + k4];
              acc[c] = fmaf(hv[t].x, w.x, acc[c]);
              acc[c] = fmaf(hv[t].y, w.y, acc[c]);
              acc[c] = fmaf(hv[t].z, w.z, acc[c]);
              acc[c] = fmaf(hv[t].w, w.w, acc[c]);
            }
          }
        }
      }
    }
    float mine = 0.f;
#pragma unroll
    for (int c = 0; c < NO; ++c) {
      if (c < n_o) {
        const float v = warp_sum(acc[c]);
        if (lane == c) mine = v;
      }
    }
    if (lane < n_o) z0[(int64_t)s * n_o + lane] = mine;
  }
}

// Per-sample softmax cross-entropy, forward and reverse, one thread per
// sample (the tensor-core path): the logits come from the partial sums
// zpart[chunk][s][c] (the forward GEMM's epilogue, or mlp_logits_kernel with
// one chunk), summed in chunk order. Statement order as mlp_head_b_kernel.
template <class T, int NO>
__global__ void __launch_bounds__(256)
mlp_head_small_kernel(const T* __restrict__ zpart, int nchunks, const T* __restrict__ lossb,
                      const T* __restrict__ y, T* __restrict__ yb, const T* __restrict__ b2,
                      T* __restrict__ z, T* __restrict__ zb, T* __restrict__ p,
                      T* __restrict__ pb, T* __restrict__ gbuf, int n_s, int n_o,
                      T* __restrict__ loss_part) {
  __shared__ T red[8];
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  const T lb = lossb[0];
  T loss_acc = T(0);
  if (s < n_s) {
    const int64_t row = (int64_t)s * n_o;
    T zv[NO], yv[NO], pv[NO], g[NO], mprev[NO];
#pragma unroll
    for (int c = 0; c < NO; ++c) {
      if (c < n_o) {
        T acc = T(0);
        for (int ch = 0; ch < nchunks; ++ch) acc += zpart[((int64_t)ch * n_s + s) * n_o + c];
        zv[c] = acc + b2[c];
        yv[c] = y[row + c];
      }
    }
    T m = zv[0];
#pragma unroll
    for (int c = 1; c < NO; ++c)
      if (c < n_o) { mprev[c] = m; m = jmax(m, zv[c]); }
#pragma unroll
    for (int c = 0; c < NO; ++c)
      if (c < n_o) pv[c] = dexp(radd(zv[c], -m));
    T rs = T(0);
#pragma unroll
    for (int c = 0; c < NO; ++c)
      if (c < n_o) rs = radd(rs, pv[c]);
#pragma unroll
    for (int c = 0; c < NO; ++c)
      if (c < n_o) loss_acc = radd(loss_acc, -rmul(yv[c], dlog(pv[c] / rs)));
    T rsb = T(0);
    T pbv[NO];
#pragma unroll
    for (int c = NO - 1; c >= 0; --c) {
      if (c < n_o) {
        const T q = pv[c] / rs;
        yb[row + c] = radd(yb[row + c], rmul(-(dlog(q)), lb));
        const T qb = rmul(T(1) / q, rmul(-(yv[c]), lb));
        pbv[c] = radd(pb[row + c], rmul(T(1) / rs, qb));
        rsb = radd(rsb, rmul(-(pv[c] / rmul(rs, rs)), qb));
      }
    }
    T mb = T(0);
#pragma unroll
    for (int c = NO - 1; c >= 0; --c) {
      if (c < n_o) {
        const T oldb = radd(pbv[c], rsb);
        const T cse = rmul(pv[c], oldb);
        g[c] = radd(zb[row + c], cse);
        mb = radd(mb, -cse);
      }
    }
#pragma unroll
    for (int c = NO - 1; c >= 1; --c) {
      if (c < n_o) {
        const T oldb = mb;
        mb = rmul(T(0.5) * (T(1) + dsign(radd(mprev[c], -zv[c]))), oldb);
        g[c] = radd(g[c], rmul(T(0.5) * (T(1) + dsign(radd(zv[c], -mprev[c]))), oldb));
      }
    }
    g[0] = radd(g[0], mb);
#pragma unroll
    for (int c = 0; c < NO; ++c) {
      if (c < n_o) {
        z[row + c] = zv[c];
        p[row + c] = pv[c];
        zb[row + c] = T(0);
        pb[row + c] = T(0);
        gbuf[row + c] = g[c];
      }
    }
  }
  loss_acc = block_sum(loss_acc, red);
  if (threadIdx.x == 0) loss_part[blockIdx.x] = loss_acc;
}

// The s1b pass of the TMA path, two adjacent hidden units per thread (8-byte
// loads and stores, few registers, many blocks in flight):
// s1b = (1 - h^2) (hb + sum_c w2[k, c] g[s, c]), c descending (the generated
// order, multiply-adds fused: this pass was issue-bound, 73 instructions per
// element), written as TF32 hi / lo planes; hb consumed to zero (stored only
// where it held a seed); the chunk's W2b (sum_s h g), b2b (sum_s g) and b1b
// (sum_s s1b) partials. NO = the class count rounded to a template (exact for
// 10 classes); a sample's g sits in shared memory at a pitch of NO rounded up
// to 4. Block = 128 threads x 2 units = 256 units of a
// chunk of samples; partial record [chunk][n_h*n_o (W2b) + n_o (b2b) + n_h
// (b1b)].
template <int NO>
__global__ void __launch_bounds__(128)
mlp_s1b_planes_kernel(const float* __restrict__ h, float* __restrict__ hb,
                      const float* __restrict__ gbuf, const float* __restrict__ w2,
                      float* __restrict__ s1b_hi, float* __restrict__ s1b_lo, int n_s, int n_h,
                      int n_o, int chunk, float* __restrict__ part) {
  constexpr int GP = (NO + 3) / 4 * 4;           // g's pitch in shared memory
  extern __shared__ __align__(16) unsigned char smraw[];
  float* gs = reinterpret_cast<float*>(smraw);  // chunk x GP (zero padded)
  const int s0 = blockIdx.x * chunk;
  const int ns = min(n_s, s0 + chunk) - s0;
  for (int e = threadIdx.x; e < ns * GP; e += blockDim.x) {
    const int i = e / GP, c = e % GP;
    gs[e] = c < n_o ? gbuf[(int64_t)(s0 + i) * n_o + c] : 0.f;
  }
  __syncthreads();
  float* my = part + (int64_t)blockIdx.x * (n_h * n_o + n_o + n_h);
  const int k = blockIdx.y * 256 + 2 * threadIdx.x;
  if (k < n_h) {
    float w[2][NO], a[2][NO];
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int c = 0; c < NO; ++c) {
        w[j][c] = c < n_o ? w2[(int64_t)(k + j) * n_o + c] : 0.f;
        a[j][c] = 0.f;
      }
    float2 bsum = make_float2(0.f, 0.f);
    auto one = [&](int i, float2 hv, float2 acc2) {
      const int64_t off = (int64_t)(s0 + i) * n_h + k;
      const float* g = gs + i * GP;
      float hh[2] = {hv.x, hv.y};
      float ac[2] = {acc2.x, acc2.y};
#pragma unroll
      for (int c = NO - 1; c >= 0; --c) {
        if (c < n_o) {
          const float gc = g[c];
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            ac[j] = fmaf(w[j][c], gc, ac[j]);
            a[j][c] = fmaf(hh[j], gc, a[j][c]);
          }
        }
      }
      float o[2], hi[2], lo[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        o[j] = __fmul_rn(__fadd_rn(1.f, -__fmul_rn(hh[j], hh[j])), ac[j]);
        tc5::tf32_split(o[j], hi[j], lo[j]);
      }
      bsum.x += o[0]; bsum.y += o[1];
      *reinterpret_cast<float2*>(s1b_hi + off) = make_float2(hi[0], hi[1]);
      *reinterpret_cast<float2*>(s1b_lo + off) = make_float2(lo[0], lo[1]);
      // hb is consumed: zero it (only where it held a seed; a zero stays zero)
      if (acc2.x != 0.f || acc2.y != 0.f)
        *reinterpret_cast<float2*>(hb + off) = make_float2(0.f, 0.f);
    };
    // eight samples' loads in flight per thread (measured: 175 -> 136 us at
    // 65,536 x 512; h and hb are read once, so they stream past the caches)
    int i = 0;
    for (; i + 8 <= ns; i += 8) {
      float2 hv[8], hbv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int64_t off = (int64_t)(s0 + i + u) * n_h + k;
        hv[u] = __ldcs(reinterpret_cast<const float2*>(h + off));
        hbv[u] = __ldcs(reinterpret_cast<const float2*>(hb + off));
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) one(i + u, hv[u], hbv[u]);
    }
    for (; i < ns; ++i) {
      const int64_t off = (int64_t)(s0 + i) * n_h + k;
      one(i, *reinterpret_cast<const float2*>(h + off), *reinterpret_cast<const float2*>(hb + off));
    }
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int c = 0; c < NO; ++c)
        if (c < n_o) my[(int64_t)(k + j) * n_o + c] = a[j][c];
    float* bb = my + (int64_t)n_h * n_o + n_o;
    bb[k] = bsum.x; bb[k + 1] = bsum.y;
  }
  if (blockIdx.y == 0 && threadIdx.x < n_o) {
    const int c = threadIdx.x;
    float acc = 0.f;
    for (int i = 0; i < ns; ++i) acc += gs[i * GP + c];
    my[(int64_t)n_h * n_o + c] = acc;
  }
}

// W2b[k, c] partial = sum over the chunk's samples of h[s,k] g[s,c]; b2b[c]
// partial = sum g[s,c]. One thread per k; partial layout [chunk][n_h*n_o + n_o].
template <class T, int NO>
__global__ void __launch_bounds__(256)
mlp_w2b_partial_kernel(const T* __restrict__ h, const T* __restrict__ gbuf, int n_s, int n_h,
                       int n_o, int chunk, T* __restrict__ part) {
  const int s0 = blockIdx.x * chunk;
  const int s1 = min(n_s, s0 + chunk);
  T* my = part + (int64_t)blockIdx.x * (n_h * n_o + n_o);
  for (int k = threadIdx.x; k < n_h; k += blockDim.x) {
    T acc[NO];
#pragma unroll
    for (int c = 0; c < NO; ++c) acc[c] = T(0);
    for (int s = s0; s < s1; ++s) {
      const T hv = h[(int64_t)s * n_h + k];
      const T* gr = gbuf + (int64_t)s * n_o;
#pragma unroll
      for (int c = 0; c < NO; ++c)
        if (c < n_o) acc[c] = fma(hv, gr[c], acc[c]);
    }
#pragma unroll
    for (int c = 0; c < NO; ++c)
      if (c < n_o) my[k * n_o + c] = acc[c];
  }
  if (threadIdx.x < n_o) {
    const int c = threadIdx.x;
    T acc = T(0);
    for (int s = s0; s < s1; ++s) acc += gbuf[(int64_t)s * n_o + c];
    my[n_h * n_o + c] = acc;
  }
}

// Sum partial vectors of length len1 + len2 in chunk order into two arrays.
template <class T>
__global__ void finish_two_kernel(const T* __restrict__ part, int count, int64_t len1,
                                  T* __restrict__ dst1, int64_t len2, T* __restrict__ dst2) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t len = len1 + len2;
  if (e >= len) return;
  const T acc = ordered_sum(part + e, count, len);
  if (e < len1) dst1[e] += acc;
  else dst2[e - len1] += acc;
}

// First level of a fixed-order sum of `count` partial records of length len:
// group g (blockIdx.y) adds records [g per, (g + 1) per) in order into
// out[g][len]. finish_three_kernel then adds the groups in order.
__global__ void sum_groups_kernel(const float* __restrict__ part, int count, int per, int64_t len,
                                  float* __restrict__ out) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= len) return;
  const int p0 = blockIdx.y * per, p1 = min(count, p0 + per);
  const float acc = ordered_sum(part + (int64_t)p0 * len + e, p1 - p0, len);
  out[(int64_t)blockIdx.y * len + e] = acc;
}

// Sums partial records [chunk][len1 + len2 + len3] in chunk order into three arrays.
__global__ void finish_three_kernel(const float* __restrict__ part, int count, int64_t len1,
                                    float* __restrict__ dst1, int64_t len2,
                                    float* __restrict__ dst2, int64_t len3,
                                    float* __restrict__ dst3) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t len = len1 + len2 + len3;
  if (e >= len) return;
  const float acc = ordered_sum(part + e, count, len);
  if (e < len1) dst1[e] += acc;
  else if (e < len1 + len2) dst2[e - len1] += acc;
  else dst3[e - len1 - len2] += acc;
}

// ---- epilogues ---------------------------------------------------------------
template <class T>
struct EpiTanh : EpiBase {  // h[m, n] = tanh(acc + b1[n])
  const T* b1;
  T* h;
  int ld;
  __device__ __forceinline__ void operator()(int m, int n, T acc) const {
    h[(int64_t)m * ld + n] = dtanh(acc + b1[n]);
  }
};
template <class T>
struct EpiAddTo : EpiBase {  // dst[m, n] += acc
  T* dst;
  int ld;
  __device__ __forceinline__ void operator()(int m, int n, T acc) const {
    T* q = dst + (int64_t)m * ld + n;
    *q = *q + acc;
  }
};
template <class T>
struct EpiWeightBias : EpiBase {  // rows < n_w: w[m, n] += acc; row n_w: bias[n] += acc
  T* w;
  T* bias;
  int n_w, ld;
  __device__ __forceinline__ void operator()(int m, int n, T acc) const {
    if (m < n_w) {
      T* q = w + (int64_t)m * ld + n;
      *q = *q + acc;
    } else {
      bias[n] = bias[n] + acc;
    }
  }
};

// ---- loaders -------------------------------------------------------------------
template <class T>
struct LdRow {  // A(m, k) = a[m * ld + k]
  const T* a;
  int ld;
  __device__ __forceinline__ T operator()(int m, int k) const { return a[(int64_t)m * ld + k]; }
};
template <class T>
struct LdB {  // B(k, n) = b[k * ld + n]
  const T* b;
  int ld;
  __device__ __forceinline__ T operator()(int k, int n) const { return b[(int64_t)k * ld + n]; }
};
template <class T>
struct LdBT {  // B(k, n) = b[n * ld + k]
  const T* b;
  int ld;
  __device__ __forceinline__ T operator()(int k, int n) const { return b[(int64_t)n * ld + k]; }
};
template <class T>
struct LdXtOnes {  // A(m, k) = x[k * ld + m] for m < n_m, 1 for m == n_m
  const T* x;
  int ld, n_m;
  __device__ __forceinline__ T operator()(int m, int k) const {
    return m < n_m ? x[(int64_t)k * ld + m] : T(1);
  }
};

constexpr int kF32RM = 2, kF32RN = 2, kF32BK = 16;
constexpr int kF64RM = 2, kF64RN = 2, kF64BK = 8;

// Float64 contractions run on the FP64 tensor cores (DMMA) unless
// STADE_F64_GEMM=simt selects the CUDA-core kernel.
inline bool f64_dmma() {
  const char* e = std::getenv("STADE_F64_GEMM");
  return !(e && std::strcmp(e, "simt") == 0);
}
template <bool A_KC, bool B_NC, class LA, class LB, class Epi>
stade_status gemm_f64(int M, int N, int K, LA la, LB lb, Epi epi, double* partial, int splits,
                      cudaStream_t s);

template <class T, int RM, int RN, int BK>
int splits_for(int M, int N, int K) {
  const int tiles = ((M + 64 * RM - 1) / (64 * RM)) * ((N + 64 * RN - 1) / (64 * RN));
  if constexpr (std::is_same<T, double>::value) {
    // the DMMA kernel's 128 x 128 tiles, one block per SM
    if (f64_dmma())
      return dmma_splits(((M + dmma::BM - 1) / dmma::BM) * ((N + dmma::BN - 1) / dmma::BN), K,
                         tc5::sm_count());
  }
  return split_plan(tiles, K, BK, 64).splits;
}


template <bool A_KC, bool B_NC, class LA, class LB, class Epi>
stade_status gemm_f64(int M, int N, int K, LA la, LB lb, Epi epi, double* partial, int splits,
                      cudaStream_t s) {
  if (f64_dmma()) return gemm_dmma<A_KC, B_NC>(M, N, K, la, lb, epi, partial, splits, s);
  return gemm_simt<double, kF64RM, kF64RN, kF64BK, A_KC, B_NC>(M, N, K, la, lb, epi, partial,
                                                                 splits, s);
}

// ---------------------------------------------------------------------------
// Per-sample head of the Float64 HVP: every statement of the head with its
// tangent twin (oracle.cc mlp2_ce_hv; hvp_double_stmt, src/STADE.jl:6904).
// One warp per sample, lane c owns class c (n_o <= 32): its logit and
// tangent as the sequential sums over hidden units, its softmax terms and
// their reverse. The class-to-class scans (the running max and its reverse)
// run in every lane over values passed by shuffle; sums over classes are
// warp sums. Lanes then own hidden units for s1b = (1 - h^2)(hb + W2 g) and
// its tangent, with g and gd broadcast class by class.
__global__ void __launch_bounds__(kHvHeadWarps * 32)
mlp_head_hv_kernel(const double* __restrict__ lossb, const double* __restrict__ lossbd,
                   const double* __restrict__ y, double* __restrict__ yb,
                   const double* __restrict__ yd, double* __restrict__ ybd,
                   const double* __restrict__ w2, const double* __restrict__ b2,
                   const double* __restrict__ w2d, const double* __restrict__ b2d,
                   const double* __restrict__ h, double* __restrict__ hb,
                   const double* __restrict__ hd, double* __restrict__ hbd,
                   double* __restrict__ z, double* __restrict__ zb, double* __restrict__ zd,
                   double* __restrict__ zbd, double* __restrict__ p, double* __restrict__ pb,
                   double* __restrict__ pd, double* __restrict__ pbd,
                   double* __restrict__ gbuf, double* __restrict__ gdbuf,
                   double* __restrict__ s1b, double* __restrict__ s1bd, int n_s, int n_h, int n_o,
                   double* __restrict__ loss_part, double* __restrict__ lossd_part, int w2_smem,
                   int rows_smem) {
  __shared__ double red[2][kHvHeadWarps];
  // w2 and w2d staged class-major with an odd row stride: the class lanes of
  // the logits loop and the hidden-unit lanes of the s1b loop both read
  // distinct banks (read from global memory instead, [k][c], when they do
  // not fit)
  extern __shared__ double w2sm[];
  const int LD = n_h + 1;
  if (w2_smem) {
    for (int e = threadIdx.x; e < n_o * n_h; e += blockDim.x) {
      const int cc = e / n_h, k = e % n_h;
      w2sm[cc * LD + k] = w2[(int64_t)k * n_o + cc];
      w2sm[n_o * LD + cc * LD + k] = w2d[(int64_t)k * n_o + cc];
    }
    __syncthreads();
  }
  auto W = [&](int k, int cc) {
    return w2_smem ? w2sm[cc * LD + k] : w2[(int64_t)k * n_o + cc];
  };
  auto WD = [&](int k, int cc) {
    return w2_smem ? w2sm[n_o * LD + cc * LD + k] : w2d[(int64_t)k * n_o + cc];
  };
  const unsigned F = 0xffffffffu;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool cl = lane < n_o;          // this lane owns class `lane`
  const int c = cl ? lane : 0;
  const double lb = lossb[0], lbd = lossbd[0];
  double loss_acc = 0.0, lossd_acc = 0.0;
  // rows_smem (with w2_smem): each warp stages its sample's h and hd rows in
  // shared memory (after w2 / w2d) with one coalesced load each, all in
  // flight at once; otherwise the rows are read from memory unit by unit
  double* hs = w2sm + 2 * (size_t)n_o * LD + (size_t)warp * 2 * n_h;
  double* hds = hs + n_h;
  for (int s = blockIdx.x * kHvHeadWarps + warp; s < n_s; s += gridDim.x * kHvHeadWarps) {
    const double* hr = h + (int64_t)s * n_h;
    const double* hdr = hd + (int64_t)s * n_h;
    const int64_t row = (int64_t)s * n_o;
    // the class lane's per-sample values, loaded together up front (read in
    // order below, each would otherwise wait out a memory latency of its own)
    double y_c = 0.0, yd_c = 0.0, yb_c = 0.0, ybd_c = 0.0, pb_c = 0.0, pbd_c = 0.0, zb_c = 0.0,
           zbd_c = 0.0;
    if (cl) {
      y_c = y[row + c]; yd_c = yd[row + c]; yb_c = yb[row + c]; ybd_c = ybd[row + c];
      pb_c = pb[row + c]; pbd_c = pbd[row + c]; zb_c = zb[row + c]; zbd_c = zbd[row + c];
    }
    if (rows_smem) {
      __syncwarp();   // the previous sample's reads of the rows are done
      for (int k0 = 0; k0 < n_h; k0 += 32 * 8) {
        double r[8], rd[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int k = k0 + 32 * j + lane;
          r[j] = k < n_h ? hr[k] : 0.0;
          rd[j] = k < n_h ? hdr[k] : 0.0;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int k = k0 + 32 * j + lane;
          if (k < n_h) { hs[k] = r[j]; hds[k] = rd[j]; }
        }
      }
      __syncwarp();
    }
    const double* hrow = rows_smem ? hs : hr;
    const double* hdrow = rows_smem ? hds : hdr;
    // logits and tangents
    double zv = b2[c], zdv = b2d[c];
    if (rows_smem && n_o <= 16) {
      // every lane sums its own hidden units (l, l + 32, ...) for all classes
      // (sixteen independent chains per array), then the lanes' sums meet in
      // a fixed halving tree: the same order on every call (the generated
      // sweep's single chain per class held ten lanes of a warp for 512
      // dependent additions per sample)
      double za[16], zda[16];
#pragma unroll
      for (int cc = 0; cc < 16; ++cc) { za[cc] = 0.0; zda[cc] = 0.0; }
      for (int k = lane; k < n_h; k += 32) {
        const double hv = hs[k], hdv = hds[k];
#pragma unroll
        for (int cc = 0; cc < 16; ++cc) {
          if (cc < n_o) {
            const double wv = W(k, cc);
            zda[cc] = zda[cc] + (hv * WD(k, cc) + wv * hdv);
            za[cc] = fma(wv, hv, za[cc]);
          }
        }
      }
      const double zs = halving_sum16(za, lane), zds = halving_sum16(zda, lane);
      const int src = class_lane16(c);
      const double zsum = __shfl_sync(F, zs, src), zdsum = __shfl_sync(F, zds, src);
      zv = zv + zsum;
      zdv = zdv + zdsum;
    } else {
#pragma unroll 8
      for (int k = 0; k < n_h; ++k) {
        const double hv = hrow[k], hdv = hdrow[k];
        const double wv = W(k, c);
        zdv = zdv + (hv * WD(k, c) + wv * hdv);
        zv = zv + wv * hv;
      }
    }
    // running max over classes with its tangent
    double m = __shfl_sync(F, zv, 0), md = __shfl_sync(F, zdv, 0);
    double mprev = 0.0;
    for (int cc = 1; cc < n_o; ++cc) {
      const double zc = __shfl_sync(F, zv, cc), zdc = __shfl_sync(F, zdv, cc);
      if (lane == cc) mprev = m;
      const double g1 = 0.5 * (1.0 + dsign(m - zc));
      const double g2 = 0.5 * (1.0 + dsign(zc - m));
      md = g1 * md + g2 * zdc;
      m = jmax(m, zc);
    }
    const double e = cl ? exp(zv - m) : 0.0;
    const double ed = cl ? e * (zdv - md) : 0.0;
    const double rs = warp_sum(e), rsd = warp_sum(ed);
    double yv = 0.0, ydv = 0.0;
    double lq = 0.0, lqd = 0.0, q = 1.0, qd = 0.0;
    if (cl) {
      yv = y_c;
      ydv = yd_c;
      q = e / rs;
      qd = ed / rs - (e / (rs * rs)) * rsd;
      lq = log(q);
      lqd = qd / q;
      lossd_acc = lossd_acc - (ydv * lq + yv * lqd);
      loss_acc = loss_acc - yv * lq;
    }
    // reverse of the loss statement with tangents
    double pbv = 0.0, pbdv = 0.0, rsb_c = 0.0, rsbd_c = 0.0;
    if (cl) {
      ybd[row + c] = ybd_c + -(lqd * lb + lq * lbd);
      yb[row + c] = yb_c + -(lq) * lb;
      const double inv_q = 1.0 / q, inv_qd = -(qd / (q * q));
      const double ny = -(yv) * lb, nyd = -(ydv * lb + yv * lbd);
      const double qbd = inv_qd * ny + inv_q * nyd;
      const double qb = inv_q * ny;
      const double inv_rs = 1.0 / rs, inv_rsd = -(rsd / (rs * rs));
      pbdv = pbd_c + (inv_rsd * qb + inv_rs * qbd);
      pbv = pb_c + inv_rs * qb;
      const double pr2 = e / (rs * rs);
      const double pr2d = ed / (rs * rs) - (e / (rs * rs)) * ((2.0 * rs * rsd) / (rs * rs));
      rsbd_c = -(pr2d * qb + pr2 * qbd);
      rsb_c = -(pr2)*qb;
    }
    const double rsb = warp_sum(rsb_c), rsbd = warp_sum(rsbd_c);
    double g = 0.0, gd = 0.0, cse = 0.0, csed = 0.0;
    if (cl) {
      const double oldbd = pbdv + rsbd, oldb = pbv + rsb;
      csed = ed * oldb + e * oldbd;
      cse = e * oldb;
      gd = zbd_c + csed;
      g = zb_c + cse;
    }
    double mb = warp_sum(-cse), mbd = warp_sum(-csed);
    // reverse of the running max, classes n_o - 1 .. 1
    for (int cc = n_o - 1; cc >= 1; --cc) {
      const double mp = __shfl_sync(F, mprev, cc), zc = __shfl_sync(F, zv, cc);
      const double g1 = 0.5 * (1.0 + dsign(mp - zc));
      const double g2 = 0.5 * (1.0 + dsign(zc - mp));
      if (lane == cc) {
        gd = gd + g2 * mbd;
        g = g + g2 * mb;
      }
      mbd = 0.0 + g1 * mbd;
      mb = 0.0 + g1 * mb;
    }
    if (lane == 0) {
      gd = gd + mbd;
      g = g + mb;
    }
    if (cl) {
      z[row + c] = zv; zd[row + c] = zdv;
      p[row + c] = e; pd[row + c] = ed;
      zb[row + c] = 0.0; zbd[row + c] = 0.0;
      pb[row + c] = 0.0; pbd[row + c] = 0.0;
      gbuf[row + c] = g; gdbuf[row + c] = gd;
    }
    // s1b, s1bd: lanes own hidden units, g and gd broadcast class by class
    double* hbr = hb + (int64_t)s * n_h;
    double* hbdr = hbd + (int64_t)s * n_h;
    double* s1br = s1b + (int64_t)s * n_h;
    double* s1bdr = s1bd + (int64_t)s * n_h;
    for (int k0 = 0; k0 < n_h; k0 += 32 * 8) {
      double acc[8], accd[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int k = k0 + 32 * j + lane;
        acc[j] = k < n_h ? hbr[k] : 0.0;
        accd[j] = k < n_h ? hbdr[k] : 0.0;
      }
      for (int cc = n_o - 1; cc >= 0; --cc) {
        const double gc = __shfl_sync(F, g, cc), gdc = __shfl_sync(F, gd, cc);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int k = k0 + 32 * j + lane;
          if (k < n_h) {
            const double wv = W(k, cc);
            accd[j] = accd[j] + (gc * WD(k, cc) + wv * gdc);
            acc[j] = acc[j] + wv * gc;
          }
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int k = k0 + 32 * j + lane;
        if (k < n_h) {
          const double th = hrow[k];
          const double thd = hdrow[k];
          const double gg = 1.0 - th * th;
          s1bdr[k] = acc[j] * -((2.0 * th) * thd) + gg * accd[j];
          s1br[k] = gg * acc[j];
          hbr[k] = 0.0;
          hbdr[k] = 0.0;
        }
      }
    }
  }
  // each lane holds its classes' terms
  loss_acc = warp_sum(loss_acc);
  lossd_acc = warp_sum(lossd_acc);
  if (lane == 0) { red[0][warp] = loss_acc; red[1][warp] = lossd_acc; }
  __syncthreads();
  if (threadIdx.x == 0) {
    double a = 0.0, b = 0.0;
    for (int w = 0; w < kHvHeadWarps; ++w) { a += red[0][w]; b += red[1][w]; }
    loss_part[blockIdx.x] = a;
    lossd_part[blockIdx.x] = b;
  }
}

// W2b, W2bd, b2b, b2bd partials of one chunk of samples; layout
// [chunk][n_h*n_o (W2b) + n_h*n_o (W2bd) + n_o (b2b) + n_o (b2bd)]. One thread
// per hidden unit k (a block's 256 units read each h / hd row coalesced, four
// samples' loads in flight), the samples of the chunk in order; the chunk's g
// and gd staged in shared memory (broadcast reads).
template <int NO>
__global__ void __launch_bounds__(256)
mlp_w2b_hv_partial_kernel(const double* __restrict__ h, const double* __restrict__ hd,
                          const double* __restrict__ gbuf, const double* __restrict__ gdbuf,
                          int n_s, int n_h, int n_o, int chunk, double* __restrict__ part) {
  extern __shared__ double gsm[];   // [chunk][2 NO]: g, then gd (zero padded)
  const int s0 = blockIdx.x * chunk;
  const int ns = min(n_s, s0 + chunk) - s0;
  for (int e = threadIdx.x; e < ns * NO; e += blockDim.x) {
    const int i = e / NO, c = e % NO;
    const int64_t src = (int64_t)(s0 + i) * n_o + c;
    gsm[i * 2 * NO + c] = c < n_o ? gbuf[src] : 0.0;
    gsm[i * 2 * NO + NO + c] = c < n_o ? gdbuf[src] : 0.0;
  }
  __syncthreads();
  const int64_t nw = (int64_t)n_h * n_o;
  double* my = part + (int64_t)blockIdx.x * (2 * nw + 2 * n_o);
  const int k = blockIdx.y * blockDim.x + threadIdx.x;
  if (k < n_h) {
    double acc[NO], accd[NO];
#pragma unroll
    for (int c = 0; c < NO; ++c) { acc[c] = 0.0; accd[c] = 0.0; }
    auto one = [&](int i, double hv, double hdv) {
      const double* gr = gsm + i * 2 * NO;
#pragma unroll
      for (int c = 0; c < NO; ++c) {
        if (c < n_o) {
          accd[c] += gr[c] * hdv + hv * gr[NO + c];
          acc[c] = fma(hv, gr[c], acc[c]);
        }
      }
    };
    int i = 0;
    for (; i + 4 <= ns; i += 4) {
      double hv[4], hdv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int64_t off = (int64_t)(s0 + i + u) * n_h + k;
        hv[u] = h[off];
        hdv[u] = hd[off];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) one(i + u, hv[u], hdv[u]);
    }
    for (; i < ns; ++i) {
      const int64_t off = (int64_t)(s0 + i) * n_h + k;
      one(i, h[off], hd[off]);
    }
#pragma unroll
    for (int c = 0; c < NO; ++c) {
      if (c < n_o) {
        my[(int64_t)k * n_o + c] = acc[c];
        my[nw + (int64_t)k * n_o + c] = accd[c];
      }
    }
  }
  if (blockIdx.y == 0 && threadIdx.x < 2 * n_o) {
    const int c = threadIdx.x % n_o, off = threadIdx.x < n_o ? 0 : NO;
    double a = 0.0;
    for (int i = 0; i < ns; ++i) a += gsm[i * 2 * NO + off + c];
    my[2 * nw + threadIdx.x] = a;
  }
}

// Sums [chunk][4 segments] partials in chunk order into four arrays.
__global__ void finish_four_kernel(const double* __restrict__ part, int count, int64_t nw,
                                   int n_o, double* __restrict__ w2b, double* __restrict__ w2bd,
                                   double* __restrict__ b2b, double* __restrict__ b2bd) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t len = 2 * nw + 2 * n_o;
  if (e >= len) return;
  const double acc = ordered_sum(part + e, count, len);
  if (e < nw) w2b[e] += acc;
  else if (e < 2 * nw) w2bd[e - nw] += acc;
  else if (e < 2 * nw + n_o) b2b[e - 2 * nw] += acc;
  else b2bd[e - 2 * nw - n_o] += acc;
}

struct EpiStore : EpiBase {  // dst[m, n] = acc
  double* dst;
  int ld;
  __device__ __forceinline__ void operator()(int m, int n, double acc) const {
    dst[(int64_t)m * ld + n] = acc;
  }
};
// s1d = acc + b1d; s1 = S1 + b1; h = tanh(s1); hd = (1 - h^2) s1d
struct EpiTanhTangent : EpiBase {
  const double *s1, *b1, *b1d;
  double *h, *hd;
  int ld;
  __device__ __forceinline__ void operator()(int m, int n, double acc) const {
    const int64_t i = (int64_t)m * ld + n;
    const double s1d = acc + b1d[n];
    const double th = tanh(s1[i] + b1[n]);
    hd[i] = (1.0 - th * th) * s1d;
    h[i] = th;
  }
};
// A(m, k) over two K segments: [a0 | a1], each row-major with leading dim ld
struct LdRow2 {
  const double *a0, *a1;
  int ld, k0;
  __device__ __forceinline__ double operator()(int m, int k) const {
    return k < k0 ? a0[(int64_t)m * ld + k] : a1[(int64_t)m * ld + (k - k0)];
  }
};
// B(k, n) over two K segments: [b0 ; b1], each row-major with leading dim ld
struct LdB2 {
  const double *b0, *b1;
  int ld, k0;
  __device__ __forceinline__ double operator()(int k, int n) const {
    return k < k0 ? b0[(int64_t)k * ld + n] : b1[(int64_t)(k - k0) * ld + n];
  }
};
// B(k, n) = [b0^T ; b1^T](k, n): b0[n * ld + k] for k < k0, b1[n * ld + k - k0] after
struct LdBT2 {
  const double *b0, *b1;
  int ld, k0;
  __device__ __forceinline__ double operator()(int k, int n) const {
    return k < k0 ? b0[(int64_t)n * ld + k] : b1[(int64_t)n * ld + (k - k0)];
  }
};
// A(m, k) = [x0^T | x1^T](m, k) with a row of ones (segment 0) / zeros (segment 1) at m == n_m
struct LdXtOnes2 {
  const double *x0, *x1;
  int ld, n_m, k0;
  __device__ __forceinline__ double operator()(int m, int k) const {
    if (k < k0) return m < n_m ? x0[(int64_t)k * ld + m] : 1.0;
    return m < n_m ? x1[(int64_t)(k - k0) * ld + m] : 0.0;
  }
};

struct MlpF64HvWs {
  double *s1, *s1b, *s1bd, *gbuf, *gdbuf, *loss_part, *lossd_part, *w2_part, *w1_part;
  int head_blocks, w2_chunks, w1_splits, w1d_splits;
};
template <class Alloc>
void mlp_hv_layout(Alloc& a, MlpF64HvWs* w, int64_t n_s, int64_t n_i, int64_t n_h, int64_t n_o) {
  // warps stride over the samples; eight blocks of eight warps per SM
  const int head_need = (int)((n_s + kHeadWarps - 1) / kHeadWarps);
  const int head_blocks = head_need < 8 * 148 ? head_need : 8 * 148;
  const int w2_chunks = (int)((n_s + kW2ChunkHv - 1) / kW2ChunkHv);
  const int w1_splits = splits_for<double, kF64RM, kF64RN, kF64BK>((int)n_i + 1, (int)n_h, (int)n_s);
  const int w1d_splits = splits_for<double, kF64RM, kF64RN, kF64BK>((int)n_i + 1, (int)n_h, 2 * (int)n_s);
  const int maxs = w1_splits > w1d_splits ? w1_splits : w1d_splits;
  auto p0 = a.template take<double>((size_t)(n_s * n_h));
  auto p1 = a.template take<double>((size_t)(n_s * n_h));
  auto p2 = a.template take<double>((size_t)(n_s * n_h));
  auto p3 = a.template take<double>((size_t)(n_s * n_o));
  auto p4 = a.template take<double>((size_t)(n_s * n_o));
  auto p5 = a.template take<double>((size_t)head_blocks);
  auto p6 = a.template take<double>((size_t)head_blocks);
  auto p7 = a.template take<double>((size_t)w2_chunks * (size_t)(2 * n_h * n_o + 2 * n_o));
  auto p8 = a.template take<double>(maxs > 1 ? (size_t)maxs * (size_t)((n_i + 1) * n_h) : 1);
  if (w) {
    w->s1 = (double*)p0; w->s1b = (double*)p1; w->s1bd = (double*)p2; w->gbuf = (double*)p3;
    w->gdbuf = (double*)p4; w->loss_part = (double*)p5; w->lossd_part = (double*)p6;
    w->w2_part = (double*)p7; w->w1_part = (double*)p8;
    w->head_blocks = head_blocks; w->w2_chunks = w2_chunks;
    w->w1_splits = w1_splits; w->w1d_splits = w1d_splits;
  }
}

}  // namespace

// ============================================================================
// Float32 adjoint
// ============================================================================
namespace {
constexpr int kW2ChunkTc = 64;  // samples per W2b partial on the tensor-core paths

constexpr int kFinGroups = 16;  // first-level groups of the W2b / b2b / b1b partial sum

struct MlpF32Ws {
  float *s1b, *gbuf, *loss_part, *w2_part, *w1_part, *zpart, *fin;
  float *x_lo, *w1_lo, *s1b_hi, *s1b_lo, *w1b_part;
  int head_blocks, w2_chunks, w1_splits;
};

// The four-rows-per-warp logits pass (STADE_LOGITS_ROWS=0 selects the
// one-row pass).
bool logits_rows_enabled() {
  const char* e = std::getenv("STADE_LOGITS_ROWS");
  return !(e && std::strcmp(e, "0") == 0);
}

// Contraction path of the Float32 adjoint: TMA-fed tcgen05 (default) or
// CUDA-core SIMT (sizes TMA cannot describe; STADE_MLP_GEMM=simt forces it).
enum class MlpPath { Tma, Simt };
MlpPath mlp_path(int64_t n_s, int64_t n_i, int64_t n_h) {
  if (!tma_mlp_supported(n_s, n_i, n_h)) return MlpPath::Simt;
  const char* sel = std::getenv("STADE_MLP_GEMM");
  if (sel && std::strcmp(sel, "simt") == 0) return MlpPath::Simt;
  return MlpPath::Tma;
}
template <class Alloc>
void mlp_f32_layout(Alloc& a, MlpF32Ws* w, int64_t n_s, int64_t n_i, int64_t n_h, int64_t n_o) {
  const int head_blocks = (int)((n_s + kHeadWarps - 1) / kHeadWarps);
  const int w2_chunks = (int)((n_s + kW2Chunk - 1) / kW2Chunk);
  const int w1_splits = splits_for<float, kF32RM, kF32RN, kF32BK>((int)n_i + 1, (int)n_h, (int)n_s);
  if (w) {
    w->head_blocks = head_blocks;
    w->w2_chunks = w2_chunks;
    w->w1_splits = w1_splits;
  }
  const int tc_chunks = (int)((n_s + kW2ChunkTc - 1) / kW2ChunkTc);
  const int w2_parts = w2_chunks > tc_chunks ? w2_chunks : tc_chunks;
  const int head_parts = head_blocks > (int)((n_s + 255) / 256) ? head_blocks : (int)((n_s + 255) / 256);
  auto s1b = a.template take<float>((size_t)(n_s * n_h));
  auto gb = a.template take<float>((size_t)(n_s * n_o));
  auto lp = a.template take<float>((size_t)head_parts);
  auto w2p = a.template take<float>((size_t)w2_parts * (size_t)(n_h * n_o + n_o + n_h));
  auto w1p = a.template take<float>(w1_splits > 1 ? (size_t)w1_splits * (size_t)((n_i + 1) * n_h) : 1);
  auto zp = a.template take<float>((size_t)tma_logit_parts(n_h) * (size_t)(n_s * n_o));
  const bool planes = tma_mlp_supported(n_s, n_i, n_h);
  // lo planes of x and W1 (each array is its own hi plane)
  auto xl = a.template take<float>(planes ? (size_t)(n_s * n_i) : 1);
  auto wl = a.template take<float>(planes ? (size_t)(n_i * n_h) : 1);
  auto sh = a.template take<float>(planes ? (size_t)(n_s * n_h) : 1);
  auto sl = a.template take<float>(planes ? (size_t)(n_s * n_h) : 1);
  auto wp = a.template take<float>(planes ? tma_w1b_part_floats(n_s, n_i, n_h) : 1);
  auto fin = a.template take<float>((size_t)kFinGroups * (size_t)(n_h * n_o + n_o + n_h));
  if (w) {
    w->fin = (float*)fin;
    w->s1b = (float*)s1b; w->gbuf = (float*)gb; w->loss_part = (float*)lp;
    w->w2_part = (float*)w2p; w->w1_part = (float*)w1p; w->zpart = (float*)zp;
    w->x_lo = (float*)xl; w->w1_lo = (float*)wl;
    w->s1b_hi = (float*)sh; w->s1b_lo = (float*)sl; w->w1b_part = (float*)wp;
  }
}
struct SizerAlloc {
  Sizer z;
  template <class T> void* take(size_t n) { z.take<T>(n); return nullptr; }
};
struct CarverAlloc {
  Carver c;
  explicit CarverAlloc(void* b) : c(b) {}
  template <class T> T* take(size_t n) { return c.take<T>(n); }
};
}  // namespace

}  // namespace stade

using namespace stade;

extern "C" size_t stade_mlp2_ce_b_f32_workspace(int64_t n_s, int64_t n_i, int64_t n_h,
                                                int64_t n_o) {
  if (n_s <= 0 || n_h <= 0 || n_o <= 0 || n_i < 0) return 256;
  SizerAlloc a;
  mlp_f32_layout(a, nullptr, n_s, n_i, n_h, n_o);
  return a.z.bytes();
}

extern "C" stade_status stade_mlp2_ce_b_f32(float* loss, const float* lossb, const float* x,
                                            float* xb, const float* y, float* yb, const float* w1,
                                            float* w1b, const float* b1, float* b1b,
                                            const float* w2, float* w2b, const float* b2,
                                            float* b2b, float* h, float* hb, float* z, float* zb,
                                            float* p, float* pb, int64_t n_s, int64_t n_i,
                                            int64_t n_h, int64_t n_o, const stade_opts* opts) {
  STADE_REQUIRE(n_s >= 0 && n_i >= 0 && n_h >= 0 && n_o >= 0, "mlp2_ce_b: negative size");
  if (n_s == 0) return STADE_OK;
  if (n_o == 0) {
    // no classes: the logits and loss loops are empty; only the hidden layer runs
    STADE_REQUIRE(n_o > 0, "mlp2_ce_b: n_o = 0 is not supported");
  }
  STADE_REQUIRE(n_o <= 32, "mlp2_ce_b: n_o = %lld > 32 classes", (long long)n_o);
  STADE_REQUIRE(n_h > 0, "mlp2_ce_b: n_h = 0 is not supported");
  STADE_REQUIRE(n_s <= (1 << 30) && n_i < (1 << 20) && n_h < (1 << 16) &&
                    n_s * n_i < (int64_t(1) << 40),
                "mlp2_ce_b: sizes out of range");
  STADE_REQUIRE(loss && lossb && x && xb && y && yb && w1 && w1b && b1 && b1b && w2 && w2b && b2 &&
                    b2b && h && hb && z && zb && p && pb,
                "mlp2_ce_b: null array argument");
  cudaStream_t s = stream_of(opts);
  void* wsp = nullptr;
  stade_status st = get_workspace(opts, stade_mlp2_ce_b_f32_workspace(n_s, n_i, n_h, n_o), &wsp);
  if (st != STADE_OK) return st;
  CarverAlloc ca(wsp);
  MlpF32Ws w;
  mlp_f32_layout(ca, &w, n_s, n_i, n_h, n_o);
  const int S = (int)n_s, I = (int)n_i, H = (int)n_h, O = (int)n_o;
  MlpPath path = mlp_path(n_s, n_i, n_h);
  // the TMA path reads x and W1 in place through TMA, and its logits and s1b
  // passes read h (and hb) with 8- and 16-byte vector loads: those base
  // addresses must be 16-byte aligned (h and xb written by the GEMMs are
  // checked there: a misaligned one takes register stores)
  if (path == MlpPath::Tma &&
      ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w1) |
        reinterpret_cast<uintptr_t>(h) | reinterpret_cast<uintptr_t>(hb)) & 15u))
    path = MlpPath::Simt;

  if (path == MlpPath::Tma) {
    // 0. TF32 lo planes of x and W1
    {
      PhaseScope ph("split", s);
      // x and W1 serve as their own hi planes (kind::tf32 reads the top 19
      // bits); only their lo planes are written
      st = tma_split_lo2(x, w.x_lo, n_s * n_i, w1, w.w1_lo, n_i * n_h, s);
    }
    if (st != STADE_OK) return st;
    // 1. h = tanh(x W1 + b1), TMA-fed tensor cores (the logits in a pass of
    // their own when w2 fits in shared memory, else in the GEMM's epilogue)
    const size_t lsm = sizeof(float) * (size_t)H * (O <= 16 ? 16 : 32);
    const bool own_logits = lsm <= 160 * 1024 && H % 4 == 0;
    {
      PhaseScope ph("fwd_gemm", s);
      st = tma_forward_tanh_logits(x, w.x_lo, w1, w.w1_lo, b1, w2, h,
                                   own_logits ? nullptr : w.zpart, S, I, H, O, s);
    }
    if (st != STADE_OK) return st;
    // 2. softmax cross-entropy and its reverse, one thread per sample
    {
      PhaseScope ph("head", s);
      const int blocks = (S + 255) / 256;
      auto kern = O <= 16 ? mlp_head_small_kernel<float, 16> : mlp_head_small_kernel<float, 32>;
      if (own_logits && O <= 16 && H % 128 == 0 && logits_rows_enabled()) {
        if (lsm > 48 * 1024)
          STADE_CUDA(cudaFuncSetAttribute(mlp_logits_rows_kernel,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)lsm));
        mlp_logits_rows_kernel<<<2 * tc5::sm_count(), 256, lsm, s>>>(h, w2, w.zpart, S, H, O);
        STADE_CHECK_LAUNCH();
      } else if (own_logits) {
        auto lk = O <= 16 ? mlp_logits_kernel<16> : mlp_logits_kernel<32>;
        if (lsm > 48 * 1024)
          STADE_CUDA(cudaFuncSetAttribute(lk, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)lsm));
        lk<<<6 * tc5::sm_count(), 256, lsm, s>>>(h, w2, w.zpart, S, H, O);
        STADE_CHECK_LAUNCH();
      }
      kern<<<blocks, 256, 0, s>>>(w.zpart, own_logits ? 1 : tma_logit_parts(n_h), lossb, y, yb,
                                  b2, z, zb, p, pb, w.gbuf, S, O, w.loss_part);
      STADE_CHECK_LAUNCH();
      st = launch_sum_to_scalar(w.loss_part, blocks, loss, true, s);
    }
    if (st != STADE_OK) return st;
    // 3. s1b as hi / lo planes, hb consumed, W2b / b2b / b1b partials
    {
      PhaseScope ph("w2b", s);
      const int chunks = (S + kW2ChunkTc - 1) / kW2ChunkTc;
      const int no = O == 10 ? 12 : O <= 16 ? 16 : 32;   // g's pitch in shared memory
      const size_t smem = sizeof(float) * (size_t)kW2ChunkTc * no;
      auto kern = O == 10 ? mlp_s1b_planes_kernel<10>
                          : O <= 16 ? mlp_s1b_planes_kernel<16> : mlp_s1b_planes_kernel<32>;
      kern<<<dim3(chunks, (H + 255) / 256), 128, smem, s>>>(h, hb, w.gbuf, w2, w.s1b_hi, w.s1b_lo,
                                                            S, H, O, kW2ChunkTc, w.w2_part);
      STADE_CHECK_LAUNCH();
      // chunk partials -> kFinGroups group sums -> the three outputs, fixed order
      const int64_t len = n_h * n_o + n_o + n_h;
      const int per = (chunks + kFinGroups - 1) / kFinGroups;
      const int groups = (chunks + per - 1) / per;
      sum_groups_kernel<<<dim3(ceil_div_u(len, 256), groups), 256, 0, s>>>(w.w2_part, chunks, per,
                                                                          len, w.fin);
      STADE_CHECK_LAUNCH();
      finish_three_kernel<<<ceil_div_u(len, 256), 256, 0, s>>>(w.fin, groups, n_h * n_o, w2b, n_o,
                                                               b2b, n_h, b1b);
      STADE_CHECK_LAUNCH();
    }
    // 4. W1b = x^T s1b, 5. xb += s1b W1^T
    {
      PhaseScope ph("w1b_gemm", s);
      st = tma_weight_grad(x, w.x_lo, w.s1b_hi, w.s1b_lo, w1b, w.w1b_part, S, I, H, s);
    }
    if (st != STADE_OK) return st;
    {
      PhaseScope ph("xb_gemm", s);
      st = tma_input_grad(w.s1b_hi, w.s1b_lo, w1, w.w1_lo, xb, S, I, H, s);
    }
    return st;
  }

  // CUDA-core path
  // 1. h = tanh(x W1 + b1)
  {
    PhaseScope ph("fwd_gemm", s);
    st = gemm_simt<float, kF32RM, kF32RN, kF32BK, true, true>(
        S, H, I, LdRow<float>{x, I}, LdB<float>{w1, H}, EpiTanh<float>{{}, b1, h, H}, nullptr,
        1, s);
  }
  if (st != STADE_OK) return st;
  // 2. per-sample head
  {
    PhaseScope ph("head", s);
    const size_t head_smem = sizeof(float) * (size_t)(n_h * n_o);
    STADE_REQUIRE(head_smem <= 200 * 1024, "mlp2_ce_b: n_h * n_o too large");
    auto kern = O <= 16 ? mlp_head_b_kernel<float, 16> : mlp_head_b_kernel<float, 32>;
    if (head_smem > 48 * 1024)
      STADE_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      (int)head_smem));
    kern<<<w.head_blocks, kHeadWarps * 32, head_smem, s>>>(lossb, y, yb, w2, b2, h, hb, z, zb, p,
                                                           pb, w.gbuf, w.s1b, S, H, O, w.loss_part);
    STADE_CHECK_LAUNCH();
    st = launch_sum_to_scalar(w.loss_part, w.head_blocks, loss, true, s);
  }
  if (st != STADE_OK) return st;
  // 3. W2b, b2b
  {
    PhaseScope ph("w2b", s);
    auto kern = O <= 16 ? mlp_w2b_partial_kernel<float, 16> : mlp_w2b_partial_kernel<float, 32>;
    kern<<<w.w2_chunks, 256, 0, s>>>(h, w.gbuf, S, H, O, kW2Chunk, w.w2_part);
    STADE_CHECK_LAUNCH();
    finish_two_kernel<float><<<ceil_div_u(n_h * n_o + n_o, 256), 256, 0, s>>>(
        w.w2_part, w.w2_chunks, n_h * n_o, w2b, n_o, b2b);
    STADE_CHECK_LAUNCH();
  }
  // 4. W1b = x^T s1b (+ b1b as the row of ones), 5. xb += s1b W1^T
  {
    PhaseScope ph("w1b_gemm", s);
    st = gemm_simt<float, kF32RM, kF32RN, kF32BK, false, true>(
        I + 1, H, S, LdXtOnes<float>{x, I, I}, LdB<float>{w.s1b, H},
        EpiWeightBias<float>{{}, w1b, b1b, I, H}, w.w1_part, w.w1_splits, s);
  }
  if (st != STADE_OK) return st;
  {
    PhaseScope ph("xb_gemm", s);
    st = gemm_simt<float, kF32RM, kF32RN, kF32BK, true, false>(
        S, I, H, LdRow<float>{w.s1b, H}, LdBT<float>{w1, H}, EpiAddTo<float>{{}, xb, I},
        nullptr, 1, s);
  }
  return st;
}

// ============================================================================
// Float64 HVP
// ============================================================================
extern "C" size_t stade_mlp2_ce_hv_f64_workspace(int64_t n_s, int64_t n_i, int64_t n_h,
                                                 int64_t n_o) {
  if (n_s <= 0 || n_h <= 0 || n_o <= 0 || n_i < 0) return 256;
  SizerAlloc a;
  mlp_hv_layout(a, nullptr, n_s, n_i, n_h, n_o);
  return a.z.bytes();
}

extern "C" stade_status stade_mlp2_ce_hv_f64(
    double* loss, const double* lossb, const double* x, double* xb, const double* y, double* yb,
    const double* w1, double* w1b, const double* b1, double* b1b, const double* w2, double* w2b,
    const double* b2, double* b2b, double* h, double* hb, double* z, double* zb, double* p,
    double* pb, int64_t n_s, int64_t n_i, int64_t n_h, int64_t n_o, double* lossd,
    const double* lossbd, const double* xd, double* xbd, const double* yd, double* ybd,
    const double* w1d, double* w1bd, const double* b1d, double* b1bd, const double* w2d,
    double* w2bd, const double* b2d, double* b2bd, double* hd, double* hbd, double* zd,
    double* zbd, double* pd, double* pbd, const stade_opts* opts) {
  STADE_REQUIRE(n_s >= 0 && n_i >= 0 && n_h >= 0 && n_o >= 0, "mlp2_ce_hv: negative size");
  if (n_s == 0) return STADE_OK;
  STADE_REQUIRE(n_o >= 1 && n_o <= 32, "mlp2_ce_hv: n_o = %lld outside 1..32", (long long)n_o);
  STADE_REQUIRE(n_h > 0, "mlp2_ce_hv: n_h = 0 is not supported");
  STADE_REQUIRE(n_s <= (1 << 29) && n_i < (1 << 20) && n_h < (1 << 16),
                "mlp2_ce_hv: sizes out of range");
  STADE_REQUIRE(loss && lossb && x && xb && y && yb && w1 && w1b && b1 && b1b && w2 && w2b && b2 &&
                    b2b && h && hb && z && zb && p && pb && lossd && lossbd && xd && xbd && yd &&
                    ybd && w1d && w1bd && b1d && b1bd && w2d && w2bd && b2d && b2bd && hd && hbd &&
                    zd && zbd && pd && pbd,
                "mlp2_ce_hv: null array argument");
  cudaStream_t s = stream_of(opts);
  void* wsp = nullptr;
  stade_status st = get_workspace(opts, stade_mlp2_ce_hv_f64_workspace(n_s, n_i, n_h, n_o), &wsp);
  if (st != STADE_OK) return st;
  CarverAlloc ca(wsp);
  MlpF64HvWs w;
  mlp_hv_layout(ca, &w, n_s, n_i, n_h, n_o);
  const int S = (int)n_s, I = (int)n_i, H = (int)n_h, O = (int)n_o;

  // forward: S1 = x W1; s1d = x W1d + xd W1, h, hd
  {
    PhaseScope ph("hv_fwd_gemms", s);
    st = gemm_f64<true, true>(S, H, I, LdRow<double>{x, I},
                                                    LdB<double>{w1, H}, EpiStore{{}, w.s1, H},
                                                    nullptr, 1, s);
    if (st == STADE_OK)
      st = gemm_f64<true, true>(
          S, H, 2 * I, LdRow2{x, xd, I, I}, LdB2{w1d, w1, H, I},
          EpiTanhTangent{{}, w.s1, b1, b1d, h, hd, H}, nullptr, 1, s);
  }
  if (st != STADE_OK) return st;
  // head
  PhaseScope ph_head("hv_head", s);
  // w2 / w2d class-major, then (where they fit) each warp's h and hd rows
  const size_t w2_bytes = sizeof(double) * 2 * (size_t)O * (size_t)(H + 1);
  const size_t rows_bytes = sizeof(double) * kHvHeadWarps * 2 * (size_t)H;
  const int w2_smem = w2_bytes <= 160 * 1024;
  const int rows_smem = w2_smem && w2_bytes + rows_bytes <= 220 * 1024;
  const size_t hsm = w2_bytes + (rows_smem ? rows_bytes : 0);
  if (w2_smem && hsm > 48 * 1024)
    STADE_CUDA(cudaFuncSetAttribute(mlp_head_hv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)hsm));
  // with w2 in shared memory, one wave of the blocks the SMs hold at once
  // (each stages w2 once)
  int head_per_sm = 0;
  STADE_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&head_per_sm, mlp_head_hv_kernel,
                                                           kHvHeadWarps * 32, w2_smem ? hsm : 0));
  if (head_per_sm < 1) head_per_sm = 1;
  const int hgrid =
      w2_smem ? std::min(w.head_blocks, head_per_sm * tc5::sm_count()) : w.head_blocks;
  mlp_head_hv_kernel<<<hgrid, kHvHeadWarps * 32, w2_smem ? hsm : 0, s>>>(
      lossb, lossbd, y, yb, yd, ybd, w2, b2, w2d, b2d, h, hb, hd, hbd, z, zb, zd, zbd, p, pb, pd,
      pbd, w.gbuf, w.gdbuf, w.s1b, w.s1bd, S, H, O, w.loss_part, w.lossd_part, w2_smem,
      rows_smem);
  STADE_CHECK_LAUNCH();
  st = launch_sum_to_scalar(w.loss_part, hgrid, loss, true, s);
  if (st != STADE_OK) return st;
  st = launch_sum_to_scalar(w.lossd_part, hgrid, lossd, true, s);
  if (st != STADE_OK) return st;
  // W2b, W2bd, b2b, b2bd
  const dim3 w2g(w.w2_chunks, (H + 255) / 256);
  const size_t w2sm = sizeof(double) * kW2ChunkHv * 2 * (O <= 16 ? 16 : 32);
  if (O <= 16)
    mlp_w2b_hv_partial_kernel<16><<<w2g, 256, w2sm, s>>>(h, hd, w.gbuf, w.gdbuf, S, H, O,
                                                         kW2ChunkHv, w.w2_part);
  else
    mlp_w2b_hv_partial_kernel<32><<<w2g, 256, w2sm, s>>>(h, hd, w.gbuf, w.gdbuf, S, H, O,
                                                         kW2ChunkHv, w.w2_part);
  STADE_CHECK_LAUNCH();
  finish_four_kernel<<<ceil_div_u(2 * n_h * n_o + 2 * n_o, 256), 256, 0, s>>>(
      w.w2_part, w.w2_chunks, n_h * n_o, O, w2b, w2bd, b2b, b2bd);
  STADE_CHECK_LAUNCH();
  ph_head.end();
  // W1b (+ b1b); W1bd = x^T s1bd + xd^T s1b (+ b1bd)
  {
    PhaseScope ph("hv_w1b_gemms", s);
    st = gemm_f64<false, true>(
        I + 1, H, S, LdXtOnes<double>{x, I, I}, LdB<double>{w.s1b, H},
        EpiWeightBias<double>{{}, w1b, b1b, I, H}, w.w1_part, w.w1_splits, s);
    if (st == STADE_OK)
      st = gemm_f64<false, true>(
          I + 1, H, 2 * S, LdXtOnes2{x, xd, I, I, S}, LdB2{w.s1bd, w.s1b, H, S},
          EpiWeightBias<double>{{}, w1bd, b1bd, I, H}, w.w1_part, w.w1d_splits, s);
  }
  if (st != STADE_OK) return st;
  // xb += s1b W1^T; xbd += s1bd W1^T + s1b W1d^T
  {
    PhaseScope ph("hv_xb_gemms", s);
    st = gemm_f64<true, false>(S, I, H, LdRow<double>{w.s1b, H},
                                                     LdBT<double>{w1, H},
                                                     EpiAddTo<double>{{}, xb, I}, nullptr, 1, s);
    if (st == STADE_OK)
      st = gemm_f64<true, false>(
          S, I, 2 * H, LdRow2{w.s1bd, w.s1b, H, H}, LdBT2{w1, w1d, H, H},
          EpiAddTo<double>{{}, xbd, I}, nullptr, 1, s);
  }
  return st;
}

// ============================================================================
// Tangent sweep mlp2_ce_d (tgen_emit, src/STADE.jl:3271-3279): the primal in
// order with every active statement preceded by its tangent line, arguments
// in tgen_signature_args order (src/STADE.jl:3306-3316). Restated in
// oracle.cc mlp2_ce_d (the forward half of the HVP sweep).
// ============================================================================
namespace stade {
namespace {

template <class T>
struct EpiStoreT : EpiBase {  // dst[m, n] = acc
  T* dst;
  int ld;
  __device__ __forceinline__ void operator()(int m, int n, T acc) const {
    dst[(int64_t)m * ld + n] = acc;
  }
};
// s1d = acc + b1d (acc = sum x w1d + xd w1); h = tanh(S1 + b1); hd = (1 - h^2) s1d
template <class T>
struct EpiTanhTangentT : EpiBase {
  const T *s1, *b1, *b1d;
  T *h, *hd;
  int ld;
  __device__ __forceinline__ void operator()(int m, int n, T acc) const {
    const int64_t i = (int64_t)m * ld + n;
    const T s1d = acc + b1d[n];
    const T th = dtanh(s1[i] + b1[n]);
    hd[i] = (T(1) - th * th) * s1d;
    h[i] = th;
  }
};
template <class T>
struct LdRow2T {  // A(m, k) over two K segments [a0 | a1]
  const T *a0, *a1;
  int ld, k0;
  __device__ __forceinline__ T operator()(int m, int k) const {
    return k < k0 ? a0[(int64_t)m * ld + k] : a1[(int64_t)m * ld + (k - k0)];
  }
};
template <class T>
struct LdB2T {  // B(k, n) over two K segments [b0 ; b1]
  const T *b0, *b1;
  int ld, k0;
  __device__ __forceinline__ T operator()(int k, int n) const {
    return k < k0 ? b0[(int64_t)k * ld + n] : b1[(int64_t)(k - k0) * ld + n];
  }
};

// Per-sample head of the tangent sweep: logits and their tangents, the
// running max through max's partials, exp, the row sum and the loss with its
// tangent. One warp per sample, blocks strided over the samples.
template <class T, int NO>
__global__ void __launch_bounds__(kHeadWarps * 32)
mlp_head_d_kernel(const T* __restrict__ y, const T* __restrict__ yd, const T* __restrict__ w2,
                  const T* __restrict__ b2, const T* __restrict__ w2d,
                  const T* __restrict__ b2d, const T* __restrict__ h,
                  const T* __restrict__ hd, T* __restrict__ z, T* __restrict__ zd,
                  T* __restrict__ p, T* __restrict__ pd, int n_s, int n_h, int n_o,
                  T* __restrict__ loss_part, T* __restrict__ lossd_part) {
  __shared__ T red[2][kHeadWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  T loss_acc = T(0), lossd_acc = T(0);
  for (int s = blockIdx.x * kHeadWarps + warp; s < n_s; s += gridDim.x * kHeadWarps) {
    const T* hr = h + (int64_t)s * n_h;
    const T* hdr = hd + (int64_t)s * n_h;
    T zp[NO], zdp[NO];
#pragma unroll
    for (int c = 0; c < NO; ++c) { zp[c] = T(0); zdp[c] = T(0); }
    for (int k = lane; k < n_h; k += 32) {
      const T hv = hr[k], hdv = hdr[k];
#pragma unroll
      for (int c = 0; c < NO; ++c) {
        if (c < n_o) {
          const T wv = __ldg(w2 + (int64_t)k * n_o + c);
          zdp[c] += hv * __ldg(w2d + (int64_t)k * n_o + c) + wv * hdv;
          zp[c] += wv * hv;
        }
      }
    }
    T zv[NO], zdv[NO];
#pragma unroll
    for (int c = 0; c < NO; ++c) {
      zv[c] = c < n_o ? warp_sum(zp[c]) + b2[c] : T(0);
      zdv[c] = c < n_o ? warp_sum(zdp[c]) + b2d[c] : T(0);
    }
    T m = zv[0], md = zdv[0];
#pragma unroll
    for (int c = 1; c < NO; ++c) {
      if (c < n_o) {
        const T g1 = T(0.5) * (T(1) + dsign(m - zv[c]));
        const T g2 = T(0.5) * (T(1) + dsign(zv[c] - m));
        md = g1 * md + g2 * zdv[c];
        m = jmax(m, zv[c]);
      }
    }
    T pv[NO], pdv[NO];
    T rs = T(0), rsd = T(0);
#pragma unroll
    for (int c = 0; c < NO; ++c) {
      pv[c] = T(0);
      pdv[c] = T(0);
      if (c < n_o) {
        const T e = dexp(zv[c] - m);
        pdv[c] = e * (zdv[c] - md);
        pv[c] = e;
      }
    }
#pragma unroll
    for (int c = 0; c < NO; ++c)
      if (c < n_o) { rsd = rsd + pdv[c]; rs = rs + pv[c]; }
    const int64_t row = (int64_t)s * n_o;
#pragma unroll
    for (int c = 0; c < NO; ++c) {
      if (c < n_o) {
        const T yv = __ldg(y + row + c), ydv = __ldg(yd + row + c);
        const T q = pv[c] / rs;
        const T qd = pdv[c] / rs - (pv[c] / (rs * rs)) * rsd;
        lossd_acc = lossd_acc - (ydv * dlog(q) + yv * (qd / q));
        loss_acc = loss_acc - yv * dlog(q);
        if (lane == c) {
          z[row + c] = zv[c]; zd[row + c] = zdv[c];
          p[row + c] = pv[c]; pd[row + c] = pdv[c];
        }
      }
    }
  }
  if (lane == 0) { red[0][warp] = loss_acc; red[1][warp] = lossd_acc; }
  __syncthreads();
  if (threadIdx.x == 0) {
    T a = T(0), b = T(0);
    for (int w = 0; w < kHeadWarps; ++w) { a += red[0][w]; b += red[1][w]; }
    loss_part[blockIdx.x] = a;
    lossd_part[blockIdx.x] = b;
  }
}

constexpr int kHeadDBlocks = 4 * 148;

template <class T>
size_t mlp_d_workspace(int64_t n_s, int64_t n_h) {
  Sizer z;
  z.take<T>((size_t)(n_s * n_h));   // s1 = x W1
  z.take<T>(kHeadDBlocks);          // loss partials
  z.take<T>(kHeadDBlocks);          // lossd partials
  return z.bytes();
}

template <class T, int RM, int RN, int BK>
stade_status mlp2_ce_d_impl(T* loss, T* lossd, const T* x, const T* xd, const T* y, const T* yd,
                            const T* w1, const T* w1d, const T* b1, const T* b1d, const T* w2,
                            const T* w2d, const T* b2, const T* b2d, T* h, T* hd, T* z, T* zd,
                            T* p, T* pd, int64_t n_s, int64_t n_i, int64_t n_h, int64_t n_o,
                            const stade_opts* opts, const char* name) {
  STADE_REQUIRE(n_s >= 0 && n_i >= 0 && n_h >= 0 && n_o >= 0, "%s: negative size", name);
  if (n_s == 0) return STADE_OK;
  STADE_REQUIRE(n_o >= 1 && n_o <= 32, "%s: n_o = %lld outside 1..32", name, (long long)n_o);
  STADE_REQUIRE(n_h > 0, "%s: n_h = 0 is not supported", name);
  STADE_REQUIRE(n_s <= (1 << 29) && n_i < (1 << 20) && n_h < (1 << 16), "%s: sizes out of range",
                name);
  STADE_REQUIRE(loss && lossd && x && xd && y && yd && w1 && w1d && b1 && b1d && w2 && w2d && b2 &&
                    b2d && h && hd && z && zd && p && pd,
                "%s: null array argument", name);
  cudaStream_t s = stream_of(opts);
  void* wsp = nullptr;
  stade_status st = get_workspace(opts, mlp_d_workspace<T>(n_s, n_h), &wsp);
  if (st != STADE_OK) return st;
  Carver c(wsp);
  T* s1 = c.take<T>((size_t)(n_s * n_h));
  T* lp = c.take<T>(kHeadDBlocks);
  T* ldp = c.take<T>(kHeadDBlocks);
  const int S = (int)n_s, I = (int)n_i, H = (int)n_h, O = (int)n_o;
  {
    PhaseScope ph("d_gemms", s);
    if constexpr (std::is_same<T, double>::value) {
      st = gemm_f64<true, true>(S, H, I, LdRow<T>{x, I}, LdB<T>{w1, H}, EpiStoreT<T>{{}, s1, H},
                                nullptr, 1, s);
      if (st == STADE_OK)
        st = gemm_f64<true, true>(S, H, 2 * I, LdRow2T<T>{x, xd, I, I}, LdB2T<T>{w1d, w1, H, I},
                                  EpiTanhTangentT<T>{{}, s1, b1, b1d, h, hd, H}, nullptr, 1, s);
    } else {
      st = gemm_simt<T, RM, RN, BK, true, true>(S, H, I, LdRow<T>{x, I}, LdB<T>{w1, H},
                                                EpiStoreT<T>{{}, s1, H}, nullptr, 1, s);
      if (st == STADE_OK)
        st = gemm_simt<T, RM, RN, BK, true, true>(
            S, H, 2 * I, LdRow2T<T>{x, xd, I, I}, LdB2T<T>{w1d, w1, H, I},
            EpiTanhTangentT<T>{{}, s1, b1, b1d, h, hd, H}, nullptr, 1, s);
    }
  }
  if (st != STADE_OK) return st;
  PhaseScope ph("d_head", s);
  const int need = (S + kHeadWarps - 1) / kHeadWarps;
  const int blocks = need < kHeadDBlocks ? need : kHeadDBlocks;
  if (O <= 16)
    mlp_head_d_kernel<T, 16><<<blocks, kHeadWarps * 32, 0, s>>>(
        y, yd, w2, b2, w2d, b2d, h, hd, z, zd, p, pd, S, H, O, lp, ldp);
  else
    mlp_head_d_kernel<T, 32><<<blocks, kHeadWarps * 32, 0, s>>>(
        y, yd, w2, b2, w2d, b2d, h, hd, z, zd, p, pd, S, H, O, lp, ldp);
  STADE_CHECK_LAUNCH();
  st = launch_sum_to_scalar(lp, blocks, loss, true, s);
  if (st == STADE_OK) st = launch_sum_to_scalar(ldp, blocks, lossd, true, s);
  return st;
}

}  // namespace
}  // namespace stade

#define MLP_D_SIG(T)                                                                          \
  T *loss, T *lossd, const T *x, const T *xd, const T *y, const T *yd, const T *w1,           \
      const T *w1d, const T *b1, const T *b1d, const T *w2, const T *w2d, const T *b2,        \
      const T *b2d, T *h, T *hd, T *z, T *zd, T *p, T *pd, int64_t n_s, int64_t n_i,          \
      int64_t n_h, int64_t n_o, const stade_opts *opts
#define MLP_D_FWD loss, lossd, x, xd, y, yd, w1, w1d, b1, b1d, w2, w2d, b2, b2d, h, hd, z, zd, p, \
      pd, n_s, n_i, n_h, n_o, opts

extern "C" size_t stade_mlp2_ce_d_f32_workspace(int64_t n_s, int64_t n_i, int64_t n_h,
                                                int64_t n_o) {
  (void)n_i; (void)n_o;
  return n_s > 0 && n_h > 0 ? stade::mlp_d_workspace<float>(n_s, n_h) : 256;
}
extern "C" size_t stade_mlp2_ce_d_f64_workspace(int64_t n_s, int64_t n_i, int64_t n_h,
                                                int64_t n_o) {
  (void)n_i; (void)n_o;
  return n_s > 0 && n_h > 0 ? stade::mlp_d_workspace<double>(n_s, n_h) : 256;
}
extern "C" stade_status stade_mlp2_ce_d_f32(MLP_D_SIG(float)) {
  return stade::mlp2_ce_d_impl<float, stade::kF32RM, stade::kF32RN, stade::kF32BK>(
      MLP_D_FWD, "mlp2_ce_d");
}
extern "C" stade_status stade_mlp2_ce_d_f64(MLP_D_SIG(double)) {
  return stade::mlp2_ce_d_impl<double, stade::kF64RM, stade::kF64RN, stade::kF64BK>(
      MLP_D_FWD, "mlp2_ce_d");
}
