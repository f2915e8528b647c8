// C1 affine_ls_b: batched affine map + least-squares loss adjoint, Float64.
//
// Generated sweep being replaced (restated in oracle.cc, pattern of
// test/val-corpus/affine_loss_b.jl:5-23 and matvec_loss_b.jl:5-27):
//   forward:  y[s,o] = b[o] + sum_k w[o,k] x[s,k];  loss += 0.5 (y - t)^2
//   backward: r = (0.5 (2 (y - t))) lossb; yb += r; tb += -r
//             g = yb (consumed, yb = 0); xb[s,k] += sum_o w[o,k] g[s,o]
//             wb[o,k] += sum_s x[s,k] g[s,o];  bb[o] += sum_s g[s,o]
//
// The generated CUDA.jl port turns `wb[o,k] += ...` into atomics on 2,048
// addresses from 1,024 samples (cgen_device_assign, src/STADE.jl:11941).
// Here each block owns a contiguous chunk of samples, stages everything it
// reads in shared memory with all of those loads in flight at once, and
// writes its partial wb / bb / loss; a second kernel sums the partials in a
// fixed order. No floating-point atomics, bit-identical results from call to
// call. The whole sweep is a few microseconds of arithmetic, so what these
// two kernels are built around is memory latency, not bandwidth.
//
// y, tb and xb follow the oracle's statement order with separate multiply and
// add roundings (no FMA contraction), so they match it bit for bit.

#include "common.cuh"

namespace stade {
namespace {

constexpr int kThreads = 512;

// Global -> shared copy with `U` loads per thread in flight before any store
// (one memory latency for a block's whole staging instead of one per pass).
template <int U>
__device__ __forceinline__ void stage(double* __restrict__ dst, const double* __restrict__ src,
                                      int n) {
  for (int base = threadIdx.x; base < n; base += U * kThreads) {
    double r[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * kThreads;
      r[u] = i < n ? src[i] : 0.0;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * kThreads;
      if (i < n) dst[i] = r[u];
    }
  }
}

// Rows of `cols` doubles copied to a pitch of `ld` (U loads in flight).
template <int U>
__device__ __forceinline__ void stage_rows(double* __restrict__ dst, int ld,
                                           const double* __restrict__ src, int rows, int cols) {
  const int n = rows * cols;
  for (int base = threadIdx.x; base < n; base += U * kThreads) {
    double r[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * kThreads;
      r[u] = i < n ? src[i] : 0.0;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = base + u * kThreads;
      if (i < n) dst[(i / cols) * ld + i % cols] = r[u];
    }
  }
}

// Pitch of w's rows in shared memory: odd, so the forward's 32 lanes (32
// outputs o, the same k) read 32 different banks instead of one.
__host__ __device__ constexpr int w_pitch(int n_i) { return n_i | 1; }

__global__ void __launch_bounds__(kThreads)
affine_ls_chunk_kernel(const double* __restrict__ lossb, const double* __restrict__ w,
                       const double* __restrict__ b, const double* __restrict__ x,
                       double* __restrict__ xb, const double* __restrict__ t,
                       double* __restrict__ tb, double* __restrict__ y,
                       double* __restrict__ yb, int64_t n_s, int n_o, int n_i,
                       int chunk, double* __restrict__ part) {
  extern __shared__ double sm[];
  const int ldw = w_pitch(n_i);
  double* ws = sm;                           // n_o rows of pitch ldw
  double* xs = ws + (size_t)n_o * ldw;       // chunk * n_i
  double* xbs = xs + (size_t)chunk * n_i;    // chunk * n_i
  double* gs = xbs + (size_t)chunk * n_i;    // chunk * n_o: t, then g
  double* tbs = gs + (size_t)chunk * n_o;    // chunk * n_o
  double* ybs = tbs + (size_t)chunk * n_o;   // chunk * n_o
  double* bs = ybs + (size_t)chunk * n_o;    // n_o
  __shared__ double red[kThreads / 32];

  const int64_t s0 = (int64_t)blockIdx.x * chunk;
  const int ns = (int)((int64_t)chunk < n_s - s0 ? (int64_t)chunk : n_s - s0);
  const int nw = n_o * n_i;
  // everything the block reads, staged up front
  stage_rows<8>(ws, ldw, w, n_o, n_i);
  stage<4>(xs, x + s0 * n_i, ns * n_i);
  stage<4>(xbs, xb + s0 * n_i, ns * n_i);
  stage<2>(gs, t + s0 * n_o, ns * n_o);
  stage<2>(tbs, tb + s0 * n_o, ns * n_o);
  stage<2>(ybs, yb + s0 * n_o, ns * n_o);
  stage<1>(bs, b, n_o);
  __syncthreads();

  const double lb = lossb[0];
  double loss_acc = 0.0;
  // forward and the residual adjoint, one thread per (sample, output)
  for (int e = threadIdx.x; e < ns * n_o; e += blockDim.x) {
    const int sl = e / n_o, o = e % n_o;
    double s = bs[o];
    const double* wr = ws + (size_t)o * ldw;
    const double* xr = xs + (size_t)sl * n_i;
    for (int k = 0; k < n_i; ++k) s = __dadd_rn(s, __dmul_rn(wr[k], xr[k]));
    const int64_t gi = s0 * n_o + e;
    y[gi] = s;
    const double d = __dadd_rn(s, -gs[e]);
    loss_acc = __dadd_rn(loss_acc, __dmul_rn(0.5, __dmul_rn(d, d)));
    const double r = __dmul_rn(__dmul_rn(0.5, __dmul_rn(2.0, d)), lb);
    tb[gi] = __dadd_rn(tbs[e], -r);
    gs[e] = __dadd_rn(ybs[e], r);  // yb += r, then consumed
    yb[gi] = 0.0;
  }
  __syncthreads();
  // xb[s,k] += sum over o = n_o-1 .. 0 of w[o,k] g[s,o] (the oracle's order);
  // each thread runs two elements' chains side by side (the additions of one
  // chain depend on each other: two chains hide half the latency)
  const int nx = ns * n_i;
  for (int e0 = threadIdx.x; e0 < nx; e0 += 2 * kThreads) {
    const int e1 = e0 + kThreads < nx ? e0 + kThreads : e0;
    const int k0 = e0 % n_i, k1 = e1 % n_i;
    const double* g0 = gs + (size_t)(e0 / n_i) * n_o;
    const double* g1 = gs + (size_t)(e1 / n_i) * n_o;
    double a0 = xbs[e0], a1 = xbs[e1];
    for (int o = n_o - 1; o >= 0; --o) {
      const double* wr = ws + (size_t)o * ldw;
      a0 = __dadd_rn(a0, __dmul_rn(wr[k0], g0[o]));
      a1 = __dadd_rn(a1, __dmul_rn(wr[k1], g1[o]));
    }
    xb[s0 * n_i + e0] = a0;
    if (e1 != e0) xb[s0 * n_i + e1] = a1;
  }
  // partial wb[o,k] and bb[o] over this chunk, samples in descending order,
  // four elements' chains side by side
  double* my = part + (size_t)blockIdx.x * (nw + n_o + 1);
  const int np = nw + n_o;
  for (int e0 = threadIdx.x; e0 < np; e0 += 4 * kThreads) {
    double acc[4];
    int oo[4], kk[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int e = e0 + u * kThreads < np ? e0 + u * kThreads : e0;
      acc[u] = 0.0;
      oo[u] = e < nw ? e / n_i : e - nw;
      kk[u] = e < nw ? e % n_i : -1;   // -1: a bb element (sum of g alone)
    }
    for (int sl = ns - 1; sl >= 0; --sl) {
      const double* xr = xs + (size_t)sl * n_i;
      const double* gr = gs + (size_t)sl * n_o;
#pragma unroll
      for (int u = 0; u < 4; ++u)
        acc[u] = kk[u] >= 0 ? fma(xr[kk[u]], gr[oo[u]], acc[u]) : acc[u] + gr[oo[u]];
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (u == 0 || e0 + u * kThreads < np) my[e0 + u * kThreads] = acc[u];
  }
  loss_acc = block_sum(loss_acc, red);
  if (threadIdx.x == 0) my[nw + n_o] = loss_acc;
}

// wb, bb and loss: each element's block partials summed by 8 lanes (lane j
// adds blocks j, j + 8, ... in order, all its loads in flight), then the 8
// lane sums in a fixed tree; the same order on every call.
constexpr int kFinLanes = 8;
__global__ void __launch_bounds__(256)
affine_ls_finish_kernel(const double* __restrict__ part, int nblk, int n_o, int n_i,
                        double* __restrict__ wb, double* __restrict__ bb,
                        double* __restrict__ loss) {
  const int nw = n_o * n_i;
  const int len = nw + n_o + 1;
  const int tid = blockIdx.x * blockDim.x + threadIdx.x;
  const int e = tid / kFinLanes, j = tid % kFinLanes;
  double acc = 0.0;
  if (e < len) {
    constexpr int U = 8;
    for (int q0 = j; q0 < nblk; q0 += U * kFinLanes) {
      double r[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int q = q0 + u * kFinLanes;
        r[u] = q < nblk ? part[(size_t)q * len + e] : 0.0;
      }
#pragma unroll
      for (int u = 0; u < U; ++u) acc += r[u];
    }
  }
#pragma unroll
  for (int off = 1; off < kFinLanes; off <<= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (e >= len || j != 0) return;
  if (e < nw) wb[e] += acc;
  else if (e < nw + n_o) bb[e - nw] += acc;
  else loss[0] += acc;
}

struct Plan {
  int chunk, nblk;
  size_t smem;
};

Plan plan(int64_t n_s, int64_t n_o, int64_t n_i) {
  Plan p;
  // 8 samples per block: the sweep is latency-bound (a few microseconds of
  // arithmetic), so it is spread over as many SMs as the batch allows (1024
  // samples: 128 blocks); the partials stay few enough to sum in one pass
  p.chunk = 8;
  p.nblk = (int)((n_s + p.chunk - 1) / p.chunk);
  p.smem = sizeof(double) * ((size_t)n_o * w_pitch((int)n_i) + 2 * (size_t)p.chunk * n_i +
                             3 * (size_t)p.chunk * n_o + n_o);
  return p;
}

}  // namespace
}  // namespace stade

using namespace stade;

extern "C" size_t stade_affine_ls_b_f64_workspace(int64_t n_s, int64_t n_o, int64_t n_i) {
  if (n_s <= 0 || n_o <= 0 || n_i < 0) return 0;
  const Plan p = plan(n_s, n_o, n_i);
  Sizer z;
  z.take<double>((size_t)p.nblk * (size_t)(n_o * n_i + n_o + 1));
  return z.bytes();
}

extern "C" stade_status stade_affine_ls_b_f64(double* loss, const double* lossb, const double* w,
                                              double* wb, const double* b, double* bb,
                                              const double* x, double* xb, const double* t,
                                              double* tb, double* y, double* yb, int64_t n_s,
                                              int64_t n_o, int64_t n_i, const stade_opts* opts) {
  STADE_REQUIRE(n_s >= 0 && n_o >= 0 && n_i >= 0, "affine_ls_b: negative size");
  if (n_s == 0 || n_o == 0) return STADE_OK;  // every loop has zero trips
  STADE_REQUIRE(loss && lossb && w && wb && b && bb && x && xb && t && tb && y && yb,
                "affine_ls_b: null array argument");
  const Plan p = plan(n_s, n_o, n_i);
  STADE_REQUIRE(p.smem <= 200 * 1024, "affine_ls_b: n_o * n_i = %lld too large for one block",
                (long long)(n_o * n_i));
  STADE_REQUIRE(n_s < (int64_t(1) << 31) / 2 && n_o * n_i < (int64_t(1) << 30),
                "affine_ls_b: size overflow");
  cudaStream_t s = stream_of(opts);
  void* wsp = nullptr;
  stade_status st = get_workspace(opts, stade_affine_ls_b_f64_workspace(n_s, n_o, n_i), &wsp);
  if (st != STADE_OK) return st;
  Carver c(wsp);
  double* part = c.take<double>((size_t)p.nblk * (size_t)(n_o * n_i + n_o + 1));
  if (p.smem > 48 * 1024)
    STADE_CUDA(cudaFuncSetAttribute(affine_ls_chunk_kernel,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem));
  PhaseScope ph("affine", s);
  affine_ls_chunk_kernel<<<p.nblk, kThreads, p.smem, s>>>(lossb, w, b, x, xb, t, tb, y, yb, n_s,
                                                          (int)n_o, (int)n_i, p.chunk, part);
  STADE_CHECK_LAUNCH();
  const int len = (int)(n_o * n_i + n_o + 1);
  affine_ls_finish_kernel<<<ceil_div_u((int64_t)len * kFinLanes, 256), 256, 0, s>>>(
      part, p.nblk, (int)n_o, (int)n_i, wb, bb, loss);
  STADE_CHECK_LAUNCH();
  return STADE_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free variant of stade_affine_ls_b_f64.
//
// Some callers cannot allocate device memory at the point where they run the
// sweep: an application that has handed all device memory to its own pool, a
// real-time loop with a fixed memory plan, or a host thread that must not
// block (cudaMalloc may synchronize the device). They also may not be able to
// size and pass a workspace. This entry point takes its scratch (the per-block
// partial sums) from a fixed array that lives in the library's own device
// memory instead, so it calls no cudaMalloc, cudaFree or allocating library
// routine. The array is created when the library's device code is loaded on
// a device and is held until the process exits.
namespace stade {
namespace {

// 4 MiB: enough for the full configuration (1024 x 64 x 32 needs 2.03 MiB).
constexpr size_t kNoAllocScratchDoubles = (size_t(4) << 20) / sizeof(double);
static __device__ __align__(256) double g_affine_noalloc_scratch[kNoAllocScratchDoubles];

// Device address of the scratch array on the current device. In host code the
// array's name is only a host-side stand-in, never a device address, so the
// address is looked up with the device current. The lookup is a query (it
// allocates nothing) and runs on every call, so a cudaDeviceReset between
// calls, which reloads the library's device code at a new address, is
// harmless; the first call on a device also loads that code there.
stade_status noalloc_scratch(double** out) {
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_affine_noalloc_scratch);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress", __FILE__, __LINE__);
  *out = static_cast<double*>(p);
  return STADE_OK;
}

}  // namespace
}  // namespace stade

extern "C" size_t stade_affine_ls_b_f64_noalloc_max_scratch(void) {
  return stade::kNoAllocScratchDoubles * sizeof(double);
}

extern "C" stade_status stade_affine_ls_b_f64_noalloc(double* loss, const double* lossb,
                                                      const double* w, double* wb, const double* b,
                                                      double* bb, const double* x, double* xb,
                                                      const double* t, double* tb, double* y,
                                                      double* yb, int64_t n_s, int64_t n_o,
                                                      int64_t n_i, const stade_opts* opts) {
  STADE_REQUIRE(n_s >= 0 && n_o >= 0 && n_i >= 0, "affine_ls_b_noalloc: negative size");
  if (n_s == 0 || n_o == 0) return STADE_OK;
  STADE_REQUIRE(loss && lossb && w && wb && b && bb && x && xb && t && tb && y && yb,
                "affine_ls_b_noalloc: null array argument");
  const Plan p = plan(n_s, n_o, n_i);
  STADE_REQUIRE(p.smem <= 200 * 1024, "affine_ls_b_noalloc: n_o * n_i = %lld too large for one block",
                (long long)(n_o * n_i));
  STADE_REQUIRE(n_s < (int64_t(1) << 31) / 2 && n_o * n_i < (int64_t(1) << 30),
                "affine_ls_b_noalloc: size overflow");
  const size_t need = (size_t)p.nblk * (size_t)(n_o * n_i + n_o + 1);
  if (need > kNoAllocScratchDoubles)
    return fail(STADE_EINVAL,
                "affine_ls_b_noalloc: %zu bytes of scratch needed, the fixed array holds %zu "
                "(n_s = %lld, n_o = %lld, n_i = %lld); use stade_affine_ls_b_f64",
                need * sizeof(double), kNoAllocScratchDoubles * sizeof(double), (long long)n_s,
                (long long)n_o, (long long)n_i);
  double* part = nullptr;
  stade_status st = noalloc_scratch(&part);
  if (st != STADE_OK) return st;
  cudaStream_t s = stream_of(opts);
  if (p.smem > 48 * 1024)
    STADE_CUDA(cudaFuncSetAttribute(affine_ls_chunk_kernel,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem));
  PhaseScope ph("affine", s);
  // every block writes all of its partial slots, so nothing needs clearing
  affine_ls_chunk_kernel<<<p.nblk, kThreads, p.smem, s>>>(lossb, w, b, x, xb, t, tb, y, yb, n_s,
                                                          (int)n_o, (int)n_i, p.chunk, part);
  STADE_CHECK_LAUNCH();
  const int len = (int)(n_o * n_i + n_o + 1);
  affine_ls_finish_kernel<<<ceil_div_u((int64_t)len * kFinLanes, 256), 256, 0, s>>>(
      part, p.nblk, (int)n_o, (int)n_i, wb, bb, loss);
  STADE_CHECK_LAUNCH();
  return STADE_OK;
}

// ---------------------------------------------------------------------------
// Tangent sweep affine_ls_d (tgen_emit, src/STADE.jl:3271-3279; restated in
// oracle.cc affine_ls_d): one thread per (sample, output) computes y and yd
// in the primal's statement order; loss / lossd per-block partials.
namespace stade {
namespace {

__global__ void __launch_bounds__(256)
affine_ls_d_kernel(const double* __restrict__ w, const double* __restrict__ wd,
                   const double* __restrict__ b, const double* __restrict__ bd,
                   const double* __restrict__ x, const double* __restrict__ xd,
                   const double* __restrict__ t, const double* __restrict__ td,
                   double* __restrict__ y, double* __restrict__ yd, int64_t n_s, int n_o,
                   int n_i, double* __restrict__ part) {
  __shared__ double red[32];
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  double l = 0.0, ld = 0.0;
  if (idx < n_s * n_o) {
    const int64_t i_s = idx / n_o;
    const int i_o = (int)(idx % n_o);
    double sd = bd[i_o], s = b[i_o];
    for (int k = 0; k < n_i; ++k) {
      const double wv = w[(int64_t)i_o * n_i + k], xv = x[i_s * n_i + k];
      sd = __dadd_rn(sd, __dadd_rn(__dmul_rn(wd[(int64_t)i_o * n_i + k], xv),
                                   __dmul_rn(wv, xd[i_s * n_i + k])));
      s = __dadd_rn(s, __dmul_rn(wv, xv));
    }
    yd[idx] = sd;
    y[idx] = s;
    const double dl = __dadd_rn(s, -t[idx]);
    ld = __dmul_rn(0.5, __dmul_rn(__dmul_rn(2.0, dl), __dadd_rn(sd, -td[idx])));
    l = __dmul_rn(0.5, __dmul_rn(dl, dl));
  }
  l = block_sum(l, red);
  __syncthreads();
  ld = block_sum(ld, red);
  if (threadIdx.x == 0) {
    part[blockIdx.x] = l;
    part[gridDim.x + blockIdx.x] = ld;
  }
}

}  // namespace
}  // namespace stade

extern "C" size_t stade_affine_ls_d_f64_workspace(int64_t n_s, int64_t n_o, int64_t n_i) {
  (void)n_i;
  if (n_s <= 0 || n_o <= 0) return 256;
  Sizer z;
  z.take<double>(2 * (size_t)ceil_div_u(n_s * n_o, 256));
  return z.bytes();
}

extern "C" stade_status stade_affine_ls_d_f64(double* loss, double* lossd, const double* w,
                                              const double* wd, const double* b,
                                              const double* bd, const double* x,
                                              const double* xd, const double* t,
                                              const double* td, double* y, double* yd,
                                              int64_t n_s, int64_t n_o, int64_t n_i,
                                              const stade_opts* opts) {
  STADE_REQUIRE(n_s >= 0 && n_o >= 0 && n_i >= 0, "affine_ls_d: negative size");
  if (n_s == 0 || n_o == 0) return STADE_OK;
  STADE_REQUIRE(loss && lossd && w && wd && b && bd && x && xd && t && td && y && yd,
                "affine_ls_d: null array argument");
  STADE_REQUIRE(n_s * n_o < (int64_t(1) << 40) && n_i < (1 << 30), "affine_ls_d: size overflow");
  cudaStream_t s = stream_of(opts);
  void* wsp = nullptr;
  stade_status st = get_workspace(opts, stade_affine_ls_d_f64_workspace(n_s, n_o, n_i), &wsp);
  if (st != STADE_OK) return st;
  const unsigned blocks = ceil_div_u(n_s * n_o, 256);
  Carver c(wsp);
  double* part = c.take<double>(2 * (size_t)blocks);
  affine_ls_d_kernel<<<blocks, 256, 0, s>>>(w, wd, b, bd, x, xd, t, td, y, yd, n_s, (int)n_o,
                                            (int)n_i, part);
  STADE_CHECK_LAUNCH();
  st = launch_sum_to_scalar(part, blocks, loss, true, s);
  if (st == STADE_OK) st = launch_sum_to_scalar(part + blocks, (int64_t)blocks, lossd, true, s);
  return st;
}
