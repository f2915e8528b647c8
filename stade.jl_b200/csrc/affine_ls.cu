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
// Here each block owns a contiguous chunk of samples and writes its partial
// wb / bb / loss; a second kernel sums the partials in block order. No
// floating-point atomics, bit-identical results from call to call.
//
// y, tb and xb follow the oracle's statement order with separate multiply and
// add roundings (no FMA contraction), so they match it bit for bit.

#include "common.cuh"

namespace stade {
namespace {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads)
affine_ls_chunk_kernel(const double* __restrict__ lossb, const double* __restrict__ w,
                       const double* __restrict__ b, const double* __restrict__ x,
                       double* __restrict__ xb, const double* __restrict__ t,
                       double* __restrict__ tb, double* __restrict__ y,
                       double* __restrict__ yb, int64_t n_s, int n_o, int n_i,
                       int chunk, double* __restrict__ part) {
  extern __shared__ double sm[];
  double* ws = sm;                     // n_o * n_i
  double* xs = ws + (size_t)n_o * n_i; // chunk * n_i
  double* gs = xs + (size_t)chunk * n_i;  // chunk * n_o
  __shared__ double red[kThreads / 32];

  const int64_t s0 = (int64_t)blockIdx.x * chunk;
  const int ns = (int)((int64_t)chunk < n_s - s0 ? (int64_t)chunk : n_s - s0);
  const int nw = n_o * n_i;
  for (int e = threadIdx.x; e < nw; e += blockDim.x) ws[e] = w[e];
  for (int e = threadIdx.x; e < ns * n_i; e += blockDim.x) xs[e] = x[s0 * n_i + e];
  __syncthreads();

  const double lb = lossb[0];
  double loss_acc = 0.0;
  // forward and the residual adjoint, one thread per (sample, output)
  for (int e = threadIdx.x; e < ns * n_o; e += blockDim.x) {
    const int sl = e / n_o, o = e % n_o;
    double s = b[o];
    const double* wr = ws + (size_t)o * n_i;
    const double* xr = xs + (size_t)sl * n_i;
    for (int k = 0; k < n_i; ++k) s = __dadd_rn(s, __dmul_rn(wr[k], xr[k]));
    const int64_t gi = s0 * n_o + e;
    y[gi] = s;
    const double d = __dadd_rn(s, -t[gi]);
    loss_acc = __dadd_rn(loss_acc, __dmul_rn(0.5, __dmul_rn(d, d)));
    const double r = __dmul_rn(__dmul_rn(0.5, __dmul_rn(2.0, d)), lb);
    tb[gi] = __dadd_rn(tb[gi], -r);
    gs[e] = __dadd_rn(yb[gi], r);  // yb += r, then consumed
    yb[gi] = 0.0;
  }
  __syncthreads();
  // xb[s,k] += sum over o = n_o-1 .. 0 of w[o,k] g[s,o] (the oracle's order)
  for (int e = threadIdx.x; e < ns * n_i; e += blockDim.x) {
    const int sl = e / n_i, k = e % n_i;
    const int64_t gi = s0 * n_i + e;
    double acc = xb[gi];
    const double* gr = gs + (size_t)sl * n_o;
    for (int o = n_o - 1; o >= 0; --o) acc = __dadd_rn(acc, __dmul_rn(ws[(size_t)o * n_i + k], gr[o]));
    xb[gi] = acc;
  }
  // partial wb[o,k] and bb[o] over this chunk, samples in descending order
  double* my = part + (size_t)blockIdx.x * (nw + n_o + 1);
  for (int e = threadIdx.x; e < nw + n_o; e += blockDim.x) {
    double acc = 0.0;
    if (e < nw) {
      const int o = e / n_i, k = e % n_i;
      for (int sl = ns - 1; sl >= 0; --sl)
        acc = fma(xs[(size_t)sl * n_i + k], gs[(size_t)sl * n_o + o], acc);
    } else {
      const int o = e - nw;
      for (int sl = ns - 1; sl >= 0; --sl) acc += gs[(size_t)sl * n_o + o];
    }
    my[e] = acc;
  }
  loss_acc = block_sum(loss_acc, red);
  if (threadIdx.x == 0) my[nw + n_o] = loss_acc;
}

// wb, bb and loss are contiguous-free caller arrays: one fixed-order pass
// over the block partials adds into each of them.
__global__ void affine_ls_finish_kernel(const double* __restrict__ part, int nblk, int n_o,
                                        int n_i, double* __restrict__ wb,
                                        double* __restrict__ bb, double* __restrict__ loss) {
  const int nw = n_o * n_i;
  const int len = nw + n_o + 1;
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= len) return;
  const double acc = ordered_sum(part + e, nblk, len, true);
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
  // about 16 samples per block: enough blocks to spread the 3 * n_s * n_o * n_i
  // multiply-adds, few enough partials to sum quickly
  p.chunk = 16;
  p.nblk = (int)((n_s + p.chunk - 1) / p.chunk);
  p.smem = sizeof(double) * ((size_t)n_o * n_i + (size_t)p.chunk * n_i + (size_t)p.chunk * n_o);
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
  affine_ls_finish_kernel<<<ceil_div_u(len, 256), 256, 0, s>>>(part, p.nblk, (int)n_o, (int)n_i,
                                                                wb, bb, loss);
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

// 2 MiB: enough for the full configuration (1024 x 64 x 32 needs 1.03 MiB).
constexpr size_t kNoAllocScratchDoubles = (size_t(2) << 20) / sizeof(double);
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
  affine_ls_finish_kernel<<<ceil_div_u(len, 256), 256, 0, s>>>(part, p.nblk, (int)n_o, (int)n_i,
                                                                wb, bb, loss);
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
