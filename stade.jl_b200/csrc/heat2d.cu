// C3 heat2d_b: adjoint of n_step explicit periodic 5-point heat steps on an
// n x n Float64 grid, with the per-step tape of the generated sweep.
//
// Generated sweep being replaced (restated in oracle.cc; time loop and tape of
// test/val-corpus/advection_b.jl:1-37, scatter adjoint of
// stencil_loss_b.jl:12-21, periodic gather of cgen_gather_loop /
// cgen_gather_periodic_inverse, src/STADE.jl:7343-7532):
//   forward  step t: un = u + alpha ((((u_up + u_dn) + u_lf) + u_rt) - 4 u);
//            tape[t] = u; u = un.           loss += sum u^2
//   backward ub += 2 u lossb; per step t (reverse): u = tape[t];
//            unb += ub, ub = 0; scatter unb through the stencil into ub and
//            alphab += (lap u) unb, unb = 0.
//
// B200 mapping. The tape IS the sequence of states: the forward step t reads
// tape[t-1] (u for t = 1) and writes tape[t] (un for the last step), so every
// state is written once and read once per sweep. The scatter adjoint is
// turned into a gather (each thread owns its output cells, no atomics); in the
// interior the five contributions are added in the order the generated
// reverse loop adds them, so interior cells match the oracle bit for bit.
// Each thread owns two adjacent columns (16-byte loads) over a strip of rows,
// keeping the rows above and below in registers; horizontal neighbours come
// from the neighbouring lanes by warp shuffle. alphab and loss are summed per
// block, then over blocks in a fixed order.
#include <cstdlib>
#include <cstring>
#include <utility>

#include "common.cuh"
#include "halo.cuh"
#include "tcgen05.cuh"

namespace stade {
namespace {

constexpr int kThreads = 128;   // 128 threads x 2 columns = 256 columns per block
constexpr int kColsPerBlock = 2 * kThreads;
constexpr int kRowsFwd = 16;
constexpr int kRowsBwd = 8;
constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ double2 ld2(const double* __restrict__ p, int64_t row, int n, int j) {
  return __ldg(reinterpret_cast<const double2*>(p + row * (int64_t)n + j));
}

// Horizontal neighbours of the thread's two columns (j, j+1) on one row.
__device__ __forceinline__ void hnbrs(const double* __restrict__ p, int64_t row, int n, int j,
                                      double2 c, int lane, double& left_of_j,
                                      double& right_of_j1) {
  left_of_j = __shfl_up_sync(kFull, c.y, 1);
  right_of_j1 = __shfl_down_sync(kFull, c.x, 1);
  if (lane == 0) left_of_j = __ldg(p + row * (int64_t)n + (j == 0 ? n - 1 : j - 1));
  if (lane == 31 || j + 2 >= n) right_of_j1 = __ldg(p + row * (int64_t)n + (j + 2 >= n ? j + 2 - n : j + 2));
}

__device__ __forceinline__ double heat_point(double c, double up, double dn, double lf, double rt,
                                             double alpha) {
  // c + alpha * ((((up + dn) + lf) + rt) - 4.0 * c), two roundings per a*b+c
  double s = __dadd_rn(__dadd_rn(__dadd_rn(up, dn), lf), rt);
  s = __dadd_rn(s, -__dmul_rn(4.0, c));
  return __dadd_rn(c, __dmul_rn(alpha, s));
}

// One forward step: dst = step(src); optionally copy_dst = src (tape slot 0)
// and a per-block partial of sum(dst^2) (the loss, last step only).
// Rows handled by one launch: block row y starts at row_lo + y * row_step and
// covers R rows, stopping at row_hi. kWrap: the whole periodic grid (row_lo 0,
// row_hi n, row indices wrap). !kWrap: a slab with one halo row above (row -1)
// and below (row `rows`) already filled, rows addressed without wrapping; the
// loads of a strip's tail past row_hi are clamped to row_hi so they stay inside
// the halo-padded slab.
template <bool kWrap>
__device__ __forceinline__ void strip_rows(int i, int n, int row_hi, int& iw, int& idn) {
  if (kWrap) {
    iw = i % n;                    // rows past n (n % R != 0) are not stored
    idn = iw + 1 == n ? 0 : iw + 1;
  } else {
    iw = i < row_hi ? i : row_hi;
    idn = i + 1 < row_hi ? i + 1 : row_hi;
  }
}

template <int R, bool kWrap>
__global__ void __launch_bounds__(kThreads)
heat_fwd_kernel(const double* __restrict__ src, double* __restrict__ dst,
                double* __restrict__ copy_dst, double alpha, int n, int row_lo, int row_step,
                int row_hi, double* __restrict__ loss_part) {
  __shared__ double red[kThreads / 32];
  const int lane = threadIdx.x & 31;
  const int j_raw = blockIdx.x * kColsPerBlock + threadIdx.x * 2;
  const bool col_ok = j_raw < n;
  const int j = col_ok ? j_raw : n - 2;
  const int i0 = row_lo + blockIdx.y * row_step;
  const int row_up = kWrap ? (i0 == 0 ? n - 1 : i0 - 1) : i0 - 1;
  double2 up = ld2(src, row_up, n, j);
  double2 cur = ld2(src, kWrap ? i0 % n : i0, n, j);
  double lsum = 0.0;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = i0 + r;
    int iw, idn;
    strip_rows<kWrap>(i, n, row_hi, iw, idn);
    const double2 dn = ld2(src, idn, n, j);
    double lf, rt;
    hnbrs(src, iw, n, j, cur, lane, lf, rt);
    double2 o;
    o.x = heat_point(cur.x, up.x, dn.x, lf, cur.y, alpha);
    o.y = heat_point(cur.y, up.y, dn.y, cur.x, rt, alpha);
    if (col_ok && i < row_hi) {
      *reinterpret_cast<double2*>(dst + (int64_t)i * n + j) = o;
      if (copy_dst) *reinterpret_cast<double2*>(copy_dst + (int64_t)i * n + j) = cur;
      if (loss_part) lsum += __dadd_rn(__dmul_rn(o.x, o.x), __dmul_rn(o.y, o.y));
    }
    up = cur;
    cur = dn;
  }
  if (loss_part) {
    lsum = block_sum(lsum, red);
    if (threadIdx.x == 0) loss_part[blockIdx.y * gridDim.x + blockIdx.x] = lsum;
  }
}

// ub_{t-1} = gather of unb_t through the stencil; alphab partial
// += sum (lap u_{t-1}) unb_t. The five contributions to a cell are added in
// the generated reverse loop's interior order: from the cell below, the cell
// to the right, the cell itself (+g, then 4 * -(alpha g)), the cell to the
// left, the cell above.
__device__ __forceinline__ double gather_point(double gc, double g_above, double g_below,
                                               double g_left, double g_right, double alpha) {
  double acc = __dadd_rn(__dmul_rn(alpha, g_below), __dmul_rn(alpha, g_right));
  acc = __dadd_rn(acc, gc);
  acc = __dadd_rn(acc, __dmul_rn(4.0, -__dmul_rn(alpha, gc)));
  acc = __dadd_rn(acc, __dmul_rn(alpha, g_left));
  acc = __dadd_rn(acc, __dmul_rn(alpha, g_above));
  return acc;
}

__device__ __forceinline__ double lap_point(double c, double up, double dn, double lf, double rt) {
  double s = __dadd_rn(__dadd_rn(__dadd_rn(up, dn), lf), rt);
  return __dadd_rn(s, -__dmul_rn(4.0, c));
}

template <int R, bool kWrap>
__global__ void __launch_bounds__(kThreads)
heat_bwd_kernel(const double* __restrict__ g, const double* __restrict__ u,
                double* __restrict__ gdst, double alpha, int n, int row_lo, int row_step,
                int row_hi, double* __restrict__ alpha_part, int first) {
  __shared__ double red[kThreads / 32];
  const int lane = threadIdx.x & 31;
  const int j_raw = blockIdx.x * kColsPerBlock + threadIdx.x * 2;
  const bool col_ok = j_raw < n;
  const int j = col_ok ? j_raw : n - 2;
  const int i0 = row_lo + blockIdx.y * row_step;
  const int row_up = kWrap ? (i0 == 0 ? n - 1 : i0 - 1) : i0 - 1;
  const int row_c = kWrap ? i0 % n : i0;
  double2 gu = ld2(g, row_up, n, j), gc = ld2(g, row_c, n, j);
  double2 uu = ld2(u, row_up, n, j), uc = ld2(u, row_c, n, j);
  double asum = 0.0;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int i = i0 + r;
    int iw, idn;
    strip_rows<kWrap>(i, n, row_hi, iw, idn);
    const double2 gd = ld2(g, idn, n, j);
    const double2 ud = ld2(u, idn, n, j);
    double g_lf, g_rt, u_lf, u_rt;
    hnbrs(g, iw, n, j, gc, lane, g_lf, g_rt);
    hnbrs(u, iw, n, j, uc, lane, u_lf, u_rt);
    double2 o;
    o.x = gather_point(gc.x, gu.x, gd.x, g_lf, gc.y, alpha);
    o.y = gather_point(gc.y, gu.y, gd.y, gc.x, g_rt, alpha);
    if (col_ok && i < row_hi) {
      *reinterpret_cast<double2*>(gdst + (int64_t)i * n + j) = o;
      asum = fma(lap_point(uc.x, uu.x, ud.x, u_lf, uc.y), gc.x, asum);
      asum = fma(lap_point(uc.y, uu.y, ud.y, uc.x, u_rt), gc.y, asum);
    }
    gu = gc; gc = gd;
    uu = uc; uc = ud;
  }
  asum = block_sum(asum, red);
  if (threadIdx.x == 0) {
    const int b = blockIdx.y * gridDim.x + blockIdx.x;
    alpha_part[b] = first ? asum : alpha_part[b] + asum;
  }
}

// General path (odd n, n < 4, or arrays not 16-byte aligned): the same steps
// with one column per thread (kColsPerBlock threads, so the block grid and the
// partials match the paired path) and the horizontal neighbours loaded, not
// shuffled. Periodic wrap on every side, so n = 1, 2 work as the generated
// code's modular indices do.
template <int R>
__global__ void __launch_bounds__(kColsPerBlock)
heat_fwd1_kernel(const double* __restrict__ src, double* __restrict__ dst,
                 double* __restrict__ copy_dst, double alpha, int n,
                 double* __restrict__ loss_part) {
  __shared__ double red[kColsPerBlock / 32];
  const int j_raw = blockIdx.x * kColsPerBlock + threadIdx.x;
  const bool col_ok = j_raw < n;
  const int j = col_ok ? j_raw : n - 1;
  const int jl = j == 0 ? n - 1 : j - 1, jr = j + 1 == n ? 0 : j + 1;
  const int i0 = blockIdx.y * R;
  double up = src[(int64_t)(i0 == 0 ? n - 1 : i0 - 1) * n + j];
  double cur = src[(int64_t)i0 * n + j];
  double lsum = 0.0;
  for (int r = 0; r < R; ++r) {
    const int i = i0 + r;
    if (i >= n) break;                       // uniform over the block
    const int64_t row = (int64_t)i * n;
    const double dn = src[(int64_t)(i + 1 == n ? 0 : i + 1) * n + j];
    const double o = heat_point(cur, up, dn, src[row + jl], src[row + jr], alpha);
    if (col_ok) {
      dst[row + j] = o;
      if (copy_dst) copy_dst[row + j] = cur;
      if (loss_part) lsum += __dmul_rn(o, o);
    }
    up = cur;
    cur = dn;
  }
  if (loss_part) {
    lsum = block_sum(lsum, red);
    if (threadIdx.x == 0) loss_part[blockIdx.y * gridDim.x + blockIdx.x] = lsum;
  }
}

template <int R>
__global__ void __launch_bounds__(kColsPerBlock)
heat_bwd1_kernel(const double* __restrict__ g, const double* __restrict__ u,
                 double* __restrict__ gdst, double alpha, int n,
                 double* __restrict__ alpha_part, int first) {
  __shared__ double red[kColsPerBlock / 32];
  const int j_raw = blockIdx.x * kColsPerBlock + threadIdx.x;
  const bool col_ok = j_raw < n;
  const int j = col_ok ? j_raw : n - 1;
  const int jl = j == 0 ? n - 1 : j - 1, jr = j + 1 == n ? 0 : j + 1;
  const int i0 = blockIdx.y * R;
  const int64_t rup = (int64_t)(i0 == 0 ? n - 1 : i0 - 1) * n;
  double gu = g[rup + j], gc = g[(int64_t)i0 * n + j];
  double uu = u[rup + j], uc = u[(int64_t)i0 * n + j];
  double asum = 0.0;
  for (int r = 0; r < R; ++r) {
    const int i = i0 + r;
    if (i >= n) break;
    const int64_t row = (int64_t)i * n, rdn = (int64_t)(i + 1 == n ? 0 : i + 1) * n;
    const double gd = g[rdn + j], ud = u[rdn + j];
    const double o = gather_point(gc, gu, gd, g[row + jl], g[row + jr], alpha);
    if (col_ok) {
      gdst[row + j] = o;
      asum = fma(lap_point(uc, uu, ud, u[row + jl], u[row + jr]), gc, asum);
    }
    gu = gc; gc = gd;
    uu = uc; uc = ud;
  }
  asum = block_sum(asum, red);
  if (threadIdx.x == 0) {
    const int b = blockIdx.y * gridDim.x + blockIdx.x;
    alpha_part[b] = first ? asum : alpha_part[b] + asum;
  }
}

__global__ void heat_bwd_init1_kernel(const double* __restrict__ ub,
                                      const double* __restrict__ unb,
                                      const double* __restrict__ ufin,
                                      const double* __restrict__ lossb,
                                      double* __restrict__ dst, int64_t nn) {
  const double lb = lossb[0];
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < nn;
       e += (int64_t)gridDim.x * blockDim.x)
    dst[e] = __dadd_rn(unb[e], __dadd_rn(ub[e], __dmul_rn(__dmul_rn(2.0, ufin[e]), lb)));
}

// g = unb + (ub + (2 u_final) lossb), written into `dst` (one of ub / unb).
__global__ void heat_bwd_init_kernel(const double* __restrict__ ub, const double* __restrict__ unb,
                                     const double* __restrict__ ufin,
                                     const double* __restrict__ lossb,
                                     double* __restrict__ dst, int64_t nn2) {
  const double lb = lossb[0];
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < nn2;
       e += (int64_t)gridDim.x * blockDim.x) {
    const double2 a = reinterpret_cast<const double2*>(ub)[e];
    const double2 b = reinterpret_cast<const double2*>(unb)[e];
    const double2 c = reinterpret_cast<const double2*>(ufin)[e];
    double2 o;
    o.x = __dadd_rn(b.x, __dadd_rn(a.x, __dmul_rn(__dmul_rn(2.0, c.x), lb)));
    o.y = __dadd_rn(b.y, __dadd_rn(a.y, __dmul_rn(__dmul_rn(2.0, c.y), lb)));
    reinterpret_cast<double2*>(dst)[e] = o;
  }
}

// n_step == 0: loss += sum u^2, ub += 2 u lossb.
__global__ void heat_nostep_kernel(const double* __restrict__ u, double* __restrict__ ub,
                                   const double* __restrict__ lossb, int64_t nn,
                                   double* __restrict__ part) {
  __shared__ double red[32];
  const double lb = lossb[0];
  double s = 0.0;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < nn;
       e += (int64_t)gridDim.x * blockDim.x) {
    const double v = u[e];
    s += __dmul_rn(v, v);
    ub[e] = __dadd_rn(ub[e], __dmul_rn(__dmul_rn(2.0, v), lb));
  }
  s = block_sum(s, red);
  if (threadIdx.x == 0) part[blockIdx.x] = s;
}

// ---- TMA-staged reverse step (one grid, n a multiple of 128) ----------------------
// A persistent kernel walks 32 x 128 tiles of the output. Per tile the
// rows i0-1 .. i0+32 and columns j0-2 .. j0+129 of the adjoint state g and of
// the taped state u are staged in shared memory by two TMA copies
// (cp.async.bulk.tensor.2d; the box starts 2 columns left of the tile so its
// innermost coordinate stays 16-byte aligned), three tiles in flight. The grid
// is periodic and TMA fills outside the tensor with zeros, so a tile on the
// grid's edge overwrites the halo cells it needs (row -1 <- row n-1, row n <-
// row 0, column -1 <- column n-1, column n <- column 0) from global memory
// before computing. Each thread owns two adjacent columns of 8 rows and
// computes them with gather_point / lap_point, exactly as heat_bwd_kernel does
// (the same ub bits); its alphab terms are summed per CTA in a fixed tile
// order. Waits on the copies are bounded (~2 s); a wait that runs out sets
// g_heat_error, the CTA stops, waits (bounded) for its copies in flight and
// returns.
template <int TR, int TC, int ST, int NT>
struct TmaTile {
  static constexpr int kHR = TR + 2, kHC = TC + 4;                   // staged region
  static constexpr int kRegionBytes = kHR * kHC * 8;
  static constexpr int kStride = (kRegionBytes + 127) / 128 * 128;   // 128-byte aligned targets
  static constexpr int kSmem = ST * 2 * kStride + 128 + 64;
  static constexpr int kRowsPerThread = TR * TC / 2 / NT;            // a thread: 2 columns
  static_assert(TR * TC % (2 * NT) == 0 && NT % (TC / 2) == 0, "tile / thread split");
  static_assert(kSmem <= 227 * 1024, "shared memory of a CTA");
  static_assert(kHC <= 256 && kHR <= 256 && (kHC * 8) % 16 == 0, "TMA box");
};
__device__ int g_heat_error = 0;

template <int TR, int TC, int ST, int NT, int MINB>
__global__ void __launch_bounds__(NT, MINB)
heat_bwd_tma_kernel(const __grid_constant__ CUtensorMap gmap,
                    const __grid_constant__ CUtensorMap umap, const double* __restrict__ g,
                    const double* __restrict__ u, double* __restrict__ gdst, double alpha, int n,
                    double* __restrict__ alpha_part, int first) {
  using namespace tc5;
  using Tl = TmaTile<TR, TC, ST, NT>;
  constexpr int kHR = Tl::kHR, kHC = Tl::kHC, RPT = Tl::kRowsPerThread;
  extern __shared__ unsigned char smraw[];
  __shared__ double red[NT / 32];
  const uint32_t raw = smem_u32(smraw);
  unsigned char* base = smraw + ((128u - (raw & 127u)) & 127u);
  auto gt = [&](int s) { return reinterpret_cast<double*>(base + (2 * s) * Tl::kStride); };
  auto ut = [&](int s) { return reinterpret_cast<double*>(base + (2 * s + 1) * Tl::kStride); };
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + 2 * ST * Tl::kStride);
  const int tid = threadIdx.x;
  const int tiles_x = n / TC, tiles = tiles_x * (n / TR);
  const int mine = (int)blockIdx.x < tiles ? (tiles - (int)blockIdx.x + (int)gridDim.x - 1) /
                                                 (int)gridDim.x
                                           : 0;
  if (tid == 0) {
    for (int s = 0; s < ST; ++s) mbar_init(smem_u32(bars + s), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  int issued = 0;
  auto issue = [&](int k) {   // thread 0: stage the k-th tile of this CTA
    const int t = (int)blockIdx.x + k * (int)gridDim.x;
    const int s = k % ST;
    const uint32_t bar = smem_u32(bars + s);
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    mbar_arrive_tx(bar, 2 * Tl::kRegionBytes);
    tma_load_2d(smem_u32(gt(s)), &gmap, (t % tiles_x) * TC - 2, (t / tiles_x) * TR - 1, bar);
    tma_load_2d(smem_u32(ut(s)), &umap, (t % tiles_x) * TC - 2, (t / tiles_x) * TR - 1, bar);
  };
  if (tid == 0)
    for (; issued < ST - 1 && issued < mine; ++issued) issue(issued);
  const int cp = tid % (TC / 2), rg = tid / (TC / 2);   // column pair, group of RPT rows
  double asum = 0.0;
  bool ok = true;
  int k = 0;
  for (; k < mine; ++k) {
    if (tid == 0 && issued < mine) issue(issued++);
    const int s = k % ST;
    const bool got = mbar_wait_for(smem_u32(bars + s), (uint32_t)(k / ST) & 1u, &g_heat_error,
                                   kWaitCycles);
    ok = __syncthreads_and(got) != 0;
    if (!ok) break;
    const int t = (int)blockIdx.x + k * (int)gridDim.x;
    const int i0 = (t / tiles_x) * TR, j0 = (t % tiles_x) * TC;
    double* G = gt(s);
    double* U = ut(s);
    // periodic halos of an edge tile (TMA filled them with zeros)
    if (i0 == 0 || i0 + TR == n || j0 == 0 || j0 + TC == n) {
      for (int e = tid; e < 2 * TC + 2 * TR; e += NT) {
        int64_t src = -1;
        int dst = 0;
        if (e < TC) {                           // row -1 <- row n-1
          if (i0 == 0) { src = (int64_t)(n - 1) * n + j0 + e; dst = 2 + e; }
        } else if (e < 2 * TC) {                // row TR <- row 0
          const int c = e - TC;
          if (i0 + TR == n) { src = j0 + c; dst = (kHR - 1) * kHC + 2 + c; }
        } else if (e < 2 * TC + TR) {           // column -1 <- column n-1
          const int r = e - 2 * TC;
          if (j0 == 0) { src = (int64_t)(i0 + r) * n + (n - 1); dst = (1 + r) * kHC + 1; }
        } else {                                // column TC <- column 0
          const int r = e - 2 * TC - TR;
          if (j0 + TC == n) { src = (int64_t)(i0 + r) * n; dst = (1 + r) * kHC + 2 + TC; }
        }
        if (src >= 0) {
          G[dst] = g[src];
          U[dst] = u[src];
        }
      }
      __syncthreads();
    }
    const int c = 2 + 2 * cp;
#pragma unroll 2
    for (int r = 0; r < RPT; ++r) {
      const int R = 1 + rg * RPT + r;
      const double2 gc = *reinterpret_cast<const double2*>(G + R * kHC + c);
      const double2 gu = *reinterpret_cast<const double2*>(G + (R - 1) * kHC + c);
      const double2 gd = *reinterpret_cast<const double2*>(G + (R + 1) * kHC + c);
      const double g_lf = G[R * kHC + c - 1], g_rt = G[R * kHC + c + 2];
      const double2 uc = *reinterpret_cast<const double2*>(U + R * kHC + c);
      const double2 uu = *reinterpret_cast<const double2*>(U + (R - 1) * kHC + c);
      const double2 ud = *reinterpret_cast<const double2*>(U + (R + 1) * kHC + c);
      const double u_lf = U[R * kHC + c - 1], u_rt = U[R * kHC + c + 2];
      double2 o;
      o.x = gather_point(gc.x, gu.x, gd.x, g_lf, gc.y, alpha);
      o.y = gather_point(gc.y, gu.y, gd.y, gc.x, g_rt, alpha);
      *reinterpret_cast<double2*>(gdst + (int64_t)(i0 + R - 1) * n + j0 + 2 * cp) = o;
      asum = fma(lap_point(uc.x, uu.x, ud.x, u_lf, uc.y), gc.x, asum);
      asum = fma(lap_point(uc.y, uu.y, ud.y, uc.x, u_rt), gc.y, asum);
    }
    __syncthreads();   // the stage is free for the copy issued next iteration
  }
  if (!ok && tid == 0) {
    // copies still in flight land before the CTA exits (bounded)
    for (int j = k; j < issued; ++j)
      mbar_wait_for(smem_u32(bars + j % ST), (uint32_t)(j / ST) & 1u, &g_heat_error,
                    kWaitCycles);
  }
  asum = block_sum(asum, red);
  if (tid == 0) alpha_part[blockIdx.x] = first ? asum : alpha_part[blockIdx.x] + asum;
}

// The launch of one tile shape: grid = min(tiles, resident CTAs).
struct TmaVariant {
  int tr, tc, smem, threads, per_sm;
  void (*kern)(CUtensorMap, CUtensorMap, const double*, const double*, double*, double, int,
               double*, int);
};
template <int TR, int TC, int ST, int NT, int MINB>
TmaVariant tma_variant() {
  using Tl = TmaTile<TR, TC, ST, NT>;
  return TmaVariant{TR, TC, Tl::kSmem, NT, MINB, heat_bwd_tma_kernel<TR, TC, ST, NT, MINB>};
}
// a: 32 x 128 tiles, 3 in flight, one CTA of 256 threads per SM; b (the
// default): 16 x 128, 2 in flight, two CTAs per SM; c: 32 x 64, 3 in flight,
// two CTAs of 128 threads per SM; d: 32 x 128, 3 in flight, 512 threads.
// Measured at 8192^2 x 16 (reverse steps, ms): a 5.03, b 4.81, c 5.23,
// d 4.97; the register-tiled kernel 4.77.
TmaVariant heat_tma_variant(char v) {
  switch (v) {
    case 'a': return tma_variant<32, 128, 3, 256, 1>();
    case 'c': return tma_variant<32, 64, 3, 128, 2>();
    case 'd': return tma_variant<32, 128, 3, 512, 1>();
    default:  return tma_variant<16, 128, 2, 256, 2>();
  }
}

// Tensor map of an n x n Float64 field for heat_bwd_tma_kernel: box of
// (tc + 4) columns x (tr + 2) rows, no swizzle, zero fill outside.
stade_status heat_map(CUtensorMap* map, const double* base, int64_t n, int tr, int tc) {
  auto fn = tc5::encode_fn();
  if (!fn) return fail(STADE_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t d[2] = {(cuuint64_t)n, (cuuint64_t)n}, st[1] = {(cuuint64_t)(n * 8)};
  cuuint32_t bx[2] = {(cuuint32_t)(tc + 4), (cuuint32_t)(tr + 2)}, es[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT64, 2, const_cast<double*>(base), d, st, bx,
                  es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(STADE_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return STADE_OK;
}

// The TMA-staged reverse step runs where its tiles cover the grid exactly.
// STADE_HEAT_TMA selects it: "0" the register-tiled kernel, a letter a tile
// shape (heat_tma_variant), unset the default shape.
char heat_tma_choice(int64_t n) {
  const char* e = std::getenv("STADE_HEAT_TMA");
  char v = 'b';   // measured fastest of the four at 8192^2 (4.81 ms per 16 steps, a: 5.03)
  if (e && std::strcmp(e, "0") == 0) return 0;
  if (e && e[0] >= 'a' && e[0] <= 'd') v = e[0];
  const TmaVariant tv = heat_tma_variant(v);
  return (n % tv.tc == 0 && n % tv.tr == 0 && n >= tv.tc && n <= 65536) ? v : 0;
}

struct Grid {
  dim3 fwd, bwd;
  int nfwd, nbwd;
};
Grid grid_of(int64_t n) {
  Grid g;
  g.fwd = dim3(ceil_div_u(n, kColsPerBlock), ceil_div_u(n, kRowsFwd));
  g.bwd = dim3(ceil_div_u(n, kColsPerBlock), ceil_div_u(n, kRowsBwd));
  g.nfwd = (int)(g.fwd.x * g.fwd.y);
  g.nbwd = (int)(g.bwd.x * g.bwd.y);
  return g;
}

constexpr int kNoStepBlocks = 1184;  // 8 per SM

// x = x + y for the two scalars (loss, alphab) after the cross-slab sum.
__global__ void add_two_kernel(double* __restrict__ loss, double* __restrict__ alphab,
                               const double* __restrict__ stage) {
  if (threadIdx.x == 0) {
    loss[0] = __dadd_rn(loss[0], stage[0]);
    alphab[0] = __dadd_rn(alphab[0], stage[1]);
  }
}

// Launch shapes of the slab path: interior rows 1 .. rows-2 in strips, and
// the two edge rows (0 and rows-1, which read the halos) one row per block.
struct SlabGrid {
  dim3 fwd_in, bwd_in, edge;
  int nfwd_in, nbwd_in, nedge;
};
SlabGrid slab_grid_of(int64_t n, int64_t rows) {
  SlabGrid g;
  const unsigned cx = ceil_div_u(n, kColsPerBlock);
  const int64_t inner = rows - 2;
  g.fwd_in = dim3(cx, inner > 0 ? ceil_div_u(inner, kRowsFwd) : 0);
  g.bwd_in = dim3(cx, inner > 0 ? ceil_div_u(inner, kRowsBwd) : 0);
  g.edge = dim3(cx, 2);
  g.nfwd_in = (int)(g.fwd_in.x * g.fwd_in.y);
  g.nbwd_in = (int)(g.bwd_in.x * g.bwd_in.y);
  g.nedge = (int)(g.edge.x * g.edge.y);
  return g;
}

}  // namespace
}  // namespace stade

using namespace stade;

extern "C" int64_t stade_initstacks_heat2d_b(int64_t n, int64_t n_step) {
  // max(0, div(n_step - 1, 1) + 1) * max(0, div(n * n - 1, 1) + 1), as initstacks_* sizes it
  if (n <= 0 || n_step <= 0) return 0;
  return n_step * n * n;
}

extern "C" size_t stade_heat2d_b_f64_workspace(int64_t n, int64_t n_step) {
  if (n <= 0) return 0;
  const Grid g = grid_of(n);
  Sizer z;
  z.take<double>((size_t)g.nfwd);                         // loss partials
  z.take<double>((size_t)(g.nbwd > kNoStepBlocks ? g.nbwd : kNoStepBlocks));  // alphab partials
  z.take<double>(2);                                      // host-scalar staging
  (void)n_step;
  return z.bytes();
}

extern "C" stade_status stade_heat2d_b_f64(double* loss, const double* lossb, double* u,
                                           double* ub, double* un, double* unb, double alpha,
                                           double* alphab, int64_t n, int64_t n_step,
                                           double* u_stack, const stade_opts* opts) {
  STADE_REQUIRE(n >= 0 && n_step >= 0, "heat2d_b: negative size");
  STADE_REQUIRE(alphab != nullptr, "heat2d_b: alphab is null");
  if (n == 0) return STADE_OK;
  STADE_REQUIRE(n <= 65536, "heat2d_b: n = %lld exceeds 65536", (long long)n);
  STADE_REQUIRE(loss && lossb && u && ub && un && unb, "heat2d_b: null array argument");
  STADE_REQUIRE(n_step == 0 || u_stack, "heat2d_b: u_stack is null");
  // Paired columns (16-byte loads, shuffled neighbours) need even n >= 4 and
  // 16-byte aligned arrays; anything else takes the one-column path.
  bool paired = n % 2 == 0 && n >= 4;
  for (const void* p : {(const void*)u, (const void*)ub, (const void*)un, (const void*)unb,
                        (const void*)u_stack})
    if (p != nullptr && (reinterpret_cast<uintptr_t>(p) & 15u) != 0) paired = false;
  const bool host_scalar = (flags_of(opts) & STADE_HOST_SCALARS) != 0;
  cudaStream_t s = stream_of(opts);
  void* wsp = nullptr;
  stade_status st = get_workspace(opts, stade_heat2d_b_f64_workspace(n, n_step), &wsp);
  if (st != STADE_OK) return st;
  const Grid g = grid_of(n);
  Carver c(wsp);
  double* loss_part = c.take<double>((size_t)g.nfwd);
  double* alpha_part = c.take<double>((size_t)(g.nbwd > kNoStepBlocks ? g.nbwd : kNoStepBlocks));
  double* stage = c.take<double>(2);
  double* alphab_dev = alphab;
  if (host_scalar) {
    STADE_CUDA(cudaMemcpyAsync(stage, alphab, sizeof(double), cudaMemcpyHostToDevice, s));
    alphab_dev = stage;
  }
  const int ni = (int)n;
  const int64_t nn = n * n;

  if (n_step == 0) {
    heat_nostep_kernel<<<kNoStepBlocks, 256, 0, s>>>(u, ub, lossb, nn, loss_part);
    STADE_CHECK_LAUNCH();
    st = launch_sum_to_scalar(loss_part, kNoStepBlocks, loss, true, s);
    if (st != STADE_OK) return st;
  } else {
    // forward sweep: tape[t] = state before step t+1
    for (int64_t t = 1; t <= n_step; ++t) {
      const double* src = t == 1 ? u : u_stack + (t - 1) * nn;
      double* dst = t == n_step ? un : u_stack + t * nn;
      double* copy = t == 1 ? u_stack : nullptr;
      PhaseScope ph("fwd_step", s);
      double* lp = t == n_step ? loss_part : nullptr;
      if (paired)
        heat_fwd_kernel<kRowsFwd, true><<<g.fwd, kThreads, 0, s>>>(src, dst, copy, alpha, ni, 0,
                                                                   kRowsFwd, ni, lp);
      else
        heat_fwd1_kernel<kRowsFwd><<<g.fwd, kColsPerBlock, 0, s>>>(src, dst, copy, alpha, ni, lp);
      STADE_CHECK_LAUNCH();
    }
    st = launch_sum_to_scalar(loss_part, g.nfwd, loss, true, s);
    if (st != STADE_OK) return st;
    // backward sweep; the first step reads the seed from `a`, steps alternate
    // a -> b -> a ... and the last one lands in ub
    double* a = (n_step % 2 == 0) ? ub : unb;
    double* b = (n_step % 2 == 0) ? unb : ub;
    {
      PhaseScope ph("bwd_init", s);
      if (paired)
        heat_bwd_init_kernel<<<kNoStepBlocks, 256, 0, s>>>(ub, unb, un, lossb, a, nn / 2);
      else
        heat_bwd_init1_kernel<<<kNoStepBlocks, 256, 0, s>>>(ub, unb, un, lossb, a, nn);
      STADE_CHECK_LAUNCH();
    }
    const char tv_id = paired ? heat_tma_choice(n) : 0;
    const bool tma = tv_id != 0;
    const TmaVariant tv = heat_tma_variant(tma ? tv_id : 'a');
    const int tma_grid =
        (int)std::min<int64_t>((n / tv.tc) * (n / tv.tr), (int64_t)tc5::sm_count() * tv.per_sm);
    if (tma)
      STADE_CUDA(cudaFuncSetAttribute(tv.kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      tv.smem));
    for (int64_t t = n_step; t >= 1; --t) {
      PhaseScope ph("bwd_step", s);
      const double* ut = u_stack + (t - 1) * nn;
      const int first = t == n_step ? 1 : 0;
      if (tma) {
        CUtensorMap gm, um;
        st = heat_map(&gm, a, n, tv.tr, tv.tc);
        if (st == STADE_OK) st = heat_map(&um, ut, n, tv.tr, tv.tc);
        if (st != STADE_OK) return st;
        tv.kern<<<tma_grid, tv.threads, tv.smem, s>>>(gm, um, a, ut, b, alpha, ni, alpha_part,
                                                      first);
      } else if (paired) {
        heat_bwd_kernel<kRowsBwd, true><<<g.bwd, kThreads, 0, s>>>(
            a, ut, b, alpha, ni, 0, kRowsBwd, ni, alpha_part, first);
      } else {
        heat_bwd1_kernel<kRowsBwd><<<g.bwd, kColsPerBlock, 0, s>>>(a, ut, b, alpha, ni,
                                                                    alpha_part, first);
      }
      STADE_CHECK_LAUNCH();
      double* tmp = a; a = b; b = tmp;
    }
    // the result is in ub (== a now); the other buffer is unb, consumed to zero
    {
      PhaseScope ph("zero_unb", s);
      STADE_CUDA(cudaMemsetAsync(unb, 0, (size_t)nn * sizeof(double), s));
    }
    st = launch_sum_to_scalar(alpha_part, tma ? tma_grid : g.nbwd, alphab_dev, true, s);
    if (st != STADE_OK) return st;
  }
  if (host_scalar) {
    STADE_CUDA(cudaMemcpyAsync(alphab, stage, sizeof(double), cudaMemcpyDeviceToHost, s));
    STADE_CUDA(cudaStreamSynchronize(s));
  }
  return STADE_OK;
}

namespace stade {
// Reads and clears the stencil kernel's error word (-1 when it cannot be read).
int heat_take_error() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_heat_error, sizeof(int)) != cudaSuccess) return -1;
  if (v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_heat_error, &zero, sizeof(int));
  }
  return v;
}
}  // namespace stade


// ---------------------------------------------------------------------------
// Slab-sharded heat2d_b: the grid's rows split into one contiguous slab per
// rank, one halo row exchanged with each neighbouring slab per step.
extern "C" int64_t stade_initstacks_heat2d_b_slab(int64_t n, int64_t n_step, int64_t rows) {
  if (n <= 0 || n_step <= 0 || rows <= 0) return 0;
  return n_step * (rows + 2) * n;
}

extern "C" size_t stade_heat2d_b_f64_slab_workspace(int64_t n, int64_t n_step, int64_t rows) {
  if (n <= 0 || rows <= 0) return 0;
  const SlabGrid g = slab_grid_of(n, rows);
  Sizer z;
  z.take<double>((size_t)(g.nfwd_in > kNoStepBlocks ? g.nfwd_in : kNoStepBlocks));  // loss, inner
  z.take<double>((size_t)g.nedge);                          // loss partials, edge rows
  z.take<double>((size_t)(g.nbwd_in > 0 ? g.nbwd_in : 1));  // alphab partials, interior
  z.take<double>((size_t)g.nedge);                          // alphab partials, edge rows
  z.take<double>(4);                                        // (loss, alphab) stage + host
  z.take<double>((size_t)((rows + 2) * n));                 // adjoint state, halo-padded
  z.take<double>((size_t)((rows + 2) * n));                 // second adjoint state
  (void)n_step;
  return z.bytes();
}

extern "C" stade_status stade_heat2d_b_f64_slab(double* loss, const double* lossb, double* u,
                                                double* ub, double* un, double* unb,
                                                double alpha, double* alphab, int64_t n,
                                                int64_t n_step, double* u_stack, int64_t rows,
                                                stade_comm* comm, const stade_opts* opts) {
  STADE_REQUIRE(n >= 0 && n_step >= 0 && rows >= 0, "heat2d_b_slab: negative size");
  STADE_REQUIRE(alphab != nullptr, "heat2d_b_slab: alphab is null");
  if (n == 0 || rows == 0) return STADE_OK;
  STADE_REQUIRE(n % 2 == 0 && n >= 4, "heat2d_b_slab: n must be even and >= 4 (got %lld)",
                (long long)n);
  STADE_REQUIRE(n <= 65536 && rows <= n, "heat2d_b_slab: n = %lld, rows = %lld out of range",
                (long long)n, (long long)rows);
  STADE_REQUIRE(rows >= 2, "heat2d_b_slab: a slab needs at least 2 rows (got %lld)",
                (long long)rows);
  STADE_REQUIRE(comm != nullptr || rows == n,
                "heat2d_b_slab: without a communicator the slab must be the whole grid");
  STADE_REQUIRE(loss && lossb && u && ub && un && unb, "heat2d_b_slab: null array argument");
  STADE_REQUIRE(n_step == 0 || u_stack, "heat2d_b_slab: u_stack is null");
  for (const void* p : {(const void*)u, (const void*)ub, (const void*)un, (const void*)unb,
                        (const void*)u_stack})
    STADE_REQUIRE(p == nullptr || (reinterpret_cast<uintptr_t>(p) & 15u) == 0,
                  "heat2d_b_slab: arrays must be 16-byte aligned");
  const bool host_scalar = (flags_of(opts) & STADE_HOST_SCALARS) != 0;
  cudaStream_t s = stream_of(opts);
  void* wsp = nullptr;
  stade_status st = get_workspace(opts, stade_heat2d_b_f64_slab_workspace(n, n_step, rows), &wsp);
  if (st != STADE_OK) return st;
  const SlabGrid g = slab_grid_of(n, rows);
  Carver c(wsp);
  double* lp_in = c.take<double>((size_t)(g.nfwd_in > kNoStepBlocks ? g.nfwd_in : kNoStepBlocks));
  double* lp_edge = c.take<double>((size_t)g.nedge);
  double* ap_in = c.take<double>((size_t)(g.nbwd_in > 0 ? g.nbwd_in : 1));
  double* ap_edge = c.take<double>((size_t)g.nedge);
  double* stage = c.take<double>(4);
  double* ga = c.take<double>((size_t)((rows + 2) * n));
  double* gb = c.take<double>((size_t)((rows + 2) * n));
  double* alphab_dev = alphab;
  if (host_scalar) {
    STADE_CUDA(cudaMemcpyAsync(stage + 2, alphab, sizeof(double), cudaMemcpyHostToDevice, s));
    alphab_dev = stage + 2;
  }
  const int ni = (int)n, ri = (int)rows;
  const int64_t nn = rows * n;            // owned cells
  const int64_t pad = (rows + 2) * n;     // one tape slot / one padded state
  const bool inner = rows > 2;
  auto slot = [&](int64_t k) { return u_stack + k * pad + n; };  // row 0 of slot k

  if (n_step == 0) {
    heat_nostep_kernel<<<kNoStepBlocks, 256, 0, s>>>(u, ub, lossb, nn, lp_in);
    STADE_CHECK_LAUNCH();
    st = launch_sum_to_scalar(lp_in, kNoStepBlocks, stage, false, s);
    if (st != STADE_OK) return st;
    STADE_CUDA(cudaMemsetAsync(stage + 1, 0, sizeof(double), s));
  } else {
    {
      PhaseScope ph("fwd_step", s);
      STADE_CUDA(cudaMemcpyAsync(slot(0), u, (size_t)nn * sizeof(double),
                                 cudaMemcpyDeviceToDevice, s));
    }
    for (int64_t t = 1; t <= n_step; ++t) {
      PhaseScope ph("fwd_step", s);
      double* src = slot(t - 1);
      double* dst = t == n_step ? un : slot(t);
      const bool last = t == n_step;
      st = halo_begin(comm, src, src + (rows - 1) * n, src - n, src + rows * n, n, s);
      if (st != STADE_OK) return st;
      if (inner) {
        heat_fwd_kernel<kRowsFwd, false><<<g.fwd_in, kThreads, 0, s>>>(
            src, dst, nullptr, alpha, ni, 1, kRowsFwd, ri - 1, last ? lp_in : nullptr);
        STADE_CHECK_LAUNCH();
      }
      st = halo_end(comm, s);
      if (st != STADE_OK) return st;
      heat_fwd_kernel<1, false><<<g.edge, kThreads, 0, s>>>(src, dst, nullptr, alpha, ni, 0,
                                                            ri - 1, ri, last ? lp_edge : nullptr);
      STADE_CHECK_LAUNCH();
    }
    st = launch_sum_to_scalar(lp_edge, g.nedge, stage, false, s);
    if (st == STADE_OK && inner) st = launch_sum_to_scalar(lp_in, g.nfwd_in, stage, true, s);
    if (st != STADE_OK) return st;
    {
      PhaseScope ph("bwd_init", s);
      heat_bwd_init_kernel<<<kNoStepBlocks, 256, 0, s>>>(ub, unb, un, lossb, ga + n, nn / 2);
      STADE_CHECK_LAUNCH();
    }
    double* a = ga + n;
    double* b = gb + n;
    for (int64_t t = n_step; t >= 1; --t) {
      PhaseScope ph("bwd_step", s);
      double* dst = t == 1 ? ub : b;
      const double* ut = slot(t - 1);
      const int first = t == n_step ? 1 : 0;
      st = halo_begin(comm, a, a + (rows - 1) * n, a - n, a + rows * n, n, s);
      if (st != STADE_OK) return st;
      if (inner) {
        heat_bwd_kernel<kRowsBwd, false><<<g.bwd_in, kThreads, 0, s>>>(
            a, ut, dst, alpha, ni, 1, kRowsBwd, ri - 1, ap_in, first);
        STADE_CHECK_LAUNCH();
      }
      st = halo_end(comm, s);
      if (st != STADE_OK) return st;
      heat_bwd_kernel<1, false><<<g.edge, kThreads, 0, s>>>(a, ut, dst, alpha, ni, 0, ri - 1,
                                                            ri, ap_edge, first);
      STADE_CHECK_LAUNCH();
      double* tmp = a; a = b; b = tmp;
    }
    {
      PhaseScope ph("zero_unb", s);
      STADE_CUDA(cudaMemsetAsync(unb, 0, (size_t)nn * sizeof(double), s));
    }
    st = launch_sum_to_scalar(ap_edge, g.nedge, stage + 1, false, s);
    if (st == STADE_OK && inner) st = launch_sum_to_scalar(ap_in, g.nbwd_in, stage + 1, true, s);
    if (st != STADE_OK) return st;
  }
  // (loss, alphab) of this slab -> sums over all slabs -> added to the outputs
  st = comm_allreduce_f64(comm, stage, 2, s);
  if (st != STADE_OK) return st;
  add_two_kernel<<<1, 32, 0, s>>>(loss, alphab_dev, stage);
  STADE_CHECK_LAUNCH();
  if (host_scalar) {
    STADE_CUDA(cudaMemcpyAsync(alphab, alphab_dev, sizeof(double), cudaMemcpyDeviceToHost, s));
    return comm_wait_stream(comm, s);
  }
  return STADE_OK;
}

// ---------------------------------------------------------------------------
// Tangent sweep heat2d_d (tgen_emit, src/STADE.jl:3271-3279; restated in
// oracle.cc heat2d_d): per step und from ud and alphad before un, then
// u = un, ud = und; loss and lossd accumulate at the end. The two state
// buffers alternate between u and un, and after the last step both hold the
// final state (the generated copy loop leaves u == un).
namespace stade {
namespace {

__global__ void __launch_bounds__(256)
heat_tan_step_kernel(const double* __restrict__ u, const double* __restrict__ ud,
                     double* __restrict__ un, double* __restrict__ und, double alpha,
                     double alphad, int n) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  const int i = blockIdx.y;
  if (j >= n) return;
  const int iu = i == 0 ? n - 1 : i - 1, id = i + 1 == n ? 0 : i + 1;
  const int jl = j == 0 ? n - 1 : j - 1, jr = j + 1 == n ? 0 : j + 1;
  const int64_t r = (int64_t)i * n;
  const double c = u[r + j], cd = ud[r + j];
  const double lap = __dadd_rn(__dadd_rn(__dadd_rn(__dadd_rn(u[(int64_t)iu * n + j],
                                                              u[(int64_t)id * n + j]),
                                                     u[r + jl]),
                                            u[r + jr]),
                               -__dmul_rn(4.0, c));
  const double lapd = __dadd_rn(__dadd_rn(__dadd_rn(__dadd_rn(ud[(int64_t)iu * n + j],
                                                               ud[(int64_t)id * n + j]),
                                                      ud[r + jl]),
                                             ud[r + jr]),
                                -__dmul_rn(4.0, cd));
  und[r + j] = __dadd_rn(cd, __dadd_rn(__dmul_rn(alphad, lap), __dmul_rn(alpha, lapd)));
  un[r + j] = __dadd_rn(c, __dmul_rn(alpha, lap));
}

// loss += sum u^2, lossd += sum 2 u ud: per-block partials.
__global__ void heat_tan_loss_kernel(const double* __restrict__ u, const double* __restrict__ ud,
                                     int64_t nn, double* __restrict__ part) {
  __shared__ double red[32];
  double a = 0.0, b = 0.0;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < nn;
       e += (int64_t)gridDim.x * blockDim.x) {
    const double v = u[e];
    a += __dmul_rn(v, v);
    b += __dmul_rn(__dmul_rn(2.0, v), ud[e]);
  }
  a = block_sum(a, red);
  b = block_sum(b, red);
  if (threadIdx.x == 0) {
    part[blockIdx.x] = a;
    part[gridDim.x + blockIdx.x] = b;
  }
}

}  // namespace
}  // namespace stade

extern "C" size_t stade_heat2d_d_f64_workspace(int64_t n, int64_t n_step) {
  (void)n; (void)n_step;
  Sizer z;
  z.take<double>(2 * (size_t)kNoStepBlocks);
  return z.bytes();
}

extern "C" stade_status stade_heat2d_d_f64(double* loss, double* lossd, double* u, double* ud,
                                           double* un, double* und, double alpha, double alphad,
                                           int64_t n, int64_t n_step, const stade_opts* opts) {
  STADE_REQUIRE(n >= 0 && n_step >= 0, "heat2d_d: negative size");
  if (n == 0) return STADE_OK;
  STADE_REQUIRE(n <= 65536, "heat2d_d: n = %lld exceeds 65536", (long long)n);
  STADE_REQUIRE(loss && lossd && u && ud && un && und, "heat2d_d: null array argument");
  cudaStream_t s = stream_of(opts);
  void* wsp = nullptr;
  stade_status st = get_workspace(opts, stade_heat2d_d_f64_workspace(n, n_step), &wsp);
  if (st != STADE_OK) return st;
  Carver c(wsp);
  double* part = c.take<double>(2 * (size_t)kNoStepBlocks);
  const int64_t nn = n * n;
  const dim3 grid(ceil_div_u(n, 256), (unsigned)n);
  double *a = u, *ad = ud, *b = un, *bd = und;
  for (int64_t t = 0; t < n_step; ++t) {
    PhaseScope ph("d_step", s);
    heat_tan_step_kernel<<<grid, 256, 0, s>>>(a, ad, b, bd, alpha, alphad, (int)n);
    STADE_CHECK_LAUNCH();
    std::swap(a, b);
    std::swap(ad, bd);
  }
  if (n_step > 0) {
    // the final state is in (a, ad); the generated copy leaves it in both pairs
    STADE_CUDA(cudaMemcpyAsync(b, a, (size_t)nn * sizeof(double), cudaMemcpyDeviceToDevice, s));
    STADE_CUDA(cudaMemcpyAsync(bd, ad, (size_t)nn * sizeof(double), cudaMemcpyDeviceToDevice, s));
  }
  heat_tan_loss_kernel<<<kNoStepBlocks, 256, 0, s>>>(a, ad, nn, part);
  STADE_CHECK_LAUNCH();
  st = launch_sum_to_scalar(part, kNoStepBlocks, loss, true, s);
  if (st == STADE_OK) st = launch_sum_to_scalar(part + kNoStepBlocks, kNoStepBlocks, lossd, true, s);
  return st;
}
