// C4 conv1d_relu_mse_b: adjoint of a valid multi-channel 1-D convolution,
// ReLU and mean squared error, Float32.
//
// Generated sweep being replaced (restated in oracle.cc; valid-convolution
// adjoint of test/val-corpus/selfrace_conv_b.jl:5-35, ReLU partial
// 0.5 * (1 + sign(a - 0.0)) of der_partials_maxmin, src/STADE.jl:1489):
//   forward  z = conv(x, w); r = max(z, 0); loss += inv_n (r - t)^2
//   backward g = relu'(z) rb_total + zb  (rb_total = rb + inv_n 2 (r - t) lossb)
//            wb[o,c,k] += sum_{b,t} g[b,o,t] x[b,c,t+k]
//            xb[b,c,t+k] += sum_{o,k} w[o,c,k] g[b,o,t]
// The generated CUDA.jl port runs the convolution contraction twins and
// scatters wb / xb with atomics (cgen_contraction_emit and
// cgen_adjoint_contraction_, src/STADE.jl:14147-14762). Here the three
// contractions are implicit GEMMs (no im2col buffer): the forward with the
// whole elementwise epilogue fused, the weight gradient split over
// (sample, position) with a fixed-order slice sum, and the input gradient
// as a gather (each output element owned by one thread, no atomics).
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "conv_tc.cuh"
#include "gemm_simt.cuh"

namespace stade {
namespace {

struct ConvDims {
  int n_b, n_c, n_l, n_o, n_k, n_lo;
};

// A(o, kk) = w[o, kk], kk = c * n_k + k
struct LdW {
  const float* w;
  int ck;
  __device__ __forceinline__ float operator()(int m, int k) const { return w[(int64_t)m * ck + k]; }
};
// B(kk, n) = x[b, c, t + k], n = b * n_lo + t
struct LdXcol {
  const float* x;
  ConvDims d;
  __device__ __forceinline__ float operator()(int kk, int n) const {
    const int b = n / d.n_lo, t = n - b * d.n_lo;
    const int c = kk / d.n_k, k = kk - c * d.n_k;
    return x[((int64_t)b * d.n_c + c) * d.n_l + t + k];
  }
};

// Forward epilogue: everything elementwise of the forward and the reverse up
// to g, plus the per-block loss partial.
struct EpiConvFwd {
  float *z, *r, *zb, *rb, *tb, *g;
  const float *t, *lossb;
  float inv_n;
  ConvDims d;
  float* loss_part;
  mutable float lsum;
  __device__ __forceinline__ void operator()(int o, int n, float a) const {
    const int b = n / d.n_lo, tt = n - b * d.n_lo;
    const int64_t idx = ((int64_t)b * d.n_o + o) * d.n_lo + tt;
    z[idx] = a;
    const float rv = a > 0.0f ? a : (a < 0.0f ? 0.0f : (a == 0.0f ? 0.0f : a));
    r[idx] = rv;
    const float dlt = __fadd_rn(rv, -t[idx]);
    lsum = __fadd_rn(lsum, __fmul_rn(inv_n, __fmul_rn(dlt, dlt)));
    const float cse1 = __fmul_rn(__fmul_rn(inv_n, __fmul_rn(2.0f, dlt)), lossb[0]);
    const float rbt = __fadd_rn(rb[idx], cse1);
    tb[idx] = __fadd_rn(tb[idx], -cse1);
    const float sg = a > 0.0f ? 1.0f : (a < 0.0f ? -1.0f : a);
    float ab = __fmul_rn(0.5f * (1.0f + sg), rbt);
    ab = __fadd_rn(ab, zb[idx]);
    g[idx] = ab;
    rb[idx] = 0.0f;
    zb[idx] = 0.0f;
  }
  __device__ __forceinline__ void finish(int64_t blk) const {
    __shared__ float red[8];
    const float v = block_sum(lsum, red);
    if (threadIdx.x == 0) loss_part[blk] = v;
  }
};

// Weight gradient: A(o, j) = g[b, o, t] with j = b * n_lo + t;
// B(j, kk) = x[b, c, t + k].
struct LdG {
  const float* g;
  ConvDims d;
  __device__ __forceinline__ float operator()(int o, int j) const {
    const int b = j / d.n_lo, t = j - b * d.n_lo;
    return g[((int64_t)b * d.n_o + o) * d.n_lo + t];
  }
};
struct LdXcolT {
  const float* x;
  ConvDims d;
  __device__ __forceinline__ float operator()(int j, int kk) const {
    const int b = j / d.n_lo, t = j - b * d.n_lo;
    const int c = kk / d.n_k, k = kk - c * d.n_k;
    return x[((int64_t)b * d.n_c + c) * d.n_l + t + k];
  }
};
struct EpiAdd : EpiBase {
  float* dst;
  int ld;
  __device__ __forceinline__ void operator()(int m, int n, float acc) const {
    float* q = dst + (int64_t)m * ld + n;
    *q = *q + acc;
  }
};

// Input gradient as a gather: A(c, ok) = w[o, c, k], ok = o * n_k + k;
// B(ok, n) = g[b, o, t' - k] (zero outside 0 <= t' - k < n_lo), n = b * n_l + t'.
struct LdWT {
  const float* w;
  ConvDims d;
  __device__ __forceinline__ float operator()(int c, int ok) const {
    const int o = ok / d.n_k, k = ok - o * d.n_k;
    return w[((int64_t)o * d.n_c + c) * d.n_k + k];
  }
};
struct LdGshift {
  const float* g;
  ConvDims d;
  __device__ __forceinline__ float operator()(int ok, int n) const {
    const int o = ok / d.n_k, k = ok - o * d.n_k;
    const int b = n / d.n_l, tp = n - b * d.n_l;
    const int t = tp - k;
    if (t < 0 || t >= d.n_lo) return 0.0f;
    return g[((int64_t)b * d.n_o + o) * d.n_lo + t];
  }
};
struct EpiAddXb : EpiBase {
  float* xb;
  ConvDims d;
  __device__ __forceinline__ void operator()(int c, int n, float acc) const {
    const int b = n / d.n_l, tp = n - b * d.n_l;
    float* q = xb + ((int64_t)b * d.n_c + c) * d.n_l + tp;
    *q = *q + acc;
  }
};

constexpr int RM = 2, RN = 2, BK = 16;

struct ConvWs {
  float *g, *loss_part, *wpart;
  int fwd_blocks, w_splits;
};
template <class Alloc>
void conv_layout(Alloc& a, ConvWs* w, const ConvDims& d) {
  const int64_t nt = (int64_t)d.n_b * d.n_o * d.n_lo;
  const int64_t ncol = (int64_t)d.n_b * d.n_lo;
  const int fwd_blocks = (int)(((d.n_o + 127) / 128) * ((ncol + 127) / 128));
  const int tiles = ((d.n_o + 127) / 128) * ((d.n_c * d.n_k + 127) / 128);
  const int w_splits = split_plan(tiles, (int)ncol, BK, 256).splits;
  auto p0 = a.template take<float>((size_t)nt);
  auto p1 = a.template take<float>((size_t)fwd_blocks);
  auto p2 = a.template take<float>(w_splits > 1 ? (size_t)w_splits * d.n_o * d.n_c * d.n_k : 1);
  if (w) {
    w->g = (float*)p0; w->loss_part = (float*)p1; w->wpart = (float*)p2;
    w->fwd_blocks = fwd_blocks; w->w_splits = w_splits;
  }
}
struct SizerA {
  Sizer z;
  template <class T> void* take(size_t n) { z.take<T>(n); return nullptr; }
};
struct CarverA {
  Carver c;
  explicit CarverA(void* b) : c(b) {}
  template <class T> T* take(size_t n) { return c.take<T>(n); }
};

// The tcgen05 path runs unless the sizes do not suit it or STADE_CONV_GEMM=simt.
bool use_tc(const ConvShape& sh) {
  const char* e = std::getenv("STADE_CONV_GEMM");
  if (e && std::strcmp(e, "simt") == 0) return false;
  return conv_tc_supported(sh);
}

}  // namespace
}  // namespace stade

using namespace stade;

extern "C" size_t stade_conv1d_relu_mse_b_f32_workspace(int64_t n_b, int64_t n_c, int64_t n_l,
                                                        int64_t n_o, int64_t n_k) {
  if (n_b <= 0 || n_c <= 0 || n_o <= 0 || n_k <= 0 || n_l < n_k) return 256;
  const ConvShape sh{n_b, n_c, n_l, n_o, n_k};
  if (use_tc(sh)) return conv_tc_workspace(sh);
  ConvDims d{(int)n_b, (int)n_c, (int)n_l, (int)n_o, (int)n_k, (int)(n_l - n_k + 1)};
  SizerA a;
  conv_layout(a, nullptr, d);
  return a.z.bytes();
}

extern "C" stade_status stade_conv1d_relu_mse_b_f32(float* loss, const float* lossb,
                                                    const float* x, float* xb, const float* w,
                                                    float* wb, const float* t, float* tb, float* z,
                                                    float* zb, float* r, float* rb, int64_t n_b,
                                                    int64_t n_c, int64_t n_l, int64_t n_o,
                                                    int64_t n_k, const stade_opts* opts) {
  STADE_REQUIRE(n_b >= 0 && n_c >= 0 && n_l >= 0 && n_o >= 0 && n_k >= 0,
                "conv1d_relu_mse_b: negative size");
  const int64_t n_lo = n_l - n_k + 1;
  if (n_b == 0 || n_o == 0 || n_lo <= 0) return STADE_OK;  // no output positions
  STADE_REQUIRE(n_c > 0 && n_k > 0, "conv1d_relu_mse_b: n_c and n_k must be positive");
  STADE_REQUIRE(n_b * n_lo < (int64_t(1) << 31) && n_b * n_l < (int64_t(1) << 31) &&
                    n_c * n_k < (1 << 20) && n_o * n_k < (1 << 20),
                "conv1d_relu_mse_b: sizes out of range");
  STADE_REQUIRE(loss && lossb && x && xb && w && wb && t && tb && z && zb && r && rb,
                "conv1d_relu_mse_b: null array argument");
  cudaStream_t s = stream_of(opts);
  void* wsp = nullptr;
  stade_status st = get_workspace(
      opts, stade_conv1d_relu_mse_b_f32_workspace(n_b, n_c, n_l, n_o, n_k), &wsp);
  if (st != STADE_OK) return st;
  const ConvShape sh{n_b, n_c, n_l, n_o, n_k};
  if (use_tc(sh)) {
    for (const void* p : {(const void*)x, (const void*)w})
      STADE_REQUIRE((reinterpret_cast<uintptr_t>(p) & 15u) == 0,
                    "conv1d_relu_mse_b: x and w must be 16-byte aligned");
    return conv_tc_run(sh, loss, lossb, x, xb, w, wb, t, tb, z, zb, r, rb, wsp, s);
  }
  const ConvDims d{(int)n_b, (int)n_c, (int)n_l, (int)n_o, (int)n_k, (int)n_lo};
  CarverA ca(wsp);
  ConvWs cw;
  conv_layout(ca, &cw, d);
  const float inv_n = 1.0f / (float)(n_b * n_o * n_lo);
  const int ncol = (int)(n_b * n_lo), ck = (int)(n_c * n_k), okk = (int)(n_o * n_k);

  EpiConvFwd ef{z, r, zb, rb, tb, cw.g, t, lossb, inv_n, d, cw.loss_part, 0.0f};
  {
    PhaseScope ph("conv_fwd", s);
    st = gemm_simt<float, RM, RN, BK, true, true>((int)n_o, ncol, ck, LdW{w, ck}, LdXcol{x, d}, ef,
                                                  nullptr, 1, s);
    if (st == STADE_OK) st = launch_sum_to_scalar(cw.loss_part, cw.fwd_blocks, loss, true, s);
  }
  if (st != STADE_OK) return st;
  {
    PhaseScope ph("conv_wgrad", s);
    st = gemm_simt<float, RM, RN, BK, true, false>((int)n_o, ck, ncol, LdG{cw.g, d},
                                                   LdXcolT{x, d}, EpiAdd{{}, wb, ck}, cw.wpart,
                                                   cw.w_splits, s);
  }
  if (st != STADE_OK) return st;
  {
    PhaseScope ph("conv_xgrad", s);
    st = gemm_simt<float, RM, RN, BK, true, true>((int)n_c, (int)(n_b * n_l), okk, LdWT{w, d},
                                                  LdGshift{cw.g, d}, EpiAddXb{{}, xb, d}, nullptr,
                                                  1, s);
  }
  return st;
}

// ---------------------------------------------------------------------------
// Tangent sweep conv1d_relu_mse_d (tgen_emit, src/STADE.jl:3271-3279;
// restated in oracle.cc conv1d_relu_mse_d): z = conv(x, w) and
// zd = conv(xd, w) + conv(x, wd) as two implicit GEMMs (the second over a
// doubled K: [w | wd] against [Xcol(xd) ; Xcol(x)]), the elementwise tail
// and the loss partials in the second one's epilogue.
namespace stade {
namespace {

struct EpiConvZ : EpiBase {  // z[b, o, t] = acc
  float* z;
  ConvDims d;
  __device__ __forceinline__ void operator()(int o, int n, float a) const {
    const int b = n / d.n_lo, tt = n - b * d.n_lo;
    z[((int64_t)b * d.n_o + o) * d.n_lo + tt] = a;
  }
};
struct LdW2 {  // A(o, kk2) = [w | wd](o, kk2)
  const float *w, *wd;
  int ck;
  __device__ __forceinline__ float operator()(int m, int k) const {
    return k < ck ? w[(int64_t)m * ck + k] : wd[(int64_t)m * ck + (k - ck)];
  }
};
struct LdXcol2 {  // B(kk2, n) = [Xcol(xd) ; Xcol(x)](kk2, n)
  const float *xd, *x;
  ConvDims d;
  __device__ __forceinline__ float operator()(int kk2, int n) const {
    const int ck = d.n_c * d.n_k;
    const float* src = kk2 < ck ? xd : x;
    const int kk = kk2 < ck ? kk2 : kk2 - ck;
    const int b = n / d.n_lo, t = n - b * d.n_lo;
    const int c = kk / d.n_k, k = kk - c * d.n_k;
    return src[((int64_t)b * d.n_c + c) * d.n_l + t + k];
  }
};
struct EpiConvTan {
  const float *z, *t, *td;
  float *zd, *r, *rd;
  float inv_n;
  ConvDims d;
  float* part;  // [2][blocks]: loss, lossd
  int64_t nblk;
  mutable float lsum, ldsum;
  __device__ __forceinline__ void operator()(int o, int n, float ad) const {
    const int b = n / d.n_lo, tt = n - b * d.n_lo;
    const int64_t idx = ((int64_t)b * d.n_o + o) * d.n_lo + tt;
    const float a = z[idx];
    zd[idx] = ad;
    const float sg = a > 0.0f ? 1.0f : (a < 0.0f ? -1.0f : a);
    const float rdv = __fmul_rn(0.5f * (1.0f + sg), ad);
    rd[idx] = rdv;
    const float rv = a > 0.0f ? a : (a < 0.0f ? 0.0f : (a == 0.0f ? 0.0f : a));
    r[idx] = rv;
    const float dlt = __fadd_rn(rv, -t[idx]);
    ldsum = __fadd_rn(ldsum, __fmul_rn(inv_n, __fmul_rn(__fmul_rn(2.0f, dlt),
                                                         __fadd_rn(rdv, -td[idx]))));
    lsum = __fadd_rn(lsum, __fmul_rn(inv_n, __fmul_rn(dlt, dlt)));
  }
  __device__ __forceinline__ void finish(int64_t blk) const {
    __shared__ float red[32];
    const float v = block_sum(lsum, red);
    __syncthreads();
    const float w = block_sum(ldsum, red);
    if (threadIdx.x == 0) {
      part[blk] = v;
      part[nblk + blk] = w;
    }
  }
};

}  // namespace
}  // namespace stade

extern "C" size_t stade_conv1d_relu_mse_d_f32_workspace(int64_t n_b, int64_t n_c, int64_t n_l,
                                                        int64_t n_o, int64_t n_k) {
  if (n_b <= 0 || n_c <= 0 || n_o <= 0 || n_k <= 0 || n_l < n_k) return 256;
  const int64_t ncol = n_b * (n_l - n_k + 1);
  const int64_t blocks = ((n_o + 127) / 128) * ((ncol + 127) / 128);
  Sizer z;
  z.take<float>((size_t)(2 * blocks));
  return z.bytes();
}

extern "C" stade_status stade_conv1d_relu_mse_d_f32(float* loss, float* lossd, const float* x,
                                                    const float* xd, const float* w,
                                                    const float* wd, const float* t,
                                                    const float* td, float* z, float* zd,
                                                    float* r, float* rd, int64_t n_b,
                                                    int64_t n_c, int64_t n_l, int64_t n_o,
                                                    int64_t n_k, const stade_opts* opts) {
  STADE_REQUIRE(n_b >= 0 && n_c >= 0 && n_l >= 0 && n_o >= 0 && n_k >= 0,
                "conv1d_relu_mse_d: negative size");
  const int64_t n_lo = n_l - n_k + 1;
  if (n_b == 0 || n_o == 0 || n_lo <= 0) return STADE_OK;
  STADE_REQUIRE(n_c > 0 && n_k > 0, "conv1d_relu_mse_d: n_c and n_k must be positive");
  STADE_REQUIRE(n_b * n_lo < (int64_t(1) << 31) && n_c * n_k < (1 << 19),
                "conv1d_relu_mse_d: sizes out of range");
  STADE_REQUIRE(loss && lossd && x && xd && w && wd && t && td && z && zd && r && rd,
                "conv1d_relu_mse_d: null array argument");
  cudaStream_t s = stream_of(opts);
  void* wsp = nullptr;
  stade_status st = get_workspace(
      opts, stade_conv1d_relu_mse_d_f32_workspace(n_b, n_c, n_l, n_o, n_k), &wsp);
  if (st != STADE_OK) return st;
  const ConvDims d{(int)n_b, (int)n_c, (int)n_l, (int)n_o, (int)n_k, (int)n_lo};
  const int ncol = (int)(n_b * n_lo), ck = (int)(n_c * n_k);
  const int64_t blocks = ((n_o + 127) / 128) * ((ncol + 127) / 128);
  Carver c(wsp);
  float* part = c.take<float>((size_t)(2 * blocks));
  const float inv_n = 1.0f / (float)(n_b * n_o * n_lo);
  {
    PhaseScope ph("d_conv", s);
    st = gemm_simt<float, RM, RN, BK, true, true>((int)n_o, ncol, ck, LdW{w, ck}, LdXcol{x, d},
                                                  EpiConvZ{{}, z, d}, nullptr, 1, s);
    if (st == STADE_OK)
      st = gemm_simt<float, RM, RN, BK, true, true>(
          (int)n_o, ncol, 2 * ck, LdW2{w, wd, ck}, LdXcol2{xd, x, d},
          EpiConvTan{z, t, td, zd, r, rd, inv_n, d, part, blocks, 0.0f, 0.0f}, nullptr, 1, s);
  }
  if (st != STADE_OK) return st;
  st = launch_sum_to_scalar(part, blocks, loss, true, s);
  if (st == STADE_OK) st = launch_sum_to_scalar(part + blocks, blocks, lossd, true, s);
  return st;
}
