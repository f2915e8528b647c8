// oracle.cc -- TEST INFRASTRUCTURE ONLY. CPU restatement of the adjoint and
// HVP sweeps that STADE.jl generates for the primals in primals.jl.
//
// Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg (and
// its --impl reference arm) may load this library. The product path
// (libstade_b200.so) never calls it.
//
// The reference cannot run here (it is Julia; no Julia toolchain), and the
// generated `_b.jl` / `_hv.jl` files for these five primals do not exist in the
// reference, so each sweep below is written by hand from STADE's generation
// rules and the pinned generated exemplars it follows (cited per function):
//   - the forward sweep is replayed verbatim before the backward sweep
//     (agen_forward_body, src/STADE.jl:6323);
//   - loops run backwards with a negated step (agen_negate_step,
//     src/STADE.jl:4656), e.g. `for i_x2 = i_n:-1:1`;
//   - a consumed adjoint is captured then zeroed, `__oldb_0 = vb; vb = 0.0`
//     (agen_backward_assign, src/STADE.jl:6605; affine_loss_b.jl:16-20);
//   - an accumulation `s = s + e` leaves sb in place and adds into e's inputs
//     (matvec_loss_b.jl:19-26);
//   - local scalars needed by a derivative are recomputed in the reverse
//     iteration instead of taped (mlp1d_b.jl:43-57); overwritten array
//     values that are needed are taped (advection_b.jl:9-10, 28-29);
//   - derivative formulas are the der_ table's: tanh' = 1 - tanh(x)^2
//     recomputed (src/STADE.jl:1462, mlp1d_b.jl:50), max(a, b)' =
//     0.5 * (1 + sign(a - b)) (src/STADE.jl:1489-1501, so 0.5 at a tie),
//     v^2' = 2 v (src/STADE.jl:1369), exp' = exp (src/STADE.jl:1391),
//     log' = 1 / x (src/STADE.jl:1397), a / b: 1 / b and -(a / b^2)
//     (transformer_b.jl:633-634);
//   - every float argument is independent (src/STADE.jl:522-525), so the
//     adjoints of inputs such as x and t are outputs too;
//   - the HVP doubles every adjoint statement with its tangent twin
//     (hvp_double_stmt, src/STADE.jl:6904; exemplar mlp1d_hv.jl).
// Build flags (Makefile): -O2 -fno-fast-math -ffp-contract=off, so no fused
// multiply-add changes the rounding of the Julia source's `a * b + c`.
//
// Index convention: 0-based here; the comments give the 1-based Julia loop.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <utility>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

using i64 = int64_t;

template <class T> inline T jl_sign(T x) { return x > T(0) ? T(1) : (x < T(0) ? T(-1) : x); }
// Julia's max for floats: NaN wins, then the larger value, +0.0 over -0.0.
template <class T> inline T jl_max(T a, T b) {
  if (a != a) return a;
  if (b != b) return b;
  if (a > b) return a;
  if (b > a) return b;
  return std::signbit(a) ? b : a;
}
// ---- Rules of the generated code, shared by the five sweeps below and by the
// restated reference exemplars at the end of this file (which pin them: the
// exemplars are compared bit for bit with the reference's own generated text,
// run by an interpreter). Each returns the expression the generator writes.
// A consumed adjoint: `__oldb = vb; vb = 0.0` (agen_backward_assign,
// src/STADE.jl:6605; affine_loss_b.jl:16-17).
template <class T> inline T take(T& vb) {
  const T o = vb;
  vb = T(0);
  return o;
}
// d(v^2)/dv = `2 * v` (der_partials_pow with a literal 2, src/STADE.jl:1369;
// affine_loss_b.jl:13, `(2__cse_0)` in mlp1d_b.jl:32).
template <class T> inline T d_sq(T v) { return T(2) * v; }
// d tanh(s)/ds = `1.0 - tanh(s) ^ 2` from the recomputed tanh (der_partials_tanh,
// src/STADE.jl:1462; mlp1d_b.jl:50); th = tanh(s), th^2 = th * th (literal_pow).
template <class T> inline T d_tanh(T th) { return T(1) - th * th; }
// d max(a, b)/da = `0.5 * (1 + sign(a - b))`, 0.5 at a tie (der_partials_maxmin,
// src/STADE.jl:1489-1501).
template <class T> inline T d_max(T a, T b);
// The HVP twin of `sb += d_tanh(th) * oldb` (hvp_double_stmt, src/STADE.jl:6904):
// `oldb * -((2 th) * (g * sd)) + g * oldbd`, g = d_tanh(th) (mlp1d_hv.jl:92-93).
template <class T> inline T d_tanh_tangent(T th, T g, T sd, T oldb, T oldbd) {
  return oldb * -((T(2) * th) * (g * sd)) + g * oldbd;
}

inline float jl_tanh(float x) { return std::tanh(x); }
inline double jl_tanh(double x) { return std::tanh(x); }
inline long double jl_tanh(long double x) { return tanhl(x); }
inline float jl_exp(float x) { return std::exp(x); }
inline double jl_exp(double x) { return std::exp(x); }
inline long double jl_exp(long double x) { return expl(x); }
inline float jl_log(float x) { return std::log(x); }
inline double jl_log(double x) { return std::log(x); }
inline long double jl_log(long double x) { return logl(x); }
template <class T> inline T d_max(T a, T b) { return T(0.5) * (T(1) + jl_sign(a - b)); }

// ---------------------------------------------------------------------------
// C1 affine_ls_b. Follows affine_loss_b.jl:5-23 (per-element adjoint with
// __oldb capture) and matvec_loss_b.jl:5-27 (flattened (sample, output) loop
// with div/mod decode; the accumulation loop's adjoint runs i_k backwards).
template <class T>
void affine_ls_b(T* loss, const T* lossb, const T* w, T* wb, const T* b, T* bb,
                 const T* x, T* xb, const T* t, T* tb, T* y, T* yb,
                 i64 n_s, i64 n_o, i64 n_i) {
  T s = T(0), sb = T(0);
  // forward sweep
  for (i64 idx = 0; idx < n_s * n_o; ++idx) {          // for idx = 1:n_s * n_o
    const i64 i_s = idx / n_o, i_o = idx % n_o;
    s = b[i_o];
    for (i64 k = 0; k < n_i; ++k) s = s + w[i_o * n_i + k] * x[i_s * n_i + k];
    y[idx] = s;
  }
  for (i64 idx2 = 0; idx2 < n_s * n_o; ++idx2) {
    const T d = y[idx2] - t[idx2];
    loss[0] = loss[0] + T(0.5) * (d * d);
  }
  // backward sweep
  for (i64 idx2 = n_s * n_o - 1; idx2 >= 0; --idx2) {  // for idx2 = n_s * n_o:-1:1
    const T cse0 = y[idx2] - t[idx2];
    const T cse1 = (T(0.5) * d_sq(cse0)) * lossb[0];
    yb[idx2] = yb[idx2] + cse1;
    tb[idx2] = tb[idx2] + -cse1;
  }
  for (i64 idx = n_s * n_o - 1; idx >= 0; --idx) {      // for idx = n_s * n_o:-1:1
    const i64 i_s = idx / n_o, i_o = idx % n_o;
    T oldb = take(yb[idx]);
    sb = sb + oldb;
    for (i64 k = n_i - 1; k >= 0; --k) {                 // for i_k = n_i:-1:1
      wb[i_o * n_i + k] = wb[i_o * n_i + k] + x[i_s * n_i + k] * sb;
      xb[i_s * n_i + k] = xb[i_s * n_i + k] + w[i_o * n_i + k] * sb;
    }
    oldb = take(sb);
    bb[i_o] = bb[i_o] + oldb;
  }
  (void)s;
}

// ---------------------------------------------------------------------------
// C2 / C5 mlp2_ce forward pieces, shared by the adjoint and the HVP.
template <class T>
void mlp2_ce_forward(T* loss, const T* x, const T* y, const T* w1, const T* b1,
                     const T* w2, const T* b2, T* h, T* z, T* p,
                     i64 n_s, i64 n_i, i64 n_h, i64 n_o) {
  for (i64 idx = 0; idx < n_s * n_h; ++idx) {
    const i64 i_s = idx / n_h, j = idx % n_h;
    T s1 = b1[j];
    for (i64 k = 0; k < n_i; ++k) s1 = s1 + x[i_s * n_i + k] * w1[k * n_h + j];
    h[idx] = jl_tanh(s1);
  }
  for (i64 idx2 = 0; idx2 < n_s * n_o; ++idx2) {
    const i64 i_s = idx2 / n_o, c = idx2 % n_o;
    T s2 = b2[c];
    for (i64 k = 0; k < n_h; ++k) s2 = s2 + h[i_s * n_h + k] * w2[k * n_o + c];
    z[idx2] = s2;
  }
  for (i64 i_s = 0; i_s < n_s; ++i_s) {
    const T* zr = z + i_s * n_o;
    T* pr = p + i_s * n_o;
    T row_max = zr[0];
    for (i64 c = 1; c < n_o; ++c) row_max = jl_max(row_max, zr[c]);
    for (i64 c = 0; c < n_o; ++c) pr[c] = jl_exp(zr[c] - row_max);
    T row_sum = T(0);
    for (i64 c = 0; c < n_o; ++c) row_sum = row_sum + pr[c];
    for (i64 c = 0; c < n_o; ++c)
      loss[0] = loss[0] - y[i_s * n_o + c] * jl_log(pr[c] / row_sum);
  }
}

// C2 mlp2_ce_b. Forward replay, then the reverse of the softmax loop (the
// loss statement, the row_sum loop, the exp loop and the row-max chain in
// that order, as transformer_b.jl:615-667 reverses the same softmax), then the
// output-logit loop (an accumulation like mlp1d_b.jl:34-42), then the hidden
// loop with s1 recomputed and tanh' = 1 - tanh(s1)^2 (mlp1d_b.jl:43-78).
template <class T>
void mlp2_ce_b(T* loss, const T* lossb, const T* x, T* xb, const T* y, T* yb,
               const T* w1, T* w1b, const T* b1, T* b1b, const T* w2, T* w2b,
               const T* b2, T* b2b, T* h, T* hb, T* z, T* zb, T* p, T* pb,
               i64 n_s, i64 n_i, i64 n_h, i64 n_o) {
  mlp2_ce_forward(loss, x, y, w1, b1, w2, b2, h, z, p, n_s, n_i, n_h, n_o);
  std::vector<T> max_tape(n_o > 0 ? n_o : 1);  // row_max before step i_c
  T s1b = T(0), s2b = T(0), row_maxb = T(0), row_sumb = T(0);
  // reverse of the softmax cross-entropy loop: for i_s = n_s:-1:1
  for (i64 i_s = n_s - 1; i_s >= 0; --i_s) {
    const T* zr = z + i_s * n_o;
    const T* pr = p + i_s * n_o;
    T* zbr = zb + i_s * n_o;
    T* pbr = pb + i_s * n_o;
    // restore the scalars of this iteration (row-max chain taped per step)
    T row_max = zr[0];
    for (i64 c = 1; c < n_o; ++c) { max_tape[c] = row_max; row_max = jl_max(row_max, zr[c]); }
    T row_sum = T(0);
    for (i64 c = 0; c < n_o; ++c) row_sum = row_sum + pr[c];
    // loss[1] = loss[1] - y * log(p / row_sum), for i_c = n_o:-1:1
    for (i64 c = n_o - 1; c >= 0; --c) {
      const T q = pr[c] / row_sum;
      yb[i_s * n_o + c] = yb[i_s * n_o + c] + -(jl_log(q)) * lossb[0];
      const T qb = (T(1) / q) * (-(y[i_s * n_o + c]) * lossb[0]);
      pbr[c] = pbr[c] + (T(1) / row_sum) * qb;
      row_sumb = row_sumb + -(pr[c] / (row_sum * row_sum)) * qb;
    }
    // row_sum = row_sum + p[c]
    for (i64 c = n_o - 1; c >= 0; --c) pbr[c] = pbr[c] + row_sumb;
    row_sumb = T(0);
    // p[c] = exp(z[c] - row_max)
    for (i64 c = n_o - 1; c >= 0; --c) {
      const T oldb = take(pbr[c]);
      const T cse = jl_exp(zr[c] - row_max) * oldb;
      zbr[c] = zbr[c] + cse;
      row_maxb = row_maxb + -cse;
    }
    // row_max = max(row_max, z[c]), for i_c = n_o:-1:2
    for (i64 c = n_o - 1; c >= 1; --c) {
      const T m_prev = max_tape[c];
      const T oldb = take(row_maxb);
      const T zc = zr[c];
      row_maxb = row_maxb + d_max(m_prev, zc) * oldb;
      zbr[c] = zbr[c] + d_max(zc, m_prev) * oldb;
    }
    // row_max = z[1]
    {
      const T oldb = take(row_maxb);
      zbr[0] = zbr[0] + oldb;
    }
  }
  // reverse of the output-logit loop: for idx2 = n_s * n_o:-1:1
  for (i64 idx2 = n_s * n_o - 1; idx2 >= 0; --idx2) {
    const i64 i_s = idx2 / n_o, c = idx2 % n_o;
    T oldb = take(zb[idx2]);
    s2b = s2b + oldb;
    for (i64 k = n_h - 1; k >= 0; --k) {
      w2b[k * n_o + c] = w2b[k * n_o + c] + h[i_s * n_h + k] * s2b;
      hb[i_s * n_h + k] = hb[i_s * n_h + k] + w2[k * n_o + c] * s2b;
    }
    oldb = take(s2b);
    b2b[c] = b2b[c] + oldb;
  }
  // reverse of the hidden loop: for idx = n_s * n_h:-1:1
  for (i64 idx = n_s * n_h - 1; idx >= 0; --idx) {
    const i64 i_s = idx / n_h, j = idx % n_h;
    T s1 = b1[j];
    for (i64 k = 0; k < n_i; ++k) s1 = s1 + x[i_s * n_i + k] * w1[k * n_h + j];
    T oldb = take(hb[idx]);
    const T th = jl_tanh(s1);
    s1b = s1b + d_tanh(th) * oldb;
    for (i64 k = 0; k < n_i; ++k) {
      const T cse_w = w1[k * n_h + j];
      const T cse_x = x[i_s * n_i + k];
      w1b[k * n_h + j] = w1b[k * n_h + j] + cse_x * s1b;
      xb[i_s * n_i + k] = xb[i_s * n_i + k] + cse_w * s1b;
    }
    oldb = take(s1b);
    b1b[j] = b1b[j] + oldb;
  }
}

// ---------------------------------------------------------------------------
// C5 mlp2_ce_hv. Every statement of mlp2_ce_b with its tangent twin, the
// tangent computed first from the primal values before the statement
// (mlp1d_hv.jl: `s2d = ...` before `s2 = ...`, `__oldb_0d` with `__oldb_0`).
template <class T>
void mlp2_ce_hv(T* loss, const T* lossb, const T* x, T* xb, const T* y, T* yb,
                const T* w1, T* w1b, const T* b1, T* b1b, const T* w2, T* w2b,
                const T* b2, T* b2b, T* h, T* hb, T* z, T* zb, T* p, T* pb,
                i64 n_s, i64 n_i, i64 n_h, i64 n_o,
                T* lossd, const T* lossbd, const T* xd, T* xbd, const T* yd, T* ybd,
                const T* w1d, T* w1bd, const T* b1d, T* b1bd, const T* w2d, T* w2bd,
                const T* b2d, T* b2bd, T* hd, T* hbd, T* zd, T* zbd, T* pd, T* pbd) {
  // ---- forward sweep with tangents (mlp1d_hv.jl:18-54)
  for (i64 idx = 0; idx < n_s * n_h; ++idx) {
    const i64 i_s = idx / n_h, j = idx % n_h;
    T s1d = b1d[j], s1 = b1[j];
    for (i64 k = 0; k < n_i; ++k) {
      const T xv = x[i_s * n_i + k], wv = w1[k * n_h + j];
      s1d = s1d + (xv * w1d[k * n_h + j] + wv * xd[i_s * n_i + k]);
      s1 = s1 + xv * wv;
    }
    const T th = jl_tanh(s1);
    hd[idx] = (T(1) - th * th) * s1d;
    h[idx] = th;
  }
  for (i64 idx2 = 0; idx2 < n_s * n_o; ++idx2) {
    const i64 i_s = idx2 / n_o, c = idx2 % n_o;
    T s2d = b2d[c], s2 = b2[c];
    for (i64 k = 0; k < n_h; ++k) {
      const T hv = h[i_s * n_h + k], wv = w2[k * n_o + c];
      s2d = s2d + (hv * w2d[k * n_o + c] + wv * hd[i_s * n_h + k]);
      s2 = s2 + wv * hv;
    }
    zd[idx2] = s2d;
    z[idx2] = s2;
  }
  std::vector<T> mt(n_o > 0 ? n_o : 1), mdt(n_o > 0 ? n_o : 1);
  for (i64 i_s = 0; i_s < n_s; ++i_s) {
    const T* zr = z + i_s * n_o; const T* zdr = zd + i_s * n_o;
    T* pr = p + i_s * n_o; T* pdr = pd + i_s * n_o;
    T m = zr[0], md = zdr[0];
    for (i64 c = 1; c < n_o; ++c) {
      const T g1 = d_max(m, zr[c]);
      const T g2 = d_max(zr[c], m);
      md = g1 * md + g2 * zdr[c];
      m = jl_max(m, zr[c]);
    }
    for (i64 c = 0; c < n_o; ++c) {
      const T e = jl_exp(zr[c] - m);
      pdr[c] = e * (zdr[c] - md);
      pr[c] = e;
    }
    T rs = T(0), rsd = T(0);
    for (i64 c = 0; c < n_o; ++c) { rsd = rsd + pdr[c]; rs = rs + pr[c]; }
    for (i64 c = 0; c < n_o; ++c) {
      const T q = pr[c] / rs;
      const T qd = pdr[c] / rs - (pr[c] / (rs * rs)) * rsd;
      lossd[0] = lossd[0] - (yd[i_s * n_o + c] * jl_log(q) + y[i_s * n_o + c] * (qd / q));
      loss[0] = loss[0] - y[i_s * n_o + c] * jl_log(q);
    }
  }
  // ---- backward sweep with tangents
  T s1b = 0, s1bd = 0, s2b = 0, s2bd = 0, mb = 0, mbd = 0, rsb = 0, rsbd = 0;
  for (i64 i_s = n_s - 1; i_s >= 0; --i_s) {
    const T* zr = z + i_s * n_o; const T* zdr = zd + i_s * n_o;
    const T* pr = p + i_s * n_o; const T* pdr = pd + i_s * n_o;
    T* zbr = zb + i_s * n_o; T* zbdr = zbd + i_s * n_o;
    T* pbr = pb + i_s * n_o; T* pbdr = pbd + i_s * n_o;
    T m = zr[0], md = zdr[0];
    for (i64 c = 1; c < n_o; ++c) {
      mt[c] = m; mdt[c] = md;
      const T g1 = d_max(m, zr[c]);
      const T g2 = d_max(zr[c], m);
      md = g1 * md + g2 * zdr[c];
      m = jl_max(m, zr[c]);
    }
    T rs = T(0), rsd = T(0);
    for (i64 c = 0; c < n_o; ++c) { rsd = rsd + pdr[c]; rs = rs + pr[c]; }
    const T lb = lossb[0], lbd = lossbd[0];
    for (i64 c = n_o - 1; c >= 0; --c) {
      const T yv = y[i_s * n_o + c], ydv = yd[i_s * n_o + c];
      const T q = pr[c] / rs;
      const T qd = pdr[c] / rs - (pr[c] / (rs * rs)) * rsd;
      const T lq = jl_log(q);
      const T lqd = qd / q;
      ybd[i_s * n_o + c] = ybd[i_s * n_o + c] + -(lqd * lb + lq * lbd);
      yb[i_s * n_o + c] = yb[i_s * n_o + c] + -(lq) * lb;
      const T inv_q = T(1) / q;
      const T inv_qd = -(qd / (q * q));
      const T ny = -(yv) * lb;
      const T nyd = -(ydv * lb + yv * lbd);
      const T qbd = inv_qd * ny + inv_q * nyd;
      const T qb = inv_q * ny;
      const T inv_rs = T(1) / rs;
      const T inv_rsd = -(rsd / (rs * rs));
      pbdr[c] = pbdr[c] + (inv_rsd * qb + inv_rs * qbd);
      pbr[c] = pbr[c] + inv_rs * qb;
      const T pr2 = pr[c] / (rs * rs);
      const T pr2d = pdr[c] / (rs * rs) - (pr[c] / (rs * rs)) * ((T(2) * rs * rsd) / (rs * rs));
      rsbd = rsbd + -(pr2d * qb + pr2 * qbd);
      rsb = rsb + -(pr2) * qb;
    }
    for (i64 c = n_o - 1; c >= 0; --c) {
      pbdr[c] = pbdr[c] + rsbd;
      pbr[c] = pbr[c] + rsb;
    }
    rsbd = T(0); rsb = T(0);
    for (i64 c = n_o - 1; c >= 0; --c) {
      const T oldbd = take(pbdr[c]), oldb = take(pbr[c]);
      const T e = jl_exp(zr[c] - m);
      const T ed = e * (zdr[c] - md);
      const T csed = ed * oldb + e * oldbd;
      const T cse = e * oldb;
      zbdr[c] = zbdr[c] + csed;
      zbr[c] = zbr[c] + cse;
      mbd = mbd + -csed;
      mb = mb + -cse;
    }
    for (i64 c = n_o - 1; c >= 1; --c) {
      const T m_prev = mt[c];
      const T oldbd = take(mbd), oldb = take(mb);
      const T zc = zr[c];
      const T g1 = d_max(m_prev, zc);
      const T g2 = d_max(zc, m_prev);
      mbd = mbd + g1 * oldbd;
      mb = mb + g1 * oldb;
      zbdr[c] = zbdr[c] + g2 * oldbd;
      zbr[c] = zbr[c] + g2 * oldb;
    }
    {
      const T oldbd = take(mbd), oldb = take(mb);
      zbdr[0] = zbdr[0] + oldbd;
      zbr[0] = zbr[0] + oldb;
    }
  }
  for (i64 idx2 = n_s * n_o - 1; idx2 >= 0; --idx2) {
    const i64 i_s = idx2 / n_o, c = idx2 % n_o;
    T oldbd = take(zbd[idx2]), oldb = take(zb[idx2]);
    s2bd = s2bd + oldbd;
    s2b = s2b + oldb;
    for (i64 k = n_h - 1; k >= 0; --k) {
      const T hv = h[i_s * n_h + k];
      w2bd[k * n_o + c] = w2bd[k * n_o + c] + (s2b * hd[i_s * n_h + k] + hv * s2bd);
      w2b[k * n_o + c] = w2b[k * n_o + c] + hv * s2b;
      const T wv = w2[k * n_o + c];
      hbd[i_s * n_h + k] = hbd[i_s * n_h + k] + (s2b * w2d[k * n_o + c] + wv * s2bd);
      hb[i_s * n_h + k] = hb[i_s * n_h + k] + wv * s2b;
    }
    oldbd = take(s2bd); oldb = take(s2b);
    b2bd[c] = b2bd[c] + oldbd;
    b2b[c] = b2b[c] + oldb;
  }
  for (i64 idx = n_s * n_h - 1; idx >= 0; --idx) {
    const i64 i_s = idx / n_h, j = idx % n_h;
    T s1d = b1d[j], s1 = b1[j];
    for (i64 k = 0; k < n_i; ++k) {
      const T xv = x[i_s * n_i + k], wv = w1[k * n_h + j];
      s1d = s1d + (xv * w1d[k * n_h + j] + wv * xd[i_s * n_i + k]);
      s1 = s1 + xv * wv;
    }
    T oldbd = take(hbd[idx]), oldb = take(hb[idx]);
    const T th = jl_tanh(s1);
    const T g = d_tanh(th);
    s1bd = s1bd + d_tanh_tangent(th, g, s1d, oldb, oldbd);
    s1b = s1b + g * oldb;
    oldbd = take(s1bd); oldb = take(s1b);
    for (i64 k = 0; k < n_i; ++k) {
      const T wdv = w1d[k * n_h + j], wv = w1[k * n_h + j];
      const T xdv = xd[i_s * n_i + k], xv = x[i_s * n_i + k];
      w1bd[k * n_h + j] = w1bd[k * n_h + j] + (oldb * xdv + xv * oldbd);
      w1b[k * n_h + j] = w1b[k * n_h + j] + xv * oldb;
      xbd[i_s * n_i + k] = xbd[i_s * n_i + k] + (oldb * wdv + wv * oldbd);
      xb[i_s * n_i + k] = xb[i_s * n_i + k] + wv * oldb;
    }
    b1bd[j] = b1bd[j] + oldbd;
    b1b[j] = b1b[j] + oldb;
  }
}

// ---------------------------------------------------------------------------
// C3 heat2d_b. Time loop with a tape of the state overwritten by the copy
// loop (advection_b.jl:1-37: slot ((i_x - 2) + (i_ - 1) * width) + 1, thread
// loop fastest), scatter adjoint of the stencil (stencil_loss_b.jl:12-21), the
// scalar float argument's adjoint returned by value (advection_b.jl:36).
template <class T>
T heat2d_b(T* loss, const T* lossb, T* u, T* ub, T* un, T* unb, T alpha, T alphab,
           i64 n, i64 n_step, T* u_stack) {
  const i64 nn = n * n;
  auto nbrs = [n](i64 idx, i64& up, i64& dn, i64& lf, i64& rt) {
    const i64 i = idx / n, j = idx % n;
    const i64 iu = (i - 1 + n) % n, id = (i + 1) % n, jl = (j - 1 + n) % n, jr = (j + 1) % n;
    up = iu * n + j; dn = id * n + j; lf = i * n + jl; rt = i * n + jr;
  };
  for (i64 it = 0; it < n_step; ++it) {                // for i_t = 1:n_step
    for (i64 idx = 0; idx < nn; ++idx) {
      i64 up, dn, lf, rt;
      nbrs(idx, up, dn, lf, rt);
      const T c = u[idx];
      un[idx] = c + alpha * ((((u[up] + u[dn]) + u[lf]) + u[rt]) - T(4) * c);
    }
    for (i64 idx2 = 0; idx2 < nn; ++idx2) {
      u_stack[idx2 + it * nn] = u[idx2];
      u[idx2] = un[idx2];
    }
  }
  for (i64 idx3 = 0; idx3 < nn; ++idx3) loss[0] = loss[0] + u[idx3] * u[idx3];
  // backward sweep
  for (i64 idx3 = nn - 1; idx3 >= 0; --idx3) ub[idx3] = ub[idx3] + d_sq(u[idx3]) * lossb[0];
  for (i64 it = n_step - 1; it >= 0; --it) {           // for i_t = n_step:-1:1
    for (i64 idx2 = nn - 1; idx2 >= 0; --idx2) {
      u[idx2] = u_stack[idx2 + it * nn];
      const T oldb = take(ub[idx2]);
      unb[idx2] = unb[idx2] + oldb;
    }
    for (i64 idx = nn - 1; idx >= 0; --idx) {
      i64 up, dn, lf, rt;
      nbrs(idx, up, dn, lf, rt);
      const T oldb = take(unb[idx]);
      const T c = u[idx];
      const T cse_a = alpha * oldb;
      ub[idx] = ub[idx] + oldb;
      alphab = alphab + ((((u[up] + u[dn]) + u[lf]) + u[rt]) - T(4) * c) * oldb;
      ub[up] = ub[up] + cse_a;
      ub[dn] = ub[dn] + cse_a;
      ub[lf] = ub[lf] + cse_a;
      ub[rt] = ub[rt] + cse_a;
      ub[idx] = ub[idx] + T(4) * -cse_a;
    }
  }
  return alphab;
}

// ---------------------------------------------------------------------------
// C4 conv1d_relu_mse_b. Valid convolution adjoint as selfrace_conv_b.jl:5-35
// (ab accumulated from the consumed zb, inner loops backwards, xb at the
// self-overlapping index t + ci - 1), ReLU through max(a, 0.0) with the der_
// partial 0.5 * (1 + sign(a - 0.0)) (src/STADE.jl:1489-1501), the local `a`
// recomputed in the reverse iteration (mlp1d_b.jl:43-47).
// inv_n is the primal's `1.0 / (n_b * n_o * n_lo)` of the whole batch: a block
// of samples (the parallel variant below) keeps the whole batch's value.
template <class T>
void conv1d_relu_mse_b_inv(T* loss, const T* lossb, const T* x, T* xb, const T* w, T* wb,
                           const T* t, T* tb, T* z, T* zb, T* r, T* rb,
                           i64 n_b, i64 n_c, i64 n_l, i64 n_o, i64 n_k, T inv_n) {
  const i64 n_lo = n_l - n_k + 1;
  const i64 nt = n_b * n_o * n_lo;
  T a = T(0), ab = T(0);
  auto conv_at = [&](i64 idx) {
    const i64 i_b = idx / (n_o * n_lo), i_o = (idx / n_lo) % n_o, i_t = idx % n_lo;
    T acc = T(0);
    for (i64 c = 0; c < n_c; ++c)
      for (i64 k = 0; k < n_k; ++k)
        acc = acc + w[(i_o * n_c + c) * n_k + k] * x[(i_b * n_c + c) * n_l + i_t + k];
    return acc;
  };
  for (i64 idx = 0; idx < nt; ++idx) {
    a = conv_at(idx);
    z[idx] = a;
    r[idx] = jl_max(a, T(0));
  }
  for (i64 idx2 = 0; idx2 < nt; ++idx2) {
    const T d = r[idx2] - t[idx2];
    loss[0] = loss[0] + inv_n * (d * d);
  }
  for (i64 idx2 = nt - 1; idx2 >= 0; --idx2) {
    const T cse0 = r[idx2] - t[idx2];
    const T cse1 = (inv_n * d_sq(cse0)) * lossb[0];
    rb[idx2] = rb[idx2] + cse1;
    tb[idx2] = tb[idx2] + -cse1;
  }
  for (i64 idx = nt - 1; idx >= 0; --idx) {
    const i64 i_b = idx / (n_o * n_lo), i_o = (idx / n_lo) % n_o, i_t = idx % n_lo;
    a = conv_at(idx);
    T oldb = take(rb[idx]);
    ab = ab + d_max(a, T(0)) * oldb;
    oldb = take(zb[idx]);
    ab = ab + oldb;
    for (i64 c = n_c - 1; c >= 0; --c) {
      for (i64 k = n_k - 1; k >= 0; --k) {
        const i64 xi = (i_b * n_c + c) * n_l + i_t + k;
        const i64 wi = (i_o * n_c + c) * n_k + k;
        wb[wi] = wb[wi] + x[xi] * ab;
        xb[xi] = xb[xi] + w[wi] * ab;
      }
    }
    ab = T(0);
  }
}
template <class T>
void conv1d_relu_mse_b(T* loss, const T* lossb, const T* x, T* xb, const T* w, T* wb,
                       const T* t, T* tb, T* z, T* zb, T* r, T* rb,
                       i64 n_b, i64 n_c, i64 n_l, i64 n_o, i64 n_k) {
  const T inv_n = T(1) / T(n_b * n_o * (n_l - n_k + 1));
  conv1d_relu_mse_b_inv(loss, lossb, x, xb, w, wb, t, tb, z, zb, r, rb, n_b, n_c, n_l, n_o, n_k,
                        inv_n);
}

// ---------------------------------------------------------------------------
// Tangent (forward-mode) sweeps `<k>_d`, tgen_emit (src/STADE.jl:3271-3279):
// one sweep in primal order; every active statement is preceded by its
// shadow line computed from the pre-statement values, `vd = sum_i partial_i
// * argd_i` (tgen_tangent_expr, src/STADE.jl:3350-3356, der_tangent_generic);
// arguments in tgen_signature_args order (src/STADE.jl:3306-3316): each float
// argument followed by its `d` shadow. No scalar argument is reassigned in
// these primals, so nothing is returned.

// C1 affine_ls_d
template <class T>
void affine_ls_d(T* loss, T* lossd, const T* w, const T* wd, const T* b, const T* bd,
                 const T* x, const T* xd, const T* t, const T* td, T* y, T* yd,
                 i64 n_s, i64 n_o, i64 n_i) {
  for (i64 idx = 0; idx < n_s * n_o; ++idx) {
    const i64 i_s = idx / n_o, i_o = idx % n_o;
    T sd = bd[i_o], s = b[i_o];
    for (i64 k = 0; k < n_i; ++k) {
      const T wv = w[i_o * n_i + k], xv = x[i_s * n_i + k];
      sd = sd + (wd[i_o * n_i + k] * xv + wv * xd[i_s * n_i + k]);
      s = s + wv * xv;
    }
    yd[idx] = sd;
    y[idx] = s;
  }
  for (i64 idx2 = 0; idx2 < n_s * n_o; ++idx2) {
    const T d = y[idx2] - t[idx2];
    lossd[0] = lossd[0] + T(0.5) * ((T(2) * d) * (yd[idx2] - td[idx2]));
    loss[0] = loss[0] + T(0.5) * (d * d);
  }
}

// C2 mlp2_ce_d (the forward half of mlp2_ce_hv: the same tangent lines)
template <class T>
void mlp2_ce_d(T* loss, T* lossd, const T* x, const T* xd, const T* y, const T* yd,
               const T* w1, const T* w1d, const T* b1, const T* b1d, const T* w2, const T* w2d,
               const T* b2, const T* b2d, T* h, T* hd, T* z, T* zd, T* p, T* pd,
               i64 n_s, i64 n_i, i64 n_h, i64 n_o) {
  for (i64 idx = 0; idx < n_s * n_h; ++idx) {
    const i64 i_s = idx / n_h, j = idx % n_h;
    T s1d = b1d[j], s1 = b1[j];
    for (i64 k = 0; k < n_i; ++k) {
      const T xv = x[i_s * n_i + k], wv = w1[k * n_h + j];
      s1d = s1d + (xv * w1d[k * n_h + j] + wv * xd[i_s * n_i + k]);
      s1 = s1 + xv * wv;
    }
    const T th = jl_tanh(s1);
    hd[idx] = (T(1) - th * th) * s1d;
    h[idx] = th;
  }
  for (i64 idx2 = 0; idx2 < n_s * n_o; ++idx2) {
    const i64 i_s = idx2 / n_o, c = idx2 % n_o;
    T s2d = b2d[c], s2 = b2[c];
    for (i64 k = 0; k < n_h; ++k) {
      const T hv = h[i_s * n_h + k], wv = w2[k * n_o + c];
      s2d = s2d + (hv * w2d[k * n_o + c] + wv * hd[i_s * n_h + k]);
      s2 = s2 + wv * hv;
    }
    zd[idx2] = s2d;
    z[idx2] = s2;
  }
  for (i64 i_s = 0; i_s < n_s; ++i_s) {
    const T* zr = z + i_s * n_o; const T* zdr = zd + i_s * n_o;
    T* pr = p + i_s * n_o; T* pdr = pd + i_s * n_o;
    T m = zr[0], md = zdr[0];
    for (i64 c = 1; c < n_o; ++c) {
      const T g1 = d_max(m, zr[c]);
      const T g2 = d_max(zr[c], m);
      md = g1 * md + g2 * zdr[c];
      m = jl_max(m, zr[c]);
    }
    for (i64 c = 0; c < n_o; ++c) {
      const T e = jl_exp(zr[c] - m);
      pdr[c] = e * (zdr[c] - md);
      pr[c] = e;
    }
    T rs = T(0), rsd = T(0);
    for (i64 c = 0; c < n_o; ++c) { rsd = rsd + pdr[c]; rs = rs + pr[c]; }
    for (i64 c = 0; c < n_o; ++c) {
      const T q = pr[c] / rs;
      const T qd = pdr[c] / rs - (pr[c] / (rs * rs)) * rsd;
      lossd[0] = lossd[0] - (yd[i_s * n_o + c] * jl_log(q) + y[i_s * n_o + c] * (qd / q));
      loss[0] = loss[0] - y[i_s * n_o + c] * jl_log(q);
    }
  }
}

// C3 heat2d_d: un's shadow from u's before each step, then u = un with ud = und
template <class T>
void heat2d_d(T* loss, T* lossd, T* u, T* ud, T* un, T* und, T alpha, T alphad, i64 n,
              i64 n_step) {
  const i64 nn = n * n;
  for (i64 it = 0; it < n_step; ++it) {
    for (i64 idx = 0; idx < nn; ++idx) {
      const i64 i = idx / n, j = idx % n;
      const i64 up = ((i - 1 + n) % n) * n + j, dn = ((i + 1) % n) * n + j;
      const i64 lf = i * n + (j - 1 + n) % n, rt = i * n + (j + 1) % n;
      const T c = u[idx], cd = ud[idx];
      const T lap = (((u[up] + u[dn]) + u[lf]) + u[rt]) - T(4) * c;
      const T lapd = (((ud[up] + ud[dn]) + ud[lf]) + ud[rt]) - T(4) * cd;
      und[idx] = cd + (alphad * lap + alpha * lapd);
      un[idx] = c + alpha * lap;
    }
    for (i64 idx2 = 0; idx2 < nn; ++idx2) {
      ud[idx2] = und[idx2];
      u[idx2] = un[idx2];
    }
  }
  for (i64 idx3 = 0; idx3 < nn; ++idx3) {
    lossd[0] = lossd[0] + (T(2) * u[idx3]) * ud[idx3];
    loss[0] = loss[0] + u[idx3] * u[idx3];
  }
}

// C4 conv1d_relu_mse_d: max(a, 0)'s tangent 0.5 (1 + sign(a - 0)) ad
template <class T>
void conv1d_relu_mse_d(T* loss, T* lossd, const T* x, const T* xd, const T* w, const T* wd,
                       const T* t, const T* td, T* z, T* zd, T* r, T* rd,
                       i64 n_b, i64 n_c, i64 n_l, i64 n_o, i64 n_k) {
  const i64 n_lo = n_l - n_k + 1;
  const i64 nt = n_b * n_o * n_lo;
  for (i64 idx = 0; idx < nt; ++idx) {
    const i64 i_b = idx / (n_o * n_lo), i_o = (idx / n_lo) % n_o, i_t = idx % n_lo;
    T a = T(0), ad = T(0);
    for (i64 c = 0; c < n_c; ++c)
      for (i64 k = 0; k < n_k; ++k) {
        const i64 wi = (i_o * n_c + c) * n_k + k, xi = (i_b * n_c + c) * n_l + i_t + k;
        ad = ad + (wd[wi] * x[xi] + w[wi] * xd[xi]);
        a = a + w[wi] * x[xi];
      }
    zd[idx] = ad;
    z[idx] = a;
    rd[idx] = d_max(a, T(0)) * ad;
    r[idx] = jl_max(a, T(0));
  }
  const T inv_n = T(1) / T(nt);
  for (i64 idx2 = 0; idx2 < nt; ++idx2) {
    const T d = r[idx2] - t[idx2];
    lossd[0] = lossd[0] + inv_n * ((T(2) * d) * (rd[idx2] - td[idx2]));
    loss[0] = loss[0] + inv_n * (d * d);
  }
}

// ---------------------------------------------------------------------------
// Parallel CPU variants (the timed CPU baseline and the checks at the full
// configuration sizes): samples split across host threads, each with private
// copies of the summed shadows, then one fixed-order sum. Same arithmetic per
// sample as the serial sweeps above; only the order in which the per-sample
// contributions to a summed shadow are added differs.

// Threads over contiguous sample blocks; each block's summed shadows go to
// private zeroed copies (`my`), added to the outputs afterwards in block
// order. `run(lo, hi, my)` runs the serial sweep on samples [lo, hi).
template <class T, class Run>
void over_sample_blocks(i64 n_s, int nthreads, size_t private_len, Run run,
                        const std::vector<std::pair<T*, i64>>& outs) {
#ifdef _OPENMP
  if (nthreads <= 0) nthreads = omp_get_max_threads();
#else
  nthreads = 1;
#endif
  std::vector<T> part((size_t)nthreads * private_len, T(0));
#pragma omp parallel num_threads(nthreads)
  {
#ifdef _OPENMP
    const int tid = omp_get_thread_num();
#else
    const int tid = 0;
#endif
    const i64 lo = n_s * tid / nthreads, hi = n_s * (tid + 1) / nthreads;
    if (hi > lo) run(lo, hi, part.data() + (size_t)tid * private_len);
  }
  for (int tid = 0; tid < nthreads; ++tid) {
    const T* my = part.data() + (size_t)tid * private_len;
    for (const auto& o : outs) {
      for (i64 i = 0; i < o.second; ++i) o.first[i] += my[i];
      my += o.second;
    }
  }
}

template <class T>
void mlp2_ce_b_omp(T* loss, const T* lossb, const T* x, T* xb, const T* y, T* yb,
                   const T* w1, T* w1b, const T* b1, T* b1b, const T* w2, T* w2b,
                   const T* b2, T* b2b, T* h, T* hb, T* z, T* zb, T* p, T* pb,
                   i64 n_s, i64 n_i, i64 n_h, i64 n_o, int nthreads) {
  const i64 nw1 = n_i * n_h, nw2 = n_h * n_o;
  over_sample_blocks<T>(
      n_s, nthreads, (size_t)(nw1 + n_h + nw2 + n_o + 1),
      [&](i64 lo, i64 hi, T* my) {
        const i64 io = lo * n_i, oo = lo * n_o, ho = lo * n_h;
        mlp2_ce_b(my + nw1 + n_h + nw2 + n_o, lossb, x + io, xb + io, y + oo, yb + oo, w1, my,
                  b1, my + nw1, w2, my + nw1 + n_h, b2, my + nw1 + n_h + nw2, h + ho, hb + ho,
                  z + oo, zb + oo, p + oo, pb + oo, hi - lo, n_i, n_h, n_o);
      },
      {{w1b, nw1}, {b1b, n_h}, {w2b, nw2}, {b2b, n_o}, {loss, 1}});
}

// C3 heat2d_b with every per-cell loop parallel over cells and bit-identical
// to the serial sweep above. The loss and alphab sums stay serial in the
// generated order. The reverse stencil loop scatters into ub[up], ub[dn],
// ub[lf], ub[rt] and ub[idx]; here each cell instead gathers, from the (at
// most five) iterations that write it, their additions sorted the way the
// serial loop performs them (iteration index descending, then statement
// order), so every cell sees the same additions in the same order. ub is zero
// when that loop starts (the restore loop above consumed it).
template <class T>
T heat2d_b_omp(T* loss, const T* lossb, T* u, T* ub, T* un, T* unb, T alpha, T alphab,
               i64 n, i64 n_step, T* u_stack, int nthreads) {
#ifdef _OPENMP
  if (nthreads <= 0) nthreads = omp_get_max_threads();
#else
  nthreads = 1;
#endif
  const i64 nn = n * n;
  // neighbours of cell (i, j) without division: rows and columns wrap
  auto up_row = [n](i64 i) { return i == 0 ? n - 1 : i - 1; };
  auto dn_row = [n](i64 i) { return i == n - 1 ? 0 : i + 1; };
  auto lf_col = [n](i64 j) { return j == 0 ? n - 1 : j - 1; };
  auto rt_col = [n](i64 j) { return j == n - 1 ? 0 : j + 1; };
  auto stencil = [&](const T* v, i64 i, i64 j) {
    const T c = v[i * n + j];
    return ((((v[up_row(i) * n + j] + v[dn_row(i) * n + j]) + v[i * n + lf_col(j)]) +
             v[i * n + rt_col(j)]) - T(4) * c);
  };
  for (i64 it = 0; it < n_step; ++it) {
#pragma omp parallel for schedule(static) num_threads(nthreads)
    for (i64 i = 0; i < n; ++i)
      for (i64 j = 0; j < n; ++j) un[i * n + j] = u[i * n + j] + alpha * stencil(u, i, j);
#pragma omp parallel for schedule(static) num_threads(nthreads)
    for (i64 idx2 = 0; idx2 < nn; ++idx2) {
      u_stack[idx2 + it * nn] = u[idx2];
      u[idx2] = un[idx2];
    }
  }
  for (i64 idx3 = 0; idx3 < nn; ++idx3) loss[0] = loss[0] + u[idx3] * u[idx3];
#pragma omp parallel for schedule(static) num_threads(nthreads)
  for (i64 idx3 = 0; idx3 < nn; ++idx3) ub[idx3] = ub[idx3] + (T(2) * u[idx3]) * lossb[0];
  for (i64 it = n_step - 1; it >= 0; --it) {
#pragma omp parallel for schedule(static) num_threads(nthreads)
    for (i64 idx2 = 0; idx2 < nn; ++idx2) {
      u[idx2] = u_stack[idx2 + it * nn];
      const T oldb = ub[idx2];
      ub[idx2] = T(0);
      unb[idx2] = unb[idx2] + oldb;
    }
    // alphab, serial in the generated (descending) order
    for (i64 i = n - 1; i >= 0; --i)
      for (i64 j = n - 1; j >= 0; --j) alphab = alphab + stencil(u, i, j) * unb[i * n + j];
    // ub from the reverse stencil loop. Iteration k of that loop adds, in
    // order: oldb_k to ub[k]; a_k = alpha oldb_k to ub[up], ub[dn], ub[lf],
    // ub[rt]; 4 * -a_k to ub[k]; and the loop runs k descending. Each cell
    // collects the additions that land on it and applies them sorted by
    // (k descending, statement ascending), as the serial loop does.
#pragma omp parallel for schedule(static) num_threads(nthreads)
    for (i64 i = 0; i < n; ++i) {
      for (i64 j = 0; j < n; ++j) {
        const i64 cell = i * n + j;
        i64 key_it[30];
        int key_st[30];
        T val[30];
        int m = 0;
        const i64 cand[5] = {dn_row(i) * n + j, up_row(i) * n + j, i * n + rt_col(j),
                             i * n + lf_col(j), cell};
        for (int a = 0; a < 5; ++a) {
          const i64 k = cand[a];
          bool seen = false;
          for (int b = 0; b < a; ++b) seen = seen || cand[b] == k;
          if (seen) continue;
          const i64 ki = k / n, kj = k % n;
          const T oldb = unb[k];
          const T cse_a = alpha * oldb;
          const i64 tgt[6] = {k, up_row(ki) * n + kj, dn_row(ki) * n + kj, ki * n + lf_col(kj),
                              ki * n + rt_col(kj), k};
          const T v[6] = {oldb, cse_a, cse_a, cse_a, cse_a, T(4) * -cse_a};
          for (int st = 0; st < 6; ++st)
            if (tgt[st] == cell) { key_it[m] = k; key_st[m] = st; val[m] = v[st]; ++m; }
        }
        for (int x = 1; x < m; ++x)
          for (int y = x; y > 0; --y) {
            const bool later = key_it[y] > key_it[y - 1] ||
                               (key_it[y] == key_it[y - 1] && key_st[y] < key_st[y - 1]);
            if (!later) break;
            std::swap(key_it[y], key_it[y - 1]);
            std::swap(key_st[y], key_st[y - 1]);
            std::swap(val[y], val[y - 1]);
          }
        T acc = ub[cell];
        for (int x = 0; x < m; ++x) acc = acc + val[x];
        ub[cell] = acc;
      }
    }
#pragma omp parallel for schedule(static) num_threads(nthreads)
    for (i64 idx = 0; idx < nn; ++idx) unb[idx] = T(0);
  }
  return alphab;
}

template <class T>
void conv1d_relu_mse_b_omp(T* loss, const T* lossb, const T* x, T* xb, const T* w, T* wb,
                           const T* t, T* tb, T* z, T* zb, T* r, T* rb,
                           i64 n_b, i64 n_c, i64 n_l, i64 n_o, i64 n_k, int nthreads) {
  const i64 n_lo = n_l - n_k + 1, nw = n_o * n_c * n_k;
  const T inv_n = T(1) / T(n_b * n_o * n_lo);
  over_sample_blocks<T>(
      n_b, nthreads, (size_t)(nw + 1),
      [&](i64 lo, i64 hi, T* my) {
        const i64 xo = lo * n_c * n_l, to = lo * n_o * n_lo;
        conv1d_relu_mse_b_inv(my + nw, lossb, x + xo, xb + xo, w, my, t + to, tb + to, z + to,
                              zb + to, r + to, rb + to, hi - lo, n_c, n_l, n_o, n_k, inv_n);
      },
      {{wb, nw}, {loss, 1}});
}

template <class T>
void mlp2_ce_hv_omp(T* loss, const T* lossb, const T* x, T* xb, const T* y, T* yb,
                    const T* w1, T* w1b, const T* b1, T* b1b, const T* w2, T* w2b,
                    const T* b2, T* b2b, T* h, T* hb, T* z, T* zb, T* p, T* pb,
                    i64 n_s, i64 n_i, i64 n_h, i64 n_o,
                    T* lossd, const T* lossbd, const T* xd, T* xbd, const T* yd, T* ybd,
                    const T* w1d, T* w1bd, const T* b1d, T* b1bd, const T* w2d, T* w2bd,
                    const T* b2d, T* b2bd, T* hd, T* hbd, T* zd, T* zbd, T* pd, T* pbd,
                    int nthreads) {
  const i64 nw1 = n_i * n_h, nw2 = n_h * n_o;
  const i64 one = nw1 + n_h + nw2 + n_o + 1;  // w1b b1b w2b b2b loss
  over_sample_blocks<T>(
      n_s, nthreads, (size_t)(2 * one),
      [&](i64 lo, i64 hi, T* my) {
        T* mb = my;          // adjoint shadows
        T* md = my + one;    // their tangents
        const i64 io = lo * n_i, oo = lo * n_o, ho = lo * n_h;
        mlp2_ce_hv(mb + nw1 + n_h + nw2 + n_o, lossb, x + io, xb + io, y + oo, yb + oo, w1, mb,
                   b1, mb + nw1, w2, mb + nw1 + n_h, b2, mb + nw1 + n_h + nw2, h + ho, hb + ho,
                   z + oo, zb + oo, p + oo, pb + oo, hi - lo, n_i, n_h, n_o,
                   md + nw1 + n_h + nw2 + n_o, lossbd, xd + io, xbd + io, yd + oo, ybd + oo, w1d,
                   md, b1d, md + nw1, w2d, md + nw1 + n_h, b2d, md + nw1 + n_h + nw2, hd + ho,
                   hbd + ho, zd + oo, zbd + oo, pd + oo, pbd + oo);
      },
      {{w1b, nw1}, {b1b, n_h}, {w2b, nw2}, {b2b, n_o}, {loss, 1},
       {w1bd, nw1}, {b1bd, n_h}, {w2bd, nw2}, {b2bd, n_o}, {lossd, 1}});
}


// ---------------------------------------------------------------------------
// Restated reference exemplars. Seven sweeps the reference ships as generated
// text (test/val-corpus/*.jl, written by STADE with keep_push_pop = false and
// fuse_ii_loops = true), restated statement for statement on the rule helpers
// above. tests/test_exemplar_pins.py runs each on seeded inputs and requires
// the results to equal, bit for bit, the reference text itself run by the
// interpreter tests/jlsub.py (fixtures written by
// tests/golden/make_exemplar_golden.py). That pins the rules the five sweeps
// use (take, d_sq, d_tanh, d_max through mlp1d's max-free form, d_tanh_tangent,
// the tape slot formula, the recompute of locals, the HVP doubling order).
// Loop direction: under fuse_ii_loops = true the generator emits an
// iteration-independent loop's adjoint un-reversed (agen_emit_ii_loop,
// src/STADE.jl:6309; mlp1d_b.jl:58, 77 run ascending), as restated here. The
// five sweeps above target the library default, fuse_ii_loops = false, under
// which every backward loop reverses (src/STADE.jl:6553-6557).

// affine_loss_b.jl:5-23
template <class T>
void ex_affine_loss_b(T* loss, const T* lossb, const T* u, T* ub, const T* a, T* ab, const T* b,
                      T* bb, T* v, T* vb, i64 n) {
  for (i64 i = 0; i < n; ++i) v[i] = a[i] * u[i] + b[i];
  for (i64 i = 0; i < n; ++i) loss[0] = loss[0] + v[i] * v[i];
  for (i64 i = n - 1; i >= 0; --i) vb[i] = vb[i] + d_sq(v[i]) * lossb[0];
  for (i64 i = n - 1; i >= 0; --i) {
    const T oldb = take(vb[i]);
    ab[i] = ab[i] + u[i] * oldb;
    ub[i] = ub[i] + a[i] * oldb;
    bb[i] = bb[i] + oldb;
  }
}

// matvec_loss_b.jl:5-27; a is i_m x i_n, column-major (a[i, j] at j * m + i)
template <class T>
void ex_matvec_loss_b(T* loss, const T* lossb, const T* a, T* ab, const T* u, T* ub, T* v, T* vb,
                      i64 m, i64 n) {
  for (i64 idx = 0; idx < m * n; ++idx) {
    const i64 i = idx / n, j = idx % n;
    v[i] = v[i] + a[j * m + i] * u[j];
  }
  for (i64 i = 0; i < m; ++i) loss[0] = loss[0] + v[i] * v[i];
  for (i64 i = m - 1; i >= 0; --i) vb[i] = vb[i] + d_sq(v[i]) * lossb[0];
  for (i64 idx = m * n - 1; idx >= 0; --idx) {
    const i64 i = idx / n, j = idx % n;
    const T cse = vb[i];
    ab[j * m + i] = ab[j * m + i] + u[j] * cse;
    ub[j] = ub[j] + a[j * m + i] * cse;
  }
}

// stencil_loss_b.jl:5-23 (the generated scatter adjoint of the 3-point stencil)
template <class T>
void ex_stencil_loss_b(T* loss, const T* lossb, const T* u, T* ub, T* w, T* wb, i64 n) {
  for (i64 i = 1; i < n - 1; ++i) w[i] = (u[i - 1] - T(2) * u[i]) + u[i + 1];
  for (i64 i = 1; i < n - 1; ++i) loss[0] = loss[0] + w[i] * w[i];
  for (i64 i = n - 2; i >= 1; --i) wb[i] = wb[i] + d_sq(w[i]) * lossb[0];
  for (i64 i = n - 2; i >= 1; --i) {
    const T oldb = take(wb[i]);
    ub[i - 1] = ub[i - 1] + oldb;
    ub[i] = ub[i] + T(2) * -oldb;
    ub[i + 1] = ub[i + 1] + oldb;
  }
}

// advection_b.jl:6-37: time loop with the overwritten du taped at slot
// ((i_x - 2) + (i_ - 1) * (nnode - 1)) + 1; the scalar arguments' adjoints
// in / out (the generated code returns (cb, dxb, dtb))
template <class T>
void ex_advection_b(T* u, T* ub, T* du, T* dub, T c, T* cb, T dx, T* dxb, T dt, T* dtb,
                    i64 nstep, i64 nnode, T* du_stack) {
  const i64 width = nnode - 1;
  for (i64 it = 0; it < nstep; ++it) {
    for (i64 x = 1; x < nnode; ++x) {
      du_stack[(x - 1) + it * width] = du[x];
      du[x] = u[x] - u[x - 1];
    }
    for (i64 x = 1; x < nnode; ++x) u[x] = u[x] - (c * dt * du[x]) / dx;
  }
  for (i64 it = nstep - 1; it >= 0; --it) {
    for (i64 x = nnode - 1; x >= 1; --x) {
      const T cse0 = du[x];
      const T cse1 = -(ub[x]);
      const T cse2 = (T(1) / dx) * cse1;
      *cb = *cb + (dt * cse0) * cse2;
      *dtb = *dtb + (c * cse0) * cse2;
      dub[x] = dub[x] + (c * dt) * cse2;
      *dxb = *dxb + -((c * dt * cse0) / (dx * dx)) * cse1;
    }
    for (i64 x = nnode - 1; x >= 1; --x) {
      du[x] = du_stack[(x - 1) + it * width];
      const T oldb = take(dub[x]);
      ub[x] = ub[x] + oldb;
      ub[x - 1] = ub[x - 1] + -oldb;
    }
  }
}

// selfrace_conv_b.jl:5-35: valid convolution, the local `a` reset per
// output, `loss += z * z` giving two adjoint adds, xb at the self-overlapping
// index t + ci - 1
template <class T>
void ex_selfrace_conv_b(const T* x, T* xb, const T* w, T* wb, T* z, T* zb, T* loss,
                        const T* lossb, i64 n, i64 nc) {
  T a = T(0), ab = T(0);
  for (i64 t = 0; t < n; ++t) {
    a = T(0);
    for (i64 ci = 0; ci < nc; ++ci) a = a + x[t + ci] * w[ci];
    z[t] = a;
  }
  for (i64 m = 0; m < n; ++m) {
    const T cse0 = z[m];
    loss[0] = loss[0] + cse0 * cse0;
  }
  for (i64 m = n - 1; m >= 0; --m) {
    const T cse1 = z[m] * lossb[0];
    zb[m] = zb[m] + cse1;
    zb[m] = zb[m] + cse1;
  }
  for (i64 t = n - 1; t >= 0; --t) {
    const T oldb = take(zb[t]);
    ab = ab + oldb;
    for (i64 ci = nc - 1; ci >= 0; --ci) {
      xb[t + ci] = xb[t + ci] + w[ci] * ab;
      wb[ci] = wb[ci] + x[t + ci] * ab;
    }
    ab = T(0);
  }
}

// mlp1d_b.jl:5-78: 1 -> n_h -> n_h -> 1 tanh MLP, squared error; the hidden
// loops' adjoints recompute their local sums and run ascending (ii loops)
template <class T>
void ex_mlp1d_b(T* loss, const T* lossb, const T* x, T* xb, const T* y, T* yb, const T* w1,
                T* w1b, const T* b1, T* b1b, const T* w2, T* w2b, const T* b2, T* b2b,
                const T* w3, T* w3b, const T* b3, T* b3b, T* h1, T* h1b, T* h2, T* h2b, T* o,
                T* ob, i64 nh) {
  T s1 = T(0), s2 = T(0), s3 = T(0), s1b = T(0), s2b = T(0), s3b = T(0);
  for (i64 j = 0; j < nh; ++j) {
    s1 = w1[j] * x[0] + b1[j];
    h1[j] = jl_tanh(s1);
  }
  for (i64 j2 = 0; j2 < nh; ++j2) {
    s2 = b2[j2];
    for (i64 k = 0; k < nh; ++k) s2 = s2 + w2[j2 * nh + k] * h1[k];
    h2[j2] = jl_tanh(s2);
  }
  s3 = b3[0];
  for (i64 k2 = 0; k2 < nh; ++k2) s3 = s3 + w3[k2] * h2[k2];
  o[0] = s3;
  const T cse0 = o[0] - y[0];
  loss[0] = loss[0] + cse0 * cse0;
  const T cse1 = d_sq(cse0) * lossb[0];
  ob[0] = ob[0] + cse1;
  yb[0] = yb[0] + -cse1;
  T oldb = take(ob[0]);
  s3b = s3b + oldb;
  for (i64 k2 = nh - 1; k2 >= 0; --k2) {
    w3b[k2] = w3b[k2] + h2[k2] * s3b;
    h2b[k2] = h2b[k2] + w3[k2] * s3b;
  }
  oldb = take(s3b);
  b3b[0] = b3b[0] + oldb;
  for (i64 j2 = 0; j2 < nh; ++j2) {
    s2 = b2[j2];
    for (i64 k = 0; k < nh; ++k) s2 = s2 + w2[j2 * nh + k] * h1[k];
    oldb = take(h2b[j2]);
    s2b = s2b + d_tanh(jl_tanh(s2)) * oldb;
    for (i64 k = 0; k < nh; ++k) {
      const T cse2 = w2[j2 * nh + k], cse3 = h1[k];
      s2 = s2 + cse2 * cse3;
      w2b[j2 * nh + k] = w2b[j2 * nh + k] + cse3 * s2b;
      h1b[k] = h1b[k] + cse2 * s2b;
    }
    oldb = take(s2b);
    b2b[j2] = b2b[j2] + oldb;
  }
  for (i64 j = 0; j < nh; ++j) {
    const T cse4 = w1[j], cse5 = x[0];
    const T cse6 = cse4 * cse5 + b1[j];
    s1 = cse6;
    oldb = take(h1b[j]);
    s1b = s1b + d_tanh(jl_tanh(s1)) * oldb;
    oldb = take(s1b);
    w1b[j] = w1b[j] + cse5 * oldb;
    xb[0] = xb[0] + cse4 * oldb;
    b1b[j] = b1b[j] + oldb;
  }
}

// mlp1d_hv.jl:5-150: the HVP of mlp1d; every statement's tangent twin first
template <class T>
void ex_mlp1d_hv(T* loss, const T* lossb, const T* x, T* xb, const T* y, T* yb, const T* w1,
                 T* w1b, const T* b1, T* b1b, const T* w2, T* w2b, const T* b2, T* b2b,
                 const T* w3, T* w3b, const T* b3, T* b3b, T* h1, T* h1b, T* h2, T* h2b, T* o,
                 T* ob, i64 nh, T* lossd, const T* lossbd, const T* xd, T* xbd, const T* yd,
                 T* ybd, const T* w1d, T* w1bd, const T* b1d, T* b1bd, const T* w2d, T* w2bd,
                 const T* b2d, T* b2bd, const T* w3d, T* w3bd, const T* b3d, T* b3bd, T* h1d,
                 T* h1bd, T* h2d, T* h2bd, T* od, T* obd) {
  T s1 = 0, s2 = 0, s3 = 0, s1b = 0, s2b = 0, s3b = 0;
  T s1d = 0, s1bd = 0, s2d = 0, s2bd = 0, s3d = 0, s3bd = 0;
  for (i64 j = 0; j < nh; ++j) {
    const T hx = x[0], hw = w1[j];
    s1d = (hx * w1d[j] + hw * xd[0]) + b1d[j];
    s1 = hw * hx + b1[j];
    const T th = jl_tanh(s1);
    h1d[j] = d_tanh(th) * s1d;
    h1[j] = th;
  }
  for (i64 j2 = 0; j2 < nh; ++j2) {
    s2d = b2d[j2];
    s2 = b2[j2];
    for (i64 k = 0; k < nh; ++k) {
      const T hh = h1[k], hw = w2[j2 * nh + k];
      s2d = s2d + (hh * w2d[j2 * nh + k] + hw * h1d[k]);
      s2 = s2 + hw * hh;
    }
    const T th = jl_tanh(s2);
    h2d[j2] = d_tanh(th) * s2d;
    h2[j2] = th;
  }
  s3d = b3d[0];
  s3 = b3[0];
  for (i64 k2 = 0; k2 < nh; ++k2) {
    const T hh = h2[k2], hw = w3[k2];
    s3d = s3d + (hh * w3d[k2] + hw * h2d[k2]);
    s3 = s3 + hw * hh;
  }
  od[0] = s3d;
  o[0] = s3;
  const T e = o[0] - y[0];
  const T e2 = d_sq(e);
  const T ed = od[0] + -(yd[0]);
  lossd[0] = lossd[0] + e2 * ed;
  loss[0] = loss[0] + e * e;
  const T lb = lossb[0];
  const T cse0d = lb * d_sq(ed) + e2 * lossbd[0];
  const T cse0 = e2 * lb;
  obd[0] = obd[0] + cse0d;
  ob[0] = ob[0] + cse0;
  ybd[0] = ybd[0] + -cse0d;
  yb[0] = yb[0] + -cse0;
  T oldbd = take(obd[0]), oldb = take(ob[0]);
  s3bd = s3bd + oldbd;
  s3b = s3b + oldb;
  for (i64 k2 = nh - 1; k2 >= 0; --k2) {
    const T hh = h2[k2];
    w3bd[k2] = w3bd[k2] + (s3b * h2d[k2] + hh * s3bd);
    w3b[k2] = w3b[k2] + hh * s3b;
    const T hw = w3[k2];
    h2bd[k2] = h2bd[k2] + (s3b * w3d[k2] + hw * s3bd);
    h2b[k2] = h2b[k2] + hw * s3b;
  }
  oldbd = take(s3bd);
  oldb = take(s3b);
  b3bd[0] = b3bd[0] + oldbd;
  b3b[0] = b3b[0] + oldb;
  for (i64 j2 = 0; j2 < nh; ++j2) {
    s2d = b2d[j2];
    s2 = b2[j2];
    for (i64 k = 0; k < nh; ++k) {
      const T hh = h1[k], hw = w2[j2 * nh + k];
      s2d = s2d + (hh * w2d[j2 * nh + k] + hw * h1d[k]);
      s2 = s2 + hw * hh;
    }
    oldbd = take(h2bd[j2]);
    oldb = take(h2b[j2]);
    const T th = jl_tanh(s2);
    const T g = d_tanh(th);
    s2bd = s2bd + d_tanh_tangent(th, g, s2d, oldb, oldbd);
    s2b = s2b + g * oldb;
    for (i64 k = 0; k < nh; ++k) {
      const T c1d = w2d[j2 * nh + k], c1 = w2[j2 * nh + k];
      const T c2d = h1d[k], c2 = h1[k];
      s2d = s2d + (c2 * c1d + c1 * c2d);
      s2 = s2 + c1 * c2;
      w2bd[j2 * nh + k] = w2bd[j2 * nh + k] + (s2b * c2d + c2 * s2bd);
      w2b[j2 * nh + k] = w2b[j2 * nh + k] + c2 * s2b;
      h1bd[k] = h1bd[k] + (s2b * c1d + c1 * s2bd);
      h1b[k] = h1b[k] + c1 * s2b;
    }
    oldbd = take(s2bd);
    oldb = take(s2b);
    b2bd[j2] = b2bd[j2] + oldbd;
    b2b[j2] = b2b[j2] + oldb;
  }
  for (i64 j = 0; j < nh; ++j) {
    const T c3d = w1d[j], c3 = w1[j], c4d = xd[0], c4 = x[0];
    const T c5d = (c4 * c3d + c3 * c4d) + b1d[j];
    const T c5 = c3 * c4 + b1[j];
    s1d = c5d;
    s1 = c5;
    oldbd = take(h1bd[j]);
    oldb = take(h1b[j]);
    const T th = jl_tanh(s1);
    const T g = d_tanh(th);
    s1bd = s1bd + d_tanh_tangent(th, g, s1d, oldb, oldbd);
    s1b = s1b + g * oldb;
    oldbd = take(s1bd);
    oldb = take(s1b);
    w1bd[j] = w1bd[j] + (oldb * c4d + c4 * oldbd);
    w1b[j] = w1b[j] + c4 * oldb;
    xbd[0] = xbd[0] + (oldb * c3d + c3 * oldbd);
    xb[0] = xb[0] + c3 * oldb;
    b1bd[j] = b1bd[j] + oldbd;
    b1b[j] = b1b[j] + oldb;
  }
}

}  // namespace

extern "C" {

// ---- restated reference exemplars, Float64 ----
void oracle_ex_affine_loss_b_f64(double* loss, const double* lossb, const double* u, double* ub,
                                 const double* a, double* ab, const double* b, double* bb,
                                 double* v, double* vb, i64 n) {
  ex_affine_loss_b(loss, lossb, u, ub, a, ab, b, bb, v, vb, n);
}
void oracle_ex_matvec_loss_b_f64(double* loss, const double* lossb, const double* a, double* ab,
                                 const double* u, double* ub, double* v, double* vb, i64 m,
                                 i64 n) {
  ex_matvec_loss_b(loss, lossb, a, ab, u, ub, v, vb, m, n);
}
void oracle_ex_stencil_loss_b_f64(double* loss, const double* lossb, const double* u, double* ub,
                                  double* w, double* wb, i64 n) {
  ex_stencil_loss_b(loss, lossb, u, ub, w, wb, n);
}
void oracle_ex_advection_b_f64(double* u, double* ub, double* du, double* dub, double c,
                               double* cb, double dx, double* dxb, double dt, double* dtb,
                               i64 nstep, i64 nnode, double* du_stack) {
  ex_advection_b(u, ub, du, dub, c, cb, dx, dxb, dt, dtb, nstep, nnode, du_stack);
}
void oracle_ex_selfrace_conv_b_f64(const double* x, double* xb, const double* w, double* wb,
                                   double* z, double* zb, double* loss, const double* lossb,
                                   i64 n, i64 nc) {
  ex_selfrace_conv_b(x, xb, w, wb, z, zb, loss, lossb, n, nc);
}
#define MLP1D_B_ARGS(T)                                                                    \
  T *loss, const T *lossb, const T *x, T *xb, const T *y, T *yb, const T *w1, T *w1b,     \
      const T *b1, T *b1b, const T *w2, T *w2b, const T *b2, T *b2b, const T *w3, T *w3b,  \
      const T *b3, T *b3b, T *h1, T *h1b, T *h2, T *h2b, T *o, T *ob, i64 nh
#define MLP1D_B_PASS                                                                       \
  loss, lossb, x, xb, y, yb, w1, w1b, b1, b1b, w2, w2b, b2, b2b, w3, w3b, b3, b3b, h1, h1b, \
      h2, h2b, o, ob, nh
void oracle_ex_mlp1d_b_f64(MLP1D_B_ARGS(double)) { ex_mlp1d_b(MLP1D_B_PASS); }
void oracle_ex_mlp1d_hv_f64(MLP1D_B_ARGS(double), double* lossd, const double* lossbd,
                            const double* xd, double* xbd, const double* yd, double* ybd,
                            const double* w1d, double* w1bd, const double* b1d, double* b1bd,
                            const double* w2d, double* w2bd, const double* b2d, double* b2bd,
                            const double* w3d, double* w3bd, const double* b3d, double* b3bd,
                            double* h1d, double* h1bd, double* h2d, double* h2bd, double* od,
                            double* obd) {
  ex_mlp1d_hv(MLP1D_B_PASS, lossd, lossbd, xd, xbd, yd, ybd, w1d, w1bd, b1d, b1bd, w2d, w2bd,
              b2d, b2bd, w3d, w3bd, b3d, b3bd, h1d, h1bd, h2d, h2bd, od, obd);
}


void oracle_affine_ls_b_f64(double* loss, const double* lossb, const double* w, double* wb,
                            const double* b, double* bb, const double* x, double* xb,
                            const double* t, double* tb, double* y, double* yb,
                            i64 n_s, i64 n_o, i64 n_i) {
  affine_ls_b<double>(loss, lossb, w, wb, b, bb, x, xb, t, tb, y, yb, n_s, n_o, n_i);
}
void oracle_affine_ls_b_f128(long double* loss, const long double* lossb, const long double* w,
                             long double* wb, const long double* b, long double* bb,
                             const long double* x, long double* xb, const long double* t,
                             long double* tb, long double* y, long double* yb,
                             i64 n_s, i64 n_o, i64 n_i) {
  affine_ls_b<long double>(loss, lossb, w, wb, b, bb, x, xb, t, tb, y, yb, n_s, n_o, n_i);
}

#define MLP_B_ARGS(T)                                                                      \
  T *loss, const T *lossb, const T *x, T *xb, const T *y, T *yb, const T *w1, T *w1b,     \
      const T *b1, T *b1b, const T *w2, T *w2b, const T *b2, T *b2b, T *h, T *hb, T *z,    \
      T *zb, T *p, T *pb, i64 n_s, i64 n_i, i64 n_h, i64 n_o
#define MLP_B_PASS loss, lossb, x, xb, y, yb, w1, w1b, b1, b1b, w2, w2b, b2, b2b, h, hb, z, zb, p, pb, n_s, n_i, n_h, n_o

void oracle_mlp2_ce_b_f32(MLP_B_ARGS(float)) { mlp2_ce_b<float>(MLP_B_PASS); }
void oracle_mlp2_ce_b_f64(MLP_B_ARGS(double)) { mlp2_ce_b<double>(MLP_B_PASS); }
void oracle_mlp2_ce_b_f128(MLP_B_ARGS(long double)) { mlp2_ce_b<long double>(MLP_B_PASS); }
void oracle_mlp2_ce_b_f32_omp(MLP_B_ARGS(float), int nthreads) {
  mlp2_ce_b_omp<float>(MLP_B_PASS, nthreads);
}
void oracle_mlp2_ce_b_f64_omp(MLP_B_ARGS(double), int nthreads) {
  mlp2_ce_b_omp<double>(MLP_B_PASS, nthreads);
}

#define MLP_HV_ARGS(T)                                                                     \
  MLP_B_ARGS(T), T *lossd, const T *lossbd, const T *xd, T *xbd, const T *yd, T *ybd,      \
      const T *w1d, T *w1bd, const T *b1d, T *b1bd, const T *w2d, T *w2bd, const T *b2d,   \
      T *b2bd, T *hd, T *hbd, T *zd, T *zbd, T *pd, T *pbd
#define MLP_HV_PASS                                                                        \
  MLP_B_PASS, lossd, lossbd, xd, xbd, yd, ybd, w1d, w1bd, b1d, b1bd, w2d, w2bd, b2d, b2bd, \
      hd, hbd, zd, zbd, pd, pbd

void oracle_mlp2_ce_hv_f64(MLP_HV_ARGS(double)) { mlp2_ce_hv<double>(MLP_HV_PASS); }
void oracle_mlp2_ce_hv_f128(MLP_HV_ARGS(long double)) { mlp2_ce_hv<long double>(MLP_HV_PASS); }
void oracle_mlp2_ce_hv_f64_omp(MLP_HV_ARGS(double), int nthreads) {
  mlp2_ce_hv_omp<double>(MLP_HV_PASS, nthreads);
}
void oracle_mlp2_ce_hv_f128_omp(MLP_HV_ARGS(long double), int nthreads) {
  mlp2_ce_hv_omp<long double>(MLP_HV_PASS, nthreads);
}

double oracle_heat2d_b_f64(double* loss, const double* lossb, double* u, double* ub, double* un,
                           double* unb, double alpha, double alphab, i64 n, i64 n_step,
                           double* u_stack) {
  return heat2d_b<double>(loss, lossb, u, ub, un, unb, alpha, alphab, n, n_step, u_stack);
}
long double oracle_heat2d_b_f128(long double* loss, const long double* lossb, long double* u,
                                 long double* ub, long double* un, long double* unb,
                                 long double alpha, long double alphab, i64 n, i64 n_step,
                                 long double* u_stack) {
  return heat2d_b<long double>(loss, lossb, u, ub, un, unb, alpha, alphab, n, n_step, u_stack);
}

void oracle_conv1d_relu_mse_b_f32(float* loss, const float* lossb, const float* x, float* xb,
                                  const float* w, float* wb, const float* t, float* tb,
                                  float* z, float* zb, float* r, float* rb,
                                  i64 n_b, i64 n_c, i64 n_l, i64 n_o, i64 n_k) {
  conv1d_relu_mse_b<float>(loss, lossb, x, xb, w, wb, t, tb, z, zb, r, rb, n_b, n_c, n_l, n_o, n_k);
}
void oracle_conv1d_relu_mse_b_f64(double* loss, const double* lossb, const double* x, double* xb,
                                  const double* w, double* wb, const double* t, double* tb,
                                  double* z, double* zb, double* r, double* rb,
                                  i64 n_b, i64 n_c, i64 n_l, i64 n_o, i64 n_k) {
  conv1d_relu_mse_b<double>(loss, lossb, x, xb, w, wb, t, tb, z, zb, r, rb, n_b, n_c, n_l, n_o, n_k);
}
void oracle_conv1d_relu_mse_b_f128(long double* loss, const long double* lossb,
                                   const long double* x, long double* xb, const long double* w,
                                   long double* wb, const long double* t, long double* tb,
                                   long double* z, long double* zb, long double* r,
                                   long double* rb, i64 n_b, i64 n_c, i64 n_l, i64 n_o, i64 n_k) {
  conv1d_relu_mse_b<long double>(loss, lossb, x, xb, w, wb, t, tb, z, zb, r, rb, n_b, n_c, n_l,
                                 n_o, n_k);
}

#define CONV_B_ARGS(T)                                                                     \
  T *loss, const T *lossb, const T *x, T *xb, const T *w, T *wb, const T *t, T *tb, T *z,   \
      T *zb, T *r, T *rb, i64 n_b, i64 n_c, i64 n_l, i64 n_o, i64 n_k
#define CONV_B_PASS loss, lossb, x, xb, w, wb, t, tb, z, zb, r, rb, n_b, n_c, n_l, n_o, n_k
double oracle_heat2d_b_f64_omp(double* loss, const double* lossb, double* u, double* ub,
                               double* un, double* unb, double alpha, double alphab, i64 n,
                               i64 n_step, double* u_stack, int nthreads) {
  return heat2d_b_omp<double>(loss, lossb, u, ub, un, unb, alpha, alphab, n, n_step, u_stack,
                              nthreads);
}
void oracle_conv1d_relu_mse_b_f32_omp(CONV_B_ARGS(float), int nthreads) {
  conv1d_relu_mse_b_omp<float>(CONV_B_PASS, nthreads);
}
void oracle_conv1d_relu_mse_b_f64_omp(CONV_B_ARGS(double), int nthreads) {
  conv1d_relu_mse_b_omp<double>(CONV_B_PASS, nthreads);
}

void oracle_affine_ls_d_f64(double* loss, double* lossd, const double* w, const double* wd,
                            const double* b, const double* bd, const double* x, const double* xd,
                            const double* t, const double* td, double* y, double* yd, i64 n_s,
                            i64 n_o, i64 n_i) {
  affine_ls_d<double>(loss, lossd, w, wd, b, bd, x, xd, t, td, y, yd, n_s, n_o, n_i);
}
void oracle_affine_ls_d_f128(long double* loss, long double* lossd, const long double* w,
                             const long double* wd, const long double* b, const long double* bd,
                             const long double* x, const long double* xd, const long double* t,
                             const long double* td, long double* y, long double* yd, i64 n_s,
                             i64 n_o, i64 n_i) {
  affine_ls_d<long double>(loss, lossd, w, wd, b, bd, x, xd, t, td, y, yd, n_s, n_o, n_i);
}

#define MLP_D_ARGS(T)                                                                      \
  T *loss, T *lossd, const T *x, const T *xd, const T *y, const T *yd, const T *w1,        \
      const T *w1d, const T *b1, const T *b1d, const T *w2, const T *w2d, const T *b2,     \
      const T *b2d, T *h, T *hd, T *z, T *zd, T *p, T *pd, i64 n_s, i64 n_i, i64 n_h, i64 n_o
#define MLP_D_PASS loss, lossd, x, xd, y, yd, w1, w1d, b1, b1d, w2, w2d, b2, b2d, h, hd, z, zd, p, pd, n_s, n_i, n_h, n_o
void oracle_mlp2_ce_d_f32(MLP_D_ARGS(float)) { mlp2_ce_d<float>(MLP_D_PASS); }
void oracle_mlp2_ce_d_f64(MLP_D_ARGS(double)) { mlp2_ce_d<double>(MLP_D_PASS); }
void oracle_mlp2_ce_d_f128(MLP_D_ARGS(long double)) { mlp2_ce_d<long double>(MLP_D_PASS); }

void oracle_heat2d_d_f64(double* loss, double* lossd, double* u, double* ud, double* un,
                         double* und, double alpha, double alphad, i64 n, i64 n_step) {
  heat2d_d<double>(loss, lossd, u, ud, un, und, alpha, alphad, n, n_step);
}
void oracle_heat2d_d_f128(long double* loss, long double* lossd, long double* u, long double* ud,
                          long double* un, long double* und, long double alpha,
                          long double alphad, i64 n, i64 n_step) {
  heat2d_d<long double>(loss, lossd, u, ud, un, und, alpha, alphad, n, n_step);
}

void oracle_conv1d_relu_mse_d_f32(float* loss, float* lossd, const float* x, const float* xd,
                                  const float* w, const float* wd, const float* t,
                                  const float* td, float* z, float* zd, float* r, float* rd,
                                  i64 n_b, i64 n_c, i64 n_l, i64 n_o, i64 n_k) {
  conv1d_relu_mse_d<float>(loss, lossd, x, xd, w, wd, t, td, z, zd, r, rd, n_b, n_c, n_l, n_o,
                           n_k);
}
void oracle_conv1d_relu_mse_d_f64(double* loss, double* lossd, const double* x, const double* xd,
                                  const double* w, const double* wd, const double* t,
                                  const double* td, double* z, double* zd, double* r, double* rd,
                                  i64 n_b, i64 n_c, i64 n_l, i64 n_o, i64 n_k) {
  conv1d_relu_mse_d<double>(loss, lossd, x, xd, w, wd, t, td, z, zd, r, rd, n_b, n_c, n_l, n_o,
                            n_k);
}
void oracle_conv1d_relu_mse_d_f128(long double* loss, long double* lossd, const long double* x,
                                   const long double* xd, const long double* w,
                                   const long double* wd, const long double* t,
                                   const long double* td, long double* z, long double* zd,
                                   long double* r, long double* rd, i64 n_b, i64 n_c, i64 n_l,
                                   i64 n_o, i64 n_k) {
  conv1d_relu_mse_d<long double>(loss, lossd, x, xd, w, wd, t, td, z, zd, r, rd, n_b, n_c, n_l,
                                 n_o, n_k);
}

}  // extern "C"
