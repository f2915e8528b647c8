"""The tangent (forward-mode) oracle `<k>_d` against the pinned adjoint
oracle: the dot-product identity lossd(v) = <grad, v> for a direction v over
every float input (the reference's dot-product check, rtol 1e-11,
src/STADE.jl:17108-17131), the primal values the two sweeps both compute
bit for bit, and lossd against a central finite difference."""
import numpy as np
import pytest

from oracle import oracle as orc
from stadeb200 import synth


def _rng(tag):
    return np.random.default_rng(int(synth.seed("tangent-tests", tag)) % (2 ** 63))


def _ip(a, b):
    return float(np.dot(a.astype(np.float64).ravel(), b.astype(np.float64).ravel()))


def test_affine_ls_d():
    n_s, n_o, n_i = 23, 7, 5
    d = synth.affine_ls_inputs(n_s, n_o, n_i)
    r = _rng("affine")
    v = {k: r.standard_normal(d[k].size) for k in ("w", "b", "x", "t")}
    z = lambda n: np.zeros(n)
    # adjoint
    g = dict(wb=z(n_o * n_i), bb=z(n_o), xb=z(n_s * n_i), tb=z(n_s * n_o))
    y_b, loss_b = z(n_s * n_o), z(1)
    orc.affine_ls_b(loss_b, d["lossb"], d["w"], g["wb"], d["b"], g["bb"], d["x"], g["xb"], d["t"],
                    g["tb"], y_b, z(n_s * n_o), n_s, n_o, n_i)
    # tangent
    loss, lossd, y, yd = z(1), z(1), z(n_s * n_o), z(n_s * n_o)
    orc.affine_ls_d(loss, lossd, d["w"], v["w"], d["b"], v["b"], d["x"], v["x"], d["t"], v["t"],
                    y, yd, n_s, n_o, n_i)
    assert np.array_equal(y, y_b) and loss[0] == loss_b[0]
    dot = sum(_ip(g[k + "b"], v[k]) for k in ("w", "b", "x", "t"))
    assert abs(lossd[0] - dot) <= 1e-11 * max(1.0, abs(dot))


@pytest.mark.parametrize("dtype,tol", [(np.float64, 1e-11)])
def test_mlp2_ce_d(dtype, tol):
    n_s, n_i, n_h, n_o = 13, 9, 11, 4
    d = synth.mlp2_ce_inputs(n_s, n_i, n_h, n_o, dtype=dtype)
    r = _rng("mlp")
    names = ("x", "y", "w1", "b1", "w2", "b2")
    v = {k: r.standard_normal(d[k].size).astype(dtype) for k in names}
    z = lambda n: np.zeros(n, dtype)
    S, I, H, O = n_s, n_i, n_h, n_o
    g = dict(xb=z(S * I), yb=z(S * O), w1b=z(I * H), b1b=z(H), w2b=z(H * O), b2b=z(O))
    hb_, zb_, pb_ = z(S * H), z(S * O), z(S * O)
    lb, hB, zB, pB = z(1), z(S * H), z(S * O), z(S * O)
    orc.mlp2_ce_b(lb, d["lossb"], d["x"], g["xb"], d["y"], g["yb"], d["w1"], g["w1b"], d["b1"],
                  g["b1b"], d["w2"], g["w2b"], d["b2"], g["b2b"], hB, hb_, zB, zb_, pB, pb_,
                  S, I, H, O)
    loss, lossd = z(1), z(1)
    h, hd, zz, zd, p, pd = z(S * H), z(S * H), z(S * O), z(S * O), z(S * O), z(S * O)
    orc.mlp2_ce_d(loss, lossd, d["x"], v["x"], d["y"], v["y"], d["w1"], v["w1"], d["b1"],
                  v["b1"], d["w2"], v["w2"], d["b2"], v["b2"], h, hd, zz, zd, p, pd, S, I, H, O)
    assert np.array_equal(h, hB) and np.array_equal(zz, zB) and np.array_equal(p, pB)
    dot = sum(_ip(g[k + "b"], v[k]) for k in names)
    assert abs(lossd[0] - dot) <= tol * max(1.0, abs(dot))


def test_heat2d_d():
    n, n_step, alpha = 10, 3, 0.2
    u0 = synth.heat2d_inputs(n)["u"]
    r = _rng("heat")
    v_u, v_a = r.standard_normal(n * n), 0.7
    z = lambda m: np.zeros(m)
    u, ub, un, unb, stack, lb = u0.copy(), z(n * n), z(n * n), z(n * n), z(n_step * n * n), z(1)
    ab = orc.heat2d_b(lb, np.ones(1), u, ub, un, unb, alpha, 0.0, n, n_step, stack)
    ut, ud, unt, und, loss, lossd = u0.copy(), v_u.copy(), z(n * n), z(n * n), z(1), z(1)
    orc.heat2d_d(loss, lossd, ut, ud, unt, und, alpha, v_a, n, n_step)
    assert loss[0] == lb[0]
    dot = _ip(ub, v_u) + ab * v_a
    assert abs(lossd[0] - dot) <= 1e-11 * max(1.0, abs(dot))
    # central difference of the loss along the direction
    def L(eps):
        uu, l1 = u0 + eps * v_u, z(1)
        orc.heat2d_d(l1, z(1), uu, z(n * n), z(n * n), z(n * n), alpha + eps * v_a, 0.0, n, n_step)
        return l1[0]
    h = 1e-6
    fd = (L(h) - L(-h)) / (2 * h)
    assert abs(fd - lossd[0]) <= 1e-6 * max(1.0, abs(lossd[0]))


def test_conv1d_relu_mse_d():
    n_b, n_c, n_l, n_o, n_k = 2, 3, 17, 4, 5
    d = synth.conv1d_relu_mse_inputs(n_b, n_c, n_l, n_o, n_k)
    d = {k: v.astype(np.float64) for k, v in d.items()}
    r = _rng("conv")
    v = {k: r.standard_normal(d[k].size) for k in ("x", "w", "t")}
    n_lo = n_l - n_k + 1
    nt = n_b * n_o * n_lo
    z = lambda m: np.zeros(m)
    g = dict(xb=z(n_b * n_c * n_l), wb=z(n_o * n_c * n_k), tb=z(nt))
    zB, rB, lb = z(nt), z(nt), z(1)
    orc.conv1d_relu_mse_b(lb, d["lossb"], d["x"], g["xb"], d["w"], g["wb"], d["t"], g["tb"], zB,
                          z(nt), rB, z(nt), n_b, n_c, n_l, n_o, n_k)
    loss, lossd, zz, zd, rr, rd = z(1), z(1), z(nt), z(nt), z(nt), z(nt)
    orc.conv1d_relu_mse_d(loss, lossd, d["x"], v["x"], d["w"], v["w"], d["t"], v["t"], zz, zd, rr,
                          rd, n_b, n_c, n_l, n_o, n_k)
    assert np.array_equal(zz, zB) and np.array_equal(rr, rB)
    dot = sum(_ip(g[k + "b"], v[k]) for k in ("x", "w", "t"))
    assert abs(lossd[0] - dot) <= 1e-11 * max(1.0, abs(dot))
