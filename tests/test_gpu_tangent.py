"""Tangent sweeps `<k>_d` on the GPU, and the full-size dot-product identity.

1. Parity: each tangent sweep through the C ABI against the tangent oracle
   (tests/test_tangent_oracle.py pins that oracle to the adjoint oracle) at
   small sizes; Float64 1e-12, Float32 1e-5 normwise.
2. At the BASELINE configurations' full sizes the size-independent identity
   lossd(v) = <grad, v> (the reference's dot-product check,
   src/STADE.jl:17108-17131) ties the GPU adjoint to the GPU tangent, two
   independent code paths: Float64 sweeps with a random direction (rtol
   1e-10); Float32 sweeps with the direction v = grad, which keeps the sum free
   of cancellation, so the identity holds to the Float32 adjoint's own
   accuracy (rtol 1e-5 against a Float64 tangent where one exists, 1e-4 for
   C4, whose only tangent is Float32 and sums 1e9 terms in Float32 partials).
   For the HVP (C5): lossd = <grad, v> from the same call, and the symmetry
   <v2, H v1> = <v1, H v2>.
"""
import numpy as np
import pytest
import torch

import cases
from oracle import oracle as orc
from refmath import rel_err
from stadeb200 import kernels, synth

pytestmark = pytest.mark.gpu


def _rng(tag):
    return np.random.default_rng(int(synth.seed("gpu-tangent", tag)) % (2 ** 63))


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _z(n, dt=torch.float64):
    return torch.zeros(n, dtype=dt, device="cuda")


def _dot(a, b):
    return float(torch.dot(a.double().ravel(), b.double().ravel()))


# ---- 1. parity against the tangent oracle -------------------------------------
@pytest.mark.parametrize("n_s,n_o,n_i", [(37, 9, 5), (1024, 64, 32), (3, 1, 70)])
def test_affine_ls_d_parity(n_s, n_o, n_i):
    d = synth.affine_ls_inputs(n_s, n_o, n_i)
    r = _rng(f"aff{n_s}")
    v = {k: r.standard_normal(d[k].size) for k in ("w", "b", "x", "t")}
    ref = dict(loss=np.full(1, 0.25), lossd=np.full(1, -0.5), y=np.zeros(n_s * n_o),
               yd=np.zeros(n_s * n_o))
    orc.affine_ls_d(ref["loss"], ref["lossd"], d["w"], v["w"], d["b"], v["b"], d["x"], v["x"],
                    d["t"], v["t"], ref["y"], ref["yd"], n_s, n_o, n_i)
    g = dict(loss=_dev(np.full(1, 0.25)), lossd=_dev(np.full(1, -0.5)), y=_z(n_s * n_o),
             yd=_z(n_s * n_o))
    kernels.affine_ls_d_cuda(g["loss"], g["lossd"], _dev(d["w"]), _dev(v["w"]), _dev(d["b"]),
                             _dev(v["b"]), _dev(d["x"]), _dev(v["x"]), _dev(d["t"]), _dev(v["t"]),
                             g["y"], g["yd"], n_s, n_o, n_i)
    for k in ("y", "yd"):
        assert np.array_equal(g[k].cpu().numpy(), ref[k]), k   # same statement order
    for k in ("loss", "lossd"):
        assert rel_err(g[k].cpu().numpy(), ref[k]) <= 1e-12, k


def _mlp_d_state(S, I, H, O, dtype):
    d = synth.mlp2_ce_inputs(S, I, H, O, dtype=dtype)
    r = _rng(f"mlp{S}{I}{H}{O}")
    st = {}
    for k in ("x", "y", "w1", "b1", "w2", "b2"):
        st[k] = d[k]
        st[k + "d"] = r.standard_normal(d[k].size).astype(dtype)
    for k in ("h", "hd"):
        st[k] = np.zeros(S * H, dtype)
    for k in ("z", "zd", "p", "pd"):
        st[k] = np.zeros(S * O, dtype)
    st["loss"] = np.full(1, 0.5, dtype)
    st["lossd"] = np.full(1, 0.25, dtype)
    return st


@pytest.mark.parametrize("sizes", [(64, 30, 40, 10), (33, 17, 19, 3), (130, 70, 129, 32),
                                   (300, 784, 512, 10)])
@pytest.mark.parametrize("dtype", [np.float64, np.float32])
def test_mlp2_ce_d_parity(sizes, dtype):
    S, I, H, O = sizes
    st = _mlp_d_state(S, I, H, O, dtype)
    ref = {k: v.copy() for k, v in st.items()}
    orc.mlp2_ce_d(*[ref[k] for k in kernels.MLP_D_ARGS], S, I, H, O)
    truth = {k: v.astype(np.float64) for k, v in st.items()}
    orc.mlp2_ce_d(*[truth[k] for k in kernels.MLP_D_ARGS], S, I, H, O)
    dev = {k: _dev(v) for k, v in st.items()}
    kernels.mlp2_ce_d_cuda(*[dev[k] for k in kernels.MLP_D_ARGS], S, I, H, O)
    for k in ("h", "hd", "z", "zd", "p", "pd", "loss", "lossd"):
        out = dev[k].cpu().numpy()
        if dtype == np.float64:
            assert rel_err(out, ref[k]) <= 1e-12, (k, rel_err(out, ref[k]))
        else:
            e = rel_err(out, truth[k])
            assert e <= max(1e-5, rel_err(ref[k], truth[k])), (k, e)


@pytest.mark.parametrize("n,n_step", [(34, 3), (64, 4), (7, 2), (10, 0), (258, 5), (1, 3),
                                      (2, 2)])
def test_heat2d_d_parity(n, n_step):
    u0 = synth.heat2d_inputs(n)["u"]
    r = _rng(f"heat{n}")
    v = r.standard_normal(n * n)
    ref = dict(loss=np.full(1, 1.5), lossd=np.full(1, 0.5), u=u0.copy(), ud=v.copy(),
               un=np.zeros(n * n), und=np.zeros(n * n))
    orc.heat2d_d(ref["loss"], ref["lossd"], ref["u"], ref["ud"], ref["un"], ref["und"], 0.2, 0.7,
                 n, n_step)
    g = {k: _dev(v) for k, v in dict(loss=np.full(1, 1.5), lossd=np.full(1, 0.5), u=u0.copy(),
                                     ud=v.copy(), un=np.zeros(n * n), und=np.zeros(n * n)).items()}
    kernels.heat2d_d_cuda(g["loss"], g["lossd"], g["u"], g["ud"], g["un"], g["und"], 0.2, 0.7, n,
                          n_step)
    for k in ("u", "un", "ud", "und"):
        if n_step > 0:
            assert np.array_equal(g[k].cpu().numpy(), ref[k]), k   # same expression order
    for k in ("loss", "lossd"):
        assert rel_err(g[k].cpu().numpy(), ref[k]) <= 1e-12, k


@pytest.mark.parametrize("sizes", [(2, 3, 30, 4, 5), (4, 16, 200, 32, 9), (1, 1, 9, 1, 9)])
def test_conv1d_relu_mse_d_parity(sizes):
    n_b, n_c, n_l, n_o, n_k = sizes
    d = synth.conv1d_relu_mse_inputs(*sizes)
    r = _rng(f"conv{sizes}")
    n_lo = n_l - n_k + 1
    nt = n_b * n_o * n_lo
    st = dict(loss=np.full(1, 0.5, np.float32), lossd=np.full(1, 0.125, np.float32))
    for k in ("x", "w", "t"):
        st[k] = d[k]
        st[k + "d"] = (0.02 * r.standard_normal(d[k].size)).astype(np.float32)
    for k in ("z", "zd", "r", "rd"):
        st[k] = np.zeros(nt, np.float32)
    order = ("loss", "lossd", "x", "xd", "w", "wd", "t", "td", "z", "zd", "r", "rd")
    ref = {k: v.copy() for k, v in st.items()}
    orc.conv1d_relu_mse_d(*[ref[k] for k in order], *sizes)
    truth = {k: v.astype(np.float64) for k, v in st.items()}
    orc.conv1d_relu_mse_d(*[truth[k] for k in order], *sizes)
    dev = {k: _dev(v) for k, v in st.items()}
    kernels.conv1d_relu_mse_d_cuda(*[dev[k] for k in order], *sizes)
    for k in ("z", "zd", "r", "rd", "loss", "lossd"):
        out = dev[k].cpu().numpy()
        e = rel_err(out, truth[k])
        assert e <= max(1e-5, rel_err(ref[k], truth[k])), (k, e)


# ---- 2. full-size dot-product identity -----------------------------------------
def test_full_c1_dot_product():
    n_s, n_o, n_i = synth.FULL["affine_ls"].values()
    d = {k: _dev(v) for k, v in synth.affine_ls_inputs(n_s, n_o, n_i).items()}
    g = dict(wb=_z(n_o * n_i), bb=_z(n_o), xb=_z(n_s * n_i), tb=_z(n_s * n_o))
    kernels.affine_ls_b_cuda(_z(1), d["lossb"], d["w"], g["wb"], d["b"], g["bb"], d["x"], g["xb"],
                             d["t"], g["tb"], _z(n_s * n_o), _z(n_s * n_o), n_s, n_o, n_i)
    r = _rng("c1full")
    v = {k: _dev(r.standard_normal(d[k].numel())) for k in ("w", "b", "x", "t")}
    lossd = _z(1)
    kernels.affine_ls_d_cuda(_z(1), lossd, d["w"], v["w"], d["b"], v["b"], d["x"], v["x"], d["t"],
                             v["t"], _z(n_s * n_o), _z(n_s * n_o), n_s, n_o, n_i)
    dot = sum(_dot(g[k + "b"], v[k]) for k in ("w", "b", "x", "t"))
    assert abs(float(lossd) - dot) <= 1e-10 * abs(dot)


def test_full_c2_dot_product():
    c = synth.FULL["mlp2_ce"]
    S, I, H, O = c["n_s"], c["n_i"], c["n_h"], c["n_o"]
    d32 = synth.mlp2_ce_inputs(S, I, H, O)
    d = {k: _dev(v) for k, v in d32.items()}
    f = torch.float32
    g = dict(xb=_z(S * I, f), yb=_z(S * O, f), w1b=_z(I * H, f), b1b=_z(H, f), w2b=_z(H * O, f),
             b2b=_z(O, f))
    kernels.mlp2_ce_b_cuda(_z(1, f), d["lossb"], d["x"], g["xb"], d["y"], g["yb"], d["w1"],
                           g["w1b"], d["b1"], g["b1b"], d["w2"], g["w2b"], d["b2"], g["b2b"],
                           _z(S * H, f), _z(S * H, f), _z(S * O, f), _z(S * O, f), _z(S * O, f),
                           _z(S * O, f), S, I, H, O)
    # direction v = the adjoint's own gradient; the tangent in Float64 on the same inputs
    names = ("x", "y", "w1", "b1", "w2", "b2")
    d64 = {k: d[k].double() for k in names}
    v = {k: g[k + "b"].double() for k in names}
    lossd = _z(1)
    kernels.mlp2_ce_d_cuda(_z(1), lossd, d64["x"], v["x"], d64["y"], v["y"], d64["w1"], v["w1"],
                           d64["b1"], v["b1"], d64["w2"], v["w2"], d64["b2"], v["b2"], _z(S * H),
                           _z(S * H), _z(S * O), _z(S * O), _z(S * O), _z(S * O), S, I, H, O)
    dot = sum(_dot(g[k + "b"], v[k]) for k in names)
    assert abs(float(lossd) - dot) <= 1e-5 * abs(dot), (float(lossd), dot)


def test_full_c3_dot_product():
    c = synth.FULL["heat2d"]
    n, ns, alpha = c["n"], c["n_step"], c["alpha"]
    u0 = _dev(synth.heat2d_inputs(n)["u"])
    stack = kernels.initstacks_heat2d_b_cuda(n, ns)
    ub, ab = _z(n * n), _z(1)
    kernels.heat2d_b_cuda_device(_z(1), _dev(np.ones(1)), u0, ub, _z(n * n), _z(n * n), alpha, ab,
                                 n, ns, stack)
    del stack
    torch.cuda.empty_cache()
    r = _rng("c3full")
    v_u = torch.randn(n * n, dtype=torch.float64, device="cuda",
                      generator=torch.Generator(device="cuda").manual_seed(5))
    v_a = float(r.standard_normal())
    lossd = _z(1)
    kernels.heat2d_d_cuda(_z(1), lossd, u0.clone(), v_u.clone(), _z(n * n), _z(n * n), alpha, v_a,
                          n, ns)
    dot = _dot(ub, v_u) + float(ab) * v_a
    assert abs(float(lossd) - dot) <= 1e-10 * abs(dot), (float(lossd), dot)


def test_full_c4_dot_product():
    c = synth.FULL["conv1d_relu_mse"]
    sizes = (c["n_b"], c["n_c"], c["n_l"], c["n_o"], c["n_k"])
    n_b, n_c, n_l, n_o, n_k = sizes
    n_lo = n_l - n_k + 1
    nt = n_b * n_o * n_lo
    d = {k: _dev(v) for k, v in synth.conv1d_relu_mse_inputs(*sizes).items()}
    f = torch.float32
    g = dict(xb=_z(n_b * n_c * n_l, f), wb=_z(n_o * n_c * n_k, f), tb=_z(nt, f))
    kernels.conv1d_relu_mse_b_cuda(_z(1, f), d["lossb"], d["x"], g["xb"], d["w"], g["wb"], d["t"],
                                   g["tb"], _z(nt, f), _z(nt, f), _z(nt, f), _z(nt, f), *sizes)
    torch.cuda.empty_cache()
    lossd = _z(1, f)
    kernels.conv1d_relu_mse_d_cuda(_z(1, f), lossd, d["x"], g["xb"], d["w"], g["wb"], d["t"],
                                   g["tb"], _z(nt, f), _z(nt, f), _z(nt, f), _z(nt, f), *sizes)
    dot = sum(_dot(g[k + "b"], g[k + "b"]) for k in ("x", "w", "t"))
    assert abs(float(lossd) - dot) <= 1e-4 * abs(dot), (float(lossd), dot)


def _hv_call(S, I, H, O, base, direction):
    t = {}
    for name in kernels.MLP_HV_ARGS + kernels.MLP_HV_TAN:
        if name in base:
            t[name] = base[name]
        elif name in direction:
            t[name] = direction[name]
        else:
            t[name] = _z(kernels._mlp_len(name, S, I, H, O))
    kernels.mlp2_ce_hv_cuda(*[t[a] for a in kernels.MLP_HV_ARGS], S, I, H, O,
                            *[t[a] for a in kernels.MLP_HV_TAN])
    return t


def test_full_c5_hvp_identities():
    c = synth.FULL["mlp2_ce_hv"]
    S, I, H, O = c["n_s"], c["n_i"], c["n_h"], c["n_o"]
    d = synth.mlp2_ce_hv_inputs(S, I, H, O)
    base = {k: _dev(d[k]) for k in ("x", "y", "w1", "b1", "w2", "b2", "lossb")}
    base.update(xd=_dev(d["xd"]), yd=_dev(d["yd"]), lossbd=_dev(d["lossbd"]))
    v1 = {k: _dev(d[k]) for k in ("w1d", "b1d", "w2d", "b2d")}
    r = _rng("c5full")
    v2 = {k: _dev(r.standard_normal(d[k].size)) for k in ("w1d", "b1d", "w2d", "b2d")}
    t1 = _hv_call(S, I, H, O, base, v1)
    t2 = _hv_call(S, I, H, O, base, v2)
    ps = ("w1", "b1", "w2", "b2")
    # lossd = <grad, v> within the same call
    for t, v in ((t1, v1), (t2, v2)):
        dot = sum(_dot(t[p + "b"], v[p + "d"]) for p in ps)
        assert abs(float(t["lossd"]) - dot) <= 1e-10 * abs(dot)
    # symmetry of the Hessian: <v2, H v1> = <v1, H v2>
    a = sum(_dot(t1[p + "bd"], v2[p + "d"]) for p in ps)
    b = sum(_dot(t2[p + "bd"], v1[p + "d"]) for p in ps)
    assert abs(a - b) <= 1e-9 * max(abs(a), abs(b)), (a, b)
