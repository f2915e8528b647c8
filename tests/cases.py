"""Argument sets of the five sweeps, in the generated argument order, and
runners for the oracle (CPU) and for libstade_b200 (GPU, through the C ABI).

A state is an ordered dict name -> numpy array (plus the integer sizes). With
`seeded=True` every adjoint array starts non-zero, which exercises the
generated semantics: outputs are accumulated (`wb += ...`) and consumed
intermediates act as seeds (`__oldb = hb; hb = 0`).
"""
from collections import OrderedDict

import numpy as np

from stadeb200 import synth

AFFINE_ARGS = ["loss", "lossb", "w", "wb", "b", "bb", "x", "xb", "t", "tb", "y", "yb"]
MLP_ARGS = ["loss", "lossb", "x", "xb", "y", "yb", "w1", "w1b", "b1", "b1b", "w2", "w2b",
            "b2", "b2b", "h", "hb", "z", "zb", "p", "pb"]
MLP_TAN = ["lossd", "lossbd", "xd", "xbd", "yd", "ybd", "w1d", "w1bd", "b1d", "b1bd",
           "w2d", "w2bd", "b2d", "b2bd", "hd", "hbd", "zd", "zbd", "pd", "pbd"]
HEAT_ARGS = ["loss", "lossb", "u", "ub", "un", "unb"]
CONV_ARGS = ["loss", "lossb", "x", "xb", "w", "wb", "t", "tb", "z", "zb", "r", "rb"]


def _rng(tag):
    return np.random.default_rng(int(synth.seed("tests", tag)) % (2 ** 63))


def affine_state(n_s, n_o, n_i, seeded=False):
    d = synth.affine_ls_inputs(n_s, n_o, n_i)
    f = np.float64
    st = OrderedDict()
    rng = _rng(f"affine{n_s}{n_o}{n_i}")
    shapes = dict(loss=1, w=n_o * n_i, b=n_o, x=n_s * n_i, t=n_s * n_o, y=n_s * n_o)
    for a in AFFINE_ARGS:
        base = a[:-1] if a.endswith("b") and a not in ("b",) and a[:-1] in shapes else a
        if a in d:
            st[a] = d[a].copy()
        elif a == "loss":
            st[a] = np.full(1, 0.25 if seeded else 0.0, f)
        else:
            n = shapes[base]
            st[a] = rng.standard_normal(n) if seeded else np.zeros(n, f)
    st["y"] = np.zeros(n_s * n_o, f)
    return st, dict(n_s=n_s, n_o=n_o, n_i=n_i)


def mlp_state(n_s, n_i, n_h, n_o, dtype=np.float32, seeded=False):
    d = synth.mlp2_ce_inputs(n_s, n_i, n_h, n_o, dtype)
    shapes = dict(loss=1, x=n_s * n_i, y=n_s * n_o, w1=n_i * n_h, b1=n_h, w2=n_h * n_o, b2=n_o,
                  h=n_s * n_h, z=n_s * n_o, p=n_s * n_o)
    rng = _rng(f"mlp{n_s}{n_i}{n_h}{n_o}")
    st = OrderedDict()
    for a in MLP_ARGS:
        base = a if a in shapes or a == "lossb" else a[:-1]
        if a in d:
            st[a] = d[a].copy()
        elif a == "loss":
            st[a] = np.full(1, 0.5 if seeded else 0.0, dtype)
        elif a in ("h", "z", "p"):
            st[a] = np.zeros(shapes[a], dtype)
        else:
            n = shapes[base]
            st[a] = (0.01 * rng.standard_normal(n)).astype(dtype) if seeded else np.zeros(n, dtype)
    return st, dict(n_s=n_s, n_i=n_i, n_h=n_h, n_o=n_o)


def mlp_hv_state(n_s, n_i, n_h, n_o, seeded=False, xd_nonzero=False):
    f = np.float64
    d = synth.mlp2_ce_hv_inputs(n_s, n_i, n_h, n_o)
    st, ints = mlp_state(n_s, n_i, n_h, n_o, f, seeded)
    for a in ("x", "y", "w1", "b1", "w2", "b2", "lossb"):
        st[a] = d[a].copy()
    shapes = dict(loss=1, x=n_s * n_i, y=n_s * n_o, w1=n_i * n_h, b1=n_h, w2=n_h * n_o, b2=n_o,
                  h=n_s * n_h, z=n_s * n_o, p=n_s * n_o)
    rng = _rng(f"mlphv{n_s}{n_i}{n_h}{n_o}")
    for a in MLP_TAN:
        base = a[:-1] if not a.endswith("bd") else a[:-2]
        if a in d:
            st[a] = d[a].copy()
        elif a in ("hd", "zd", "pd"):
            st[a] = np.zeros(shapes[base], f)
        elif a == "lossd":
            st[a] = np.full(1, 0.125 if seeded else 0.0, f)
        else:
            n = shapes[base]
            st[a] = 0.01 * rng.standard_normal(n) if seeded else np.zeros(n, f)
    if xd_nonzero:
        st["xd"] = 0.1 * rng.standard_normal(n_s * n_i)
        st["yd"] = 0.1 * rng.standard_normal(n_s * n_o)
        st["lossbd"] = np.full(1, 0.3, f)
    return st, ints


def heat_state(n, n_step, alpha=0.2, seeded=False):
    f = np.float64
    d = synth.heat2d_inputs(n)
    rng = _rng(f"heat{n}{n_step}")
    st = OrderedDict()
    st["loss"] = np.full(1, 1.5 if seeded else 0.0, f)
    st["lossb"] = d["lossb"].copy()
    st["u"] = d["u"].copy()
    st["ub"] = rng.standard_normal(n * n) * 0.1 if seeded else np.zeros(n * n, f)
    st["un"] = np.zeros(n * n, f)
    st["unb"] = rng.standard_normal(n * n) * 0.1 if seeded else np.zeros(n * n, f)
    st["u_stack"] = np.zeros(max(n_step * n * n, 1), f)
    return st, dict(n=n, n_step=n_step, alpha=alpha, alphab=0.75 if seeded else 0.0)


def conv_state(n_b, n_c, n_l, n_o, n_k, dtype=np.float32, seeded=False):
    d = synth.conv1d_relu_mse_inputs(n_b, n_c, n_l, n_o, n_k)
    n_lo = n_l - n_k + 1
    shapes = dict(loss=1, x=n_b * n_c * n_l, w=n_o * n_c * n_k, t=n_b * n_o * n_lo,
                  z=n_b * n_o * n_lo, r=n_b * n_o * n_lo)
    rng = _rng(f"conv{n_b}{n_c}{n_l}{n_o}{n_k}")
    st = OrderedDict()
    for a in CONV_ARGS:
        base = a if a in shapes or a == "lossb" else a[:-1]
        if a in d:
            st[a] = d[a].astype(dtype)
        elif a == "loss":
            st[a] = np.full(1, 0.5 if seeded else 0.0, dtype)
        elif a in ("z", "r"):
            st[a] = np.zeros(shapes[a], dtype)
        else:
            n = shapes[base]
            st[a] = (0.001 * rng.standard_normal(n)).astype(dtype) if seeded else np.zeros(n, dtype)
    return st, dict(n_b=n_b, n_c=n_c, n_l=n_l, n_o=n_o, n_k=n_k)


def copy_state(st):
    return OrderedDict((k, v.copy()) for k, v in st.items())


# ---- runners ---------------------------------------------------------------------
def oracle_affine(st, ints):
    from oracle import oracle as orc
    orc.affine_ls_b(*[st[a] for a in AFFINE_ARGS], ints["n_s"], ints["n_o"], ints["n_i"])


def oracle_mlp(st, ints):
    from oracle import oracle as orc
    orc.mlp2_ce_b(*[st[a] for a in MLP_ARGS], ints["n_s"], ints["n_i"], ints["n_h"], ints["n_o"])


def oracle_mlp_hv(st, ints, truth=False):
    from oracle import oracle as orc
    orc.mlp2_ce_hv(*[st[a] for a in MLP_ARGS], ints["n_s"], ints["n_i"], ints["n_h"], ints["n_o"],
                   *[st[a] for a in MLP_TAN], truth=truth)


def oracle_heat(st, ints):
    from oracle import oracle as orc
    return orc.heat2d_b(*[st[a] for a in HEAT_ARGS], ints["alpha"], ints["alphab"], ints["n"],
                        ints["n_step"], st["u_stack"])


def oracle_conv(st, ints):
    from oracle import oracle as orc
    orc.conv1d_relu_mse_b(*[st[a] for a in CONV_ARGS], ints["n_b"], ints["n_c"], ints["n_l"],
                          ints["n_o"], ints["n_k"])


def _to_dev(st):
    import torch
    return OrderedDict((k, torch.from_numpy(v).cuda()) for k, v in st.items())


def _back(dev, st):
    for k, v in dev.items():
        st[k] = v.cpu().numpy()


def gpu_affine(st, ints):
    import stadeb200
    dev = _to_dev(st)
    stadeb200.affine_ls_b_cuda(*[dev[a] for a in AFFINE_ARGS], ints["n_s"], ints["n_o"], ints["n_i"])
    _back(dev, st)


def gpu_mlp(st, ints):
    import stadeb200
    dev = _to_dev(st)
    stadeb200.mlp2_ce_b_cuda(*[dev[a] for a in MLP_ARGS], ints["n_s"], ints["n_i"], ints["n_h"],
                             ints["n_o"])
    _back(dev, st)


def gpu_mlp_hv(st, ints):
    import stadeb200
    dev = _to_dev(st)
    stadeb200.mlp2_ce_hv_cuda(*[dev[a] for a in MLP_ARGS], ints["n_s"], ints["n_i"], ints["n_h"],
                              ints["n_o"], *[dev[a] for a in MLP_TAN])
    _back(dev, st)


def gpu_heat(st, ints):
    import stadeb200
    dev = _to_dev(st)
    ab = stadeb200.heat2d_b_cuda(*[dev[a] for a in HEAT_ARGS], ints["alpha"], ints["alphab"],
                                 ints["n"], ints["n_step"], dev["u_stack"])
    _back(dev, st)
    return ab


def gpu_conv(st, ints):
    import stadeb200
    dev = _to_dev(st)
    stadeb200.conv1d_relu_mse_b_cuda(*[dev[a] for a in CONV_ARGS], ints["n_b"], ints["n_c"],
                                     ints["n_l"], ints["n_o"], ints["n_k"])
    _back(dev, st)


def conv_kink_adjust(st0, truth, out, ints, band=1e-5):
    """The exact adjoint of the ReLU branch the GPU took, where it took the
    other one at a kink. max(z, 0)' = 0.5 (1 + sign z) jumps at z = 0; where
    the exact pre-activation |z| is within `band` * max|z| (the contraction's
    Float32 rounding) and the GPU's z has the other sign, the GPU's g = dz
    differs from the exact one by (d_gpu - d_exact) * rb_total. Returns a copy
    of `truth` with wb and xb moved by exactly that, and the number of such
    elements. Everything else (z, r, tb, loss) is continuous at the kink."""
    n_b, n_c, n_l, n_o, n_k = (ints[k] for k in ("n_b", "n_c", "n_l", "n_o", "n_k"))
    n_lo = n_l - n_k + 1
    zt = truth["z"].reshape(n_b, n_o, n_lo)
    zg = out["z"].astype(np.float64).reshape(n_b, n_o, n_lo)
    flip = (np.sign(zt) != np.sign(zg)) & (np.abs(zt) <= band * np.abs(zt).max())
    adj = OrderedDict((k, v.copy()) for k, v in truth.items())
    idx = np.argwhere(flip)
    if len(idx) == 0:
        return adj, 0
    inv_n = 1.0 / (n_b * n_o * n_lo)
    tt = st0["t"].astype(np.float64).reshape(n_b, n_o, n_lo)
    rb0 = st0["rb"].astype(np.float64).reshape(n_b, n_o, n_lo)
    lb = float(st0["lossb"][0])
    x = st0["x"].astype(np.float64).reshape(n_b, n_c, n_l)
    w = st0["w"].astype(np.float64).reshape(n_o, n_c, n_k)
    wb = adj["wb"].reshape(n_o, n_c, n_k)
    xb = adj["xb"].reshape(n_b, n_c, n_l)
    for b, o, t in idx:
        rt = max(zt[b, o, t], 0.0)
        rbt = rb0[b, o, t] + inv_n * 2.0 * (rt - tt[b, o, t]) * lb
        dg = (0.5 * (1.0 + np.sign(zg[b, o, t])) - 0.5 * (1.0 + np.sign(zt[b, o, t]))) * rbt
        wb[o, :, :] += dg * np.stack([x[b, :, t + k] for k in range(n_k)], axis=1)
        for k in range(n_k):
            xb[b, :, t + k] += dg * w[o, :, k]
    return adj, len(idx)
