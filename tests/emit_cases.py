"""Inputs for the .cu emitter's corpus (tests/emit_corpus/*.jl): per sweep,
the generated positional arguments (without the stacks) for a size, seeded."""
from collections import OrderedDict

import numpy as np

CORPUS = "emit_corpus"


def _rng(tag):
    import zlib
    return np.random.default_rng(zlib.crc32(tag.encode()))


def _n(r, n, scale=1.0):
    return scale * r.standard_normal(n)


def affine(size, r):
    n_s, n_o, n_i = size
    a = OrderedDict()
    a["loss"], a["lossb"] = np.full(1, 0.25), np.full(1, 1.5)
    for k, n in (("w", n_o * n_i), ("b", n_o), ("x", n_s * n_i), ("t", n_s * n_o),
                 ("y", n_s * n_o)):
        a[k] = _n(r, n)
        a[k + "b"] = _n(r, n, 0.1)
    a["n_s"], a["n_o"], a["n_i"] = n_s, n_o, n_i
    return a


def heat(size, r):
    n, n_step = size
    a = OrderedDict()
    a["loss"], a["lossb"] = np.full(1, 1.5), np.full(1, 0.5)
    a["u"], a["ub"] = _n(r, n * n), _n(r, n * n, 0.1)
    a["un"], a["unb"] = _n(r, n * n), _n(r, n * n, 0.1)
    a["alpha"], a["alphab"] = 0.2, 0.75
    a["n"], a["n_step"] = n, n_step
    return a


def decay(size, r):
    n, nstep = size
    a = OrderedDict()
    a["u"], a["ub"] = _n(r, n), _n(r, n)
    a["k"], a["kb"] = 0.7, 0.3
    a["dt"], a["dtb"] = 0.05, -0.2
    a["i_n"], a["i_nstep"] = n, nstep
    return a


def edge_relu(size, r):
    nn, ne = size
    a = OrderedDict()
    a["loss"], a["lossb"] = np.full(1, 0.5), np.full(1, 1.25)
    a["x"], a["xb"] = _n(r, nn), _n(r, nn, 0.1)
    a["w"], a["wb"] = _n(r, ne), _n(r, ne, 0.1)
    e2n = r.integers(1, nn + 1, size=(ne, 2)).astype(np.int64)   # column-major 2 x ne
    a["i_e2n"] = np.ascontiguousarray(e2n.reshape(-1))
    a["i_ne"] = ne
    return a


def bilin(size, r):
    m, n = size
    a = OrderedDict()
    a["loss"], a["lossb"] = np.full(1, 0.0), np.full(1, 0.75)
    a["a"], a["ab"] = _n(r, m * n), _n(r, m * n, 0.1)
    a["x"], a["xb"] = _n(r, m), _n(r, m, 0.1)
    a["z"], a["zb"] = _n(r, n), _n(r, n, 0.1)
    a["i_m"], a["i_n"] = m, n
    return a


def cumsum_sq(size, r):
    (n,) = size
    a = OrderedDict()
    a["loss"], a["lossb"] = np.full(1, 0.0), np.full(1, 1.0)
    a["x"], a["xb"] = _n(r, n), _n(r, n, 0.1)
    a["c"], a["cb"] = _n(r, n), _n(r, n, 0.1)
    a["i_n"] = n
    return a


def window(size, r):
    n, k = size
    a = OrderedDict()
    a["loss"], a["lossb"] = np.full(1, 0.0), np.full(1, 0.5)
    a["x"], a["xb"] = _n(r, n + k - 1), _n(r, n + k - 1, 0.1)
    a["w"], a["wb"] = _n(r, k, 0.5), _n(r, k, 0.1)
    a["z"], a["zb"] = _n(r, n), _n(r, n, 0.1)
    a["i_n"], a["i_k"] = n, k
    return a


def smooth(size, r):
    (n,) = size
    a = OrderedDict()
    a["loss"], a["lossb"] = np.full(1, 0.0), np.full(1, 0.75)
    a["u"], a["ub"] = _n(r, n), _n(r, n, 0.1)
    a["v"], a["vb"] = _n(r, n), _n(r, n, 0.1)
    a["i_n"] = n
    return a


def halving(size, r):
    (n,) = size
    a = OrderedDict()
    a["x"], a["xb"] = _n(r, n), _n(r, n, 0.1)
    a["i_n"] = n
    return a


def divmod(size, r):
    n, d = size
    a = OrderedDict()
    a["x"], a["xb"] = _n(r, n), _n(r, n, 0.1)
    a["i_n"], a["i_d"] = n, d
    return a


def ragged(size, r):
    (n,) = size
    a = OrderedDict()
    a["loss"], a["lossb"] = np.full(1, 0.0), np.full(1, 0.75)
    a["x"], a["xb"] = _n(r, n), _n(r, n, 0.1)
    a["w"], a["wb"] = _n(r, 3, 0.8), _n(r, 3, 0.1)
    a["i_n"] = n
    return a


# name -> (file, builder, dims, initstacks argument names, sizes: small, odd, zero-trip, large)
CASES = {
    "affine_ls_b": ("affine_ls_b.jl", affine, None, ("n_s", "n_o", "n_i"),
                    [(37, 9, 5), (1, 1, 1), (0, 3, 2), (1024, 64, 32)]),
    "heat2d_b": ("heat2d_b.jl", heat, None, ("n", "n_step"),
                 [(7, 3), (1, 2), (5, 0), (96, 4)]),
    "decay_b": ("decay_b.jl", decay, None, ("i_n", "i_nstep"),
                [(33, 4), (1, 1), (0, 3), (4096, 8)]),
    "edge_relu_b": ("edge_relu_b.jl", edge_relu, {"i_e2n": ["2"]}, ("i_ne",),
                    [(20, 57), (2, 1), (3, 0), (2000, 50000)]),
    "bilin_b": ("bilin_b.jl", bilin, {"a": ["i_m"], "ab": ["i_m"]}, ("i_m", "i_n"),
                [(7, 5), (1, 1), (0, 4), (300, 200)]),
    "cumsum_sq_b": ("cumsum_sq_b.jl", cumsum_sq, None, ("i_n",), [(17,), (1,), (2000,)]),
    "window_b": ("window_b.jl", window, None, ("i_n", "i_k"),
                 [(40, 5), (1, 1), (0, 3), (5000, 17)]),
    "halving_b": ("halving_b.jl", halving, None, None, [(16,), (13,), (1,), (4096,)]),
    "smooth_b": ("smooth_b.jl", smooth, None, ("i_n",), [(12,), (3,), (2,), (100000,)]),
    "ragged_b": ("ragged_b.jl", ragged, None, ("i_n",), [(10,), (1,), (0,), (5000,)]),
    "divmod_b": ("divmod_b.jl", divmod, None, None,
                 [(50, 7), (777, 1), (0, 3), (500, 3), (1000, 64), (3000, 2147483647),
                  (3000, 2147483648), (20000, 97)]),
}


def source(name):
    """The C1 and C3 sweeps ship with the package (the bench's emitted arm
    runs them); the others are this directory's corpus."""
    import os
    from stadeb200 import emit
    if name in ("affine_ls_b", "heat2d_b"):
        return emit.generated_source(name)
    here = os.path.dirname(os.path.abspath(__file__))
    with open(os.path.join(here, CORPUS, CASES[name][0])) as f:
        return f.read()


def make(name, size, tag=""):
    _, builder, _, _, _ = CASES[name]
    return builder(size, _rng(f"{name}{size}{tag}"))


def stack_ints(name, args):
    keys = CASES[name][3]
    return [] if keys is None else [args[k] for k in keys]


def copy_args(a):
    return OrderedDict((k, v.copy() if isinstance(v, np.ndarray) else v) for k, v in a.items())
