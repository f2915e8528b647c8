"""Seeded synthetic inputs of the five benchmark configurations.

No dataset is involved: the reference quotes no public benchmark for this path,
so every input is drawn here with the shapes and distributions the
configurations name. Seeds are FNV-1a-64 of "<kernel>:<array>" (the scheme
of val_stable_seed, src/STADE.jl:16619-16626) fed to a documented generator
(xoshiro256** per 2^20-element chunk, Box-Muller cosine normals), so the oracle
and the GPU see the same bits.

`Generator` draws through any shared library exporting `<prefix>fnv1a64` and
`<prefix>fill_{normal,uniform,onehot}_{f64,f32}`: by default the product
library's `stade_` functions; the test side builds one over its own
restatement of the generator, so a CPU-only run never loads this library.
"""
from __future__ import annotations

import math

import numpy as np

# Full sizes of the configurations (BASELINE configs C1..C5).
FULL = {
    "affine_ls": dict(n_s=1024, n_o=64, n_i=32),
    "mlp2_ce": dict(n_s=65536, n_i=784, n_h=512, n_o=10),
    "heat2d": dict(n=8192, n_step=16, alpha=0.2),
    "conv1d_relu_mse": dict(n_b=4096, n_c=64, n_l=2048, n_o=128, n_k=9),
    "mlp2_ce_hv": dict(n_s=16384, n_i=784, n_h=512, n_o=10),
}


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class Generator:
    """The input recipes of the five configurations over one library's fill
    functions (`lib` a ctypes library or a callable returning one)."""

    def __init__(self, lib, prefix: str):
        self._lib, self._prefix = lib, prefix

    def _fn(self, name):
        import ctypes as C
        L = self._lib() if callable(self._lib) else self._lib
        f = getattr(L, self._prefix + name)
        if name == "fnv1a64":
            f.restype, f.argtypes = C.c_uint64, [C.c_char_p]
        elif name.startswith("fill_onehot"):
            f.restype, f.argtypes = None, [C.c_void_p, C.c_int64, C.c_int64, C.c_uint64]
        else:
            f.restype = None
            f.argtypes = [C.c_void_p, C.c_int64, C.c_uint64, C.c_double, C.c_double]
        return f

    def seed(self, kernel: str, array: str) -> int:
        return int(self._fn("fnv1a64")(f"{kernel}:{array}".encode()))

    def normal(self, n: int, seed_: int, dtype, mean=0.0, std=1.0) -> np.ndarray:
        a = np.empty(n, dtype=dtype)
        self._fn("fill_normal_f64" if dtype == np.float64 else "fill_normal_f32")(
            _ptr(a), n, seed_, mean, std)
        return a

    def uniform(self, n: int, seed_: int, dtype, lo=0.0, hi=1.0) -> np.ndarray:
        a = np.empty(n, dtype=dtype)
        self._fn("fill_uniform_f64" if dtype == np.float64 else "fill_uniform_f32")(
            _ptr(a), n, seed_, lo, hi)
        return a

    def onehot(self, n_rows: int, n_o: int, seed_: int, dtype) -> np.ndarray:
        a = np.empty(n_rows * n_o, dtype=dtype)
        self._fn("fill_onehot_f64" if dtype == np.float64 else "fill_onehot_f32")(
            _ptr(a), n_rows, n_o, seed_)
        return a

    def affine_ls_inputs(self, n_s, n_o, n_i, kernel="affine_ls"):
        """C1: W, b, X, T ~ N(0,1), Float64; lossb = 1."""
        f, sd = np.float64, self.seed
        return dict(w=self.normal(n_o * n_i, sd(kernel, "w"), f),
                    b=self.normal(n_o, sd(kernel, "b"), f),
                    x=self.normal(n_s * n_i, sd(kernel, "x"), f),
                    t=self.normal(n_s * n_o, sd(kernel, "t"), f), lossb=np.ones(1, f))

    def mlp2_ce_inputs(self, n_s, n_i, n_h, n_o, dtype=np.float32, kernel="mlp2_ce"):
        """C2: X ~ U(0,1), one-hot Y, Xavier-uniform W1 / W2, b = 0; lossb = 1."""
        r1 = math.sqrt(6.0 / (n_i + n_h))
        r2 = math.sqrt(6.0 / (n_h + n_o))
        sd = self.seed
        return dict(x=self.uniform(n_s * n_i, sd(kernel, "x"), dtype),
                    y=self.onehot(n_s, n_o, sd(kernel, "y"), dtype),
                    w1=self.uniform(n_i * n_h, sd(kernel, "w1"), dtype, -r1, r1),
                    b1=np.zeros(n_h, dtype),
                    w2=self.uniform(n_h * n_o, sd(kernel, "w2"), dtype, -r2, r2),
                    b2=np.zeros(n_o, dtype), lossb=np.ones(1, dtype))

    def mlp2_ce_hv_inputs(self, n_s, n_i, n_h, n_o, kernel="mlp2_ce_hv"):
        """C5: the C2 model in Float64 plus a N(0,1) direction over W1, b1, W2,
        b2; xd = yd = 0, lossbd = 0."""
        d = self.mlp2_ce_inputs(n_s, n_i, n_h, n_o, np.float64, kernel)
        f, sd = np.float64, self.seed
        d.update(w1d=self.normal(n_i * n_h, sd(kernel, "w1d"), f),
                 b1d=self.normal(n_h, sd(kernel, "b1d"), f),
                 w2d=self.normal(n_h * n_o, sd(kernel, "w2d"), f),
                 b2d=self.normal(n_o, sd(kernel, "b2d"), f),
                 xd=np.zeros(n_s * n_i, f), yd=np.zeros(n_s * n_o, f), lossbd=np.zeros(1, f))
        return d

    def heat2d_inputs(self, n, kernel="heat2d"):
        """C3: u0 ~ N(0,1), Float64; lossb = 1."""
        return dict(u=self.normal(n * n, self.seed(kernel, "u"), np.float64),
                    lossb=np.ones(1, np.float64))

    def conv1d_relu_mse_inputs(self, n_b, n_c, n_l, n_o, n_k, kernel="conv1d_relu_mse"):
        """C4: X, W ~ N(0, 0.02), T ~ N(0, 1), Float32; lossb = 1."""
        f, sd = np.float32, self.seed
        n_lo = n_l - n_k + 1
        return dict(x=self.normal(n_b * n_c * n_l, sd(kernel, "x"), f, 0.0, 0.02),
                    w=self.normal(n_o * n_c * n_k, sd(kernel, "w"), f, 0.0, 0.02),
                    t=self.normal(n_b * n_o * n_lo, sd(kernel, "t"), f), lossb=np.ones(1, f))


def _product_lib():
    from ._lib import lib
    return lib()


_default = Generator(_product_lib, "stade_")
seed = _default.seed
normal = _default.normal
uniform = _default.uniform
onehot = _default.onehot
affine_ls_inputs = _default.affine_ls_inputs
mlp2_ce_inputs = _default.mlp2_ce_inputs
mlp2_ce_hv_inputs = _default.mlp2_ce_hv_inputs
heat2d_inputs = _default.heat2d_inputs
conv1d_relu_mse_inputs = _default.conv1d_relu_mse_inputs
