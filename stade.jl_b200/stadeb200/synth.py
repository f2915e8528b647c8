"""Seeded synthetic inputs of the five benchmark configurations.

No dataset is involved: the reference quotes no public benchmark for this path,
so every input is drawn here with the shapes and distributions the
configurations name. Seeds are FNV-1a-64 of "<kernel>:<array>" (the scheme
of val_stable_seed, src/STADE.jl:16619-16626) fed to the library's
documented generator (stade_fill_*), so the oracle and the GPU see the same
bits.
"""
from __future__ import annotations

import math

import numpy as np

from ._lib import lib

# Full sizes of the configurations (BASELINE configs C1..C5).
FULL = {
    "affine_ls": dict(n_s=1024, n_o=64, n_i=32),
    "mlp2_ce": dict(n_s=65536, n_i=784, n_h=512, n_o=10),
    "heat2d": dict(n=8192, n_step=16, alpha=0.2),
    "conv1d_relu_mse": dict(n_b=4096, n_c=64, n_l=2048, n_o=128, n_k=9),
    "mlp2_ce_hv": dict(n_s=16384, n_i=784, n_h=512, n_o=10),
}


def seed(kernel: str, array: str) -> int:
    return int(lib().stade_fnv1a64(f"{kernel}:{array}".encode()))


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def normal(n: int, seed_: int, dtype, mean=0.0, std=1.0) -> np.ndarray:
    a = np.empty(n, dtype=dtype)
    f = lib().stade_fill_normal_f64 if dtype == np.float64 else lib().stade_fill_normal_f32
    f(_ptr(a), n, seed_, mean, std)
    return a


def uniform(n: int, seed_: int, dtype, lo=0.0, hi=1.0) -> np.ndarray:
    a = np.empty(n, dtype=dtype)
    f = lib().stade_fill_uniform_f64 if dtype == np.float64 else lib().stade_fill_uniform_f32
    f(_ptr(a), n, seed_, lo, hi)
    return a


def onehot(n_rows: int, n_o: int, seed_: int, dtype) -> np.ndarray:
    a = np.empty(n_rows * n_o, dtype=dtype)
    f = lib().stade_fill_onehot_f64 if dtype == np.float64 else lib().stade_fill_onehot_f32
    f(_ptr(a), n_rows, n_o, seed_)
    return a


def affine_ls_inputs(n_s, n_o, n_i, kernel="affine_ls"):
    """C1: W, b, X, T ~ N(0,1), Float64; lossb = 1."""
    f = np.float64
    return dict(w=normal(n_o * n_i, seed(kernel, "w"), f), b=normal(n_o, seed(kernel, "b"), f),
                x=normal(n_s * n_i, seed(kernel, "x"), f), t=normal(n_s * n_o, seed(kernel, "t"), f),
                lossb=np.ones(1, f))


def mlp2_ce_inputs(n_s, n_i, n_h, n_o, dtype=np.float32, kernel="mlp2_ce"):
    """C2: X ~ U(0,1), one-hot Y, Xavier-uniform W1 / W2, b = 0; lossb = 1."""
    r1 = math.sqrt(6.0 / (n_i + n_h))
    r2 = math.sqrt(6.0 / (n_h + n_o))
    return dict(x=uniform(n_s * n_i, seed(kernel, "x"), dtype),
                y=onehot(n_s, n_o, seed(kernel, "y"), dtype),
                w1=uniform(n_i * n_h, seed(kernel, "w1"), dtype, -r1, r1),
                b1=np.zeros(n_h, dtype),
                w2=uniform(n_h * n_o, seed(kernel, "w2"), dtype, -r2, r2),
                b2=np.zeros(n_o, dtype), lossb=np.ones(1, dtype))


def mlp2_ce_hv_inputs(n_s, n_i, n_h, n_o, kernel="mlp2_ce_hv"):
    """C5: the C2 model in Float64 plus a N(0,1) direction over W1, b1, W2,
    b2; xd = yd = 0, lossbd = 0."""
    d = mlp2_ce_inputs(n_s, n_i, n_h, n_o, np.float64, kernel)
    f = np.float64
    d.update(w1d=normal(n_i * n_h, seed(kernel, "w1d"), f), b1d=normal(n_h, seed(kernel, "b1d"), f),
             w2d=normal(n_h * n_o, seed(kernel, "w2d"), f), b2d=normal(n_o, seed(kernel, "b2d"), f),
             xd=np.zeros(n_s * n_i, f), yd=np.zeros(n_s * n_o, f), lossbd=np.zeros(1, f))
    return d


def heat2d_inputs(n, kernel="heat2d"):
    """C3: u0 ~ N(0,1), Float64; lossb = 1."""
    return dict(u=normal(n * n, seed(kernel, "u"), np.float64), lossb=np.ones(1, np.float64))


def conv1d_relu_mse_inputs(n_b, n_c, n_l, n_o, n_k, kernel="conv1d_relu_mse"):
    """C4: X, W ~ N(0, 0.02), T ~ N(0, 1), Float32; lossb = 1."""
    f = np.float32
    n_lo = n_l - n_k + 1
    return dict(x=normal(n_b * n_c * n_l, seed(kernel, "x"), f, 0.0, 0.02),
                w=normal(n_o * n_c * n_k, seed(kernel, "w"), f, 0.0, 0.02),
                t=normal(n_b * n_o * n_lo, seed(kernel, "t"), f), lossb=np.ones(1, f))
