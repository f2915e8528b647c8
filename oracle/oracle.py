"""TEST INFRASTRUCTURE ONLY: numpy/ctypes front end of the CPU oracle
(oracle.cc), the restatement of the adjoint / HVP sweeps STADE.jl generates.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module, as the checker or as the timed CPU baseline; the product path
(libstade_b200.so) never does.

Each function takes numpy arrays, runs the oracle IN PLACE on them exactly
as the generated code mutates its arguments, and returns what the generated
Julia returns (nothing, or the scalar adjoint for heat2d_b).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

_lib = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        P, I64, D = C.c_void_p, C.c_int64, C.c_double
        L.oracle_affine_ls_b_f64.argtypes = [P] * 12 + [I64] * 3
        L.oracle_affine_ls_b_f128.argtypes = [P] * 12 + [I64] * 3
        for n in ("oracle_mlp2_ce_b_f32", "oracle_mlp2_ce_b_f64", "oracle_mlp2_ce_b_f128"):
            getattr(L, n).argtypes = [P] * 20 + [I64] * 4
        for n in ("oracle_mlp2_ce_b_f32_omp", "oracle_mlp2_ce_b_f64_omp"):
            getattr(L, n).argtypes = [P] * 20 + [I64] * 4 + [C.c_int]
        for n in ("oracle_mlp2_ce_hv_f64_omp", "oracle_mlp2_ce_hv_f128_omp"):
            getattr(L, n).argtypes = [P] * 20 + [I64] * 4 + [P] * 20 + [C.c_int]
        for n in ("oracle_conv1d_relu_mse_b_f32_omp", "oracle_conv1d_relu_mse_b_f64_omp"):
            getattr(L, n).argtypes = [P] * 12 + [I64] * 5 + [C.c_int]
        for n in ("oracle_mlp2_ce_hv_f64", "oracle_mlp2_ce_hv_f128"):
            getattr(L, n).argtypes = [P] * 20 + [I64] * 4 + [P] * 20
        L.oracle_heat2d_b_f64.argtypes = [P] * 6 + [D, D, I64, I64, P]
        L.oracle_heat2d_b_f64.restype = D
        L.oracle_heat2d_b_f64_omp.argtypes = [P] * 6 + [D, D, I64, I64, P, C.c_int]
        L.oracle_heat2d_b_f64_omp.restype = D
        L.oracle_heat2d_b_f128.argtypes = [P] * 6 + [C.c_longdouble] * 2 + [I64, I64, P]
        L.oracle_heat2d_b_f128.restype = C.c_longdouble
        for n in ("oracle_conv1d_relu_mse_b_f32", "oracle_conv1d_relu_mse_b_f64",
                  "oracle_conv1d_relu_mse_b_f128"):
            getattr(L, n).argtypes = [P] * 12 + [I64] * 5
        for n in ("oracle_affine_ls_d_f64", "oracle_affine_ls_d_f128"):
            getattr(L, n).argtypes = [P] * 12 + [I64] * 3
        for n in ("oracle_mlp2_ce_d_f32", "oracle_mlp2_ce_d_f64", "oracle_mlp2_ce_d_f128"):
            getattr(L, n).argtypes = [P] * 20 + [I64] * 4
        L.oracle_heat2d_d_f64.argtypes = [P] * 6 + [D, D, I64, I64]
        L.oracle_heat2d_d_f128.argtypes = [P] * 6 + [C.c_longdouble] * 2 + [I64, I64]
        for n in ("oracle_conv1d_relu_mse_d_f32", "oracle_conv1d_relu_mse_d_f64",
                  "oracle_conv1d_relu_mse_d_f128"):
            getattr(L, n).argtypes = [P] * 12 + [I64] * 5
        for f in L.oracle_affine_ls_b_f64, L.oracle_mlp2_ce_b_f32:
            f.restype = None
        _lib = L
    return _lib


def _p(a: np.ndarray, dtype) -> int:
    assert a.dtype == dtype and a.flags.c_contiguous, (a.dtype, dtype)
    return a.ctypes.data


def affine_ls_b(loss, lossb, w, wb, b, bb, x, xb, t, tb, y, yb, n_s, n_o, n_i, truth=False):
    if truth:
        ld = np.longdouble
        arrs = [np.asarray(a, dtype=ld) for a in (loss, lossb, w, wb, b, bb, x, xb, t, tb, y, yb)]
        lib().oracle_affine_ls_b_f128(*[_p(a, ld) for a in arrs], n_s, n_o, n_i)
        for dst, src in zip((loss, lossb, w, wb, b, bb, x, xb, t, tb, y, yb), arrs):
            dst[...] = src
        return None
    f = np.float64
    lib().oracle_affine_ls_b_f64(*[_p(a, f) for a in (loss, lossb, w, wb, b, bb, x, xb, t, tb, y,
                                                       yb)], n_s, n_o, n_i)
    return None


def _truth_run(fn, arrs, *rest):
    """Runs the long-double (x87 80-bit) instantiation on widened copies of
    `arrs` and writes the results back into `arrs`, whose dtype stays as it
    was: the caller passes float64 arrays to keep the truth at full width."""
    ld = np.longdouble
    conv = [np.asarray(a, dtype=ld).copy() for a in arrs]
    r = fn(*[_p(a, ld) for a in conv], *rest)
    for dst, src in zip(arrs, conv):
        dst[...] = src
    return r


def mlp2_ce_b(loss, lossb, x, xb, y, yb, w1, w1b, b1, b1b, w2, w2b, b2, b2b, h, hb, z, zb, p, pb,
              n_s, n_i, n_h, n_o, threads=None, truth=False):
    arrs = (loss, lossb, x, xb, y, yb, w1, w1b, b1, b1b, w2, w2b, b2, b2b, h, hb, z, zb, p, pb)
    dt = arrs[0].dtype
    if truth:
        _truth_run(lib().oracle_mlp2_ce_b_f128, arrs, n_s, n_i, n_h, n_o)
        return None
    tag = "f32" if dt == np.float32 else "f64"
    if threads is not None:
        getattr(lib(), f"oracle_mlp2_ce_b_{tag}_omp")(*[_p(a, dt) for a in arrs], n_s, n_i, n_h,
                                                      n_o, threads)
    else:
        getattr(lib(), f"oracle_mlp2_ce_b_{tag}")(*[_p(a, dt) for a in arrs], n_s, n_i, n_h, n_o)
    return None


def mlp2_ce_hv(*args, truth=False, threads=None):
    """threads: samples split over that many host threads (0 = all), each
    block's summed shadows added in block order."""
    assert len(args) == 44
    arrs, ints, tans = list(args[:20]), args[20:24], list(args[24:])
    omp = () if threads is None else (threads,)
    sfx = "" if threads is None else "_omp"
    if truth:
        ld = np.longdouble
        conv = [np.asarray(a, dtype=ld) for a in arrs + tans]
        getattr(lib(), "oracle_mlp2_ce_hv_f128" + sfx)(*[_p(a, ld) for a in conv[:20]], *ints,
                                                       *[_p(a, ld) for a in conv[20:]], *omp)
        for dst, src in zip(arrs + tans, conv):
            dst[...] = src
        return None
    f = np.float64
    getattr(lib(), "oracle_mlp2_ce_hv_f64" + sfx)(*[_p(a, f) for a in arrs], *ints,
                                                  *[_p(a, f) for a in tans], *omp)
    return None


def heat2d_b(loss, lossb, u, ub, un, unb, alpha, alphab, n, n_step, u_stack, truth=False,
             threads=None):
    """threads: the per-cell loops over that many host threads (0 = all),
    bit-identical to the serial sweep."""
    f = np.float64
    if threads is not None and not truth:
        return lib().oracle_heat2d_b_f64_omp(_p(loss, f), _p(lossb, f), _p(u, f), _p(ub, f),
                                             _p(un, f), _p(unb, f), float(alpha), float(alphab),
                                             n, n_step, _p(u_stack, f), threads)
    if truth:
        return float(_truth_run(
            lambda *a: lib().oracle_heat2d_b_f128(*a[:6], alpha, alphab, n, n_step, a[6]),
            (loss, lossb, u, ub, un, unb, u_stack)))
    return lib().oracle_heat2d_b_f64(_p(loss, f), _p(lossb, f), _p(u, f), _p(ub, f), _p(un, f),
                                     _p(unb, f), float(alpha), float(alphab), n, n_step,
                                     _p(u_stack, f))


def conv1d_relu_mse_b(loss, lossb, x, xb, w, wb, t, tb, z, zb, r, rb, n_b, n_c, n_l, n_o, n_k,
                      truth=False, threads=None):
    """threads: samples split over that many host threads (0 = all), the mean
    loss's 1 / (n_b n_o n_lo) of the whole batch kept in every block."""
    arrs = (loss, lossb, x, xb, w, wb, t, tb, z, zb, r, rb)
    dt = arrs[0].dtype
    if truth:
        _truth_run(lib().oracle_conv1d_relu_mse_b_f128, arrs, n_b, n_c, n_l, n_o, n_k)
        return None
    tag = "f32" if dt == np.float32 else "f64"
    if threads is not None:
        getattr(lib(), f"oracle_conv1d_relu_mse_b_{tag}_omp")(*[_p(a, dt) for a in arrs], n_b,
                                                              n_c, n_l, n_o, n_k, threads)
    else:
        getattr(lib(), f"oracle_conv1d_relu_mse_b_{tag}")(*[_p(a, dt) for a in arrs], n_b, n_c,
                                                          n_l, n_o, n_k)
    return None


# ---- tangent (forward-mode) sweeps <k>_d, tgen_signature_args order ---------
def affine_ls_d(loss, lossd, w, wd, b, bd, x, xd, t, td, y, yd, n_s, n_o, n_i, truth=False):
    f = np.float64
    if truth:
        _truth_run(lib().oracle_affine_ls_d_f128, (loss, lossd, w, wd, b, bd, x, xd, t, td, y, yd),
                   n_s, n_o, n_i)
        return
    lib().oracle_affine_ls_d_f64(*[_p(a, f) for a in (loss, lossd, w, wd, b, bd, x, xd, t, td,
                                                      y, yd)], n_s, n_o, n_i)


def mlp2_ce_d(*args, truth=False):
    assert len(args) == 24
    arrs, ints = args[:20], args[20:]
    dt = arrs[0].dtype
    if truth:
        _truth_run(lib().oracle_mlp2_ce_d_f128, arrs, *ints)
        return
    fn = lib().oracle_mlp2_ce_d_f32 if dt == np.float32 else lib().oracle_mlp2_ce_d_f64
    fn(*[_p(a, dt) for a in arrs], *ints)


def heat2d_d(loss, lossd, u, ud, un, und, alpha, alphad, n, n_step, truth=False):
    f = np.float64
    if truth:
        _truth_run(lambda *a: lib().oracle_heat2d_d_f128(*a, alpha, alphad, n, n_step),
                   (loss, lossd, u, ud, un, und))
        return
    lib().oracle_heat2d_d_f64(*[_p(a, f) for a in (loss, lossd, u, ud, un, und)], float(alpha),
                              float(alphad), n, n_step)


def conv1d_relu_mse_d(loss, lossd, x, xd, w, wd, t, td, z, zd, r, rd, n_b, n_c, n_l, n_o, n_k,
                      truth=False):
    arrs = (loss, lossd, x, xd, w, wd, t, td, z, zd, r, rd)
    dt = arrs[0].dtype
    if truth:
        _truth_run(lib().oracle_conv1d_relu_mse_d_f128, arrs, n_b, n_c, n_l, n_o, n_k)
        return
    fn = lib().oracle_conv1d_relu_mse_d_f32 if dt == np.float32 else \
        lib().oracle_conv1d_relu_mse_d_f64
    fn(*[_p(a, dt) for a in arrs], n_b, n_c, n_l, n_o, n_k)


# ---- the oracle side's own input generator (synth.cc) ----------------------
def generator():
    """The configurations' seeded inputs drawn by liboracle's restatement of
    the generator, bit-identical to the product library's (checked in
    tests/test_seeds.py); the bench's reference arm uses it so that it never
    loads the product library."""
    import sys
    pkg = os.path.join(os.path.dirname(HERE), "stade.jl_b200")
    if pkg not in sys.path:
        sys.path.insert(0, pkg)
    from stadeb200.synth import Generator
    return Generator(lib, "oracle_")
