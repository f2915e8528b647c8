"""Host mirror of the generated GPU entry points, by their generated names.

Each function here stands where STADE's CUDA port puts a host function
`<k>_b_cuda` (cgen_emit, src/STADE.jl:12062-12111) or `<k>_hv_cuda`, with the
generated argument order (agen_signature_args, src/STADE.jl:3455-3465; HVP
pairs per hvp_emit, src/STADE.jl:6751-6758), and calls libstade_b200 through
its C ABI. Arrays are CUDA tensors (the caller's device memory, as CuArrays
are for the generated code); integers are Python ints; a scalar float
argument's adjoint is passed in and returned, as the generated Julia returns
it by value (emit_return_scalars, src/STADE.jl:2072).

Every array is checked for device, dtype and length before the call; the
library raises StadeError on a CUDA or shape failure. There is no CPU path.
"""
from __future__ import annotations

import ctypes as C

import torch

from ._lib import STADE_HOST_SCALARS, check, lib, make_opts


def _stream_ptr(stream) -> int:
    if stream is None:
        stream = torch.cuda.current_stream()
    return stream.cuda_stream


def _arr(t: torch.Tensor, dtype: torch.dtype, n: int, name: str) -> int:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name}: expected a CUDA tensor, got {type(t).__name__}")
    if not t.is_cuda:
        raise ValueError(f"{name}: tensor must live on a CUDA device")
    if t.dtype != dtype:
        raise TypeError(f"{name}: dtype {t.dtype}, expected {dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name}: tensor must be contiguous")
    if t.numel() < n:
        raise ValueError(f"{name}: {t.numel()} elements, the kernel indexes {n}")
    return t.data_ptr()


def _opts(stream, workspace, flags=0):
    ws_ptr, ws_bytes = None, 0
    if workspace is not None:
        ws_ptr, ws_bytes = workspace.data_ptr(), workspace.numel() * workspace.element_size()
    return make_opts(_stream_ptr(stream), ws_ptr, ws_bytes, flags)


# ---------------------------------------------------------------------------
def affine_ls_b_cuda(loss, lossb, w, wb, b, bb, x, xb, t, tb, y, yb, n_s, n_o, n_i,
                     *, stream=None, workspace=None):
    """Adjoint of affine_ls (C1), Float64. Returns nothing (no scalar args)."""
    f64 = torch.float64
    ptrs = [_arr(loss, f64, 1, "loss"), _arr(lossb, f64, 1, "lossb"),
            _arr(w, f64, n_o * n_i, "w"), _arr(wb, f64, n_o * n_i, "wb"),
            _arr(b, f64, n_o, "b"), _arr(bb, f64, n_o, "bb"),
            _arr(x, f64, n_s * n_i, "x"), _arr(xb, f64, n_s * n_i, "xb"),
            _arr(t, f64, n_s * n_o, "t"), _arr(tb, f64, n_s * n_o, "tb"),
            _arr(y, f64, n_s * n_o, "y"), _arr(yb, f64, n_s * n_o, "yb")]
    o = _opts(stream, workspace)
    check(lib().stade_affine_ls_b_f64(*ptrs, n_s, n_o, n_i, C.byref(o)))


def affine_ls_b_workspace(n_s, n_o, n_i) -> int:
    return lib().stade_affine_ls_b_f64_workspace(n_s, n_o, n_i)


# ---------------------------------------------------------------------------
def mlp2_ce_b_cuda(loss, lossb, x, xb, y, yb, w1, w1b, b1, b1b, w2, w2b, b2, b2b,
                   h, hb, z, zb, p, pb, n_s, n_i, n_h, n_o, *, stream=None, workspace=None):
    """Adjoint of mlp2_ce (C2), Float32 (STADE's precision conversion)."""
    f = torch.float32
    ptrs = [_arr(loss, f, 1, "loss"), _arr(lossb, f, 1, "lossb"),
            _arr(x, f, n_s * n_i, "x"), _arr(xb, f, n_s * n_i, "xb"),
            _arr(y, f, n_s * n_o, "y"), _arr(yb, f, n_s * n_o, "yb"),
            _arr(w1, f, n_i * n_h, "w1"), _arr(w1b, f, n_i * n_h, "w1b"),
            _arr(b1, f, n_h, "b1"), _arr(b1b, f, n_h, "b1b"),
            _arr(w2, f, n_h * n_o, "w2"), _arr(w2b, f, n_h * n_o, "w2b"),
            _arr(b2, f, n_o, "b2"), _arr(b2b, f, n_o, "b2b"),
            _arr(h, f, n_s * n_h, "h"), _arr(hb, f, n_s * n_h, "hb"),
            _arr(z, f, n_s * n_o, "z"), _arr(zb, f, n_s * n_o, "zb"),
            _arr(p, f, n_s * n_o, "p"), _arr(pb, f, n_s * n_o, "pb")]
    o = _opts(stream, workspace)
    check(lib().stade_mlp2_ce_b_f32(*ptrs, n_s, n_i, n_h, n_o, C.byref(o)))


def mlp2_ce_b_workspace(n_s, n_i, n_h, n_o) -> int:
    return lib().stade_mlp2_ce_b_f32_workspace(n_s, n_i, n_h, n_o)


# ---------------------------------------------------------------------------
def initstacks_heat2d_b_cuda(n, n_step, device=None):
    """Tape of heat2d_b: n_step * n * n Float64 values (initstacks_heat2d_b)."""
    m = lib().stade_initstacks_heat2d_b(n, n_step)
    return torch.empty(max(m, 1), dtype=torch.float64, device=device or "cuda")


def heat2d_b_cuda(loss, lossb, u, ub, un, unb, alpha, alphab, n, n_step, u_stack,
                  *, stream=None, workspace=None):
    """Adjoint of heat2d (C3), Float64. Returns alphab (the scalar argument's
    adjoint, starting from the given value), as the generated Julia does."""
    f64 = torch.float64
    nn = n * n
    ptrs = [_arr(loss, f64, 1, "loss"), _arr(lossb, f64, 1, "lossb"),
            _arr(u, f64, nn, "u"), _arr(ub, f64, nn, "ub"),
            _arr(un, f64, nn, "un"), _arr(unb, f64, nn, "unb")]
    stack = _arr(u_stack, f64, lib().stade_initstacks_heat2d_b(n, n_step), "u_stack")
    box = C.c_double(float(alphab))
    o = _opts(stream, workspace, STADE_HOST_SCALARS)
    check(lib().stade_heat2d_b_f64(*ptrs, float(alpha), C.addressof(box), n, n_step, stack,
                                   C.byref(o)))
    return box.value


def heat2d_b_cuda_device(loss, lossb, u, ub, un, unb, alpha, alphab_dev, n, n_step, u_stack,
                         *, stream=None, workspace=None):
    """heat2d_b with alphab as a 1-element device tensor (no host sync)."""
    f64 = torch.float64
    nn = n * n
    ptrs = [_arr(loss, f64, 1, "loss"), _arr(lossb, f64, 1, "lossb"),
            _arr(u, f64, nn, "u"), _arr(ub, f64, nn, "ub"),
            _arr(un, f64, nn, "un"), _arr(unb, f64, nn, "unb")]
    stack = _arr(u_stack, f64, lib().stade_initstacks_heat2d_b(n, n_step), "u_stack")
    o = _opts(stream, workspace)
    check(lib().stade_heat2d_b_f64(*ptrs, float(alpha), _arr(alphab_dev, f64, 1, "alphab"), n,
                                   n_step, stack, C.byref(o)))


def heat2d_b_workspace(n, n_step) -> int:
    return lib().stade_heat2d_b_f64_workspace(n, n_step)


def initstacks_heat2d_b_slab_cuda(n, n_step, rows, device=None):
    """Tape of one slab: n_step states of (rows + 2) x n values (halo rows)."""
    m = lib().stade_initstacks_heat2d_b_slab(n, n_step, rows)
    return torch.empty(max(m, 1), dtype=torch.float64, device=device or "cuda")


def heat2d_b_slab_cuda(loss, lossb, u, ub, un, unb, alpha, alphab_dev, n, n_step, u_stack, rows,
                       comm=None, *, stream=None, workspace=None):
    """heat2d_b on this rank's slab of `rows` grid rows (rank order = slab
    order, periodic); loss and alphab_dev (1-element device tensors) receive
    the sums over all slabs. comm: a ddp.NcclComm, or None when the slab is
    the whole grid."""
    f = torch.float64
    nn = rows * n
    ptrs = [_arr(loss, f, 1, "loss"), _arr(lossb, f, 1, "lossb"), _arr(u, f, nn, "u"),
            _arr(ub, f, nn, "ub"), _arr(un, f, nn, "un"), _arr(unb, f, nn, "unb")]
    stack = _arr(u_stack, f, lib().stade_initstacks_heat2d_b_slab(n, n_step, rows), "u_stack")
    ab = _arr(alphab_dev, f, 1, "alphab")
    o = _opts(stream, workspace)
    handle = comm.handle if comm is not None else None
    check(lib().stade_heat2d_b_f64_slab(*ptrs, float(alpha), ab, n, n_step, stack, rows, handle,
                                        C.byref(o)))


def heat2d_b_slab_workspace(n, n_step, rows) -> int:
    return lib().stade_heat2d_b_f64_slab_workspace(n, n_step, rows)


# ---------------------------------------------------------------------------
def conv1d_relu_mse_b_cuda(loss, lossb, x, xb, w, wb, t, tb, z, zb, r, rb,
                           n_b, n_c, n_l, n_o, n_k, *, stream=None, workspace=None):
    """Adjoint of conv1d_relu_mse (C4), Float32."""
    f = torch.float32
    n_lo = n_l - n_k + 1
    nt = n_b * n_o * max(n_lo, 0)
    ptrs = [_arr(loss, f, 1, "loss"), _arr(lossb, f, 1, "lossb"),
            _arr(x, f, n_b * n_c * n_l, "x"), _arr(xb, f, n_b * n_c * n_l, "xb"),
            _arr(w, f, n_o * n_c * n_k, "w"), _arr(wb, f, n_o * n_c * n_k, "wb"),
            _arr(t, f, nt, "t"), _arr(tb, f, nt, "tb"),
            _arr(z, f, nt, "z"), _arr(zb, f, nt, "zb"),
            _arr(r, f, nt, "r"), _arr(rb, f, nt, "rb")]
    o = _opts(stream, workspace)
    check(lib().stade_conv1d_relu_mse_b_f32(*ptrs, n_b, n_c, n_l, n_o, n_k, C.byref(o)))


def conv1d_relu_mse_b_workspace(n_b, n_c, n_l, n_o, n_k) -> int:
    return lib().stade_conv1d_relu_mse_b_f32_workspace(n_b, n_c, n_l, n_o, n_k)


# ---------------------------------------------------------------------------
MLP_HV_ARGS = ["loss", "lossb", "x", "xb", "y", "yb", "w1", "w1b", "b1", "b1b", "w2", "w2b",
               "b2", "b2b", "h", "hb", "z", "zb", "p", "pb"]
MLP_HV_TAN = ["lossd", "lossbd", "xd", "xbd", "yd", "ybd", "w1d", "w1bd", "b1d", "b1bd",
              "w2d", "w2bd", "b2d", "b2bd", "hd", "hbd", "zd", "zbd", "pd", "pbd"]


def _mlp_len(name: str, n_s, n_i, n_h, n_o) -> int:
    base = {"loss": 1, "x": n_s * n_i, "y": n_s * n_o, "w1": n_i * n_h, "b1": n_h,
            "w2": n_h * n_o, "b2": n_o, "h": n_s * n_h, "z": n_s * n_o, "p": n_s * n_o}
    for key in sorted(base, key=len, reverse=True):   # "lossbd" -> "loss", "w1bd" -> "w1"
        if name.startswith(key):
            return base[key]
    raise KeyError(name)


def mlp2_ce_hv_cuda(*args, stream=None, workspace=None):
    """HVP of mlp2_ce (C5), Float64, argument layout of hvp_emit: the 20
    adjoint arrays, n_s, n_i, n_h, n_o, then the 20 (tangent, adjoint-of-
    tangent) arrays."""
    if len(args) != 44:
        raise TypeError(f"mlp2_ce_hv_cuda takes 44 positional arguments, got {len(args)}")
    arrs, (n_s, n_i, n_h, n_o), tans = args[:20], args[20:24], args[24:]
    f64 = torch.float64
    ptrs = []
    for name, t in zip(MLP_HV_ARGS, arrs):
        ptrs.append(_arr(t, f64, _mlp_len(name, n_s, n_i, n_h, n_o), name))
    tptrs = []
    for name, t in zip(MLP_HV_TAN, tans):
        tptrs.append(_arr(t, f64, _mlp_len(name, n_s, n_i, n_h, n_o), name))
    o = _opts(stream, workspace)
    check(lib().stade_mlp2_ce_hv_f64(*ptrs, n_s, n_i, n_h, n_o, *tptrs, C.byref(o)))


def mlp2_ce_hv_workspace(n_s, n_i, n_h, n_o) -> int:
    return lib().stade_mlp2_ce_hv_f64_workspace(n_s, n_i, n_h, n_o)


def kernel_launches() -> int:
    return lib().stade_kernel_launches()


def reset_kernel_launches() -> None:
    lib().stade_reset_kernel_launches()


# ---- tangent (forward-mode) sweeps <k>_d, tgen_signature_args order ----------
def affine_ls_d_cuda(loss, lossd, w, wd, b, bd, x, xd, t, td, y, yd, n_s, n_o, n_i, *,
                     stream=None, workspace=None):
    """Tangent of affine_ls (C1), Float64: lossd += directional derivative."""
    f = torch.float64
    sz = dict(loss=1, lossd=1, w=n_o * n_i, wd=n_o * n_i, b=n_o, bd=n_o, x=n_s * n_i,
              xd=n_s * n_i, t=n_s * n_o, td=n_s * n_o, y=n_s * n_o, yd=n_s * n_o)
    arrs = dict(loss=loss, lossd=lossd, w=w, wd=wd, b=b, bd=bd, x=x, xd=xd, t=t, td=td, y=y, yd=yd)
    ptrs = [_arr(arrs[k], f, sz[k], k) for k in sz]
    o = _opts(stream, workspace)
    check(lib().stade_affine_ls_d_f64(*ptrs, n_s, n_o, n_i, C.byref(o)))


MLP_D_ARGS = ["loss", "lossd", "x", "xd", "y", "yd", "w1", "w1d", "b1", "b1d", "w2", "w2d",
              "b2", "b2d", "h", "hd", "z", "zd", "p", "pd"]


def mlp2_ce_d_cuda(*args, stream=None, workspace=None):
    """Tangent of mlp2_ce: the 20 arrays of tgen_signature_args, then n_s,
    n_i, n_h, n_o. Float32 or Float64 by the arrays' dtype."""
    if len(args) != 24:
        raise TypeError(f"mlp2_ce_d_cuda takes 24 positional arguments, got {len(args)}")
    arrs, (n_s, n_i, n_h, n_o) = args[:20], args[20:]
    dt = arrs[0].dtype
    if dt not in (torch.float32, torch.float64):
        raise TypeError(f"mlp2_ce_d_cuda: unsupported dtype {dt}")
    ptrs = [_arr(t, dt, _mlp_len(nm, n_s, n_i, n_h, n_o), nm) for nm, t in zip(MLP_D_ARGS, arrs)]
    o = _opts(stream, workspace)
    fn = lib().stade_mlp2_ce_d_f32 if dt == torch.float32 else lib().stade_mlp2_ce_d_f64
    check(fn(*ptrs, n_s, n_i, n_h, n_o, C.byref(o)))


def heat2d_d_cuda(loss, lossd, u, ud, un, und, alpha, alphad, n, n_step, *, stream=None,
                  workspace=None):
    """Tangent of heat2d (C3), Float64."""
    f = torch.float64
    nn = n * n
    ptrs = [_arr(loss, f, 1, "loss"), _arr(lossd, f, 1, "lossd"), _arr(u, f, nn, "u"),
            _arr(ud, f, nn, "ud"), _arr(un, f, nn, "un"), _arr(und, f, nn, "und")]
    o = _opts(stream, workspace)
    check(lib().stade_heat2d_d_f64(*ptrs, float(alpha), float(alphad), n, n_step, C.byref(o)))


def conv1d_relu_mse_d_cuda(loss, lossd, x, xd, w, wd, t, td, z, zd, r, rd, n_b, n_c, n_l, n_o,
                           n_k, *, stream=None, workspace=None):
    """Tangent of conv1d_relu_mse (C4), Float32."""
    f = torch.float32
    n_lo = n_l - n_k + 1
    nt = n_b * n_o * max(n_lo, 0)
    nx, nw = n_b * n_c * n_l, n_o * n_c * n_k
    sz = [("loss", 1), ("lossd", 1), ("x", nx), ("xd", nx), ("w", nw), ("wd", nw), ("t", nt),
          ("td", nt), ("z", nt), ("zd", nt), ("r", nt), ("rd", nt)]
    arrs = (loss, lossd, x, xd, w, wd, t, td, z, zd, r, rd)
    ptrs = [_arr(a, f, n, nm) for a, (nm, n) in zip(arrs, sz)]
    o = _opts(stream, workspace)
    check(lib().stade_conv1d_relu_mse_d_f32(*ptrs, n_b, n_c, n_l, n_o, n_k, C.byref(o)))
