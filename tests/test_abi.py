"""The C ABI library loads on a machine without a GPU and exports every
function include/stade_b200.h declares; argument checks that precede any
CUDA call return STADE_EINVAL; workspace queries are pure host functions."""
import ctypes as C
import os
import re

import pytest

import stadeb200
from stadeb200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "stade_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(stade_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = stadeb200.lib()
    names = declared_functions()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(L, n)]
    assert missing == []


def test_python_binding_covers_the_header():
    assert set(declared_functions()) <= set(_lib.SIGNATURES)


def test_version_and_launch_counter():
    L = stadeb200.lib()
    assert b"sm_100a" in L.stade_version()
    L.stade_reset_kernel_launches()
    assert L.stade_kernel_launches() == 0


def test_workspace_queries():
    L = stadeb200.lib()
    assert L.stade_initstacks_heat2d_b(8192, 16) == 16 * 8192 * 8192
    assert L.stade_initstacks_heat2d_b(0, 16) == 0
    assert L.stade_affine_ls_b_f64_workspace(1024, 64, 32) > 0
    assert L.stade_mlp2_ce_b_f32_workspace(65536, 784, 512, 10) >= 65536 * 512 * 4
    assert L.stade_mlp2_ce_hv_f64_workspace(16384, 784, 512, 10) >= 3 * 16384 * 512 * 8
    assert L.stade_conv1d_relu_mse_b_f32_workspace(4096, 64, 2048, 128, 9) >= 4096 * 128 * 2040 * 4
    assert L.stade_heat2d_b_f64_workspace(8192, 16) > 0


def test_argument_errors_before_any_cuda_call():
    L = stadeb200.lib()
    o = _lib.make_opts()
    nul = [None] * 12
    assert L.stade_affine_ls_b_f64(*nul, -1, 4, 4, C.byref(o)) == _lib.STADE_EINVAL
    assert L.stade_affine_ls_b_f64(*nul, 4, 4, 4, C.byref(o)) == _lib.STADE_EINVAL
    assert b"null" in L.stade_last_error()
    assert L.stade_mlp2_ce_b_f32(*([None] * 20), 4, 4, 4, 64, C.byref(o)) == _lib.STADE_EINVAL
    assert L.stade_heat2d_b_f64(*([None] * 6), 0.2, None, 8, 2, None, C.byref(o)) == _lib.STADE_EINVAL
    box = C.c_double(0.0)
    assert L.stade_heat2d_b_f64(*([None] * 6), 0.2, C.addressof(box), 7, 2, None,
                                C.byref(o)) == _lib.STADE_EINVAL
    assert L.stade_conv1d_relu_mse_b_f32(*([None] * 12), 1, 1, 8, 1, 3, C.byref(o)) == _lib.STADE_EINVAL
    # zero-trip loops: nothing to do, nothing touched
    assert L.stade_affine_ls_b_f64(*nul, 0, 4, 4, C.byref(o)) == _lib.STADE_OK
    assert L.stade_conv1d_relu_mse_b_f32(*([None] * 12), 1, 1, 2, 1, 3, C.byref(o)) == _lib.STADE_OK


def test_kernels_refuse_host_tensors():
    import torch
    t = torch.zeros(4, dtype=torch.float64)
    with pytest.raises(ValueError):
        stadeb200.affine_ls_b_cuda(*([t] * 12), 1, 2, 2)
