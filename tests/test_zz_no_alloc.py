"""The allocation-free entry point stade_affine_ls_b_f64_noalloc, through the
C ABI, against the workspace entry point stade_affine_ls_b_f64.

It serves callers that cannot allocate device memory where they run the
sweep (all device memory handed to their own pool, a fixed memory plan, a
thread that must not block on cudaMalloc): its scratch is a fixed array in
the library's device memory. Two calls in a row, so the second call runs on
the array the first one left behind. This file is collected last so that a
run stopping at its first failure has already run every other test.
"""
import ctypes as C

import pytest

import cases
from refmath import rel_err
from stadeb200 import _lib

pytestmark = pytest.mark.gpu

F64_TOL = 1e-12


def _to_dev(st):
    import torch
    return {k: torch.from_numpy(v.copy()).cuda() for k, v in st.items()}


def _call(name, dev, ints):
    import torch
    o = _lib.make_opts(torch.cuda.current_stream().cuda_stream)
    code = getattr(_lib.lib(), name)(*[dev[a].data_ptr() for a in cases.AFFINE_ARGS],
                                     ints["n_s"], ints["n_o"], ints["n_i"], C.byref(o))
    _lib.check(code)


@pytest.mark.parametrize("sizes", [(1024, 64, 32), (37, 9, 5)])
def test_noalloc_matches_workspace_entry_point(sizes):
    import torch
    st, ints = cases.affine_state(*sizes, seeded=True)
    ref, new = _to_dev(st), _to_dev(st)
    for _ in range(2):
        _call("stade_affine_ls_b_f64", ref, ints)
        _call("stade_affine_ls_b_f64_noalloc", new, ints)
        torch.cuda.synchronize()
        for k in cases.AFFINE_ARGS:
            a, b = new[k].cpu().numpy(), ref[k].cpu().numpy()
            assert rel_err(a, b) <= F64_TOL, k


def test_noalloc_rejects_sizes_beyond_its_array():
    import torch
    st, ints = cases.affine_state(16, 4, 4)
    dev = _to_dev(st)
    o = _lib.make_opts(torch.cuda.current_stream().cuda_stream)
    limit = _lib.lib().stade_affine_ls_b_f64_noalloc_max_scratch()
    assert limit == 2 << 20
    # 65,536 samples x 64 x 32 need 4096 blocks x 2,113 partials = 69 MB of scratch
    code = _lib.lib().stade_affine_ls_b_f64_noalloc(
        *[dev[a].data_ptr() for a in cases.AFFINE_ARGS], 65536, 64, 32, C.byref(o))
    assert code == _lib.STADE_EINVAL
    assert b"scratch" in _lib.lib().stade_last_error()
