"""The allocation-free entry point stade_affine_ls_b_f64_noalloc, through the
C ABI, against the workspace entry point stade_affine_ls_b_f64.

It serves callers that cannot allocate device memory where they run the
sweep (all device memory handed to their own pool, a fixed memory plan, a
thread that must not block on cudaMalloc): its scratch is a fixed array in
the library's device memory. Both entry points launch the same two kernels
with the same fixed-order sums, so their outputs must agree bit for bit. Two
calls in a row, so the second call runs on the array the first one left
behind. This file is collected last so that a run stopping at its first
failure has already run every other test.
"""
import ctypes as C
import os
import subprocess
import sys

import numpy as np
import pytest

import cases
from stadeb200 import _lib

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
CHUNK = 8    # samples per block of the C1 kernels: one partial record per block


def _to_dev(st):
    import torch
    return {k: torch.from_numpy(v.copy()).cuda() for k, v in st.items()}


def _call(name, dev, ints):
    import torch
    o = _lib.make_opts(torch.cuda.current_stream().cuda_stream)
    return getattr(_lib.lib(), name)(*[dev[a].data_ptr() for a in cases.AFFINE_ARGS],
                                     ints["n_s"], ints["n_o"], ints["n_i"], C.byref(o))


def _max_samples(n_o, n_i):
    """The largest batch whose partial records fit the fixed array."""
    per_block = n_o * n_i + n_o + 1
    limit = _lib.lib().stade_affine_ls_b_f64_noalloc_max_scratch() // 8
    return (limit // per_block) * CHUNK


@pytest.mark.parametrize("sizes", [(1024, 64, 32), (37, 9, 5), ("max", 64, 32)])
def test_noalloc_matches_workspace_entry_point(sizes):
    import torch
    if sizes[0] == "max":
        # the last partial slot of the array is in use
        sizes = (_max_samples(sizes[1], sizes[2]), sizes[1], sizes[2])
    st, ints = cases.affine_state(*sizes, seeded=True)
    ref, new = _to_dev(st), _to_dev(st)
    for _ in range(2):
        _lib.check(_call("stade_affine_ls_b_f64", ref, ints))
        _lib.check(_call("stade_affine_ls_b_f64_noalloc", new, ints))
        torch.cuda.synchronize()
        for k in cases.AFFINE_ARGS:
            assert np.array_equal(new[k].cpu().numpy(), ref[k].cpu().numpy()), k


def test_noalloc_rejects_sizes_beyond_its_array():
    import torch
    limit = _lib.lib().stade_affine_ls_b_f64_noalloc_max_scratch()
    assert limit == 4 << 20
    n_s = _max_samples(64, 32) + 1          # one block more than the array holds
    st, ints = cases.affine_state(n_s, 64, 32)
    dev = _to_dev(st)
    code = _call("stade_affine_ls_b_f64_noalloc", dev, ints)
    assert code == _lib.STADE_EINVAL
    assert b"scratch" in _lib.lib().stade_last_error()
    torch.cuda.synchronize()


_FRESH = r"""
import sys
sys.path[:0] = [{root!r}, {pkg!r}, {tests!r}]
import numpy as np, torch
import cases
from stadeb200 import _lib
import ctypes as C
torch.cuda.set_device(0)
st, ints = cases.affine_state(1024, 64, 32, seeded=True)
dev = {{k: torch.from_numpy(v.copy()).cuda() for k, v in st.items()}}
o = _lib.make_opts(torch.cuda.current_stream().cuda_stream)
for _ in range(2):
    _lib.check(_lib.lib().stade_affine_ls_b_f64_noalloc(
        *[dev[a].data_ptr() for a in cases.AFFINE_ARGS], 1024, 64, 32, C.byref(o)))
torch.cuda.synchronize()
print("cached", _lib.lib().stade_workspace_cached_bytes())
"""


def test_noalloc_first_in_a_fresh_process_allocates_nothing():
    """Run alone in a new process, before any other entry point: the
    library's workspace cache stays empty, so nothing was allocated for the
    call."""
    root = os.path.dirname(HERE)
    code = _FRESH.format(root=root, pkg=os.path.join(root, "stade.jl_b200"), tests=HERE)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    assert "cached 0" in r.stdout, r.stdout
