"""Failure detection without a GPU fault.

A rank that never joins: one process creates a two-rank communicator alone;
the library's bounded host-side wait gives up after the communicator's
timeout, aborts the half-made communicator and returns STADE_ETIMEDOUT, and
the process's GPU context keeps working (a sweep runs correctly afterwards).
Nothing is launched on the GPU while the wait runs.

A device-side wait that nothing satisfies: stade_check_bounded_wait runs the
tensor-core kernels' own bounded mbarrier wait on a barrier no thread arrives
on, with a ~0.1 s limit; the wait gives up, the device error word is set,
the kernel returns, and the context stays usable (a tensor-core sweep runs
correctly afterwards and leaves the error word clear). No __trap, no bad
address, no endless loop: the wait is bounded by the SM clock.

The reference has no run-time guard beyond check_replicas
(src/STADE.jl:17665); these are the library's own.
"""
import ctypes as C
import os
import subprocess
import sys

import numpy as np
import pytest

import cases
from refmath import rel_err
from stadeb200 import _lib

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

_NEVER_JOINS = r"""
import sys, time, ctypes as C
sys.path[:0] = [{root!r}, {pkg!r}, {tests!r}]
import numpy as np, torch
import cases
from refmath import rel_err
from stadeb200 import _lib
torch.cuda.set_device(0)
L = _lib.lib()
uid = C.create_string_buffer(128)
_lib.check(L.stade_comm_unique_id(uid))
h = C.c_void_p()
t0 = time.time()
code = L.stade_comm_init(uid.raw, 2, 0, 1500, C.byref(h))   # rank 1 never joins
dt = time.time() - t0
print("code", code, "elapsed", round(dt, 2), "msg", L.stade_last_error().decode())
assert code == _lib.STADE_ETIMEDOUT and not h.value, code
# the context still works: a C1 sweep against the oracle
st, ints = cases.affine_state(37, 9, 5, seeded=True)
ref, out = cases.copy_state(st), cases.copy_state(st)
cases.oracle_affine(ref, ints)
cases.gpu_affine(out, ints)
assert all(rel_err(out[k], ref[k]) <= 1e-12 for k in cases.AFFINE_ARGS)
print("context ok")
"""


def test_comm_init_times_out_when_a_rank_never_joins():
    code = _NEVER_JOINS.format(root=ROOT, pkg=os.path.join(ROOT, "stade.jl_b200"), tests=HERE)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=180,
                       env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "context ok" in r.stdout
    line = [l for l in r.stdout.splitlines() if l.startswith("code")][0]
    elapsed = float(line.split()[3])
    assert 1.0 <= elapsed <= 60.0, line        # waited about the timeout, then gave up


def test_device_wait_guard_returns_and_reports():
    import torch
    L = _lib.lib()
    L.stade_device_error()                       # start from a clear error word
    o = _lib.make_opts(torch.cuda.current_stream().cuda_stream)
    code = L.stade_check_bounded_wait(200_000_000, C.byref(o))   # ~0.1 s of SM clock
    assert code == _lib.STADE_ETIMEDOUT, L.stade_last_error()
    assert L.stade_device_error() != 0           # the guard recorded the timeout
    assert L.stade_device_error() == 0           # reading cleared it
    # out-of-range limits are refused before any launch
    assert L.stade_check_bounded_wait(10, C.byref(o)) == _lib.STADE_EINVAL
    # the context keeps working: a tensor-core sweep, no wait runs out
    st, ints = cases.mlp_state(300, 132, 200, 10, seeded=True)
    ref, out = cases.copy_state(st), cases.copy_state(st)
    truth = cases.OrderedDict((k, v.astype(np.float64)) for k, v in st.items())
    cases.oracle_mlp(truth, ints)
    cases.gpu_mlp(out, ints)
    assert L.stade_device_error() == 0
    for k in ("h", "z", "w1b", "xb", "loss"):
        assert rel_err(out[k], truth[k]) <= 1e-5, k
