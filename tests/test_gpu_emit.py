"""The .cu emitter's output on the B200: every corpus sweep emitted, built for
sm_100a and called through its C ABI on device arrays, against the
sequential interpreter (or, at the C1 / C3 sizes the interpreter is too slow
for, the C++ oracle it is pinned to). Atomics reorder sums, so float arrays
and returned scalars are compared with the Float64 bound 1e-12 (normwise
relative); integer arrays and tables bit for bit, float tapes within the same
bound (a tape of tanh values holds the device's tanh, ulps from the host's)."""
import numpy as np
import pytest
import torch

import cases
import emit_cases as ec
import jlsub
from oracle import oracle as orc
from refmath import rel_err
from stadeb200 import emit

pytestmark = pytest.mark.gpu


def _dev(args):
    return [torch.from_numpy(v.copy()).cuda() if isinstance(v, np.ndarray) else v
            for v in args.values()]


def _reference(name, args):
    a = ec.copy_args(args)
    size = None
    if name == "affine_ls_b" and a["n_s"] * a["n_o"] > 5000:
        orc.affine_ls_b(*[a[k] for k in cases.AFFINE_ARGS], a["n_s"], a["n_o"], a["n_i"])
        return a, None, ()
    if name == "heat2d_b" and a["n"] > 32:
        n, n_step = a["n"], a["n_step"]
        stack = np.zeros(max(n_step * n * n, 0))
        r = orc.heat2d_b(*[a[k] for k in cases.HEAT_ARGS], a["alpha"], a["alphab"], n, n_step,
                         stack if n_step else np.zeros(1))
        return a, r, (stack,)
    del size
    I = jlsub.Interp(ec.source(name), 64, ec.CASES[name][2])
    stacks = ()
    if f"initstacks_{name}" in I.funcs:
        stacks = I.initstacks(f"initstacks_{name}", *ec.stack_ints(name, a))
    r = I.call(name, *a.values(), *stacks)
    return a, r, stacks


@pytest.mark.parametrize("name", sorted(ec.CASES))
def test_emitted_sweep_on_gpu(name):
    sw = emit.load(ec.source(name), dims=ec.CASES[name][2])
    for size in ec.CASES[name][4]:
        args = ec.make(name, size)
        ref, r_ref, st_ref = _reference(name, args)
        dev = _dev(args)
        stacks = sw.initstacks(*ec.stack_ints(name, args))
        r_gpu = sw(*dev, *stacks)
        torch.cuda.synchronize()
        if r_ref is None:
            assert r_gpu is None
        else:
            rr = r_ref if isinstance(r_ref, tuple) else (r_ref,)
            rg = r_gpu if isinstance(r_gpu, tuple) else (r_gpu,)
            for x, y in zip(rr, rg):
                assert abs(x - y) <= 1e-12 * max(1.0, abs(x)), (name, size, x, y)
        for (k, v), d in zip(args.items(), dev):
            if not isinstance(v, np.ndarray):
                continue
            got = d.cpu().numpy()
            if v.dtype == np.int64:
                assert np.array_equal(got, ref[k]), (name, size, k)
            else:
                assert rel_err(got, ref[k]) <= 1e-12, (name, size, k, rel_err(got, ref[k]))
        for s_gpu, s_ref in zip(stacks, st_ref):
            got = s_gpu if isinstance(s_gpu, int) else s_gpu.cpu().numpy()
            if isinstance(got, np.ndarray) and got.dtype.kind == "f" and got.size:
                # taped values of device tanh / exp differ from the host's by ulps
                assert rel_err(got, s_ref) <= 1e-12, (name, size, "stack")
            else:
                assert np.array_equal(got, s_ref), (name, size, "stack")


def test_emitted_c1_matches_hand_written_sweep():
    """The generated C1 sweep and libstade_b200's hand-written one agree at the
    BASELINE size (both against the oracle, 1e-12)."""
    import stadeb200
    name = "affine_ls_b"
    args = ec.make(name, (1024, 64, 32), "hw")
    sw = emit.load(ec.source(name))
    d1, d2 = _dev(args), _dev(args)
    sw(*d1)
    stadeb200.affine_ls_b_cuda(*d2)
    torch.cuda.synchronize()
    for a, b in zip(d1, d2):
        if isinstance(a, torch.Tensor):
            assert rel_err(a.cpu().numpy(), b.cpu().numpy()) <= 1e-12


@pytest.mark.parametrize("name", ["affine_ls_b", "window_b", "smooth_b"])
def test_emitted_float32_on_gpu(name):
    """The Float32 build (cgen_convert_precision) against the interpreter in
    Float32, 1e-5 normwise (the north star's Float32 bound)."""
    sw = emit.load(ec.source(name), precision=32, dims=ec.CASES[name][2])
    args = ec.make(name, ec.CASES[name][4][0], "f32")
    for k, v in args.items():
        if isinstance(v, np.ndarray) and v.dtype == np.float64:
            args[k] = v.astype(np.float32)
    ref = ec.copy_args(args)
    I = jlsub.Interp(ec.source(name), 32, ec.CASES[name][2])
    stacks = ()
    if f"initstacks_{name}" in I.funcs:
        stacks = I.initstacks(f"initstacks_{name}", *ec.stack_ints(name, ref))
    I.call(name, *ref.values(), *stacks)
    dev = _dev(args)
    sw(*dev, *sw.initstacks(*ec.stack_ints(name, args)))
    torch.cuda.synchronize()
    for (k, v), d in zip(args.items(), dev):
        if isinstance(v, np.ndarray):
            got = d.cpu().numpy()
            assert got.dtype == np.float32
            assert rel_err(got, ref[k]) <= 1e-5, (name, k, rel_err(got, ref[k]))
