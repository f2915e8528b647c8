"""libstade_b200 on the golden fixtures' inputs (tests/golden/*.npz), judged
with the parity verdict against the fixtures' stored truth and oracle
outputs: the GPU's worst element-wise error against the truth within
max(rtol, 20 × the oracle's, ceiling) (Float64: 2.5e-14 / 1e-10; Float32:
1e-5 / 1e-5); heat2d's tape bit for bit."""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

import make_golden as mg  # noqa: E402
import parity  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", sorted(mg.SIZES))
def test_gpu_on_golden_fixture(name):
    kern = parity.KERNELS[name]
    meta, st, out, truth, ret, ret_truth = mg.load(name)
    ints, sc = meta["ints"], meta["scalars"]
    got = parity.cases.copy_state(st)
    r = kern.gpu(got, ints, sc) or []
    f32 = kern.dtype == np.float32
    rtol = parity.TOL_F32 if f32 else parity.RTOL_F64
    ceiling = parity.TOL_F32 if f32 else parity.TRUTH_CEILING_F64
    t_cpu, _ = parity._kink_truth(kern, st, truth, out, ints)
    t_gpu, _ = parity._kink_truth(kern, st, truth, got, ints)
    tr_cpu = tr_gpu = 0.0
    changed = 0
    for k in parity._float_arrays(kern, st):
        assert got[k].dtype == st[k].dtype, k
        tr_cpu = max(tr_cpu, parity.relerr_arr(t_cpu[k], out[k]))
        tr_gpu = max(tr_gpu, parity.relerr_arr(t_gpu[k], got[k]))
        changed += int(np.count_nonzero(got[k] != st[k]))
    assert len(r) == len(ret)
    for a, b, t in zip(r, ret, ret_truth):
        tr_cpu = max(tr_cpu, parity.relerr_scalar(t, b))
        tr_gpu = max(tr_gpu, parity.relerr_scalar(t, a))
    ok, tr_tol = parity.verdict(tr_cpu, tr_gpu, 1, True, changed, rtol, parity.TRUTH_FACTOR,
                                ceiling)
    assert ok, (name, tr_gpu, tr_tol, tr_cpu)
    if kern.stack:
        assert np.array_equal(got[kern.stack], out[kern.stack])
