"""The golden fixtures (tests/golden/*.npz, written by make_golden.py): the
input generator rebuilds their inputs bit for bit, the oracle reproduces
their outputs bit for bit and their long-double truth to 1e-15, and the
stored oracle outputs lie within the parity tolerances of the stored truth
(Float64 1e-10, the verdict's ceiling; Float32 1e-5; C4's ReLU kinks judged
against the branch taken)."""
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

import make_golden as mg  # noqa: E402
import parity  # noqa: E402

NAMES = sorted(mg.SIZES)


def test_every_sweep_has_a_fixture():
    assert set(NAMES) == set(parity.KERNELS)
    for n in NAMES:
        assert os.path.exists(os.path.join(HERE, "golden", n + ".npz")), n


@pytest.mark.parametrize("name", NAMES)
def test_inputs_regenerate(name):
    kern, ints, st, sc = mg.trial(name)
    meta, st_g, _, _, _, _ = mg.load(name)
    assert meta["ints"] == ints and meta["scalars"] == sc
    assert list(st) == list(st_g)
    for k in st:
        assert st[k].dtype == st_g[k].dtype and np.array_equal(st[k], st_g[k]), k


@pytest.mark.parametrize("name", NAMES)
def test_oracle_reproduces_outputs(name):
    kern = parity.KERNELS[name]
    meta, st, out, truth, ret, ret_truth = mg.load(name)
    ints, sc = meta["ints"], meta["scalars"]
    got = parity.cases.copy_state(st)
    r = kern.cpu(got, ints, sc, False) or []
    for k in st:
        assert np.array_equal(got[k], out[k]), k
    assert r == ret
    big = parity.OrderedDict((k, v.astype(np.float64)) for k, v in st.items())
    rb = kern.cpu(big, ints, sc, True) or []
    for k in st:
        assert parity.relerr_arr(big[k], truth[k]) <= 1e-15, k
    for a, b in zip(rb, ret_truth):
        assert parity.relerr_scalar(a, b) <= 1e-15


@pytest.mark.parametrize("name", NAMES)
def test_oracle_within_tolerance_of_truth(name):
    kern = parity.KERNELS[name]
    meta, st, out, truth, ret, ret_truth = mg.load(name)
    tol = parity.TOL_F32 if kern.dtype == np.float32 else parity.TRUTH_CEILING_F64
    t_adj, _ = parity._kink_truth(kern, st, truth, out, meta["ints"])
    changed = 0
    for k in parity._float_arrays(kern, st):
        assert parity.relerr_arr(t_adj[k], out[k]) <= tol, k
        changed += int(np.count_nonzero(out[k] != st[k]))
    for a, b in zip(ret, ret_truth):
        assert parity.relerr_scalar(a, b) <= tol
    assert changed > 0
