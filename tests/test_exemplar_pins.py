"""Pins of the oracle's generation rules on the reference's own generated
code: seven sweeps the reference ships as generated text
(test/val-corpus/{affine_loss_b, matvec_loss_b, stencil_loss_b, advection_b,
selfrace_conv_b, mlp1d_b, mlp1d_hv}.jl), restated in oracle/oracle.cc on the
same rule helpers its five sweeps use, must reproduce bit for bit what that
text computes. The expected values are the reference text run by the
interpreter tests/jlsub.py on seeded inputs (tests/golden/exemplars/*.npz,
written by tests/golden/make_exemplar_golden.py, which records each text's
sha256)."""
import ctypes as C
import json
import os

import numpy as np
import pytest

from oracle import oracle as orc

HERE = os.path.dirname(os.path.abspath(__file__))
FIX = os.path.join(HERE, "golden", "exemplars")
NAMES = ("affine_loss_b", "matvec_loss_b", "stencil_loss_b", "advection_b", "selfrace_conv_b",
         "mlp1d_b", "mlp1d_hv")


def load(name):
    d = np.load(os.path.join(FIX, name + ".npz"))
    order = json.loads(str(d["order"]))
    ins = {k: d["in_" + k] for k in order}
    outs = {k: d["out_" + k] for k in order}
    stacks = [d[f"stack_{i}"] for i in range(int(d["n_stacks"]))]
    return order, ins, outs, stacks, d


def _run_oracle(name, order, ins, stacks):
    a = {k: (v.copy() if v.ndim else v.item()) for k, v in ins.items()}
    L = orc.lib()
    fn = getattr(L, f"oracle_ex_{name}_f64")
    ret = ()
    if name == "advection_b":
        boxes = {k: C.c_double(a[k]) for k in ("cb", "dxb", "dtb")}
        st = [np.zeros_like(s) for s in stacks]     # initstacks: a zeroed tape
        fn.restype = None
        fn(*[a[k].ctypes.data for k in ("u", "ub", "du", "dub")], C.c_double(a["c"]),
           C.byref(boxes["cb"]), C.c_double(a["dx"]), C.byref(boxes["dxb"]), C.c_double(a["dt"]),
           C.byref(boxes["dtb"]), C.c_int64(a["i_nstep"]), C.c_int64(a["i_nnode"]),
           st[0].ctypes.data)
        ret = tuple(boxes[k].value for k in ("cb", "dxb", "dtb"))
        for k in ("cb", "dxb", "dtb"):
            a[k] = boxes[k].value
        return a, ret, st
    args = []
    for k in order:
        v = a[k]
        args.append(C.c_void_p(v.ctypes.data) if isinstance(v, np.ndarray) else C.c_int64(v))
    fn.restype = None
    fn(*args)
    return a, ret, []


@pytest.mark.parametrize("name", NAMES)
def test_oracle_rules_reproduce_the_reference_generated_sweep(name):
    order, ins, outs, stacks, d = load(name)
    a, ret, st = _run_oracle(name, order, ins, stacks)
    changed = 0
    for k in order:
        if isinstance(a[k], np.ndarray):
            assert a[k].dtype == outs[k].dtype
            assert np.array_equal(a[k], outs[k]), (name, k, np.max(np.abs(a[k] - outs[k])))
            changed += int(not np.array_equal(ins[k], outs[k]))
    assert changed >= 3, name     # the call did something
    assert np.array_equal(np.array(ret, dtype=np.float64), d["ret"]), (name, ret, d["ret"])
    if name == "advection_b":
        # the tape the sweep wrote equals the interpreter's, slot for slot
        assert np.any(stacks[0] != 0)
        assert np.array_equal(st[0], stacks[0]), name
