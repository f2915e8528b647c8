"""Sweeps the reference generated, run on the B200: the .cu emitter's sm_100a
build of seven of the reference's generated texts (test/val-corpus:
affine_loss_b, matvec_loss_b, stencil_loss_b, advection_b, selfrace_conv_b,
mlp1d_b, mlp1d_hv), called through its C ABI on device arrays, against what
that text computes (the interpreter tests/jlsub.py on the same seeded
inputs, tests/golden/exemplars/*.npz). The builds are made, with the
fixtures, by tests/golden/make_exemplar_golden.py where the reference
checkout exists, and travel with the working tree as stade.jl_b200/_gen/
libraries (the reference text does not). Atomic accumulation reorders sums,
so float arrays and returned scalars must agree within 1e-12 (the
reference's element-wise form, and normwise); tapes within the same bound."""
import json
import os

import numpy as np
import pytest
import torch

from refmath import ref_rel_err, rel_err
from stadeb200 import emit

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
FIX = os.path.join(HERE, "golden", "exemplars")
NAMES = ("affine_loss_b", "matvec_loss_b", "stencil_loss_b", "advection_b", "selfrace_conv_b",
         "mlp1d_b", "mlp1d_hv")


@pytest.mark.parametrize("name", NAMES)
def test_reference_generated_sweep_on_gpu(name):
    d = np.load(os.path.join(FIX, name + ".npz"))
    so = os.path.join(emit.GEN_DIR, str(d["so_name"]))
    if not os.path.exists(so):
        pytest.skip(f"{so} not built: run tests/golden/make_exemplar_golden.py")
    man = json.loads(str(d["manifest"]))
    sw = emit.Sweep(so, man)
    order = json.loads(str(d["order"]))
    ins = {k: d["in_" + k] for k in order}
    dev = {}
    for k in order:
        v = ins[k]
        dev[k] = torch.from_numpy(v.copy()).cuda() if v.ndim else v.item()
    stacks = sw.initstacks(*[dev[a] for a in man["initstacks"]["args"]]) \
        if man["initstacks"]["symbol"] else ()
    r = sw(*[dev[k] for k in order], *stacks)
    torch.cuda.synchronize()
    ret = () if r is None else (r if isinstance(r, tuple) else (r,))
    want = d["ret"]
    assert len(ret) == len(want)
    for x, y in zip(ret, want):
        assert abs(x - y) <= 1e-12 * max(1.0, abs(y)), (name, x, y)
    for k in order:
        if not isinstance(dev[k], torch.Tensor):
            continue
        got, exp = dev[k].cpu().numpy(), d["out_" + k]
        assert ref_rel_err(got, exp) <= 1e-12 and rel_err(got, exp) <= 1e-12, (name, k)
    for i, s in enumerate(stacks):
        got = s.cpu().numpy() if isinstance(s, torch.Tensor) else s
        exp = d[f"stack_{i}"]
        assert rel_err(got, exp) <= 1e-12, (name, "stack", i)
