"""The reference's GPU parity verdict (tests/parity.py, restating
val_gpu_parity_script, src/STADE.jl:18939-19175) on every sweep
libstade_b200 exports: three seeded trials, every shadow drawn at random,
the long-double truth, `ok` by the reference's rule. (The north star's
normwise 1e-5 bound for the Float32 sweeps is tests/test_gpu_parity.py's.)"""
import subprocess
import sys
import json

import pytest

import parity

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", sorted(parity.KERNELS))
def test_parity_script_verdict(name):
    k = parity.KERNELS[name]
    r = parity.run(k, dict(k.defaults), trials=3)
    assert r["ok"] and not r["vacuous"], r
    assert r["truth_trials"] == 3
    if k.stack:
        # the tape holds the forward states, computed in the generated order
        assert r["stack_max_rel_err"] == 0.0, r


@pytest.mark.parametrize("name,sizes", [
    ("mlp2_ce_b", ["n_s=37", "n_i=20", "n_h=12", "n_o=3"]),
    ("heat2d_b", ["n=5", "n_step=3"]),
    ("conv1d_relu_mse_b", ["n_b=3", "n_c=5", "n_l=17", "n_o=6", "n_k=4"]),
    ("mlp2_ce_hv", ["n_s=9", "n_i=7", "n_h=5", "n_o=4"]),
])
def test_parity_script_cli_odd_sizes(name, sizes):
    p = subprocess.run([sys.executable, parity.__file__, "--kernel", name, "--trials", "2",
                        "--size", *sizes], capture_output=True, text=True, cwd=parity.ROOT)
    r = json.loads(p.stdout.strip().splitlines()[-1])
    assert p.returncode == 0 and r["ok"], (p.stderr[-2000:], r)
