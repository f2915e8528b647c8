"""The parity driver (tests/parity.py) on the CPU: its verdict rule against the
cases the reference documents for it (src/STADE.jl:18915-18932), and whole
runs in which the oracle stands in for the device, with mistakes planted in
the oracle's output."""
import json
import subprocess
import sys

import numpy as np
import pytest

import parity


def test_verdict_rule_cases():
    # passes by the ceiling: GPU 6.3e-12 against a CPU error of 9e-14 (ratio 71)
    ok, tol = parity.verdict(9e-14, 6.3e-12, 3, True, 10, 2.5e-14)
    assert ok and tol == 1e-10
    # passes by the factor: GPU 1.5e-10 against a CPU error of 4.5e-11
    ok, tol = parity.verdict(4.5e-11, 1.5e-10, 3, True, 10, 2.5e-14)
    assert ok and tol == pytest.approx(9e-10)
    # above both is no longer rounding
    assert not parity.verdict(1e-13, 2e-10, 3, True, 10, 2.5e-14)[0]
    # a run that changed nothing is not a pass
    assert not parity.verdict(0.0, 0.0, 3, True, 0, 2.5e-14)[0]
    # no truth run: the GPU-vs-CPU check decides
    assert not parity.verdict(0.0, 0.0, 0, False, 10, 2.5e-14)[0]
    assert parity.verdict(0.0, 0.0, 0, True, 10, 2.5e-14)[0]


def test_relerr_matches_generated_helpers():
    a = np.array([0.5, 200.0, -3.0])
    b = np.array([0.5 + 1e-9, 200.0 * (1 + 1e-9), -3.0])
    assert parity.relerr_arr(a, b) == pytest.approx(1e-9, rel=1e-6)   # |a| < 1: absolute
    assert parity.relerr_arr(np.zeros(0), np.zeros(0)) == 0.0        # empty compares nothing
    assert parity.relerr_scalar(2.0, 2.0 + 2e-12) == pytest.approx(1e-12, rel=1e-6)


def _self(kern, mutate=None):
    def run(st, ints, sc):
        r = kern.cpu(st, ints, sc, False)
        if mutate:
            mutate(st)
        return r
    return run


@pytest.mark.parametrize("name", ["affine_ls_b", "heat2d_b", "conv1d_relu_mse_b", "heat2d_d"])
def test_oracle_as_device_passes(name):
    k = parity.KERNELS[name]
    r = parity.run(k, dict(k.defaults), trials=2, gpu=_self(k), device="cpu")
    assert r["ok"] and not r["vacuous"] and r["max_rel_err"] == 0.0
    assert r["truth_trials"] == 2 and r["tr_gpu"] == r["tr_cpu"]
    assert r["elements_changed"] > 0
    if k.stack:
        assert r["stacks_compared"] == 2 and r["stack_max_rel_err"] == 0.0


def test_planted_gradient_error_fails():
    k = parity.KERNELS["affine_ls_b"]

    def bump(st):
        st["wb"][5] += 1e-8 * max(1.0, abs(st["wb"][5]))
    r = parity.run(k, dict(k.defaults), trials=2, gpu=_self(k, bump), device="cpu")
    assert not r["ok"]
    assert r["tr_gpu"] == pytest.approx(1e-8, rel=1e-3) and r["max_rel_err"] > 1e-9


def test_planted_scalar_return_error_fails():
    k = parity.KERNELS["heat2d_b"]

    def run(st, ints, sc):
        return [v + 1e-7 for v in k.cpu(st, ints, sc, False)]
    r = parity.run(k, dict(k.defaults), trials=1, gpu=run, device="cpu")
    assert not r["ok"]


def test_planted_stack_error_is_reported_not_failed():
    k = parity.KERNELS["heat2d_b"]

    def bump(st):
        st["u_stack"][7] += 0.5
    r = parity.run(k, dict(k.defaults), trials=1, gpu=_self(k, bump), device="cpu")
    assert r["ok"] and r["stack_max_rel_err"] > 0.1


def test_float32_floor_and_kink_count():
    k = parity.KERNELS["conv1d_relu_mse_b"]

    def bump(st):
        st["wb"][0] += 5e-4 * max(1.0, abs(st["wb"][0]))
    r = parity.run(k, dict(k.defaults), trials=1, gpu=_self(k, bump), device="cpu")
    assert not r["ok"] and r["tr_tol"] >= parity.TOL_F32 and r["kinks"] == 0


def test_zero_trip_run_is_vacuous():
    k = parity.KERNELS["affine_ls_d"]
    r = parity.run(k, dict(n_s=0, n_o=0, n_i=0), trials=1, gpu=_self(k), device="cpu")
    assert r["vacuous"] and not r["ok"]


def test_seeds_fresh_per_trial_baseline_shared():
    k = parity.KERNELS["mlp2_ce_b"]
    ints = dict(n_s=4, n_i=6, n_h=5, n_o=3)
    base, seeds = parity.make_trials(k, ints, 3)
    base2, seeds2 = parity.make_trials(k, ints, 3)
    assert all(np.array_equal(base[a], base2[a]) for a in base)              # reproducible
    assert not np.array_equal(seeds[0]["w1b"], seeds[1]["w1b"])               # fresh per trial
    assert set(seeds[0]) == {a for a in k.args if a not in k.primal}
    assert base["x"].dtype == np.float32 and seeds[0]["lossb"].dtype == np.float32


def test_cli_prints_one_json_line():
    # --kernel with an unknown size name is refused before anything runs
    p = subprocess.run([sys.executable, parity.__file__, "--kernel", "affine_ls_b", "--size",
                        "n_q=3"], capture_output=True, text=True)
    assert p.returncode != 0 and "no integer argument n_q" in p.stderr
    out = subprocess.run([sys.executable, "-c",
                          "import sys; sys.argv[0] = 'parity'; sys.path.insert(0, 'tests');"
                          "import parity, json;"
                          "k = parity.KERNELS['affine_ls_b'];"
                          "r = parity.run(k, dict(n_s=8, n_o=3, n_i=2), 1,"
                          " gpu=lambda st, i, sc: k.cpu(st, i, sc, False), device='cpu');"
                          "print(json.dumps(r))"],
                         capture_output=True, text=True, cwd=parity.ROOT)
    line = out.stdout.strip().splitlines()[-1]
    r = json.loads(line)
    for key in ("ok", "mode", "max_rel_err", "truth_trials", "tr_cpu", "tr_gpu", "tr_tol",
                "tr_trials", "stack_max_rel_err", "stacks_compared", "elements_compared",
                "elements_changed", "vacuous", "device"):
        assert key in r, key
    assert r["ok"] and r["mode"] == "adjoint"
