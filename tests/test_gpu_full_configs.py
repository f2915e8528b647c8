"""Element-wise parity at the full BASELINE configuration sizes.

Each configuration runs once on the B200 through the C ABI on exactly the
bench's inputs (seeded synthetic data, zero shadows, lossb = 1), and every
output array is compared element by element with the CPU oracle on the same
inputs: the sweep in the kernel's own precision (what the generated Julia
computes on the CPU) and the same sweep at higher precision (Float64 for the
Float32 sweeps, 80-bit long double for the Float64 HVP) as the exact result.
The oracle runs with its summed shadows split over host threads in sample
blocks (oracle.cc over_sample_blocks; C3's parallel sweep is bit-identical
to the serial one).

Metrics per array (refmath):
  elem(phi)  max_i |a_i - b_i| / max(|b_i|, phi * max_j |b_j|), phi = 1e-3:
             element-wise relative error with a floor at 1e-3 of the array's
             largest magnitude (the floor keeps cancelled sums, whose exact
             value is far below their terms, from dividing rounding noise by
             nothing); also recorded at phi = 1e-2 and 0;
  ref        the reference's own element-wise form, |a - b| / max(|a|, |b|, 1)
             (src/STADE.jl:18980);
  norm       max|a - b| / max|b|.
Gate per array, with tol = 1e-5 (Float32) or 1e-12 (Float64), the north
star's tolerances:
  elem(1e-3)(gpu, exact) <= max(tol, 20 * elem(1e-3)(cpu, exact)), and
  norm(gpu, exact) <= tol,
where cpu is the oracle in the kernel's precision (the generated sweep as the
reference runs it on the CPU). A Float32 evaluation cannot hold 1e-5
element-wise at elements far below the array's largest: the CPU sweep itself
misses it (tanh outputs near zero, sums with cancellation), so the GPU is
judged by the reference's own GPU verdict (val_truth_verdict_lines,
src/STADE.jl:18915-18932: worst GPU error at most 20 times the worst CPU
error against the exact result) without its 1e-10 ceiling, element-wise.
Measured on the B200 at the full sizes: the per-sample outputs are within
1.6x of the CPU's own error; C2's sums over 65,536 samples (w1b, b1b, w2b,
b2b) within 18x, from the tensor core's Float32 accumulation, which
truncates toward zero and so shifts every sample of a hidden unit the same
way (halved by chains of two K blocks, at +0.11 ms per grad-eval).
Where the sweep has no higher-precision truth
here (C1, C3 in Float64) the GPU is compared with the Float64 oracle at tol
directly. Set STADE_PARITY_RECORD to a path to also write every figure as
JSON.
"""
import json
import os

import numpy as np
import pytest

import cases
from refmath import elem_rel_err, ref_rel_err, rel_err

pytestmark = pytest.mark.gpu

F32_TOL = 1e-5
F64_TOL = 1e-12
CPU_FACTOR = 20.0    # the reference's verdict (val_truth_verdict_lines)
PHI = 1e-3
THREADS = 0          # the oracle on every host thread
RECORD = {}


def _metrics(a, b):
    return {"elem_1e-3": elem_rel_err(a, b, 1e-3), "elem_1e-2": elem_rel_err(a, b, 1e-2),
            "elem_0": elem_rel_err(a, b, 0.0), "ref": ref_rel_err(a, b), "norm": rel_err(a, b)}


def _record(config, name, **pairs):
    RECORD.setdefault(config, {})[name] = {k: _metrics(a, b) for k, (a, b) in pairs.items()}
    return RECORD[config][name]


def _check(fails, config, name, gate, tol, cpu=None, **pairs):
    """Records every pair's metrics; notes a failure when pair `gate` (the
    GPU against the exact result) misses the gate above, with pair `cpu` (the
    same-precision oracle against the exact result) as the CPU's own error.
    The caller asserts once all arrays are recorded."""
    m = _record(config, name, **pairs)
    bound = max(tol, CPU_FACTOR * m[cpu]["elem_1e-3"]) if cpu else tol
    if not (m[gate]["elem_1e-3"] <= bound and m[gate]["norm"] <= tol):
        fails.append((name, m[gate], m[cpu] if cpu else None))


@pytest.fixture(scope="module", autouse=True)
def _write_record():
    yield
    path = os.environ.get("STADE_PARITY_RECORD")
    if path and RECORD:
        with open(path, "w") as f:
            json.dump(RECORD, f, indent=1)


def _oracle_mlp(st, ints):
    from oracle import oracle as orc
    orc.mlp2_ce_b(*[st[a] for a in cases.MLP_ARGS], ints["n_s"], ints["n_i"], ints["n_h"],
                  ints["n_o"], threads=THREADS)


def test_c1_affine_ls_full():
    """C1 at 1024 x 64 x 32: y, xb, tb bit for bit (same operation order),
    wb, bb, loss within 1e-12 element-wise."""
    st, ints = cases.affine_state(1024, 64, 32)
    ref, out = cases.copy_state(st), cases.copy_state(st)
    cases.oracle_affine(ref, ints)
    cases.gpu_affine(out, ints)
    for k in ("y", "xb", "tb"):
        assert np.array_equal(out[k], ref[k]), k
    fails = []
    for k in ("wb", "bb", "loss", "y", "xb", "tb"):
        _check(fails, "C1", k, "gpu_vs_f64", F64_TOL, gpu_vs_f64=(out[k], ref[k]))
    assert not fails, fails


def test_c2_mlp2_ce_full():
    """C2 at 65,536 x 784 x 512 x 10, Float32, against the exact result
    (the sweep in Float64) with the Float32 oracle's own error as the CPU's."""
    st, ints = cases.mlp_state(65536, 784, 512, 10)
    out = cases.copy_state(st)
    cases.gpu_mlp(out, ints)
    ref = cases.copy_state(st)
    _oracle_mlp(ref, ints)
    truth = cases.OrderedDict((k, v.astype(np.float64)) for k, v in st.items())
    _oracle_mlp(truth, ints)
    for k in ("hb", "zb", "pb"):
        assert not np.any(out[k]), k
    fails = []
    for k in ("h", "z", "p", "yb", "xb", "w1b", "b1b", "w2b", "b2b", "loss"):
        _check(fails, "C2", k, "gpu_vs_f64", F32_TOL, "f32_oracle_vs_f64",
               gpu_vs_f64=(out[k], truth[k]),
               f32_oracle_vs_f64=(ref[k], truth[k]), gpu_vs_f32_oracle=(out[k], ref[k]))
    assert not fails, fails


def test_c3_heat2d_full():
    """C3 at 8192^2 x 16 steps, Float64: the 8 GiB tape and the restored
    field bit for bit, ub / alphab / loss within 1e-12 element-wise."""
    from oracle import oracle as orc
    n, n_step = 8192, 16
    st, ints = cases.heat_state(n, n_step)
    out = cases.copy_state(st)
    a_gpu = cases.gpu_heat(out, ints)
    ref = cases.copy_state(st)
    del st
    a_ref = orc.heat2d_b(*[ref[k] for k in cases.HEAT_ARGS], ints["alpha"], ints["alphab"], n,
                         n_step, ref["u_stack"], threads=THREADS)
    assert np.array_equal(out["u_stack"], ref["u_stack"])
    assert np.array_equal(out["u"], ref["u"])
    out.pop("u_stack"), ref.pop("u_stack")
    fails = []
    for k in ("ub", "un", "loss"):
        _check(fails, "C3", k, "gpu_vs_f64", F64_TOL, gpu_vs_f64=(out[k], ref[k]))
    _check(fails, "C3", "alphab", "gpu_vs_f64", F64_TOL,
           gpu_vs_f64=(np.array([a_gpu]), np.array([a_ref])))
    assert not fails, fails
    assert not np.any(out["unb"])


def test_c4_conv1d_relu_mse_512_samples():
    """C4 at full channels, length and taps with 512 samples (the weight
    gradient sums 512 x 2040 = 1.04 M terms per element), Float32, against
    the sweep in Float64 moved to the ReLU branch the GPU took where the exact
    pre-activation lies within Float32 rounding of the kink (those must be
    rare), with the Float32 oracle's own error as the CPU's."""
    from oracle import oracle as orc
    n_b, n_c, n_l, n_o, n_k = 512, 64, 2048, 128, 9
    st, ints = cases.conv_state(n_b, n_c, n_l, n_o, n_k)
    out = cases.copy_state(st)
    cases.gpu_conv(out, ints)
    ref = cases.copy_state(st)
    orc.conv1d_relu_mse_b(*[ref[a] for a in cases.CONV_ARGS], n_b, n_c, n_l, n_o, n_k,
                          threads=THREADS)
    truth = cases.OrderedDict((k, v.astype(np.float64)) for k, v in st.items())
    orc.conv1d_relu_mse_b(*[truth[a] for a in cases.CONV_ARGS], n_b, n_c, n_l, n_o, n_k,
                          threads=THREADS)
    adj, flips = cases.conv_kink_adjust(st, truth, out, ints)
    RECORD.setdefault("C4", {})["kink_flips"] = int(flips)
    assert flips <= 1e-4 * out["z"].size
    for k in ("zb", "rb"):
        assert not np.any(out[k]), k
    fails = []
    for k in ("z", "r", "tb", "xb", "wb", "loss"):
        _check(fails, "C4", k, "gpu_vs_f64", F32_TOL, "f32_oracle_vs_f64",
               gpu_vs_f64=(out[k], adj[k]),
               f32_oracle_vs_f64=(ref[k], truth[k]), gpu_vs_f32_oracle=(out[k], ref[k]))
    assert not fails, fails


def test_c5_mlp2_ce_hv_full():
    """C5 at 16,384 samples, Float64: every HVP output (the *bd shadows) and
    adjoint against the 80-bit long-double sweep, with the Float64 oracle's
    own error as the CPU's."""
    from oracle import oracle as orc
    st, ints = cases.mlp_hv_state(16384, 784, 512, 10)
    out = cases.copy_state(st)
    cases.gpu_mlp_hv(out, ints)
    dims = (ints["n_s"], ints["n_i"], ints["n_h"], ints["n_o"])
    ref = cases.copy_state(st)
    orc.mlp2_ce_hv(*[ref[a] for a in cases.MLP_ARGS], *dims, *[ref[a] for a in cases.MLP_TAN],
                   threads=THREADS)
    truth = cases.copy_state(st)
    orc.mlp2_ce_hv(*[truth[a] for a in cases.MLP_ARGS], *dims, *[truth[a] for a in cases.MLP_TAN],
                   threads=THREADS, truth=True)
    for k in ("hb", "zb", "pb", "hbd", "zbd", "pbd"):
        assert not np.any(out[k]), k
    fails = []
    for k in ("w1bd", "b1bd", "w2bd", "b2bd", "lossd", "xbd", "ybd", "w1b", "b1b", "w2b", "b2b",
              "loss", "xb", "yb", "h", "hd", "z", "zd", "p", "pd"):
        _check(fails, "C5", k, "gpu_vs_truth", F64_TOL, "f64_oracle_vs_truth",
               gpu_vs_truth=(out[k], truth[k]),
               f64_oracle_vs_truth=(ref[k], truth[k]), gpu_vs_f64_oracle=(out[k], ref[k]))
    assert not fails, fails
