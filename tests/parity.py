"""TEST INFRASTRUCTURE: the GPU parity driver, a restatement of the script
STADE.jl writes to validate a generated GPU sweep (val_gpu_parity_script,
src/STADE.jl:18939-19175; driver stade_validate_gpu_file,
src/STADE.jl:19186-19240), run against libstade_b200 through its C ABI.

Per kernel and mode, for each of `trials` seeded draws:
  - the primal values are one shared baseline (the synthetic inputs; every
    float array the inputs do not supply, intermediates and `loss` included,
    is drawn once at random, as the reference's baseline YAML holds a value
    for every argument); every shadow (adjoint seed, or the HVP's two
    directions) is a fresh N(0, 1) draw per trial (val_random_values_like,
    src/STADE.jl:16880-16891);
  - the CPU oracle (the generated code's arithmetic in the kernel's own type)
    and the GPU sweep run on copies; stacks are zero-filled first on both
    sides (_val_init_stacks_local, src/STADE.jl:18968);
  - the same oracle code runs in long double (x87, 64-bit significand) on the
    same inputs as the truth, in place of the reference's 192-bit BigFloat;
  - every float array (primal value and shadow; HVP tangents too) and every
    returned scalar is compared element-wise with
    |a - b| / max(|a|, |b|, 1) (_relerr_arr, src/STADE.jl:18976).

Verdict (val_truth_verdict_lines, src/STADE.jl:18925-18932):
    tr_tol = max(rtol, truth_factor * tr_cpu_worst, truth_ceiling)
    ok     = tr_gpu_worst <= tr_tol  and  elements_changed > 0
with rtol = 2.5e-14, truth_factor = 20, truth_ceiling = 1e-10 for Float64
sweeps (the reference's defaults). The reference generates Float64 code only;
for the Float32 sweeps the floor and the ceiling are the Float32 tolerance,
1e-5. `elements_changed` counts the CPU elements the call changed, so a run
that executed nothing is `vacuous`, never `ok` (src/STADE.jl:19035-19040).
The tape (heat2d's u_stack) is compared GPU against CPU and reported as
`stack_max_rel_err`, beside the verdict, as the reference reports it.

C4's ReLU has a kink at z = 0; where a Float32 pre-activation lies within
rounding of 0, the branch a sweep took may differ from the exact one. Its
error there is judged against the exact adjoint of the branch that sweep took
(tests/cases.py, conv_kink_adjust), separately for the CPU and the GPU run,
and the number of such elements is reported as `kinks`.

Usage: python tests/parity.py --kernel mlp2_ce_b [--trials 3] [--size n_s=256 ...]
Prints one JSON line and exits 0 when `ok`, 1 otherwise.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from collections import OrderedDict

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for _p in (HERE, ROOT, os.path.join(ROOT, "stade.jl_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import cases  # noqa: E402
from oracle import oracle as orc  # noqa: E402
from stadeb200 import synth  # noqa: E402

RTOL_F64, TRUTH_CEILING_F64, TRUTH_FACTOR = 2.5e-14, 1.0e-10, 20.0
TOL_F32 = 1.0e-5


# ---- element-wise errors, as the generated script computes them ----------------
def relerr_arr(a, b) -> float:
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    if a.size == 0:
        return 0.0
    return float(np.max(np.abs(a - b) / np.maximum(np.maximum(np.abs(a), np.abs(b)), 1.0)))


def relerr_scalar(a, b) -> float:
    return abs(a - b) / max(abs(a), abs(b), 1.0)


def verdict(tr_cpu_worst, tr_gpu_worst, truth_trials, local_ok, elements_changed, rtol,
            truth_factor=TRUTH_FACTOR, truth_ceiling=TRUTH_CEILING_F64):
    """(ok, tr_tol). `local_ok` is the GPU-vs-CPU check of the trials that had
    no truth run (all of them pass it vacuously when every trial had one)."""
    tr_tol = max(rtol, truth_factor * tr_cpu_worst, truth_ceiling)
    ok = local_ok and (truth_trials == 0 or tr_gpu_worst <= tr_tol)
    return ok and elements_changed > 0, tr_tol


# ---- kernels: generated argument order, shapes, runners ---------------------------
def _np_to_dev(st):
    import torch
    return OrderedDict((k, torch.from_numpy(np.ascontiguousarray(v)).cuda()) for k, v in st.items())


def _dev_back(dev, st):
    for k, v in dev.items():
        st[k] = v.cpu().numpy()


class Kernel:
    """One generated sweep. `args`: its float arrays in signature order;
    `primal`: those that are primal values (the rest are shadows, drawn per
    trial); `scalar`: (primal name, value, shadow name) of a float scalar
    argument, whose shadow the sweep returns; `stack`: the tape array."""

    def __init__(self, name, mode, dtype, args, primal, shapes, inputs, cpu, gpu, defaults,
                 scalar=None, stack=None, kink=False):
        self.name, self.mode, self.dtype = name, mode, dtype
        self.args, self.primal, self.shapes, self.inputs = args, primal, shapes, inputs
        self.cpu, self.gpu, self.defaults = cpu, gpu, defaults
        self.scalar, self.stack, self.kink = scalar, stack, kink


def _affine_shapes(i):
    n_s, n_o, n_i = i["n_s"], i["n_o"], i["n_i"]
    return dict(loss=1, w=n_o * n_i, b=n_o, x=n_s * n_i, t=n_s * n_o, y=n_s * n_o)


def _mlp_shapes(i):
    n_s, n_i, n_h, n_o = i["n_s"], i["n_i"], i["n_h"], i["n_o"]
    return dict(loss=1, x=n_s * n_i, y=n_s * n_o, w1=n_i * n_h, b1=n_h, w2=n_h * n_o, b2=n_o,
                h=n_s * n_h, z=n_s * n_o, p=n_s * n_o)


def _heat_shapes(i):
    return dict(loss=1, u=i["n"] ** 2, un=i["n"] ** 2)


def _conv_shapes(i):
    n_lo = i["n_l"] - i["n_k"] + 1
    return dict(loss=1, x=i["n_b"] * i["n_c"] * i["n_l"], w=i["n_o"] * i["n_c"] * i["n_k"],
                t=i["n_b"] * i["n_o"] * n_lo, z=i["n_b"] * i["n_o"] * n_lo,
                r=i["n_b"] * i["n_o"] * n_lo)


def _ints(i, keys):
    return [i[k] for k in keys]


AFF_I, MLP_I, CONV_I = ("n_s", "n_o", "n_i"), ("n_s", "n_i", "n_h", "n_o"), \
    ("n_b", "n_c", "n_l", "n_o", "n_k")
HEAT_I = ("n", "n_step")
MLP_D = ["loss", "lossd", "x", "xd", "y", "yd", "w1", "w1d", "b1", "b1d", "w2", "w2d", "b2",
         "b2d", "h", "hd", "z", "zd", "p", "pd"]
AFF_D = ["loss", "lossd", "w", "wd", "b", "bd", "x", "xd", "t", "td", "y", "yd"]
HEAT_D = ["loss", "lossd", "u", "ud", "un", "und"]
CONV_D = ["loss", "lossd", "x", "xd", "w", "wd", "t", "td", "z", "zd", "r", "rd"]
MLP_PRIMAL = ["loss", "x", "y", "w1", "b1", "w2", "b2", "h", "z", "p"]


def _cpu_call(fn, args, keys, scalars=(), tail=()):
    """The oracle in the generated positional order: float arrays, float
    scalars, integer sizes, then `tail` arrays (HVP tangents, the tape)."""
    def run(st, i, sc, truth):
        r = fn(*[st[a] for a in args], *[sc[k] for k in scalars], *_ints(i, keys),
               *[st[a] for a in tail], truth=truth)
        return [] if r is None else [float(r)]
    return run


def _gpu_call(fn_name, args, keys, scalars=(), tail=()):
    """The same call through libstade_b200's C ABI on device copies."""
    def run(st, i, sc):
        import stadeb200
        dev = _np_to_dev(st)
        r = getattr(stadeb200, fn_name)(*[dev[a] for a in args], *[sc[k] for k in scalars],
                                        *_ints(i, keys), *[dev[a] for a in tail])
        _dev_back(dev, st)
        return [] if r is None else [float(r)]
    return run


def _build_kernels():
    K = {}
    A, M, H, C = cases.AFFINE_ARGS, cases.MLP_ARGS, cases.HEAT_ARGS, cases.CONV_ARGS
    # C1 affine least squares, adjoint (Float64)
    K["affine_ls_b"] = Kernel(
        "affine_ls_b", "adjoint", np.float64, A, ["loss", "w", "b", "x", "t", "y"],
        _affine_shapes, lambda i: synth.affine_ls_inputs(*_ints(i, AFF_I)),
        _cpu_call(orc.affine_ls_b, A, AFF_I), _gpu_call("affine_ls_b_cuda", A, AFF_I),
        dict(n_s=1024, n_o=64, n_i=32))
    # C2 two-layer MLP, softmax cross-entropy, adjoint (Float32)
    K["mlp2_ce_b"] = Kernel(
        "mlp2_ce_b", "adjoint", np.float32, M, MLP_PRIMAL, _mlp_shapes,
        lambda i: synth.mlp2_ce_inputs(*_ints(i, MLP_I), np.float32),
        _cpu_call(orc.mlp2_ce_b, M, MLP_I), _gpu_call("mlp2_ce_b_cuda", M, MLP_I),
        dict(n_s=256, n_i=784, n_h=512, n_o=10))
    # C3 periodic heat equation, adjoint with a tape; returns alpha's adjoint (Float64)
    K["heat2d_b"] = Kernel(
        "heat2d_b", "adjoint", np.float64, H, ["loss", "u", "un"], _heat_shapes,
        lambda i: synth.heat2d_inputs(i["n"]),
        _cpu_call(orc.heat2d_b, H, HEAT_I, ("alpha", "alphab"), ("u_stack",)),
        _gpu_call("heat2d_b_cuda", H, HEAT_I, ("alpha", "alphab"), ("u_stack",)),
        dict(n=192, n_step=16), scalar=("alpha", 0.2, "alphab"), stack="u_stack")
    # C4 conv1d + ReLU + MSE, adjoint (Float32)
    K["conv1d_relu_mse_b"] = Kernel(
        "conv1d_relu_mse_b", "adjoint", np.float32, C, ["loss", "x", "w", "t", "z", "r"],
        _conv_shapes, lambda i: synth.conv1d_relu_mse_inputs(*_ints(i, CONV_I)),
        _cpu_call(orc.conv1d_relu_mse_b, C, CONV_I),
        _gpu_call("conv1d_relu_mse_b_cuda", C, CONV_I),
        dict(n_b=4, n_c=16, n_l=256, n_o=32, n_k=9), kink=True)
    # C5 HVP of C2 (Float64): tangents of the primals and of the adjoint seeds
    K["mlp2_ce_hv"] = Kernel(
        "mlp2_ce_hv", "hvp", np.float64, M + cases.MLP_TAN, MLP_PRIMAL, _mlp_shapes,
        lambda i: {k: v for k, v in synth.mlp2_ce_hv_inputs(*_ints(i, MLP_I)).items()
                   if k in MLP_PRIMAL},
        _cpu_call(orc.mlp2_ce_hv, M, MLP_I, tail=cases.MLP_TAN),
        _gpu_call("mlp2_ce_hv_cuda", M, MLP_I, tail=cases.MLP_TAN),
        dict(n_s=128, n_i=784, n_h=512, n_o=10))
    # Tangent sweeps <k>_d (forward mode). The reference script validates the
    # adjoint and the HVP; the same comparison applies unchanged.
    K["affine_ls_d"] = Kernel(
        "affine_ls_d", "tangent", np.float64, AFF_D, ["loss", "w", "b", "x", "t", "y"],
        _affine_shapes, lambda i: synth.affine_ls_inputs(*_ints(i, AFF_I)),
        _cpu_call(orc.affine_ls_d, AFF_D, AFF_I), _gpu_call("affine_ls_d_cuda", AFF_D, AFF_I),
        dict(n_s=1024, n_o=64, n_i=32))
    for dt, tag in ((np.float32, "f32"), (np.float64, "f64")):
        K[f"mlp2_ce_d_{tag}"] = Kernel(
            f"mlp2_ce_d_{tag}", "tangent", dt, MLP_D, MLP_PRIMAL, _mlp_shapes,
            lambda i, dt=dt: synth.mlp2_ce_inputs(*_ints(i, MLP_I), dt),
            _cpu_call(orc.mlp2_ce_d, MLP_D, MLP_I), _gpu_call("mlp2_ce_d_cuda", MLP_D, MLP_I),
            dict(n_s=256, n_i=784, n_h=512, n_o=10))
    K["heat2d_d"] = Kernel(
        "heat2d_d", "tangent", np.float64, HEAT_D, ["loss", "u", "un"], _heat_shapes,
        lambda i: synth.heat2d_inputs(i["n"]),
        _cpu_call(orc.heat2d_d, HEAT_D, HEAT_I, ("alpha", "alphad")),
        _gpu_call("heat2d_d_cuda", HEAT_D, HEAT_I, ("alpha", "alphad")),
        dict(n=192, n_step=16), scalar=("alpha", 0.2, "alphad"))
    K["conv1d_relu_mse_d"] = Kernel(
        "conv1d_relu_mse_d", "tangent", np.float32, CONV_D, ["loss", "x", "w", "t", "z", "r"],
        _conv_shapes, lambda i: synth.conv1d_relu_mse_inputs(*_ints(i, CONV_I)),
        _cpu_call(orc.conv1d_relu_mse_d, CONV_D, CONV_I),
        _gpu_call("conv1d_relu_mse_d_cuda", CONV_D, CONV_I),
        dict(n_b=4, n_c=16, n_l=256, n_o=32, n_k=9), kink=True)
    return K


KERNELS = _build_kernels()


def _base_of(name, kern: Kernel, ints):
    """The primal that a float array shadows ('w1b' -> 'w1', 'w1bd' -> 'w1b'
    -> 'w1', 'lossb' -> 'loss')."""
    shapes = kern.shapes(ints)
    s = name
    while s not in shapes:
        s = s[:-1]
    return s


def make_trials(kern: Kernel, ints, trials, seed_tag="parity"):
    """(baseline, [per-trial seeds]) as numpy dicts in the kernel's dtype."""
    dt = kern.dtype
    shapes = kern.shapes(ints)
    tag = f"{kern.name}:" + ",".join(f"{k}={v}" for k, v in sorted(ints.items()))
    rng = np.random.default_rng(int(synth.seed(seed_tag, tag)) % (2 ** 63))
    given = kern.inputs(ints)
    base = OrderedDict()
    for a in kern.primal:
        if a in given and np.asarray(given[a]).size == shapes[a]:
            base[a] = np.asarray(given[a]).astype(dt).copy()
        else:
            base[a] = rng.standard_normal(shapes[a]).astype(dt)
    seeds = []
    for _ in range(trials):
        sd = OrderedDict()
        for a in kern.args:
            if a not in kern.primal:
                sd[a] = rng.standard_normal(shapes[_base_of(a, kern, ints)]).astype(dt)
        if kern.scalar:
            sd[kern.scalar[2]] = float(rng.standard_normal())
        seeds.append(sd)
    return base, seeds


def _state(kern, ints, base, seed):
    st = OrderedDict()
    for a in kern.args:
        st[a] = (base[a] if a in base else seed[a]).copy()
    if kern.stack:
        st[kern.stack] = np.zeros(max(ints["n_step"] * ints["n"] ** 2, 1), kern.dtype)
    sc = {}
    if kern.scalar:
        sc[kern.scalar[0]] = kern.scalar[1]
        sc[kern.scalar[2]] = seed[kern.scalar[2]]
    return st, sc


def _float_arrays(kern, st):
    return [a for a in kern.args if a != kern.stack]


def _kink_truth(kern, pre, truth, out, ints):
    """Exact adjoint of the ReLU branch `out` took (adjoint conv only)."""
    if not kern.kink or kern.mode != "adjoint":
        return truth, 0
    adj, n = cases.conv_kink_adjust(pre, truth, out, ints)
    return adj, n


def run(kern: Kernel, ints, trials=3, gpu=None, device=None):
    gpu = gpu or kern.gpu
    f32 = kern.dtype == np.float32
    rtol = TOL_F32 if f32 else RTOL_F64
    ceiling = TOL_F32 if f32 else TRUTH_CEILING_F64
    base, seeds = make_trials(kern, ints, trials)
    all_ok = True
    tr_cpu_worst = tr_gpu_worst = 0.0
    truth_trials = 0
    tr_pairs = []
    max_rel = stack_rel = 0.0
    stacks_compared = elements_compared = elements_changed = kinks = 0
    worst = ("", 0.0)
    for seed in seeds:
        st0, sc = _state(kern, ints, base, seed)
        cpu = cases.copy_state(st0)
        gpu_st = cases.copy_state(st0)
        ret_cpu = kern.cpu(cpu, ints, sc, False) or []
        big = None
        try:
            big = OrderedDict((k, v.astype(np.float64)) for k, v in st0.items())
            ret_big = kern.cpu(big, ints, sc, True) or []
        except Exception:  # the truth run is optional, as the reference's BigFloat run is
            big = None
        ret_gpu = gpu(gpu_st, ints, sc) or []
        names = _float_arrays(kern, st0)
        trc = trg = 0.0
        if big is not None:
            t_cpu, k1 = _kink_truth(kern, st0, big, cpu, ints)
            t_gpu, k2 = _kink_truth(kern, st0, big, gpu_st, ints)
            kinks += k1 + k2
            for a in names:
                trc = max(trc, relerr_arr(t_cpu[a], cpu[a]))
                e = relerr_arr(t_gpu[a], gpu_st[a])
                trg = max(trg, e)
                worst = max(worst, (a, e), key=lambda w: w[1])
            for rb, rc, rg in zip(ret_big, ret_cpu, ret_gpu):
                trc = max(trc, relerr_scalar(rb, rc))
                trg = max(trg, relerr_scalar(rb, rg))
                worst = max(worst, ("<return>", relerr_scalar(rb, rg)), key=lambda w: w[1])
        local_max = 0.0
        for a in names:
            elements_compared += cpu[a].size
            elements_changed += int(np.count_nonzero(cpu[a] != st0[a]))
            local_max = max(local_max, relerr_arr(cpu[a], gpu_st[a]))
        for rc, rg in zip(ret_cpu, ret_gpu):
            elements_compared += 1
            local_max = max(local_max, relerr_scalar(rc, rg))
        if kern.stack:
            stack_rel = max(stack_rel, relerr_arr(cpu[kern.stack], gpu_st[kern.stack]))
            stacks_compared += 1
        max_rel = max(max_rel, local_max)
        if big is None:
            all_ok = all_ok and local_max <= rtol
        else:
            tr_cpu_worst, tr_gpu_worst = max(tr_cpu_worst, trc), max(tr_gpu_worst, trg)
            truth_trials += 1
            tr_pairs.append([trc, trg])
    ok, tr_tol = verdict(tr_cpu_worst, tr_gpu_worst, truth_trials, all_ok, elements_changed,
                         rtol, TRUTH_FACTOR, ceiling)
    out = OrderedDict(ok=bool(ok), mode=kern.mode, max_rel_err=max_rel, truth_trials=truth_trials,
                      tr_cpu=tr_cpu_worst, tr_gpu=tr_gpu_worst, tr_tol=tr_tol, tr_trials=tr_pairs,
                      stack_max_rel_err=stack_rel, stacks_compared=stacks_compared,
                      elements_compared=elements_compared, elements_changed=elements_changed,
                      vacuous=elements_changed == 0, device=device or _device_name())
    out["kernel"] = kern.name
    out["tr_gpu_worst_array"] = worst[0]
    out["dtype"] = "f32" if f32 else "f64"
    out["sizes"] = dict(ints)
    if kern.kink:
        out["kinks"] = kinks
    return out


def _device_name():
    try:
        import torch
        return torch.cuda.get_device_name(0) if torch.cuda.is_available() else "cpu"
    except Exception:
        return "unknown"


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--kernel", required=True, choices=sorted(KERNELS))
    ap.add_argument("--trials", type=int, default=3)
    ap.add_argument("--size", nargs="*", default=[], help="integer arguments, e.g. n_s=512")
    a = ap.parse_args(argv)
    kern = KERNELS[a.kernel]
    ints = dict(kern.defaults)
    for kv in a.size:
        k, v = kv.split("=")
        if k not in ints:
            ap.error(f"{a.kernel} has no integer argument {k}")
        ints[k] = int(v)
    res = run(kern, ints, a.trials)
    print(json.dumps(res))
    return 0 if res["ok"] else 1


if __name__ == "__main__":
    sys.exit(main())
