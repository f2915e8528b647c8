"""Run one sweep of libstade_b200 on seeded synthetic inputs of a chosen size.

Meant for profiling one kernel at a controlled size (for example under ncu)
and for quick timing; it checks nothing.

    python tests/run_case.py heat2d --n 4096 --n-step 4 --repeat 2
    python tests/run_case.py mlp2_ce --n-s 8192
    python tests/run_case.py mlp2_ce_hv --n-s 2048
    python tests/run_case.py conv1d_relu_mse --n-b 64
    python tests/run_case.py affine_ls

(a profiling driver kept beside the tests; pytest does not collect it)
"""
from __future__ import annotations

import argparse
import os
import sys

import torch

sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                "stade.jl_b200"))
from stadeb200 import kernels, synth  # noqa: E402


def _dev(d):
    return {k: torch.from_numpy(v).cuda() for k, v in d.items()}


def _zeros(n, dt):
    return torch.zeros(n, dtype=dt, device="cuda")


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("config", choices=list(synth.FULL))
    ap.add_argument("--repeat", type=int, default=1)
    ap.add_argument("--n", type=int)
    ap.add_argument("--n-step", type=int)
    ap.add_argument("--n-s", type=int)
    ap.add_argument("--n-b", type=int)
    ap.add_argument("--n-l", type=int)
    a = ap.parse_args(argv)
    c = dict(synth.FULL[a.config])
    for key in ("n", "n_step", "n_s", "n_b", "n_l"):
        v = getattr(a, key)
        if v is not None:
            c[key] = v
    f32, f64 = torch.float32, torch.float64
    if a.config == "heat2d":
        n, ns = c["n"], c["n_step"]
        t = _dev(synth.heat2d_inputs(n))
        stack = kernels.initstacks_heat2d_b_cuda(n, ns)
        run = lambda: kernels.heat2d_b_cuda(_zeros(1, f64), t["lossb"], t["u"], _zeros(n * n, f64),
                                            _zeros(n * n, f64), _zeros(n * n, f64), c["alpha"], 0.0,
                                            n, ns, stack)
    elif a.config in ("mlp2_ce", "mlp2_ce_hv"):
        S, I, H, O = c["n_s"], c["n_i"], c["n_h"], c["n_o"]
        if a.config == "mlp2_ce":
            t = _dev(synth.mlp2_ce_inputs(S, I, H, O))
            z = lambda n: _zeros(n, f32)
            run = lambda: kernels.mlp2_ce_b_cuda(
                z(1), t["lossb"], t["x"], z(S * I), t["y"], z(S * O), t["w1"], z(I * H), t["b1"],
                z(H), t["w2"], z(H * O), t["b2"], z(O), z(S * H), z(S * H), z(S * O), z(S * O),
                z(S * O), z(S * O), S, I, H, O)
        else:
            t = _dev(synth.mlp2_ce_hv_inputs(S, I, H, O))
            z = lambda n: _zeros(n, f64)
            def run():
                args = []
                for name in kernels.MLP_HV_ARGS:
                    args.append(t[name] if name in t else z(kernels._mlp_len(name, S, I, H, O)))
                tans = []
                for name in kernels.MLP_HV_TAN:
                    tans.append(t[name] if name in t else z(kernels._mlp_len(name, S, I, H, O)))
                kernels.mlp2_ce_hv_cuda(*args, S, I, H, O, *tans)
    elif a.config == "conv1d_relu_mse":
        B, Cc, L, O, K = c["n_b"], c["n_c"], c["n_l"], c["n_o"], c["n_k"]
        t = _dev(synth.conv1d_relu_mse_inputs(B, Cc, L, O, K))
        nt = B * O * (L - K + 1)
        z = lambda n: _zeros(n, f32)
        run = lambda: kernels.conv1d_relu_mse_b_cuda(
            z(1), t["lossb"], t["x"], z(B * Cc * L), t["w"], z(O * Cc * K), t["t"], z(nt), z(nt),
            z(nt), z(nt), z(nt), B, Cc, L, O, K)
    else:
        S, O, I = c["n_s"], c["n_o"], c["n_i"]
        t = _dev(synth.affine_ls_inputs(S, O, I))
        z = lambda n: _zeros(n, f64)
        run = lambda: kernels.affine_ls_b_cuda(z(1), t["lossb"], t["w"], z(O * I), t["b"], z(O),
                                               t["x"], z(S * I), t["t"], z(S * O), z(S * O),
                                               z(S * O), S, O, I)
    for i in range(a.repeat):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        run()
        e1.record()
        torch.cuda.synchronize()
        print(f"{a.config} {c} call {i}: {e0.elapsed_time(e1):.3f} ms")


if __name__ == "__main__":
    main()
