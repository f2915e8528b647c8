"""Writes tests/golden/exemplars/<name>.npz: seven sweeps the reference ships
as generated text (test/val-corpus/<name>.jl), run by the interpreter
tests/jlsub.py on seeded inputs, with the reference text's sha256.

Run here, where the reference checkout exists (it does not travel to the GPU
box): python tests/golden/make_exemplar_golden.py <path to the reference>

Each fixture holds the generated argument order, the inputs ("in_<arg>"),
the outputs after the call ("out_<arg>"), the returned scalars ("ret"), and
for the B200 test the .cu emitter's manifest of that text and the name of
its sm_100a build under stade.jl_b200/_gen/ (built by this script; the build
travels with the working tree, the reference text does not).
"""
import hashlib
import json
import os
import sys
import zlib

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [os.path.dirname(HERE), os.path.join(ROOT, "stade.jl_b200")]

import jlsub  # noqa: E402

OUT = os.path.join(HERE, "exemplars")


def _rng(name):
    return np.random.default_rng(zlib.crc32(("exemplar:" + name).encode()))


def _args(name):
    """Generated positional arguments (arrays, ints, float scalars), seeded,
    with non-zero adjoint seeds so accumulation into shadows is exercised."""
    r = _rng(name)
    nrm = lambda n, s=1.0: s * r.standard_normal(n)
    a = {}
    if name == "affine_loss_b":
        n = 37
        a.update(loss=np.full(1, 0.25), lossb=np.full(1, 1.5))
        for k in ("u", "a", "b", "v"):
            a[k], a[k + "b"] = nrm(n), nrm(n, 0.1)
        a["i_n"] = n
        dims = None
    elif name == "matvec_loss_b":
        m, n = 7, 5
        a.update(loss=np.full(1, 0.5), lossb=np.full(1, 0.75), a=nrm(m * n), ab=nrm(m * n, 0.1),
                 u=nrm(n), ub=nrm(n, 0.1), v=nrm(m, 0.3), vb=nrm(m, 0.1), i_m=m, i_n=n)
        dims = {"a": ["i_m"], "ab": ["i_m"]}
    elif name == "stencil_loss_b":
        n = 29
        a.update(loss=np.full(1, 0.125), lossb=np.full(1, 2.0), u=nrm(n), ub=nrm(n, 0.1),
                 w=nrm(n), wb=nrm(n, 0.1), i_n=n)
        dims = None
    elif name == "advection_b":
        nnode, nstep = 23, 6
        a.update(u=nrm(nnode), ub=nrm(nnode), du=nrm(nnode), dub=nrm(nnode, 0.1), c=0.8, cb=0.3,
                 dx=0.05, dxb=-0.2, dt=0.01, dtb=0.7, i_nstep=nstep, i_nnode=nnode)
        dims = None
    elif name == "selfrace_conv_b":
        n, nc = 31, 5
        a.update(x=nrm(n + nc - 1), xb=nrm(n + nc - 1, 0.1), w=nrm(nc), wb=nrm(nc, 0.1),
                 z=nrm(n), zb=nrm(n, 0.1), loss=np.full(1, 0.5), lossb=np.full(1, 1.25), i_n=n,
                 i_nc=nc)
        dims = None
    elif name in ("mlp1d_b", "mlp1d_hv"):
        nh = 9
        lens = dict(loss=1, x=1, y=1, w1=nh, b1=nh, w2=nh * nh, b2=nh, w3=nh, b3=1, h1=nh, h2=nh,
                    o=1)
        for k, n in lens.items():
            a[k] = np.full(1, 0.5) if k == "loss" else nrm(n, 0.5)
            a[k + "b"] = np.full(1, 1.0) if k == "loss" else nrm(n, 0.1)
        a["n_h"] = nh
        if name == "mlp1d_hv":
            for k, n in lens.items():
                a[k + "d"] = nrm(n, 0.3)
                a[k + "bd"] = nrm(n, 0.05)
        dims = None
    else:
        raise ValueError(name)
    return a, dims


EXEMPLARS = ("affine_loss_b", "matvec_loss_b", "stencil_loss_b", "advection_b",
             "selfrace_conv_b", "mlp1d_b", "mlp1d_hv")


def main(ref_root):
    from stadeb200 import emit
    corpus = os.path.join(ref_root, "test", "val-corpus")
    os.makedirs(OUT, exist_ok=True)
    for name in EXEMPLARS:
        path = os.path.join(corpus, name + ".jl")
        with open(path) as f:
            text = f.read()
        a, dims = _args(name)
        I = jlsub.Interp(text, 64, dims)
        stacks = ()
        init = "initstacks_" + (name if name.endswith("_b") else name[:-3] + "_b")
        if init in I.funcs:
            params = I.funcs[init][0]
            stacks = I.initstacks(init, *[a[p] for p in params])
        ins = {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in a.items()}
        call = [a[p] for p in I.funcs[name][0] if p in a] + list(stacks)
        ret = I.call(name, *call)
        ret = () if ret is None else (ret if isinstance(ret, tuple) else (ret,))
        cu, man = emit.emit(text, dims=dims)
        so = emit.build(cu)
        man = {k: v for k, v in man.items() if k != "loops"}   # keeps no text of the reference
        fx = {"order": np.array(json.dumps([p for p in I.funcs[name][0] if p in a])),
              "sha256": np.array(hashlib.sha256(text.encode()).hexdigest()),
              "manifest": np.array(json.dumps(man)), "so_name": np.array(os.path.basename(so)),
              "dims": np.array(json.dumps(dims)), "ret": np.array(ret, dtype=np.float64),
              "n_stacks": np.array(len(stacks))}
        for k, v in ins.items():
            fx["in_" + k] = np.asarray(v)
            fx["out_" + k] = np.asarray(a[k])
        for i, s in enumerate(stacks):
            fx[f"stack_{i}"] = np.asarray(s)
        np.savez_compressed(os.path.join(OUT, name + ".npz"), **fx)
        print(name, "ok", os.path.basename(so))


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("STADE_REFERENCE_DIR")
    if not ref:
        sys.exit("usage: make_exemplar_golden.py <path to the STADE.jl checkout> "
                 "(or set STADE_REFERENCE_DIR)")
    main(ref)
