"""Writes the golden fixtures of this directory: per generated sweep, one
seeded trial at a small size — its inputs (primal baseline and shadow seeds,
the tape zero-filled, the float scalars), the CPU oracle's outputs in the
sweep's own type, and the same oracle run in long double (the truth the
parity verdict measures against). Arrays are stored as written by the
sweeps, in the generated argument order.

The reference cannot run here (no Julia), so the expected outputs are the
oracle's; the fixtures pin the oracle and the input generator against drift,
and the GPU tests judge libstade_b200 against them with the parity verdict.

    python tests/golden/make_golden.py        # rewrites tests/golden/*.npz
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))

import parity  # noqa: E402

SIZES = {
    "affine_ls_b": dict(n_s=37, n_o=9, n_i=5),
    "affine_ls_d": dict(n_s=37, n_o=9, n_i=5),
    "mlp2_ce_b": dict(n_s=48, n_i=36, n_h=32, n_o=10),
    "mlp2_ce_d_f32": dict(n_s=32, n_i=24, n_h=20, n_o=10),
    "mlp2_ce_d_f64": dict(n_s=32, n_i=24, n_h=20, n_o=10),
    "mlp2_ce_hv": dict(n_s=16, n_i=20, n_h=16, n_o=10),
    "heat2d_b": dict(n=12, n_step=3),
    "heat2d_d": dict(n=12, n_step=3),
    "conv1d_relu_mse_b": dict(n_b=2, n_c=8, n_l=40, n_o=8, n_k=5),
    "conv1d_relu_mse_d": dict(n_b=2, n_c=8, n_l=40, n_o=8, n_k=5),
}
SEED_TAG = "golden"


def trial(name):
    """(kernel, ints, inputs, scalars) of the one golden trial of `name`."""
    kern = parity.KERNELS[name]
    ints = dict(SIZES[name])
    base, seeds = parity.make_trials(kern, ints, 1, SEED_TAG)
    st, sc = parity._state(kern, ints, base, seeds[0])
    return kern, ints, st, sc


def compute(name):
    kern, ints, st, sc = trial(name)
    out = parity.cases.copy_state(st)
    ret = kern.cpu(out, ints, sc, False) or []
    big = parity.OrderedDict((k, v.astype(np.float64)) for k, v in st.items())
    ret_big = kern.cpu(big, ints, sc, True) or []
    return kern, ints, st, sc, out, ret, big, ret_big


def write(name):
    kern, ints, st, sc, out, ret, big, ret_big = compute(name)
    arrs = {}
    for k in st:   # outputs equal to their input (read-only arrays) are not stored twice
        arrs["in_" + k] = st[k]
        if not np.array_equal(out[k], st[k]):
            arrs["out_" + k] = out[k]
        if not np.array_equal(big[k], st[k].astype(np.float64)):
            arrs["truth_" + k] = big[k]
    arrs["ret"] = np.asarray(ret, np.float64)
    arrs["ret_truth"] = np.asarray(ret_big, np.float64)
    arrs["meta"] = np.frombuffer(json.dumps(dict(
        kernel=name, ints=ints, scalars=sc, dtype=np.dtype(kern.dtype).name,
        seed_tag=SEED_TAG)).encode(), np.uint8)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **arrs)


def load(name):
    """(meta, inputs, outputs, truth, returned scalars, their truth) of a
    stored fixture; an array the sweep left unchanged has out == truth == in."""
    with np.load(os.path.join(HERE, name + ".npz")) as z:
        d = {k: z[k] for k in z.files}
    meta = json.loads(d.pop("meta").tobytes().decode())
    keys = [k[3:] for k in d if k.startswith("in_")]
    st = parity.OrderedDict((k, d["in_" + k]) for k in keys)
    out = parity.OrderedDict((k, d.get("out_" + k, st[k])) for k in keys)
    truth = parity.OrderedDict((k, d.get("truth_" + k, st[k].astype(np.float64))) for k in keys)
    return meta, st, out, truth, list(d["ret"]), list(d["ret_truth"])


if __name__ == "__main__":
    for n in SIZES:
        write(n)
        print(n, os.path.getsize(os.path.join(HERE, n + ".npz")), "bytes")
