"""The input generator: FNV-1a seeds pinned by the reference's own golden
values (test/validate_seed_stable.jl:37-38), Box-Muller normals with the
statistics the reference checks (validate_seed_stable.jl:60-62), and
chunked generation that does not depend on the host thread count."""
import os
import subprocess
import sys

import numpy as np

import stadeb200
from stadeb200 import synth


def test_fnv1a_goldens_of_the_reference():
    """The reference's own golden values, kept as a fixture (tests/golden)."""
    import json
    here = os.path.dirname(os.path.abspath(__file__))
    with open(os.path.join(here, "golden", "fnv1a_seeds.json")) as f:
        gold = json.load(f)["seeds"]
    L = stadeb200.lib()
    assert len(gold) == 2
    for s, v in gold.items():
        assert L.stade_fnv1a64(s.encode()) == int(v, 16), s


def test_normals_mean_and_variance():
    x = synth.normal(10 ** 6, 11, np.float64)
    assert abs(x.mean()) < 5e-3 and abs((x * x).mean() - 1) < 5e-3


def test_uniform_range_and_onehot():
    u = synth.uniform(100000, 3, np.float32, -0.5, 0.25)
    assert u.min() >= -0.5 and u.max() < 0.25
    y = synth.onehot(1000, 10, 9, np.float64).reshape(1000, 10)
    assert np.all(y.sum(1) == 1.0)
    counts = y.sum(0)
    assert counts.min() > 60


def test_generation_independent_of_thread_count():
    code = ("import sys; sys.path.insert(0, %r); import numpy as np; from stadeb200 import synth;"
            "a = synth.normal(3 * 2**20 + 5, 77, np.float32); print(float(a.sum()), a[123456])")
    root = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "stade.jl_b200")
    outs = []
    for nt in ("1", "4"):
        env = dict(os.environ, OMP_NUM_THREADS=nt)
        outs.append(subprocess.run([sys.executable, "-c", code % root], env=env, check=True,
                                   capture_output=True, text=True).stdout)
    assert outs[0] == outs[1]


def test_oracle_generator_matches_the_library_bit_for_bit():
    """The oracle side's own generator (oracle/synth.cc, used by the bench's
    reference arm so that it never loads the product library) draws the same
    bits as the library's, for every configuration's recipe and across the
    2^20-element chunk boundary."""
    from oracle import oracle as orc
    og = orc.generator()
    cases = [("affine_ls_inputs", (37, 9, 5)),
             ("mlp2_ce_inputs", (300, 132, 20, 10)),
             ("mlp2_ce_hv_inputs", (64, 16, 8, 10)),
             ("heat2d_inputs", (1100,)),                  # 1.21 M > 2^20 elements
             ("conv1d_relu_mse_inputs", (3, 5, 40, 4, 3))]
    for name, args in cases:
        a, b = getattr(synth, name)(*args), getattr(og, name)(*args)
        assert a.keys() == b.keys(), name
        for k in a:
            assert a[k].dtype == b[k].dtype and np.array_equal(a[k], b[k]), (name, k)
    assert og.seed("abc", "x") == synth.seed("abc", "x")
    for dt in (np.float32, np.float64):
        assert np.array_equal(og.onehot(2 ** 20 + 7, 10, 5, dt), synth.onehot(2 ** 20 + 7, 10, 5, dt))
