"""Pins of the CPU oracle (the restated generated sweeps) on the CPU.

The reference cannot run here (Julia) and ships no numeric gradients for
these primals, so the oracle is pinned by what the reference's own tests
check (test/validate_corpus.jl, src/STADE.jl:16334-17159):
  - agreement with the textbook gradients of the same functions (refmath),
  - central finite differences (the reference's FD oracle, rtol 1e-3),
  - the dot-product identity <grad, v> = lossd of the HVP's forward tangent
    (the reference's exact identity, rtol 1e-11, src/STADE.jl:17108-17131),
  - HVP against finite differences of the gradient (src/STADE.jl:17133-17159)
    and against an 80-bit long-double run of the same sweep (the
    BigFloat-truth idea of val_gpu_parity_script, src/STADE.jl:18939).
"""
import numpy as np
import pytest

import cases
import refmath
from refmath import rel_err


def test_affine_matches_closed_form():
    st, ints = cases.affine_state(37, 9, 5, seeded=True)
    ref = refmath.affine_ls(st["w"], st["b"], st["x"], st["t"], st["lossb"], **ints)
    st0 = cases.copy_state(st)
    cases.oracle_affine(st, ints)
    assert rel_err(st["y"], ref["y"]) < 1e-14
    assert abs(st["loss"][0] - (st0["loss"][0] + ref["loss"])) < 1e-12 * abs(ref["loss"])
    # accumulated outputs: output = seed + gradient; consumed yb ends at zero
    g = st0["yb"].reshape(ints["n_s"], ints["n_o"])  # yb seed flows like the residual
    W = st["w"].reshape(ints["n_o"], ints["n_i"])
    X = st["x"].reshape(ints["n_s"], ints["n_i"])
    assert rel_err(st["wb"] - st0["wb"], ref["wb"] + (g.T @ X).ravel()) < 1e-12
    assert rel_err(st["bb"] - st0["bb"], ref["bb"] + g.sum(0)) < 1e-12
    assert rel_err(st["xb"] - st0["xb"], ref["xb"] + (g @ W).ravel()) < 1e-12
    assert rel_err(st["tb"] - st0["tb"], ref["tb"]) < 1e-12
    assert np.all(st["yb"] == 0.0)


def test_affine_finite_differences():
    st, ints = cases.affine_state(6, 4, 3)
    run = cases.copy_state(st)
    cases.oracle_affine(run, ints)
    eps = 1e-6
    for name in ("w", "b", "x", "t"):
        for i in range(0, st[name].size, max(1, st[name].size // 5)):
            lp, lm = cases.copy_state(st), cases.copy_state(st)
            lp[name][i] += eps
            lm[name][i] -= eps
            cases.oracle_affine(lp, ints)
            cases.oracle_affine(lm, ints)
            fd = (lp["loss"][0] - lm["loss"][0]) / (2 * eps)
            assert abs(run[name + "b"][i] - fd) <= 1e-3 * max(1.0, abs(fd))


def test_mlp_f64_matches_closed_form():
    st, ints = cases.mlp_state(13, 11, 7, 5, np.float64, seeded=False)
    ref = refmath.mlp2_ce(st["x"], st["y"], st["w1"], st["b1"], st["w2"], st["b2"], st["lossb"],
                          **ints)
    cases.oracle_mlp(st, ints)
    for k in ("h", "z", "p"):
        assert rel_err(st[k], ref[k]) < 1e-13, k
    assert abs(st["loss"][0] - ref["loss"]) < 1e-12 * abs(ref["loss"])
    for k in ("yb", "w2b", "b2b", "w1b", "b1b", "xb"):
        assert rel_err(st[k], ref[k]) < 1e-12, k
    for k in ("hb", "zb", "pb"):
        assert np.all(st[k] == 0.0), k


def test_mlp_f32_close_to_f64():
    s32, ints = cases.mlp_state(16, 20, 12, 10, np.float32, seeded=True)
    s64 = cases.OrderedDict((k, v.astype(np.float64)) for k, v in s32.items())
    cases.oracle_mlp(s32, ints)
    cases.oracle_mlp(s64, ints)
    for k in ("yb", "w2b", "b2b", "w1b", "b1b", "xb", "h", "z", "p"):
        assert rel_err(s32[k], s64[k]) < 2e-5, k


def test_mlp_seeds_act_like_generated_code():
    """hb / zb / pb seeds enter the reverse sweep; outputs accumulate."""
    st, ints = cases.mlp_state(5, 6, 4, 3, np.float64, seeded=True)
    st0 = cases.copy_state(st)
    cases.oracle_mlp(st, ints)
    clean = cases.copy_state(st0)
    for k in ("xb", "yb", "w1b", "b1b", "w2b", "b2b", "hb", "zb", "pb"):
        clean[k][:] = 0.0
    cases.oracle_mlp(clean, ints)
    # a non-zero hb seed changes w1b beyond the accumulated starting value
    assert rel_err(st["w1b"] - st0["w1b"], clean["w1b"]) > 1e-6
    for k in ("hb", "zb", "pb"):
        assert np.all(st[k] == 0.0)


def _heat_fd_alpha(st, ints, eps=1e-6):
    vals = []
    for sgn in (+1, -1):
        s = cases.copy_state(st)
        i = dict(ints)
        i["alpha"] = ints["alpha"] + sgn * eps
        s["loss"][0] = 0.0
        cases.oracle_heat(s, i)
        vals.append(s["loss"][0])
    return (vals[0] - vals[1]) / (2 * eps)


@pytest.mark.parametrize("n,n_step", [(6, 3), (8, 4), (10, 1)])
def test_heat_matches_closed_form(n, n_step):
    st, ints = cases.heat_state(n, n_step)
    ref = refmath.heat2d(st["u"], ints["alpha"], n, n_step, st["lossb"])
    u0 = st["u"].copy()
    ab = cases.oracle_heat(st, ints)
    # the tape holds the forward states bit for bit, u is restored, un final
    for k in range(n_step):
        assert np.array_equal(st["u_stack"][k * n * n:(k + 1) * n * n], ref["states"][k].ravel())
    assert np.array_equal(st["u"], u0)
    assert np.array_equal(st["un"], ref["final"].ravel())
    assert abs(st["loss"][0] - ref["loss"]) < 1e-13 * ref["loss"]
    assert rel_err(st["ub"], ref["ub"]) < 1e-13
    assert abs(ab - ref["alphab"]) < 1e-12 * max(1.0, abs(ref["alphab"]))
    assert np.all(st["unb"] == 0.0)


def test_heat_alpha_finite_difference_and_homogeneity():
    st, ints = cases.heat_state(8, 3)
    fd = _heat_fd_alpha(st, ints)
    s = cases.copy_state(st)
    ab = cases.oracle_heat(s, ints)
    assert abs(ab - fd) <= 1e-3 * max(1.0, abs(fd))
    # loss is homogeneous of degree 2 in u0: <ub, u0> = 2 loss
    assert abs(np.dot(s["ub"], st["u"]) - 2 * s["loss"][0]) < 1e-11 * s["loss"][0]


def test_heat_no_steps():
    st, ints = cases.heat_state(6, 0, seeded=True)
    st0 = cases.copy_state(st)
    ab = cases.oracle_heat(st, ints)
    assert ab == ints["alphab"]
    assert np.allclose(st["ub"], st0["ub"] + 2 * st0["u"])
    assert np.isclose(st["loss"][0], st0["loss"][0] + np.sum(st0["u"] ** 2))


def test_conv_f64_matches_closed_form():
    st, ints = cases.conv_state(3, 4, 21, 5, 3, np.float64)
    ref = refmath.conv1d_relu_mse(st["x"], st["w"], st["t"], st["lossb"], **ints)
    cases.oracle_conv(st, ints)
    for k in ("z", "r", "wb", "xb", "tb"):
        assert rel_err(st[k], ref[k]) < 1e-12, k
    assert abs(st["loss"][0] - ref["loss"]) < 1e-12 * ref["loss"]
    assert np.all(st["zb"] == 0.0) and np.all(st["rb"] == 0.0)


def test_conv_f32_close_to_f64():
    s32, ints = cases.conv_state(2, 3, 30, 4, 5, np.float32, seeded=True)
    s64 = cases.OrderedDict((k, v.astype(np.float64)) for k, v in s32.items())
    cases.oracle_conv(s32, ints)
    cases.oracle_conv(s64, ints)
    for k in ("wb", "xb", "tb", "z", "r"):
        assert rel_err(s32[k], s64[k]) < 1e-5, k


def _grad_vec(st):
    return np.concatenate([st[k] for k in ("w1b", "b1b", "w2b", "b2b")])


def test_hvp_dot_product_identity_and_gradient():
    """lossd = <grad, v> at rtol 1e-11; the HVP's adjoint part equals the
    adjoint sweep."""
    st, ints = cases.mlp_hv_state(9, 7, 6, 4)
    cases.oracle_mlp_hv(st, ints)
    adj, _ = cases.mlp_state(9, 7, 6, 4, np.float64)
    for k in ("x", "y", "w1", "b1", "w2", "b2", "lossb"):
        adj[k] = cases.synth.mlp2_ce_hv_inputs(9, 7, 6, 4)[k].copy()
    cases.oracle_mlp(adj, ints)
    for k in ("w1b", "b1b", "w2b", "b2b", "xb", "yb"):
        assert rel_err(st[k], adj[k]) < 1e-14, k
    v = np.concatenate([st[k] for k in ("w1d", "b1d", "w2d", "b2d")])
    dot = float(np.dot(_grad_vec(st), v))
    assert abs(st["lossd"][0] - dot) <= 1e-11 * max(1.0, abs(dot))


def test_hvp_matches_gradient_finite_differences():
    n = (6, 5, 4, 3)
    st, ints = cases.mlp_hv_state(*n)
    cases.oracle_mlp_hv(st, ints)
    hv = np.concatenate([st[k] for k in ("w1bd", "b1bd", "w2bd", "b2bd")])
    eps = 1e-5
    grads = []
    for sgn in (+1, -1):
        s, _ = cases.mlp_state(*n, dtype=np.float64)
        base = cases.synth.mlp2_ce_hv_inputs(*n)
        for k in ("x", "y", "lossb"):
            s[k] = base[k].copy()
        for k in ("w1", "b1", "w2", "b2"):
            s[k] = base[k] + sgn * eps * base[k + "d"]
        cases.oracle_mlp(s, ints)
        grads.append(_grad_vec(s))
    fd = (grads[0] - grads[1]) / (2 * eps)
    assert rel_err(hv, fd) < 1e-6


def test_hvp_against_long_double_truth():
    st, ints = cases.mlp_hv_state(8, 6, 5, 4, seeded=True, xd_nonzero=True)
    tr = cases.copy_state(st)
    cases.oracle_mlp_hv(st, ints)
    cases.oracle_mlp_hv(tr, ints, truth=True)
    for k in ("w1bd", "b1bd", "w2bd", "b2bd", "xbd", "ybd", "w1b", "xb", "hd", "zd", "pd"):
        assert rel_err(st[k], tr[k]) < 1e-12, k


# ---- the sample-parallel oracle variants (full-size checks, CPU baseline) ----
def _omp_vs_serial(state_fn, args, ints_keys, run, summed, threads=3):
    """Per-sample outputs bit-identical to the serial sweep; the summed
    shadows differ only in the order the blocks' sums are added."""
    st, ints = state_fn()
    a, b = cases.copy_state(st), cases.copy_state(st)
    run(a, ints, None)
    run(b, ints, threads)
    for k in args:
        if k in summed:
            scale = max(1.0, float(np.abs(a[k]).max()))
            assert float(np.abs(a[k] - b[k]).max()) <= 1e-5 * scale, k
        else:
            assert np.array_equal(a[k], b[k]), k


def test_parallel_mlp2_ce_b_matches_serial():
    from oracle import oracle as orc
    for dt in (np.float32, np.float64):
        def run(st, ints, threads):
            orc.mlp2_ce_b(*[st[a] for a in cases.MLP_ARGS], ints["n_s"], ints["n_i"], ints["n_h"],
                          ints["n_o"], threads=threads)
        _omp_vs_serial(lambda: cases.mlp_state(37, 12, 8, 5, dtype=dt, seeded=True),
                       cases.MLP_ARGS, None, run, {"w1b", "b1b", "w2b", "b2b", "loss"})


def test_parallel_conv1d_relu_mse_b_keeps_the_whole_batch_mean():
    from oracle import oracle as orc
    for dt in (np.float32, np.float64):
        def run(st, ints, threads):
            orc.conv1d_relu_mse_b(*[st[a] for a in cases.CONV_ARGS], ints["n_b"], ints["n_c"],
                                  ints["n_l"], ints["n_o"], ints["n_k"], threads=threads)
        _omp_vs_serial(lambda: cases.conv_state(5, 3, 20, 4, 3, dtype=dt, seeded=True),
                       cases.CONV_ARGS, None, run, {"wb", "loss"})


def test_parallel_mlp2_ce_hv_matches_serial():
    from oracle import oracle as orc

    def run(st, ints, threads, truth=False):
        orc.mlp2_ce_hv(*[st[a] for a in cases.MLP_ARGS], ints["n_s"], ints["n_i"], ints["n_h"],
                       ints["n_o"], *[st[a] for a in cases.MLP_TAN], threads=threads, truth=truth)
    summed = {"w1b", "b1b", "w2b", "b2b", "loss", "w1bd", "b1bd", "w2bd", "b2bd", "lossd"}
    _omp_vs_serial(lambda: cases.mlp_hv_state(23, 12, 8, 5, seeded=True),
                   cases.MLP_ARGS + cases.MLP_TAN, None, run, summed)
    # the long-double instantiation as well
    st, ints = cases.mlp_hv_state(23, 12, 8, 5, seeded=True)
    a, b = cases.copy_state(st), cases.copy_state(st)
    run(a, ints, None, truth=True)
    run(b, ints, 3, truth=True)
    for k in cases.MLP_ARGS + cases.MLP_TAN:
        scale = max(1.0, float(np.abs(a[k]).max()))
        assert float(np.abs(a[k] - b[k]).max()) <= 1e-15 * scale, k


@pytest.mark.parametrize("n,n_step", [(1, 3), (2, 2), (3, 4), (5, 3), (17, 5), (64, 2)])
def test_parallel_heat2d_b_bit_identical_to_serial(n, n_step):
    """The parallel C3 oracle gathers each cell's additions in the serial
    scatter's order: every field, the tape, loss and alphab bit for bit
    (wrapped neighbours, n = 1 and 2 where neighbours coincide, included)."""
    from oracle import oracle as orc
    st, ints = cases.heat_state(n, n_step, seeded=True)
    a, b = cases.copy_state(st), cases.copy_state(st)
    ra = orc.heat2d_b(*[a[k] for k in cases.HEAT_ARGS], ints["alpha"], ints["alphab"], n, n_step,
                      a["u_stack"])
    rb = orc.heat2d_b(*[b[k] for k in cases.HEAT_ARGS], ints["alpha"], ints["alphab"], n, n_step,
                      b["u_stack"], threads=4)
    assert ra == rb
    for k in st:
        assert np.array_equal(a[k], b[k]), k
