"""The .cu emitter on the CPU: its checker (the Julia-subset interpreter) pinned
to the C++ oracle, the loop decisions it records, the emitted program built
for the host and compared bit for bit with the interpreter, the sm_100a build,
the corpus adjoints checked against finite differences of their primals, and
the refusals."""
import json
import os
import subprocess

import numpy as np
import pytest

import cases
import emit_cases as ec
import jlsub
from oracle import oracle as orc
from stadeb200 import emit

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _interp_run(name, args, precision=64):
    I = jlsub.Interp(ec.source(name), precision, ec.CASES[name][2])
    fn = name
    stacks = ()
    if f"initstacks_{fn}" in I.funcs:
        stacks = I.initstacks(f"initstacks_{fn}", *ec.stack_ints(name, args))
    ret = I.call(fn, *args.values(), *stacks)
    return ret, stacks


# ---- the checker, pinned to the oracle ----------------------------------------------
@pytest.mark.parametrize("sizes", [(37, 9, 5), (1, 1, 1), (0, 3, 2), (64, 32, 16)])
def test_interp_matches_oracle_affine(sizes):
    st, _ = cases.affine_state(*sizes, seeded=True)
    a, b = cases.copy_state(st), cases.copy_state(st)
    orc.affine_ls_b(*[a[k] for k in cases.AFFINE_ARGS], *sizes)
    jlsub.Interp(ec.source("affine_ls_b")).call("affine_ls_b",
                                                *[b[k] for k in cases.AFFINE_ARGS], *sizes)
    for k in a:
        assert np.array_equal(a[k], b[k]), k


@pytest.mark.parametrize("n,n_step", [(7, 3), (1, 2), (4, 0), (12, 5)])
def test_interp_matches_oracle_heat(n, n_step):
    st, ints = cases.heat_state(n, n_step, seeded=True)
    a, b = cases.copy_state(st), cases.copy_state(st)
    r1 = orc.heat2d_b(*[a[k] for k in cases.HEAT_ARGS], 0.2, 0.75, n, n_step, a["u_stack"])
    I = jlsub.Interp(ec.source("heat2d_b"))
    (stack,) = I.initstacks("initstacks_heat2d_b", n, n_step)
    assert stack.size == max(n_step * n * n, 0) or (n_step == 0 and stack.size == 0)
    r2 = I.call("heat2d_b", *[b[k] for k in cases.HEAT_ARGS], 0.2, 0.75, n, n_step,
                b["u_stack"][:stack.size])
    assert r1 == r2
    for k in cases.HEAT_ARGS + ["u_stack"]:
        assert np.array_equal(a[k], b[k]), k


# ---- loop decisions -----------------------------------------------------------------------
def _loops(name):
    _, man = emit.emit(ec.source(name), dims=ec.CASES[name][2])
    return man, [(l["line"], l["mode"], set(l["atomics"]), set(l["reductions"]),
                  set(l["private"])) for l in man["loops"]]


def test_decisions_affine():
    man, L = _loops("affine_ls_b")
    assert [m for _, m, *_ in L] == ["parallel"] * 4
    assert L[1][2] == {"loss"}                           # the loss sum: atomics
    assert L[2][2] == set()                              # yb, tb at the thread's own index
    assert L[3][2] == {"wb", "xb", "bb"} and "sb=0.0" in L[3][4]   # convergent constant
    assert man["returns"] == [] and man["initstacks"]["stacks"] == []


def test_decisions_heat():
    man, L = _loops("heat2d_b")
    modes = [m for _, m, *_ in L]
    assert modes == ["host", "parallel", "parallel", "parallel", "parallel", "host", "parallel",
                     "gather", "parallel"]
    # the stencil's scatter into ub becomes a gather over the periodic grid;
    # the rest of that loop (unb consumed, alphab summed) stays a thread per cell
    assert man["loops"][7]["gathered"] == ["ub"]
    assert L[8][2] == set() and L[8][3] == {"alphab"}
    assert L[6][2] == set()                               # tape restore: own index
    assert man["returns"] == ["alphab"]
    kinds = {a["name"]: a["kind"] for a in man["args"]}
    assert kinds["alpha"] == "scalar_float" and kinds["alphab"] == "scalar_float_inout"
    assert kinds["n"] == "scalar_int" and man["initstacks"]["stacks"] == [
        {"name": "u_stack", "dtype": "f64"}]


def test_heat_kernel_rewrites():
    """The emitted C3 kernels carry the rewrites their speed rests on: alpha
    (never assigned) goes by value, the block-sum kernels stride over a
    resident grid, the consumed adjoints' zero stores wait for their loads,
    and the divisions by n multiply by a per-launch magic number."""
    cu, _ = emit.emit(ec.source("heat2d_b"))
    assert "g_fbox[0] = v0" in cu and "double j_alpha" in cu   # alphab boxed, alpha by value
    assert cu.count("stade_resident_blocks((const void*)") == 2   # loss and the stencil rest
    assert "tid_ += (int64_t)gridDim.x * blockDim.x" in cu
    assert "jl_after((double)(0.0), jl_bits(j___oldb_1) & z_)" in cu   # unb[idx] = 0.0
    assert "jl_after((double)(0.0), jl_bits(j___oldb_0) & z_)" in cu   # ub[idx2] = 0.0
    assert "jl_divf((j_idx - ((int64_t)1)), j_n, fd_n)" in cu and "jl_fd_make(j_n)" in cu
    assert "jl_div((j_idx" not in cu


def test_decisions_generic():
    _, L = _loops("decay_b")
    assert [m for _, m, *_ in L] == ["host", "parallel", "host", "parallel"]
    assert L[3][3] == {"kb", "dtb"}
    _, L = _loops("edge_relu_b")
    assert [m for _, m, *_ in L] == ["parallel", "parallel"]
    assert L[1][2] == {"xb"} and "db=0.0" in L[1][4]       # scatter through the table
    _, L = _loops("bilin_b")
    assert L[1][2] == {"xb", "zb"}                        # ab[i_i, i_j]: the decode is injective
    _, L = _loops("cumsum_sq_b")
    assert [m for _, m, *_ in L] == ["sequential", "parallel", "parallel", "sequential"]
    _, L = _loops("window_b")
    assert L[3][2] == {"wb", "xb"}
    man, L = _loops("halving_b")
    assert [m for _, m, *_ in L] == ["sequential", "parallel"]
    man, L = _loops("smooth_b")
    assert [m for _, m, *_ in L] == ["parallel", "parallel", "parallel", "gather", "parallel"]
    assert man["loops"][3]["gathered"] == ["ub"] and L[4][2] == set()
    # a Tier-B tape: initstacks fills the prefix table and returns the total;
    # the taping loop is parallel because each iteration owns its span of slots
    man, L = _loops("ragged_b")
    assert [m for _, m, *_ in L] == ["parallel", "parallel"]
    assert L[0][2] == {"loss"} and L[1][2] == {"wb"}
    assert man["initstacks"]["stacks"] == [
        {"name": "v_stack", "dtype": "f64"}, {"name": "prefix_v_stack_1", "dtype": "i64_table"},
        {"name": "__tot_v_stack_1", "dtype": "int"}]


# ---- the emitted program, host build, against the interpreter -----------------------------
@pytest.mark.parametrize("name", sorted(ec.CASES))
def test_host_build_matches_interpreter(name):
    sw = emit.load(ec.source(name), dims=ec.CASES[name][2], host=True)
    gathered = {a for l in sw.m["loops"] for a in l["gathered"]}
    for size in ec.CASES[name][4][:3]:
        args = ec.make(name, size)
        ref = ec.copy_args(args)
        r_ref, st_ref = _interp_run(name, ref)
        out = ec.copy_args(args)
        stacks = sw.initstacks(*ec.stack_ints(name, out))
        sig = lambda s: s if isinstance(s, (int, np.integer)) else ("array", s.size)
        assert [sig(s) for s in stacks] == [sig(s) for s in st_ref]
        r_out = sw(*out.values(), *stacks)
        if gathered and r_ref is not None:   # the gathered values feed later statements
            assert np.allclose(r_out, r_ref, rtol=1e-13, atol=1e-13), (name, size)
        else:
            assert r_out == r_ref, (name, size)
        for k, v in out.items():
            if isinstance(v, np.ndarray):
                if gathered and v.dtype != np.int64:   # a gather sums in another order
                    assert np.allclose(v, ref[k], rtol=1e-13, atol=1e-13), (name, size, k)
                else:
                    assert np.array_equal(v, ref[k]), (name, size, k)
        for s1, s2 in zip(stacks, st_ref):
            assert np.array_equal(s1, s2), (name, size, "stack")


@pytest.mark.parametrize("name", ["affine_ls_b", "window_b"])
def test_host_build_float32(name):
    sw = emit.load(ec.source(name), precision=32, dims=ec.CASES[name][2], host=True)
    args = ec.make(name, ec.CASES[name][4][0])
    a32 = ec.copy_args(args)
    for k, v in a32.items():
        if isinstance(v, np.ndarray) and v.dtype == np.float64:
            a32[k] = v.astype(np.float32)
    ref = ec.copy_args(a32)
    _interp_run(name, ref, precision=32)
    sw(*a32.values())
    for k, v in a32.items():
        if isinstance(v, np.ndarray):
            assert v.dtype == np.float32
            err = np.abs(v - ref[k]).max() / max(np.abs(ref[k]).max(), 1e-30)
            assert err <= 1e-6, (k, err)


# ---- the corpus adjoints are the derivatives of their primals ---------------------------
def _primal_loss(I, name, args, wseed):
    """<seed, outputs> of the primal: loss-style primals report loss[1];
    decay reports <w, u_final>."""
    a = ec.copy_args(args)
    prim = name[:-2]
    params = I.funcs[prim][0]
    I.call(prim, *[a[p] for p in params])
    if "loss" in a:
        return float(a["loss"][0])
    return float(np.dot(wseed, a["u"]))


@pytest.mark.parametrize("name", ["decay_b", "edge_relu_b", "bilin_b", "cumsum_sq_b",
                                  "window_b", "smooth_b", "ragged_b"])
def test_corpus_adjoint_is_the_derivative(name):
    size = ec.CASES[name][4][0]
    args = ec.make(name, size, "fd")
    I = jlsub.Interp(ec.source(name), 64, ec.CASES[name][2])
    prim_params = I.funcs[name[:-2]][0]
    floats = [p for p in prim_params if isinstance(args.get(p), (np.ndarray, float))
              and not (isinstance(args.get(p), np.ndarray) and args[p].dtype == np.int64)
              and p != "loss" and p not in ("c", "z")]
    r = np.random.default_rng(7)
    v = {p: (r.standard_normal(args[p].shape) if isinstance(args[p], np.ndarray)
             else float(r.standard_normal())) for p in floats}
    wseed = r.standard_normal(args["u"].shape) if name == "decay_b" else None
    # adjoint: zero shadows, seed lossb = 1 (or ub = w for decay)
    adj = ec.copy_args(args)
    for p in list(adj):
        if p.endswith("b") and p[:-1] in adj and p not in ("b",):
            adj[p] = np.zeros_like(adj[p]) if isinstance(adj[p], np.ndarray) else 0.0
    if "lossb" in adj:
        adj["lossb"][:] = 1.0
    if name == "decay_b":
        adj["ub"] = wseed.copy()
    stacks = I.initstacks(f"initstacks_{name}", *ec.stack_ints(name, adj))
    ret = I.call(name, *adj.values(), *stacks)
    rets = dict(zip([p + "b" for p in prim_params if not isinstance(args.get(p), np.ndarray)
                     and p not in ec.CASES[name][3] and not p.startswith("i_")],
                    ret if isinstance(ret, tuple) else ([ret] if ret is not None else [])))
    grad_dot = 0.0
    for p in floats:
        g = rets[p + "b"] if not isinstance(args[p], np.ndarray) else adj[p + "b"]
        grad_dot += float(np.sum(np.asarray(g) * v[p]))
    eps = 1e-6

    def at(s):
        a = ec.copy_args(args)
        for p in floats:
            a[p] = a[p] + s * v[p]
        return _primal_loss(I, name, a, wseed)
    fd = (at(eps) - at(-eps)) / (2 * eps)
    assert abs(fd - grad_dot) <= 1e-6 * max(1.0, abs(fd)), (fd, grad_dot)


# ---- builds and refusals --------------------------------------------------------------------
@pytest.mark.parametrize("name", sorted(ec.CASES))
def test_builds_for_sm100a(name):
    cu, _ = emit.emit(ec.source(name), dims=ec.CASES[name][2])
    assert os.path.exists(emit.build(cu))


@pytest.mark.parametrize("src,msg", [
    ("function f_b(x, i_n)\n for i = 1:i_n\n x[i] = gamma(x[i])\n end\nend\n",
     "function gamma is not supported"),
    ("function f_b(a, i_n)\n for k = 1:i_n\n a[div(k, 2), k] = 1.0\n end\nend\n",
     "cannot infer dimension 1 of a"),
    ("function f_b(x, i_n)\n for i = 1:i_n\n if x[i] > 0.0\n return nothing\n end\n end\nend\n",
     "return inside a loop or branch"),
    ("function f_b(x, i_n)\n for i = 1:i_n\n x[i] = 1.0\n", "missing 'end'"),
])
def test_refusals(src, msg):
    with pytest.raises(emit.EmitError, match=msg):
        emit.emit(src)


def test_cli_and_cuda_file(tmp_path):
    src = os.path.join(ROOT, "tests", ec.CORPUS, "bilin_b.jl")
    exe = os.path.join(ROOT, "stade.jl_b200", "stade_emit")
    out = tmp_path / "bilin_b.cu"
    man = tmp_path / "bilin_b.json"
    subprocess.run([exe, src, str(out), "--dims", "a=i_m;ab=i_m", "--manifest", str(man)],
                   check=True)
    m = json.loads(man.read_text())
    assert m["symbol"] == "stade_bilin_b" and "extern \"C\" int stade_bilin_b(" in out.read_text()
    m2 = emit.cuda_file(src, str(tmp_path / "b2.cu"), dims={"a": ["i_m"], "ab": ["i_m"]})
    assert m2 == m and (tmp_path / "b2.json").exists()
    # without --dims the leading extent comes from the flattened nest's decode
    inferred = tmp_path / "bilin_inferred.cu"
    subprocess.run([exe, src, str(inferred)], check=True)
    assert inferred.read_text() == out.read_text()
    # an extent nothing gives is refused with a pointer to --dims
    odd = tmp_path / "odd_b.jl"
    odd.write_text("function odd_b(a, ab, i_r, i_c)\n    for k = 1:i_c\n"
                   "        ab[i_r, k] = ab[i_r, k] + a[i_r, k]\n    end\nend\n")
    bad = subprocess.run([exe, str(odd), str(out)], capture_output=True, text=True)
    assert bad.returncode == 1 and "cannot infer dimension" in bad.stderr


# ---- the reference's own generated adjoints, read as input text ----------------------------
_REF_CORPUS = os.path.join(os.path.dirname(ROOT), "reference", "test", "val-corpus")


@pytest.mark.skipif(not os.path.isdir(_REF_CORPUS), reason="the reference checkout is not here")
@pytest.mark.parametrize("suffix,least", [("_b", 133), ("_hv", 133), ("_d", 136)])
def test_reference_corpus_emits(suffix, least):
    """STADE's generated adjoints, HVP and tangent sweeps (its test corpus,
    read from the reference checkout beside this repository): the emitter
    accepts all but those that index a multi-dimensional argument whose
    leading extent neither a loop nor a flattened nest's decode gives (they
    need dims) and two tangents that
    reassign an integer argument inside device loops; a sample of the
    emitted programs compiles."""
    names = sorted(f for f in os.listdir(_REF_CORPUS) if f.endswith(suffix + ".jl"))
    accepted, refused = [], []
    for f in names:
        with open(os.path.join(_REF_CORPUS, f)) as fh:
            src = fh.read()
        try:
            cu, _ = emit.emit(src)
            accepted.append((f, cu))
        except emit.EmitError as e:
            refused.append((f, str(e)))
    assert len(names) >= 139 and len(accepted) >= least, refused
    for f, msg in refused:
        assert "cannot infer dimension" in msg or "assigned on the device and on the host" in msg, (
            f, msg)
    for f, cu in accepted[::16]:
        r = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-DSTADE_EMIT_HOST", "-x", "c++",
                            "-"], input=cu, capture_output=True, text=True)
        assert r.returncode == 0, (f, r.stderr[-2000:])


@pytest.mark.skipif(not os.path.isdir(_REF_CORPUS), reason="the reference checkout is not here")
def test_reference_tier_b_sweep():
    """The reference's raggedind_b (a row length that grows with the row: a
    Tier-B tape with prefix tables), emitted and built for the host: bit for
    bit the interpreter's result and tables, and its x adjoint the central
    difference of the primal raggedind (sizes from the primal's header: out
    and u of length n, x of length m0 + n)."""
    rd = lambda f: open(os.path.join(_REF_CORPUS, f)).read()
    src = rd("raggedind_b.jl")
    sw = emit.load(src, host=True)
    assert [l["mode"] for l in sw.m["loops"]] == ["parallel", "parallel"]
    n, m0 = 7, 3
    r = np.random.default_rng(1)
    args = dict(out=np.zeros(n), outb=r.standard_normal(n), u=r.standard_normal(n),
                ub=np.zeros(n), x=r.standard_normal(m0 + n), xb=np.zeros(m0 + n))
    ref = {k: v.copy() for k, v in args.items()}
    I = jlsub.Interp(src)
    st_ref = I.initstacks("initstacks_raggedind_b", m0, n)
    I.call("raggedind_b", *ref.values(), n, m0, *st_ref)
    out = {k: v.copy() for k, v in args.items()}
    st = sw.initstacks(m0, n)
    sw(*out.values(), n, m0, *st)
    for k in args:
        assert np.array_equal(out[k], ref[k]), k
    for a, b in zip(st, st_ref):
        assert np.array_equal(a, b)
    P = jlsub.Interp(rd("raggedind.jl"))

    def loss(x):
        o = np.zeros(n)
        P.call("raggedind", o, args["u"].copy(), x, n, m0)
        return float(np.dot(o, args["outb"]))
    v = r.standard_normal(m0 + n)
    fd = (loss(args["x"] + 1e-6 * v) - loss(args["x"] - 1e-6 * v)) / 2e-6
    assert abs(fd - float(np.dot(out["xb"], v))) <= 1e-6 * max(1.0, abs(fd))


@pytest.mark.skipif(not os.path.isdir(_REF_CORPUS), reason="the reference checkout is not here")
def test_reference_hvp_sweep():
    """The reference's advection_hv (an HVP sweep that allocates the tangent
    of its tape in Julia): the allocation becomes a trailing argument the
    caller provides (sized by stade_advection_hv_locals), the stacks come
    from initstacks_advection_b, and the host build agrees with the
    interpreter (1e-13: its stencil adjoint is gathered, summing in another
    order)."""
    src = open(os.path.join(_REF_CORPUS, "advection_hv.jl")).read()
    sw = emit.load(src, host=True)
    assert sw.m["initstacks"]["symbol"] == "stade_initstacks_advection_b"
    assert sw.m["locals"]["arrays"] == [{"name": "du_stack_d", "dtype": "f64"}]
    assert sw.m["args"][-1] == {"name": "du_stack_d", "kind": "array_float", "stack": False,
                                "local": True}
    nn, ns = 9, 4
    r = np.random.default_rng(2)
    arr = lambda: r.standard_normal(nn)
    a = dict(u=arr(), ub=arr(), du=np.zeros(nn), dub=arr(), c=0.7, cb=0.1, dx=0.5, dxb=0.2,
             dt=0.05, dtb=-0.3, i_nstep=ns, i_nnode=nn, ud=arr(), ubd=arr(), dud=np.zeros(nn),
             dubd=arr(), cd=0.3, cbd=0.0, dxd=-0.2, dxbd=0.0, dtd=0.4, dtbd=0.0)
    cp = lambda d: {k: (v.copy() if isinstance(v, np.ndarray) else v) for k, v in d.items()}
    ref, out = cp(a), cp(a)
    I = jlsub.Interp(src)
    (st_ref,) = I.initstacks("initstacks_advection_b", nn, ns)
    r_ref = I.call("advection_hv", *ref.values(), st_ref)
    (st,) = sw.initstacks(nn, ns)
    r_out = sw(*out.values(), st)
    assert np.allclose(r_out, r_ref, rtol=1e-13, atol=1e-13)
    assert np.array_equal(st, st_ref)
    for k, v in a.items():
        if isinstance(v, np.ndarray):
            assert np.allclose(out[k], ref[k], rtol=1e-13, atol=1e-13), k


@pytest.mark.skipif(not os.path.isdir(_REF_CORPUS), reason="the reference checkout is not here")
def test_reference_tangent_sweep():
    """The reference's advection_d (forward mode), emitted and built for the
    host: bit for bit the interpreter, and its tangent ud the central
    difference of the primal advection along (ud, cd, dxd, dtd)."""
    src = open(os.path.join(_REF_CORPUS, "advection_d.jl")).read()
    sw = emit.load(src, host=True)
    nn, ns = 9, 4
    r = np.random.default_rng(3)
    u0, ud0 = r.standard_normal(nn), r.standard_normal(nn)
    c, dx, dt, cd, dxd, dtd = 0.7, 0.5, 0.05, 0.3, -0.2, 0.4
    out = dict(u=u0.copy(), ud=ud0.copy(), du=np.zeros(nn), dud=np.zeros(nn))
    ref = {k: v.copy() for k, v in out.items()}
    jlsub.Interp(src).call("advection_d", ref["u"], ref["ud"], ref["du"], ref["dud"], c, cd, dx,
                           dxd, dt, dtd, ns, nn)
    sw(out["u"], out["ud"], out["du"], out["dud"], c, cd, dx, dxd, dt, dtd, ns, nn)
    for k in out:
        assert np.array_equal(out[k], ref[k]), k
    P = jlsub.Interp(src)

    def prim(h):
        u = u0 + h * ud0
        P.call("advection", u, np.zeros(nn), c + h * cd, dx + h * dxd, dt + h * dtd, ns, nn)
        return u
    fd = (prim(1e-6) - prim(-1e-6)) / 2e-6
    assert np.max(np.abs(fd - out["ud"])) <= 1e-6 * max(1.0, np.max(np.abs(fd)))


@pytest.mark.skipif(not os.path.isdir(_REF_CORPUS), reason="the reference checkout is not here")
def test_reference_flattened_nest_extent():
    """The reference's matvec_loss_b indexes a[i_i, i_j] with i_i, i_j decoded
    from one flattened loop over 1:i_m * i_n (div / mod by i_n): the emitter
    takes a's leading extent i_m from that decode, and the host build agrees
    bit for bit with the interpreter given a = i_m x i_n explicitly."""
    src = open(os.path.join(_REF_CORPUS, "matvec_loss_b.jl")).read()
    sw = emit.load(src, host=True)
    m, n = 5, 3
    r = np.random.default_rng(4)
    a = dict(loss=np.zeros(1), lossb=np.ones(1), a=r.standard_normal(m * n), ab=np.zeros(m * n),
             u=r.standard_normal(n), ub=np.zeros(n), v=np.zeros(m), vb=np.zeros(m))
    ref = {k: v.copy() for k, v in a.items()}
    jlsub.Interp(src, 64, {"a": ["i_m"], "ab": ["i_m"]}).call("matvec_loss_b", *ref.values(), m, n)
    out = {k: v.copy() for k, v in a.items()}
    sw(*out.values(), m, n)
    for k in a:
        assert np.array_equal(out[k], ref[k]), k
    assert np.any(out["ab"] != 0)
