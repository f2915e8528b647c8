"""Host logic of the data-parallel epilogue, on the CPU.

Role tables and refusals restate test/validate_ddp_roles.jl (hand-written
tables for the val-corpus subjects, the refusal list with its message
fragments). The rank-invariance tests restate test/validate_ddp.jl
(batch_run, :97 and :160-179): each of two `gloo` ranks runs the oracle sweep
on its own samples between the epilogue's resets and sums, and the summed
:accum / :reduced buffers must match one run over all samples within
rtol 1e-12; the global sample count comes back from allreduce_accum. The
epilogue here runs through ddp.Epilogue, the class the CUDA path drives with
the NCCL backend, with a gloo backend over numpy arrays standing in for it.
"""
import os
import socket

import numpy as np
import pytest

from stadeb200 import ddp

A = "array_float"
I = "scalar_int"


def sig(name, args, floats, written, reduced_outputs, ambiguous=()):
    kinds = {a: (A if a in floats else I) for a in args}
    return ddp.KernelSig(name, tuple(args), kinds, frozenset(written),
                         frozenset(reduced_outputs), frozenset(ambiguous))


# the val-corpus subjects of validate_ddp_roles.jl, with the write facts their
# bodies show (test/val-corpus/<name>.jl)
SUBJECTS = {
    "ddp_affine": sig("ddp_affine", ["loss", "u", "a", "b", "v", "i_n"],
                      {"loss", "u", "a", "b", "v"}, {"v", "loss"}, {"loss"}),
    "ddp_twoparam": sig("ddp_twoparam", ["loss", "u", "w", "b", "h", "o", "i_n", "i_m"],
                        {"loss", "u", "w", "b", "h", "o"}, {"h", "o", "loss"}, {"loss"}),
    "ddp_ragged": sig("ddp_ragged", ["loss", "u", "a", "v", "i_n", "m0"],
                      {"loss", "u", "a", "v"}, {"v", "loss"}, {"loss"}),
    "ddp_branch": sig("ddp_branch", ["loss", "u", "a", "b", "v", "i_n"],
                      {"loss", "u", "a", "b", "v"}, {"v", "loss"}, {"loss"}),
    "ddp_tangent_input": sig("ddp_tangent_input", ["loss", "u", "a", "v", "i_n"],
                             {"loss", "u", "a", "v"}, {"v", "loss"}, {"loss"}),
    "ddp_batch_hist": sig("ddp_batch_hist", ["loss", "u", "a", "hist", "v", "i_n", "i_k"],
                          {"loss", "u", "a", "hist", "v"}, {"v", "hist", "loss"}, {"loss"},
                          {"hist"}),
    "affine_loss": sig("affine_loss", ["loss", "u", "a", "b", "v", "i_n"],
                       {"loss", "u", "a", "b", "v"}, {"v", "loss"}, {"loss"}),
    "matvec_loss": sig("matvec_loss", ["loss", "a", "u", "v", "i_m", "i_n"],
                       {"loss", "a", "u", "v"}, {"v", "loss"}, {"loss"}, {"v"}),
    "ddp_written_per_sample": sig("ddp_written_per_sample", ["loss", "u", "a", "v", "i_n"],
                                  {"loss", "u", "a", "v"}, {"v", "loss"}, {"loss"}),
    "ddp_ambiguous_reduce": sig("ddp_ambiguous_reduce", ["loss", "u", "a", "v", "i_n"],
                                {"loss", "u", "a", "v"}, {"v", "loss"}, {"loss"}, {"v"}),
}

EXPECTED = {
    "ddp_affine": (["u"], {}, dict(loss="reduced", lossb="seed", u="per_sample", ub="local",
                                   a="shared", ab="accum", b="shared", bb="accum", v="scratch",
                                   vb="local")),
    "ddp_twoparam": (["u"], {}, dict(loss="reduced", lossb="seed", u="per_sample", ub="local",
                                     w="shared", wb="accum", b="shared", bb="accum",
                                     h="scratch", hb="local", o="scratch", ob="local")),
    "ddp_ragged": (["u"], {}, dict(loss="reduced", lossb="seed", u="per_sample", ub="local",
                                   a="shared", ab="accum", v="scratch", vb="local")),
    "ddp_branch": (["u"], {}, dict(loss="reduced", lossb="seed", u="per_sample", ub="local",
                                   a="shared", ab="accum", b="shared", bb="accum", v="scratch",
                                   vb="local")),
    "ddp_tangent_input": (["u"], {}, dict(loss="reduced", lossb="seed", u="per_sample",
                                          ub="local", a="shared", ab="accum", v="scratch",
                                          vb="local")),
    "ddp_batch_hist": (["u"], {"reduced": ["hist"]},
                       dict(loss="reduced", lossb="seed", u="per_sample", ub="local",
                            a="shared", ab="accum", hist="reduced", histb="seed", v="scratch",
                            vb="local")),
    "affine_loss": (["u"], {}, dict(loss="reduced", lossb="seed", u="per_sample", ub="local",
                                    a="shared", ab="accum", b="shared", bb="accum", v="scratch",
                                    vb="local")),
}


@pytest.mark.parametrize("name", sorted(EXPECTED))
def test_role_table(name):
    per_sample, kw, table = EXPECTED[name]
    roles = ddp.derive_roles(SUBJECTS[name], per_sample, "adjoint", **kw)
    assert roles == table


def test_role_table_hvp_and_tangent():
    roles = ddp.derive_roles(SUBJECTS["ddp_affine"], ["u"], "hvp")
    assert roles["ad"] == "shared" and roles["abd"] == "accum" and roles["ab"] == "accum"
    assert roles["lossd"] == "reduced" and roles["lossbd"] == "seed"
    assert roles["vd"] == "scratch" and roles["vbd"] == "local"
    t = ddp.derive_roles(SUBJECTS["ddp_affine"], ["u"], "tangent")
    assert "ab" not in t and t["ad"] == "shared"


@pytest.mark.parametrize("name,per_sample,reduced,fragment", [
    ("ddp_written_per_sample", ["v"], [], "plain overwrite"),
    ("ddp_ambiguous_reduce", ["u"], [], "does not say which"),
    ("matvec_loss", ["u"], [], "does not say which"),
    ("ddp_batch_hist", ["u"], [], "does not say which"),
    ("ddp_affine", ["nosuch"], [], "not an argument"),
    ("ddp_affine", ["i_n"], [], "not a float array argument"),
    ("ddp_affine", ["u"], ["loss"], "already derived"),
    ("ddp_batch_hist", ["hist"], ["hist"], "per_sample and in reduced"),
    ("ddp_affine", ["u", "u"], [], "more than once"),
])
def test_refusals(name, per_sample, reduced, fragment):
    with pytest.raises(ValueError, match=fragment):
        ddp.derive_roles(SUBJECTS[name], per_sample, "adjoint", reduced)


@pytest.mark.parametrize("name,per_sample,reduced,arr,cls", [
    ("matvec_loss", ["u", "v"], [], "v", "scratch"),
    ("ddp_batch_hist", ["u"], ["hist"], "hist", "reduced"),
])
def test_ambiguity_resolutions(name, per_sample, reduced, arr, cls):
    assert ddp.derive_roles(SUBJECTS[name], per_sample, "adjoint", reduced)[arr] == cls


def test_benchmark_kernels_roles():
    r = ddp.derive_roles(ddp.MLP2_CE, ["x", "y"], "adjoint")
    assert ddp.role_args(ddp.MLP2_CE, r, "adjoint", "accum") == ["w1b", "b1b", "w2b", "b2b"]
    assert ddp.role_args(ddp.MLP2_CE, r, "adjoint", "reduced") == ["loss"]
    assert ddp.role_args(ddp.MLP2_CE, r, "adjoint", "local") == ["xb", "yb", "hb", "zb", "pb"]
    assert ddp.role_args(ddp.MLP2_CE, r, "adjoint", "shared") == ["w1", "b1", "w2", "b2"]
    assert ddp.role_args(ddp.MLP2_CE, r, "adjoint", "seed") == ["lossb"]
    h = ddp.derive_roles(ddp.MLP2_CE, ["x", "y"], "hvp")
    assert ddp.role_args(ddp.MLP2_CE, h, "hvp", "accum") == [
        "w1b", "b1b", "w2b", "b2b", "w1bd", "b1bd", "w2bd", "b2bd"]
    a = ddp.derive_roles(ddp.AFFINE_LS, ["x", "t"], "adjoint")
    assert ddp.role_args(ddp.AFFINE_LS, a, "adjoint", "accum") == ["wb", "bb"]
    assert ddp.role_args(ddp.AFFINE_LS, a, "adjoint", "local") == ["xb", "tb", "yb"]


@pytest.mark.parametrize("mode", ["block", "mod"])
@pytest.mark.parametrize("n,p", [(6, 2), (7, 2), (5, 4), (65536, 8), (3, 4)])
def test_shard_partition(mode, n, p):
    seen = []
    for r in range(p):
        seen += list(ddp.shard(n, r, p, mode))
    assert sorted(seen) == list(range(n))


# ---------------------------------------------------------------------------
class GlooBackend:
    """The epilogue's three operations on numpy arrays over a gloo group."""

    def __init__(self):
        import torch.distributed as dist
        self.dist = dist

    def zero(self, bufs):
        for b in bufs:
            b[...] = 0

    def allreduce_sum(self, bufs, n_local=None):
        import torch
        flat = torch.from_numpy(np.concatenate([b.ravel() for b in bufs]).astype(np.float64))
        self.dist.all_reduce(flat)
        off = 0
        for b in bufs:
            b[...] = flat[off:off + b.size].numpy().reshape(b.shape).astype(b.dtype)
            off += b.size
        if n_local is None:
            return None
        c = torch.tensor([n_local], dtype=torch.int64)
        self.dist.all_reduce(c)
        return int(c.item())

    def check(self, bufs, names):
        import torch
        s = torch.tensor([[float(np.sum(b)), float(np.sum(np.abs(b)))] for b in bufs],
                         dtype=torch.float64)
        lo, hi = s.clone(), s.clone()
        self.dist.all_reduce(lo, op=self.dist.ReduceOp.MIN)
        self.dist.all_reduce(hi, op=self.dist.ReduceOp.MAX)
        bad = [names[i] for i in range(len(bufs)) if not torch.equal(lo[i], hi[i])]
        if bad:
            raise RuntimeError(f"`{'`, `'.join(bad)}` differ across ranks")


def _affine_bank(rows, n_o, n_i, full):
    f = np.float64
    m = len(rows)
    bank = dict(loss=np.zeros(1, f), lossb=full["lossb"].copy(), w=full["w"].copy(),
                wb=np.zeros(n_o * n_i, f), b=full["b"].copy(), bb=np.zeros(n_o, f),
                x=full["x"].reshape(-1, n_i)[rows].ravel().copy(), xb=np.full(m * n_i, 7.0),
                t=full["t"].reshape(-1, n_o)[rows].ravel().copy(), tb=np.full(m * n_o, 7.0),
                y=np.zeros(m * n_o, f), yb=np.full(m * n_o, 7.0))
    return bank


def _affine_sweep(bank, m, n_o, n_i):
    from oracle import oracle as orc
    orc.affine_ls_b(bank["loss"], bank["lossb"], bank["w"], bank["wb"], bank["b"], bank["bb"],
                    bank["x"], bank["xb"], bank["t"], bank["tb"], bank["y"], bank["yb"], m, n_o,
                    n_i)


def _mlp_bank(rows, n_i, n_h, n_o, full):
    f = np.float64
    m = len(rows)
    z = lambda n: np.zeros(n, f)
    return dict(loss=z(1), lossb=full["lossb"].copy(),
                x=full["x"].reshape(-1, n_i)[rows].ravel().copy(), xb=np.full(m * n_i, 3.0),
                y=full["y"].reshape(-1, n_o)[rows].ravel().copy(), yb=np.full(m * n_o, 3.0),
                w1=full["w1"].copy(), w1b=np.full(n_i * n_h, 5.0), b1=full["b1"].copy(),
                b1b=z(n_h), w2=full["w2"].copy(), w2b=z(n_h * n_o), b2=full["b2"].copy(),
                b2b=z(n_o), h=z(m * n_h), hb=np.full(m * n_h, 2.0), z=z(m * n_o),
                zb=np.full(m * n_o, 2.0), p=z(m * n_o), pb=np.full(m * n_o, 2.0))


def _mlp_sweep(bank, m, n_i, n_h, n_o):
    from oracle import oracle as orc
    orc.mlp2_ce_b(*[bank[k] for k in ("loss", "lossb", "x", "xb", "y", "yb", "w1", "w1b", "b1",
                                       "b1b", "w2", "w2b", "b2", "b2b", "h", "hb", "z", "zb", "p",
                                       "pb")], m, n_i, n_h, n_o)


def _rank_main(rank, world, port, case, mode, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from stadeb200 import synth
        if case == "affine_ls":
            n_s, n_o, n_i = 37, 6, 5
            full = synth.affine_ls_inputs(n_s, n_o, n_i)
            rows = list(ddp.shard(n_s, rank, world, mode))
            bank = _affine_bank(rows, n_o, n_i, full)
            epi = ddp.Epilogue(ddp.AFFINE_LS, ["x", "t"], "adjoint", GlooBackend())
            sweep = lambda: _affine_sweep(bank, len(rows), n_o, n_i)
        else:
            n_s, n_i, n_h, n_o = 29, 11, 7, 4
            full = synth.mlp2_ce_inputs(n_s, n_i, n_h, n_o, dtype=np.float64)
            rows = list(ddp.shard(n_s, rank, world, mode))
            bank = _mlp_bank(rows, n_i, n_h, n_o, full)
            epi = ddp.Epilogue(ddp.MLP2_CE, ["x", "y"], "adjoint", GlooBackend())
            sweep = lambda: _mlp_sweep(bank, len(rows), n_i, n_h, n_o)
        epi.check_replicas(bank)
        epi.reset_accum(bank)
        epi.reset_reduced(bank)
        epi.reset_local(bank)
        sweep()
        n_global = epi.allreduce_accum(bank, len(rows))
        epi.allreduce_reduced(bank)
        out = {b: bank[b].copy() for b in epi.accum + epi.reduced}
        # a :shared buffer that differs on one rank is caught
        if rank == 1:
            bank[epi.checked[0]][0] += 1e-9
        try:
            epi.check_replicas(bank)
            caught = None
        except RuntimeError as e:
            caught = str(e)
        q.put((rank, n_global, out, caught))
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _single_rank(case):
    from stadeb200 import synth
    if case == "affine_ls":
        n_s, n_o, n_i = 37, 6, 5
        full = synth.affine_ls_inputs(n_s, n_o, n_i)
        bank = _affine_bank(list(range(n_s)), n_o, n_i, full)
        epi = ddp.Epilogue(ddp.AFFINE_LS, ["x", "t"], "adjoint", GlooBackend())
        epi.backend.zero([bank[b] for b in epi.accum + epi.reduced + epi.local])
        _affine_sweep(bank, n_s, n_o, n_i)
    else:
        n_s, n_i, n_h, n_o = 29, 11, 7, 4
        full = synth.mlp2_ce_inputs(n_s, n_i, n_h, n_o, dtype=np.float64)
        bank = _mlp_bank(list(range(n_s)), n_i, n_h, n_o, full)
        epi = ddp.Epilogue(ddp.MLP2_CE, ["x", "y"], "adjoint", GlooBackend())
        epi.backend.zero([bank[b] for b in epi.accum + epi.reduced + epi.local])
        _mlp_sweep(bank, n_s, n_i, n_h, n_o)
    return n_s, {b: bank[b] for b in epi.accum + epi.reduced}


@pytest.mark.parametrize("case", ["affine_ls", "mlp2_ce"])
@pytest.mark.parametrize("mode", ["mod", "block"])
def test_rank_invariance_gloo(case, mode):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, case, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        rank, n_global, out, caught = q.get(timeout=120)
        res[rank] = (n_global, out, caught)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    n_s, ref = _single_rank(case)
    for rank in (0, 1):
        n_global, out, caught = res[rank]
        assert n_global == n_s
        assert caught is not None and "differ across ranks" in caught
        for b, v in ref.items():
            err = np.max(np.abs(out[b] - v)) / max(np.max(np.abs(v)), 1e-300)
            assert err <= 1e-12, (b, err)
    # both ranks hold the same sums
    for b in ref:
        assert np.array_equal(res[0][1][b], res[1][1][b])


# ---- C4: a mean loss over sample blocks ---------------------------------------------
CONV_SIZES = (8, 3, 12, 4, 3)   # n_b, n_c, n_l, n_o, n_k


def _conv_bank(rows, dtype, factor):
    from stadeb200 import synth
    n_b, n_c, n_l, n_o, n_k = CONV_SIZES
    n_lo = n_l - n_k + 1
    full = synth.conv1d_relu_mse_inputs(*CONV_SIZES)
    rng = np.random.default_rng(5)          # the same non-zero local seeds on every rank
    seeds = {k: rng.standard_normal(n_b * n) for k, n in
             (("xb", n_c * n_l), ("tb", n_o * n_lo), ("zb", n_o * n_lo), ("rb", n_o * n_lo))}
    per = dict(x=n_c * n_l, xb=n_c * n_l, t=n_o * n_lo, tb=n_o * n_lo, zb=n_o * n_lo,
               rb=n_o * n_lo)
    lo, hi = rows.start, rows.stop
    sl = lambda a, k: np.ascontiguousarray(a[lo * per[k]:hi * per[k]]).astype(dtype)
    m = hi - lo
    return dict(loss=np.zeros(1, dtype), lossb=(full["lossb"] * factor).astype(dtype),
                x=sl(full["x"], "x"), xb=sl(seeds["xb"], "xb"), w=full["w"].astype(dtype),
                wb=np.zeros(n_o * n_c * n_k, dtype), t=sl(full["t"], "t"),
                tb=sl(seeds["tb"], "tb"), z=np.zeros(m * n_o * n_lo, dtype),
                zb=sl(seeds["zb"], "zb"), r=np.zeros(m * n_o * n_lo, dtype),
                rb=sl(seeds["rb"], "rb"))


def _conv_sweep(bank, m):
    from oracle import oracle as orc
    n_b, n_c, n_l, n_o, n_k = CONV_SIZES
    orc.conv1d_relu_mse_b(*[bank[k] for k in ("loss", "lossb", "x", "xb", "w", "wb", "t", "tb",
                                              "z", "zb", "r", "rb")], m, n_c, n_l, n_o, n_k)


def _conv_rank_main(rank, world, port, dtype, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        factor = ddp.mean_loss_factor(CONV_SIZES[0], world)
        rows = ddp.shard(CONV_SIZES[0], rank, world)
        bank = _conv_bank(rows, dtype, factor)
        epi = ddp.Epilogue(ddp.CONV1D_RELU_MSE, ["x", "t"], "adjoint", GlooBackend())
        assert epi.accum == ["wb"] and epi.reduced == ["loss"]
        epi.reset_accum(bank)
        epi.reset_reduced(bank)
        _conv_sweep(bank, len(rows))
        n_global = epi.allreduce_accum(bank, len(rows))
        epi.allreduce_reduced(bank)
        bank["loss"] *= bank["loss"].dtype.type(factor)
        q.put((rank, rows.start, rows.stop, n_global, bank))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_conv_mean_loss_shards_exactly(dtype):
    """C4 on two gloo ranks, each on its block of samples with the loss seed
    and the summed loss scaled by 1/2: every per-sample array (z, r and the
    adjoints xb, tb, zb, rb) equals the whole-batch run's rows bit for bit;
    wb and loss agree to summation order."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_conv_rank_main, args=(r, 2, port, dtype, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    n_b, n_c, n_l, n_o, n_k = CONV_SIZES
    n_lo = n_l - n_k + 1
    ref = _conv_bank(range(0, n_b), dtype, 1.0)
    _conv_sweep(ref, n_b)
    per = dict(xb=n_c * n_l, tb=n_o * n_lo, z=n_o * n_lo, zb=n_o * n_lo, r=n_o * n_lo,
               rb=n_o * n_lo)
    tol = 1e-5 if dtype == np.float32 else 1e-12
    for rank, lo, hi, n_global, bank in res:
        assert n_global == n_b
        for k, n in per.items():
            assert np.array_equal(bank[k], ref[k][lo * n:hi * n]), (rank, k)
        for k in ("wb", "loss"):
            err = np.max(np.abs(bank[k] - ref[k])) / np.max(np.abs(ref[k]))
            assert err <= tol, (rank, k, err)
    assert np.array_equal(res[0][4]["wb"], res[1][4]["wb"])


def test_mean_loss_factor_refusals():
    assert ddp.mean_loss_factor(4096, 8) == 0.125
    for n, p in ((4096, 3), (6, 4), (10, 0)):
        with pytest.raises(ValueError):
            ddp.mean_loss_factor(n, p)


# ---- C5: the hvp-mode bucket (b and bd shadows) over sample blocks ------------
def _hv_rank_main(rank, world, port, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q.put((rank,) + _hv_run(rank, world))
    finally:
        dist.destroy_process_group()


def _hv_run(rank, world):
    """One rank's hvp sweep between the epilogue's resets and sums (world = 1:
    the whole batch, no communication)."""
    import cases
    from oracle import oracle as orc
    n_s, n_i, n_h, n_o = 23, 9, 6, 4
    st, _ = cases.mlp_hv_state(n_s, n_i, n_h, n_o, seeded=True, xd_nonzero=True)
    rows = ddp.shard(n_s, rank, world)
    lo, hi = rows.start, rows.stop
    per = dict(x=n_i, xb=n_i, y=n_o, yb=n_o, h=n_h, hb=n_h, z=n_o, zb=n_o, p=n_o, pb=n_o)
    bank = {}
    for k, v in st.items():
        base = k[:-1] if k.endswith("d") and k[:-1] in per else k
        w = per.get(base)
        bank[k] = v[lo * w:hi * w].copy() if w else v.copy()
    backend = GlooBackend() if world > 1 else _NoComm()
    epi = ddp.Epilogue(ddp.MLP2_CE, ["x", "y"], "hvp", backend)
    epi.check_replicas(bank) if world > 1 else None
    epi.reset_accum(bank)
    epi.reset_reduced(bank)
    epi.reset_local(bank)
    orc.mlp2_ce_hv(*[bank[a] for a in cases.MLP_ARGS], hi - lo, n_i, n_h, n_o,
                   *[bank[a] for a in cases.MLP_TAN])
    n_global = epi.allreduce_accum(bank, hi - lo) if world > 1 else hi - lo
    if world > 1:
        epi.allreduce_reduced(bank)
    return n_global, {b: bank[b].copy() for b in epi.accum + epi.reduced}


class _NoComm:
    def zero(self, bufs):
        for b in bufs:
            b[...] = 0


def test_hvp_bucket_rank_invariance_gloo():
    """C5's epilogue in hvp mode: two gloo ranks each run the HVP sweep on
    their block of samples; the one bucket of the eight :accum shadows (b and
    bd of w1, b1, w2, b2) and the :reduced loss / lossd summed across ranks
    match one run over the whole batch (rtol 1e-12, test/validate_ddp.jl:
    160-179), and the global sample count comes back."""
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_hv_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        rank, n_global, out = q.get(timeout=120)
        res[rank] = (n_global, out)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    n_s, ref = _hv_run(0, 1)
    assert sorted(ref) == sorted(["w1b", "b1b", "w2b", "b2b", "w1bd", "b1bd", "w2bd", "b2bd",
                                  "loss", "lossd"])
    for rank in (0, 1):
        n_global, out = res[rank]
        assert n_global == n_s
        for b, v in ref.items():
            err = np.max(np.abs(out[b] - v)) / max(np.max(np.abs(v)), 1e-300)
            assert err <= 1e-12, (b, err)
            assert np.array_equal(out[b], res[0][1][b])


# ---- C3: row slabs with a halo row per neighbour per step ---------------------
def _exchange(dist, first, last, rank, world):
    """Sends this slab's first row to the rank above and its last row to the
    rank below (periodic); returns (top halo, bottom halo): the rank above's
    last row and the rank below's first row."""
    import torch
    up, down = (rank - 1) % world, (rank + 1) % world
    top, bottom = torch.empty(first.size, dtype=torch.float64), torch.empty(first.size,
                                                                             dtype=torch.float64)
    reqs = [dist.isend(torch.from_numpy(first.copy()), up, tag=1),
            dist.isend(torch.from_numpy(last.copy()), down, tag=2),
            dist.irecv(bottom, down, tag=1), dist.irecv(top, up, tag=2)]
    for r in reqs:
        r.wait()
    return top.numpy(), bottom.numpy()


def _slab_gather(a_pad, lo, rows, n, alpha):
    """ub of the slab's rows from the adjoint state a (halo-padded, rows + 2)
    by the reverse stencil loop's additions, applied per cell in the order the
    serial loop makes them (iteration index descending, then statement): the
    schedule stade_heat2d_b_f64_slab's kernels follow."""
    i = (lo + np.arange(rows))[:, None] % n
    j = np.arange(n)[None, :]
    own = a_pad[1:rows + 1]
    k_self = i * n + j
    k_b, k_a = ((i + 1) % n) * n + j, ((i - 1) % n) * n + j
    k_r, k_l = i * n + (j + 1) % n, i * n + (j - 1) % n
    a_b, a_a = alpha * a_pad[2:rows + 2], alpha * a_pad[0:rows]
    a_r, a_l = alpha * np.roll(own, -1, axis=1), alpha * np.roll(own, 1, axis=1)
    keys = np.stack([k_self + 0 * j, k_b + 0 * j, k_a + 0 * j, k_r + 0 * j, k_l + 0 * j,
                     k_self + 0 * j]).astype(np.int64)
    stmt = np.array([0, 1, 2, 3, 4, 5])[:, None, None]
    vals = np.stack([own, a_b, a_a, a_r, a_l, 4.0 * -(alpha * own)])
    order = np.lexsort((np.broadcast_to(stmt, keys.shape), -keys), axis=0)
    acc = np.zeros_like(own)
    for s in range(6):
        acc = acc + np.take_along_axis(vals, order[s:s + 1], axis=0)[0]
    return acc


def _slab_sweep(dist, rank, world, u0, n, n_step, alpha):
    """The slab form of heat2d_b on this rank's rows, as stade_heat2d_b_f64_slab
    runs it: tape slots hold each state with a halo row above and below, the
    forward exchanges the state's edge rows per step, the reverse exchanges the
    adjoint state's edge rows per step, loss and alphab are summed across
    slabs at the end."""
    lo, hi = n * rank // world, n * (rank + 1) // world
    rows = hi - lo
    pad = lambda s, top, bot: np.vstack([top[None], s, bot[None]])
    state = u0.reshape(n, n)[lo:hi].copy()
    tape = []
    for _ in range(n_step):
        top, bot = _exchange(dist, state[0], state[-1], rank, world)
        p = pad(state, top, bot)
        tape.append(p)
        c = p[1:rows + 1]
        lap = (((p[0:rows] + p[2:rows + 2]) + np.roll(c, 1, axis=1)) + np.roll(c, -1, axis=1)) \
            - 4.0 * c
        state = c + alpha * lap
    un = state
    loss = 0.0
    for v in un.ravel():
        loss = loss + v * v
    a = 0.0 + (2.0 * un)                     # unb (zero) + the loss seed's ub (lossb = 1)
    alphab = 0.0
    for t in range(n_step - 1, -1, -1):
        top, bot = _exchange(dist, a[0], a[-1], rank, world)
        a_pad = pad(a, top, bot)
        p = tape[t]
        c = p[1:rows + 1]
        lap = (((p[0:rows] + p[2:rows + 2]) + np.roll(c, 1, axis=1)) + np.roll(c, -1, axis=1)) \
            - 4.0 * c
        for v in (lap * a).ravel()[::-1]:
            alphab = alphab + v
        a = _slab_gather(a_pad, lo, rows, n, alpha)
    return lo, hi, a, un, tape, loss, alphab


def _slab_rank_main(rank, world, port, n, n_step, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from stadeb200 import synth
        u0 = synth.heat2d_inputs(n)["u"]
        lo, hi, ub, un, tape, loss, alphab = _slab_sweep(dist, rank, world, u0, n, n_step, 0.2)
        s = torch.tensor([loss, alphab], dtype=torch.float64)
        dist.all_reduce(s)
        q.put((rank, lo, hi, ub, un, tape, float(s[0]), float(s[1])))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n,n_step", [(2, 12, 3), (3, 17, 4)])
def test_heat2d_slabs_gloo(world, n, n_step):
    """C3 on row slabs across gloo ranks, emulating the GPU slab schedule:
    every rank's ub, final state and halo-padded tape slots equal the
    single-grid oracle's bit for bit (the halo rows are the neighbours' edge
    rows, periodic across the first and last rank); loss and alphab, summed
    across slabs, within 1e-12."""
    import torch.multiprocessing as mp
    from oracle import oracle as orc
    from stadeb200 import synth
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_slab_rank_main, args=(r, world, port, n, n_step, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    u = synth.heat2d_inputs(n)["u"].copy()
    z = lambda: np.zeros(n * n)
    loss, ub, un, unb, stack = np.zeros(1), z(), z(), z(), np.zeros(n_step * n * n)
    alphab = orc.heat2d_b(loss, np.ones(1), u, ub, un, unb, 0.2, 0.0, n, n_step, stack)
    tape = stack.reshape(n_step, n, n)
    for rank, lo, hi, s_ub, s_un, s_tape, s_loss, s_alphab in res:
        assert np.array_equal(s_ub, ub.reshape(n, n)[lo:hi]), rank
        assert np.array_equal(s_un, un.reshape(n, n)[lo:hi]), rank
        for t in range(n_step):
            assert np.array_equal(s_tape[t][1:-1], tape[t][lo:hi]), (rank, t)
            assert np.array_equal(s_tape[t][0], tape[t][(lo - 1) % n]), (rank, t)
            assert np.array_equal(s_tape[t][-1], tape[t][hi % n]), (rank, t)
        assert abs(s_loss - loss[0]) <= 1e-12 * abs(loss[0])
        assert abs(s_alphab - alphab) <= 1e-12 * max(1.0, abs(alphab))
