"""The generated epilogue functions of C4 (conv1d_relu_mse_b_*, adjoint mode)
and C5 (mlp2_ce_hv_*, hvp mode, the `_hv` names of ddpgen_fname,
src/STADE.jl:17578-17582) through the C ABI on a one-rank communicator: the
resets zero exactly the buffers the role table gives each role, the
all-reduces return the sample count and leave a one-rank sum unchanged, and
check_replicas accepts the :shared and :seed buffers. Two ranks are covered by
the gloo tests of the same role tables (test_ddp_host.py) and by
test_gpu_ddp_conv.py on a box with two GPUs."""
import ctypes as C

import numpy as np
import pytest
import torch

from stadeb200 import _lib, ddp

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def comm():
    L = _lib.lib()
    uid = C.create_string_buffer(128)
    _lib.check(L.stade_comm_unique_id(uid))
    c = ddp.NcclComm(0, 1, unique_id=uid.raw, timeout_ms=30000)
    yield c
    c.close()


def _bank(names, lens, dtype):
    g = torch.Generator().manual_seed(7)
    return {n: (torch.rand(lens[n], generator=g, dtype=torch.float64) + 0.5).to(dtype).cuda()
            for n in names}


def _p(t):
    return C.c_void_p(t.data_ptr())


def test_conv1d_relu_mse_b_epilogue(comm):
    L = _lib.lib()
    B, Cc, Ln, O, K = 3, 4, 20, 5, 3
    nt = B * O * (Ln - K + 1)
    lens = dict(x=B * Cc * Ln, xb=B * Cc * Ln, w=O * Cc * K, wb=O * Cc * K, t=nt, tb=nt, z=nt,
                zb=nt, r=nt, rb=nt, loss=1, lossb=1)
    bank = _bank(lens, lens, torch.float32)
    roles = ddp.derive_roles(ddp.CONV1D_RELU_MSE, ["x", "t"], "adjoint")
    role = lambda want: ddp.role_args(ddp.CONV1D_RELU_MSE, roles, "adjoint", want)
    o = C.byref(_lib.make_opts(torch.cuda.current_stream().cuda_stream))
    before = {k: v.clone() for k, v in bank.items()}
    _lib.check(L.stade_conv1d_relu_mse_b_reset_local_f32(*[_p(bank[k]) for k in role("local")],
                                                         B, Cc, Ln, O, K, o))
    _lib.check(L.stade_conv1d_relu_mse_b_reset_accum_f32(_p(bank["wb"]), O, Cc, K, o))
    torch.cuda.synchronize()
    for k in bank:
        zeroed = k in role("local") or k in role("accum")
        assert bool((bank[k] == 0).all()) == zeroed, k
        if not zeroed:
            assert torch.equal(bank[k], before[k]), k
    bank["wb"].fill_(1.5)
    n_global = C.c_int64(0)
    _lib.check(L.stade_conv1d_relu_mse_b_allreduce_accum_f32(_p(bank["wb"]), O, Cc, K, 11,
                                                             comm.handle, C.byref(n_global), o))
    _lib.check(L.stade_conv1d_relu_mse_b_allreduce_reduced_f32(_p(bank["loss"]), comm.handle, o))
    torch.cuda.synchronize()
    assert n_global.value == 11 and bool((bank["wb"] == 1.5).all())
    assert torch.equal(bank["loss"], before["loss"])
    mask = C.c_uint64(99)
    _lib.check(L.stade_conv1d_relu_mse_b_check_replicas_f32(_p(bank["w"]), _p(bank["lossb"]), O,
                                                            Cc, K, comm.handle, C.byref(mask), o))
    assert mask.value == 0
    _lib.check(L.stade_conv1d_relu_mse_b_reset_reduced_f32(_p(bank["loss"]), o))
    torch.cuda.synchronize()
    assert float(bank["loss"][0]) == 0.0
    assert role("accum") == ["wb"] and role("reduced") == ["loss"]
    assert role("shared") + role("seed") == ["w", "lossb"]


def test_mlp2_ce_hv_epilogue(comm):
    L = _lib.lib()
    S, I, H, O = 6, 5, 4, 3
    base = dict(loss=1, lossb=1, x=S * I, y=S * O, w1=I * H, b1=H, w2=H * O, b2=O, h=S * H,
                z=S * O, p=S * O)
    lens = {}
    for k, n in base.items():
        for suffix in ("", "b", "d", "bd"):
            nm = k + suffix if k != "lossb" else ("lossb" + ("d" if suffix in ("d", "bd") else ""))
            lens[nm] = n
    bank = _bank(lens, lens, torch.float64)
    roles = ddp.derive_roles(ddp.MLP2_CE, ["x", "y"], "hvp")
    role = lambda want: ddp.role_args(ddp.MLP2_CE, roles, "hvp", want)
    o = C.byref(_lib.make_opts(torch.cuda.current_stream().cuda_stream))
    before = {k: v.clone() for k, v in bank.items()}
    _lib.check(L.stade_mlp2_ce_hv_reset_local_f64(*[_p(bank[k]) for k in role("local")],
                                                  S, I, H, O, o))
    _lib.check(L.stade_mlp2_ce_hv_reset_accum_f64(*[_p(bank[k]) for k in role("accum")],
                                                  I, H, O, o))
    _lib.check(L.stade_mlp2_ce_hv_reset_reduced_f64(*[_p(bank[k]) for k in role("reduced")], o))
    torch.cuda.synchronize()
    zeroed = set(role("local") + role("accum") + role("reduced"))
    for k in bank:
        if k in zeroed:
            assert bool((bank[k] == 0).all()), k
        else:
            assert torch.equal(bank[k], before[k]), k
    for k in role("accum"):
        bank[k].fill_(2.25)
    n_global = C.c_int64(0)
    _lib.check(L.stade_mlp2_ce_hv_allreduce_accum_f64(*[_p(bank[k]) for k in role("accum")],
                                                      I, H, O, S, comm.handle, C.byref(n_global),
                                                      o))
    _lib.check(L.stade_mlp2_ce_hv_allreduce_reduced_f64(*[_p(bank[k]) for k in role("reduced")],
                                                        comm.handle, o))
    torch.cuda.synchronize()
    assert n_global.value == S
    assert all(bool((bank[k] == 2.25).all()) for k in role("accum"))
    mask = C.c_uint64(99)
    _lib.check(L.stade_mlp2_ce_hv_check_replicas_f64(
        *[_p(bank[k]) for k in role("shared") + role("seed")], I, H, O, comm.handle,
        C.byref(mask), o))
    assert mask.value == 0
    assert role("shared") + role("seed") == ["w1", "b1", "w2", "b2", "w1d", "b1d", "w2d", "b2d",
                                             "lossb", "lossbd"]


def test_ddp_zero_runs_of_adjacent_buffers():
    """stade_ddp_zero clears buffers that follow each other in memory with one
    memset per run: a mix of adjacent and separate buffers (in any order) is
    zeroed exactly, and the elements around them are left alone."""
    L = _lib.lib()
    big = torch.arange(1, 1001, dtype=torch.float32, device="cuda")
    other = torch.arange(1, 65, dtype=torch.float32, device="cuda")
    spans = [(10, 30), (30, 31), (31, 100), (200, 260), (500, 500), (600, 700)]
    bufs = [big[a:b] for a, b in spans] + [other[8:40]]
    ptrs = (C.c_void_p * len(bufs))(*[C.c_void_p(b.data_ptr()) for b in bufs])
    counts = (C.c_int64 * len(bufs))(*[b.numel() for b in bufs])
    _lib.check(L.stade_ddp_zero(ptrs, counts, len(bufs), 0, None))
    torch.cuda.synchronize()
    want = np.arange(1, 1001, dtype=np.float32)
    for a, b in spans:
        want[a:b] = 0
    want_o = np.arange(1, 65, dtype=np.float32)
    want_o[8:40] = 0
    assert np.array_equal(big.cpu().numpy(), want)
    assert np.array_equal(other.cpu().numpy(), want_o)


def test_ddp_zero_large_runs():
    """A 6 MB run of two adjacent buffers (one memset) that ends mid-array and
    not on a 16-byte boundary: cleared exactly, the bytes around it kept."""
    L = _lib.lib()
    n = (6 << 20) // 4 + 3                       # 6 MB + 12 bytes of Float32
    big = torch.full((n + 64,), 7.0, dtype=torch.float32, device="cuda")
    bufs = [big[16:16 + n // 2], big[16 + n // 2:16 + n]]   # adjacent: one run
    ptrs = (C.c_void_p * 2)(*[C.c_void_p(b.data_ptr()) for b in bufs])
    counts = (C.c_int64 * 2)(*[b.numel() for b in bufs])
    _lib.check(L.stade_ddp_zero(ptrs, counts, 2, 0, None))
    torch.cuda.synchronize()
    host = big.cpu().numpy()
    assert not np.any(host[16:16 + n])
    assert np.all(host[:16] == 7.0) and np.all(host[16 + n:] == 7.0)
