"""C3 on row slabs (stade_heat2d_b_f64_slab): the grid split into one slab of
rows per rank with a halo row exchanged with each neighbour per step.

Every cell goes through the same arithmetic as in the one-GPU sweep, so the
fields (ub, un, unb, the tape's owned rows) match the one-GPU path bit for
bit; loss and alphab are sums over slabs and agree within the Float64
tolerance 1e-12. The multi-rank cases run one process per GPU (NCCL through
libstade_b200) and are skipped on a box with fewer GPUs.
"""
import os
import socket

import numpy as np
import pytest

import cases

pytestmark = pytest.mark.gpu

F64_TOL = 1e-12


def _full_gpu(n, n_step, seeded):
    st, ints = cases.heat_state(n, n_step, seeded=seeded)
    u0 = st["u"].copy()
    ab = cases.gpu_heat(st, ints)
    return st, ints, ab, u0


def _slab_run(st0, ints, rows_lo, rows, comm):
    import torch
    import stadeb200
    n, n_step = ints["n"], ints["n_step"]
    sl = slice(rows_lo * n, (rows_lo + rows) * n)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()
    loss = dev(st0["loss"].copy())
    lossb = dev(st0["lossb"])
    u, ub = dev(st0["u"][sl]), dev(st0["ub"][sl])
    un, unb = dev(np.zeros(rows * n)), dev(st0["unb"][sl])
    ab = dev(np.array([ints["alphab"]]))
    stack = stadeb200.initstacks_heat2d_b_slab_cuda(n, n_step, rows)
    stadeb200.heat2d_b_slab_cuda(loss, lossb, u, ub, un, unb, ints["alpha"], ab, n, n_step, stack,
                                 rows, comm)
    torch.cuda.synchronize()
    tape = stack.cpu().numpy()
    owned = None
    if n_step > 0:
        owned = tape.reshape(n_step, rows + 2, n)[:, 1:rows + 1, :].copy()
    return dict(loss=loss.cpu().numpy(), u=u.cpu().numpy(), ub=ub.cpu().numpy(),
                un=un.cpu().numpy(), unb=unb.cpu().numpy(), alphab=float(ab.cpu().numpy()[0]),
                tape=owned)


@pytest.mark.parametrize("n,n_step,seeded", [(64, 4, True), (34, 3, False), (6, 2, True),
                                             (258, 5, True), (4, 1, True), (10, 0, True)])
def test_single_slab_matches_grid_path(n, n_step, seeded):
    st0, ints = cases.heat_state(n, n_step, seeded=seeded)
    full, _, ab_full, _ = _full_gpu(n, n_step, seeded)
    out = _slab_run(st0, ints, 0, n, None)
    for k in ("u", "un", "unb", "ub"):
        assert np.array_equal(out[k], full[k]), k
    if n_step > 0:
        assert np.array_equal(out["tape"].ravel(), full["u_stack"][:n_step * n * n])
    assert abs(out["loss"][0] - full["loss"][0]) <= F64_TOL * abs(full["loss"][0])
    assert abs(out["alphab"] - ab_full) <= F64_TOL * max(1.0, abs(ab_full))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, n, n_step, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    comm = None
    try:
        from stadeb200 import ddp
        comm = ddp.NcclComm(rank, world, timeout_ms=60000)
        st0, ints = cases.heat_state(n, n_step, seeded=True)
        lo, hi = n * rank // world, n * (rank + 1) // world
        out = _slab_run(st0, ints, lo, hi - lo, comm)
        q.put((rank, lo, hi, out, None))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, 0, 0, None, repr(e)))
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n,n_step", [(2, 64, 4), (2, 258, 5), (2, 8, 3), (4, 130, 3),
                                            (4, 8, 2)])
def test_slabs_across_gpus_match_grid_path(world, n, n_step):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    full, ints, ab_full, _ = _full_gpu(n, n_step, True)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, n, n_step, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    errs = [r[4] for r in res if r[4]]
    assert not errs, errs
    for rank, lo, hi, out, _ in res:
        sl = slice(lo * n, hi * n)
        for k in ("u", "un", "unb", "ub"):
            assert np.array_equal(out[k], full[k][sl]), (rank, k)
        tape = full["u_stack"][:n_step * n * n].reshape(n_step, n, n)[:, lo:hi, :]
        assert np.array_equal(out["tape"], tape), rank
        assert abs(out["loss"][0] - full["loss"][0]) <= F64_TOL * abs(full["loss"][0])
        assert abs(out["alphab"] - ab_full) <= F64_TOL * max(1.0, abs(ab_full))
    for p in procs:
        assert p.exitcode == 0
