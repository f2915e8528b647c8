"""C4 over sample blocks on several GPUs (one process per GPU, NCCL through
libstade_b200): each rank runs the sweep on its block with the loss seed
scaled by 1/N (ddp.mean_loss_factor), sums wb and the loss in one bucket and
scales the loss by 1/N. Every per-sample array (z, r and the adjoints xb, tb,
zb, rb) equals the one-GPU whole-batch run's rows bit for bit; wb and the
loss agree within the Float32 tolerance 1e-5. Skipped on a box with fewer
GPUs than ranks."""
import os
import socket

import numpy as np
import pytest

import cases

pytestmark = pytest.mark.gpu

SIZES = dict(n_b=8, n_c=16, n_l=96, n_o=32, n_k=9)
PER_SAMPLE = ("xb", "tb", "z", "zb", "r", "rb")


def _per(k):
    n_lo = SIZES["n_l"] - SIZES["n_k"] + 1
    return SIZES["n_c"] * SIZES["n_l"] if k in ("x", "xb") else SIZES["n_o"] * n_lo


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    comm = None
    try:
        import stadeb200
        from stadeb200 import ddp
        comm = ddp.NcclComm(rank, world, timeout_ms=60000)
        factor = ddp.mean_loss_factor(SIZES["n_b"], world)
        rows = ddp.shard(SIZES["n_b"], rank, world)
        st, _ = cases.conv_state(**SIZES, seeded=True)
        st["loss"][:] = 0
        st["wb"][:] = 0
        st["lossb"] = (st["lossb"] * np.float32(factor)).astype(np.float32)
        for k in ("x", "t") + PER_SAMPLE:
            st[k] = np.ascontiguousarray(st[k][rows.start * _per(k):rows.stop * _per(k)])
        dev = {k: torch.from_numpy(v).cuda() for k, v in st.items()}
        stadeb200.conv1d_relu_mse_b_cuda(*[dev[a] for a in cases.CONV_ARGS], len(rows),
                                         SIZES["n_c"], SIZES["n_l"], SIZES["n_o"], SIZES["n_k"])
        ddp.allreduce_sum_(comm, dev["wb"], dev["loss"])
        dev["loss"].mul_(factor)
        torch.cuda.synchronize()
        q.put((rank, rows.start, rows.stop, {k: v.cpu().numpy() for k, v in dev.items()}, None))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, 0, 0, None, repr(e)))
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_conv_sample_blocks_match_one_gpu(world):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    full, ints = cases.conv_state(**SIZES, seeded=True)
    full["loss"][:] = 0
    full["wb"][:] = 0
    cases.gpu_conv(full, ints)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=120)
    errs = [r[4] for r in res if r[4]]
    assert not errs, errs
    for rank, lo, hi, out, _ in res:
        for k in PER_SAMPLE:
            assert np.array_equal(out[k], full[k][lo * _per(k):hi * _per(k)]), (rank, k)
        for k in ("wb", "loss"):
            err = np.max(np.abs(out[k] - full[k])) / np.max(np.abs(full[k]))
            assert err <= 1e-5, (rank, k, err)
    for p in procs:
        assert p.exitcode == 0
