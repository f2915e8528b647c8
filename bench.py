#!/usr/bin/env python
"""Benchmark of libstade_b200 on the configurations of BASELINE.json.

Default workload: configuration C2 (the config the
headline metric "adjoint grad-evals/sec at 1/2/4/8 B200" is quoted on for
data parallelism): the adjoint of a 2-layer tanh MLP 784-512-10 with softmax
cross-entropy, Float32, global mini-batch 65,536 samples. One step = one
data-parallel gradient evaluation of the whole global batch:
reset_accum / reset_reduced / reset_local (the generated epilogue's zeroing),
the adjoint sweep on this rank's block of samples, and (N > 1) the NCCL sum of
the :accum bucket and of the loss. With N GPUs each rank owns 65,536 / N
samples (strong scaling: the grad-eval is fixed, its work is split).

Also selectable with --config: heat2d (C3; row slabs with a halo exchange per
step at N > 1), affine_ls (C1; replicas at N > 1), mlp2_ce_hv (C5; sample
blocks), conv1d_relu_mse (C4; sample blocks, the mean loss's seed and sum
scaled by 1/N). The default run at N = 1 also measures C1, C3, C4 and C5 the
same way and reports them under "configs" (C2 stays the headline value).

--impl reference times the reference's CPU implementation of the path: the
oracle (the generated sweep restated in C++, OpenMP over all host threads)
on inputs from the oracle's own generator, one whole grad-eval per step for
C1, C2 and C5; no product library is loaded on that arm.

    python bench.py [--gpus N --steps K --warmup W] [--config NAME] [--impl reference]
    python bench.py --config affine_ls|heat2d --impl emitted

Rank 0 prints one JSON line. Timing: W untimed warm-up steps, then exactly K
steps between a barrier + synchronize on both sides; each step is bracketed by
CUDA events on the launching stream and the L2 is flushed (256 MiB write)
between steps, outside the events; the reported time is the max over ranks.
`e2e` times the same step through the public Python / C-ABI entry points with
the step's inputs copied from pinned host memory and the gradient and loss
copied back, inside the timed region.
"""
from __future__ import annotations

import argparse
import gc
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "stade.jl_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "adjoint grad-evals/sec at 1/2/4/8 B200; % of HBM or tensor-pipe roofline"
UNIT = "grad-evals/s"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
L2_FLUSH_BYTES = 256 << 20
L2_BYTES = 126 * 1000 * 1000  # B200 L2; a rank whose step inputs are smaller gets its L2 flushed


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference", "emitted"], default="ours",
                    help="emitted: C1 / C3 through the .cu emitter's output for the "
                         "generated sweep text (one GPU)")
    ap.add_argument("--config", default="mlp2_ce",
                    choices=["mlp2_ce", "heat2d", "affine_ls", "mlp2_ce_hv", "conv1d_relu_mse"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-graph", action="store_true",
                    help="time eager launches instead of a replayed CUDA graph of one step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="N = 1 default run: skip the C1 / C3 / C4 / C5 blocks of \"configs\"")
    ap.add_argument("--cpu-seconds", type=float, default=12.0,
                    help="target length of the CPU-baseline sample")
    return ap.parse_args()


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return {k: float(d[k]) for k in FALLBACK_PEAKS}, "measured"
    except Exception:
        return dict(FALLBACK_PEAKS), "fallback"


# ---------------------------------------------------------------------------
class ClockSampler:
    """nvidia-smi clock / throttle samples of this rank's GPU during the timed
    region (200 ms period)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap,"
              "timestamp")

    def __init__(self, device_index: int):
        self.proc = None
        self.lines = []
        try:
            import torch
            uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            sel = uuid if uuid.startswith("GPU-") else "GPU-" + uuid
        except Exception:
            sel = str(device_index)
        self.cmd = ["nvidia-smi", "-i", sel, f"--query-gpu={self.FIELDS}",
                    "--format=csv,noheader,nounits", "-lms", "200"]

    def start(self):
        """Starts sampling; call well before the timed region (nvidia-smi's
        start-up must not overlap the timing) and bracket each timed region
        with mark_begin / mark_end (summary(i) covers the i-th)."""
        self.windows = []
        self._t0 = None
        try:
            self.proc = subprocess.Popen(self.cmd, stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def mark_begin(self):
        self._t0 = time.time()

    def mark_end(self):
        self.windows.append((self._t0, time.time()))
        return len(self.windows) - 1

    def stop(self):
        if not self.proc:
            return
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self, i=0):
        import datetime
        window = self.windows[i] if i < len(self.windows) else None
        rows = []
        for l in self.lines:
            parts = [p.strip() for p in l.split(",")]
            if len(parts) < 10:
                continue
            try:
                ts = datetime.datetime.strptime(parts[9], "%Y/%m/%d %H:%M:%S.%f").timestamp()
            except ValueError:
                ts = None
            if window and ts is not None and not (window[0] - 0.25 <= ts <= window[1] + 0.25):
                continue
            try:
                rows.append(dict(sm=float(parts[1]), smax=float(parts[2]),
                                 power=float(parts[3]) if parts[3] not in ("[N/A]", "") else 0.0,
                                 hw=parts[5], hwt=parts[6], swt=parts[7], pcap=parts[8]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no nvidia-smi samples"]}
        smax = max(r["smax"] for r in rows)
        loaded = [r for r in rows if r["power"] > 250.0] or rows
        reasons = set()
        for r in loaded:
            for key, name in (("hw", "hw_slowdown"), ("hwt", "hw_thermal_slowdown"),
                              ("swt", "sw_thermal_slowdown"), ("pcap", "sw_power_cap")):
                if r[key].lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(r["sm"] for r in loaded), "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(rows), "samples_under_load": len(loaded)}


# ---------------------------------------------------------------------------
def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def timed_loop(torch, step, steps, warmup, world, dist, flush, stream):
    """W warm-up steps, barrier + sync, K steps, barrier + sync. With `flush`
    (workloads whose inputs fit in L2) each step sits between CUDA events on
    the launching stream and the L2 is flushed between steps, outside the
    events; without it (inputs larger than L2) one event pair brackets all K
    steps back to back, gaps included. Returns (max-over-ranks total ms,
    per-step ms list)."""
    if flush is not None:
        flush.add_(1)   # the flush kernel's first launch (module load) happens here
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    # the interpreter's cycle collector pauses for ~10 ms at a time; a pause
    # on one rank inside the timed steps holds every rank at the next
    # all-reduce, so it is run before the timing and held off during it
    gc.collect()
    gc.disable()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    h0 = time.perf_counter()
    if flush is None:
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        for _ in range(steps):
            step()
        t1.record(stream)
        host = time.perf_counter() - h0
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        total = t0.elapsed_time(t1)
        per = [total / steps] * steps
    else:
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(steps)]
        for i in range(steps):
            flush.add_(1)
            evs[i][0].record(stream)
            step()
            evs[i][1].record(stream)
        host = time.perf_counter() - h0
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        per = [a.elapsed_time(b) for a, b in evs]
        total = sum(per)
    gc.enable()
    timed_loop.host_ms = host * 1e3   # host time to enqueue the K steps (this rank)
    if world > 1:
        t = torch.tensor([total, timed_loop.host_ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total, timed_loop.host_ms = float(t[0].item()), float(t[1].item())
    return total, per


def roofline(phases, phase_work, steps, peaks, peak_src, traffic):
    """Dominant phase by device time; achieved = algorithmic work per launch /
    average launch time."""
    best = None
    for name, (ms, cnt) in phases.items():
        if name not in phase_work or cnt == 0:
            continue
        if best is None or ms > best[1]:
            best = (name, ms, cnt)
    if best is None:
        return None
    name, ms, cnt = best
    kind, work, note = phase_work[name]
    avg_s = ms / cnt / 1e3
    if kind == "hbm":
        achieved = work / avg_s / 1e9
        peak = peaks["hbm_gbs"]
        unit = "GB/s"
    elif kind == "fp64":
        # the Float64 tensor-core rate measured in this run (cuBLAS DGEMM,
        # fp64_peak()); MEASURED_PEAKS.json carries no Float64 figure
        achieved = work / avg_s / 1e12
        peak = peaks.get("fp64_tflops") or 37.2
        unit = "TFLOP/s"
        peak_src = peaks.get("fp64_source", "nominal fp64 (no measured figure)")
    else:
        achieved = work / avg_s / 1e12
        peak = peaks["bf16_tflops"]
        unit = "TFLOP/s"
    total_ms = sum(v[0] for v in phases.values())
    extra = {}
    if kind == "tensor":
        # 3xTF32: three TF32 MMAs per product, TF32 at half the bf16 rate
        ceil = peak / 6.0
        extra = {"ceiling_3xtf32": ceil, "frac_of_3xtf32_ceiling": achieved / ceil}
    t = traffic.get(name) if traffic else None
    return {**{"bound": "hbm" if kind == "hbm" else "tensor", "pipe": kind, "kernel": name,
            "achieved": achieved,
            "peak": peak, "unit": unit, "frac": achieved / peak, "peak_source": peak_src,
            "traffic": t,
            "launch_ms": ms / cnt, "share_of_step": ms / total_ms if total_ms else None,
            "note": note}, **extra}


def fp64_peak(torch, n=8192, reps=5):
    """Float64 GEMM throughput of this GPU: cuBLAS DGEMM (torch.matmul) on
    n x n x n, best of `reps` launches after one warm-up, CUDA events on the
    current stream. The denominator of the Float64 (DMMA) phases' roofline."""
    a = torch.randn(n, n, dtype=torch.float64, device="cuda")
    b = torch.randn(n, n, dtype=torch.float64, device="cuda")
    c = a @ b
    torch.cuda.synchronize()
    best = None
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch.matmul(a, b, out=c)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        best = ms if best is None else min(best, ms)
    del a, b, c
    return 2.0 * n ** 3 / (best / 1e3) / 1e12


def load_traffic(config):
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(config, {})
    except Exception:
        return {}


# ---------------------------------------------------------------------------
# The CPU side (the reference arm and each line's cpu_baseline): the oracle,
# the generated sweeps restated in C++ (oracle/oracle.cc) with OpenMP over
# samples (C3: over grid cells, bit-identical to the serial sweep), on inputs
# from the oracle's own restatement of the generator, so this side never
# loads the product library.
FULL_UNITS = {"affine_ls": (1, "evaluation"), "mlp2_ce": (65536, "samples"),
              "heat2d": (16, "time steps of the 8192^2 grid"),
              "conv1d_relu_mse": (4096, "samples"), "mlp2_ce_hv": (16384, "samples")}


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


class CpuSweep:
    """One configuration's oracle sweep over `units` of one grad-eval's work
    (FULL_UNITS: samples of the batch, or time steps of the C3 grid), inputs
    drawn once; run() times one sweep."""

    def __init__(self, config, units, threads):
        import numpy as np
        from oracle import oracle as orc
        self.config, self.units, self.threads = config, units, threads
        self.orc, self.np = orc, np
        g = orc.generator()
        full = _synth_full()[config]
        z = lambda n, dt: np.zeros(n, dt)
        if config == "affine_ls":
            S, O, I = full["n_s"], full["n_o"], full["n_i"]
            d = g.affine_ls_inputs(S, O, I)
            f = np.float64
            self.args = [z(1, f), d["lossb"], d["w"], z(O * I, f), d["b"], z(O, f), d["x"],
                         z(S * I, f), d["t"], z(S * O, f), z(S * O, f), z(S * O, f), S, O, I]
        elif config in ("mlp2_ce", "mlp2_ce_hv"):
            S, I, H, O = units, full["n_i"], full["n_h"], full["n_o"]
            if config == "mlp2_ce":
                d, f = g.mlp2_ce_inputs(S, I, H, O), np.float32
            else:
                d, f = g.mlp2_ce_hv_inputs(S, I, H, O, kernel="mlp2_ce_hv"), np.float64
            lens = dict(loss=1, x=S * I, y=S * O, w1=I * H, b1=H, w2=H * O, b2=O, h=S * H, z=S * O,
                        p=S * O)
            names = ["loss", "lossb", "x", "xb", "y", "yb", "w1", "w1b", "b1", "b1b", "w2", "w2b",
                     "b2", "b2b", "h", "hb", "z", "zb", "p", "pb"]

            def arr(nm, tan=False):
                key = nm + ("d" if tan else "")
                if key in d:
                    return d[key]
                base = nm[:-1] if nm not in lens and nm != "lossb" else nm
                return z(1 if nm == "lossb" else lens[base], f)
            self.args = [arr(a) for a in names] + [S, I, H, O]
            if config == "mlp2_ce_hv":
                tan = [arr(a, True) for a in names]
                tan[1] = d["lossbd"]   # lossbd
                self.args += tan
        elif config == "heat2d":
            n = full["n"]
            d = g.heat2d_inputs(n)
            f = np.float64
            self.args = [z(1, f), d["lossb"], d["u"], z(n * n, f), z(n * n, f), z(n * n, f),
                         full["alpha"], 0.0, n, units, z(units * n * n, f)]
        elif config == "conv1d_relu_mse":
            B, C, L, O, K = units, full["n_c"], full["n_l"], full["n_o"], full["n_k"]
            d = g.conv1d_relu_mse_inputs(B, C, L, O, K)
            nt, f = B * O * (L - K + 1), np.float32
            self.args = [z(1, f), d["lossb"], d["x"], z(B * C * L, f), d["w"], z(O * C * K, f),
                         d["t"], z(nt, f), z(nt, f), z(nt, f), z(nt, f), z(nt, f), B, C, L, O, K]
        else:
            raise ValueError(config)

    def run(self):
        orc, c, t = self.orc, self.config, self.threads
        t0 = time.perf_counter()
        if c == "affine_ls":
            orc.affine_ls_b(*self.args)
        elif c == "mlp2_ce":
            orc.mlp2_ce_b(*self.args, threads=t)
        elif c == "mlp2_ce_hv":
            orc.mlp2_ce_hv(*self.args, threads=t)
        elif c == "heat2d":
            orc.heat2d_b(*self.args, threads=t)
        else:
            orc.conv1d_relu_mse_b(*self.args, threads=t)
        return time.perf_counter() - t0

    def describe(self):
        full, what = FULL_UNITS[self.config]
        par = (f"OpenMP over {'grid cells' if self.config == 'heat2d' else 'samples'}, "
               f"{self.threads} threads") if self.threads > 1 else "serial"
        part = ("the whole grad-eval" if self.units >= full else
                f"{self.units} of {full} {what}, scaled to the whole grad-eval")
        return f"{part} (oracle.cc, the generated sweep restated; {par})"


def _synth_full():
    from stadeb200.synth import FULL
    return FULL


def cpu_baseline(config, seconds):
    """The oracle timed on the host on a bounded sample of the configuration
    (about `seconds` of work, at most the whole grad-eval); grad-evals/s."""
    full, _ = FULL_UNITS[config]
    threads = 1 if config == "affine_ls" else cpu_threads()
    if config == "affine_ls":
        sw = CpuSweep(config, 1, threads)
        reps, t = 0, 0.0
        while t < min(seconds, 3.0):
            t += sw.run()
            reps += 1
        return {"value": reps / t, "unit": UNIT, "cores": 1, "kind": "port",
                "sample": f"{reps} whole grad-evals, {t:.2f} s (oracle.cc, the generated sweep "
                          "restated; serial: 1.6 MB of work per evaluation)"}
    probe = {"mlp2_ce": 4 * threads, "mlp2_ce_hv": 2 * threads, "heat2d": 1,
             "conv1d_relu_mse": threads}[config]
    t0 = CpuSweep(config, probe, threads).run()
    units = int(min(full, max(probe, probe * seconds / max(t0, 1e-3))))
    if config == "heat2d":
        units = max(1, min(full, units))
    sw = CpuSweep(config, units, threads)
    t = sw.run()
    return {"value": (units / full) / t, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": sw.describe() + f", {t:.2f} s"}


# ---------------------------------------------------------------------------
# Workloads
class Mlp2Ce:
    name = "mlp2_ce"
    dtype = "f32"
    scaling = "strong"

    def __init__(self, torch, rank, world, comm_factory):
        import numpy as np
        from stadeb200 import synth, kernels, ddp
        self.torch, self.np, self.kernels, self.ddp = torch, np, kernels, ddp
        self.world = world
        c = synth.FULL["mlp2_ce"]
        self.G, self.n_i, self.n_h, self.n_o = c["n_s"], c["n_i"], c["n_h"], c["n_o"]
        rng = ddp.shard(self.G, rank, world)
        self.n_s = len(rng)
        lo, hi = rng.start, rng.stop
        d = synth.mlp2_ce_inputs(self.G, self.n_i, self.n_h, self.n_o)
        f32 = torch.float32
        dev = "cuda"
        self.host = {k: torch.from_numpy(v) for k, v in d.items()}
        self.host["x"] = self.host["x"][lo * self.n_i:hi * self.n_i].contiguous()
        self.host["y"] = self.host["y"][lo * self.n_o:hi * self.n_o].contiguous()
        self.pinned = {k: v.pin_memory() for k, v in self.host.items()}
        t = {k: v.to(dev) for k, v in self.host.items()}
        S, I, H, O = self.n_s, self.n_i, self.n_h, self.n_o
        z = lambda n: torch.zeros(n, dtype=f32, device=dev)
        t.update(h=z(S * H), zz=z(S * O), p=z(S * O))
        # the local shadows back to back too: reset_local! clears them with one memset
        local = z(S * I + S * O + S * H + S * O + S * O)
        off = 0
        for k, n in (("xb", S * I), ("yb", S * O), ("hb", S * H), ("zb", S * O), ("pb", S * O)):
            t[k] = local[off:off + n]
            off += n
        # the :accum shadows and the :reduced loss back to back in one allocation:
        # the step sums them with one NCCL all-reduce in place (no gather /
        # scatter into a bucket)
        self.bucket = z(I * H + H + H * O + O + 1)
        off = 0
        for k, n in (("w1b", I * H), ("b1b", H), ("w2b", H * O), ("b2b", O), ("loss", 1)):
            t[k] = self.bucket[off:off + n]
            off += n
        self.t = t
        self.ws = torch.empty(kernels.mlp2_ce_b_workspace(S, I, H, O), dtype=torch.uint8, device=dev)
        self.comm = comm_factory() if world > 1 else None
        self.grad_host = {k: torch.empty(t[k].numel(), dtype=f32).pin_memory()
                          for k in ("w1b", "b1b", "w2b", "b2b", "loss")}
        self.flush_l2 = self.static_flush(world)

    def step(self):
        t, d = self.t, self.ddp
        d.mlp2_ce_b_reset_accum_(t["w1b"], t["b1b"], t["w2b"], t["b2b"])
        d.mlp2_ce_b_reset_reduced_(t["loss"])
        d.mlp2_ce_b_reset_local_(t["xb"], t["yb"], t["hb"], t["zb"], t["pb"])
        self.kernels.mlp2_ce_b_cuda(t["loss"], t["lossb"], t["x"], t["xb"], t["y"], t["yb"],
                                    t["w1"], t["w1b"], t["b1"], t["b1b"], t["w2"], t["w2b"],
                                    t["b2"], t["b2b"], t["h"], t["hb"], t["zz"], t["zb"], t["p"],
                                    t["pb"], self.n_s, self.n_i, self.n_h, self.n_o,
                                    workspace=self.ws)
        if self.comm is not None:
            # :accum and :reduced are summed every step here, so one collective
            d.allreduce_sum_(self.comm, t["w1b"], t["b1b"], t["w2b"], t["b2b"], t["loss"])

    E2E_CHUNKS = 8

    def e2e_step(self):
        """The grad-eval from host buffers, pipelined as a caller would: the
        batch's rows go up in 8 chunks on a copy stream while the sweep runs on
        the chunks already there (the sweep accumulates its weight gradients
        and loss, so chunk calls add up to the whole-batch call)."""
        torch, t, p, d = self.torch, self.t, self.pinned, self.ddp
        main = torch.cuda.current_stream()
        if not hasattr(self, "copy_stream"):
            self.copy_stream = torch.cuda.Stream()
            self.copied = [torch.cuda.Event() for _ in range(self.E2E_CHUNKS)]
        for k in ("w1", "b1", "w2", "b2"):
            t[k].copy_(p[k], non_blocking=True)
        d.mlp2_ce_b_reset_accum_(t["w1b"], t["b1b"], t["w2b"], t["b2b"])
        d.mlp2_ce_b_reset_reduced_(t["loss"])
        d.mlp2_ce_b_reset_local_(t["xb"], t["yb"], t["hb"], t["zb"], t["pb"])
        S, I, H, O = self.n_s, self.n_i, self.n_h, self.n_o
        bounds = [S * c // self.E2E_CHUNKS for c in range(self.E2E_CHUNKS + 1)]
        self.copy_stream.wait_stream(main)   # the previous step's use of x and y is done
        with torch.cuda.stream(self.copy_stream):
            for c in range(self.E2E_CHUNKS):
                lo, hi = bounds[c], bounds[c + 1]
                t["x"][lo * I:hi * I].copy_(p["x"][lo * I:hi * I], non_blocking=True)
                t["y"][lo * O:hi * O].copy_(p["y"][lo * O:hi * O], non_blocking=True)
                self.copied[c].record(self.copy_stream)
        for c in range(self.E2E_CHUNKS):
            lo, hi = bounds[c], bounds[c + 1]
            main.wait_event(self.copied[c])
            sl = lambda k, w: t[k][lo * w:hi * w]
            self.kernels.mlp2_ce_b_cuda(t["loss"], t["lossb"], sl("x", I), sl("xb", I), sl("y", O),
                                        sl("yb", O), t["w1"], t["w1b"], t["b1"], t["b1b"], t["w2"],
                                        t["w2b"], t["b2"], t["b2b"], sl("h", H), sl("hb", H),
                                        sl("zz", O), sl("zb", O), sl("p", O), sl("pb", O),
                                        hi - lo, I, H, O, workspace=self.ws)
        if self.comm is not None:
            d.allreduce_sum_(self.comm, t["w1b"], t["b1b"], t["w2b"], t["b2b"], t["loss"])
        for k, v in self.grad_host.items():
            v.copy_(t[k], non_blocking=True)

    e2e_note = ("inputs and weights up every step; the weight gradients and the loss come "
                "back (a data-parallel caller's view); xb, which the sweep also writes, stays on "
                "the device")

    def e2e_bytes(self):
        h2d = sum(self.pinned[k].numel() * 4 for k in ("x", "y", "w1", "b1", "w2", "b2"))
        d2h = sum(v.numel() * 4 for v in self.grad_host.values())
        return h2d, d2h

    def phase_work(self):
        S, I, H, O = self.n_s, self.n_i, self.n_h, self.n_o
        gemm = 2.0 * S * I * H
        return {"fwd_gemm": ("tensor", gemm, "x W1 (2 S I H flops), tanh epilogue"),
                "w1b_gemm": ("tensor", gemm + S * H, "x^T s1b + colsum (2 S I H + S H flops)"),
                "xb_gemm": ("tensor", gemm, "s1b W1^T (2 S I H flops)"),
                "head": ("hbm", 4.0 * S * H * 4 + 8.0 * S * O * 4,
                         "reads h, hb; writes s1b, hb (4 S H floats) + per-class arrays"),
                "w2b": ("hbm", 4.0 * S * H + 4.0 * S * O, "reads h and g once")}

    @staticmethod
    def static_flush(world):
        c = _synth_full()["mlp2_ce"]
        S = c["n_s"] // world
        return 4 * (S * (c["n_i"] + c["n_o"]) + c["n_i"] * c["n_h"] + c["n_h"] +
                    c["n_h"] * c["n_o"] + c["n_o"] + 1) < L2_BYTES

    @classmethod
    def static_config(cls, world):
        c = _synth_full()["mlp2_ce"]
        return {"workload": "C2 mlp2_ce_b: 2-layer tanh MLP 784-512-10 softmax cross-entropy "
                            "adjoint, Float32, per-sample shadow-weight accumulation",
                "global_batch": c["n_s"], "per_rank_batch": c["n_s"] // world, "n_i": c["n_i"],
                "n_h": c["n_h"], "n_o": c["n_o"], "parallelism": f"dp{world}",
                "l2": ("L2 flushed between timed steps (256 MiB write outside the events)"
                       if cls.static_flush(world) else
                       "inputs larger than L2, steps timed back to back")}

    def config(self):
        return self.static_config(self.world)

class Heat2d:
    """C3. At N = 1 the generated signature (stade_heat2d_b_f64) on the whole
    grid; at N > 1 the grid's rows split into one slab per rank
    (stade_heat2d_b_f64_slab, a halo row to each neighbour per step over
    NCCL): the grad-eval is fixed and its work split (strong scaling)."""
    name = "heat2d"
    dtype = "f64"
    scaling = "strong"

    def __init__(self, torch, rank, world, comm_factory):
        import numpy as np
        from stadeb200 import synth, kernels
        self.torch, self.np, self.kernels = torch, np, kernels
        c = synth.FULL["heat2d"]
        self.n, self.n_step, self.alpha = c["n"], c["n_step"], c["alpha"]
        self.world = world
        n = self.n
        lo, hi = n * rank // world, n * (rank + 1) // world
        self.rows = hi - lo
        m = self.rows * n
        d = synth.heat2d_inputs(n)
        f64 = torch.float64
        self.pinned = {"u": torch.from_numpy(d["u"][lo * n:hi * n].copy()).pin_memory()}
        z = lambda k: torch.zeros(k, dtype=f64, device="cuda")
        self.t = dict(loss=z(1), lossb=torch.ones(1, dtype=f64, device="cuda"),
                      u=self.pinned["u"].to("cuda"), ub=z(m), un=z(m), unb=z(m), alphab=z(1))
        self.comm = comm_factory() if world > 1 else None
        if world > 1:
            self.stack = kernels.initstacks_heat2d_b_slab_cuda(n, self.n_step, self.rows)
            ws = kernels.heat2d_b_slab_workspace(n, self.n_step, self.rows)
        else:
            self.stack = kernels.initstacks_heat2d_b_cuda(n, self.n_step)
            ws = kernels.heat2d_b_workspace(n, self.n_step)
        self.ws = torch.empty(ws, dtype=torch.uint8, device="cuda")
        self.out_host = torch.empty(m, dtype=f64).pin_memory()
        self.ab_host = torch.empty(1, dtype=f64).pin_memory()
        self.flush_l2 = self.static_flush(world)

    def step(self):
        t = self.t
        t["ub"].zero_()
        t["loss"].zero_()
        t["alphab"].zero_()
        if self.comm is None:
            self.kernels.heat2d_b_cuda_device(t["loss"], t["lossb"], t["u"], t["ub"], t["un"],
                                              t["unb"], self.alpha, t["alphab"], self.n,
                                              self.n_step, self.stack, workspace=self.ws)
        else:
            self.kernels.heat2d_b_slab_cuda(t["loss"], t["lossb"], t["u"], t["ub"], t["un"],
                                            t["unb"], self.alpha, t["alphab"], self.n,
                                            self.n_step, self.stack, self.rows, self.comm,
                                            workspace=self.ws)

    def e2e_step(self):
        self.t["u"].copy_(self.pinned["u"], non_blocking=True)
        self.step()
        self.out_host.copy_(self.t["ub"], non_blocking=True)
        self.ab_host.copy_(self.t["alphab"], non_blocking=True)

    def e2e_bytes(self):
        # per rank; the caller multiplies by the rank count for strong scaling
        return self.rows * self.n * 8, self.rows * self.n * 8 + 8

    def phase_work(self):
        N = float(self.rows) * self.n
        return {"fwd_step": ("hbm", 16.0 * N, "read u_k, write u_k+1 (tape)"),
                "bwd_step": ("hbm", 24.0 * N, "read unb_k, read tape u_k-1, write ub_k-1"),
                "bwd_init": ("hbm", 32.0 * N, "read ub, unb, u_final; write seed")}

    @staticmethod
    def static_flush(world):
        n = _synth_full()["heat2d"]["n"]
        return (n // world) * n * 8 < L2_BYTES

    @classmethod
    def static_config(cls, world):
        c = _synth_full()["heat2d"]
        return {"workload": "C3 heat2d_b: periodic 5-point heat adjoint, 8192^2 Float64, 16 taped "
                            "steps, alpha 0.2", "n": c["n"], "n_step": c["n_step"],
                "rows_per_rank": c["n"] // world,
                "parallelism": f"slabs{world}" if world > 1 else "single",
                "l2": ("L2 flushed between timed steps" if cls.static_flush(world) else
                       "inputs larger than L2 (the slab's fields), steps timed back to back")}

    def config(self):
        return self.static_config(self.world)

class AffineLs:
    name = "affine_ls"
    dtype = "f64"
    scaling = "weak"
    flush_l2 = True

    def __init__(self, torch, rank, world, comm_factory):
        import numpy as np
        from stadeb200 import synth, kernels
        self.torch, self.np, self.kernels = torch, np, kernels
        c = synth.FULL["affine_ls"]
        self.n_s, self.n_o, self.n_i = c["n_s"], c["n_o"], c["n_i"]
        self.world = world
        d = synth.affine_ls_inputs(self.n_s, self.n_o, self.n_i)
        f64 = torch.float64
        self.pinned = {k: torch.from_numpy(v).pin_memory() for k, v in d.items()}
        t = {k: v.to("cuda") for k, v in self.pinned.items()}
        z = lambda m: torch.zeros(m, dtype=f64, device="cuda")
        S, O, I = self.n_s, self.n_o, self.n_i
        t.update(loss=z(1), wb=z(O * I), bb=z(O), xb=z(S * I), tb=z(S * O), y=z(S * O), yb=z(S * O))
        self.t = t
        self.ws = torch.empty(kernels.affine_ls_b_workspace(S, O, I), dtype=torch.uint8,
                              device="cuda")
        self.grad_host = {k: torch.empty(t[k].numel(), dtype=f64).pin_memory()
                          for k in ("wb", "bb", "loss")}
        self.graph = None

    def _eval(self):
        t = self.t
        for k in ("wb", "bb", "xb", "tb", "loss"):
            t[k].zero_()
        self.kernels.affine_ls_b_cuda(t["loss"], t["lossb"], t["w"], t["wb"], t["b"], t["bb"],
                                      t["x"], t["xb"], t["t"], t["tb"], t["y"], t["yb"],
                                      self.n_s, self.n_o, self.n_i, workspace=self.ws)

    def step(self):
        self._eval()

    def e2e_step(self):
        t, p = self.t, self.pinned
        for k in ("w", "b", "x", "t"):
            t[k].copy_(p[k], non_blocking=True)
        self._eval()
        for k, v in self.grad_host.items():
            v.copy_(t[k], non_blocking=True)

    def e2e_bytes(self):
        h2d = sum(self.pinned[k].numel() * 8 for k in ("w", "b", "x", "t"))
        return h2d, sum(v.numel() * 8 for v in self.grad_host.values())

    def phase_work(self):
        S, O, I = self.n_s, self.n_o, self.n_i
        byts = 8.0 * (S * I + S * O + O * I + O + O * I + O + S * I + S * O)
        return {"affine": ("hbm", byts, "read X, T, W, b; write Wb, bb, Xb, Tb (1,606,656 B); "
                                        "two launches, latency-bound")}

    @classmethod
    def static_config(cls, world):
        c = _synth_full()["affine_ls"]
        return {"workload": "C1 affine_ls_b: y = W x + b, 0.5 sum (y - t)^2 adjoint, W 64x32, "
                            "batch 1024, Float64", "n_s": c["n_s"], "n_o": c["n_o"],
                "n_i": c["n_i"], "parallelism": f"replicas{world}",
                "l2": "working set 1.6 MB fits in L2; L2 flushed between timed steps"}

    def config(self):
        return self.static_config(self.world)

class EmittedAffineLs(AffineLs):
    """C1 through the .cu emitter: the generated affine_ls_b text
    (julia/generated/affine_ls_b.jl) emitted, built for sm_100a and called
    through its C ABI in place of the hand-written sweep."""

    def __init__(self, torch, rank, world, comm_factory):
        super().__init__(torch, rank, world, comm_factory)
        from stadeb200 import emit
        self.sweep = emit.load(emit.generated_source("affine_ls_b"))

    def _eval(self):
        t = self.t
        for k in ("wb", "bb", "xb", "tb", "loss"):
            t[k].zero_()
        self.sweep(t["loss"], t["lossb"], t["w"], t["wb"], t["b"], t["bb"], t["x"], t["xb"],
                   t["t"], t["tb"], t["y"], t["yb"], self.n_s, self.n_o, self.n_i)

    def phase_work(self):
        kind, work, note = super().phase_work()["affine"]
        return {"emitted_sweep": (kind, work, "whole emitted call; " + note)}

    def config(self):
        c = super().config()
        c["workload"] += " (the .cu emitter's output for the generated sweep text)"
        return c


class EmittedHeat2d(Heat2d):
    """C3 through the .cu emitter's output for julia/generated/heat2d_b.jl
    (one GPU: the emitted sweep has no slab form)."""

    graphable = False   # returns alphab to the host: synchronises, cannot be captured

    def __init__(self, torch, rank, world, comm_factory):
        if world > 1:
            raise SystemExit("--impl emitted runs on one GPU")
        super().__init__(torch, rank, world, comm_factory)
        from stadeb200 import emit
        self.sweep = emit.load(emit.generated_source("heat2d_b"))
        self.stack = None
        self.stack = self.sweep.initstacks(self.n, self.n_step)[0]

    def step(self):
        t = self.t
        t["ub"].zero_()
        t["loss"].zero_()
        ab = self.sweep(t["loss"], t["lossb"], t["u"], t["ub"], t["un"], t["unb"], self.alpha,
                        0.0, self.n, self.n_step, self.stack)
        self.ab_host[0] = ab

    def e2e_step(self):
        self.t["u"].copy_(self.pinned["u"], non_blocking=True)
        self.step()
        self.out_host.copy_(self.t["ub"], non_blocking=True)

    def phase_work(self):
        N = float(self.rows) * self.n
        return {"emitted_sweep": ("hbm", 80.0 * 8.0 * N / 16 * self.n_step,
                                  "whole emitted call; algorithmic 80 N x 8 B per 16 steps")}

    def config(self):
        c = super().config()
        c["workload"] += " (the .cu emitter's output for the generated sweep text)"
        return c


class Conv1dReluMse:
    """C4. At N > 1 (a power of two) each rank takes a block of the 4,096
    samples; the loss is a mean, so the loss seed goes in scaled by 1/N and
    the summed loss comes out scaled by 1/N (ddp.mean_loss_factor), and the
    :accum wb and the loss are summed in one bucket."""
    name = "conv1d_relu_mse"
    dtype = "f32"
    flush_l2 = False  # x alone is 2.1 GB

    def __init__(self, torch, rank, world, comm_factory):
        import numpy as np
        from stadeb200 import synth, kernels, ddp
        self.torch, self.np, self.kernels, self.ddp = torch, np, kernels, ddp
        c = synth.FULL["conv1d_relu_mse"]
        self.G, self.C, self.L, self.O, self.K = c["n_b"], c["n_c"], c["n_l"], c["n_o"], c["n_k"]
        self.world = world
        self.factor = ddp.mean_loss_factor(self.G, world) if world > 1 else 1.0
        self.scaling = "strong"
        rng = ddp.shard(self.G, rank, world)
        self.B = len(rng)
        B, C, L, O, K = self.B, self.C, self.L, self.O, self.K
        lo_ = L - K + 1
        self.nt = B * O * lo_
        d = synth.conv1d_relu_mse_inputs(self.G, C, L, O, K)
        d["x"] = d["x"][rng.start * C * L:rng.stop * C * L]
        d["t"] = d["t"][rng.start * O * lo_:rng.stop * O * lo_]
        d["lossb"] = (d["lossb"] * np.float32(self.factor)).astype(np.float32)
        f32 = torch.float32
        self.pinned = {k: torch.from_numpy(np.ascontiguousarray(v)).pin_memory()
                       for k, v in d.items()}
        t = {k: v.to("cuda") for k, v in self.pinned.items()}
        z = lambda m: torch.zeros(m, dtype=f32, device="cuda")
        t.update(loss=z(1), xb=z(B * C * L), wb=z(O * C * K), tb=z(self.nt), z=z(self.nt),
                 zb=z(self.nt), r=z(self.nt), rb=z(self.nt))
        self.t = t
        self.ws = torch.empty(kernels.conv1d_relu_mse_b_workspace(B, C, L, O, K), dtype=torch.uint8,
                              device="cuda")
        self.grad_host = {k: torch.empty(t[k].numel(), dtype=f32).pin_memory()
                          for k in ("wb", "loss")}
        self.comm = comm_factory() if world > 1 else None

    def step(self):
        t = self.t
        for k in ("wb", "xb", "tb", "loss"):
            t[k].zero_()
        self.kernels.conv1d_relu_mse_b_cuda(t["loss"], t["lossb"], t["x"], t["xb"], t["w"], t["wb"],
                                            t["t"], t["tb"], t["z"], t["zb"], t["r"], t["rb"],
                                            self.B, self.C, self.L, self.O, self.K,
                                            workspace=self.ws)
        if self.comm is not None:
            self.ddp.allreduce_sum_(self.comm, t["wb"], t["loss"])
            t["loss"].mul_(self.factor)

    def e2e_step(self):
        t, p = self.t, self.pinned
        for k in ("x", "w", "t"):
            t[k].copy_(p[k], non_blocking=True)
        self.step()
        for k, v in self.grad_host.items():
            v.copy_(t[k], non_blocking=True)

    def e2e_bytes(self):
        h2d = sum(self.pinned[k].numel() * 4 for k in ("x", "w", "t"))
        return h2d, sum(v.numel() * 4 for v in self.grad_host.values())

    def phase_work(self):
        fl = 2.0 * self.B * self.O * (self.L - self.K + 1) * self.C * self.K
        nx = float(self.B) * self.C * self.L
        return {"conv_split": ("hbm", 12.0 * nx, "x read, x^T hi / lo planes written"),
                "conv_fwd": ("tensor", fl, "implicit GEMM 2 B O Lo C K flops + elementwise"),
                "conv_wgrad": ("tensor", fl, "weight gradient 2 B O Lo C K flops"),
                "conv_xgrad": ("tensor", fl, "input gradient 2 B O Lo C K flops")}

    @classmethod
    def static_config(cls, world):
        c = _synth_full()["conv1d_relu_mse"]
        return {"workload": "C4 conv1d_relu_mse_b: 1-D conv 128x64x9 + ReLU + MSE adjoint, batch "
                            "4096 x 64 x 2048, Float32", "global_batch": c["n_b"],
                "per_rank_batch": c["n_b"] // world, "n_c": c["n_c"], "n_l": c["n_l"],
                "n_o": c["n_o"], "n_k": c["n_k"], "parallelism": f"dp{world}",
                "l2": "inputs larger than L2"}

    def config(self):
        return self.static_config(self.world)

class _LocalZero:
    """The epilogue's zeroing at N = 1 (no communicator)."""

    def zero(self, bufs):
        from stadeb200 import ddp
        ddp.zero_(*bufs)


class Mlp2CeHv:
    """C5. At N > 1 each rank takes a block of the 16,384 samples and the hvp
    epilogue (ddp.Epilogue over NCCL) sums the 8 :accum shadows (b and bd of
    w1, b1, w2, b2) in one bucket and the :reduced loss / lossd."""
    name = "mlp2_ce_hv"
    dtype = "f64"
    scaling = "strong"

    def __init__(self, torch, rank, world, comm_factory):
        import numpy as np
        from stadeb200 import synth, kernels, ddp
        self.torch, self.np, self.kernels = torch, np, kernels
        c = synth.FULL["mlp2_ce_hv"]
        self.G, self.I, self.H, self.O = c["n_s"], c["n_i"], c["n_h"], c["n_o"]
        self.world = world
        rng = ddp.shard(self.G, rank, world)
        lo, hi = rng.start, rng.stop
        self.S = hi - lo
        d = synth.mlp2_ce_hv_inputs(self.G, self.I, self.H, self.O)
        for k, w in (("x", self.I), ("y", self.O), ("xd", self.I), ("yd", self.O)):
            d[k] = d[k][lo * w:hi * w].copy()
        self.pinned = {k: torch.from_numpy(v).pin_memory() for k, v in d.items()}
        t = {k: v.to("cuda") for k, v in self.pinned.items()}
        S, I, H, O = self.S, self.I, self.H, self.O
        from stadeb200 import ddp as _ddp
        roles = _ddp.derive_roles(_ddp.MLP2_CE, ["x", "y"], "hvp")
        summed = (_ddp.role_args(_ddp.MLP2_CE, roles, "hvp", "accum") +
                  _ddp.role_args(_ddp.MLP2_CE, roles, "hvp", "reduced"))
        # the eight :accum shadows and loss / lossd back to back: one NCCL
        # all-reduce in place per step
        lens = [kernels._mlp_len(nm, S, I, H, O) for nm in summed]
        self.bucket = torch.zeros(sum(lens), dtype=torch.float64, device="cuda")
        off = 0
        for nm, n in zip(summed, lens):
            t[nm] = self.bucket[off:off + n]
            off += n
        self.summed = summed
        for name in kernels.MLP_HV_ARGS + kernels.MLP_HV_TAN:
            if name not in t:
                t[name] = torch.zeros(kernels._mlp_len(name, S, I, H, O), dtype=torch.float64,
                                      device="cuda")
        self.t = t
        self.ws = torch.empty(kernels.mlp2_ce_hv_workspace(S, I, H, O), dtype=torch.uint8,
                              device="cuda")
        self.comm = comm_factory() if world > 1 else None
        backend = ddp.NcclBackend(self.comm) if self.comm is not None else _LocalZero()
        self.epi = ddp.Epilogue(ddp.MLP2_CE, ["x", "y"], "hvp", backend)
        self.flush_l2 = self.static_flush(world)
        self.out_names = ("w1bd", "b1bd", "w2bd", "b2bd", "lossd")
        self.grad_host = {k: torch.empty(t[k].numel(), dtype=torch.float64).pin_memory()
                          for k in self.out_names}

    def step(self):
        t, e = self.t, self.epi
        e.reset_accum(t)
        e.reset_reduced(t)
        e.reset_local(t)
        self.kernels.mlp2_ce_hv_cuda(*[t[a] for a in self.kernels.MLP_HV_ARGS], self.S, self.I,
                                     self.H, self.O, *[t[a] for a in self.kernels.MLP_HV_TAN],
                                     workspace=self.ws)
        if self.comm is not None:
            # :accum and :reduced summed every step: one collective over the bucket
            e.backend.allreduce_sum([t[b] for b in self.summed])

    def e2e_step(self):
        t, p = self.t, self.pinned
        for k in ("x", "y", "w1", "b1", "w2", "b2", "w1d", "b1d", "w2d", "b2d"):
            t[k].copy_(p[k], non_blocking=True)
        self.step()
        for k, v in self.grad_host.items():
            v.copy_(t[k], non_blocking=True)

    def e2e_bytes(self):
        h2d = sum(self.pinned[k].numel() * 8 for k in ("x", "y", "w1", "b1", "w2", "b2", "w1d",
                                                         "b1d", "w2d", "b2d"))
        return h2d, sum(v.numel() * 8 for v in self.grad_host.values())

    def phase_work(self):
        u = 2.0 * self.S * self.I * self.H
        return {"hv_fwd_gemms": ("fp64", 3 * u, "x W1, x W1d + xd W1 (3 units of 2 S I H flops)"),
                "hv_w1b_gemms": ("fp64", 3 * u, "x^T s1b, x^T s1bd + xd^T s1b (3 units)"),
                "hv_xb_gemms": ("fp64", 3 * u, "s1b W1^T, s1bd W1^T + s1b W1d^T (3 units)")}

    @staticmethod
    def static_flush(world):
        c = _synth_full()["mlp2_ce_hv"]
        S, I, H, O = c["n_s"] // world, c["n_i"], c["n_h"], c["n_o"]
        return 8 * (2 * S * (I + O) + 2 * (I * H + H + H * O + O) + 2) < L2_BYTES

    @classmethod
    def static_config(cls, world):
        c = _synth_full()["mlp2_ce_hv"]
        return {"workload": "C5 mlp2_ce_hv: HVP of the C2 loss, batch 16384, Float64, direction "
                            "over all 407,050 parameters", "global_batch": c["n_s"],
                "per_rank_batch": c["n_s"] // world, "n_i": c["n_i"], "n_h": c["n_h"],
                "n_o": c["n_o"], "parallelism": f"dp{world}",
                "l2": ("L2 flushed between timed steps" if cls.static_flush(world) else
                       "inputs (x, xd) larger than L2, steps timed back to back")}

    def config(self):
        return self.static_config(self.world)

WORKLOADS = {"mlp2_ce": Mlp2Ce, "heat2d": Heat2d, "affine_ls": AffineLs,
             "conv1d_relu_mse": Conv1dReluMse, "mlp2_ce_hv": Mlp2CeHv}
EMITTED = {"affine_ls": EmittedAffineLs, "heat2d": EmittedHeat2d}


# ---------------------------------------------------------------------------
REF_FULL_STEPS = ("mlp2_ce", "affine_ls", "mlp2_ce_hv")   # whole grad-evals per step


def run_reference(args):
    """The reference's CPU implementation of the path on the host cores: the
    oracle (the generated sweep restated in C++; the reference's Julia cannot
    run on these machines) with OpenMP over all host threads, on the oracle's
    own inputs, so no product library is loaded. Each step is one whole
    grad-eval of the configuration (C3 and C4, whose whole grad-eval takes
    minutes on the host, run a bounded sample per step, stated in the line).
    Under torchrun only rank 0 runs it."""
    world, rank, _ = dist_setup(args)
    if rank != 0:
        return
    config = args.config
    full, _ = FULL_UNITS[config]
    threads = 1 if config == "affine_ls" else cpu_threads()
    if config in REF_FULL_STEPS:
        units = full
    elif config == "heat2d":
        units = 2
    else:
        units = 4 * threads
    sw = CpuSweep(config, units, threads)
    for _ in range(args.warmup):
        sw.run()
    h0 = time.perf_counter()
    times = [sw.run() for _ in range(args.steps)]
    wall = time.perf_counter() - h0
    ms_per_step = 1e3 * sum(times) / args.steps
    value = (units / full) * 1e3 / ms_per_step
    cls = WORKLOADS[config]
    cpu = {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
           "sample": sw.describe()}
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": cls.scaling,
            "vs_baseline": None, "dtype": cls.dtype, "data": "synthetic (seeded, shapes and "
                                                            "distributions of the BASELINE config)",
            "config": cls.static_config(world),
            "cpu_baseline": cpu,
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "timing": "host wall clock around each step (perf_counter)",
            "timed_region_s": wall}
    print(json.dumps(line), flush=True)


EXTRA_CONFIGS = ("affine_ls", "heat2d", "conv1d_relu_mse", "mlp2_ce_hv")


def measure(W, args, torch, world, rank, dist, stream, flush, clocks, peaks, peak_src):
    """Times one workload: W warm-up steps, K timed steps of a replayed CUDA
    graph of one step (eager where capture is not possible), then the same
    steps eagerly with the phase profiler on (roofline, launch count), then
    the end-to-end steps from host buffers, then the CPU baseline (rank 0,
    N = 1). Returns the JSON-line fields of this workload."""
    from stadeb200 import _lib
    t_setup = time.time()
    for _ in range(args.warmup):
        W.step()
    torch.cuda.synchronize()
    step_fn, graph = W.step, None
    if not args.no_graph and getattr(W, "graphable", True):
        try:
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                W.step()                     # workspace / attributes settled outside capture
            torch.cuda.current_stream().wait_stream(side)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                W.step()
            torch.cuda.synchronize()
            step_fn = graph.replay
            for _ in range(2):
                step_fn()
            torch.cuda.synchronize()
        except Exception as e:  # fall back to eager launches, and say so
            graph = None
            step_fn = W.step
            print(f"# graph capture failed, timing eager launches: {e!r}", file=sys.stderr)
        if world > 1:
            # every rank replays its graph or none does (the steps hold collectives)
            ok = torch.tensor([1.0 if graph is not None else 0.0], device="cuda")
            dist.all_reduce(ok, op=dist.ReduceOp.MIN)
            if float(ok.item()) < 1.0:
                graph = None
                step_fn = W.step
    time.sleep(max(0.0, 1.5 - (time.time() - t_setup)))  # nvidia-smi is up and sampling
    # the warm-up steps again right before timing: the GPU idled during the
    # wait above and its clocks are back at speed only after some work
    clocks.mark_begin()
    total_ms, per = timed_loop(torch, step_fn, args.steps, args.warmup, world, dist,
                               flush if W.flush_l2 else None, stream)
    window = clocks.mark_end()
    host_ms = timed_loop.host_ms / args.steps
    ms_per_step = total_ms / args.steps
    value = 1000.0 / ms_per_step if W.scaling == "strong" else world * 1000.0 / ms_per_step

    # the same steps eagerly with the phase profiler on: per-phase device time
    # for the roofline, and the launch count (a replayed graph holds the same
    # kernels)
    _lib.profile_read()
    _lib.profile_enable(True)
    launches0 = _lib.lib().stade_kernel_launches()
    e0 = W.sweep.launches() if args.impl == "emitted" else 0
    p_ms, _ = timed_loop(torch, W.step, args.steps, 0, world, dist,
                         flush if W.flush_l2 else None, stream)
    launches = _lib.lib().stade_kernel_launches() - launches0
    _lib.profile_enable(False)
    phases = _lib.profile_read()
    if args.impl == "emitted":
        # the emitted sweep's own launch counter, and the whole call as its phase
        launches = W.sweep.launches() - e0
        phases = {"emitted_sweep": (p_ms, args.steps)}

    # end to end through the public entry points with host buffers
    e2e = None
    if not args.no_e2e:
        e_ms, _ = timed_loop(torch, W.e2e_step, args.steps, args.warmup, world, dist, None, stream)
        h2d, d2h = W.e2e_bytes()
        ev = 1000.0 / (e_ms / args.steps)
        if W.scaling != "strong":
            ev *= world
        e2e = {"value": ev, "unit": UNIT,
               "h2d_bytes_per_step": h2d * (world if W.scaling == "strong" else 1),
               "d2h_bytes_per_step": d2h * (world if W.scaling == "strong" else 1),
               "ms_per_step": e_ms / args.steps}
        note = getattr(W, "e2e_note", None)
        if note:
            e2e["note"] = note
    torch.cuda.synchronize()
    timing = "CUDA graph of one step, replayed" if graph is not None else "eager launches"
    graph_note = ("the step's NCCL calls are captured in the graph"
                  if graph is not None and world > 1 else None)
    # a graph that holds NCCL calls goes before the communicators
    step_fn = graph = None
    torch.cuda.synchronize()
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(W.name, args.cpu_seconds)
    return {"value": value, "ms_per_step": ms_per_step, "scaling": W.scaling, "dtype": W.dtype,
            "config": W.config(),
            "roofline": roofline(phases, W.phase_work(), args.steps, peaks, peak_src,
                                 load_traffic(W.name) if world == 1 else None),
            "cpu_baseline": cpu, "e2e": e2e, "clocks_window": window,
            "gpu_launches": launches,
            "timing": timing, "graph_note": graph_note,
            "eager_profiled_ms_per_step": p_ms / args.steps,
            "host_enqueue_ms_per_step": host_ms,
            "phases_ms_per_step": {k: v[0] / args.steps for k, v in phases.items()},
            "step_ms_min_max": [min(per), max(per)]}


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    import torch
    world, rank, local = dist_setup(args)
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    from stadeb200 import ddp

    def comm_factory():
        return ddp.NcclComm(rank, world)

    def make(name):
        if args.impl == "emitted":
            if name not in EMITTED:
                raise SystemExit(f"--impl emitted: one of {sorted(EMITTED)}")
            return EMITTED[name](torch, rank, world, comm_factory)
        return WORKLOADS[name](torch, rank, world, comm_factory)

    stream = torch.cuda.current_stream()
    flush = torch.zeros(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")
    peaks, peak_src = load_peaks()
    if args.config == "mlp2_ce_hv" or (world == 1 and args.config == "mlp2_ce" and not args.no_extra):
        peaks["fp64_tflops"] = fp64_peak(torch)
        peaks["fp64_source"] = "measured (cuBLAS DGEMM 8192^3 in this run, best of 5)"
    clocks = ClockSampler(local)
    clocks.start()

    W = make(args.config)
    head = measure(W, args, torch, world, rank, dist, stream, flush, clocks, peaks, peak_src)
    comm = getattr(W, "comm", None)
    del W
    # the other configurations at N = 1 (the default run), each measured the
    # same way, reported in "configs"
    extras = {}
    if (world == 1 and args.impl == "ours" and args.config == "mlp2_ce" and not args.no_extra):
        for name in EXTRA_CONFIGS:
            gc.collect()
            torch.cuda.empty_cache()
            Wx = make(name)
            extras[name] = measure(Wx, args, torch, world, rank, dist, stream, flush, clocks,
                                   peaks, peak_src)
            del Wx
    clocks.stop()

    if rank == 0:
        def finish(m):
            m["clocks"] = clocks.summary(m.pop("clocks_window"))
            return m
        head = finish(head)
        line = {"metric": METRIC, "value": head.pop("value"), "unit": UNIT, "n_gpus": world,
                **({"impl": "emitted"} if args.impl == "emitted" else {}),
                "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": head.pop("ms_per_step"), "higher_is_better": True,
                "scaling": head.pop("scaling"), "vs_baseline": None, "dtype": head.pop("dtype"),
                "data": "synthetic (seeded, shapes and distributions of the BASELINE config)",
                **head}
        if "fp64_tflops" in peaks:
            line["fp64_peak"] = {"tflops": peaks["fp64_tflops"], "source": peaks["fp64_source"]}
        if extras:
            line["configs"] = {k: finish(v) for k, v in extras.items()}
            line["gpu_launches_all_configs"] = line["gpu_launches"] + sum(
                v["gpu_launches"] for v in extras.values())
        print(json.dumps(line), flush=True)
    torch.cuda.synchronize()
    if world > 1:
        if comm is not None:
            comm.close()
        dist.barrier()
        dist.destroy_process_group()

if __name__ == "__main__":
    main()
