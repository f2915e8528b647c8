"""Data-parallel epilogue: role table, sample sharding and the generated
epilogue functions, over NCCL through libstade_b200.

Restates `ddpgen_roles` (src/STADE.jl:17404-17440): every float argument gets
a class from two facts the caller states (`per_sample`, `reduced`) and two the
kernel shows (which arrays it writes, which outputs are reductions), and
every buffer of the generated layout gets a role:

    class         input buffer     adjoint-valued buffer
    :shared       :shared          :accum
    :reduced      :reduced         :seed
    :per_sample   :per_sample      :local
    :scratch      :scratch         :local

(a scalar float argument's adjoint is :returned). The epilogue zeroes :accum
and :reduced once per step, :local before each sample, sums :accum (with the
sample count) and :reduced across ranks, and checks :shared / :seed for
agreement (src/STADE.jl:17595-17696). Here the sums are one NCCL collective
per call over one bucket instead of one MPI.Allreduce! per buffer.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch

from ._lib import STADE_F32, STADE_F64, check, lib, make_opts


@dataclass(frozen=True)
class KernelSig:
    """What ddpgen_ reads from a parsed primal: argument order, kinds
    (:array_float, :scalar_float, :array_int, :scalar_int), the arrays the body
    writes, and the outputs every write of which adds to the array itself."""
    name: str
    args: tuple
    kinds: dict
    written: frozenset
    reduced_outputs: frozenset
    # arrays whose writes all add the array to itself at an index that varies
    # with an enclosing loop: a per-sample result or a cross-sample sum, which
    # the caller must resolve (ddpgen_reduced_outputs, src/STADE.jl:17282)
    ambiguous: frozenset = frozenset()


def adjoint_layout(sig: KernelSig) -> list:
    """agen_signature_args (src/STADE.jl:3455-3465): each float argument
    followed by its adjoint."""
    out = []
    for a in sig.args:
        out.append(a)
        if sig.kinds[a] in ("array_float", "scalar_float"):
            out.append(a + "b")
    return out


def hvp_layout(sig: KernelSig) -> list:
    """ddpgen_hvp_signature_args (src/STADE.jl:17475-17484): the adjoint
    layout, then (tangent, adjoint-of-tangent) per float argument."""
    out = adjoint_layout(sig)
    for a in sig.args:
        if sig.kinds[a] in ("array_float", "scalar_float"):
            out += [a + "d", a + "bd"]
    return out


def check_declaration(sig: KernelSig, per_sample, reduced=()) -> None:
    """The refusals of ddpgen_check_declaration (src/STADE.jl:17218-17270):
    names that are not float array arguments, duplicates, an array in both
    lists, a per_sample array the kernel overwrites, a `reduced` array whose
    role is already derived, and an ambiguous array left unresolved. Raises
    ValueError with the reference's wording."""
    per_sample, reduced = list(per_sample), list(reduced)
    for kw, names in (("per_sample", per_sample), ("reduced", reduced)):
        not_args = [p for p in names if p not in sig.args]
        if not_args:
            verb = "is" if len(not_args) == 1 else "are"
            raise ValueError(f"{kw} names `{'`, `'.join(not_args)}`, which {verb} not an "
                             f"argument of {sig.name}")
        not_fa = [p for p in names if sig.kinds[p] != "array_float"]
        if not_fa:
            raise ValueError(f"{kw} names `{'`, `'.join(not_fa)}`, which is not a float array "
                             "argument")
        dups = sorted({p for p in names if names.count(p) > 1})
        if dups:
            raise ValueError(f"{kw} names `{'`, `'.join(dups)}` more than once")
    both = [p for p in per_sample if p in reduced]
    if both:
        raise ValueError(f"`{'`, `'.join(both)}` appears in per_sample and in reduced. An array "
                         "is one or the other")
    bad_ps = [p for p in per_sample if p in sig.written and p not in sig.ambiguous]
    if bad_ps:
        raise ValueError(f"per_sample names `{'`, `'.join(bad_ps)}`, which the kernel writes by "
                         "plain overwrite. That array already takes a derived role, so naming it "
                         "here would give it two")
    bad_rd = [p for p in reduced if p not in sig.ambiguous]
    if bad_rd:
        raise ValueError(f"reduced names `{'`, `'.join(bad_rd)}`, whose role is already derived. "
                         "`reduced` resolves an array whose writes are all additive at an index "
                         "that varies with an enclosing loop, and no other")
    unresolved = [a for a in sorted(sig.ambiguous) if a not in per_sample and a not in reduced]
    if unresolved:
        raise ValueError(f"`{'`, `'.join(unresolved)}` takes only additive writes at an index "
                         "that varies with an enclosing loop. Two readings fit that shape and the "
                         "kernel does not say which. Name it in `per_sample` if it holds one "
                         "sample's own result, which needs no communication. Name it in `reduced` "
                         "if it accumulates across samples, which is summed across ranks")


def derive_roles(sig: KernelSig, per_sample, mode: str, reduced=()) -> dict:
    """Role of every buffer of the mode's layout (ddpgen_roles)."""
    if mode not in ("tangent", "adjoint", "hvp"):
        raise ValueError(f"mode must be tangent, adjoint or hvp, got {mode}")
    per_sample, reduced = list(per_sample), list(reduced)
    check_declaration(sig, per_sample, reduced)
    all_reduced = set(sig.reduced_outputs) | set(reduced)
    roles = {}
    for a in sig.args:
        kind = sig.kinds[a]
        if kind not in ("array_float", "scalar_float"):
            continue
        readonly = kind == "array_float" and a not in sig.written
        if a in per_sample and a not in sig.written:
            cls = "per_sample"
        elif a in per_sample:
            cls = "scratch"
        elif a in all_reduced:
            cls = "reduced"
        elif readonly:
            cls = "shared"
        else:
            cls = "scratch"
        out_role = ("returned" if kind == "scalar_float" else
                    "accum" if cls == "shared" else "seed" if cls == "reduced" else "local")
        roles[a] = cls
        if mode in ("tangent", "hvp"):
            roles[a + "d"] = cls
        if mode in ("adjoint", "hvp"):
            roles[a + "b"] = out_role
        if mode == "hvp":
            roles[a + "bd"] = out_role
    return roles


def role_args(sig: KernelSig, roles: dict, mode: str, want: str) -> list:
    """Buffers with one role, in layout order, arrays only (ddpgen_role_args)."""
    layout = adjoint_layout(sig) if mode == "adjoint" else hvp_layout(sig)
    scalars = set()
    for a in sig.args:
        if sig.kinds[a] == "scalar_float":
            scalars |= {a, a + "b", a + "d", a + "bd"}
    return [b for b in layout if roles.get(b) == want and b not in scalars]


# The primal mlp2_ce (oracle/primals.jl): h, z, p and loss are written; every
# write of loss adds to loss itself.
MLP2_CE = KernelSig(
    name="mlp2_ce",
    args=("loss", "x", "y", "w1", "b1", "w2", "b2", "h", "z", "p", "n_s", "n_i", "n_h", "n_o"),
    kinds={**{a: "array_float" for a in ("loss", "x", "y", "w1", "b1", "w2", "b2", "h", "z", "p")},
           **{a: "scalar_int" for a in ("n_s", "n_i", "n_h", "n_o")}},
    written=frozenset({"h", "z", "p", "loss"}),
    reduced_outputs=frozenset({"loss"}),
)


# The primal affine_ls (oracle/primals.jl): y is overwritten, every write of
# loss adds to loss itself.
AFFINE_LS = KernelSig(
    name="affine_ls",
    args=("loss", "w", "b", "x", "t", "y", "n_s", "n_o", "n_i"),
    kinds={**{a: "array_float" for a in ("loss", "w", "b", "x", "t", "y")},
           **{a: "scalar_int" for a in ("n_s", "n_o", "n_i")}},
    written=frozenset({"y", "loss"}),
    reduced_outputs=frozenset({"loss"}),
)


# The primal conv1d_relu_mse (oracle/primals.jl): z, r are overwritten, every
# write of loss adds to loss itself; its loss is a mean over all outputs
# (inv_n = 1 / (n_b n_o n_lo) inside the sweep).
CONV1D_RELU_MSE = KernelSig(
    name="conv1d_relu_mse",
    args=("loss", "x", "w", "t", "z", "r", "n_b", "n_c", "n_l", "n_o", "n_k"),
    kinds={**{a: "array_float" for a in ("loss", "x", "w", "t", "z", "r")},
           **{a: "scalar_int" for a in ("n_b", "n_c", "n_l", "n_o", "n_k")}},
    written=frozenset({"z", "r", "loss"}),
    reduced_outputs=frozenset({"loss"}),
)


def mean_loss_factor(n_samples: int, nranks: int) -> float:
    """For a primal whose loss is a mean over its samples (C4's inv_n), a
    rank of a sample-sharded run computes inv_n over its own block, nranks
    times the whole batch's. Multiplying the loss seed by the returned factor
    before the sweep and the summed :reduced loss by it after the sum makes
    the sharded run the whole-batch function. The factor is 1 / nranks and is
    required to be a power of two with equal blocks: then every product that
    carries it is exact, the per-sample adjoints equal the whole-batch ones
    bit for bit, and the :accum sums differ only in summation order."""
    if nranks < 1 or nranks & (nranks - 1) or n_samples % nranks:
        raise ValueError(f"a mean loss shards exactly over a power-of-two rank count that "
                         f"divides the samples; got {n_samples} samples on {nranks} ranks")
    return 1.0 / nranks


def shard(n_samples: int, rank: int, nranks: int, mode: str = "block") -> range | list:
    """Samples of one rank. "mod": sample s (1-based) on rank mod(s - 1, P),
    as test/validate_ddp.jl:52-53; "block": contiguous blocks, which keeps
    each rank's batch one strided array (the layout a batch-loop kernel
    takes)."""
    if mode == "mod":
        return list(range(rank, n_samples, nranks))
    lo = n_samples * rank // nranks
    hi = n_samples * (rank + 1) // nranks
    return range(lo, hi)


# ---------------------------------------------------------------------------
class NcclComm:
    """One NCCL communicator per process / GPU (stade_comm_init). The 128-byte
    id is made on rank 0 and broadcast with whatever the caller has: here a
    torch.distributed group (any backend), as a Julia caller would use MPI."""

    def __init__(self, rank: int, nranks: int, group=None, timeout_ms: int = 60000,
                 unique_id: bytes | None = None):
        if unique_id is None:
            import torch.distributed as dist
            buf = [None]
            if rank == 0:
                raw = C.create_string_buffer(128)
                check(lib().stade_comm_unique_id(raw))
                buf[0] = bytes(raw.raw)
            dist.broadcast_object_list(buf, src=0, group=group)
            unique_id = buf[0]
        self.rank, self.size = rank, nranks
        handle = C.c_void_p()
        check(lib().stade_comm_init(unique_id, nranks, rank, timeout_ms, C.byref(handle)))
        self.handle = handle

    def close(self) -> None:
        if self.handle:
            lib().stade_comm_destroy(self.handle)
            self.handle = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _dtype_code(ts) -> int:
    dt = ts[0].dtype
    if any(t.dtype != dt for t in ts):
        raise TypeError("all buffers of one epilogue call must share a dtype")
    if dt == torch.float32:
        return STADE_F32
    if dt == torch.float64:
        return STADE_F64
    raise TypeError(f"unsupported dtype {dt}")


def _bufs(ts):
    for t in ts:
        if not (t.is_cuda and t.is_contiguous()):
            raise ValueError("epilogue buffers must be contiguous CUDA tensors")
    n = len(ts)
    ptrs = (C.c_void_p * n)(*[t.data_ptr() for t in ts])
    counts = (C.c_int64 * n)(*[t.numel() for t in ts])
    return ptrs, counts, n


def _opts(stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return make_opts(s.cuda_stream)


def zero_(*bufs, stream=None) -> None:
    """fill!(b, 0.0) for each buffer (ddpgen_fill_fn)."""
    if not bufs:
        return
    ptrs, counts, n = _bufs(bufs)
    o = _opts(stream)
    check(lib().stade_ddp_zero(ptrs, counts, n, _dtype_code(bufs), C.byref(o)))


def allreduce_sum_(comm: NcclComm, *bufs, n_local=None, stream=None):
    """Sums the buffers across ranks in one collective. With n_local given,
    also sums the sample counts and returns the global count (the value
    allreduce_accum! returns; reading it waits for the stream). With
    n_local=None nothing is counted and the call stays asynchronous."""
    if not bufs:
        return n_local
    ptrs, counts, n = _bufs(bufs)
    o = _opts(stream)
    ng = C.c_int64(0)
    check(lib().stade_ddp_allreduce_sum(comm.handle, ptrs, counts, n, _dtype_code(bufs),
                                        0 if n_local is None else int(n_local),
                                        None if n_local is None else C.byref(ng), C.byref(o)))
    return None if n_local is None else ng.value


def check_replicas(comm: NcclComm, *bufs, names=None, stream=None) -> None:
    """Raises when a :shared / :seed buffer differs across ranks."""
    if not bufs:
        return
    ptrs, counts, n = _bufs(bufs)
    o = _opts(stream)
    mask = C.c_uint64(0)
    code = lib().stade_ddp_check_replicas(comm.handle, ptrs, counts, n, _dtype_code(bufs),
                                          C.byref(mask), C.byref(o))
    if code != 0 and mask.value:
        names = names or [f"buffer {i}" for i in range(n)]
        bad = [names[i] for i in range(n) if mask.value >> i & 1]
        raise RuntimeError(f"`{'`, `'.join(bad)}` differ across ranks. A :shared or :seed buffer "
                           "must hold identical values on every rank. The usual cause is a "
                           "per-sample array left out of per_sample")
    check(code)


class NcclBackend:
    """Epilogue operations on CUDA tensors through libstade_b200 (one bucketed
    NCCL collective per call)."""

    def __init__(self, comm: NcclComm, stream=None):
        self.comm, self.stream = comm, stream

    def zero(self, bufs):
        zero_(*bufs, stream=self.stream)

    def allreduce_sum(self, bufs, n_local=None):
        return allreduce_sum_(self.comm, *bufs, n_local=n_local, stream=self.stream)

    def check(self, bufs, names):
        check_replicas(self.comm, *bufs, names=names, stream=self.stream)


class Epilogue:
    """The five functions the reference's `stade_ddp_file` writes for one
    kernel and mode (ddpgen_emit, src/STADE.jl:17578-17696), driven by the
    role table: reset_accum / reset_reduced / reset_local zero the :accum,
    :reduced and :local buffers, allreduce_accum sums :accum across ranks with
    the sample count and returns the global count, allreduce_reduced sums
    :reduced, check_replicas checks :shared and :seed buffers for agreement.
    `bank` maps buffer names to the caller's arrays; the backend does the
    work (NcclBackend on CUDA tensors)."""

    def __init__(self, sig: KernelSig, per_sample, mode: str, backend, reduced=()):
        if mode not in ("adjoint", "hvp"):
            raise ValueError("an epilogue exists for the adjoint and hvp modes")
        self.sig, self.mode, self.backend = sig, mode, backend
        self.roles = derive_roles(sig, per_sample, mode, reduced)
        r = lambda want: role_args(sig, self.roles, mode, want)
        self.accum, self.reduced, self.local = r("accum"), r("reduced"), r("local")
        self.checked = r("shared") + r("seed")
        self.returned = [b for b, v in self.roles.items() if v == "returned"]

    def reset_accum(self, bank):
        self.backend.zero([bank[b] for b in self.accum])

    def reset_reduced(self, bank):
        self.backend.zero([bank[b] for b in self.reduced])

    def reset_local(self, bank):
        self.backend.zero([bank[b] for b in self.local])

    def allreduce_accum(self, bank, n_local: int) -> int:
        return self.backend.allreduce_sum([bank[b] for b in self.accum], n_local=n_local)

    def allreduce_reduced(self, bank):
        self.backend.allreduce_sum([bank[b] for b in self.reduced])

    def check_replicas(self, bank):
        self.backend.check([bank[b] for b in self.checked], self.checked)


# ---- generated names of the mlp2_ce epilogue (adjoint mode) ------------------
_ROLES_B = derive_roles(MLP2_CE, ["x", "y"], "adjoint")


def mlp2_ce_b_reset_accum_(w1b, b1b, w2b, b2b, stream=None):
    zero_(w1b, b1b, w2b, b2b, stream=stream)


def mlp2_ce_b_reset_reduced_(loss, stream=None):
    zero_(loss, stream=stream)


def mlp2_ce_b_reset_local_(xb, yb, hb, zb, pb, stream=None):
    zero_(xb, yb, hb, zb, pb, stream=stream)


def mlp2_ce_b_allreduce_accum_(w1b, b1b, w2b, b2b, n_local, comm, stream=None) -> int:
    return allreduce_sum_(comm, w1b, b1b, w2b, b2b, n_local=n_local, stream=stream)


def mlp2_ce_b_allreduce_reduced_(loss, comm, stream=None) -> None:
    allreduce_sum_(comm, loss, stream=stream)


def mlp2_ce_b_check_replicas(w1, b1, w2, b2, lossb, comm, stream=None) -> None:
    check_replicas(comm, w1, b1, w2, b2, lossb, names=["w1", "b1", "w2", "b2", "lossb"],
                   stream=stream)


# ---- generated names of the mlp2_ce epilogue (hvp mode) ----------------------
def mlp2_ce_hv_reset_accum_(w1b, b1b, w2b, b2b, w1bd, b1bd, w2bd, b2bd, stream=None):
    zero_(w1b, b1b, w2b, b2b, w1bd, b1bd, w2bd, b2bd, stream=stream)


def mlp2_ce_hv_reset_reduced_(loss, lossd, stream=None):
    zero_(loss, lossd, stream=stream)


def mlp2_ce_hv_reset_local_(xb, yb, hb, zb, pb, xbd, ybd, hbd, zbd, pbd, stream=None):
    zero_(xb, yb, hb, zb, pb, xbd, ybd, hbd, zbd, pbd, stream=stream)


def mlp2_ce_hv_allreduce_accum_(w1b, b1b, w2b, b2b, w1bd, b1bd, w2bd, b2bd, n_local, comm,
                                stream=None) -> int:
    return allreduce_sum_(comm, w1b, b1b, w2b, b2b, w1bd, b1bd, w2bd, b2bd, n_local=n_local,
                          stream=stream)


def mlp2_ce_hv_allreduce_reduced_(loss, lossd, comm, stream=None) -> None:
    allreduce_sum_(comm, loss, lossd, stream=stream)
