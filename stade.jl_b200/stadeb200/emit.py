"""The .cu emitter (include/stade_emit.h) from Python: STADE-generated Julia
sweep text in, a CUDA source, a built library and a callable out.

    cu, manifest = emit(open("foo_b.jl").read())            # C++ emitter, via ctypes
    so = build(cu)                                          # nvcc, sm_100a
    sweep = Sweep(so, manifest)
    stacks = sweep.initstacks(n, n_step)                   # the tape, on the device
    ret = sweep(*args, *stacks)                             # the generated call

`cuda_file(in_path, out_path)` is the file-to-file form of STADE.jl's
stade_cuda_file (src/STADE.jl:12062-12111): it writes the .cu and, beside it,
the manifest (.json) with the loop decisions. `build(..., host=True)` compiles
the same source for the CPU (kernels as loops over their threads), which the
tests use to check the translation without a GPU.
"""
from __future__ import annotations

import ctypes as C
import hashlib
import json
import os
import subprocess

_HERE = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(_HERE)
EMIT_LIB = os.path.join(PKG, "libstade_emit.so")
GEN_DIR = os.path.join(PKG, "_gen")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

GENERATED = os.path.join(PKG, "julia", "generated")

_lib = None


def generated_source(name: str) -> str:
    """The text of a generated sweep shipped with the package
    (julia/generated/<name>.jl: the C1 and C3 adjoints in STADE's output
    style)."""
    with open(os.path.join(GENERATED, name + ".jl")) as f:
        return f.read()


class EmitError(RuntimeError):
    pass


# The generated sweeps shipped in julia/generated/ and the precisions the
# package builds them in (the bench's emitted arm and its Julia binding load
# these).
SHIPPED = {"affine_ls_b": (64, 32), "heat2d_b": (64,)}


def build_shipped() -> list:
    """Emits and builds every shipped generated sweep for sm_100a (cached by
    content under _gen/); returns the library paths."""
    return [build(emit(generated_source(name), precision=prec)[0])
            for name, precs in SHIPPED.items() for prec in precs]


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(EMIT_LIB):
            raise EmitError(f"{EMIT_LIB} is missing: run `make -C {PKG}`")
        L = C.CDLL(EMIT_LIB)
        L.stade_emit_cuda.restype = C.c_int
        L.stade_emit_cuda.argtypes = [C.c_char_p, C.c_char_p, C.c_int, C.c_char_p, C.c_char_p,
                                      C.c_size_t, C.POINTER(C.c_size_t), C.c_char_p, C.c_size_t,
                                      C.POINTER(C.c_size_t)]
        L.stade_emit_last_error.restype = C.c_char_p
        _lib = L
    return _lib


def _dims_spec(dims) -> str:
    if not dims:
        return ""
    if isinstance(dims, str):
        return dims
    return ";".join(f"{k}=" + ",".join(str(x) for x in v) for k, v in dims.items())


def emit(source: str, function: str | None = None, precision: int = 64, dims=None):
    """(CUDA source, manifest dict). dims: {"a": ["i_m"]} or "a=i_m"."""
    L = lib()
    src = source.encode()
    fn = function.encode() if function else None
    ds = _dims_spec(dims).encode()
    n_cu, n_m = C.c_size_t(0), C.c_size_t(0)
    if L.stade_emit_cuda(src, fn, precision, ds, None, 0, C.byref(n_cu), None, 0, C.byref(n_m)):
        raise EmitError(L.stade_emit_last_error().decode())
    cu = C.create_string_buffer(n_cu.value + 1)
    man = C.create_string_buffer(n_m.value + 1)
    if L.stade_emit_cuda(src, fn, precision, ds, cu, n_cu.value + 1, C.byref(n_cu), man,
                         n_m.value + 1, C.byref(n_m)):
        raise EmitError(L.stade_emit_last_error().decode())
    return cu.value.decode(), json.loads(man.value.decode())


def cuda_file(in_path: str, out_path: str, function: str | None = None, precision: int = 64,
              dims=None) -> dict:
    """stade_cuda_file: reads a generated .jl, writes the .cu and its manifest
    (out_path with .json). Returns the manifest."""
    with open(in_path) as f:
        cu, man = emit(f.read(), function, precision, dims)
    with open(out_path, "w") as f:
        f.write(cu)
    with open(os.path.splitext(out_path)[0] + ".json", "w") as f:
        json.dump(man, f, indent=1)
    return man


def build(cu: str, out_dir: str | None = None, host: bool = False) -> str:
    """Compiles the source into a shared library (cached by content) and
    returns its path. GPU: nvcc for sm_100a with -fmad=false (each a * b + c
    rounded twice, as the generated Julia evaluates it). host: g++ with the
    same rounding."""
    out_dir = out_dir or GEN_DIR
    os.makedirs(out_dir, exist_ok=True)
    h = hashlib.sha256((cu + ("host" if host else "sm_100a")).encode()).hexdigest()[:16]
    so = os.path.join(out_dir, f"gen_{h}{'_host' if host else ''}.so")
    if os.path.exists(so):
        return so
    src = os.path.join(out_dir, f"gen_{h}.cu")
    with open(src, "w") as f:
        f.write(cu)
    tmp = so + f".{os.getpid()}.tmp"
    if host:
        cmd = ["/usr/bin/g++", "-std=c++17", "-O2", "-ffp-contract=off", "-fPIC", "-shared",
               "-DSTADE_EMIT_HOST", "-x", "c++", src, "-o", tmp]
    else:
        cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-fmad=false", "-std=c++17", "-shared",
               "-Xcompiler", "-fPIC", "-diag-suppress", "177", src, "-o", tmp]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise EmitError(f"compiling {src} failed:\n{r.stderr[-4000:]}")
    os.replace(tmp, so)
    return so


_DT = {"f64": ("float64", C.c_double), "f32": ("float32", C.c_float)}


class Sweep:
    """A built sweep. Call it with the generated positional arguments: device
    arrays (torch CUDA tensors; numpy arrays for a host build), Python ints
    and floats. Returns what the generated Julia returns: None, the one
    returned scalar, or the tuple of them."""

    def __init__(self, so_path: str, manifest: dict, host: bool = False):
        self.m = manifest
        self.host = host
        self.lib = C.CDLL(so_path)
        self.fdt, self.cf = _DT[manifest["precision"]]
        args = []
        for a in manifest["args"]:
            k = a["kind"]
            if k in ("array_float", "array_int"):
                args.append(C.c_void_p)
            elif k == "scalar_int":
                args.append(C.c_int64)
            elif k == "scalar_float":
                args.append(self.cf)
            else:
                args.append(C.POINTER(self.cf))
        self.fn = getattr(self.lib, manifest["symbol"])
        self.fn.restype = C.c_int
        self.fn.argtypes = args + [C.c_void_p]
        ini = manifest["initstacks"]
        self.init = None
        if ini["symbol"]:
            self.init = getattr(self.lib, ini["symbol"])
            self.init.restype = C.c_int64
            self.init.argtypes = [C.c_int64] * len(ini["args"]) + [
                C.POINTER(C.c_int64), C.POINTER(C.c_int), C.POINTER(C.c_void_p)]

    def launches(self) -> int:
        """Kernels this library has launched so far (all calls)."""
        f = getattr(self.lib, self.m["symbol"] + "_launches")
        f.restype = C.c_int64
        return int(f())

    def _init_args(self, args):
        """initstacks' integer arguments; one it reads through `length(a)`
        may be given as the array (or as its length)."""
        import numpy as np
        ini = self.m["initstacks"]
        lens = set(ini.get("length_args", []))
        vals = []
        for name, a in zip(ini["args"], args):
            if name in lens and not isinstance(a, int) and hasattr(a, "__len__"):
                a = a.numel() if hasattr(a, "numel") else int(np.asarray(a).size)
            vals.append(int(a))
        return vals

    def stack_sizes(self, *args):
        """(size, kind) per item initstacks_<k> returns: kind "float64",
        "float32" or "int64" for a stack the caller zero-fills, "int" for a
        returned integer (size = its value), "int64_table" / "float_table"
        for a table initstacks fills."""
        ini = self.m["initstacks"]
        if not self.init:
            return []
        n = len(ini["stacks"])
        sizes = (C.c_int64 * max(n, 1))()
        dts = (C.c_int * max(n, 1))()
        got = self.init(*self._init_args(args), sizes, dts, None)
        if got < 0:
            raise EmitError(f"{ini['symbol']}: a table write fell outside its table")
        kinds = ("float64", "float32", "int64", "int", "int64_table", "float_table")
        return [(int(sizes[i]), kinds[dts[i]]) for i in range(got)]

    def initstacks(self, *args, device="cuda"):
        """What initstacks_<k> returns: its stacks zero-filled, its tables
        with the contents it computes, its integers as ints."""
        import numpy as np
        items = self.stack_sizes(*args)
        host = []
        fill = (C.c_void_p * max(len(items), 1))()
        for i, (n, kind) in enumerate(items):
            if kind == "int":
                host.append(n)
                continue
            dt = {"int64_table": "int64", "float_table": self.fdt}.get(kind, kind)
            on_host = self.host or kind.endswith("_table")
            a = np.zeros(max(n, 0) if on_host else 0, dt)
            if kind.endswith("_table") and n > 0:
                fill[i] = a.ctypes.data
            host.append(a)
        if any(k.endswith("_table") for _, k in items):
            if self.init(*self._init_args(args), None, None, fill) < 0:
                raise EmitError(f"{self.m['initstacks']['symbol']}: a table write fell outside its table")
        if self.host:
            return tuple(host)
        import torch
        out = []
        for h, (n, kind) in zip(host, items):   # stacks straight on the device, tables copied up
            if isinstance(h, int):
                out.append(h)
            elif kind.endswith("_table"):
                out.append(torch.from_numpy(h).to(device))
            else:
                out.append(torch.zeros(max(n, 0), dtype=getattr(torch, kind), device=device))
        return tuple(out)

    def _ptr(self, a, spec):
        want = "int64" if spec["kind"] == "array_int" else self.fdt
        if self.host:
            import numpy as np
            if not isinstance(a, np.ndarray) or a.dtype != np.dtype(want) or not a.flags.c_contiguous:
                raise TypeError(f"{spec['name']}: expected a contiguous numpy {want} array")
            return a.ctypes.data
        import torch
        if not (isinstance(a, torch.Tensor) and a.is_cuda and a.is_contiguous()
                and str(a.dtype) == f"torch.{want}"):
            raise TypeError(f"{spec['name']}: expected a contiguous CUDA {want} tensor")
        return a.data_ptr()

    def local_arrays(self, *args, device="cuda"):
        """The arrays the sweep allocates for itself in Julia (hoisted to
        trailing arguments), zero-filled, sized by stade_<k>_locals from the
        sweep's other arguments (everything but these locals, in order)."""
        loc = self.m.get("locals")
        if not loc:
            return ()
        import numpy as np
        by_name = dict(zip([a["name"] for a in self.m["args"]], args))
        f = getattr(self.lib, loc["symbol"])
        f.restype = C.c_int64
        vals = [int(by_name[n]) for n in loc["args"]]
        for n in loc["length_args"]:
            a = by_name[n]
            vals.append(a.numel() if hasattr(a, "numel") else int(np.asarray(a).size))
        n = len(loc["arrays"])
        sizes = (C.c_int64 * n)()
        dts = (C.c_int * n)()
        f.argtypes = [C.c_int64] * len(vals) + [C.POINTER(C.c_int64), C.POINTER(C.c_int)]
        f(*vals, sizes, dts)
        kinds = ("float64", "float32", "int64")
        if self.host:
            return tuple(np.zeros(sizes[i], kinds[dts[i]]) for i in range(n))
        import torch
        return tuple(torch.zeros(sizes[i], dtype=getattr(torch, kinds[dts[i]]), device=device)
                     for i in range(n))

    def __call__(self, *args, stream=None):
        specs = self.m["args"]
        n_local = sum(1 for a in specs if a.get("local"))
        if n_local and len(args) == len(specs) - n_local:
            args = tuple(args) + self.local_arrays(*args)
        if len(args) != len(specs):
            raise TypeError(f"{self.m['function']} takes {len(specs)} arguments, got {len(args)}")
        cargs, boxes = [], {}
        for a, s in zip(args, specs):
            k = s["kind"]
            if k in ("array_float", "array_int"):
                cargs.append(self._ptr(a, s))
            elif k == "scalar_int":
                cargs.append(int(a))
            elif k == "scalar_float":
                cargs.append(float(a))
            else:
                b = self.cf(float(a))
                boxes[s["name"]] = b
                cargs.append(C.pointer(b))
        if stream is None and not self.host:
            import torch
            stream = torch.cuda.current_stream().cuda_stream
        rc = self.fn(*cargs, stream or None)
        if rc != 0:
            raise EmitError(f"{self.m['symbol']} returned {rc}")
        ret = [boxes[r].value for r in self.m["returns"]]
        if not ret:
            return None
        return ret[0] if len(ret) == 1 else tuple(ret)


def load(source: str, function: str | None = None, precision: int = 64, dims=None,
         host: bool = False) -> Sweep:
    """emit + build + Sweep in one call."""
    cu, man = emit(source, function, precision, dims)
    return Sweep(build(cu, host=host), man, host=host)
