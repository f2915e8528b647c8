"""ctypes binding of libstade_b200.so (the C ABI in include/stade_b200.h).

The library is built in-tree (stade.jl_b200/libstade_b200.so). Loading it
fails loudly when it is missing: there is no fallback implementation.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "libstade_b200.so")

STADE_OK = 0
STADE_EINVAL = 1
STADE_ECUDA = 2
STADE_ENCCL = 3
STADE_ETIMEDOUT = 4
STADE_ENOTSUP = 5
STADE_EREPLICA = 6
STADE_HOST_SCALARS = 0x1
STADE_F32 = 0
STADE_F64 = 1

_STATUS_NAMES = {
    0: "STADE_OK", 1: "STADE_EINVAL", 2: "STADE_ECUDA", 3: "STADE_ENCCL",
    4: "STADE_ETIMEDOUT", 5: "STADE_ENOTSUP", 6: "STADE_EREPLICA",
}


class StadeError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{_STATUS_NAMES.get(code, code)}: {msg}")
        self.code = code


class stade_opts(C.Structure):
    _fields_ = [("stream", C.c_void_p), ("workspace", C.c_void_p),
                ("workspace_bytes", C.c_size_t), ("flags", C.c_uint32)]


P = C.c_void_p          # device array
I64 = C.c_int64
D = C.c_double
OPTS = C.POINTER(stade_opts)
ST = C.c_int


# name -> (restype, argtypes)
SIGNATURES = {
    "stade_last_error": (C.c_char_p, []),
    "stade_version": (C.c_char_p, []),
    "stade_kernel_launches": (C.c_int, []),
    "stade_reset_kernel_launches": (None, []),
    "stade_workspace_cached_bytes": (C.c_size_t, []),
    "stade_device_error": (C.c_int, []),
    "stade_check_bounded_wait": (ST, [I64, OPTS]),
    "stade_profile_enable": (None, [C.c_int]),
    "stade_profile_read": (C.c_int, [C.c_char_p, C.c_int, C.POINTER(D), C.POINTER(C.c_int),
                                     C.c_int]),
    "stade_affine_ls_b_f64_workspace": (C.c_size_t, [I64, I64, I64]),
    "stade_affine_ls_b_f64": (ST, [P] * 12 + [I64] * 3 + [OPTS]),
    "stade_affine_ls_b_f64_noalloc_max_scratch": (C.c_size_t, []),
    "stade_affine_ls_b_f64_noalloc": (ST, [P] * 12 + [I64] * 3 + [OPTS]),
    "stade_mlp2_ce_b_f32_workspace": (C.c_size_t, [I64] * 4),
    "stade_mlp2_ce_b_f32": (ST, [P] * 20 + [I64] * 4 + [OPTS]),
    "stade_initstacks_heat2d_b": (I64, [I64, I64]),
    "stade_heat2d_b_f64_workspace": (C.c_size_t, [I64, I64]),
    "stade_heat2d_b_f64": (ST, [P] * 6 + [D, P, I64, I64, P, OPTS]),
    "stade_affine_ls_d_f64_workspace": (C.c_size_t, [I64] * 3),
    "stade_affine_ls_d_f64": (ST, [P] * 12 + [I64] * 3 + [OPTS]),
    "stade_mlp2_ce_d_f32_workspace": (C.c_size_t, [I64] * 4),
    "stade_mlp2_ce_d_f64_workspace": (C.c_size_t, [I64] * 4),
    "stade_mlp2_ce_d_f32": (ST, [P] * 20 + [I64] * 4 + [OPTS]),
    "stade_mlp2_ce_d_f64": (ST, [P] * 20 + [I64] * 4 + [OPTS]),
    "stade_heat2d_d_f64_workspace": (C.c_size_t, [I64] * 2),
    "stade_heat2d_d_f64": (ST, [P] * 6 + [D, D, I64, I64, OPTS]),
    "stade_conv1d_relu_mse_d_f32_workspace": (C.c_size_t, [I64] * 5),
    "stade_conv1d_relu_mse_d_f32": (ST, [P] * 12 + [I64] * 5 + [OPTS]),
    "stade_initstacks_heat2d_b_slab": (I64, [I64, I64, I64]),
    "stade_heat2d_b_f64_slab_workspace": (C.c_size_t, [I64, I64, I64]),
    "stade_heat2d_b_f64_slab": (ST, [P] * 6 + [D, P, I64, I64, P, I64, P, OPTS]),
    "stade_conv1d_relu_mse_b_f32_workspace": (C.c_size_t, [I64] * 5),
    "stade_conv1d_relu_mse_b_f32": (ST, [P] * 12 + [I64] * 5 + [OPTS]),
    "stade_mlp2_ce_hv_f64_workspace": (C.c_size_t, [I64] * 4),
    "stade_mlp2_ce_hv_f64": (ST, [P] * 20 + [I64] * 4 + [P] * 20 + [OPTS]),
    "stade_comm_unique_id": (ST, [C.c_char_p]),
    "stade_comm_init": (ST, [C.c_char_p, C.c_int, C.c_int, C.c_int, C.POINTER(C.c_void_p)]),
    "stade_comm_destroy": (ST, [C.c_void_p]),
    "stade_comm_rank": (C.c_int, [C.c_void_p]),
    "stade_comm_size": (C.c_int, [C.c_void_p]),
    "stade_ddp_zero": (ST, [C.POINTER(C.c_void_p), C.POINTER(I64), C.c_int, C.c_int, OPTS]),
    "stade_ddp_allreduce_sum": (ST, [C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(I64), C.c_int,
                                     C.c_int, I64, C.POINTER(I64), OPTS]),
    "stade_ddp_check_replicas": (ST, [C.c_void_p, C.POINTER(C.c_void_p), C.POINTER(I64), C.c_int,
                                      C.c_int, C.POINTER(C.c_uint64), OPTS]),
    "stade_mlp2_ce_b_reset_accum_f32": (ST, [P] * 4 + [I64] * 3 + [OPTS]),
    "stade_mlp2_ce_b_reset_reduced_f32": (ST, [P, OPTS]),
    "stade_mlp2_ce_b_reset_local_f32": (ST, [P] * 5 + [I64] * 4 + [OPTS]),
    "stade_mlp2_ce_b_allreduce_accum_f32": (ST, [P] * 4 + [I64] * 4 + [C.c_void_p,
                                                                      C.POINTER(I64), OPTS]),
    "stade_mlp2_ce_b_allreduce_reduced_f32": (ST, [P, C.c_void_p, OPTS]),
    "stade_mlp2_ce_b_check_replicas_f32": (ST, [P] * 5 + [I64] * 3 + [C.c_void_p,
                                                                      C.POINTER(C.c_uint64), OPTS]),
    "stade_conv1d_relu_mse_b_reset_accum_f32": (ST, [P] + [I64] * 3 + [OPTS]),
    "stade_conv1d_relu_mse_b_reset_reduced_f32": (ST, [P, OPTS]),
    "stade_conv1d_relu_mse_b_reset_local_f32": (ST, [P] * 4 + [I64] * 5 + [OPTS]),
    "stade_conv1d_relu_mse_b_allreduce_accum_f32": (ST, [P] + [I64] * 4 + [C.c_void_p,
                                                                         C.POINTER(I64), OPTS]),
    "stade_conv1d_relu_mse_b_allreduce_reduced_f32": (ST, [P, C.c_void_p, OPTS]),
    "stade_conv1d_relu_mse_b_check_replicas_f32": (ST, [P] * 2 + [I64] * 3 + [
        C.c_void_p, C.POINTER(C.c_uint64), OPTS]),
    "stade_mlp2_ce_hv_reset_accum_f64": (ST, [P] * 8 + [I64] * 3 + [OPTS]),
    "stade_mlp2_ce_hv_reset_reduced_f64": (ST, [P, P, OPTS]),
    "stade_mlp2_ce_hv_reset_local_f64": (ST, [P] * 10 + [I64] * 4 + [OPTS]),
    "stade_mlp2_ce_hv_allreduce_accum_f64": (ST, [P] * 8 + [I64] * 4 + [C.c_void_p,
                                                                        C.POINTER(I64), OPTS]),
    "stade_mlp2_ce_hv_allreduce_reduced_f64": (ST, [P, P, C.c_void_p, OPTS]),
    "stade_mlp2_ce_hv_check_replicas_f64": (ST, [P] * 10 + [I64] * 3 + [
        C.c_void_p, C.POINTER(C.c_uint64), OPTS]),
    "stade_fnv1a64": (C.c_uint64, [C.c_char_p]),
    "stade_fill_normal_f64": (None, [P, I64, C.c_uint64, D, D]),
    "stade_fill_normal_f32": (None, [P, I64, C.c_uint64, D, D]),
    "stade_fill_uniform_f64": (None, [P, I64, C.c_uint64, D, D]),
    "stade_fill_uniform_f32": (None, [P, I64, C.c_uint64, D, D]),
    "stade_fill_onehot_f32": (None, [P, I64, I64, C.c_uint64]),
    "stade_fill_onehot_f64": (None, [P, I64, I64, C.c_uint64]),
}

_lib = None


def lib() -> C.CDLL:
    """The loaded library; raises if it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `make -C stade.jl_b200` "
                              "(or __graft_entry__.build()); there is no CPU fallback")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def profile_enable(on: bool) -> None:
    lib().stade_profile_enable(1 if on else 0)


def profile_read(max_phases: int = 64) -> dict:
    """{phase: (total device ms, launches)} since the last read; waits for
    the recorded events."""
    name_len = 64
    names = C.create_string_buffer(name_len * max_phases)
    ms = (D * max_phases)()
    cnt = (C.c_int * max_phases)()
    n = lib().stade_profile_read(names, name_len, ms, cnt, max_phases)
    out = {}
    for i in range(min(n, max_phases)):
        nm = names.raw[i * name_len:(i + 1) * name_len].split(b"\0", 1)[0].decode()
        out[nm] = (ms[i], cnt[i])
    return out


def check(code: int) -> None:
    if code != STADE_OK:
        raise StadeError(code, lib().stade_last_error().decode(errors="replace"))


def make_opts(stream=None, workspace=None, workspace_bytes=0, flags=0) -> stade_opts:
    o = stade_opts()
    o.stream = stream
    o.workspace = workspace
    o.workspace_bytes = workspace_bytes
    o.flags = flags
    return o
