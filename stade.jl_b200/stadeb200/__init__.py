"""stadeb200: Python host side of libstade_b200, a B200 (sm_100a) backend for
the adjoint / HVP sweeps and the data-parallel epilogue that STADE.jl
generates. The functions carry the generated names (`<k>_b_cuda`,
`<k>_hv_cuda`, `initstacks_<k>_b_cuda`, `<k>_b_reset_accum_` ...)."""
from ._lib import StadeError, lib, LIB_PATH  # noqa: F401
from .kernels import (  # noqa: F401
    affine_ls_b_cuda, mlp2_ce_b_cuda, heat2d_b_cuda, heat2d_b_cuda_device,
    initstacks_heat2d_b_cuda, conv1d_relu_mse_b_cuda, mlp2_ce_hv_cuda,
    heat2d_b_slab_cuda, initstacks_heat2d_b_slab_cuda,
    affine_ls_d_cuda, mlp2_ce_d_cuda, heat2d_d_cuda, conv1d_relu_mse_d_cuda,
    kernel_launches, reset_kernel_launches,
)
