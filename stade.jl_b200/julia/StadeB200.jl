# StadeB200.jl -- Julia binding of libstade_b200 (the C ABI in include/stade_b200.h).
#
# Defines the functions STADE.jl's CUDA port generates, by their generated
# names and argument order (`<k>_b_cuda`, `initstacks_<k>_b_cuda`, the ddpgen_
# epilogue), so a caller that `include`s the generated file can use these
# instead. Arrays are CuArrays (device pointers); integers Int64; a scalar
# float argument's adjoint is passed in and returned by value, as the generated
# code returns it. Every call runs on the task-local CUDA.jl stream.
#
# Not exercised in this repository (no Julia toolchain on the build machines);
# the Python host mirror (stadeb200/kernels.py) binds the same symbols and is
# what the tests run.
module StadeB200

using CUDA

const libstade = joinpath(@__DIR__, "..", "libstade_b200.so")

struct StadeOpts
    stream::Ptr{Cvoid}
    workspace::Ptr{Cvoid}
    workspace_bytes::Csize_t
    flags::UInt32
end

const STADE_HOST_SCALARS = UInt32(1)

opts(; flags = UInt32(0)) = Ref(StadeOpts(CUDA.stream().handle, C_NULL, 0, flags))

function check(code::Cint)
    code == 0 && return nothing
    msg = unsafe_string(ccall((:stade_last_error, libstade), Cstring, ()))
    error("libstade_b200: status $code: $msg")
end

# C1 -- replaces affine_ls_b_cuda
function affine_ls_b_cuda(loss, lossb, w, wb, b, bb, x, xb, t, tb, y, yb, n_s, n_o, n_i)
    check(ccall((:stade_affine_ls_b_f64, libstade), Cint,
        (CuPtr{Float64}, CuPtr{Float64}, CuPtr{Float64}, CuPtr{Float64}, CuPtr{Float64},
         CuPtr{Float64}, CuPtr{Float64}, CuPtr{Float64}, CuPtr{Float64}, CuPtr{Float64},
         CuPtr{Float64}, CuPtr{Float64}, Int64, Int64, Int64, Ref{StadeOpts}),
        loss, lossb, w, wb, b, bb, x, xb, t, tb, y, yb, n_s, n_o, n_i, opts()))
    return nothing
end

# C2 -- replaces mlp2_ce_b_cuda (Float32 after precision conversion)
function mlp2_ce_b_cuda(loss, lossb, x, xb, y, yb, w1, w1b, b1, b1b, w2, w2b, b2, b2b,
                        h, hb, z, zb, p, pb, n_s, n_i, n_h, n_o)
    check(ccall((:stade_mlp2_ce_b_f32, libstade), Cint,
        (ntuple(_ -> CuPtr{Float32}, 20)..., Int64, Int64, Int64, Int64, Ref{StadeOpts}),
        loss, lossb, x, xb, y, yb, w1, w1b, b1, b1b, w2, w2b, b2, b2b, h, hb, z, zb, p, pb,
        n_s, n_i, n_h, n_o, opts()))
    return nothing
end

# C3 -- replaces initstacks_heat2d_b and heat2d_b_cuda; returns alphab
function initstacks_heat2d_b_cuda(n, n_step)
    m = ccall((:stade_initstacks_heat2d_b, libstade), Int64, (Int64, Int64), n, n_step)
    return CuArray{Float64}(undef, max(m, 1))
end

function heat2d_b_cuda(loss, lossb, u, ub, un, unb, alpha, alphab, n, n_step, u_stack)
    box = Ref{Float64}(alphab)
    check(ccall((:stade_heat2d_b_f64, libstade), Cint,
        (CuPtr{Float64}, CuPtr{Float64}, CuPtr{Float64}, CuPtr{Float64}, CuPtr{Float64},
         CuPtr{Float64}, Float64, Ptr{Float64}, Int64, Int64, CuPtr{Float64}, Ref{StadeOpts}),
        loss, lossb, u, ub, un, unb, alpha, box, n, n_step, u_stack,
        opts(flags = STADE_HOST_SCALARS)))
    return box[]
end

# C4 -- replaces conv1d_relu_mse_b_cuda
function conv1d_relu_mse_b_cuda(loss, lossb, x, xb, w, wb, t, tb, z, zb, r, rb,
                                n_b, n_c, n_l, n_o, n_k)
    check(ccall((:stade_conv1d_relu_mse_b_f32, libstade), Cint,
        (ntuple(_ -> CuPtr{Float32}, 12)..., Int64, Int64, Int64, Int64, Int64, Ref{StadeOpts}),
        loss, lossb, x, xb, w, wb, t, tb, z, zb, r, rb, n_b, n_c, n_l, n_o, n_k, opts()))
    return nothing
end

# Tangent sweeps -- replace the `<k>_d` functions stade_tangent_file writes
# (tgen_signature_args: each float argument followed by its `d` shadow)
function affine_ls_d_cuda(loss, lossd, w, wd, b, bd, x, xd, t, td, y, yd, n_s, n_o, n_i)
    check(ccall((:stade_affine_ls_d_f64, libstade), Cint,
        (ntuple(_ -> CuPtr{Float64}, 12)..., Int64, Int64, Int64, Ref{StadeOpts}),
        loss, lossd, w, wd, b, bd, x, xd, t, td, y, yd, n_s, n_o, n_i, opts()))
    return nothing
end

function mlp2_ce_d_cuda(loss, lossd, x, xd, y, yd, w1, w1d, b1, b1d, w2, w2d, b2, b2d,
                        h, hd, z, zd, p, pd, n_s, n_i, n_h, n_o)
    T = eltype(loss)
    sym = T == Float32 ? :stade_mlp2_ce_d_f32 : :stade_mlp2_ce_d_f64
    check(ccall((sym, libstade), Cint,
        (ntuple(_ -> CuPtr{T}, 20)..., Int64, Int64, Int64, Int64, Ref{StadeOpts}),
        loss, lossd, x, xd, y, yd, w1, w1d, b1, b1d, w2, w2d, b2, b2d, h, hd, z, zd, p, pd,
        n_s, n_i, n_h, n_o, opts()))
    return nothing
end

function heat2d_d_cuda(loss, lossd, u, ud, un, und, alpha, alphad, n, n_step)
    check(ccall((:stade_heat2d_d_f64, libstade), Cint,
        (ntuple(_ -> CuPtr{Float64}, 6)..., Float64, Float64, Int64, Int64, Ref{StadeOpts}),
        loss, lossd, u, ud, un, und, alpha, alphad, n, n_step, opts()))
    return nothing
end

function conv1d_relu_mse_d_cuda(loss, lossd, x, xd, w, wd, t, td, z, zd, r, rd,
                                n_b, n_c, n_l, n_o, n_k)
    check(ccall((:stade_conv1d_relu_mse_d_f32, libstade), Cint,
        (ntuple(_ -> CuPtr{Float32}, 12)..., Int64, Int64, Int64, Int64, Int64, Ref{StadeOpts}),
        loss, lossd, x, xd, w, wd, t, td, z, zd, r, rd, n_b, n_c, n_l, n_o, n_k, opts()))
    return nothing
end

# C5 -- replaces mlp2_ce_hv_cuda (hvp_emit layout: adjoint args, then pairs)
function mlp2_ce_hv_cuda(loss, lossb, x, xb, y, yb, w1, w1b, b1, b1b, w2, w2b, b2, b2b,
                         h, hb, z, zb, p, pb, n_s, n_i, n_h, n_o,
                         lossd, lossbd, xd, xbd, yd, ybd, w1d, w1bd, b1d, b1bd, w2d, w2bd,
                         b2d, b2bd, hd, hbd, zd, zbd, pd, pbd)
    check(ccall((:stade_mlp2_ce_hv_f64, libstade), Cint,
        (ntuple(_ -> CuPtr{Float64}, 20)..., Int64, Int64, Int64, Int64,
         ntuple(_ -> CuPtr{Float64}, 20)..., Ref{StadeOpts}),
        loss, lossb, x, xb, y, yb, w1, w1b, b1, b1b, w2, w2b, b2, b2b, h, hb, z, zb, p, pb,
        n_s, n_i, n_h, n_o, lossd, lossbd, xd, xbd, yd, ybd, w1d, w1bd, b1d, b1bd, w2d, w2bd,
        b2d, b2bd, hd, hbd, zd, zbd, pd, pbd, opts()))
    return nothing
end

# ---- data-parallel epilogue (ddpgen_ names; NCCL instead of MPI) ----------------
mutable struct Comm
    handle::Ptr{Cvoid}
end

"""Create the communicator: `id` (128 bytes) from `unique_id()` on rank 0,
broadcast by the caller (e.g. MPI.Bcast!)."""
function unique_id()
    id = Vector{UInt8}(undef, 128)
    check(ccall((:stade_comm_unique_id, libstade), Cint, (Ptr{UInt8},), id))
    return id
end

function Comm(id::Vector{UInt8}, nranks::Integer, rank::Integer; timeout_ms::Integer = 60000)
    h = Ref{Ptr{Cvoid}}(C_NULL)
    check(ccall((:stade_comm_init, libstade), Cint,
        (Ptr{UInt8}, Cint, Cint, Cint, Ptr{Ptr{Cvoid}}), id, nranks, rank, timeout_ms, h))
    return Comm(h[])
end

"""Sum the buffers (all Float32 or all Float64) across ranks in one
collective; with `n_local` given, also the sample counts, returning the
global count (the generic form of `<k>_b_allreduce_accum!`)."""
function ddp_allreduce_sum!(comm::Comm, bufs::CuArray{T}...; n_local = nothing) where {T}
    dt = T === Float32 ? Cint(0) : T === Float64 ? Cint(1) : error("Float32 or Float64 buffers")
    ptrs = [Ptr{Cvoid}(UInt(pointer(b))) for b in bufs]   # device addresses
    counts = Int64[length(b) for b in bufs]
    ng = Ref{Int64}(0)
    check(ccall((:stade_ddp_allreduce_sum, libstade), Cint,
        (Ptr{Cvoid}, Ptr{Ptr{Cvoid}}, Ptr{Int64}, Cint, Cint, Int64, Ptr{Int64}, Ref{StadeOpts}),
        comm.handle, ptrs, counts, length(bufs), dt, n_local === nothing ? 0 : n_local,
        n_local === nothing ? C_NULL : ng, opts()))
    return n_local === nothing ? nothing : ng[]
end

mlp2_ce_b_reset_accum!(w1b, b1b, w2b, b2b) =(foreach(b -> fill!(b, 0f0), (w1b, b1b, w2b, b2b)); nothing)
mlp2_ce_b_reset_reduced!(loss) = (fill!(loss, 0f0); nothing)
mlp2_ce_b_reset_local!(xb, yb, hb, zb, pb) = (foreach(b -> fill!(b, 0f0), (xb, yb, hb, zb, pb)); nothing)

function mlp2_ce_b_allreduce_accum!(w1b, b1b, w2b, b2b, n_local, comm::Comm)
    ng = Ref{Int64}(0)
    check(ccall((:stade_mlp2_ce_b_allreduce_accum_f32, libstade), Cint,
        (CuPtr{Float32}, CuPtr{Float32}, CuPtr{Float32}, CuPtr{Float32}, Int64, Int64, Int64,
         Int64, Ptr{Cvoid}, Ptr{Int64}, Ref{StadeOpts}),
        w1b, b1b, w2b, b2b, div(length(w1b), length(b1b)), length(b1b), length(b2b),
        n_local, comm.handle, ng, opts()))
    return ng[]
end

function mlp2_ce_b_allreduce_reduced!(loss, comm::Comm)
    check(ccall((:stade_mlp2_ce_b_allreduce_reduced_f32, libstade), Cint,
        (CuPtr{Float32}, Ptr{Cvoid}, Ref{StadeOpts}), loss, comm.handle, opts()))
    return nothing
end

function mlp2_ce_b_check_replicas(w1, b1, w2, b2, lossb, comm::Comm)
    mask = Ref{UInt64}(0)
    code = ccall((:stade_mlp2_ce_b_check_replicas_f32, libstade), Cint,
        (CuPtr{Float32}, CuPtr{Float32}, CuPtr{Float32}, CuPtr{Float32}, CuPtr{Float32},
         Int64, Int64, Int64, Ptr{Cvoid}, Ptr{UInt64}, Ref{StadeOpts}),
        w1, b1, w2, b2, lossb, div(length(w1), length(b1)), length(b1), length(b2),
        comm.handle, mask, opts())
    if code == 6
        names = ["w1", "b1", "w2", "b2", "lossb"]
        bad = [names[i + 1] for i in 0:4 if (mask[] >> i) & 1 == 1]
        error("mlp2_ce_b_check_replicas: `" * join(bad, "`, `") * "` differ across ranks. " *
              "A :shared or :seed buffer must hold identical values on every rank.")
    end
    check(code)
    return nothing
end

# conv1d_relu_mse, adjoint mode, per_sample = [:x, :t] (:accum wb, :reduced loss,
# :local xb tb zb rb, :shared w, :seed lossb). Sizes from the arrays: w is
# n_o x n_c x n_k, x is n_b x n_c x n_l.
conv1d_relu_mse_b_reset_accum!(wb) = (fill!(wb, 0f0); nothing)
conv1d_relu_mse_b_reset_reduced!(loss) = (fill!(loss, 0f0); nothing)
conv1d_relu_mse_b_reset_local!(xb, tb, zb, rb) = (foreach(b -> fill!(b, 0f0), (xb, tb, zb, rb)); nothing)

function conv1d_relu_mse_b_allreduce_accum!(wb, n_local, comm::Comm)
    ng = Ref{Int64}(0)
    check(ccall((:stade_conv1d_relu_mse_b_allreduce_accum_f32, libstade), Cint,
        (CuPtr{Float32}, Int64, Int64, Int64, Int64, Ptr{Cvoid}, Ptr{Int64}, Ref{StadeOpts}),
        wb, length(wb), 1, 1, n_local, comm.handle, ng, opts()))
    return ng[]
end

function conv1d_relu_mse_b_allreduce_reduced!(loss, comm::Comm)
    check(ccall((:stade_conv1d_relu_mse_b_allreduce_reduced_f32, libstade), Cint,
        (CuPtr{Float32}, Ptr{Cvoid}, Ref{StadeOpts}), loss, comm.handle, opts()))
    return nothing
end

function conv1d_relu_mse_b_check_replicas(w, lossb, comm::Comm)
    mask = Ref{UInt64}(0)
    code = ccall((:stade_conv1d_relu_mse_b_check_replicas_f32, libstade), Cint,
        (CuPtr{Float32}, CuPtr{Float32}, Int64, Int64, Int64, Ptr{Cvoid}, Ptr{UInt64},
         Ref{StadeOpts}), w, lossb, length(w), 1, 1, comm.handle, mask, opts())
    if code == 6
        bad = [n for (i, n) in enumerate(["w", "lossb"]) if (mask[] >> (i - 1)) & 1 == 1]
        error("conv1d_relu_mse_b_check_replicas: `" * join(bad, "`, `") *
              "` differ across ranks. A :shared or :seed buffer must hold identical values " *
              "on every rank.")
    end
    check(code)
    return nothing
end

# mlp2_ce, hvp mode: the `_hv` names (ddpgen_mode_suffix), per_sample = [:x, :y].
mlp2_ce_hv_reset_accum!(w1b, b1b, w2b, b2b, w1bd, b1bd, w2bd, b2bd) =
    (foreach(b -> fill!(b, 0.0), (w1b, b1b, w2b, b2b, w1bd, b1bd, w2bd, b2bd)); nothing)
mlp2_ce_hv_reset_reduced!(loss, lossd) = (fill!(loss, 0.0); fill!(lossd, 0.0); nothing)
mlp2_ce_hv_reset_local!(xb, yb, hb, zb, pb, xbd, ybd, hbd, zbd, pbd) =
    (foreach(b -> fill!(b, 0.0), (xb, yb, hb, zb, pb, xbd, ybd, hbd, zbd, pbd)); nothing)

function mlp2_ce_hv_allreduce_accum!(w1b, b1b, w2b, b2b, w1bd, b1bd, w2bd, b2bd, n_local,
                                     comm::Comm)
    ng = Ref{Int64}(0)
    check(ccall((:stade_mlp2_ce_hv_allreduce_accum_f64, libstade), Cint,
        (ntuple(_ -> CuPtr{Float64}, 8)..., Int64, Int64, Int64, Int64, Ptr{Cvoid}, Ptr{Int64},
         Ref{StadeOpts}),
        w1b, b1b, w2b, b2b, w1bd, b1bd, w2bd, b2bd, div(length(w1b), length(b1b)),
        length(b1b), length(b2b), n_local, comm.handle, ng, opts()))
    return ng[]
end

function mlp2_ce_hv_allreduce_reduced!(loss, lossd, comm::Comm)
    check(ccall((:stade_mlp2_ce_hv_allreduce_reduced_f64, libstade), Cint,
        (CuPtr{Float64}, CuPtr{Float64}, Ptr{Cvoid}, Ref{StadeOpts}), loss, lossd, comm.handle,
        opts()))
    return nothing
end

function mlp2_ce_hv_check_replicas(w1, b1, w2, b2, w1d, b1d, w2d, b2d, lossb, lossbd, comm::Comm)
    mask = Ref{UInt64}(0)
    code = ccall((:stade_mlp2_ce_hv_check_replicas_f64, libstade), Cint,
        (ntuple(_ -> CuPtr{Float64}, 10)..., Int64, Int64, Int64, Ptr{Cvoid}, Ptr{UInt64},
         Ref{StadeOpts}),
        w1, b1, w2, b2, w1d, b1d, w2d, b2d, lossb, lossbd, div(length(w1), length(b1)),
        length(b1), length(b2), comm.handle, mask, opts())
    if code == 6
        names = ["w1", "b1", "w2", "b2", "w1d", "b1d", "w2d", "b2d", "lossb", "lossbd"]
        bad = [names[i + 1] for i in 0:9 if (mask[] >> i) & 1 == 1]
        error("mlp2_ce_hv_check_replicas: `" * join(bad, "`, `") * "` differ across ranks. " *
              "A :shared or :seed buffer must hold identical values on every rank.")
    end
    check(code)
    return nothing
end

end # module
