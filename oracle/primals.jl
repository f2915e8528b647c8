# Primal kernels of the five benchmark configurations, written in STADE's
# input style (claude/skill-stade.md rules 1-14: flattened independent nests
# with div/mod-recovered indices, no allocation, length-1 arrays for scalar
# outputs, every float argument positional). STADE.jl differentiates these;
# oracle.cc restates, loop for loop, the adjoint / HVP sweeps it generates for
# them with indexed tapes and STADE's default loop handling (keep_push_pop =
# false, fuse_ii_loops = false: every backward loop runs reversed,
# src/STADE.jl:6553-6557), and libstade_b200 runs the same sweeps on the GPU.
#
# This file is a specification for readers and for a Julia caller that wants to
# regenerate the adjoints with STADE; nothing in this repository executes it.

# affine_ls(loss, w, b, x, t, y, n_s, n_o, n_i)
#
# Batched affine map and least-squares loss (configuration C1).
# loss: length-1 output, accumulated in place
# w: weights n_o x n_i, row-major ((i_o - 1) * n_i + i_k)
# b: bias, length n_o
# x: inputs n_s x n_i, row-major
# t: targets n_s x n_o, row-major
# y: predictions n_s x n_o, scratch, overwritten
function affine_ls(loss, w, b, x, t, y, n_s, n_o, n_i)
    # every (sample, output) pair is independent: one flattened loop
    for idx = 1:n_s * n_o
        i_s = div(idx - 1, n_o) + 1
        i_o = mod(idx - 1, n_o) + 1
        s = b[i_o]
        # the dot product over inputs is a genuine accumulation
        for i_k = 1:n_i
            s = s + w[(i_o - 1) * n_i + i_k] * x[(i_s - 1) * n_i + i_k]
        end
        y[idx] = s
    end
    for idx2 = 1:n_s * n_o
        loss[1] = loss[1] + 0.5 * (y[idx2] - t[idx2]) ^ 2
    end
    return nothing
end

# mlp2_ce(loss, x, y, w1, b1, w2, b2, h, z, p, n_s, n_i, n_h, n_o)
#
# Two-layer tanh MLP with a softmax cross-entropy loss, a batch loop in the
# kernel (configurations C2 in Float32 and C5 as its HVP in Float64).
# loss: length-1 output, accumulated in place
# x: inputs n_s x n_i; y: one-hot targets n_s x n_o
# w1: n_i x n_h ((i_k - 1) * n_h + i_j); b1: n_h
# w2: n_h x n_o ((i_k - 1) * n_o + i_c); b2: n_o
# h: hidden activations n_s x n_h, scratch
# z: logits n_s x n_o, scratch; p: shifted exponentials n_s x n_o, scratch
function mlp2_ce(loss, x, y, w1, b1, w2, b2, h, z, p, n_s, n_i, n_h, n_o)
    # hidden layer: every (sample, unit) is independent
    for idx = 1:n_s * n_h
        i_s = div(idx - 1, n_h) + 1
        i_j = mod(idx - 1, n_h) + 1
        s1 = b1[i_j]
        for i_k = 1:n_i
            s1 = s1 + x[(i_s - 1) * n_i + i_k] * w1[(i_k - 1) * n_h + i_j]
        end
        h[idx] = tanh(s1)
    end
    # output logits: every (sample, class) is independent
    for idx2 = 1:n_s * n_o
        i_s = div(idx2 - 1, n_o) + 1
        i_c = mod(idx2 - 1, n_o) + 1
        s2 = b2[i_c]
        for i_k = 1:n_h
            s2 = s2 + h[(i_s - 1) * n_h + i_k] * w2[(i_k - 1) * n_o + i_c]
        end
        z[idx2] = s2
    end
    # softmax cross-entropy, one sample per iteration
    for i_s = 1:n_s
        row_max = z[(i_s - 1) * n_o + 1]
        # running max is a sequential scan; max() avoids a branch
        for i_c = 2:n_o
            row_max = max(row_max, z[(i_s - 1) * n_o + i_c])
        end
        for i_c = 1:n_o
            p[(i_s - 1) * n_o + i_c] = exp(z[(i_s - 1) * n_o + i_c] - row_max)
        end
        row_sum = 0.0
        for i_c = 1:n_o
            row_sum = row_sum + p[(i_s - 1) * n_o + i_c]
        end
        for i_c = 1:n_o
            loss[1] = loss[1] - y[(i_s - 1) * n_o + i_c] * log(p[(i_s - 1) * n_o + i_c] / row_sum)
        end
    end
    return nothing
end

# heat2d(loss, u, un, alpha, n, n_step)
#
# Explicit periodic 5-point heat diffusion (configuration C3).
# loss: length-1 output, accumulated in place
# u: field n x n, row-major, advanced in place
# un: next-state scratch n x n
# alpha: diffusivity times dt / dx^2
function heat2d(loss, u, un, alpha, n, n_step)
    for i_t = 1:n_step
        # every cell is independent; periodic neighbours by mod
        for idx = 1:n * n
            i = div(idx - 1, n) + 1
            j = mod(idx - 1, n) + 1
            i_up = mod(i - 2, n) + 1
            i_dn = mod(i, n) + 1
            j_lf = mod(j - 2, n) + 1
            j_rt = mod(j, n) + 1
            c = u[idx]
            un[idx] = c + alpha * ((((u[(i_up - 1) * n + j] + u[(i_dn - 1) * n + j]) + u[(i - 1) * n + j_lf]) + u[(i - 1) * n + j_rt]) - 4.0 * c)
        end
        # the new state becomes the current one
        for idx2 = 1:n * n
            u[idx2] = un[idx2]
        end
    end
    for idx3 = 1:n * n
        loss[1] = loss[1] + u[idx3] ^ 2
    end
    return nothing
end

# conv1d_relu_mse(loss, x, w, t, z, r, n_b, n_c, n_l, n_o, n_k)
#
# Valid multi-channel 1-D convolution, ReLU, mean squared error
# (configuration C4).
# x: n_b x n_c x n_l; w: n_o x n_c x n_k
# t, z, r: n_b x n_o x (n_l - n_k + 1); z and r are scratch
function conv1d_relu_mse(loss, x, w, t, z, r, n_b, n_c, n_l, n_o, n_k)
    n_lo = n_l - n_k + 1
    # every (sample, output channel, position) is independent
    for idx = 1:n_b * n_o * n_lo
        i_b = div(idx - 1, n_o * n_lo) + 1
        i_o = mod(div(idx - 1, n_lo), n_o) + 1
        i_t = mod(idx - 1, n_lo) + 1
        a = 0.0
        for i_c = 1:n_c
            for i_k = 1:n_k
                a = a + w[((i_o - 1) * n_c + i_c - 1) * n_k + i_k] * x[((i_b - 1) * n_c + i_c - 1) * n_l + i_t + i_k - 1]
            end
        end
        z[idx] = a
        r[idx] = max(a, 0.0)
    end
    inv_n = 1.0 / (n_b * n_o * n_lo)
    for idx2 = 1:n_b * n_o * n_lo
        loss[1] = loss[1] + inv_n * (r[idx2] - t[idx2]) ^ 2
    end
    return nothing
end
