# C3 periodic heat equation: the adjoint STADE generates for oracle/primals.jl's
# heat2d (the state overwritten by the copy loop is taped, thread loop fastest),
# written out in its output style; the same sweep oracle/oracle.cc restates.
function initstacks_heat2d_b(n, n_step)
    u_stack = Vector{Float64}(undef, max(0, div(n_step - 1, 1) + 1) * max(0, div(n * n - 1, 1) + 1))
    return u_stack
end

function heat2d_b(loss, lossb, u, ub, un, unb, alpha, alphab, n, n_step, u_stack)
    for i_t = 1:n_step
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
        for idx2 = 1:n * n
            __idx_u_stack_0 = ((idx2 - 1) + (i_t - 1) * (div(n * n - 1, 1) + 1)) + 1
            u_stack[__idx_u_stack_0] = u[idx2]
            u[idx2] = un[idx2]
        end
    end
    for idx3 = 1:n * n
        loss[1] = loss[1] + u[idx3] ^ 2
    end
    for idx3 = n * n:-1:1
        ub[idx3] = ub[idx3] + (2 * u[idx3]) * lossb[1]
    end
    for i_t = n_step:-1:1
        for idx2 = n * n:-1:1
            __idx_u_stack_0 = ((idx2 - 1) + (i_t - 1) * (div(n * n - 1, 1) + 1)) + 1
            u[idx2] = u_stack[__idx_u_stack_0]
            __oldb_0 = ub[idx2]
            ub[idx2] = 0.0
            unb[idx2] = unb[idx2] + __oldb_0
        end
        for idx = n * n:-1:1
            i = div(idx - 1, n) + 1
            j = mod(idx - 1, n) + 1
            i_up = mod(i - 2, n) + 1
            i_dn = mod(i, n) + 1
            j_lf = mod(j - 2, n) + 1
            j_rt = mod(j, n) + 1
            __oldb_1 = unb[idx]
            unb[idx] = 0.0
            c = u[idx]
            __cse_0 = alpha * __oldb_1
            ub[idx] = ub[idx] + __oldb_1
            alphab = alphab + ((((u[(i_up - 1) * n + j] + u[(i_dn - 1) * n + j]) + u[(i - 1) * n + j_lf]) + u[(i - 1) * n + j_rt]) - 4.0 * c) * __oldb_1
            ub[(i_up - 1) * n + j] = ub[(i_up - 1) * n + j] + __cse_0
            ub[(i_dn - 1) * n + j] = ub[(i_dn - 1) * n + j] + __cse_0
            ub[(i - 1) * n + j_lf] = ub[(i - 1) * n + j_lf] + __cse_0
            ub[(i - 1) * n + j_rt] = ub[(i - 1) * n + j_rt] + __cse_0
            ub[idx] = ub[idx] + 4.0 * -__cse_0
        end
    end
    return alphab
end
