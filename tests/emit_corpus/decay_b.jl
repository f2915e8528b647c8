# Explicit decay du/dt = -k u over i_nstep steps (u overwritten in place, so the
# reverse sweep restores it from a tape), float scalar arguments k and dt whose
# adjoints the sweep returns. Generated-code style; the primal is below.
function initstacks_decay_b(i_n, i_nstep)
    u_stack = Vector{Float64}(undef, max(0, div(i_nstep - 1, 1) + 1) * max(0, div(i_n - 1, 1) + 1))
    return u_stack
end

function decay_b(u, ub, k, kb, dt, dtb, i_n, i_nstep, u_stack)
    for i_ = 1:i_nstep
        for i_x = 1:i_n
            __idx_u_stack_0 = ((i_x - 1) + (i_ - 1) * (div(i_n - 1, 1) + 1)) + 1
            u_stack[__idx_u_stack_0] = u[i_x]
            u[i_x] = u[i_x] - (k * dt) * u[i_x]
        end
    end
    for i_ = i_nstep:-1:1
        for i_x = i_n:-1:1
            __idx_u_stack_0 = ((i_x - 1) + (i_ - 1) * (div(i_n - 1, 1) + 1)) + 1
            u[i_x] = u_stack[__idx_u_stack_0]
            __oldb_0 = ub[i_x]
            ub[i_x] = 0.0
            __cse_0 = -__oldb_0
            ub[i_x] = ub[i_x] + __oldb_0
            kb = kb + (dt * u[i_x]) * __cse_0
            dtb = dtb + (k * u[i_x]) * __cse_0
            ub[i_x] = ub[i_x] + (k * dt) * __cse_0
        end
    end
    return (kb, dtb)
end

function decay(u, k, dt, i_n, i_nstep)
    for i_ = 1:i_nstep
        for i_x = 1:i_n
            u[i_x] = u[i_x] - (k * dt) * u[i_x]
        end
    end
end
