# A ragged nest: the inner trip count i_m depends on the outer iteration, so
# the tape layout is Tier-B. initstacks runs the sizing loop, filling the
# prefix table of per-iteration offsets and the running total, as
# agen_tier_b_block_stmts writes it; the sweep tapes each inner value at
# prefix + i_k. Generated-code style; the primal is below.
function initstacks_ragged_b(i_n)
    prefix_v_stack_1 = Vector{Int}(undef, max(0, div(i_n - 1, 1) + 1))
    __tot_v_stack_1 = 0
    for i_i = 1:i_n
        prefix_v_stack_1[(i_i - 1) + 1] = __tot_v_stack_1
        i_m = mod(i_i, 3) + 1
        __tot_v_stack_1 = __tot_v_stack_1 + max(0, div(i_m - 1, 1) + 1)
    end
    v_stack = Vector{Float64}(undef, __tot_v_stack_1)
    return (v_stack, prefix_v_stack_1, __tot_v_stack_1)
end

function ragged_b(loss, lossb, x, xb, w, wb, i_n, v_stack, prefix_v_stack_1, __tot_v_stack_1)
    for i_i = 1:i_n
        i_m = mod(i_i, 3) + 1
        v = x[i_i]
        for i_k = 1:i_m
            v_stack[prefix_v_stack_1[(i_i - 1) + 1] + i_k] = v
            v = tanh(v * w[i_k])
        end
        loss[1] = loss[1] + v
    end
    for i_i = i_n:-1:1
        i_m = mod(i_i, 3) + 1
        vb = lossb[1]
        for i_k = i_m:-1:1
            v = v_stack[prefix_v_stack_1[(i_i - 1) + 1] + i_k]
            t = tanh(v * w[i_k])
            __cse_0 = (1 - t ^ 2) * vb
            wb[i_k] = wb[i_k] + v * __cse_0
            vb = w[i_k] * __cse_0
        end
        xb[i_i] = xb[i_i] + vb
    end
    return nothing
end

function ragged(loss, x, w, i_n)
    for i_i = 1:i_n
        i_m = mod(i_i, 3) + 1
        v = x[i_i]
        for i_k = 1:i_m
            v = tanh(v * w[i_k])
        end
        loss[1] = loss[1] + v
    end
end
