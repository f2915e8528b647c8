# Edge loss over a graph: each edge's endpoints come from an integer table
# i_e2n (2 x i_ne, column-major), a branch taken per edge is recorded on an
# integer stack, and the endpoint adjoints scatter through the table.
function initstacks_edge_relu_b(i_ne)
    branch_stack = Vector{Int64}(undef, max(0, div(i_ne - 1, 1) + 1))
    return branch_stack
end

function edge_relu_b(loss, lossb, x, xb, w, wb, i_e2n, i_ne, branch_stack)
    d = 0.0
    db = 0.0
    for i_e = 1:i_ne
        d = x[i_e2n[1, i_e]] - x[i_e2n[2, i_e]]
        if d > 0.0
            __idx_branch_stack_0 = (i_e - 1) + 1
            branch_stack[__idx_branch_stack_0] = 1
            loss[1] = loss[1] + w[i_e] * d ^ 2
        else
            __idx_branch_stack_0 = (i_e - 1) + 1
            branch_stack[__idx_branch_stack_0] = 0
        end
    end
    for i_e = i_ne:-1:1
        d = x[i_e2n[1, i_e]] - x[i_e2n[2, i_e]]
        __idx_branch_stack_0 = (i_e - 1) + 1
        __branch = branch_stack[__idx_branch_stack_0]
        if __branch == 1
            __cse_0 = lossb[1]
            wb[i_e] = wb[i_e] + d ^ 2 * __cse_0
            db = db + (w[i_e] * (2 * d)) * __cse_0
        end
        __oldb_0 = db
        db = 0.0
        xb[i_e2n[1, i_e]] = xb[i_e2n[1, i_e]] + __oldb_0
        xb[i_e2n[2, i_e]] = xb[i_e2n[2, i_e]] + -__oldb_0
    end
    return nothing
end

function edge_relu(loss, x, w, i_e2n, i_ne)
    for i_e = 1:i_ne
        d = x[i_e2n[1, i_e]] - x[i_e2n[2, i_e]]
        if d > 0.0
            loss[1] = loss[1] + w[i_e] * d ^ 2
        end
    end
end
