# C1 affine least squares: the adjoint STADE generates for oracle/primals.jl's
# affine_ls (keep_push_pop = false), written out in its output style; the same
# sweep oracle/oracle.cc restates in C++.
function initstacks_affine_ls_b(n_s, n_o, n_i)
    return nothing
end

function affine_ls_b(loss, lossb, w, wb, b, bb, x, xb, t, tb, y, yb, n_s, n_o, n_i)
    s = 0.0
    sb = 0.0
    for idx = 1:n_s * n_o
        i_s = div(idx - 1, n_o) + 1
        i_o = mod(idx - 1, n_o) + 1
        s = b[i_o]
        for i_k = 1:n_i
            s = s + w[(i_o - 1) * n_i + i_k] * x[(i_s - 1) * n_i + i_k]
        end
        y[idx] = s
    end
    for idx2 = 1:n_s * n_o
        loss[1] = loss[1] + 0.5 * (y[idx2] - t[idx2]) ^ 2
    end
    for idx2 = n_s * n_o:-1:1
        __cse_0 = y[idx2] - t[idx2]
        __cse_1 = (0.5 * (2 * __cse_0)) * lossb[1]
        yb[idx2] = yb[idx2] + __cse_1
        tb[idx2] = tb[idx2] + -__cse_1
    end
    for idx = n_s * n_o:-1:1
        i_s = div(idx - 1, n_o) + 1
        i_o = mod(idx - 1, n_o) + 1
        __oldb_0 = yb[idx]
        yb[idx] = 0.0
        sb = sb + __oldb_0
        for i_k = n_i:-1:1
            wb[(i_o - 1) * n_i + i_k] = wb[(i_o - 1) * n_i + i_k] + x[(i_s - 1) * n_i + i_k] * sb
            xb[(i_s - 1) * n_i + i_k] = xb[(i_s - 1) * n_i + i_k] + w[(i_o - 1) * n_i + i_k] * sb
        end
        __oldb_1 = sb
        sb = 0.0
        bb[i_o] = bb[i_o] + __oldb_1
    end
    return nothing
end
