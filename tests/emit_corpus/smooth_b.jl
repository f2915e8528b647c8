# Three-point smoothing then a sum of squares: the reverse sweep scatters each
# cell's adjoint to its two neighbours (constant offsets -1, 0, +1), which the
# emitter turns into a gather over the cells.
function initstacks_smooth_b(i_n)
    return nothing
end

function smooth_b(loss, lossb, u, ub, v, vb, i_n)
    for i_x = 2:i_n - 1
        v[i_x] = (u[i_x - 1] + 2.0 * u[i_x]) + u[i_x + 1]
    end
    for i_x2 = 2:i_n - 1
        loss[1] = loss[1] + v[i_x2] ^ 2
    end
    for i_x2 = i_n - 1:-1:2
        vb[i_x2] = vb[i_x2] + (2 * v[i_x2]) * lossb[1]
    end
    for i_x = i_n - 1:-1:2
        __oldb_0 = vb[i_x]
        vb[i_x] = 0.0
        ub[i_x - 1] = ub[i_x - 1] + __oldb_0
        ub[i_x] = ub[i_x] + 2.0 * __oldb_0
        ub[i_x + 1] = ub[i_x + 1] + __oldb_0
    end
    return nothing
end

function smooth(loss, u, v, i_n)
    for i_x = 2:i_n - 1
        v[i_x] = (u[i_x - 1] + 2.0 * u[i_x]) + u[i_x + 1]
    end
    for i_x2 = 2:i_n - 1
        loss[1] = loss[1] + v[i_x2] ^ 2
    end
end
