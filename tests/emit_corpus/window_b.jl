# Sliding window z[t] = tanh(sum_c w[c] x[t + c - 1]): the window's adjoint
# scalar is reset after every iteration (a convergent constant), and the
# windows overlap, so xb is accumulated from several iterations.
function initstacks_window_b(i_n, i_k)
    return nothing
end

function window_b(loss, lossb, x, xb, w, wb, z, zb, i_n, i_k)
    s = 0.0
    sb = 0.0
    for i_t = 1:i_n
        s = 0.0
        for i_c = 1:i_k
            s = s + w[i_c] * x[(i_t + i_c) - 1]
        end
        z[i_t] = tanh(s)
    end
    for i_t = 1:i_n
        loss[1] = loss[1] + z[i_t]
    end
    for i_t = i_n:-1:1
        zb[i_t] = zb[i_t] + lossb[1]
    end
    for i_t = i_n:-1:1
        s = 0.0
        for i_c = 1:i_k
            s = s + w[i_c] * x[(i_t + i_c) - 1]
        end
        __oldb_0 = zb[i_t]
        zb[i_t] = 0.0
        sb = sb + (1 - tanh(s) ^ 2) * __oldb_0
        for i_c = i_k:-1:1
            wb[i_c] = wb[i_c] + x[(i_t + i_c) - 1] * sb
            xb[(i_t + i_c) - 1] = xb[(i_t + i_c) - 1] + w[i_c] * sb
        end
        sb = 0.0
    end
    return nothing
end

function window(loss, x, w, z, i_n, i_k)
    for i_t = 1:i_n
        s = 0.0
        for i_c = 1:i_k
            s = s + w[i_c] * x[(i_t + i_c) - 1]
        end
        z[i_t] = tanh(s)
    end
    for i_t = 1:i_n
        loss[1] = loss[1] + z[i_t]
    end
end
