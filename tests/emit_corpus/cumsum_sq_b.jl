# Prefix sum then a sum of squares: the prefix recurrence carries a value
# between iterations in both sweeps, so those loops stay sequential.
function initstacks_cumsum_sq_b(i_n)
    return nothing
end

function cumsum_sq_b(loss, lossb, x, xb, c, cb, i_n)
    c[1] = x[1]
    for i_k = 2:i_n
        c[i_k] = c[i_k - 1] + x[i_k]
    end
    for i_k = 1:i_n
        loss[1] = loss[1] + c[i_k] ^ 2
    end
    for i_k = i_n:-1:1
        cb[i_k] = cb[i_k] + (2 * c[i_k]) * lossb[1]
    end
    for i_k = i_n:-1:2
        __oldb_0 = cb[i_k]
        cb[i_k] = 0.0
        cb[i_k - 1] = cb[i_k - 1] + __oldb_0
        xb[i_k] = xb[i_k] + __oldb_0
    end
    __oldb_1 = cb[1]
    cb[1] = 0.0
    xb[1] = xb[1] + __oldb_1
    return nothing
end

function cumsum_sq(loss, x, c, i_n)
    c[1] = x[1]
    for i_k = 2:i_n
        c[i_k] = c[i_k - 1] + x[i_k]
    end
    for i_k = 1:i_n
        loss[1] = loss[1] + c[i_k] ^ 2
    end
end
