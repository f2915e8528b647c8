# Bilinear form x' A z over a flattened (i, j) nest with div / mod decoded
# indices and a column-major 2-D array a (i_m x i_n).
function initstacks_bilin_b(i_m, i_n)
    return nothing
end

function bilin_b(loss, lossb, a, ab, x, xb, z, zb, i_m, i_n)
    for idx = 1:i_m * i_n
        i_i = div(idx - 1, i_n) + 1
        i_j = mod(idx - 1, i_n) + 1
        loss[1] = loss[1] + x[i_i] * a[i_i, i_j] * z[i_j]
    end
    for idx = i_m * i_n:-1:1
        __icse_0 = idx - 1
        i_i = div(__icse_0, i_n) + 1
        i_j = mod(__icse_0, i_n) + 1
        __cse_1 = lossb[1]
        __cse_2 = a[i_i, i_j] * z[i_j]
        xb[i_i] = xb[i_i] + __cse_2 * __cse_1
        ab[i_i, i_j] = ab[i_i, i_j] + (x[i_i] * z[i_j]) * __cse_1
        zb[i_j] = zb[i_j] + (x[i_i] * a[i_i, i_j]) * __cse_1
    end
    return nothing
end

function bilin(loss, a, x, z, i_m, i_n)
    for idx = 1:i_m * i_n
        i_i = div(idx - 1, i_n) + 1
        i_j = mod(idx - 1, i_n) + 1
        loss[1] = loss[1] + x[i_i] * a[i_i, i_j] * z[i_j]
    end
end
