# A while loop (trip count known only at run time): it runs in a one-thread
# kernel, in order. Not a derivative; it exercises the sequential path.
function halving_b(x, xb, i_n)
    i_m = i_n
    while i_m > 1
        for i_k = 1:div(i_m, 2)
            x[i_k] = x[i_k] + x[i_k + div(i_m, 2)]
        end
        i_m = div(i_m, 2)
    end
    for i_k = 1:i_n
        xb[i_k] = xb[i_k] + 2.0 * x[1]
    end
    return nothing
end
