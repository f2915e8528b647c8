# Integer division by a divisor fixed for the loop (a host integer): every
# iteration indexes with div / mod / rem of its own number, negative and
# beyond 2^31 included. Not a derivative; it exercises the index arithmetic.
function divmod_b(x, xb, i_n, i_d)
    for i_k = 1:i_n
        i_q = div(i_k * 7919 - 1, i_d) + div(i_k - 3, i_d)
        i_r = mod(i_k * 104729 - 5, i_d) + mod(3 - i_k, i_d)
        i_s = rem(i_k * 1000003 - 7, i_d) + rem(2 - i_k, i_d)
        xb[i_k] = xb[i_k] + x[mod(i_q, i_n) + 1] * (i_r + 1) + x[mod(i_s, i_n) + 1]
    end
    return nothing
end
