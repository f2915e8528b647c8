"""Independent closed-form derivatives (numpy, Float64) of the five primals.

These do not follow the generated statement order; they are the textbook
gradients of the same functions, used to pin the oracle (which does follow
it) from outside.
"""
import numpy as np


def affine_ls(w, b, x, t, lossb, n_s, n_o, n_i):
    W = w.reshape(n_o, n_i)
    X = x.reshape(n_s, n_i)
    T = t.reshape(n_s, n_o)
    Y = X @ W.T + b
    r = (Y - T) * lossb[0]
    return dict(y=Y.ravel(), loss=0.5 * np.sum((Y - T) ** 2), wb=(r.T @ X).ravel(), bb=r.sum(0),
                xb=(r @ W).ravel(), tb=(-r).ravel())


def mlp2_ce(x, y, w1, b1, w2, b2, lossb, n_s, n_i, n_h, n_o):
    X = x.reshape(n_s, n_i)
    Y = y.reshape(n_s, n_o)
    W1 = w1.reshape(n_i, n_h)
    W2 = w2.reshape(n_h, n_o)
    H = np.tanh(X @ W1 + b1)
    Z = H @ W2 + b2
    m = Z.max(1, keepdims=True)
    E = np.exp(Z - m)
    rs = E.sum(1, keepdims=True)
    logq = np.log(E / rs)
    loss = -np.sum(Y * logq)
    lb = lossb[0]
    g = (E / rs * Y.sum(1, keepdims=True) - Y) * lb
    hb = g @ W2.T
    s1b = (1 - H ** 2) * hb
    return dict(h=H.ravel(), z=Z.ravel(), p=E.ravel(), loss=loss, yb=(-logq * lb).ravel(),
                w2b=(H.T @ g).ravel(), b2b=g.sum(0), w1b=(X.T @ s1b).ravel(), b1b=s1b.sum(0),
                xb=(s1b @ W1.T).ravel(), g=g, s1b=s1b)


def heat2d(u0, alpha, n, n_step, lossb):
    """Forward states (bit-for-bit the primal's arithmetic order), loss,
    gradient w.r.t. u0 and dloss/dalpha."""
    U = u0.reshape(n, n).copy()
    states = []
    for _ in range(n_step):
        states.append(U.copy())
        up = np.roll(U, 1, 0)
        dn = np.roll(U, -1, 0)
        lf = np.roll(U, 1, 1)
        rt = np.roll(U, -1, 1)
        U = U + alpha * ((((up + dn) + lf) + rt) - 4.0 * U)
    loss = np.sum(U * U)
    G = 2.0 * U * lossb[0]
    alphab = 0.0
    for k in range(n_step - 1, -1, -1):
        S = states[k]
        lap = (np.roll(S, 1, 0) + np.roll(S, -1, 0) + np.roll(S, 1, 1) + np.roll(S, -1, 1)) - 4.0 * S
        alphab += np.sum(lap * G)
        G = G + alpha * ((np.roll(G, 1, 0) + np.roll(G, -1, 0) + np.roll(G, 1, 1)
                          + np.roll(G, -1, 1)) - 4.0 * G)
    return dict(states=states, final=U, loss=loss, ub=G.ravel(), alphab=alphab)


def conv1d_relu_mse(x, w, t, lossb, n_b, n_c, n_l, n_o, n_k):
    n_lo = n_l - n_k + 1
    X = x.reshape(n_b, n_c, n_l)
    W = w.reshape(n_o, n_c, n_k)
    T = t.reshape(n_b, n_o, n_lo)
    # windows[b, c, t, k] = X[b, c, t + k]
    win = np.stack([X[:, :, k:k + n_lo] for k in range(n_k)], axis=-1)
    Z = np.einsum("ock,bctk->bot", W, win)
    R = np.maximum(Z, 0.0)
    inv_n = 1.0 / (n_b * n_o * n_lo)
    loss = inv_n * np.sum((R - T) ** 2)
    relu_d = 0.5 * (1.0 + np.sign(Z))
    G = relu_d * (inv_n * 2.0 * (R - T)) * lossb[0]
    wb = np.einsum("bot,bctk->ock", G, win)
    xb = np.zeros_like(X)
    for k in range(n_k):
        xb[:, :, k:k + n_lo] += np.einsum("oc,bot->bct", W[:, :, k], G)
    tb = -(inv_n * 2.0 * (R - T)) * lossb[0]
    return dict(z=Z.ravel(), r=R.ravel(), loss=loss, wb=wb.ravel(), xb=xb.ravel(), tb=tb.ravel(),
                g=G)


def rel_err(a, b) -> float:
    """Normwise relative error max|a - b| / max|b| (0 when both are zero)."""
    a = np.asarray(a, dtype=np.float64).ravel()
    b = np.asarray(b, dtype=np.float64).ravel()
    den = np.max(np.abs(b)) if b.size else 0.0
    num = np.max(np.abs(a - b)) if a.size else 0.0
    if den == 0.0:
        return float(num)
    return float(num / den)


def ref_rel_err(a, b) -> float:
    """The reference's element-wise relative error, max_i |a_i - b_i| /
    max(|a_i|, |b_i|, 1) (_relerr_arr of the generated GPU parity script,
    src/STADE.jl:18980)."""
    a = np.asarray(a, dtype=np.float64).ravel()
    b = np.asarray(b, dtype=np.float64).ravel()
    if a.size == 0:
        return 0.0
    return float(np.max(np.abs(a - b) / np.maximum(np.maximum(np.abs(a), np.abs(b)), 1.0)))


def elem_rel_err(a, b, floor_frac) -> float:
    """Element-wise relative error against b with a floor scaled to the
    array: max_i |a_i - b_i| / max(|b_i|, floor_frac * max_j |b_j|). With
    floor_frac = 0 every element counts relative to itself (exact zeros in b
    must then be exact in a)."""
    a = np.asarray(a, dtype=np.float64).ravel()
    b = np.asarray(b, dtype=np.float64).ravel()
    if a.size == 0:
        return 0.0
    d = np.abs(a - b)
    den = np.maximum(np.abs(b), floor_frac * float(np.max(np.abs(b))))
    with np.errstate(divide="ignore", invalid="ignore"):
        r = np.where(d == 0.0, 0.0, d / den)
    return float(np.max(r))
