"""Checks, on the CPU in fp64, the chunked form of the gated delta rule that the CUDA kernels compute.

The kernels in ``sorernn_b200/csrc`` do not run the per-token recurrence of the reference
(sore/model/gdn_ref.py:17-22); they run a chunk decomposition of it (WY/UT transform inside a chunk,
a dk x dv state pass between chunks) and its hand-derived reverse mode. This file restates exactly
that algebra in numpy, with the same padding rule the kernels use for a partial last chunk (padded
rows carry k = v = q = 0, beta = 0, g = 0), and checks it against the oracle. A wrong formula here
would be a wrong kernel, so the check runs without a GPU.
"""
import numpy as np
import pytest

from inputs import make_inputs, make_state_inputs
from oracle import gdn_oracle as orc

C = 16  # small chunk so that the cases below cross several chunk boundaries


def _pad(x, n):
    out = np.zeros((n,) + x.shape[1:], x.dtype)
    out[: x.shape[0]] = x
    return out


def _chunk_terms(q, k, v, g, beta, S0, scale):
    Gam = np.cumsum(g)
    idx = np.arange(len(g))
    low_incl = idx[:, None] >= idx[None, :]
    low_strict = idx[:, None] > idx[None, :]
    E = np.where(low_incl, np.exp(np.where(low_incl, Gam[:, None] - Gam[None, :], 0.0)), 0.0)
    G = k @ k.T
    A = np.where(low_strict, beta[:, None] * G * E, 0.0)
    Tm = np.linalg.inv(np.eye(len(g)) + A)
    eG = np.exp(Gam)
    W = Tm @ ((beta * eG)[:, None] * k)
    U = Tm @ (beta[:, None] * v)
    D = U - W @ S0
    P = scale * np.where(low_incl, (q @ k.T) * E, 0.0)
    O_inter = scale * eG[:, None] * (q @ S0)
    O = O_inter + P @ D
    dec = np.exp(Gam[-1] - Gam)
    S1 = np.exp(Gam[-1]) * S0 + (k * dec[:, None]).T @ D
    return dict(Gam=Gam, E=E, G=G, A=A, T=Tm, eG=eG, W=W, U=U, D=D, P=P, O=O, O_inter=O_inter, dec=dec,
                S1=S1, low_incl=low_incl, low_strict=low_strict)


def chunked_forward(q, k, v, g, beta, scale, S0):
    """One (sequence, head): q,k [T,dk], v [T,dv], g,beta [T]. Returns o, final state, chunk-start states."""
    T = q.shape[0]
    o = np.zeros_like(v)
    S = S0.copy()
    starts = []
    for t0 in range(0, T, C):
        n = min(C, T - t0)
        sl = slice(t0, t0 + n)
        starts.append(S.copy())
        r = _chunk_terms(_pad(q[sl], C), _pad(k[sl], C), _pad(v[sl], C), _pad(g[sl], C), _pad(beta[sl], C), S, scale)
        o[sl] = r["O"][:n]
        S = r["S1"]
    return o, S, starts


def chunked_backward(q, k, v, g, beta, do, scale, S0, dht):
    T = q.shape[0]
    _, _, starts = chunked_forward(q, k, v, g, beta, scale, S0)
    dq, dk, dv = np.zeros_like(q), np.zeros_like(k), np.zeros_like(v)
    dg, db = np.zeros_like(g), np.zeros_like(beta)
    dS = dht.copy()
    for ci in reversed(range(len(starts))):
        t0 = ci * C
        n = min(C, T - t0)
        sl = slice(t0, t0 + n)
        Q, K, V, Gg, Bt, dO = (_pad(x[sl], C) for x in (q, k, v, g, beta, do))
        Sc = starts[ci]
        r = _chunk_terms(Q, K, V, Gg, Bt, Sc, scale)
        Tm, W, D, P, E, eG, dec, A, G = (r[x] for x in ("T", "W", "D", "P", "E", "eG", "dec", "A", "G"))
        Kd = K * dec[:, None]
        dD = P.T @ dO + Kd @ dS
        dS0 = scale * (Q * eG[:, None]).T @ dO + np.exp(r["Gam"][-1]) * dS - W.T @ dD
        dP = dO @ D.T
        dPs = np.where(r["low_incl"], dP * scale * E, 0.0)
        dQ = scale * eG[:, None] * (dO @ Sc.T) + dPs @ K
        dKst = (D @ dS.T) * dec[:, None]
        dK = dPs.T @ Q + dKst
        dW = -dD @ Sc.T
        dT = dD @ (Bt[:, None] * V).T + dW @ ((Bt * eG)[:, None] * K).T
        dVb = Tm.T @ dD
        dKb = Tm.T @ dW
        dV = Bt[:, None] * dVb
        dB = (dVb * V).sum(1) + eG * (dKb * K).sum(1)
        dK += (Bt * eG)[:, None] * dKb
        dA = np.where(r["low_strict"], -Tm.T @ dT @ Tm.T, 0.0)
        dB += (dA * G * E).sum(1)
        dG = dA * Bt[:, None] * E
        dK += (dG + dG.T) @ K
        XA = dA * A
        XP = np.where(r["low_incl"], dP * P, 0.0)
        dGam = XA.sum(1) - XA.sum(0) + XP.sum(1) - XP.sum(0)
        dGam += (dO * r["O_inter"]).sum(1)
        dGam += Bt * eG * (dKb * K).sum(1)
        term = (K * dKst).sum(1)
        dGam -= term
        dGam[-1] += term.sum() + np.exp(r["Gam"][-1]) * (dS * Sc).sum()
        dgc = np.cumsum(dGam[::-1])[::-1]
        dq[sl], dk[sl], dv[sl], dg[sl], db[sl] = dQ[:n], dK[:n], dV[:n], dgc[:n], dB[:n]
        dS = dS0
    return dq, dk, dv, dg, db, dS


@pytest.mark.parametrize("T", [1, 5, 16, 37, 64])
def test_chunked_forward_and_backward_equal_recurrence(T):
    dk_, dv_ = 8, 6
    x = make_inputs(100 + T, 1, T, 1, 1, dk_, dv_, g_mode="uniform")
    h0, dht = make_state_inputs(100 + T, 1, 1, dk_, dv_)
    scale = 0.4
    o_ref, ht_ref = orc.gdn_forward(x["q"], x["k"], x["v"], x["g"], x["beta"], scale, initial_state=h0)
    grads_ref = orc.gdn_backward(x["q"], x["k"], x["v"], x["g"], x["beta"], x["do"], scale,
                                 initial_state=h0, dht=dht)
    sq = lambda a: a[0, :, 0]  # noqa: E731
    o, ht, _ = chunked_forward(sq(x["q"]), sq(x["k"]), sq(x["v"]), sq(x["g"]), sq(x["beta"]), scale, h0[0, 0])
    np.testing.assert_allclose(o, sq(o_ref), atol=1e-12)
    np.testing.assert_allclose(ht, ht_ref[0, 0], atol=1e-12)
    got = chunked_backward(sq(x["q"]), sq(x["k"]), sq(x["v"]), sq(x["g"]), sq(x["beta"]), sq(x["do"]), scale,
                           h0[0, 0], dht[0, 0])
    names = ("dq", "dk", "dv", "dg", "dbeta", "dh0")
    for name, a, b in zip(names, got, grads_ref):
        b = b[0, 0] if name == "dh0" else sq(b)
        np.testing.assert_allclose(a, b, atol=1e-10, err_msg=name)


def block_doubling_inverse(A):
    """The kernels' (I + A)^-1 for a strictly lower 64 x 64 A (chunk_common.cuh, tri_inverse64): 16 x 16
    diagonal blocks by forward substitution, then 16 -> 32 and 32 -> 64 merges via the lower-left block
    -T1 (A10 T0) of [[I + A00, 0], [A10, I + A11]]^-1."""
    T = np.array(A, dtype=np.float64)
    for b in range(4):
        s = slice(16 * b, 16 * b + 16)
        L = np.eye(16) + np.tril(A[s, s], -1)
        X = np.zeros((16, 16))
        for c in range(16):  # column c: forward substitution
            for i in range(16):
                X[i, c] = (1.0 if i == c else 0.0) - L[i, :i] @ X[:i, c] if i >= c else 0.0
        T[s, s] = X
    for size in (16, 32):
        for p in range(0, 64, 2 * size):
            r0, c0 = p + size, p
            Y = A[r0:r0 + size, c0:c0 + size] @ T[c0:c0 + size, c0:c0 + size]
            T[r0:r0 + size, c0:c0 + size] = -T[r0:r0 + size, r0:r0 + size] @ Y
    return T


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_block_doubling_inverse(seed):
    rng = np.random.default_rng(seed)
    A = np.tril(rng.standard_normal((64, 64)) * 0.3, -1)
    T = block_doubling_inverse(A)
    np.testing.assert_allclose(T, np.linalg.inv(np.eye(64) + A), rtol=1e-9, atol=1e-9)
    assert np.all(np.triu(T, 1) == 0)
