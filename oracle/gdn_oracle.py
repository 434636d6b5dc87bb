"""CPU oracle for the gated delta rule: TEST INFRASTRUCTURE ONLY.

This module is the checker for the CUDA path. Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import it. The product path
(``sorernn_b200``) never calls it and has no CPU fallback.

It restates, in numpy, the reference's sequential gated delta rule
(soreRNN ``sore/model/gdn_ref.py``):

* ``_recurrence`` (gdn_ref.py:11-22): per token, in this order
  ``S <- exp(g_t) * S``; ``delta = beta_t * (v_t - S^T k_t)``; ``S <- S + k_t delta^T``;
  ``o_t = scale * S^T q_t``. The state is ``[dk, dv]`` per (sequence, head) and starts at zero.
* ``naive_gated_delta_rule`` (gdn_ref.py:25-61): fp32 compute (fp64 kept), output in the dtype of
  ``v``, ``cu_seqlens`` requires B == 1 and resets the state at each document start.
* GVA head mapping (gdn.py:171-174, ``repeat_interleave``): value head ``i`` reads q/k head
  ``i // (HV // H)``.
* q/k L2 norm (gdn.py:177, ``F.normalize``): ``x / max(||x||_2, 1e-12)``.

Three things the reference oracle does not have are restated from the same recurrence and are
therefore *parity unpinned* by the reference's own tests: a seeded ``initial_state``, the returned
final state, and the single-token decode step. The backward is the hand-derived reverse-mode of the
same per-token recurrence (the reference obtains it from torch autograd through gdn_ref.py:17-22);
it is pinned against autograd outputs of the reference in ``tests/golden``.
"""
from __future__ import annotations

import numpy as np

L2_EPS = 1e-12


def _compute_dtype(dtype) -> np.dtype:
    # gdn_ref.py:45-46 promotes to at least fp32 and keeps fp64.
    return np.promote_types(np.dtype(dtype), np.float32)


def _bounds(T: int, B: int, cu_seqlens) -> list[tuple[int, int, int]]:
    """(batch row, start, end) of every sequence; gdn_ref.py:42-43,53-56 validation rules."""
    if cu_seqlens is None:
        return [(b, 0, T) for b in range(B)]
    cu = [int(x) for x in np.asarray(cu_seqlens).tolist()]
    if B != 1:
        raise ValueError(f"cu_seqlens requires B == 1, got B = {B}")
    if cu[0] != 0 or cu[-1] != T:
        raise ValueError(f"cu_seqlens must run from 0 to T = {T}, got {cu[0]}..{cu[-1]}")
    return [(0, a, b) for a, b in zip(cu[:-1], cu[1:])]


def l2norm(x: np.ndarray) -> np.ndarray:
    n = np.sqrt((x * x).sum(-1, keepdims=True))
    return x / np.maximum(n, L2_EPS)


def l2norm_backward(x: np.ndarray, dy: np.ndarray) -> np.ndarray:
    """Gradient of ``x / max(||x||, eps)`` (the ``F.normalize`` of gdn.py:177)."""
    n = np.sqrt((x * x).sum(-1, keepdims=True))
    nn_ = np.maximum(n, L2_EPS)
    y = x / nn_
    return (dy - y * (y * dy).sum(-1, keepdims=True) * (n > L2_EPS)) / nn_


def _head_map(H: int, HV: int) -> np.ndarray:
    if HV % H:
        raise ValueError(f"HV={HV} must be a multiple of H={H}")
    return np.arange(HV) // (HV // H)


def gdn_forward(q, k, v, g, beta, scale=None, initial_state=None, cu_seqlens=None,
                use_qk_l2norm=False, output_final_state=True):
    """Sequential gated delta rule forward.

    Shapes: ``q, k [B,T,H,dk]``, ``v [B,T,HV,dv]``, ``g, beta [B,T,HV]``,
    ``initial_state [N,HV,dk,dv]`` (N sequences). Returns ``(o [B,T,HV,dv], final [N,HV,dk,dv])``.
    """
    B, T, H, dk = q.shape
    HV, dv = v.shape[2], v.shape[3]
    scale = dk ** -0.5 if scale is None else scale
    cdt = _compute_dtype(v.dtype)
    q, k, v, g, beta = (np.asarray(x, dtype=cdt) for x in (q, k, v, g, beta))
    if use_qk_l2norm:
        q, k = l2norm(q), l2norm(k)
    hm = _head_map(H, HV)
    seqs = _bounds(T, B, cu_seqlens)
    o = np.zeros((B, T, HV, dv), dtype=cdt)
    final = np.zeros((len(seqs), HV, dk, dv), dtype=cdt)
    for n, (b, a, e) in enumerate(seqs):
        S = np.zeros((HV, dk, dv), dtype=cdt)
        if initial_state is not None:
            S[...] = np.asarray(initial_state[n], dtype=cdt)
        for t in range(a, e):
            qt, kt = q[b, t, hm], k[b, t, hm]  # [HV, dk]
            S = S * np.exp(g[b, t])[:, None, None]
            delta = (v[b, t] - np.einsum("hkv,hk->hv", S, kt)) * beta[b, t][:, None]
            S = S + kt[:, :, None] * delta[:, None, :]
            o[b, t] = np.einsum("hk,hkv->hv", qt * scale, S)
        final[n] = S
    return o, (final if output_final_state else None)


def gdn_backward(q, k, v, g, beta, do, scale=None, initial_state=None, dht=None, cu_seqlens=None,
                 use_qk_l2norm=False):
    """Reverse-mode of :func:`gdn_forward` (per-token reverse recurrence).

    With ``dH`` the gradient of the state after token t:
    ``dH += scale q do^T``; ``dq = scale S_t do``; ``ddelta = dH^T k``;
    ``dk = dH delta - beta S' ddelta``; ``dv = beta ddelta``; ``dbeta = ddelta . (v - S'^T k)``;
    ``dS' = dH - beta k ddelta^T``; ``dg = <dS', S'>``; ``dH <- exp(g) dS'``,
    where ``S' = exp(g_t) S_{t-1}``. Returns ``dq, dk, dv, dg, dbeta, dh0``.
    """
    B, T, H, dk = q.shape
    HV, dv = v.shape[2], v.shape[3]
    scale = dk ** -0.5 if scale is None else scale
    cdt = _compute_dtype(v.dtype)
    q_raw, k_raw = np.asarray(q, dtype=cdt), np.asarray(k, dtype=cdt)
    v, g, beta, do = (np.asarray(x, dtype=cdt) for x in (v, g, beta, do))
    q, k = (l2norm(q_raw), l2norm(k_raw)) if use_qk_l2norm else (q_raw, k_raw)
    hm = _head_map(H, HV)
    seqs = _bounds(T, B, cu_seqlens)
    dq = np.zeros((B, T, H, dk), dtype=cdt)
    dk_ = np.zeros((B, T, H, dk), dtype=cdt)
    dv_ = np.zeros((B, T, HV, dv), dtype=cdt)
    dg = np.zeros((B, T, HV), dtype=cdt)
    db = np.zeros((B, T, HV), dtype=cdt)
    dh0 = np.zeros((len(seqs), HV, dk, dv), dtype=cdt)
    for n, (b, a, e) in enumerate(seqs):
        S = np.zeros((HV, dk, dv), dtype=cdt)
        if initial_state is not None:
            S[...] = np.asarray(initial_state[n], dtype=cdt)
        states = []  # S_{t-1} for every t (oracle sizes only)
        for t in range(a, e):
            states.append(S)
            kt = k[b, t, hm]
            Sd = S * np.exp(g[b, t])[:, None, None]
            delta = (v[b, t] - np.einsum("hkv,hk->hv", Sd, kt)) * beta[b, t][:, None]
            S = Sd + kt[:, :, None] * delta[:, None, :]
        dH = np.zeros((HV, dk, dv), dtype=cdt)
        if dht is not None:
            dH[...] = np.asarray(dht[n], dtype=cdt)
        for t in range(e - 1, a - 1, -1):
            qt, kt = q[b, t, hm], k[b, t, hm]
            gam = np.exp(g[b, t])
            Sd = states[t - a] * gam[:, None, None]
            p = np.einsum("hkv,hk->hv", Sd, kt)
            u = v[b, t] - p
            delta = u * beta[b, t][:, None]
            St = Sd + kt[:, :, None] * delta[:, None, :]
            dH = dH + scale * qt[:, :, None] * do[b, t][:, None, :]
            dqt = scale * np.einsum("hkv,hv->hk", St, do[b, t])
            ddelta = np.einsum("hkv,hk->hv", dH, kt)
            dkt = np.einsum("hkv,hv->hk", dH, delta) - beta[b, t][:, None] * np.einsum("hkv,hv->hk", Sd, ddelta)
            dv_[b, t] = beta[b, t][:, None] * ddelta
            db[b, t] = (ddelta * u).sum(-1)
            dSd = dH - beta[b, t][:, None, None] * kt[:, :, None] * ddelta[:, None, :]
            dg[b, t] = (dSd * Sd).sum((-1, -2))
            dH = dSd * gam[:, None, None]
            np.add.at(dq[b, t], hm, dqt)
            np.add.at(dk_[b, t], hm, dkt)
        dh0[n] = dH
    if use_qk_l2norm:
        dq = l2norm_backward(q_raw, dq)
        dk_ = l2norm_backward(k_raw, dk_)
    return dq, dk_, dv_, dg, db, dh0


def gdn_decode_step(q, k, v, g, beta, state, scale=None, use_qk_l2norm=False):
    """One token of the recurrence on a resident state (gdn_ref.py:18-21), state updated in place.

    ``q, k [N,H,dk]``, ``v [N,HV,dv]``, ``g, beta [N,HV]``, ``state [N,HV,dk,dv]``. Returns ``o``.
    """
    N, H, dk = q.shape
    HV = v.shape[1]
    scale = dk ** -0.5 if scale is None else scale
    cdt = _compute_dtype(state.dtype)
    q, k, v, g, beta = (np.asarray(x, dtype=cdt) for x in (q, k, v, g, beta))
    if use_qk_l2norm:
        q, k = l2norm(q), l2norm(k)
    hm = _head_map(H, HV)
    qt, kt = q[:, hm], k[:, hm]
    S = state * np.exp(g)[..., None, None]
    delta = (v - np.einsum("nhkv,nhk->nhv", S, kt)) * beta[..., None]
    S = S + kt[..., :, None] * delta[..., None, :]
    state[...] = S
    return np.einsum("nhk,nhkv->nhv", qt * scale, S)


def gate_and_beta(a, b, A_log, dt_bias):
    """``g = -exp(A_log) * softplus(a + dt_bias)`` and ``beta = sigmoid(b)`` (gdn.py:191-194)."""
    x = np.asarray(a, np.float64) + np.asarray(dt_bias, np.float64)
    sp = np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, 20))))
    g = -np.exp(np.asarray(A_log, np.float64)) * sp
    beta = 1.0 / (1.0 + np.exp(-np.asarray(b, np.float64)))
    return g, beta


def rms_norm_gated(x, g, weight, eps):
    """The layer's output step (gdn.py:180-188; RMSNorm of layers.py:15-18):
    ``x * rsqrt(mean(x^2, -1) + eps) * weight * silu(g)``, in fp64."""
    x, g, w = (np.asarray(t, np.float64) for t in (x, g, weight))
    r = 1.0 / np.sqrt((x * x).mean(-1, keepdims=True) + eps)
    return x * r * w * (g / (1.0 + np.exp(-g)))


def causal_conv1d(x, weight, doc_ids=None, silu=True):
    """The layer's q/k/v prologue (sore/model/conv.py:6-23, then F.silu at gdn.py:210):
    ``z_t = sum_j weight[:, K-1-j] x_{t-j}`` over taps of t's document; ``x [B,T,C]``, ``weight [C,K]``,
    ``doc_ids [T]`` (None = one document per batch row). fp64."""
    x, w = np.asarray(x, np.float64), np.asarray(weight, np.float64)
    T, K = x.shape[1], w.shape[1]
    z = x * w[:, K - 1]
    for j in range(1, min(K, T)):
        term = x[:, : T - j] * w[:, K - 1 - j]
        if doc_ids is not None:
            same = np.asarray(doc_ids)[j:] == np.asarray(doc_ids)[: T - j]
            term = np.where(same[None, :, None], term, 0.0)
        z[:, j:] += term
    return z / (1.0 + np.exp(-z)) if silu else z
