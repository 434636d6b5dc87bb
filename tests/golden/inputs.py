"""Seeded input generator shared by the golden-fixture script and the tests (numpy PCG64 only)."""
from __future__ import annotations

import numpy as np


def make_inputs(seed, B, T, H, HV, dk, dv, normalized=True, g_mode="logsigmoid16"):
    """Config-0 value distributions: q,k ~ N(0,1) (L2-normalised if ``normalized``); v ~ N(0,1);
    beta = sigmoid(N(0,1)); g = logsigmoid(N(0,1)) / 16; upstream gradient ~ N(0,1)."""
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, T, H, dk))
    k = rng.standard_normal((B, T, H, dk))
    if normalized:
        q /= np.linalg.norm(q, axis=-1, keepdims=True)
        k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((B, T, HV, dv))
    x = rng.standard_normal((B, T, HV))
    if g_mode == "logsigmoid16":
        g = -np.logaddexp(0.0, -x) / 16.0
    else:  # "uniform": the reference test's g = -U(0,1)
        g = -rng.random((B, T, HV))
    beta = 1.0 / (1.0 + np.exp(-rng.standard_normal((B, T, HV))))
    do = rng.standard_normal((B, T, HV, dv))
    return dict(q=q, k=k, v=v, g=g, beta=beta, do=do)


def make_state_inputs(seed, N, HV, dk, dv):
    """Initial state ~ 0.1 * N(0,1) and final-state cotangent ~ N(0,1), both ``[N,HV,dk,dv]``."""
    h0 = np.random.default_rng(seed + 1000).standard_normal((N, HV, dk, dv)) * 0.1
    dht = np.random.default_rng(seed + 2000).standard_normal((N, HV, dk, dv))
    return h0, dht
