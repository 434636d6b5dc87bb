"""Seeded weights and inputs of one GatedDeltaNet layer, shared by the layer fixture script and the layer
tests (numpy PCG64 only, so both sides draw identical values).

Parameter names and shapes are those of the reference layer's ``state_dict`` (sore/model/gdn.py:110-135):
``q_proj/k_proj.weight [Hqk*D, d_model]``, ``v_proj/g_proj.weight [Hv*D, d_model]``,
``a_proj/b_proj.weight [Hv, d_model]``, ``conv_q/conv_k [Hqk*D, K]``, ``conv_v [Hv*D, K]``,
``A_log, dt_bias [Hv]``, ``o_norm.weight [D]``, ``o_proj.weight [d_model, Hv*D]``. The distributions follow
the reference's initialisation (linear layers ~ U(+-1/sqrt(fan_in)), convolutions ~ U(+-1/sqrt(K)),
A ~ U(1, 16), dt log-uniform in [1e-3, 1e-1] with dt_bias = softplus^-1(dt)); the RMSNorm weight is drawn
around 1 instead of left at 1, so that its gradient path is exercised.
"""
from __future__ import annotations

import numpy as np


def layer_weights(seed: int, d_model: int, qk_heads: int, v_heads: int, head_dim: int, K: int = 4) -> dict:
    rng = np.random.default_rng(seed)
    qk, vd = qk_heads * head_dim, v_heads * head_dim

    def lin(out_f, in_f):
        b = in_f ** -0.5
        return rng.uniform(-b, b, (out_f, in_f))

    w = {
        "q_proj.weight": lin(qk, d_model),
        "k_proj.weight": lin(qk, d_model),
        "v_proj.weight": lin(vd, d_model),
        "g_proj.weight": lin(vd, d_model),
        "a_proj.weight": lin(v_heads, d_model),
        "b_proj.weight": lin(v_heads, d_model),
        "conv_q": rng.uniform(-K ** -0.5, K ** -0.5, (qk, K)),
        "conv_k": rng.uniform(-K ** -0.5, K ** -0.5, (qk, K)),
        "conv_v": rng.uniform(-K ** -0.5, K ** -0.5, (vd, K)),
        "A_log": np.log(rng.uniform(1.0, 16.0, v_heads)),
    }
    log_dt = rng.random(v_heads) * (np.log(1e-1) - np.log(1e-3)) + np.log(1e-3)
    dt = np.exp(log_dt)
    w["dt_bias"] = dt + np.log(-np.expm1(-dt))
    w["o_norm.weight"] = 1.0 + 0.1 * rng.standard_normal(head_dim)
    w["o_proj.weight"] = lin(d_model, vd)
    return w


def layer_io(seed: int, T: int, d_model: int) -> tuple[np.ndarray, np.ndarray]:
    """``x [1, T, d_model] ~ N(0,1)`` and the output cotangent ``~ N(0,1)``."""
    rng = np.random.default_rng(seed)
    return rng.standard_normal((1, T, d_model)), rng.standard_normal((1, T, d_model))


def grad_sample_indices(seed: int, numel: int, n: int = 2048) -> np.ndarray:
    """The flat indices at which a parameter's gradient is stored (all of them for small tensors)."""
    if numel <= n:
        return np.arange(numel)
    return np.sort(np.random.default_rng(seed).choice(numel, n, replace=False))
