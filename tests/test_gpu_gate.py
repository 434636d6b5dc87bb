"""GPU parity of the gate / beta activations (gdn.py:157-162 and 191-194) and of the op with
``use_gate_in_kernel`` / ``use_beta_sigmoid_in_kernel``.

Expected values: the oracle's ``gate_and_beta`` (fp64 restatement of ``_gate_and_beta``) and its analytic
derivatives; for the whole op, the same op fed the activations computed by torch, with torch autograd
through them. Tolerances: fp32 1e-4 x RMS; bf16 outputs 2e-2 beyond output rounding, gradients 3e-2.
"""
import numpy as np
import pytest
import torch

from helpers import assert_bf16_close, assert_rms_close, to_np
from inputs import make_inputs
from oracle.gdn_oracle import gate_and_beta

pytestmark = pytest.mark.gpu


def _raw(seed, T, HV, dtype):
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((2, T, HV)) * 4.0
    a[0, :3, 0] = [25.0, -40.0, 19.9]  # both sides of the softplus threshold, and deep underflow
    b = rng.standard_normal((2, T, HV)) * 3.0
    A_log = rng.standard_normal(HV) * 0.5
    dt_bias = rng.standard_normal(HV) * 0.5
    dev = lambda x, dt=torch.float32: torch.tensor(x, device="cuda").to(dt)  # noqa: E731
    return dev(a, dtype), dev(b, dtype), dev(A_log), dev(dt_bias)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("with_bias", [True, False])
def test_gate_and_beta_forward_backward(dtype, with_bias):
    from sorernn_b200.gated_delta_rule import gdn_beta_sigmoid, gdn_gate

    T, HV = 300, 6
    a, b, A_log, dt_bias = _raw(5, T, HV, dtype)
    a.requires_grad_(True)
    b.requires_grad_(True)
    A_log.requires_grad_(True)
    dt_bias.requires_grad_(with_bias)
    g = gdn_gate(a, A_log, dt_bias if with_bias else None)
    beta = gdn_beta_sigmoid(b)
    an, bn = to_np(a).astype(np.float64), to_np(b).astype(np.float64)
    Al, dtb = to_np(A_log).astype(np.float64), (to_np(dt_bias).astype(np.float64) if with_bias else np.zeros(HV))
    g_ref, beta_ref = gate_and_beta(an, bn, Al, dtb)
    assert g.dtype == torch.float32 and beta.dtype == torch.float32
    assert_rms_close(to_np(g), g_ref, 1e-4, "g")
    assert_rms_close(to_np(beta), beta_ref, 1e-4, "beta")

    rng = np.random.default_rng(6)
    dg = rng.standard_normal(g.shape)
    db = rng.standard_normal(beta.shape)
    (g * torch.tensor(dg, device="cuda", dtype=torch.float32)).sum().backward(retain_graph=True)
    (beta * torch.tensor(db, device="cuda", dtype=torch.float32)).sum().backward()
    x = an + dtb
    sig = np.where(x > 20, 1.0, 1.0 / (1.0 + np.exp(-x)))
    da_ref = dg * (-np.exp(Al)) * sig
    db_ref = db * beta_ref * (1.0 - beta_ref)
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    check = assert_rms_close if dtype == torch.float32 else assert_bf16_close
    check(to_np(a.grad), da_ref, tol, "da")
    check(to_np(b.grad), db_ref, tol, "db")
    assert_rms_close(to_np(A_log.grad), (dg * g_ref).sum(axis=(0, 1)), 1e-4, "dA_log")
    if with_bias:
        assert_rms_close(to_np(dt_bias.grad), da_ref.sum(axis=(0, 1)), 1e-4, "ddt_bias")
    else:
        assert dt_bias.grad is None


def test_op_with_in_kernel_gate_matches_precomputed_activations():
    """use_gate_in_kernel / use_beta_sigmoid_in_kernel == the op fed torch-computed g and beta."""
    from sorernn_b200 import chunk_gated_delta_rule

    B, T, H, HV, D = 1, 200, 2, 4, 128
    x = make_inputs(31, B, T, H, HV, D, D, normalized=False)
    q, k, v = (torch.tensor(x[n], device="cuda").bfloat16() for n in ("q", "k", "v"))
    do = torch.tensor(x["do"], device="cuda").bfloat16()
    rng = np.random.default_rng(32)
    a = torch.tensor(rng.standard_normal((B, T, HV)) - 2.0, device="cuda").bfloat16()
    bb = torch.tensor(rng.standard_normal((B, T, HV)), device="cuda").bfloat16()
    A_log = torch.tensor(rng.standard_normal(HV) * 0.3 - 1.0, device="cuda", dtype=torch.float32)
    dt_bias = torch.tensor(rng.standard_normal(HV) * 0.3, device="cuda", dtype=torch.float32)

    def leaves():
        return [t.clone().requires_grad_(True) for t in (a, bb, A_log, dt_bias)]

    a1, b1, A1, d1 = leaves()
    o1, _ = chunk_gated_delta_rule(q, k, v, a1, b1, use_qk_l2norm_in_kernel=True, use_gate_in_kernel=True,
                                   A_log=A1, dt_bias=d1, use_beta_sigmoid_in_kernel=True)
    (o1.float() * do.float()).sum().backward()

    a2, b2, A2, d2 = leaves()
    g2 = -A2.exp() * torch.nn.functional.softplus(a2.float() + d2)
    beta2 = b2.float().sigmoid()
    o2, _ = chunk_gated_delta_rule(q, k, v, g2, beta2, use_qk_l2norm_in_kernel=True)
    (o2.float() * do.float()).sum().backward()

    assert_bf16_close(to_np(o1), to_np(o2), 2e-2, "o")
    for name, t1, t2 in (("da", a1, a2), ("db", b1, b2), ("dA_log", A1, A2), ("ddt_bias", d1, d2)):
        assert_rms_close(to_np(t1.grad), to_np(t2.grad), 3e-2, name)
