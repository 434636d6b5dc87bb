"""Host-side checks of the Python boundary (no GPU needed): argument validation happens before any
library call, and CPU tensors are refused (no CPU fallback)."""
import pytest
import torch


def _x(B=1, T=8, H=2, HV=2, D=16):
    q = torch.randn(B, T, H, D)
    v = torch.randn(B, T, HV, D)
    return q, q.clone(), v, torch.randn(B, T, HV), torch.rand(B, T, HV)


def test_gate_in_kernel_requires_A_log():
    from sorernn_b200 import chunk_gated_delta_rule

    q, k, v, g, beta = _x()
    with pytest.raises(ValueError, match="A_log"):
        chunk_gated_delta_rule(q, k, v, g, beta, use_gate_in_kernel=True)


def test_unknown_keyword_is_rejected():
    from sorernn_b200 import chunk_gated_delta_rule

    q, k, v, g, beta = _x()
    with pytest.raises(TypeError, match="unexpected keyword"):
        chunk_gated_delta_rule(q, k, v, g, beta, use_gate_in_kernal=True)


def test_cpu_tensors_are_refused():
    from sorernn_b200 import chunk_gated_delta_rule, fused_recurrent_gated_delta_rule_step

    q, k, v, g, beta = _x()
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        chunk_gated_delta_rule(q, k, v, g, beta)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        chunk_gated_delta_rule(q, k, v, g, beta, use_gate_in_kernel=True, A_log=torch.zeros(2))
    state = torch.zeros(1, 2, 16, 16)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        fused_recurrent_gated_delta_rule_step(q[:, 0], k[:, 0], v[:, 0], g[:, 0], beta[:, 0], state)

