"""The GatedDeltaNet token-mixer layer on this package's CUDA ops: a drop-in for soreRNN's
``sore.model.gdn.GatedDeltaNet`` (sore/model/gdn.py:92-206) at the layer boundary.

``o_proj(RMSNorm(o) * silu(g_proj(x)))`` with ``o`` the gated delta rule over the q/k/v projections after
a short causal convolution + SiLU. The parameters carry the reference layer's names and shapes, so its
``state_dict`` loads unchanged (and back). Every step between the projections is one of this package's
kernels: the convolution (``layer_ops.causal_conv1d``, per-document resets from ``cu_seqlens``), the gate
and beta activations (with ``kernel_gate``: ``-exp(A_log) softplus(a + dt_bias)`` and ``sigmoid(b)`` as
fused kernels with their backward), the gated delta rule with the in-kernel q/k L2 norm and native
grouped value heads (``chunk_gated_delta_rule``), and, with ``fused_norm_gate``, RMSNorm(o)·silu(gate) in one
kernel (``layer_ops.rms_norm_gated``). The projections are plain ``nn.Linear`` (library GEMMs).
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F
from torch import Tensor, nn

from .gated_delta_rule import chunk_gated_delta_rule
from .layer_ops import causal_conv1d, rms_norm_gated


class _RMSNormWeight(nn.Module):
    """The output norm's weight (state_dict key ``o_norm.weight``) and its eps; unfused path in fp32."""

    def __init__(self, dim: int, eps: float) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x: Tensor) -> Tensor:
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * self.weight.float()).to(x.dtype)


class GatedDeltaNet(nn.Module):
    """``GatedDeltaNet(d_model, qk_heads, v_heads, head_dim=128, conv_kernel=4, norm_eps=1e-6,
    kernel_gate=True, fused_norm_gate=True)``; ``forward(x [B,T,d_model], cu_seqlens=None,
    cu_seqlens_cpu=None)``: with ``cu_seqlens`` (int64 ``[S+1]``, B == 1) the convolution and the recurrent
    state restart at every document; without it every batch row is a document. ``cu_seqlens_cpu`` (the same
    values on the host) only sizes buffers; nothing synchronises the host."""

    def __init__(self, d_model: int, qk_heads: int, v_heads: int, head_dim: int = 128, conv_kernel: int = 4,
                 norm_eps: float = 1e-6, kernel_gate: bool = True, fused_norm_gate: bool = True) -> None:
        super().__init__()
        if v_heads % qk_heads:
            raise ValueError(f"v_heads = {v_heads} must be a multiple of qk_heads = {qk_heads}")
        self.qk_heads, self.v_heads, self.head_dim = qk_heads, v_heads, head_dim
        self.kernel_gate, self.fused_norm_gate = kernel_gate, fused_norm_gate
        qk, vd = qk_heads * head_dim, v_heads * head_dim
        self.q_proj = nn.Linear(d_model, qk, bias=False)
        self.k_proj = nn.Linear(d_model, qk, bias=False)
        self.v_proj = nn.Linear(d_model, vd, bias=False)
        self.g_proj = nn.Linear(d_model, vd, bias=False)
        self.a_proj = nn.Linear(d_model, v_heads, bias=False)
        self.b_proj = nn.Linear(d_model, v_heads, bias=False)
        bound = conv_kernel ** -0.5
        self.conv_q = nn.Parameter(torch.empty(qk, conv_kernel).uniform_(-bound, bound))
        self.conv_k = nn.Parameter(torch.empty(qk, conv_kernel).uniform_(-bound, bound))
        self.conv_v = nn.Parameter(torch.empty(vd, conv_kernel).uniform_(-bound, bound))
        self.A_log = nn.Parameter(torch.empty(v_heads).uniform_(1, 16).log())
        log_dt = torch.rand(v_heads) * (math.log(1e-1) - math.log(1e-3)) + math.log(1e-3)
        dt = log_dt.exp()
        self.dt_bias = nn.Parameter(dt + torch.log(-torch.expm1(-dt)))
        self.o_norm = _RMSNormWeight(head_dim, norm_eps)
        self.o_proj = nn.Linear(vd, d_model, bias=False)

    def forward(self, x: Tensor, cu_seqlens: Optional[Tensor] = None,
                cu_seqlens_cpu: Optional[Tensor] = None) -> Tensor:
        b, t, _ = x.shape

        def conv(h: Tensor, w: Tensor) -> Tensor:
            return causal_conv1d(h, w, activation="silu", cu_seqlens=cu_seqlens, cu_seqlens_cpu=cu_seqlens_cpu)[0]

        q = conv(self.q_proj(x), self.conv_q).view(b, t, self.qk_heads, self.head_dim)
        k = conv(self.k_proj(x), self.conv_k).view(b, t, self.qk_heads, self.head_dim)
        v = conv(self.v_proj(x), self.conv_v).view(b, t, self.v_heads, self.head_dim)
        if self.kernel_gate:  # raw a/b projections; the activations run as fused kernels
            gate_kw = dict(use_gate_in_kernel=True, A_log=self.A_log, dt_bias=self.dt_bias,
                           use_beta_sigmoid_in_kernel=True)
            g, beta = self.a_proj(x), self.b_proj(x)
        else:
            gate_kw = {}
            g = -self.A_log.float().exp() * F.softplus(self.a_proj(x).float() + self.dt_bias.float())
            beta = self.b_proj(x).sigmoid()
        o, _ = chunk_gated_delta_rule(q, k, v, g, beta, scale=self.head_dim ** -0.5, cu_seqlens=cu_seqlens,
                                      cu_seqlens_cpu=cu_seqlens_cpu, use_qk_l2norm_in_kernel=True, **gate_kw)
        gate = self.g_proj(x).view(b, t, self.v_heads, self.head_dim)
        if self.fused_norm_gate:
            o = rms_norm_gated(o, gate, self.o_norm.weight, None, activation="swish", eps=self.o_norm.eps)
        else:
            o = self.o_norm(o) * F.silu(gate)
        return self.o_proj(o.flatten(-2))
