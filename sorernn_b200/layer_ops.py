"""The GDN layer's neighbouring steps as fused CUDA ops (the rows after the mixer itself):

* :func:`rms_norm_gated` — ``RMSNorm(o) * weight * silu(gate)`` in one pass, the drop-in for FLA's
  ``fla.modules.fused_norm_gate.rms_norm_gated`` as soreRNN calls it (sore/model/gdn.py:186:
  ``rms_norm_gated(o, gate, self.o_norm.weight, None, activation="swish", eps=self.o_norm.eps)``);
* :func:`causal_conv1d` — the short causal depthwise convolution + SiLU of the q/k/v prologue, the
  drop-in for FLA's ``fla.modules.conv.causal_conv1d`` (gdn.py:204-206) with per-document resets.

Each is a ``torch.library`` custom op with a registered autograd formula and a fake kernel, calling the
C ABI (include/gdn_b200.h); CUDA tensors only.
"""
from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor

from . import _lib
from .gated_delta_rule import _DT, _ptr, _stream


@torch.library.custom_op("sorernn_b200::rms_norm_gated_fwd", mutates_args=())
def _ng_fwd(x: Tensor, gate: Tensor, weight: Tensor, eps: float) -> Tensor:
    D = x.shape[-1]
    y = torch.empty_like(x)
    _lib.check(_lib.lib().gdn_rms_norm_gated_fwd(x.numel() // D, D, _ptr(x), _ptr(gate), _DT[x.dtype], _ptr(weight),
                                                 _DT[weight.dtype], eps, _ptr(y), _stream(x)), "gdn_rms_norm_gated_fwd")
    return y


@_ng_fwd.register_fake
def _(x, gate, weight, eps):
    return torch.empty_like(x)


@torch.library.custom_op("sorernn_b200::rms_norm_gated_bwd", mutates_args=())
def _ng_bwd(x: Tensor, gate: Tensor, weight: Tensor, eps: float, dy: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    D = x.shape[-1]
    dx, dg = torch.empty_like(x), torch.empty_like(gate)
    dw = torch.empty(D, dtype=torch.float32, device=x.device)
    _lib.check(_lib.lib().gdn_rms_norm_gated_bwd(x.numel() // D, D, _ptr(x), _ptr(gate), _DT[x.dtype], _ptr(weight),
                                                 _DT[weight.dtype], eps, _ptr(dy.to(x.dtype).contiguous()), _ptr(dx),
                                                 _ptr(dg), _ptr(dw), _stream(x)), "gdn_rms_norm_gated_bwd")
    return dx, dg, dw


@_ng_bwd.register_fake
def _(x, gate, weight, eps, dy):
    return torch.empty_like(x), torch.empty_like(gate), x.new_empty(x.shape[-1], dtype=torch.float32)


def _ng_setup(ctx, inputs, output):
    x, gate, weight, eps = inputs
    ctx.save_for_backward(x, gate, weight)
    ctx.eps = eps


def _ng_backward(ctx, dy):
    x, gate, weight = ctx.saved_tensors
    dx, dg, dw = _ng_bwd(x, gate, weight, ctx.eps, dy)
    return dx, dg, dw.to(weight.dtype), None


torch.library.register_autograd("sorernn_b200::rms_norm_gated_fwd", _ng_backward, setup_context=_ng_setup)


def rms_norm_gated(x: Tensor, g: Tensor, weight: Tensor, bias: Optional[Tensor] = None, activation: str = "swish",
                   residual: Optional[Tensor] = None, prenorm: bool = False, residual_in_fp32: bool = False,
                   eps: float = 1e-5) -> Tensor:
    """``x * rsqrt(mean(x^2, -1) + eps) * weight * silu(g)`` over the last dim, fp32 math, output in x's
    dtype (FLA signature; soreRNN passes bias=None, activation="swish"). The last dim must be a multiple
    of 32 and at most 1024; ``bias``, ``residual`` and ``prenorm`` are not supported."""
    if bias is not None or residual is not None or prenorm:
        raise NotImplementedError("rms_norm_gated: bias, residual and prenorm are not supported")
    if activation not in ("swish", "silu"):
        raise NotImplementedError(f"rms_norm_gated: activation {activation!r} (only swish/silu)")
    if not x.is_cuda:
        raise RuntimeError("sorernn_b200 runs on CUDA tensors only (no CPU fallback)")
    if g.shape != x.shape or weight.shape != (x.shape[-1],):
        raise ValueError(f"shapes: x {tuple(x.shape)}, g {tuple(g.shape)}, weight {tuple(weight.shape)}")
    return _ng_fwd(x.contiguous(), g.to(x.dtype).contiguous(), weight.contiguous(), float(eps))


@torch.library.custom_op("sorernn_b200::causal_conv1d_fwd", mutates_args=())
def _conv_fwd(x: Tensor, weight: Tensor, cu_seqlens: Optional[Tensor], silu: bool) -> Tensor:
    B, T, C = x.shape
    y = torch.empty_like(x)
    N = 0 if cu_seqlens is None else cu_seqlens.numel() - 1
    _lib.check(_lib.lib().gdn_causal_conv1d_fwd(B, T, C, weight.shape[1], _ptr(x), _DT[x.dtype], _ptr(weight),
                                                _DT[weight.dtype], _ptr(cu_seqlens), N, int(silu), _ptr(y),
                                                _stream(x)), "gdn_causal_conv1d_fwd")
    return y


@_conv_fwd.register_fake
def _(x, weight, cu_seqlens, silu):
    return torch.empty_like(x)


@torch.library.custom_op("sorernn_b200::causal_conv1d_bwd", mutates_args=())
def _conv_bwd(x: Tensor, weight: Tensor, cu_seqlens: Optional[Tensor], silu: bool, dy: Tensor) -> tuple[Tensor, Tensor]:
    B, T, C = x.shape
    dx = torch.empty_like(x)
    dw = torch.empty(weight.shape, dtype=torch.float32, device=x.device)
    N = 0 if cu_seqlens is None else cu_seqlens.numel() - 1
    _lib.check(_lib.lib().gdn_causal_conv1d_bwd(B, T, C, weight.shape[1], _ptr(x), _DT[x.dtype], _ptr(weight),
                                                _DT[weight.dtype], _ptr(cu_seqlens), N, int(silu),
                                                _ptr(dy.to(x.dtype).contiguous()), _ptr(dx), _ptr(dw), _stream(x)),
               "gdn_causal_conv1d_bwd")
    return dx, dw


@_conv_bwd.register_fake
def _(x, weight, cu_seqlens, silu, dy):
    return torch.empty_like(x), x.new_empty(weight.shape, dtype=torch.float32)


def _conv_setup(ctx, inputs, output):
    x, weight, cu_seqlens, silu = inputs
    ctx.save_for_backward(x, weight, cu_seqlens)
    ctx.silu = silu


def _conv_backward(ctx, dy):
    x, weight, cu_seqlens = ctx.saved_tensors
    dx, dw = _conv_bwd(x, weight, cu_seqlens, ctx.silu, dy)
    return dx, dw.to(weight.dtype), None, None


torch.library.register_autograd("sorernn_b200::causal_conv1d_fwd", _conv_backward, setup_context=_conv_setup)


def causal_conv1d(x: Tensor, weight: Tensor, bias: Optional[Tensor] = None, residual: Optional[Tensor] = None,
                  initial_state: Optional[Tensor] = None, output_final_state: bool = False,
                  activation: Optional[str] = None, backend: Optional[str] = None,
                  cu_seqlens: Optional[Tensor] = None, cu_seqlens_cpu: Optional[Tensor] = None, **kwargs):
    """Short causal depthwise convolution over ``x [B, T, C]`` with ``weight [C, K]`` (K <= 4), optional SiLU,
    the state reset at each document start (``cu_seqlens``, B == 1) — FLA's ``causal_conv1d`` signature as
    soreRNN calls it (gdn.py:204-206). Returns ``(y, None)``; bias, residual and conv states are not
    supported. ``cu_seqlens_cpu`` is accepted and not needed."""
    if bias is not None or residual is not None or initial_state is not None or output_final_state:
        raise NotImplementedError("causal_conv1d: bias, residual and conv states are not supported")
    if activation not in (None, "silu", "swish"):
        raise NotImplementedError(f"causal_conv1d: activation {activation!r}")
    if not x.is_cuda:
        raise RuntimeError("sorernn_b200 runs on CUDA tensors only (no CPU fallback)")
    if x.dim() != 3 or weight.dim() != 2 or weight.shape[0] != x.shape[2]:
        raise ValueError(f"x must be [B,T,C] and weight [C,K], got {tuple(x.shape)} and {tuple(weight.shape)}")
    if cu_seqlens is not None:
        if x.shape[0] != 1:
            raise ValueError(f"cu_seqlens requires B == 1, got B = {x.shape[0]}")
        cu_seqlens = cu_seqlens.to(device=x.device, dtype=torch.int64).contiguous()
    y = _conv_fwd(x.contiguous(), weight.contiguous(), cu_seqlens, activation is not None)
    return y, None
