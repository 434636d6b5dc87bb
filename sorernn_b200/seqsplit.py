"""Sequence-split (context-parallel) prefill of the gated delta rule across ranks.

The reference has no context parallelism (soreRNN grows context by curriculum only,
configs/b0_8_pretrain.yaml:18-20); this is the long-context prefill path of the B200 build.

A segment of tokens is an affine map on the state entering it (gdn_ref.py:18-21 is linear in (S, v)):
``S_out = M S_in + C`` with ``M = prod_t exp(g_t)(I - beta_t k_t k_t^T)`` (later tokens on the left,
``[dk, dk]``) and ``C`` the segment's final state from a zero state (``[dk, dv]``). Rank r of P:

1. runs the forward of its segment from a zero state (rank 0: from ``h0``): local outputs and ``C_r``;
   ranks r > 0 also compute ``M_r`` (``gdn_segment_transition``);
2. exclusive scan over ranks: rank 0's outgoing state is ``C_0`` (or ``M_0 h0 + C_0``); rank r receives
   ``S_in`` from rank r-1 over NCCL (NVLink), forms ``S_out = M_r S_in + C_r`` and sends it to rank r+1;
3. ranks r > 0 add the incoming state's contribution to their outputs (``gdn_segment_apply_state``:
   the recurrence with v = 0 from ``S_in``), and the last rank's ``S_out`` is the sequence's final state.

Only step 2 crosses GPUs: one ``[N, HV, dk, dv]`` fp32 state per boundary (2 MiB at HV=16, d=128),
received into this GPU's memory by NCCL before any kernel reads it.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch
import torch.distributed as dist
from torch import Tensor

from . import _lib
from .gated_delta_rule import _DT, _ptr, _stream, chunk_gated_delta_rule


def _problem(q_like: Tensor, v_shape, g: Tensor, beta: Tensor, scale: float, l2norm: bool) -> _lib.Problem:
    B, T, H, DK = q_like.shape
    HV, DV = v_shape[2], v_shape[3]
    return _lib.Problem(B=B, T=T, H=H, HV=HV, DK=DK, DV=DV, N=B, cu_seqlens=None, max_seqlen=T, scale=scale,
                        act_dtype=_DT[q_like.dtype], g_dtype=_DT[g.dtype], beta_dtype=_DT[beta.dtype],
                        use_qk_l2norm=int(l2norm), ckpt_every=4)


def _ws(p: _lib.Problem, device) -> tuple[Tensor, int]:
    n = _lib.lib().gdn_segment_workspace_size(ctypes.byref(p))
    return torch.empty(max(n, 1), dtype=torch.uint8, device=device), n


def segment_transition(k: Tensor, g: Tensor, beta: Tensor, use_qk_l2norm: bool = False,
                       num_v_heads: Optional[int] = None) -> Tensor:
    """``M [B, HV, dk, dk]`` fp32 for each batch row (one segment per row)."""
    k, g, beta = k.contiguous(), g.contiguous(), beta.contiguous()
    B, T, H, DK = k.shape
    HV = g.shape[2] if num_v_heads is None else num_v_heads
    p = _problem(k, (B, T, HV, DK), g, beta, 1.0, use_qk_l2norm)
    M = torch.empty(B, HV, DK, DK, dtype=torch.float32, device=k.device)
    ws, n = _ws(p, k.device)
    _lib.check(_lib.lib().gdn_segment_transition(ctypes.byref(p), _ptr(k), _ptr(g), _ptr(beta), _ptr(M), _ptr(ws), n,
                                                 _stream(k)), "gdn_segment_transition")
    return M


def combine(M: Tensor, C: Tensor, S_in: Tensor) -> Tensor:
    """``S_out = M S_in + C`` (fp32, batched over [N, HV])."""
    return torch.matmul(M, S_in.to(M.dtype)) + C


def apply_incoming_state(q: Tensor, k: Tensor, g: Tensor, beta: Tensor, S_in: Tensor, o: Tensor, scale: float,
                         use_qk_l2norm: bool = False, final_state: Optional[Tensor] = None) -> None:
    """In place: ``o += scale (M_{<=t} S_in)^T q_t`` and ``final_state += M S_in`` (if given)."""
    q, k, g, beta = (x.contiguous() for x in (q, k, g, beta))
    assert o.is_contiguous()
    p = _problem(q, o.shape, g, beta, scale, use_qk_l2norm)
    ws, n = _ws(p, q.device)
    S_in = S_in.float().contiguous()
    _lib.check(_lib.lib().gdn_segment_apply_state(ctypes.byref(p), _ptr(q), _ptr(k), _ptr(g), _ptr(beta), _ptr(S_in),
                                                  _ptr(o), _ptr(final_state), _ptr(ws), n, _stream(q)),
               "gdn_segment_apply_state")


def exchange_boundary_states(C: Tensor, M: Optional[Tensor], group=None) -> tuple[Optional[Tensor], Tensor]:
    """Step 2, the only cross-rank step: the exclusive scan of segment maps along the rank chain.

    Rank r receives ``S_in`` (the state entering its segment) from rank r-1, forms ``S_out = M S_in + C``
    and sends it to rank r+1; rank 0's ``S_out`` is ``C`` (its forward already started from ``h0``).
    Returns ``(S_in, S_out)``; ``S_in`` is None on rank 0. ``M`` is read on ranks r > 0 only.
    Every rank issues its receive before its send, so the chain completes in rank order.
    """
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    glob = (lambda r: dist.get_global_rank(group, r)) if group is not None else (lambda r: r)
    S_in = None
    if rank > 0:
        S_in = torch.empty_like(C)
        dist.recv(S_in, src=glob(rank - 1), group=group)
        S_out = combine(M, C, S_in)
    else:
        S_out = C
    if rank < world - 1:
        dist.send(S_out.contiguous(), dst=glob(rank + 1), group=group)
    return S_in, S_out


def sequence_split_prefill(q: Tensor, k: Tensor, v: Tensor, g: Tensor, beta: Tensor, scale: Optional[float] = None,
                           use_qk_l2norm_in_kernel: bool = False, group=None,
                           initial_state: Optional[Tensor] = None) -> tuple[Tensor, Optional[Tensor]]:
    """Forward of this rank's segment of a sequence split across the ranks of ``group`` (rank order =
    token order). Every rank passes its own contiguous slice ``[B, T_r, ...]``. Returns
    ``(o_r, final_state)``; ``final_state`` (the whole sequence's) is returned on the last rank only.
    ``initial_state`` is read on rank 0 only.
    """
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    scale = q.shape[-1] ** -0.5 if scale is None else float(scale)
    h0 = initial_state if rank == 0 else None
    o, C = chunk_gated_delta_rule(q, k, v, g, beta, scale=scale, initial_state=h0, output_final_state=True,
                                  use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel)
    if world == 1:
        return o, C
    M = segment_transition(k, g, beta, use_qk_l2norm_in_kernel, v.shape[2]) if rank > 0 else None
    S_in, S_out = exchange_boundary_states(C, M, group)
    if rank > 0:
        apply_incoming_state(q, k, g, beta, S_in, o, scale, use_qk_l2norm_in_kernel)
    return o, (S_out if rank == world - 1 else None)
