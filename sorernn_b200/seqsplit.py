"""Sequence-split (context-parallel) prefill of the gated delta rule across ranks.

The reference has no context parallelism (soreRNN grows context by curriculum only,
configs/b0_8_pretrain.yaml:18-20); this is the long-context prefill path of the B200 build.

A segment of tokens is an affine map on the state entering it (gdn_ref.py:18-21 is linear in (S, v)):
``S_out = M S_in + C`` with ``M = prod_t exp(g_t)(I - beta_t k_t k_t^T)`` (later tokens on the left,
``[dk, dk]``) and ``C`` the segment's final state from a zero state (``[dk, dv]``). Rank r of P:

1. runs the forward of its segment from a zero state (rank 0: from ``h0``): local outputs and ``C_r``;
   ranks r > 0 also compute ``M_r`` (``gdn_segment_transition``);
2. exclusive scan over ranks: one NCCL all_gather (NVLink) of every rank's map ``(M_r, C_r)``; rank r
   composes the maps of ranks 0 .. r-1 locally into ``S_in`` (rank 0's ``C_0`` already includes ``h0``);
3. ranks r > 0 add the incoming state's contribution to their outputs (``gdn_segment_apply_state``:
   the recurrence with v = 0 from ``S_in``), and the last rank's ``S_out`` is the sequence's final state.

On the chunked kernels (bf16, d = 128) steps 1 and 3 share one chunk-parallel prep pass: ``gdn_segment_maps``
writes its records and runs the C and M state passes over them, and ``gdn_segment_outputs`` reruns the state
pass from the true incoming state with outputs, in place of the zero-state outputs plus a correction.

Only step 2 crosses GPUs: one ``[N, HV, dk, dk]`` map and one ``[N, HV, dk, dv]`` state per rank (2 MiB at
HV=16, d=128), gathered into this GPU's memory by NCCL before any kernel reads them.
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


def affine_inclusive_scan(M: Tensor, C: Tensor) -> tuple[Tensor, Tensor]:
    """Inclusive scan of segment maps along dim 0: entry s becomes ``(M_s, C_s) o ... o (M_0, C_0)`` with
    ``(M2, C2) o (M1, C1) = (M2 M1, M2 C1 + C2)`` (apply map 1, then map 2). Hillis-Steele: ceil(log2 P)
    rounds, each two batched products over all entries at once, instead of P - 1 dependent steps.
    The C part of an entry never reads M_0, so M_0 may be a placeholder when only states are wanted."""
    P = M.shape[0]
    d = 1
    while d < P:
        C = torch.cat([C[:d], torch.matmul(M[d:], C[:-d]) + C[d:]])
        M = torch.cat([M[:d], torch.matmul(M[d:], M[:-d])])
        d *= 2
    return M, C


def exchange_boundary_states(C: Tensor, M: Optional[Tensor], group=None) -> tuple[Optional[Tensor], Tensor]:
    """Step 2, the only cross-rank step: the exclusive scan of segment maps over the ranks.

    One ``all_gather`` brings every rank's map ``(M_r, C_r)`` (2 MiB per rank at HV = 16, d = 128) into
    this GPU's memory; each rank then composes the maps of the ranks before it locally
    (``affine_inclusive_scan``, log-depth batched products). There is no dependent chain of transfers:
    every rank takes the same single collective. Rank 0's ``M`` is not needed (it starts the sequence) and
    goes as zeros. Returns ``(S_in, S_out)``: the state entering and leaving this rank's segment; ``S_in``
    is None on rank 0, whose ``S_out`` is ``C``.
    """
    rank = dist.get_rank(group)
    world = dist.get_world_size(group)
    dk = C.shape[-2]
    if M is None:
        M = torch.zeros(*C.shape[:-2], dk, dk, dtype=C.dtype, device=C.device)
    flat = torch.cat([M.reshape(-1), C.to(M.dtype).reshape(-1)])
    gathered = torch.empty(world * flat.numel(), dtype=flat.dtype, device=flat.device)
    dist.all_gather_into_tensor(gathered, flat, group=group)
    parts = gathered.view(world, -1)
    Ms = parts[:, :M.numel()].reshape(world, *M.shape)
    Cs = parts[:, M.numel():].reshape(world, *C.shape)
    if rank == 0:
        return None, C
    _, Cin = affine_inclusive_scan(Ms[:rank + 1], Cs[:rank + 1])
    return Cin[rank - 1].to(C.dtype), Cin[rank].to(C.dtype)


class _Records:
    """Prep records of one sequence-split problem, kept between ``gdn_segment_maps`` and
    ``gdn_segment_outputs`` (chunked kernels only)."""

    def __init__(self, q, v, g, beta, scale, l2):
        self.p = _problem(q, v.shape, g, beta, scale, l2)
        n = _lib.lib().gdn_segment_records_size(ctypes.byref(self.p))
        self.buf = torch.empty(max(n, 1), dtype=torch.uint8, device=q.device)
        self.n = n

    def maps(self, q, k, v, g, beta, h0, want_m):
        B, HV, dk, dv = q.shape[0], v.shape[2], q.shape[3], v.shape[3]
        C = torch.empty(B, HV, dk, dv, dtype=torch.float32, device=q.device)
        M = torch.empty(B, HV, dk, dk, dtype=torch.float32, device=q.device) if want_m else None
        h0 = None if h0 is None else h0.float().contiguous()
        _lib.check(_lib.lib().gdn_segment_maps(ctypes.byref(self.p), _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta),
                                               _ptr(h0), _ptr(C), _ptr(M), _ptr(self.buf), self.n, _stream(q)),
                   "gdn_segment_maps")
        return C, M

    def outputs(self, q, k, v, g, beta, incoming):
        o = torch.empty_like(v)
        inc = None if incoming is None else incoming.float().contiguous()
        _lib.check(_lib.lib().gdn_segment_outputs(ctypes.byref(self.p), _ptr(q), _ptr(k), _ptr(v), _ptr(g),
                                                  _ptr(beta), _ptr(inc), _ptr(o), None, _ptr(self.buf), self.n,
                                                  _stream(q)), "gdn_segment_outputs")
        return o


def _chunk_path(q, v) -> bool:
    return q.dtype == torch.bfloat16 and q.shape[-1] == 128 and v.shape[-1] == 128


def _local_split(q, k, v, g, beta, scale, l2, P, h0):
    """Forward of one rank's sequence cut into P sub-segments run side by side as a batch of P (the
    tensors are [1, T, ...] and contiguous, so the cut is a view). Sub-segment 0 starts from h0, the
    others from zero. Returns the per-piece views, ``o``, the incoming state of every sub-segment that its
    outputs still lack (zero for sub-segment 0), the prefix maps ``Mpre[s] = M_{s-1} ... M_0`` (identity
    for s = 0) and the rank's map ``(M, C)`` (C = the outgoing state for a zero rank input)."""
    T = q.shape[1]
    Ts = T // P
    seg = lambda x: x.view(P, Ts, *x.shape[2:])  # noqa: E731
    qs, ks, vs, gs, bs = (seg(x) for x in (q, k, v, g, beta))
    HV, dk, dv = v.shape[2], q.shape[3], v.shape[3]
    init = None
    if h0 is not None:
        init = torch.zeros(P, HV, dk, dv, dtype=torch.float32, device=q.device)
        init[0] = h0[0].float()
    o, C = chunk_gated_delta_rule(qs, ks, vs, gs, bs, scale=scale, initial_state=init, output_final_state=True,
                                  use_qk_l2norm_in_kernel=l2)
    M = segment_transition(ks, gs, bs, l2, HV)  # [P, HV, dk, dk]
    # prefix of the piece maps (log-depth batched products): piece s's incoming state from a zero rank input,
    # and the map from the rank's input to piece s's input
    Mi, Ci = affine_inclusive_scan(M, C)
    S_loc = torch.cat([torch.zeros_like(C[:1]), Ci[:-1]])
    eye = torch.eye(dk, dtype=M.dtype, device=q.device).expand(1, HV, dk, dk)
    Mpre = torch.cat([eye, Mi[:-1]])
    M_rank, C_rank = Mi[P - 1], Ci[P - 1]
    return qs, ks, gs, bs, o, S_loc, Mpre, M_rank.unsqueeze(0), C_rank.unsqueeze(0)


def segmented_prefill(q: Tensor, k: Tensor, v: Tensor, g: Tensor, beta: Tensor, scale: Optional[float] = None,
                      use_qk_l2norm_in_kernel: bool = False, initial_state: Optional[Tensor] = None,
                      local_segments: int = 8, group=None) -> tuple[Tensor, Optional[Tensor]]:
    """Forward of a long sequence ``[1, T, ...]`` cut into ``local_segments`` pieces per rank that run side by
    side (a batch of pieces fills the SMs when there are few heads), joined by the same affine maps as the
    cross-rank split. With a process group of P ranks, every rank passes its contiguous slice (rank order =
    token order) and the boundary states cross ranks over NCCL; without one, the whole sequence is local.
    Returns ``(o, final_state)``; ``final_state`` on the last rank only. ``initial_state`` is read on rank
    0 only. Each rank's slice length must be a multiple of ``local_segments``."""
    if q.shape[0] != 1:
        raise ValueError("segmented_prefill takes one sequence ([1, T, ...])")
    dist_on = group is not None or (dist.is_available() and dist.is_initialized())
    rank = dist.get_rank(group) if dist_on else 0
    world = dist.get_world_size(group) if dist_on else 1
    scale = q.shape[-1] ** -0.5 if scale is None else float(scale)
    P = int(local_segments)
    if P < 1 or q.shape[1] % P:
        raise ValueError(f"slice length {q.shape[1]} is not a multiple of local_segments = {P}")
    q, k, v, g, beta = (x.contiguous() for x in (q, k, v, g, beta))
    h0 = initial_state if rank == 0 else None
    if _chunk_path(q, v):
        return _segmented_prefill_chunked(q, k, v, g, beta, scale, use_qk_l2norm_in_kernel, P, h0, rank, world,
                                          group)
    qs, ks, gs, bs, o, S_loc, Mpre, M_r, C_r = _local_split(q, k, v, g, beta, scale, use_qk_l2norm_in_kernel,
                                                           P, h0)
    if world > 1:
        S_in, S_out = exchange_boundary_states(C_r, M_r if rank > 0 else None, group)
    else:
        S_in, S_out = None, C_r
    # every sub-segment's incoming state that its outputs still lack: the local part and the rank's input
    S_tot = S_loc if S_in is None else S_loc + torch.matmul(Mpre, S_in.expand(P, -1, -1, -1))
    if P > 1 or S_in is not None:
        apply_incoming_state(qs, ks, gs, bs, S_tot, o, scale, use_qk_l2norm_in_kernel)
    o = o.view(1, q.shape[1], *o.shape[2:])
    return o, (S_out if rank == world - 1 else None)


def piece_chain(n_seq: int, pieces: int, HV: int, maps: Optional[Tensor], terms: Tensor, start: Optional[Tensor],
                out: Optional[Tensor], final: Optional[Tensor], mode: int) -> None:
    """``gdn_piece_chain`` on the current stream: the chain of affine maps along ``pieces`` consecutive pieces
    of each of ``n_seq`` sequences (fp32, one launch). mode 0: ``out[p]`` = the state entering piece p (``start``
    for piece 0; ``terms[p]`` = piece p's final state from its own start), ``final`` = the state leaving the last
    piece; mode 1: the reverse chain of the transposed maps (end-state gradients); mode 2: with ``terms`` = the
    maps, ``final`` = the composite map M_{P-1} ... M_0."""
    _lib.check(_lib.lib().gdn_piece_chain(n_seq, pieces, HV, 128, 128, _ptr(maps), _ptr(terms), _ptr(start),
                                          _ptr(out), _ptr(final), mode, _stream(terms)), "gdn_piece_chain")


def _gather(x: Tensor, world: int, group) -> Tensor:
    """all_gather of a contiguous tensor into ``[world, *x.shape]`` (one NCCL collective)."""
    out = torch.empty(world * x.numel(), dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(out, x.reshape(-1), group=group)
    return out.view(world, *x.shape)


def _segmented_prefill_chunked(q, k, v, g, beta, scale, l2, P, h0, rank, world, group):
    """segmented_prefill on the chunked kernels: one prep pass for all pieces, then three state passes over
    its records: each piece's C (from zero; piece 0 of rank 0 from h0) and M, then each piece's outputs from
    its true incoming state. The maps are joined by chain kernels (gdn_piece_chain), across ranks after one
    all_gather of every rank's composite map (M_r, C_r)."""
    T = q.shape[1]
    Ts = T // P
    seg = lambda x: x.view(P, Ts, *x.shape[2:])  # noqa: E731
    qs, ks, vs, gs, bs = (seg(x) for x in (q, k, v, g, beta))
    HV, dk, dv = v.shape[2], q.shape[3], v.shape[3]
    f32 = dict(dtype=torch.float32, device=q.device)
    init = None
    if h0 is not None:
        init = torch.zeros(P, HV, dk, dv, **f32)
        init[0] = h0[0].float()
    rec = _Records(qs, vs, gs, bs, scale, l2)
    need_m = P > 1 or (world > 1 and rank > 0)
    C, M = rec.maps(qs, ks, vs, gs, bs, init, need_m)
    inc = torch.empty(P, HV, dk, dv, **f32)  # every piece's true incoming state
    final = torch.empty(1, HV, dk, dv, **f32)
    if rank == 0:  # the pieces' incoming states from h0; final: the state leaving this rank (C_r)
        h0f = None if h0 is None else h0.float().contiguous()
        piece_chain(1, P, HV, M, C, h0f, inc, final, 0)
    else:  # this rank's composite map and its final state from a zero input, for the exchange
        piece_chain(1, P, HV, M, C, None, inc, final, 0)
    if world == 1:
        return rec.outputs(qs, ks, vs, gs, bs, inc).view(1, T, HV, dv), final
    M_r = torch.zeros(1, HV, dk, dk, **f32)  # rank 0's map is never read (it starts the sequence)
    if rank > 0:
        piece_chain(1, P, HV, M, M, None, None, M_r, 2)
    Ms, Cs = _gather(M_r, world, group), _gather(final, world, group)
    # the state entering every rank: the chain of the ranks' maps (rank 0's C_r already holds h0)
    S_ranks = torch.empty(world, HV, dk, dv, **f32)
    S_out = torch.empty(1, HV, dk, dv, **f32)
    piece_chain(1, world, HV, Ms.view(world, HV, dk, dk), Cs.view(world, HV, dk, dv), None, S_ranks, S_out, 0)
    if rank > 0:  # piece 0 leaves with M_0 S_in + C_0; the pieces' chain from S_in
        S_in = S_ranks[rank:rank + 1]
        C[0] = torch.baddbmm(C[0], M[0], S_in[0])
        piece_chain(1, P, HV, M, C, S_in, inc, None, 0)
    o = rec.outputs(qs, ks, vs, gs, bs, inc)
    return o.view(1, T, *o.shape[2:]), (S_out if rank == world - 1 else None)


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
    if rank > 0 and _chunk_path(q, v):  # one prep pass; C and M, then the outputs from the incoming state
        q, k, v, g, beta = (x.contiguous() for x in (q, k, v, g, beta))
        rec = _Records(q, v, g, beta, scale, use_qk_l2norm_in_kernel)
        C, M = rec.maps(q, k, v, g, beta, None, True)
        S_in, S_out = exchange_boundary_states(C, M, group)
        o = rec.outputs(q, k, v, g, beta, S_in)
        return o, (S_out if rank == world - 1 else None)
    o, C = chunk_gated_delta_rule(q, k, v, g, beta, scale=scale, initial_state=h0, output_final_state=True,
                                  use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel)
    if world == 1:
        return o, C
    M = segment_transition(k, g, beta, use_qk_l2norm_in_kernel, v.shape[2]) if rank > 0 else None
    S_in, S_out = exchange_boundary_states(C, M, group)
    if rank > 0:
        apply_incoming_state(q, k, g, beta, S_in, o, scale, use_qk_l2norm_in_kernel)
    return o, (S_out if rank == world - 1 else None)
