"""Training on pieces: the chunked gated delta rule with every sequence cut into P pieces that run side by
side on one GPU.

The chunked kernels walk the chunks of one (sequence, value head) pair serially in one CTA, so a GPU that
holds few pairs leaves most of its 148 SMs idle: config 1 (B=8, T=4096, H=16) split by batch rows over 8 GPUs
gives each GPU 16 pairs. A piece of a sequence is an affine map on the state entering it,
``S_out = M S_in + C`` (the recurrence of gdn_ref.py:18-21 is linear in (S, v)), and the same holds for the
backward: the gradient reaching a piece's incoming state is ``M^T dS_end + R``, with ``R`` that gradient for
a zero end-state gradient. So, over the B*P pieces as independent sequences:

forward   one chunk-parallel prep pass over every piece's chunks and, from its records, the C and M state
          passes (``gdn_segment_maps_save``); the chain of the maps along each sequence (``gdn_piece_chain``)
          gives every piece its true incoming state, and the outputs pass runs every piece from it, writing the
          backward's per-chunk records (``gdn_segment_outputs_save``). Outputs and records are those of the
          unsplit forward.
backward  a reverse sweep that carries dS alone over every piece from a zero end-state gradient yields every
          ``R`` (``gdn_chunk_state_grad_saved``); the reverse chain of the transposed maps gives every piece's
          true end-state gradient; the full sweep from those writes the gradients.

Three state passes, a dS-only sweep and a full sweep of T/P tokens each replace one state pass and one sweep
of T tokens, so the split pays when B*HV*P pairs fill the SMs that B*HV pairs leave idle. Nothing here crosses
GPUs.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch
from torch import Tensor

from . import _lib
from .gated_delta_rule import DEFAULT_CKPT_EVERY, _check_inputs, _problem, _ptr, _stream
from .seqsplit import affine_inclusive_scan


# The two chains in torch (log-depth scans of batched products). The op runs them as one kernel each
# (gdn_piece_chain); these state the same algebra and check it on the CPU against the oracle.
def incoming_states(M: Tensor, C: Tensor, h0: Optional[Tensor]) -> tuple[Tensor, Tensor]:
    """Forward scan along the pieces. ``M [B, P, HV, dk, dk]`` and ``C [B, P, HV, dk, dv]`` are every piece's
    map (``C`` of piece 0 already started from ``h0``). Returns ``(S_in [B, P, HV, dk, dv], S_final [B, HV,
    dk, dv])``: the state entering each piece (``h0`` or zeros for piece 0) and the one leaving the last."""
    B, P = C.shape[:2]
    _, Ci = affine_inclusive_scan(M.transpose(0, 1), C.transpose(0, 1))  # [P, B, ...]
    first = torch.zeros_like(C[:, 0]) if h0 is None else h0.to(C.dtype).expand_as(C[:, 0])
    S_in = torch.cat([first.unsqueeze(0), Ci[:-1]]).transpose(0, 1)
    return S_in.contiguous(), Ci[P - 1].contiguous()


def end_state_grads(MT: Tensor, R: Tensor, dht: Optional[Tensor]) -> Tensor:
    """Reverse scan along the pieces. ``MT [B, P, HV, dk, dk]`` holds every piece's transposed map, ``R [B, P,
    HV, dk, dv]`` the gradient of each piece's incoming state for a zero end-state gradient, ``dht`` the
    gradient of the sequences' final states (None: zero). Returns the gradient of every piece's end state
    ``X [B, P, HV, dk, dv]``: ``X[:, P-1] = dht``, ``X[:, p] = MT[:, p+1] X[:, p+1] + R[:, p+1]``."""
    B, P = R.shape[:2]
    last = torch.zeros_like(R[:, 0]) if dht is None else dht.to(R.dtype).expand_as(R[:, 0])
    if P == 1:
        return last.unsqueeze(1).contiguous()
    # entry s = piece P-1-s for s = 0 .. P-2; dht enters through the first entry's constant term
    A = MT[:, 1:].flip(1).transpose(0, 1)
    Bc = R[:, 1:].flip(1).transpose(0, 1).clone()
    if dht is not None:
        Bc[0] = Bc[0] + torch.matmul(A[0], last)
    _, Cs = affine_inclusive_scan(A, Bc)  # Cs[s] = gradient entering piece P-1-s = X[:, P-2-s]
    X = torch.cat([Cs.flip(0), last.unsqueeze(0)])  # [P, B, ...] in piece order
    return X.transpose(0, 1).contiguous()


def _chain(B, P, HV, maps, terms, start, out, final, reverse, stream):
    """``gdn_piece_chain``: the forward chain of :func:`incoming_states` (reverse = 0) or the reverse chain of
    :func:`end_state_grads` (reverse = 1) in one launch (fp32 FMAs, one CTA per (sequence, head, 16 columns)) on
    ``stream``."""
    _lib.check(_lib.lib().gdn_piece_chain(B, P, HV, 128, 128, _ptr(maps), _ptr(terms), _ptr(start), _ptr(out),
                                          _ptr(final), reverse, stream), "gdn_piece_chain")


class _PiecesFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, g, beta, h0, scale, l2, P):
        B, T = q.shape[:2]
        Ts = T // P
        view = lambda x: x.reshape(B * P, Ts, *x.shape[2:])  # noqa: E731  (contiguous: a view)
        qs, ks, vs, gs, bs = (view(x) for x in (q, k, v, g, beta))
        HV, dk, dv = v.shape[2], q.shape[3], v.shape[3]
        p = _problem(qs, ks, vs, gs, bs, scale, None, Ts, l2, DEFAULT_CKPT_EVERY)
        L = _lib.lib()
        n_rec = L.gdn_segment_records_size(ctypes.byref(p))
        rec = torch.empty(max(n_rec, 1), dtype=torch.uint8, device=q.device)
        saved = torch.empty(max(L.gdn_chunk_saved_bytes(ctypes.byref(p)), 1), dtype=torch.uint8, device=q.device)
        init = None
        if h0 is not None:
            init = torch.zeros(B, P, HV, dk, dv, dtype=torch.float32, device=q.device)
            init[:, 0] = h0.float()
            init = init.view(B * P, HV, dk, dv)
        C = torch.empty(B * P, HV, dk, dv, dtype=torch.float32, device=q.device)
        M = torch.empty(B * P, HV, dk, dk, dtype=torch.float32, device=q.device) if P > 1 else None
        stream = _stream(q)
        _lib.check(L.gdn_segment_maps_save(ctypes.byref(p), _ptr(qs), _ptr(ks), _ptr(vs), _ptr(gs), _ptr(bs),
                                           _ptr(init), _ptr(C), _ptr(M), _ptr(saved), _ptr(rec), n_rec, stream),
                   "gdn_segment_maps_save")
        if P > 1:
            S_in = torch.empty(B * P, HV, dk, dv, dtype=torch.float32, device=q.device)
            final = torch.empty(B, HV, dk, dv, dtype=torch.float32, device=q.device)
            h0f = None if h0 is None else h0.float().contiguous()
            _chain(B, P, HV, M, C, h0f, S_in, final, 0, stream)
        else:
            S_in, final = init, C.view(B, HV, dk, dv)
        o = torch.empty_like(vs)
        _lib.check(L.gdn_segment_outputs_save(ctypes.byref(p), _ptr(qs), _ptr(ks), _ptr(vs), _ptr(gs), _ptr(bs),
                                              _ptr(S_in), _ptr(o), None, _ptr(saved), _ptr(rec), n_rec, stream),
                   "gdn_segment_outputs_save")
        del rec
        ctx.save_for_backward(q, k, v, g, beta, saved, M)
        ctx.args = (scale, l2, P, h0 is not None)
        ctx.set_materialize_grads(False)
        return o.view(B, T, HV, dv), final

    @staticmethod
    def backward(ctx, do, dht):
        q, k, v, g, beta, saved, M = ctx.saved_tensors
        scale, l2, P, has_h0 = ctx.args
        B, T = q.shape[:2]
        Ts = T // P
        HV, dk, dv = v.shape[2], q.shape[3], v.shape[3]
        view = lambda x: x.reshape(B * P, Ts, *x.shape[2:])  # noqa: E731
        qs, ks, vs, gs, bs = (view(x) for x in (q, k, v, g, beta))
        if do is None:
            do = torch.zeros_like(v)
        dos = view(do.contiguous())
        p = _problem(qs, ks, vs, gs, bs, scale, None, Ts, l2, DEFAULT_CKPT_EVERY)
        L = _lib.lib()
        ws_bytes = L.gdn_chunk_bwd_saved_workspace_size(ctypes.byref(p))
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
        dq, dk_, dv_ = torch.empty_like(qs), torch.empty_like(ks), torch.empty_like(vs)
        dg = torch.empty(gs.shape, dtype=torch.float32, device=q.device)
        db = torch.empty(bs.shape, dtype=torch.float32, device=q.device)
        dS0 = torch.empty(B * P, HV, dk, dv, dtype=torch.float32, device=q.device)
        stream = _stream(q)

        def sweep(dht_pieces):
            _lib.check(L.gdn_chunk_bwd_saved(ctypes.byref(p), _ptr(qs), _ptr(ks), _ptr(vs), _ptr(gs), _ptr(bs),
                                             _ptr(saved), _ptr(dos), _ptr(dht_pieces), _ptr(dq), _ptr(dk_),
                                             _ptr(dv_), _ptr(dg), _ptr(db), _ptr(dS0), _ptr(ws), ws_bytes, stream),
                       "gdn_chunk_bwd_saved")

        dht_ = None if dht is None else dht.float().contiguous()
        if P > 1:
            # R of every piece (dS0), for a zero end-state gradient: the sweep carrying dS alone
            _lib.check(L.gdn_chunk_state_grad_saved(ctypes.byref(p), _ptr(qs), _ptr(ks), _ptr(vs), _ptr(gs),
                                                    _ptr(bs), _ptr(saved), _ptr(dos), None, _ptr(dS0), _ptr(ws),
                                                    ws_bytes, stream), "gdn_chunk_state_grad_saved")
            X = torch.empty(B * P, HV, dk, dv, dtype=torch.float32, device=q.device)
            _chain(B, P, HV, M, dS0, dht_, X, None, 1, stream)
            sweep(X)
        else:
            sweep(dht_)
        dh0 = dS0.view(B, P, HV, dk, dv)[:, 0] if has_h0 else None
        shape = lambda x: x.view(B, T, *x.shape[2:])  # noqa: E731
        return (shape(dq), shape(dk_), shape(dv_), shape(dg).to(g.dtype), shape(db).to(beta.dtype), dh0,
                None, None, None)


def chunk_gated_delta_rule_pieces(q: Tensor, k: Tensor, v: Tensor, g: Tensor, beta: Tensor, pieces: int,
                                  scale: Optional[float] = None, initial_state: Optional[Tensor] = None,
                                  output_final_state: bool = False,
                                  use_qk_l2norm_in_kernel: bool = False) -> tuple[Tensor, Optional[Tensor]]:
    """``chunk_gated_delta_rule`` (same arguments and results, no ``cu_seqlens``) computed on ``pieces`` pieces
    of every sequence side by side, forward and backward. Needs the chunked kernels (bf16 q/k/v with dk = dv =
    128) and T a multiple of ``pieces``; T / pieces a multiple of 64 keeps every piece's chunks
    full. Results match the unsplit op within its bf16 tolerance (the pieces are joined in fp32)."""
    _check_inputs(q, k, v, g, beta, None)
    P = int(pieces)
    if P < 1 or q.shape[1] % P:
        raise ValueError(f"sequence length {q.shape[1]} is not a multiple of pieces = {P}")
    if not (q.dtype == torch.bfloat16 and q.shape[-1] == 128 and v.shape[-1] == 128):
        raise ValueError("chunk_gated_delta_rule_pieces needs the chunked kernels (bf16, dk = dv = 128)")
    scale = q.shape[-1] ** -0.5 if scale is None else float(scale)
    q, k, v, g, beta = (x.contiguous() for x in (q, k, v, g, beta))
    h0 = None if initial_state is None else initial_state.contiguous()
    o, final = _PiecesFn.apply(q, k, v, g, beta, h0, scale, bool(use_qk_l2norm_in_kernel), P)
    return o, (final if output_final_state else None)
