"""PyTorch-facing API: the drop-in for ``fla.ops.gated_delta_rule.chunk_gated_delta_rule``.

soreRNN calls (sore/model/gdn.py:166-169)::

    o, _ = chunk_gated_delta_rule(q, k, v, g, beta, scale=scale, cu_seqlens=cu_seqlens,
                                  cu_seqlens_cpu=cu_seqlens_cpu, use_qk_l2norm_in_kernel=True)

:func:`chunk_gated_delta_rule` here takes the same arguments (FLA 0.5.x signature,
fla/ops/gated_delta_rule/chunk.py:365-380, minus ``cp_context``/``transpose_state_layout``) and returns
``(o, final_state or None)``. It is built from two ``torch.library`` custom ops (``sorernn_b200::gdn_fwd``,
``sorernn_b200::gdn_bwd``) with a registered autograd formula and fake (meta) kernels, so
``torch.compile`` treats the mixer as one opaque op and activation checkpointing sees it. Each op is a
thin ctypes call into the C ABI (include/gdn_b200.h); there is no Triton and no CPU fallback: on a
CPU tensor, or without the built library, the call raises.

:func:`fused_recurrent_gated_delta_rule_step` is the single-token decode step on a resident fp32 state.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch
from torch import Tensor

from . import _lib

_DT = {torch.bfloat16: _lib.BF16, torch.float16: _lib.FP16, torch.float32: _lib.FP32}
# Backward modes of the chunked kernels, chosen by ``ckpt_every``:
#   SAVE_RECORDS (0): the forward saves every chunk's backward record (88 KB per 64-token chunk and value head:
#     the chunk-start state and the chunk's operand tiles), the backward runs the reverse sweep alone;
#   k >= 1: the forward keeps one fp32 state every k chunks (64 KB each), the backward rebuilds the records from
#     them in a recompute pass first (less memory held between the passes, one pass more).
SAVE_RECORDS = 0
DEFAULT_CKPT_EVERY = 8  # the checkpoint interval of the recompute mode
_BWD_RECORD_BYTES = 90112  # kBwdRecordBytes (csrc/kernels.h)


def _ptr(t: Optional[Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(t: Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def _problem(q, k, v, g, beta, scale, cu_seqlens, max_seqlen, use_qk_l2norm, ckpt_every) -> _lib.Problem:
    B, T, H, DK = q.shape
    HV, DV = v.shape[2], v.shape[3]
    N = B if cu_seqlens is None else cu_seqlens.numel() - 1
    return _lib.Problem(B=B, T=T, H=H, HV=HV, DK=DK, DV=DV, N=N,
                        cu_seqlens=None if cu_seqlens is None else cu_seqlens.data_ptr(),
                        max_seqlen=max_seqlen, scale=scale, act_dtype=_DT[q.dtype], g_dtype=_DT[g.dtype],
                        beta_dtype=_DT[beta.dtype], use_qk_l2norm=int(use_qk_l2norm), ckpt_every=ckpt_every)


def checkpoint_count(B: int, T: int, N: int, ckpt_every: int, varlen: bool) -> int:
    """Number of forward state checkpoints, the same count as ``gdn_checkpoint_count`` (gdn_abi.cu) computes:
    one per ``ckpt_every`` 64-token chunks of each sequence; with ``cu_seqlens`` an upper bound from the
    packed length and the number of sequences alone (no device read)."""
    if not varlen:
        nc = (T + 63) // 64
        return N * ((nc + ckpt_every - 1) // ckpt_every)
    nc = (B * T + 63 * N) // 64
    return nc // ckpt_every + N + 1


def _uses_chunk_kernels(q: Tensor, v: Tensor) -> bool:
    """The library's kernel-family choice (``gdn_uses_chunk_kernels``): chunked tcgen05 kernels for bf16 with
    dk = dv = 128, recurrent kernels otherwise."""
    return q.dtype == torch.bfloat16 and q.shape[-1] == 128 and v.shape[-1] == 128


def _saves_records(q: Tensor, v: Tensor, ckpt_every: int) -> bool:
    return ckpt_every == SAVE_RECORDS and _uses_chunk_kernels(q, v)


def saved_record_bytes(B: int, T: int, N: int, HV: int, varlen: bool) -> int:
    """Bytes of the backward records the forward saves (``gdn_chunk_saved_bytes``): one per 64-token chunk and
    value head; with ``cu_seqlens`` sized for the worst split of the packed tokens into N sequences."""
    chunks = (B * T + 63 * N) // 64 + N if varlen else N * ((T + 63) // 64)
    return chunks * HV * _BWD_RECORD_BYTES


def _check_inputs(q, k, v, g, beta, cu_seqlens):
    if not q.is_cuda:
        raise RuntimeError("sorernn_b200 runs on CUDA tensors only (no CPU fallback)")
    if q.shape != k.shape or q.dim() != 4:
        raise ValueError(f"q and k must be [B,T,H,K] with equal shapes, got {tuple(q.shape)} and {tuple(k.shape)}")
    B, T, H, _ = q.shape
    if v.dim() != 4 or v.shape[:2] != (B, T) or v.shape[2] % H:
        raise ValueError(f"v must be [B,T,HV,V] with HV a multiple of H, got {tuple(v.shape)}")
    HV = v.shape[2]
    for name, x in (("g", g), ("beta", beta)):
        if x.shape != (B, T, HV):
            raise ValueError(f"{name} must be [B,T,HV] = {(B, T, HV)}, got {tuple(x.shape)}")
    if q.dtype != k.dtype or q.dtype != v.dtype:
        raise ValueError("q, k and v must share one dtype")
    if cu_seqlens is not None and B != 1:  # gdn_ref.py:42-43
        raise ValueError(f"cu_seqlens requires B == 1, got B = {B}")


# ------------------------------------------------------------------------------------------------
# custom ops
# ------------------------------------------------------------------------------------------------
@torch.library.custom_op("sorernn_b200::gdn_fwd", mutates_args=())
def gdn_fwd(q: Tensor, k: Tensor, v: Tensor, g: Tensor, beta: Tensor, initial_state: Optional[Tensor],
            cu_seqlens: Optional[Tensor], scale: float, use_qk_l2norm: bool, max_seqlen: int,
            ckpt_every: int) -> tuple[Tensor, Tensor, Tensor]:
    """Returns ``(o, final_state, saved)``; ``saved`` feeds :func:`gdn_bwd`: the backward records (uint8) when
    ``ckpt_every == SAVE_RECORDS`` and the chunked kernels run, else fp32 state checkpoints."""
    saves = _saves_records(q, v, ckpt_every)
    p = _problem(q, k, v, g, beta, scale, cu_seqlens, max_seqlen, use_qk_l2norm,
                 DEFAULT_CKPT_EVERY if ckpt_every == SAVE_RECORDS else ckpt_every)
    L = _lib.lib()
    o = torch.empty_like(v)
    final = torch.empty(p.N, p.HV, p.DK, p.DV, dtype=torch.float32, device=q.device)
    # with cu_seqlens the sizes are upper bounds: the slots no sequence fills are zeros (the library zeroes
    # the records' unused tail itself), so the output is deterministic (the same in eager mode and under tracing)
    if saves:
        ck = torch.empty(L.gdn_chunk_saved_bytes(ctypes.byref(p)), dtype=torch.uint8, device=q.device)
    else:
        alloc = torch.zeros if cu_seqlens is not None else torch.empty
        n_ck = L.gdn_checkpoint_count(ctypes.byref(p))
        ck = alloc(max(n_ck, 0), p.HV, p.DK, p.DV, dtype=torch.float32, device=q.device)
    ws_bytes = L.gdn_chunk_fwd_workspace_size(ctypes.byref(p))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
    h0 = None if initial_state is None else initial_state.float().contiguous()
    fn, name = (L.gdn_chunk_fwd_save, "gdn_chunk_fwd_save") if saves else (L.gdn_chunk_fwd, "gdn_chunk_fwd")
    _lib.check(fn(ctypes.byref(p), _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(h0), _ptr(o), _ptr(final),
                  _ptr(ck), _ptr(ws), ws_bytes, _stream(q)), name)
    return o, final, ck


@gdn_fwd.register_fake
def _(q, k, v, g, beta, initial_state, cu_seqlens, scale, use_qk_l2norm, max_seqlen, ckpt_every):
    B, T, H, DK = q.shape
    HV, DV = v.shape[2], v.shape[3]
    N = B if cu_seqlens is None else cu_seqlens.shape[0] - 1
    varlen = cu_seqlens is not None
    if _saves_records(q, v, ckpt_every):  # no library call while tracing
        saved = q.new_empty(saved_record_bytes(B, T, N, HV, varlen), dtype=torch.uint8)
    else:
        k_ = DEFAULT_CKPT_EVERY if ckpt_every == SAVE_RECORDS else ckpt_every
        saved = q.new_empty(max(checkpoint_count(B, T, N, k_, varlen), 0), HV, DK, DV, dtype=torch.float32)
    return torch.empty_like(v), q.new_empty(N, HV, DK, DV, dtype=torch.float32), saved


@torch.library.custom_op("sorernn_b200::gdn_bwd", mutates_args=())
def gdn_bwd(q: Tensor, k: Tensor, v: Tensor, g: Tensor, beta: Tensor, initial_state: Optional[Tensor],
            checkpoints: Tensor, do: Tensor, dht: Optional[Tensor], cu_seqlens: Optional[Tensor], scale: float,
            use_qk_l2norm: bool, max_seqlen: int, ckpt_every: int) -> tuple[Tensor, Tensor, Tensor, Tensor, Tensor,
                                                                             Tensor]:
    """Returns ``(dq, dk, dv, dg, dbeta, dh0)``; dg, dbeta in the dtypes of g, beta; dh0 fp32.
    ``checkpoints`` is the third output of :func:`gdn_fwd` called with the same ``ckpt_every``."""
    saves = _saves_records(q, v, ckpt_every)
    p = _problem(q, k, v, g, beta, scale, cu_seqlens, max_seqlen, use_qk_l2norm,
                 DEFAULT_CKPT_EVERY if ckpt_every == SAVE_RECORDS else ckpt_every)
    L = _lib.lib()
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    dg = torch.empty(g.shape, dtype=torch.float32, device=q.device)
    db = torch.empty(beta.shape, dtype=torch.float32, device=q.device)
    dh0 = torch.empty(p.N, p.HV, p.DK, p.DV, dtype=torch.float32, device=q.device)
    dht_ = None if dht is None else dht.float().contiguous()
    if saves:  # the reverse sweep over the records the forward saved
        ws_bytes = L.gdn_chunk_bwd_saved_workspace_size(ctypes.byref(p))
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
        _lib.check(L.gdn_chunk_bwd_saved(ctypes.byref(p), _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta),
                                         _ptr(checkpoints), _ptr(do.contiguous()), _ptr(dht_), _ptr(dq), _ptr(dk),
                                         _ptr(dv), _ptr(dg), _ptr(db), _ptr(dh0), _ptr(ws), ws_bytes, _stream(q)),
                   "gdn_chunk_bwd_saved")
    else:
        ws_bytes = L.gdn_chunk_bwd_workspace_size(ctypes.byref(p))
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=q.device)
        h0 = None if initial_state is None else initial_state.float().contiguous()
        _lib.check(L.gdn_chunk_bwd(ctypes.byref(p), _ptr(q), _ptr(k), _ptr(v), _ptr(g), _ptr(beta), _ptr(h0),
                                   _ptr(checkpoints), _ptr(do.contiguous()), _ptr(dht_), _ptr(dq), _ptr(dk),
                                   _ptr(dv), _ptr(dg), _ptr(db), _ptr(dh0), _ptr(ws), ws_bytes, _stream(q)),
                   "gdn_chunk_bwd")
    return dq, dk, dv, dg.to(g.dtype), db.to(beta.dtype), dh0


@gdn_bwd.register_fake
def _(q, k, v, g, beta, initial_state, checkpoints, do, dht, cu_seqlens, scale, use_qk_l2norm, max_seqlen,
      ckpt_every):
    N = q.shape[0] if cu_seqlens is None else cu_seqlens.shape[0] - 1
    HV, DK, DV = v.shape[2], q.shape[3], v.shape[3]
    return (torch.empty_like(q), torch.empty_like(k), torch.empty_like(v), torch.empty_like(g),
            torch.empty_like(beta), q.new_empty(N, HV, DK, DV, dtype=torch.float32))


def _setup_context(ctx, inputs, output):
    q, k, v, g, beta, initial_state, cu_seqlens, scale, use_qk_l2norm, max_seqlen, ckpt_every = inputs
    o, _, ck = output
    ctx.save_for_backward(q, k, v, g, beta, initial_state, ck, cu_seqlens)
    ctx.args = (scale, use_qk_l2norm, max_seqlen, ckpt_every)
    ctx.has_h0 = initial_state is not None
    ctx.o_meta = (o.shape, o.dtype)
    # outputs the loss does not reach get None, not zero tensors: no zero fill of the saved records (hundreds
    # of MB) or of the final-state gradient on every backward
    ctx.set_materialize_grads(False)


def _backward(ctx, do, dht, _dck):
    q, k, v, g, beta, initial_state, ck, cu_seqlens = ctx.saved_tensors
    scale, l2, max_seqlen, ckpt_every = ctx.args
    if do is None:  # only the final state reaches the loss
        do = q.new_zeros(ctx.o_meta[0], dtype=ctx.o_meta[1])
    dq, dk, dv, dg, db, dh0 = gdn_bwd(q, k, v, g, beta, initial_state, ck, do, dht, cu_seqlens, scale, l2,
                                      max_seqlen, ckpt_every)
    return dq, dk, dv, dg, db, (dh0 if ctx.has_h0 else None), None, None, None, None, None


torch.library.register_autograd("sorernn_b200::gdn_fwd", _backward, setup_context=_setup_context)


# ------------------------------------------------------------------------------------------------
# gate and beta activations (the layer's use_gate_in_kernel / use_beta_sigmoid_in_kernel, gdn.py:157-162)
# ------------------------------------------------------------------------------------------------
@torch.library.custom_op("sorernn_b200::gdn_gate", mutates_args=())
def gdn_gate(a: Tensor, A_log: Tensor, dt_bias: Optional[Tensor]) -> Tensor:
    """``g = -exp(A_log) * softplus(a + dt_bias)`` in fp32 for raw ``a [..., HV]`` (gdn.py:191-194)."""
    HV = a.shape[-1]
    g = torch.empty(a.shape, dtype=torch.float32, device=a.device)
    A, dtb = A_log.float().contiguous(), None if dt_bias is None else dt_bias.float().contiguous()
    _lib.check(_lib.lib().gdn_gate_fwd(a.numel() // HV, HV, _ptr(a), _DT[a.dtype], _ptr(A), _ptr(dtb), _lib.FP32,
                                       _ptr(g), _stream(a)), "gdn_gate_fwd")
    return g


@gdn_gate.register_fake
def _(a, A_log, dt_bias):
    return torch.empty(a.shape, dtype=torch.float32, device=a.device)


@torch.library.custom_op("sorernn_b200::gdn_gate_bwd", mutates_args=())
def gdn_gate_bwd(a: Tensor, A_log: Tensor, dt_bias: Optional[Tensor], dg: Tensor) -> tuple[Tensor, Tensor, Tensor]:
    """Returns ``(da, dA_log, ddt_bias)``; ``ddt_bias`` is empty when ``dt_bias`` is None."""
    HV = a.shape[-1]
    da = torch.empty_like(a)
    dA = torch.empty(HV, dtype=torch.float32, device=a.device)
    ddt = torch.empty(HV if dt_bias is not None else 0, dtype=torch.float32, device=a.device)
    A, dtb = A_log.float().contiguous(), None if dt_bias is None else dt_bias.float().contiguous()
    _lib.check(_lib.lib().gdn_gate_bwd(a.numel() // HV, HV, _ptr(a), _DT[a.dtype], _ptr(A), _ptr(dtb), _lib.FP32,
                                       _ptr(dg.float().contiguous()), _ptr(da), _ptr(dA),
                                       _ptr(ddt) if dt_bias is not None else None, _stream(a)), "gdn_gate_bwd")
    return da, dA, ddt


@gdn_gate_bwd.register_fake
def _(a, A_log, dt_bias, dg):
    HV = a.shape[-1]
    return (torch.empty_like(a), a.new_empty(HV, dtype=torch.float32),
            a.new_empty(HV if dt_bias is not None else 0, dtype=torch.float32))


def _gate_setup(ctx, inputs, output):
    a, A_log, dt_bias = inputs
    ctx.save_for_backward(a, A_log, dt_bias)
    ctx.has_bias = dt_bias is not None


def _gate_backward(ctx, dg):
    a, A_log, dt_bias = ctx.saved_tensors
    da, dA, ddt = gdn_gate_bwd(a, A_log, dt_bias, dg)
    return da, dA.to(A_log.dtype), (ddt.to(dt_bias.dtype) if ctx.has_bias else None)


torch.library.register_autograd("sorernn_b200::gdn_gate", _gate_backward, setup_context=_gate_setup)


@torch.library.custom_op("sorernn_b200::gdn_beta_sigmoid", mutates_args=())
def gdn_beta_sigmoid(b: Tensor) -> Tensor:
    """``beta = sigmoid(b)`` in fp32."""
    beta = torch.empty(b.shape, dtype=torch.float32, device=b.device)
    _lib.check(_lib.lib().gdn_beta_sigmoid_fwd(b.numel(), _ptr(b), _DT[b.dtype], _ptr(beta), _stream(b)),
               "gdn_beta_sigmoid_fwd")
    return beta


@gdn_beta_sigmoid.register_fake
def _(b):
    return torch.empty(b.shape, dtype=torch.float32, device=b.device)


@torch.library.custom_op("sorernn_b200::gdn_beta_sigmoid_bwd", mutates_args=())
def gdn_beta_sigmoid_bwd(b: Tensor, dbeta: Tensor) -> Tensor:
    db = torch.empty_like(b)
    _lib.check(_lib.lib().gdn_beta_sigmoid_bwd(b.numel(), _ptr(b), _DT[b.dtype], _ptr(dbeta.float().contiguous()),
                                               _ptr(db), _stream(b)), "gdn_beta_sigmoid_bwd")
    return db


@gdn_beta_sigmoid_bwd.register_fake
def _(b, dbeta):
    return torch.empty_like(b)


def _beta_setup(ctx, inputs, output):
    ctx.save_for_backward(inputs[0])


def _beta_backward(ctx, dbeta):
    (b,) = ctx.saved_tensors
    return gdn_beta_sigmoid_bwd(b, dbeta)


torch.library.register_autograd("sorernn_b200::gdn_beta_sigmoid", _beta_backward, setup_context=_beta_setup)


# ------------------------------------------------------------------------------------------------
# public API
# ------------------------------------------------------------------------------------------------
def auto_pieces(q: Tensor, v: Tensor, cu_seqlens: Optional[Tensor]) -> int:
    """Pieces per sequence the op picks by itself: 1 unless the problem runs on the chunked kernels as a padded
    batch (no ``cu_seqlens``) of at most 64 (sequence, value head) pairs; then the largest of 2, 4, 8 that keeps
    pairs x pieces <= 128 (one wave of CTAs) and the pieces at least 512 tokens (8 chunks), in whole chunks.
    Measured on one B200 (config-1 rows, T = 4,096, fwd+bwd): 16 pairs 1.83 -> 0.56 ms on 8 pieces, 32 pairs
    1.88 -> 0.95 ms on 4, 64 pairs 1.98 -> 1.70 ms on 2. Never under torch.compile (the pieces path is not one of the registered custom
    ops)."""
    if cu_seqlens is not None or not _uses_chunk_kernels(q, v) or torch.compiler.is_compiling():
        return 1
    B, T = q.shape[:2]
    units = B * v.shape[2]
    if units > 64:
        return 1
    P = 1
    while P < 8 and units * P * 2 <= 128 and T % (64 * P * 2) == 0 and T // (P * 2) >= 512:
        P *= 2
    return P


def chunk_gated_delta_rule(q: Tensor, k: Tensor, v: Tensor, g: Tensor, beta: Tensor, scale: Optional[float] = None,
                           initial_state: Optional[Tensor] = None, output_final_state: bool = False,
                           use_qk_l2norm_in_kernel: bool = False, cu_seqlens: Optional[Tensor] = None,
                           cu_seqlens_cpu: Optional[Tensor] = None, ckpt_every: Optional[int] = None,
                           pieces: Optional[int] = None, **kwargs):
    """Gated delta rule, same contract as FLA's ``chunk_gated_delta_rule`` (q, k, v, g, beta order).

    q, k ``[B,T,H,K]``; v ``[B,T,HV,V]`` (HV a multiple of H: grouped value attention); g (log decay) and
    beta ``[B,T,HV]``; initial_state ``[N,HV,K,V]``. Returns ``(o [B,T,HV,V], final_state [N,HV,K,V] fp32 or
    None)``. ``cu_seqlens`` (int64 ``[N+1]``, B == 1) resets the state at each document start;
    ``cu_seqlens_cpu`` (same values on the host) is read only to size buffers, never to synchronise.

    FLA's gate keywords are accepted as the layer passes them (gdn.py:157-162): with
    ``use_gate_in_kernel=True`` (and ``A_log [HV]``, optional ``dt_bias [HV]``), ``g`` is the raw a_proj
    output and the log decay is ``-exp(A_log) * softplus(g + dt_bias)``; with
    ``use_beta_sigmoid_in_kernel=True``, ``beta`` is the raw b_proj output and ``sigmoid(beta)`` is used.
    Both activations run as fused CUDA kernels with their own backward (gradients reach a, b, A_log,
    dt_bias).

    ``ckpt_every`` picks what the chunked kernels keep for the backward: ``SAVE_RECORDS`` (0) saves every
    chunk's backward record (88 KB per 64-token chunk and value head) and the backward runs its reverse sweep
    alone; k >= 1 keeps one fp32 state every k chunks and the backward first rebuilds the records from them
    (less memory held between the passes, one pass more). ``None`` (the default): ``SAVE_RECORDS`` when
    autograd will need the backward, else ``DEFAULT_CKPT_EVERY`` (nothing per chunk is written for a
    forward without gradients).

    ``pieces`` (extra keyword): cut every sequence into that many pieces that run side by side, forward and
    backward (:mod:`sorernn_b200.pieces`), for problems with few (sequence, value head) pairs per GPU, whose
    serial per-pair chains would leave most SMs idle. ``None`` (the default) picks it when autograd will run
    a backward on a padded batch (no ``cu_seqlens``) of at most 64 pairs on the chunked kernels, with pieces
    of at least 512 tokens (``auto_pieces``); ``1`` never splits.
    """
    use_gate = bool(kwargs.pop("use_gate_in_kernel", False))
    A_log, dt_bias = kwargs.pop("A_log", None), kwargs.pop("dt_bias", None)
    use_beta_sigmoid = bool(kwargs.pop("use_beta_sigmoid_in_kernel", False))
    if kwargs.pop("cp_context", None) is not None:
        raise NotImplementedError("cp_context is not supported by this op (see sorernn_b200.seqsplit)")
    if kwargs:
        raise TypeError(f"unexpected keyword arguments: {sorted(kwargs)}")
    if use_gate:
        if A_log is None:
            raise ValueError("A_log must be provided when use_gate_in_kernel=True")
        if not g.is_cuda:
            raise RuntimeError("sorernn_b200 runs on CUDA tensors only (no CPU fallback)")
        HV = g.shape[-1]
        if A_log.numel() != HV or (dt_bias is not None and dt_bias.numel() != HV):
            raise ValueError(f"A_log and dt_bias must have HV = {HV} elements")
        g = gdn_gate(g.contiguous(), A_log.reshape(HV), None if dt_bias is None else dt_bias.reshape(HV))
    if use_beta_sigmoid:
        beta = gdn_beta_sigmoid(beta.contiguous())
    _check_inputs(q, k, v, g, beta, cu_seqlens)
    scale = q.shape[-1] ** -0.5 if scale is None else float(scale)
    if cu_seqlens is not None:
        cu_seqlens = cu_seqlens.to(device=q.device, dtype=torch.int64).contiguous()
        if cu_seqlens_cpu is not None:
            max_seqlen = int((cu_seqlens_cpu[1:] - cu_seqlens_cpu[:-1]).max()) if cu_seqlens_cpu.numel() > 1 else 0
        else:
            max_seqlen = q.shape[1]
    else:
        max_seqlen = q.shape[1]
    q, k, v, g, beta = (x.contiguous() for x in (q, k, v, g, beta))
    if ckpt_every is None:
        grads = torch.is_grad_enabled() and any(
            t is not None and t.requires_grad for t in (q, k, v, g, beta, initial_state))
        ckpt_every = SAVE_RECORDS if grads else DEFAULT_CKPT_EVERY
    elif ckpt_every < 0:
        raise ValueError(f"ckpt_every must be >= 0, got {ckpt_every}")
    if pieces is None:
        grads = torch.is_grad_enabled() and any(
            t is not None and t.requires_grad for t in (q, k, v, g, beta, initial_state))
        pieces = auto_pieces(q, v, cu_seqlens) if grads and ckpt_every == SAVE_RECORDS else 1
    if int(pieces) > 1:
        if cu_seqlens is not None:
            raise ValueError("pieces > 1 needs a padded batch (no cu_seqlens)")
        from .pieces import chunk_gated_delta_rule_pieces

        return chunk_gated_delta_rule_pieces(q, k, v, g, beta, int(pieces), scale=scale, initial_state=initial_state,
                                             output_final_state=output_final_state,
                                             use_qk_l2norm_in_kernel=use_qk_l2norm_in_kernel)
    o, final, _ = gdn_fwd(q, k, v, g, beta, initial_state, cu_seqlens, scale, bool(use_qk_l2norm_in_kernel),
                          int(max_seqlen), int(ckpt_every))
    return o, (final if output_final_state else None)


def fused_recurrent_gated_delta_rule_step(q: Tensor, k: Tensor, v: Tensor, g: Tensor, beta: Tensor, state: Tensor,
                                          scale: Optional[float] = None, use_qk_l2norm_in_kernel: bool = False,
                                          out: Optional[Tensor] = None) -> Tensor:
    """One decode token: ``q, k [N,H,K]``, ``v [N,HV,V]``, ``g, beta [N,HV]``, ``state [N,HV,K,V]`` fp32
    (updated in place). Returns ``o [N,HV,V]`` in v's dtype (written into ``out`` if given)."""
    if not q.is_cuda:
        raise RuntimeError("sorernn_b200 runs on CUDA tensors only (no CPU fallback)")
    if state.dtype != torch.float32 or not state.is_contiguous():
        raise ValueError("state must be a contiguous fp32 tensor")
    N, H, DK = q.shape
    HV, DV = v.shape[1], v.shape[2]
    if state.shape != (N, HV, DK, DV):
        raise ValueError(f"state must be {(N, HV, DK, DV)}, got {tuple(state.shape)}")
    scale = DK ** -0.5 if scale is None else float(scale)
    o = torch.empty_like(v) if out is None else out
    _lib.check(_lib.lib().gdn_decode_step(N, H, HV, DK, DV, scale, _DT[q.dtype], _DT[g.dtype], _DT[beta.dtype],
                                          int(use_qk_l2norm_in_kernel), _ptr(q.contiguous()), _ptr(k.contiguous()),
                                          _ptr(v.contiguous()), _ptr(g.contiguous()), _ptr(beta.contiguous()),
                                          _ptr(state), _ptr(o), _stream(q)), "gdn_decode_step")
    return o
