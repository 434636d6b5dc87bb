"""Sequence-split prefill across ranks, host side: the boundary-state exchange of
``sorernn_b200.seqsplit.exchange_boundary_states`` (one all_gather of the segment maps, composed locally)
run over ``gloo`` ranks on CPU.

Each rank computes its segment's pieces with the oracle (the reference recurrence, gdn_ref.py:18-21):
outputs and final state ``C_r`` from a zero state (rank 0 from ``h0``), the transition ``M_r`` (the same
recurrence with ``v = 0`` started from the identity), and after the exchange the contribution of the
incoming state (the recurrence with ``v = 0`` started from ``S_in``). Concatenated over ranks, outputs and
the last rank's final state must equal one unsplit oracle run. The CUDA kernels behind those three pieces
have their own parity tests (tests/test_gpu_chunk.py, tests/test_gpu_recurrent.py).
"""
from __future__ import annotations

import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from inputs import make_inputs
from oracle.gdn_oracle import gdn_forward


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _segment_bounds(T: int, splits: list[int]) -> list[tuple[int, int]]:
    edges = [0] + list(np.cumsum(splits))
    assert edges[-1] == T
    return [(int(edges[r]), int(edges[r + 1])) for r in range(len(splits))]


def _case(l2: bool):
    B, T, H, HV, dk, dv = 2, 47, 2, 4, 8, 6
    x = make_inputs(77, B, T, H, HV, dk, dv, normalized=not l2)
    h0 = np.random.default_rng(5).standard_normal((B, HV, dk, dv)) * 0.1
    return x, h0


def _chain_worker(rank: int, world: int, port: int, splits: list[int], l2: bool):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    try:
        from sorernn_b200 import seqsplit

        x, h0 = _case(l2)
        B, T, H, dk = x["q"].shape
        HV, dv = x["v"].shape[2], x["v"].shape[3]
        a, e = _segment_bounds(T, splits)[rank]
        seg = {n: x[n][:, a:e] for n in ("q", "k", "v", "g", "beta")}
        o, C = gdn_forward(seg["q"], seg["k"], seg["v"], seg["g"], seg["beta"],
                           initial_state=h0 if rank == 0 else None, use_qk_l2norm=l2)
        M = None
        if rank > 0:
            eye = np.broadcast_to(np.eye(dk), (B, HV, dk, dk))
            _, M = gdn_forward(seg["q"], seg["k"], np.zeros((B, e - a, HV, dk)), seg["g"], seg["beta"],
                               initial_state=eye, use_qk_l2norm=l2)
            M = torch.from_numpy(np.ascontiguousarray(M))
        S_in, S_out = seqsplit.exchange_boundary_states(torch.from_numpy(C), M)
        if rank > 0:
            o_in, _ = gdn_forward(seg["q"], seg["k"], np.zeros((B, e - a, HV, dv)), seg["g"], seg["beta"],
                                  initial_state=S_in.numpy(), use_qk_l2norm=l2)
            o = o + o_in
        o_ref, s_ref = gdn_forward(x["q"], x["k"], x["v"], x["g"], x["beta"], initial_state=h0, use_qk_l2norm=l2)
        np.testing.assert_allclose(o, o_ref[:, a:e], rtol=1e-10, atol=1e-10)
        if rank == world - 1:
            np.testing.assert_allclose(S_out.numpy(), s_ref, rtol=1e-10, atol=1e-10)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("splits,l2", [([20, 27], False), ([20, 27], True), ([11, 16, 20], True),
                                       ([5, 30, 1, 11], False)])
def test_boundary_state_chain_matches_unsplit_oracle(splits, l2):
    mp.spawn(_chain_worker, args=(len(splits), _free_port(), splits, l2), nprocs=len(splits), join=True)


def _lost_sender_worker(rank: int, world: int, port: int, result):
    """Rank 0 leaves without joining the exchange; rank 1's all_gather must end with an error inside the
    group timeout."""
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
    from sorernn_b200 import seqsplit

    C = torch.zeros(1, 1, 4, 4, dtype=torch.float64)
    M = torch.eye(4, dtype=torch.float64).reshape(1, 1, 4, 4)
    if rank == 0:
        result[0] = 1  # left without joining the collective
        return
    try:
        seqsplit.exchange_boundary_states(C, M)
        result[1] = 2  # completed (must not happen)
    except RuntimeError:
        result[1] = 1  # the collective ended with an error


def test_lost_sender_ends_the_receive_with_an_error():
    ctx = mp.get_context("spawn")
    result = ctx.Array("i", [0, 0])
    port = _free_port()
    procs = [ctx.Process(target=_lost_sender_worker, args=(r, 2, port, result)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank did not finish within 60 s"
    assert list(result) == [1, 1]


def test_affine_scan_matches_sequential_composition():
    from sorernn_b200.seqsplit import affine_inclusive_scan

    g = torch.Generator().manual_seed(3)
    for P in (1, 2, 3, 5, 8):
        M = torch.randn(P, 2, 6, 6, generator=g, dtype=torch.float64) * 0.4
        C = torch.randn(P, 2, 6, 5, generator=g, dtype=torch.float64)
        Mi, Ci = affine_inclusive_scan(M, C)
        m, c = M[0], C[0]
        for s in range(P):
            if s:
                m, c = M[s] @ m, M[s] @ c + C[s]
            torch.testing.assert_close(Mi[s], m, rtol=1e-12, atol=1e-12)
            torch.testing.assert_close(Ci[s], c, rtol=1e-12, atol=1e-12)
