"""Sequence-split prefill over NCCL: one sequence cut into per-rank segments on 2 GPUs.

Each rank runs ``sequence_split_prefill`` (one segment per rank) or ``segmented_prefill`` (local pieces too)
on its own slice: the segment maps on the chunk kernels, one NCCL all_gather of every rank's map, the
composition of the maps before it, and the outputs from its true incoming state. The outputs of every rank
and the last rank's final state must match the oracle (the reference recurrence) on the whole sequence,
within the bf16 bar. Needs 2 GPUs; skipped otherwise. NVLS is off (NCCL_NVLS_ENABLE=0).
"""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

D = 128


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, splits, result, local_segments):
    import torch.distributed as dist

    from helpers import assert_bf16_close, assert_rms_close, to_np
    from inputs import make_inputs
    from oracle import cgdn
    from sorernn_b200 import seqsplit

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        B, H, HV = (1 if local_segments else 2), 2, 4  # segmented_prefill takes one sequence
        T = sum(splits)
        x = make_inputs(321, B, T, H, HV, D, D, normalized=False)
        h0 = np.random.default_rng(8).standard_normal((B, HV, D, D)) * 0.05
        a = sum(splits[:rank])
        e = a + splits[rank]
        dev = {n: torch.tensor(x[n][:, a:e], device="cuda").to(torch.bfloat16 if n in ("q", "k", "v") else
                                                                torch.float32).contiguous()
               for n in ("q", "k", "v", "g", "beta")}
        h0_dev = torch.tensor(h0, dtype=torch.float32, device="cuda")
        if local_segments:
            o, fin = seqsplit.segmented_prefill(dev["q"], dev["k"], dev["v"], dev["g"], dev["beta"],
                                                use_qk_l2norm_in_kernel=True, initial_state=h0_dev,
                                                local_segments=local_segments)
        else:
            o, fin = seqsplit.sequence_split_prefill(dev["q"], dev["k"], dev["v"], dev["g"], dev["beta"],
                                                     use_qk_l2norm_in_kernel=True, initial_state=h0_dev)
        torch.cuda.synchronize()
        # oracle on the whole sequence, from the same rounded inputs
        full = {n: x[n] for n in ("q", "k", "v", "g", "beta")}
        for n in ("q", "k", "v"):
            full[n] = to_np(torch.tensor(full[n]).to(torch.bfloat16))
        o_ref, s_ref = cgdn.forward(full["q"], full["k"], full["v"], full["g"], full["beta"], D ** -0.5,
                                    initial_state=h0, use_qk_l2norm=True)
        assert_bf16_close(to_np(o), o_ref[:, a:e], 2e-2, f"o rank {rank}")
        if rank == world - 1:
            assert fin is not None
            assert_rms_close(to_np(fin), s_ref, 2e-2, "final state")
        else:
            assert fin is None
        result[rank] = 1
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("local_segments", [0, 4])
def test_sequence_split_prefill_two_ranks_nccl(local_segments):
    ctx = torch.multiprocessing.get_context("spawn")
    result = ctx.Array("i", [0, 0])
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, [640, 448], result, local_segments)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank did not finish within 300 s"
    assert [p.exitcode for p in procs] == [0, 0] and list(result) == [1, 1]
