"""Config 4 at its own length: one sequence of T = 262,144 tokens (bf16, d = 128, chunk 64, in-kernel q/k L2
norm), forward only, against the C oracle (the reference recurrence, pinned by test_oracle_golden.py) run
on the same bf16-rounded inputs. Two heads instead of sixteen keep the oracle's host time to seconds; the
heads are independent, so the check covers every code path of the 16-head run.

Checked: the segmented prefill (the sequence cut into 8 local pieces joined by affine maps, the path
bench.py times for config 4 on one GPU) and the single chunked forward, outputs within the bf16 bar
beyond output rounding and final states within 2e-2 x RMS. The same inputs also run through 4 pieces, so
the piece count is covered. The cross-rank split of the same path is tests/test_gpu_seqsplit_nccl.py.
"""
import numpy as np
import pytest
import torch

from helpers import assert_bf16_close, assert_rms_close, to_np
from oracle import cgdn

pytestmark = pytest.mark.gpu
T, H, D = 262144, 2, 128


@pytest.fixture(scope="module")
def case():
    gen = torch.Generator(device="cuda").manual_seed(262144)
    x = dict(q=torch.randn(1, T, H, D, device="cuda", generator=gen).bfloat16(),
             k=torch.randn(1, T, H, D, device="cuda", generator=gen).bfloat16(),
             v=torch.randn(1, T, H, D, device="cuda", generator=gen).bfloat16(),
             g=torch.nn.functional.logsigmoid(torch.randn(1, T, H, device="cuda", generator=gen)) / 16,
             beta=torch.sigmoid(torch.randn(1, T, H, device="cuda", generator=gen)).bfloat16())
    xn = {n: to_np(t) for n, t in x.items()}
    o_ref, s_ref = cgdn.forward(xn["q"], xn["k"], xn["v"], xn["g"], xn["beta"], D ** -0.5, use_qk_l2norm=True)
    return x, o_ref, s_ref


@pytest.mark.parametrize("pieces", [8, 4])
def test_segmented_prefill_full_length_matches_oracle(case, pieces):
    from sorernn_b200.seqsplit import segmented_prefill

    x, o_ref, s_ref = case
    o, s = segmented_prefill(x["q"], x["k"], x["v"], x["g"], x["beta"], use_qk_l2norm_in_kernel=True,
                             local_segments=pieces)
    torch.cuda.synchronize()
    assert_bf16_close(to_np(o), o_ref, 2e-2, "long prefill o")
    assert_rms_close(to_np(s), s_ref, 2e-2, "long prefill final state")


def test_chunked_forward_full_length_matches_oracle(case):
    from sorernn_b200 import chunk_gated_delta_rule

    x, o_ref, s_ref = case
    o, s = chunk_gated_delta_rule(x["q"], x["k"], x["v"], x["g"], x["beta"], output_final_state=True,
                                  use_qk_l2norm_in_kernel=True)
    torch.cuda.synchronize()
    assert np.isfinite(to_np(s)).all()
    assert_bf16_close(to_np(o), o_ref, 2e-2, "long forward o")
    assert_rms_close(to_np(s), s_ref, 2e-2, "long forward final state")
