"""GPU parity of the layer's neighbouring steps (sorernn_b200.layer_ops) against the oracle's restatement
(forward) and torch fp64 autograd of the same formula (backward). Tolerances: fp32 1e-4 x RMS; bf16 2e-2
beyond the output's rounding, gradients 3e-2."""
import numpy as np
import pytest
import torch

from helpers import assert_bf16_close, assert_rms_close, to_np
from oracle.gdn_oracle import rms_norm_gated as rms_norm_gated_ref

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("D", [128, 64, 32, 1024])
def test_rms_norm_gated_forward_backward(dtype, D):
    from sorernn_b200.layer_ops import rms_norm_gated

    gen = torch.Generator(device="cuda").manual_seed(D)
    x = (torch.randn(3, 257, 4, D, device="cuda", generator=gen) * 2.0).to(dtype).requires_grad_(True)
    g = (torch.randn(3, 257, 4, D, device="cuda", generator=gen) * 2.0).to(dtype).requires_grad_(True)
    w = (1.0 + 0.2 * torch.randn(D, device="cuda", generator=gen)).requires_grad_(True)
    eps = 1e-6
    y = rms_norm_gated(x, g, w, None, activation="swish", eps=eps)
    y_ref = rms_norm_gated_ref(to_np(x), to_np(g), to_np(w), eps)
    fwd_check = assert_rms_close if dtype == torch.float32 else assert_bf16_close
    fwd_check(to_np(y), y_ref, 1e-4 if dtype == torch.float32 else 2e-2, "y")

    dy = torch.randn(y.shape, device="cuda", generator=gen).to(dtype)
    y.backward(dy)
    x64, g64, w64 = (t.detach().double().cpu().requires_grad_(True) for t in (x, g, w))
    r = torch.rsqrt(x64.pow(2).mean(-1, keepdim=True) + eps)
    (x64 * r * w64 * torch.nn.functional.silu(g64)).backward(dy.double().cpu())
    tol = 1e-4 if dtype == torch.float32 else 3e-2
    grad_check = assert_rms_close if dtype == torch.float32 else assert_bf16_close
    grad_check(to_np(x.grad), x64.grad.numpy(), tol, "dx")
    grad_check(to_np(g.grad), g64.grad.numpy(), tol, "dgate")
    assert_rms_close(to_np(w.grad), w64.grad.numpy(), 1e-4 if dtype == torch.float32 else 3e-2, "dweight")


def _doc_ids(cu, T):
    ids = np.zeros(T, dtype=np.int64)
    for n in range(len(cu) - 1):
        ids[cu[n]:cu[n + 1]] = n
    return ids


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
# C = 2144: several channel slabs per row (one block covers 4 KB of a row), the last one narrow
@pytest.mark.parametrize("K,varlen,C", [(4, False, 64), (4, True, 96), (3, True, 96), (2, False, 64), (1, False, 64),
                                        (4, True, 2144), (3, False, 2144)])
def test_causal_conv1d_silu_forward_backward(dtype, K, varlen, C):
    from oracle.gdn_oracle import causal_conv1d as conv_ref
    from sorernn_b200.layer_ops import causal_conv1d

    gen = torch.Generator(device="cuda").manual_seed(K * 10 + int(varlen) + C)
    B, T = (1, 301) if varlen else (2, 150)
    cu = [0, 1, 3, 90, 91, 200, 301] if varlen else None
    x = torch.randn(B, T, C, device="cuda", generator=gen).to(dtype).requires_grad_(True)
    w = (torch.randn(C, K, device="cuda", generator=gen) * K ** -0.5).requires_grad_(True)
    cu_t = None if cu is None else torch.tensor(cu, device="cuda")
    y, st = causal_conv1d(x, w, activation="silu", cu_seqlens=cu_t)
    assert st is None
    ids = None if cu is None else _doc_ids(cu, T)
    y_ref = conv_ref(to_np(x), to_np(w), ids)
    fwd_check = assert_rms_close if dtype == torch.float32 else assert_bf16_close
    fwd_check(to_np(y), y_ref, 1e-4 if dtype == torch.float32 else 2e-2, "y")

    dy = torch.randn(y.shape, device="cuda", generator=gen).to(dtype)
    y.backward(dy)
    # torch fp64 autograd of the reference formula (masked shifted sum, conv.py:6-23)
    x64, w64 = (t.detach().double().cpu().requires_grad_(True) for t in (x, w))
    z = x64 * w64[:, K - 1]
    for j in range(1, min(K, T)):
        term = x64[:, : T - j] * w64[:, K - 1 - j]
        if ids is not None:
            same = torch.tensor(ids[j:] == ids[: T - j])
            term = term.masked_fill(~same[None, :, None], 0.0)
        z = z + torch.nn.functional.pad(term, (0, 0, j, 0))
    torch.nn.functional.silu(z).backward(dy.double().cpu())
    tol = 1e-4 if dtype == torch.float32 else 3e-2
    grad_check = assert_rms_close if dtype == torch.float32 else assert_bf16_close
    grad_check(to_np(x.grad), x64.grad.numpy(), tol, "dx")
    assert_rms_close(to_np(w.grad), w64.grad.numpy(), 1e-4 if dtype == torch.float32 else 3e-2, "dweight")


@pytest.mark.parametrize("K", [4, 3])
def test_causal_conv1d_ranges_over_many_tiles(K):
    """Rows of 4 KB (2,048 bf16 channels) over 8,880 tokens: every block's token range spans several tiles of
    its two-stage ring (stages refilled), with document boundaries at arbitrary rows, inside tiles and across
    ranges."""
    from oracle.gdn_oracle import causal_conv1d as conv_ref
    from sorernn_b200.layer_ops import causal_conv1d

    gen = torch.Generator(device="cuda").manual_seed(100 + K)
    T, C = 8880, 2048
    rng = np.random.default_rng(K)
    cu = [0] + sorted(rng.choice(np.arange(1, T), 40, replace=False).tolist()) + [T]
    x = torch.randn(1, T, C, device="cuda", generator=gen).bfloat16().requires_grad_(True)
    w = (torch.randn(C, K, device="cuda", generator=gen) * K ** -0.5).requires_grad_(True)
    y, _ = causal_conv1d(x, w, activation="silu", cu_seqlens=torch.tensor(cu, device="cuda"))
    ids = _doc_ids(cu, T)
    assert_bf16_close(to_np(y), conv_ref(to_np(x), to_np(w), ids), 2e-2, "y")
    dy = torch.randn(y.shape, device="cuda", generator=gen).bfloat16()
    y.backward(dy)
    x64, w64 = (t.detach().double().cpu().requires_grad_(True) for t in (x, w))
    z = x64 * w64[:, K - 1]
    for j in range(1, K):
        same = torch.tensor(ids[j:] == ids[: T - j])
        z = z + torch.nn.functional.pad((x64[:, : T - j] * w64[:, K - 1 - j]).masked_fill(~same[None, :, None], 0.0),
                                        (0, 0, j, 0))
    torch.nn.functional.silu(z).backward(dy.double().cpu())
    assert_bf16_close(to_np(x.grad), x64.grad.numpy(), 3e-2, "dx")
    assert_rms_close(to_np(w.grad), w64.grad.numpy(), 3e-2, "dweight")


def test_rms_norm_gated_blocks_over_many_tiles():
    """94,720 rows of 128 bf16 features: every block walks about ten 32-row tiles, so its four-stage ring is
    refilled several times, in both directions."""
    from sorernn_b200.layer_ops import rms_norm_gated

    gen = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(94720, 128, device="cuda", generator=gen).bfloat16().requires_grad_(True)
    g = torch.randn(94720, 128, device="cuda", generator=gen).bfloat16().requires_grad_(True)
    w = (1.0 + 0.2 * torch.randn(128, device="cuda", generator=gen)).requires_grad_(True)
    y = rms_norm_gated(x, g, w, None, activation="swish", eps=1e-6)
    assert_bf16_close(to_np(y), rms_norm_gated_ref(to_np(x), to_np(g), to_np(w), 1e-6), 2e-2, "y")
    dy = torch.randn(y.shape, device="cuda", generator=gen).bfloat16()
    y.backward(dy)
    x64, g64, w64 = (t.detach().double().cpu().requires_grad_(True) for t in (x, g, w))
    r = torch.rsqrt(x64.pow(2).mean(-1, keepdim=True) + 1e-6)
    (x64 * r * w64 * torch.nn.functional.silu(g64)).backward(dy.double().cpu())
    assert_bf16_close(to_np(x.grad), x64.grad.numpy(), 3e-2, "dx")
    assert_bf16_close(to_np(g.grad), g64.grad.numpy(), 3e-2, "dgate")
    assert_rms_close(to_np(w.grad), w64.grad.numpy(), 3e-2, "dweight")
