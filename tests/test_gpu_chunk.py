"""GPU parity of the chunked tcgen05 path (bf16 activations, dk = dv = 128) through the C ABI.

Expected values: the C oracle (the reference recurrence, gdn_ref.py:17-22, restated and pinned by
test_oracle_golden.py) run in fp32 on exactly the bf16-rounded inputs the GPU sees. Bars: fp32 outputs
(states, transition maps) max-abs error <= 2e-2 x RMS(reference); bf16 outputs: the same bound on the
error beyond the output's own bf16 rounding (helpers.assert_bf16_close); gradients 3e-2.
"""
import ctypes

import numpy as np
import pytest
import torch

from helpers import assert_bf16_close, assert_rms_close, to_np
from oracle import cgdn

pytestmark = pytest.mark.gpu
D = 128


def _inputs(seed, B, T, H, HV, normalized=True, g_scale=16.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B, T, H, D, device="cuda", generator=g)
    k = torch.randn(B, T, H, D, device="cuda", generator=g)
    if normalized:
        q, k = torch.nn.functional.normalize(q, dim=-1), torch.nn.functional.normalize(k, dim=-1)
    v = torch.randn(B, T, HV, D, device="cuda", generator=g)
    gg = torch.nn.functional.logsigmoid(torch.randn(B, T, HV, device="cuda", generator=g)) / g_scale
    beta = torch.sigmoid(torch.randn(B, T, HV, device="cuda", generator=g))
    do = torch.randn(B, T, HV, D, device="cuda", generator=g)
    bf = lambda x: x.bfloat16()  # noqa: E731
    return dict(q=bf(q), k=bf(k), v=bf(v), g=gg.float(), beta=bf(beta), do=bf(do))


def _np(x):
    return {n: to_np(t) for n, t in x.items()}


def test_chunk_kernels_selected_for_bf16_d128():
    from sorernn_b200 import _lib

    p = _lib.Problem(B=1, T=64, H=1, HV=1, DK=128, DV=128, N=1, cu_seqlens=None, max_seqlen=64, scale=1.0,
                     act_dtype=_lib.BF16, g_dtype=_lib.FP32, beta_dtype=_lib.BF16, use_qk_l2norm=1, ckpt_every=4)
    assert _lib.lib().gdn_uses_chunk_kernels(ctypes.byref(p)) == 1


@pytest.mark.parametrize("B,T,H,HV,l2", [(1, 64, 1, 1, False), (2, 300, 2, 2, True), (1, 130, 1, 2, True),
                                         (3, 1, 2, 2, False), (1, 1000, 2, 4, True)])
def test_chunk_forward_matches_oracle(B, T, H, HV, l2):
    from sorernn_b200 import chunk_gated_delta_rule

    x = _inputs(B * 1000 + T, B, T, H, HV, normalized=not l2)
    h0 = torch.randn(B, HV, D, D, device="cuda") * 0.05
    o, ht = chunk_gated_delta_rule(x["q"], x["k"], x["v"], x["g"], x["beta"], initial_state=h0,
                                   output_final_state=True, use_qk_l2norm_in_kernel=l2)
    xn = _np(x)
    o_ref, ht_ref = cgdn.forward(xn["q"], xn["k"], xn["v"], xn["g"], xn["beta"], D ** -0.5,
                                 initial_state=to_np(h0), use_qk_l2norm=l2)
    assert_bf16_close(to_np(o), o_ref, 2e-2, "o")
    assert_rms_close(to_np(ht), ht_ref, 2e-2, "final_state")


def test_chunk_forward_varlen_short_documents():
    from sorernn_b200 import chunk_gated_delta_rule

    cu = [0, 1, 3, 4, 70, 200, 512]
    x = _inputs(7, 1, 512, 2, 2, normalized=False)
    cu_t = torch.tensor(cu, device="cuda")
    o, ht = chunk_gated_delta_rule(x["q"], x["k"], x["v"], x["g"], x["beta"], output_final_state=True,
                                   use_qk_l2norm_in_kernel=True, cu_seqlens=cu_t, cu_seqlens_cpu=torch.tensor(cu))
    xn = _np(x)
    o_ref, ht_ref = cgdn.forward(xn["q"], xn["k"], xn["v"], xn["g"], xn["beta"], D ** -0.5, cu_seqlens=cu,
                                 use_qk_l2norm=True)
    assert_bf16_close(to_np(o), o_ref, 2e-2, "o")
    assert_rms_close(to_np(ht), ht_ref, 2e-2, "final_state")
    # documents are isolated: changing document [4, 70) leaves later documents bit-identical
    x2 = dict(x)
    x2["v"] = x["v"].clone()
    x2["v"][:, 4:70] = torch.randn_like(x2["v"][:, 4:70].float()).bfloat16()
    o2, _ = chunk_gated_delta_rule(x2["q"], x2["k"], x2["v"], x2["g"], x2["beta"], use_qk_l2norm_in_kernel=True,
                                   cu_seqlens=cu_t)
    assert torch.equal(o2[:, 70:], o[:, 70:]) and torch.equal(o2[:, :4], o[:, :4])
    assert not torch.equal(o2[:, 4:70], o[:, 4:70])


def test_chunk_forward_checkpoints_are_chunk_start_states():
    from sorernn_b200.gated_delta_rule import gdn_fwd

    T, K = 700, 2  # checkpoints at chunks 0, 2, 4, ... -> tokens 0, 128, 256, ...
    x = _inputs(11, 1, T, 1, 1)
    h0 = torch.randn(1, 1, D, D, device="cuda") * 0.05
    _, _, ck = gdn_fwd(x["q"], x["k"], x["v"], x["g"], x["beta"], h0, None, D ** -0.5, False, T, K)
    xn = _np(x)
    n_ck = (T + 63) // 64
    n_ck = (n_ck + K - 1) // K
    assert ck.shape[0] == n_ck
    assert_rms_close(to_np(ck[0]), to_np(h0[0]), 1e-6, "ckpt 0 = h0")
    for m in range(1, n_ck):
        t = 64 * K * m
        _, st = cgdn.forward(xn["q"][:, :t], xn["k"][:, :t], xn["v"][:, :t], xn["g"][:, :t], xn["beta"][:, :t],
                             D ** -0.5, initial_state=to_np(h0))
        assert_rms_close(to_np(ck[m]), st[0], 2e-2, f"ckpt {m}")


def test_chunk_forward_large_row_config1_shape():
    """One batch row of config 1 (T = 4096, H = 16) against the oracle (all 64 chunks of a sequence)."""
    from sorernn_b200 import chunk_gated_delta_rule

    x = _inputs(12, 1, 4096, 16, 16, normalized=False)
    o, ht = chunk_gated_delta_rule(x["q"], x["k"], x["v"], x["g"], x["beta"], output_final_state=True,
                                   use_qk_l2norm_in_kernel=True)
    xn = _np(x)
    o_ref, ht_ref = cgdn.forward(xn["q"], xn["k"], xn["v"], xn["g"], xn["beta"], D ** -0.5, use_qk_l2norm=True)
    assert_bf16_close(to_np(o), o_ref, 2e-2, "o")
    assert_rms_close(to_np(ht), ht_ref, 2e-2, "final_state")


def test_chunk_forward_strong_decay_stays_finite():
    """Large |g| (e.g. -exp(A_log) softplus(.) with A up to 16) must not overflow inside a chunk."""
    from sorernn_b200 import chunk_gated_delta_rule

    x = _inputs(13, 1, 256, 2, 2, g_scale=0.05)  # g ~ -20 x logsigmoid magnitude
    o, ht = chunk_gated_delta_rule(x["q"], x["k"], x["v"], x["g"], x["beta"], output_final_state=True)
    xn = _np(x)
    o_ref, ht_ref = cgdn.forward(xn["q"], xn["k"], xn["v"], xn["g"], xn["beta"], D ** -0.5)
    assert torch.isfinite(o.float()).all() and torch.isfinite(ht).all()
    assert_bf16_close(to_np(o), o_ref, 2e-2, "o")


def test_sequence_split_passes_bf16():
    from sorernn_b200 import chunk_gated_delta_rule, seqsplit

    B, T, H = 1, 640, 2
    x = _inputs(14, B, T, H, H)
    o_full, ht_full = chunk_gated_delta_rule(x["q"], x["k"], x["v"], x["g"], x["beta"], output_final_state=True)
    cut = 320
    segs = [{n: t[:, a:b].contiguous() for n, t in x.items()} for a, b in ((0, cut), (cut, T))]
    o1, c1 = chunk_gated_delta_rule(segs[0]["q"], segs[0]["k"], segs[0]["v"], segs[0]["g"], segs[0]["beta"],
                                    output_final_state=True)
    o2, c2 = chunk_gated_delta_rule(segs[1]["q"], segs[1]["k"], segs[1]["v"], segs[1]["g"], segs[1]["beta"],
                                    output_final_state=True)
    M = seqsplit.segment_transition(segs[1]["k"], segs[1]["g"], segs[1]["beta"])
    # M against the product of the per-token transitions (fp64, host)
    xn = {n: to_np(t).astype(np.float64) for n, t in segs[1].items()}
    Mref = np.broadcast_to(np.eye(D), (B, H, D, D)).copy()
    for t in range(T - cut):
        kk = xn["k"][:, t]
        Mt = np.exp(xn["g"][:, t])[..., None, None] * (np.eye(D) - xn["beta"][:, t][..., None, None]
                                                       * kk[..., :, None] * kk[..., None, :])
        Mref = Mt @ Mref
    assert_rms_close(to_np(M), Mref, 2e-2, "transition")
    s_out = seqsplit.combine(M, c2, c1)
    assert_rms_close(to_np(s_out), to_np(ht_full), 2e-2, "combined state")
    seqsplit.apply_incoming_state(segs[1]["q"], segs[1]["k"], segs[1]["g"], segs[1]["beta"], c1, o2, D ** -0.5)
    assert_bf16_close(to_np(torch.cat([o1, o2], 1)), to_np(o_full), 2e-2, "o")


# the two backward modes: records saved by the forward (the default when gradients are needed), and the
# recompute pass from state checkpoints (every 4 chunks here: several segments per sequence)
MODES = {"saved": 0, "recompute": 4}


def _grads_vs_oracle(x, h0, dht, l2, cu=None, tol=3e-2, mode="saved"):
    """fwd+bwd through the public op; compare every gradient with the oracle on the same inputs."""
    from sorernn_b200 import chunk_gated_delta_rule

    t = {n: x[n].clone().requires_grad_(n != "do") for n in x}
    h0t = None if h0 is None else h0.clone().requires_grad_(True)
    cu_t = None if cu is None else torch.tensor(cu, device="cuda")
    o, ht = chunk_gated_delta_rule(t["q"], t["k"], t["v"], t["g"], t["beta"], initial_state=h0t,
                                   output_final_state=True, use_qk_l2norm_in_kernel=l2, cu_seqlens=cu_t,
                                   cu_seqlens_cpu=None if cu is None else torch.tensor(cu),
                                   ckpt_every=MODES[mode])
    loss = (o.float() * t["do"].float()).sum() + (0 if dht is None else (ht * dht).sum())
    loss.backward()
    xn = _np(x)
    ref = cgdn.backward(xn["q"], xn["k"], xn["v"], xn["g"], xn["beta"], xn["do"], D ** -0.5,
                        initial_state=None if h0 is None else to_np(h0), dht=None if dht is None else to_np(dht),
                        cu_seqlens=cu, use_qk_l2norm=l2)
    got = [t["q"].grad, t["k"].grad, t["v"].grad, t["g"].grad, t["beta"].grad]
    for name, a, r in zip(("dq", "dk", "dv"), got[:3], ref[:3]):
        assert_bf16_close(to_np(a), r, tol, name)
    assert_rms_close(to_np(got[3]), ref[3], tol, "dg")
    assert_rms_close(to_np(got[4]), ref[4], tol, "dbeta")  # beta is bf16: its grad is rounded on return
    if h0 is not None:
        assert_rms_close(to_np(h0t.grad), ref[5], tol, "dh0")


@pytest.mark.parametrize("mode", sorted(MODES))
@pytest.mark.parametrize("B,T,H,HV,l2", [(1, 64, 1, 1, False), (2, 300, 2, 2, True), (1, 200, 1, 2, True),
                                         (1, 130, 2, 2, False)])
def test_chunk_backward_matches_oracle(B, T, H, HV, l2, mode):
    x = _inputs(B * 7 + T, B, T, H, HV, normalized=not l2)
    gen = torch.Generator(device="cuda").manual_seed(B * 7 + T + 1)
    h0 = torch.randn(B, HV, D, D, device="cuda", generator=gen) * 0.05
    dht = torch.randn(B, HV, D, D, device="cuda", generator=gen) * 0.1
    _grads_vs_oracle(x, h0, dht, l2, mode=mode)


@pytest.mark.parametrize("mode", sorted(MODES))
def test_chunk_backward_varlen_short_documents(mode):
    cu = [0, 1, 3, 4, 70, 200, 512]
    x = _inputs(21, 1, 512, 2, 2, normalized=False)
    _grads_vs_oracle(x, None, None, True, cu=cu, mode=mode)


@pytest.mark.parametrize("mode", sorted(MODES))
def test_chunk_backward_large_row_config1_shape(mode):
    x = _inputs(22, 1, 4096, 16, 16, normalized=False)
    _grads_vs_oracle(x, None, None, True, mode=mode)


def test_backward_mode_follows_autograd():
    """Without ckpt_every the op saves per-chunk records only when a backward will run: a forward without
    gradients keeps the small checkpoints, and both modes give the same gradients within the bf16 bar."""
    from sorernn_b200 import chunk_gated_delta_rule

    x = _inputs(31, 1, 640, 2, 2, normalized=False)
    with torch.no_grad():
        base = torch.cuda.memory_allocated()
        o, _ = chunk_gated_delta_rule(x["q"], x["k"], x["v"], x["g"], x["beta"], use_qk_l2norm_in_kernel=True)
        held_nograd = torch.cuda.memory_allocated() - base - o.numel() * o.element_size()
    del o
    assert held_nograd < 10 * 2 * 128 * 128 * 4  # no records (88 KB per chunk-head would be 1.8 MB here)
    grads = {}
    for mode, ck in (("auto", None), ("recompute", 8)):
        t = {n: x[n].clone().requires_grad_(n != "do") for n in x}
        o, _ = chunk_gated_delta_rule(t["q"], t["k"], t["v"], t["g"], t["beta"], use_qk_l2norm_in_kernel=True,
                                      ckpt_every=ck)
        o.backward(t["do"])
        grads[mode] = [to_np(t[n].grad) for n in ("q", "k", "v", "g", "beta")]
    for name, a, r in zip(("dq", "dk", "dv", "dg", "dbeta"), grads["auto"], grads["recompute"]):
        assert_rms_close(a, r, 2e-2, f"{name} saved vs recompute")


def test_saved_records_tail_is_zeroed_varlen():
    """With cu_seqlens the record buffer is sized for the worst split; the slots past the last sequence's
    chunks come back zero even when the allocator hands out a dirty block, so the op's outputs are a
    function of its inputs."""
    from sorernn_b200.gated_delta_rule import SAVE_RECORDS, gdn_fwd, saved_record_bytes

    cu = [0, 1, 3, 4, 70, 200, 512]
    x = _inputs(32, 1, 512, 2, 2, normalized=False)
    cu_t = torch.tensor(cu, device="cuda")
    nbytes = saved_record_bytes(1, 512, len(cu) - 1, 2, True)
    dirty = torch.full((nbytes,), 0xA5, dtype=torch.uint8, device="cuda")
    del dirty  # the caching allocator hands this block to the op's buffer of the same size
    _, _, rec = gdn_fwd(x["q"], x["k"], x["v"], x["g"], x["beta"], None, cu_t, D ** -0.5, True, 312, SAVE_RECORDS)
    assert rec.dtype == torch.uint8 and rec.numel() == nbytes
    used = sum((b - a + 63) // 64 for a, b in zip(cu[:-1], cu[1:])) * 2 * 90112
    assert used < nbytes
    assert int(rec[used:].count_nonzero()) == 0
    assert int(rec[:used].count_nonzero()) > 0


@pytest.mark.parametrize("l2", [True, False])
def test_segment_maps_and_outputs_share_one_prep(l2):
    """gdn_segment_maps / gdn_segment_outputs over one set of prep records: the C pass and the output pass
    are the forward's own state pass, so C and o equal the plain forward's bit for bit; M matches the
    transition map of the fused kernel (gdn_segment_transition) within the fp32 bar."""
    from sorernn_b200 import chunk_gated_delta_rule, seqsplit

    B, T, H, HV = 3, 300, 2, 4
    # weak decay (g / 256): M keeps entries of order 0.1 over 300 tokens, so the 2e-2 bar relative to its RMS
    # measures the kernel, not noise on a matrix that has decayed to ~1e-8
    x = _inputs(41, B, T, H, HV, normalized=not l2, g_scale=256.0)
    gen = torch.Generator(device="cuda").manual_seed(42)
    h0 = torch.randn(B, HV, D, D, device="cuda", generator=gen) * 0.05
    rec = seqsplit._Records(x["q"], x["v"], x["g"], x["beta"], D ** -0.5, l2)
    C, M = rec.maps(x["q"], x["k"], x["v"], x["g"], x["beta"], h0, True)
    o = rec.outputs(x["q"], x["k"], x["v"], x["g"], x["beta"], h0)
    o_ref, C_ref = chunk_gated_delta_rule(x["q"], x["k"], x["v"], x["g"], x["beta"], initial_state=h0,
                                          output_final_state=True, use_qk_l2norm_in_kernel=l2)
    assert torch.equal(C, C_ref)
    assert torch.equal(o, o_ref)
    M_ref = seqsplit.segment_transition(x["k"], x["g"], x["beta"], l2, HV)
    assert_rms_close(to_np(M), to_np(M_ref), 2e-2, "transition")
    xn = _np(x)  # M against the oracle: the final state of the recurrence from the identity with v = 0
    Mo = []
    for b in range(B):
        _, s_b = cgdn.forward(xn["q"][b:b + 1], xn["k"][b:b + 1], np.zeros_like(xn["v"][b:b + 1]),
                              xn["g"][b:b + 1], xn["beta"][b:b + 1], D ** -0.5,
                              initial_state=np.broadcast_to(np.eye(D, dtype=np.float32), (1, HV, D, D)).copy(),
                              use_qk_l2norm=l2)
        Mo.append(s_b)
    assert_rms_close(to_np(M), np.concatenate(Mo), 2e-2, "transition vs oracle")


@pytest.mark.parametrize("P,with_h0", [(4, True), (8, False), (1, True)])
def test_segmented_prefill_matches_one_forward(P, with_h0):
    """The sequence cut into P local pieces joined by affine maps == one chunk forward (bf16 bar)."""
    from sorernn_b200 import chunk_gated_delta_rule
    from sorernn_b200.seqsplit import segmented_prefill

    T, H, HV = 2048, 2, 4
    x = _inputs(15, 1, T, H, HV, normalized=False)
    h0 = (torch.randn(1, HV, D, D, device="cuda", generator=torch.Generator(device="cuda").manual_seed(4)) * 0.1
          if with_h0 else None)
    o_ref, s_ref = chunk_gated_delta_rule(x["q"], x["k"], x["v"], x["g"], x["beta"], initial_state=h0,
                                          output_final_state=True, use_qk_l2norm_in_kernel=True)
    o, s = segmented_prefill(x["q"], x["k"], x["v"], x["g"], x["beta"], use_qk_l2norm_in_kernel=True,
                             initial_state=h0, local_segments=P)
    assert_bf16_close(to_np(o), to_np(o_ref), 2e-2, "o")
    assert_rms_close(to_np(s), to_np(s_ref), 2e-2, "final state")


@pytest.mark.parametrize("mode", sorted(MODES))
def test_chunk_varlen_empty_documents_fwd_bwd(mode):
    """Zero-length documents at the start, middle and end: their final state is their initial state, their
    dh0 is their dht, and the neighbours are unaffected (forward and backward against the oracle)."""
    cu = [0, 0, 5, 5, 70, 70, 200, 200]
    N = len(cu) - 1
    x = _inputs(23, 1, 200, 2, 2, normalized=False)
    gen = torch.Generator(device="cuda").manual_seed(24)
    h0 = torch.randn(N, 2, D, D, device="cuda", generator=gen) * 0.05
    dht = torch.randn(N, 2, D, D, device="cuda", generator=gen) * 0.1
    _grads_vs_oracle(x, h0, dht, True, cu=cu, mode=mode)


def test_zero_length_sequences():
    """T = 0: empty outputs, the final state is the initial state and dh0 is dht."""
    from sorernn_b200 import chunk_gated_delta_rule

    B, H = 2, 2
    x = _inputs(25, B, 64, H, H)
    x0 = {n: t[:, :0].contiguous() for n, t in x.items()}
    gen = torch.Generator(device="cuda").manual_seed(26)
    h0 = (torch.randn(B, H, D, D, device="cuda", generator=gen) * 0.05).requires_grad_(True)
    leaves = {n: x0[n].clone().requires_grad_(True) for n in ("q", "k", "v", "g", "beta")}
    o, ht = chunk_gated_delta_rule(leaves["q"], leaves["k"], leaves["v"], leaves["g"], leaves["beta"],
                                   initial_state=h0, output_final_state=True, use_qk_l2norm_in_kernel=True)
    assert o.shape == (B, 0, H, D)
    assert torch.equal(ht, h0.detach())
    dht = torch.randn(B, H, D, D, device="cuda", generator=gen)
    (ht * dht).sum().backward()
    assert torch.equal(h0.grad, dht)
