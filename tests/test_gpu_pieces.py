"""GPU parity of training on pieces (sorernn_b200.pieces): every sequence cut into P pieces that run side by
side, joined by their affine maps in the forward and by the transposed maps in the backward.

Expected values: the C oracle on the same bf16-rounded inputs (unsplit sequences). Bars as in
test_gpu_chunk.py: bf16 outputs and gradients beyond their own rounding 2e-2 / 3e-2 x RMS; fp32 states 2e-2.
"""
import pytest
import torch

from helpers import assert_bf16_close, assert_rms_close, to_np
from oracle import cgdn

pytestmark = pytest.mark.gpu
D = 128


def _inputs(seed, B, T, H, HV):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B, T, H, D, device="cuda", generator=g)
    k = torch.randn(B, T, H, D, device="cuda", generator=g)
    v = torch.randn(B, T, HV, D, device="cuda", generator=g)
    gg = torch.nn.functional.logsigmoid(torch.randn(B, T, HV, device="cuda", generator=g)) / 16
    beta = torch.sigmoid(torch.randn(B, T, HV, device="cuda", generator=g))
    do = torch.randn(B, T, HV, D, device="cuda", generator=g)
    h0 = torch.randn(B, HV, D, D, device="cuda", generator=g) * 0.05
    dht = torch.randn(B, HV, D, D, device="cuda", generator=g) * 0.1
    bf = lambda x: x.bfloat16()  # noqa: E731
    return dict(q=bf(q), k=bf(k), v=bf(v), g=gg.float(), beta=bf(beta), do=bf(do)), h0, dht


# (1, 300, 1, 2, 3): pieces of 100 tokens, so every piece ends in a partial chunk
@pytest.mark.parametrize("B,T,H,HV,P,with_state", [(2, 1024, 2, 2, 4, True), (1, 4096, 1, 2, 8, False),
                                                   (2, 640, 2, 4, 5, True), (1, 512, 1, 1, 1, True),
                                                   (1, 300, 1, 2, 3, True)])
def test_pieces_fwd_bwd_match_oracle(B, T, H, HV, P, with_state):
    from sorernn_b200.pieces import chunk_gated_delta_rule_pieces

    x, h0, dht = _inputs(B * 31 + T + P, B, T, H, HV)
    if not with_state:
        h0 = dht = None
    t = {n: x[n].clone().requires_grad_(n != "do") for n in x}
    h0t = None if h0 is None else h0.clone().requires_grad_(True)
    o, ht = chunk_gated_delta_rule_pieces(t["q"], t["k"], t["v"], t["g"], t["beta"], pieces=P, initial_state=h0t,
                                          output_final_state=True, use_qk_l2norm_in_kernel=True)
    loss = (o.float() * t["do"].float()).sum() + (0 if dht is None else (ht * dht).sum())
    loss.backward()
    xn = {n: to_np(v) for n, v in x.items()}
    h0n = None if h0 is None else to_np(h0)
    o_ref, s_ref = cgdn.forward(xn["q"], xn["k"], xn["v"], xn["g"], xn["beta"], D ** -0.5, initial_state=h0n,
                                use_qk_l2norm=True)
    ref = cgdn.backward(xn["q"], xn["k"], xn["v"], xn["g"], xn["beta"], xn["do"], D ** -0.5, initial_state=h0n,
                        dht=None if dht is None else to_np(dht), use_qk_l2norm=True)
    assert_bf16_close(to_np(o), o_ref, 2e-2, "pieces o")
    assert_rms_close(to_np(ht), s_ref, 2e-2, "pieces final state")
    got = [t["q"].grad, t["k"].grad, t["v"].grad, t["g"].grad, t["beta"].grad]
    for name, a, r in zip(("dq", "dk", "dv"), got[:3], ref[:3]):
        assert_bf16_close(to_np(a), r, 3e-2, "pieces " + name)
    assert_rms_close(to_np(got[3]), ref[3], 3e-2, "pieces dg")
    assert_rms_close(to_np(got[4]), ref[4], 3e-2, "pieces dbeta")
    if h0 is not None:
        assert_rms_close(to_np(h0t.grad), ref[5], 3e-2, "pieces dh0")


def test_pieces_match_the_unsplit_op():
    """Same inputs through the unsplit op and on 4 pieces: outputs and gradients agree within the bf16 bar
    (the pieces differ only in where the state is rounded to bf16 operand tiles)."""
    from sorernn_b200 import chunk_gated_delta_rule
    from sorernn_b200.pieces import chunk_gated_delta_rule_pieces

    x, _, _ = _inputs(7, 1, 2048, 2, 2)
    res = {}
    for name, fn in (("one", lambda *a, **kw: chunk_gated_delta_rule(*a, pieces=1, **kw)),
                     ("pieces", lambda *a, **kw: chunk_gated_delta_rule_pieces(*a, pieces=4, **kw))):
        t = {n: x[n].clone().requires_grad_(n != "do") for n in x}
        o, _ = fn(t["q"], t["k"], t["v"], t["g"], t["beta"], use_qk_l2norm_in_kernel=True)
        o.backward(t["do"])
        res[name] = [to_np(o)] + [to_np(t[n].grad) for n in ("q", "k", "v", "g", "beta")]
    for name, a, r in zip(("o", "dq", "dk", "dv", "dg", "dbeta"), res["pieces"], res["one"]):
        assert_rms_close(a, r, 3e-2, "pieces vs one " + name)


def test_pieces_reject_bad_arguments():
    from sorernn_b200.pieces import chunk_gated_delta_rule_pieces

    x, _, _ = _inputs(3, 1, 300, 1, 1)
    with pytest.raises(ValueError):
        chunk_gated_delta_rule_pieces(x["q"], x["k"], x["v"], x["g"], x["beta"], pieces=7)
    with pytest.raises(ValueError):
        chunk_gated_delta_rule_pieces(x["q"].float(), x["k"].float(), x["v"].float(), x["g"], x["beta"].float(),
                                      pieces=2)


@pytest.mark.parametrize("P", [1, 2, 5, 8])
@pytest.mark.parametrize("with_start", [False, True])
def test_piece_chain_kernel_matches_the_torch_scans(P, with_start):
    """gdn_piece_chain (fp32 FMAs on the CUDA cores) against the torch log-depth scans that the CPU test pins
    to the oracle: both directions, with and without a start state."""
    from sorernn_b200.pieces import _chain, end_state_grads, incoming_states
    from sorernn_b200.gated_delta_rule import _stream

    B, HV = 2, 3
    gen = torch.Generator(device="cuda").manual_seed(P * 2 + with_start)
    M = torch.randn(B, P, HV, D, D, device="cuda", generator=gen) / D ** 0.5
    C = torch.randn(B, P, HV, D, D, device="cuda", generator=gen)
    start = torch.randn(B, HV, D, D, device="cuda", generator=gen) if with_start else None
    S_in = torch.empty(B * P, HV, D, D, device="cuda")
    final = torch.empty(B, HV, D, D, device="cuda")
    _chain(B, P, HV, M, C, start, S_in, final, 0, _stream(M))
    ref_in, ref_final = incoming_states(M.double(), C.double(), None if start is None else start.double())
    assert_rms_close(to_np(S_in.view(B, P, HV, D, D)), to_np(ref_in), 1e-4, "piece chain states")
    assert_rms_close(to_np(final), to_np(ref_final), 1e-4, "piece chain final")
    X = torch.empty(B * P, HV, D, D, device="cuda")
    _chain(B, P, HV, M, C, start, X, None, 1, _stream(M))
    ref_x = end_state_grads(M.double().transpose(-1, -2), C.double(), None if start is None else start.double())
    assert_rms_close(to_np(X.view(B, P, HV, D, D)), to_np(ref_x), 1e-4, "piece chain gradients")


@pytest.mark.parametrize("HV,with_dht", [(2, True), (4, False)])
def test_state_grad_sweep_equals_the_full_sweeps_dh0(HV, with_dht):
    """gdn_chunk_state_grad_saved carries dS with the full sweep's own steps, so its dh0 is the full
    sweep's dh0 bit for bit (grouped value heads included)."""
    import ctypes

    from sorernn_b200 import _lib
    from sorernn_b200.gated_delta_rule import SAVE_RECORDS, _problem, _ptr, _stream, gdn_bwd, gdn_fwd

    x, _, dht = _inputs(41 + HV, 2, 700, 2, HV)
    dht = dht if with_dht else None
    scale = D ** -0.5
    _, _, rec = gdn_fwd(x["q"], x["k"], x["v"], x["g"], x["beta"], None, None, scale, True, 700, SAVE_RECORDS)
    full = gdn_bwd(x["q"], x["k"], x["v"], x["g"], x["beta"], None, rec, x["do"], dht, None, scale, True, 700,
                   SAVE_RECORDS)[5]
    p = _problem(x["q"], x["k"], x["v"], x["g"], x["beta"], scale, None, 700, True, 8)
    L = _lib.lib()
    n = L.gdn_chunk_bwd_saved_workspace_size(ctypes.byref(p))
    ws = torch.empty(n, dtype=torch.uint8, device="cuda")
    dh0 = torch.full_like(full, float("nan"))
    _lib.check(L.gdn_chunk_state_grad_saved(ctypes.byref(p), _ptr(x["q"]), _ptr(x["k"]), _ptr(x["v"]), _ptr(x["g"]),
                                            _ptr(x["beta"]), _ptr(rec), _ptr(x["do"]),
                                            _ptr(None if dht is None else dht.contiguous()), _ptr(dh0), _ptr(ws), n,
                                            _stream(x["q"])), "gdn_chunk_state_grad_saved")
    torch.cuda.synchronize()
    assert torch.equal(dh0, full)


@pytest.mark.parametrize("B,T,want", [(1, 4096, 8), (4, 1024, 2)])
def test_op_picks_pieces_by_itself_for_few_sequence_heads(B, T, want):
    """chunk_gated_delta_rule on a padded batch of 16 or 64 (sequence, head) pairs with gradients runs on 8 or
    2 pieces (auto_pieces), and its outputs and gradients match the unsplit op's (pieces=1) within the bf16
    bar."""
    from sorernn_b200 import chunk_gated_delta_rule
    from sorernn_b200.gated_delta_rule import auto_pieces

    x, _, _ = _inputs(9 + B, B, T, 16, 16)
    assert auto_pieces(x["q"], x["v"], None) == want
    res = {}
    for name, P in (("auto", None), ("one", 1)):
        t = {n: x[n].clone().requires_grad_(n != "do") for n in x}
        o, _ = chunk_gated_delta_rule(t["q"], t["k"], t["v"], t["g"], t["beta"], use_qk_l2norm_in_kernel=True,
                                      pieces=P)
        o.backward(t["do"])
        res[name] = [to_np(o)] + [to_np(t[n].grad) for n in ("q", "k", "v", "g", "beta")]
    for name, a, r in zip(("o", "dq", "dk", "dv", "dg", "dbeta"), res["auto"], res["one"]):
        assert_rms_close(a, r, 3e-2, "auto pieces vs one " + name)
