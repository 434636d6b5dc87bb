"""GPU parity of the recurrent kernels (fp32 path, decode step, sequence-split passes) via the C ABI.

Every expected value comes from the reference: the golden fixtures (soreRNN's naive_gated_delta_rule
with autograd, fp64) or the CPU oracle that those fixtures pin. Tolerances: max-abs <= 1e-4 x RMS for
fp32 outputs, states and gradients; 2e-2 for bf16 inputs.
"""
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from helpers import assert_bf16_close, assert_rms_close, to_np
from inputs import make_inputs, make_state_inputs
from oracle import cgdn

pytestmark = pytest.mark.gpu

GOLD = Path(__file__).resolve().parent / "golden"
META = json.loads((GOLD / "golden.json").read_text())
CASES = [n for n in META if n not in ("config0_checksum", "initial_state")]


def _dev(x, dtype=torch.float32, grad=False):
    return torch.tensor(x, dtype=dtype, device="cuda", requires_grad=grad)


def _run(x, m, dtype=torch.float32, h0=None, dht=None, cu=None):
    from sorernn_b200 import chunk_gated_delta_rule

    t = {n: _dev(x[n], dtype, grad=(n != "do")) for n in ("q", "k", "v", "g", "beta", "do")}
    h0_t = None if h0 is None else _dev(h0, grad=True)
    cu_t = None if cu is None else torch.tensor(cu, dtype=torch.long, device="cuda")
    o, ht = chunk_gated_delta_rule(t["q"], t["k"], t["v"], t["g"], t["beta"], scale=m["scale"], initial_state=h0_t,
                                   output_final_state=True, use_qk_l2norm_in_kernel=m.get("l2norm", False),
                                   cu_seqlens=cu_t, cu_seqlens_cpu=None if cu is None else torch.tensor(cu))
    loss = (o.float() * t["do"].float()).sum()
    if dht is not None:
        loss = loss + (ht * _dev(dht)).sum()
    loss.backward()
    grads = {"d" + n: to_np(t[n].grad) for n in ("q", "k", "v", "g", "beta")}
    if h0_t is not None:
        grads["dh0"] = to_np(h0_t.grad)
    return to_np(o), to_np(ht), grads


@pytest.mark.parametrize("name", CASES)
def test_fp32_matches_reference_golden(name):
    m = META[name]
    x = make_inputs(m["seed"], m["B"], m["T"], m["H"], m["HV"], m["dk"], m["dv"], normalized=not m["l2norm"],
                    g_mode=m["g_mode"])
    ref = dict(np.load(GOLD / f"{name}.npz"))
    o, _, grads = _run(x, m, cu=m["cu"])
    assert_rms_close(o, ref["o"], 1e-4, "o")
    for n, a in grads.items():
        assert_rms_close(a, ref[n], 1e-4, n)


def test_fp32_initial_state_and_final_state():
    m = META["initial_state"]
    x = make_inputs(m["seed"], m["B"], m["T"], m["H"], m["HV"], m["dk"], m["dv"])
    h0, dht = make_state_inputs(m["seed"], m["B"], m["HV"], m["dk"], m["dv"])
    ref = dict(np.load(GOLD / "initial_state.npz"))
    o, ht, grads = _run(x, m, h0=h0, dht=dht)
    assert_rms_close(o, ref["o"], 1e-4, "o")
    assert_rms_close(ht, ref["ht"], 1e-4, "final_state")
    for n, a in grads.items():
        assert_rms_close(a, ref[n], 1e-4, n)


def test_fp32_config0_against_reference_checksum():
    m = META["config0_checksum"]
    x = {n: a.astype(np.float32) for n, a in
         make_inputs(m["seed"], m["B"], m["T"], m["H"], m["HV"], m["dk"], m["dv"]).items()}
    o, _, grads = _run(x, m)
    outs = dict(o=o, **grads)
    for n, s in m["outputs"].items():
        flat = outs[n].reshape(-1).astype(np.float64)
        rms_ref = np.sqrt(s["sumsq"] / flat.size)
        err = np.abs(flat[s["idx"]] - np.asarray(s["val"])).max()
        assert err <= 1e-4 * rms_ref, f"{n}: sampled max err {err:.3e} > 1e-4 RMS {rms_ref:.3e}"
        assert abs(np.sqrt((flat ** 2).sum()) - np.sqrt(s["sumsq"])) <= 1e-4 * np.sqrt(s["sumsq"]), n


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-4), (torch.bfloat16, 2e-2)])
def test_decode_steps_match_oracle(dtype, tol):
    from sorernn_b200 import fused_recurrent_gated_delta_rule_step

    N, H, HV, d = 6, 2, 4, 128
    rng = np.random.default_rng(3)
    state = (rng.standard_normal((N, HV, d, d)) * 0.02).astype(np.float32)
    st_dev = torch.tensor(state, device="cuda")
    st_ref = state.copy()
    for step in range(3):
        x = make_inputs(40 + step, N, 1, H, HV, d, d)
        xs = {n: x[n][:, 0] for n in ("q", "k", "v", "g", "beta")}
        dev = {n: torch.tensor(a, device="cuda").to(dtype) for n, a in xs.items()}
        o = fused_recurrent_gated_delta_rule_step(dev["q"], dev["k"], dev["v"], dev["g"], dev["beta"], st_dev,
                                                  scale=d ** -0.5)
        # the oracle sees the same (rounded) inputs
        xr = {n: to_np(t) for n, t in dev.items()}
        o_ref = cgdn.decode_step(xr["q"], xr["k"], xr["v"], xr["g"], xr["beta"], st_ref, d ** -0.5)
        assert_rms_close(to_np(o), o_ref, tol, f"o step {step}")
        assert_rms_close(to_np(st_dev), st_ref, 1e-4, f"state step {step}")


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-4), (torch.bfloat16, 2e-2)])
def test_decode_many_heads_per_cta(dtype, tol):
    """600 heads: every CTA of the persistent d=128 decode kernel streams several heads through its
    shared-memory stages (stage reuse, bulk-store / bulk-load ordering); L2 norm on, GVA 2."""
    from sorernn_b200 import fused_recurrent_gated_delta_rule_step

    N, H, HV, d = 75, 4, 8, 128
    rng = np.random.default_rng(11)
    state = (rng.standard_normal((N, HV, d, d)) * 0.05).astype(np.float32)
    st_dev = torch.tensor(state, device="cuda")
    st_ref = state.copy()
    for step in range(2):
        x = make_inputs(70 + step, N, 1, H, HV, d, d, normalized=False)
        dev = {n: torch.tensor(x[n][:, 0], device="cuda").to(dtype) for n in ("q", "k", "v", "g", "beta")}
        o = fused_recurrent_gated_delta_rule_step(dev["q"], dev["k"], dev["v"], dev["g"], dev["beta"], st_dev,
                                                  scale=d ** -0.5, use_qk_l2norm_in_kernel=True)
        xr = {n: to_np(t) for n, t in dev.items()}
        o_ref = cgdn.decode_step(xr["q"], xr["k"], xr["v"], xr["g"], xr["beta"], st_ref, d ** -0.5,
                                 use_qk_l2norm=True)
        if dtype == torch.bfloat16:  # o is rounded to bf16: check the error beyond that rounding
            assert_bf16_close(to_np(o), o_ref, tol, f"o step {step}")
        else:
            assert_rms_close(to_np(o), o_ref, tol, f"o step {step}")
        assert_rms_close(to_np(st_dev), st_ref, 1e-4, f"state step {step}")


def test_decode_l2norm_and_gva_small_head():
    from sorernn_b200 import fused_recurrent_gated_delta_rule_step

    N, H, HV, dk, dv = 5, 1, 3, 24, 40
    x = make_inputs(9, N, 1, H, HV, dk, dv, normalized=False)
    h0, _ = make_state_inputs(9, N, HV, dk, dv)
    st_dev = torch.tensor(h0, dtype=torch.float32, device="cuda")
    dev = {n: torch.tensor(x[n][:, 0], dtype=torch.float32, device="cuda") for n in ("q", "k", "v", "g", "beta")}
    o = fused_recurrent_gated_delta_rule_step(dev["q"], dev["k"], dev["v"], dev["g"], dev["beta"], st_dev, 0.3,
                                              use_qk_l2norm_in_kernel=True)
    st_ref = h0.astype(np.float32)
    o_ref = cgdn.decode_step(x["q"][:, 0], x["k"][:, 0], x["v"][:, 0], x["g"][:, 0], x["beta"][:, 0], st_ref, 0.3,
                             use_qk_l2norm=True)
    assert_rms_close(to_np(o), o_ref, 1e-4, "o")
    assert_rms_close(to_np(st_dev), st_ref, 1e-4, "state")


def test_segment_passes_rebuild_the_unsplit_sequence_fp32():
    """Split one sequence in two segments: zero-state run + transition + apply_state == one run."""
    from sorernn_b200 import chunk_gated_delta_rule
    from sorernn_b200 import seqsplit

    B, T, H, d = 2, 150, 2, 32
    x = make_inputs(21, B, T, H, H, d, d)
    dev = {n: torch.tensor(a, dtype=torch.float32, device="cuda") for n, a in x.items()}
    o_full, ht_full = chunk_gated_delta_rule(dev["q"], dev["k"], dev["v"], dev["g"], dev["beta"],
                                             output_final_state=True)
    cut = 70
    seg = [{n: t[:, a:b].contiguous() for n, t in dev.items()} for a, b in ((0, cut), (cut, T))]
    o1, c1 = chunk_gated_delta_rule(seg[0]["q"], seg[0]["k"], seg[0]["v"], seg[0]["g"], seg[0]["beta"],
                                    output_final_state=True)
    o2, c2 = chunk_gated_delta_rule(seg[1]["q"], seg[1]["k"], seg[1]["v"], seg[1]["g"], seg[1]["beta"],
                                    output_final_state=True)
    M2 = seqsplit.segment_transition(seg[1]["k"], seg[1]["g"], seg[1]["beta"])
    s_out = seqsplit.combine(M2, c2, c1)
    assert_rms_close(to_np(s_out), to_np(ht_full), 1e-4, "combined final state")
    seqsplit.apply_incoming_state(seg[1]["q"], seg[1]["k"], seg[1]["g"], seg[1]["beta"], c1, o2, d ** -0.5)
    assert_rms_close(to_np(torch.cat([o1, o2], 1)), to_np(o_full), 1e-4, "o")
