"""Pins the CPU oracle (``oracle/gdn_oracle.py``) to outputs of the reference itself.

The fixtures in ``tests/golden`` were produced by ``tests/golden/make_golden.py`` from soreRNN's
``naive_gated_delta_rule`` (sore/model/gdn_ref.py:25) with torch autograd, and, for the seeded
initial state, from flash-linear-attention's ``naive_recurrent_gated_delta_rule``.
"""
import json
from pathlib import Path

import numpy as np
import pytest

from inputs import make_inputs, make_state_inputs
from oracle import gdn_oracle as orc

GOLD = Path(__file__).resolve().parent / "golden"
META = json.loads((GOLD / "golden.json").read_text())
CASES = [n for n in META if n not in ("config0_checksum", "initial_state")]


def _case(name):
    m = META[name]
    inp = make_inputs(m["seed"], m["B"], m["T"], m["H"], m["HV"], m["dk"], m["dv"],
                      normalized=not m["l2norm"], g_mode=m["g_mode"])
    return m, inp, dict(np.load(GOLD / f"{name}.npz"))


@pytest.mark.parametrize("name", CASES)
def test_oracle_forward_matches_reference(name):
    m, x, ref = _case(name)
    o, _ = orc.gdn_forward(x["q"], x["k"], x["v"], x["g"], x["beta"], m["scale"], cu_seqlens=m["cu"],
                           use_qk_l2norm=m["l2norm"])
    np.testing.assert_allclose(o, ref["o"], atol=1e-12, rtol=0)


@pytest.mark.parametrize("name", CASES)
def test_oracle_backward_matches_reference_autograd(name):
    m, x, ref = _case(name)
    dq, dk, dv, dg, db, _ = orc.gdn_backward(x["q"], x["k"], x["v"], x["g"], x["beta"], x["do"], m["scale"],
                                             cu_seqlens=m["cu"], use_qk_l2norm=m["l2norm"])
    for n, a in dict(dq=dq, dk=dk, dv=dv, dg=dg, dbeta=db).items():
        np.testing.assert_allclose(a, ref[n], atol=1e-11, rtol=0, err_msg=n)


def test_oracle_initial_state_matches_fla_naive():
    m = META["initial_state"]
    x = make_inputs(m["seed"], m["B"], m["T"], m["H"], m["HV"], m["dk"], m["dv"])
    h0, dht = make_state_inputs(m["seed"], m["B"], m["HV"], m["dk"], m["dv"])
    ref = dict(np.load(GOLD / "initial_state.npz"))
    # FLA's naive function computes in fp32 internally, so this pin is at fp32 rounding level.
    o, ht = orc.gdn_forward(x["q"], x["k"], x["v"], x["g"], x["beta"], m["scale"], initial_state=h0)
    np.testing.assert_allclose(o, ref["o"], atol=1e-6 * np.abs(ref["o"]).max(), rtol=0)
    np.testing.assert_allclose(ht, ref["ht"], atol=1e-6 * np.abs(ref["ht"]).max(), rtol=0)
    dq, dk, dv, dg, db, dh0 = orc.gdn_backward(x["q"], x["k"], x["v"], x["g"], x["beta"], x["do"], m["scale"],
                                               initial_state=h0, dht=dht)
    for n, a in dict(dq=dq, dk=dk, dv=dv, dg=dg, dbeta=db, dh0=dh0).items():
        np.testing.assert_allclose(a, ref[n], atol=1e-6 * np.abs(ref[n]).max(), rtol=0, err_msg=n)


def test_oracle_config0_checksum():
    m = META["config0_checksum"]
    x = {n: a.astype(np.float32) for n, a in
         make_inputs(m["seed"], m["B"], m["T"], m["H"], m["HV"], m["dk"], m["dv"]).items()}
    o, _ = orc.gdn_forward(x["q"], x["k"], x["v"], x["g"], x["beta"], m["scale"])
    dq, dk, dv, dg, db, _ = orc.gdn_backward(x["q"], x["k"], x["v"], x["g"], x["beta"], x["do"], m["scale"])
    outs = dict(o=o, dq=dq, dk=dk, dv=dv, dg=dg, dbeta=db)
    for n, s in m["outputs"].items():
        flat = outs[n].reshape(-1).astype(np.float64)
        tol = 2e-5 * s["absmax"]  # both sides are fp32 (different summation orders)
        np.testing.assert_allclose(flat[s["idx"]], s["val"], atol=tol, rtol=0, err_msg=n)
        assert abs(np.sqrt((flat * flat).sum()) - np.sqrt(s["sumsq"])) <= 1e-5 * np.sqrt(s["sumsq"]), n


def test_decode_step_equals_one_token_of_forward():
    x = make_inputs(5, 3, 1, 2, 4, 16, 8)
    h0, _ = make_state_inputs(5, 3, 4, 16, 8)
    o_ref, ht = orc.gdn_forward(x["q"], x["k"], x["v"], x["g"], x["beta"], 0.25, initial_state=h0)
    st = h0.copy()
    o = orc.gdn_decode_step(x["q"][:, 0], x["k"][:, 0], x["v"][:, 0], x["g"][:, 0], x["beta"][:, 0], st, 0.25)
    np.testing.assert_allclose(o, o_ref[:, 0], atol=1e-13)
    np.testing.assert_allclose(st, ht, atol=1e-13)


def test_validation_errors_match_reference():
    x = make_inputs(1, 2, 6, 1, 1, 4, 4)
    with pytest.raises(ValueError, match="B == 1"):
        orc.gdn_forward(x["q"], x["k"], x["v"], x["g"], x["beta"], 1.0, cu_seqlens=[0, 3, 6])
    x = make_inputs(1, 1, 6, 1, 1, 4, 4)
    with pytest.raises(ValueError, match="cu_seqlens"):
        orc.gdn_forward(x["q"], x["k"], x["v"], x["g"], x["beta"], 1.0, cu_seqlens=[0, 3, 5])


@pytest.mark.parametrize("name", CASES + ["initial_state"])
def test_c_oracle_matches_numpy_oracle(name):
    from oracle import cgdn

    m = META[name]
    x = make_inputs(m["seed"], m["B"], m["T"], m["H"], m["HV"], m["dk"], m["dv"],
                    normalized=not m["l2norm"], g_mode=m["g_mode"])
    h0 = dht = None
    if name == "initial_state":
        h0, dht = make_state_inputs(m["seed"], m["B"], m["HV"], m["dk"], m["dv"])
    kw = dict(cu_seqlens=m["cu"], use_qk_l2norm=m["l2norm"])
    o, ht = orc.gdn_forward(x["q"], x["k"], x["v"], x["g"], x["beta"], m["scale"], initial_state=h0, **kw)
    o_c, ht_c = cgdn.forward(x["q"], x["k"], x["v"], x["g"], x["beta"], m["scale"], initial_state=h0, **kw)
    np.testing.assert_allclose(o_c, o, atol=2e-6 * max(1, np.abs(o).max()))
    np.testing.assert_allclose(ht_c, ht, atol=2e-6 * max(1, np.abs(ht).max()))
    ref = orc.gdn_backward(x["q"], x["k"], x["v"], x["g"], x["beta"], x["do"], m["scale"], initial_state=h0,
                           dht=dht, **kw)
    got = cgdn.backward(x["q"], x["k"], x["v"], x["g"], x["beta"], x["do"], m["scale"], initial_state=h0,
                        dht=dht, **kw)
    for n, a, b in zip(("dq", "dk", "dv", "dg", "dbeta", "dh0"), got, ref):
        np.testing.assert_allclose(a, b, atol=1e-5 * max(1, np.abs(b).max()), err_msg=n)


def test_c_oracle_decode_step():
    from oracle import cgdn

    x = make_inputs(5, 3, 1, 2, 4, 16, 8)
    h0, _ = make_state_inputs(5, 3, 4, 16, 8)
    st = h0.copy()
    o = orc.gdn_decode_step(x["q"][:, 0], x["k"][:, 0], x["v"][:, 0], x["g"][:, 0], x["beta"][:, 0], st, 0.25)
    st_c = h0.astype(np.float32)
    o_c = cgdn.decode_step(x["q"][:, 0], x["k"][:, 0], x["v"][:, 0], x["g"][:, 0], x["beta"][:, 0], st_c, 0.25)
    np.testing.assert_allclose(o_c, o, atol=1e-5)
    np.testing.assert_allclose(st_c, st, atol=1e-5)


def test_oracles_agree_on_empty_documents():
    """Zero-length documents: both restatements (numpy, C) keep h0 as the final state, pass dht through
    as dh0, and agree elsewhere."""
    from inputs import make_inputs, make_state_inputs
    from oracle import cgdn
    from oracle import gdn_oracle as orc

    cu = [0, 0, 5, 5, 17, 17]
    x = make_inputs(3, 1, 17, 1, 2, 8, 8)
    h0, dht = make_state_inputs(3, len(cu) - 1, 2, 8, 8)
    o_n, s_n = orc.gdn_forward(x["q"], x["k"], x["v"], x["g"], x["beta"], initial_state=h0, cu_seqlens=cu)
    o_c, s_c = cgdn.forward(x["q"], x["k"], x["v"], x["g"], x["beta"], 8 ** -0.5, initial_state=h0, cu_seqlens=cu)
    np.testing.assert_allclose(o_c, o_n, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(s_c, s_n, rtol=1e-5, atol=1e-6)
    for n in (0, 2, 4):
        np.testing.assert_allclose(s_n[n], h0[n])
    g_n = orc.gdn_backward(x["q"], x["k"], x["v"], x["g"], x["beta"], x["do"], initial_state=h0, dht=dht,
                           cu_seqlens=cu)
    g_c = cgdn.backward(x["q"], x["k"], x["v"], x["g"], x["beta"], x["do"], 8 ** -0.5, initial_state=h0, dht=dht,
                        cu_seqlens=cu)
    for a, b in zip(g_c, g_n):
        np.testing.assert_allclose(a, b, rtol=1e-4, atol=1e-5)
    for n in (0, 2, 4):
        np.testing.assert_allclose(g_n[5][n], dht[n])
