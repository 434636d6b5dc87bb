"""Layer-level parity of ``sorernn_b200.layer.GatedDeltaNet`` against the reference's own layer.

The expected values are the reference ``GatedDeltaNet`` (sore/model/gdn.py, pure-PyTorch backend) run in
fp64 by ``tests/golden/make_layer_golden.py`` on the seeded weights and inputs of
``tests/golden/layer_inputs.py``, with the document boundaries of the reference's own matrix test
(tests/model/test_gdn.py:104-162: documents of 1-3 tokens, or one document; GVA 1x and 2x). Here the same
weights are loaded into this package's layer, whose every step between the projections is one of this
package's CUDA kernels, and output, input gradient and every parameter gradient are compared:

* fp32 (head size 64, the reference test's preset): the reference test's own bars (output atol 1e-3;
  gradients rtol 1e-2 with atol 5e-3 x max|ref|, 5e-2 x max|ref| for A_log and dt_bias), for each option
  set of this layer (in-kernel gate, fused norm-gate, both, neither);
* bf16 autocast (head size 128: the chunked tcgen05 kernels): max-abs error <= 5e-2 x max|ref| and
  RMS error <= 2e-2 x RMS(ref) for the output and every gradient (bf16 projections and activations against
  an fp64 reference);
* document isolation: perturbing earlier documents leaves later outputs bit-identical, with the reference
  test's negative control (without cu_seqlens the same check must see the change;
  tests/model/test_gdn.py:165-193), and packed == separate.
"""
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
from layer_inputs import grad_sample_indices, layer_io, layer_weights  # noqa: E402

pytestmark = pytest.mark.gpu
OPTION_SETS = {"none": dict(kernel_gate=False, fused_norm_gate=False),
               "kernel_gate": dict(kernel_gate=True, fused_norm_gate=False),
               "fused_norm_gate": dict(kernel_gate=False, fused_norm_gate=True),
               "all": dict(kernel_gate=True, fused_norm_gate=True)}


def _fixture(name):
    return np.load(GOLDEN / f"layer_{name}.npz")


def _layer(fx, **options):
    from sorernn_b200.layer import GatedDeltaNet

    d, hqk, hv, hd = int(fx["d_model"]), int(fx["qk_heads"]), int(fx["v_heads"]), int(fx["head_dim"])
    layer = GatedDeltaNet(d, hqk, hv, hd, int(fx["conv_kernel"]), float(fx["norm_eps"]), **options)
    w = layer_weights(int(fx["wseed"]), d, hqk, hv, hd, int(fx["conv_kernel"]))
    layer.load_state_dict({n: torch.tensor(a, dtype=torch.float32) for n, a in w.items()})
    return layer.cuda()


def _run(layer, fx, bf16=False):
    x_np, cot_np = layer_io(int(fx["xseed"]), int(fx["T"]), int(fx["d_model"]))
    x = torch.tensor(x_np, dtype=torch.float32, device="cuda", requires_grad=True)
    cot = torch.tensor(cot_np, dtype=torch.float32, device="cuda")
    cu = torch.tensor(fx["cu"], dtype=torch.int64)
    with torch.autocast("cuda", dtype=torch.bfloat16, enabled=bf16):
        out = layer(x, cu_seqlens=cu.cuda(), cu_seqlens_cpu=cu)
    (out.float() * cot).sum().backward()
    torch.cuda.synchronize()
    grads = {n: p.grad.detach().float().cpu().numpy().reshape(-1) for n, p in layer.named_parameters()}
    return out.detach().float().cpu().numpy(), x.grad.float().cpu().numpy(), grads


def _check_grads(fx, gx, grads, tol_fn):
    """Every parameter gradient at the stored sample indices, and the input gradient in full."""
    tol_fn("x", gx, fx["gx"], float(np.abs(fx["gx"]).max()))
    for j, pn in enumerate(fx["param_names"]):
        g = grads[str(pn)]
        idx = grad_sample_indices(1000 + j, g.size)
        tol_fn(str(pn), g[idx], fx["g_" + str(pn)], float(fx["gmax_" + str(pn)]))


@pytest.mark.parametrize("option_set", sorted(OPTION_SETS))
@pytest.mark.parametrize("case", ["hd64_rep1_short_docs", "hd64_rep2_short_docs", "hd64_rep1_one_doc",
                                  "hd64_rep2_one_doc"])
def test_layer_matches_reference_fp32(case, option_set):
    fx = _fixture(case)
    out, gx, grads = _run(_layer(fx, **OPTION_SETS[option_set]), fx)
    torch.testing.assert_close(torch.tensor(out), torch.tensor(fx["out"]), atol=1e-3, rtol=0)

    def tol(name, a, r, rmax):
        atol = (5e-2 if name in ("A_log", "dt_bias") else 5e-3) * rmax
        torch.testing.assert_close(torch.tensor(a), torch.tensor(r), rtol=1e-2, atol=atol,
                                   msg=lambda m, n=name: f"{n}: {m}")

    _check_grads(fx, gx, grads, tol)


@pytest.mark.parametrize("option_set", ["all", "none"])
@pytest.mark.parametrize("case", ["hd128_rep1_short_docs", "hd128_rep2_short_docs"])
def test_layer_bf16_chunked_matches_reference(case, option_set):
    """bf16 autocast with head size 128: the chunked tcgen05 kernels run the mixer."""
    from helpers import PARITY_LOG

    fx = _fixture(case)
    out, gx, grads = _run(_layer(fx, **OPTION_SETS[option_set]), fx, bf16=True)

    def tol(name, a, r, rmax):
        a, r = np.asarray(a, np.float64), np.asarray(r, np.float64)
        err = np.abs(a - r)
        rms_r = max(float(np.sqrt((r * r).mean())), 1e-30)
        PARITY_LOG.append((f"layer {name}", float(err.max() / max(rmax, 1e-30)), None, 5e-2, case))
        assert err.max() <= 5e-2 * rmax, f"{name}: max err {err.max():.3e} > 5e-2 x max|ref| {rmax:.3e}"
        assert np.sqrt((err * err).mean()) <= 2e-2 * rms_r, f"{name}: RMS err above 2e-2 x RMS(ref)"

    tol("out", out, fx["out"], float(np.abs(fx["out"]).max()))
    _check_grads(fx, gx, grads, tol)


@pytest.mark.parametrize("option_set", ["all", "none"])
@pytest.mark.parametrize("case", ["hd64_rep2_short_docs", "hd128_rep1_short_docs"])
def test_layer_isolates_documents(case, option_set):
    """Perturbing earlier documents (the 1-3-token ones, then [4, 70)) leaves every later output
    bit-identical; the same check without cu_seqlens (no resets) must see the change."""
    fx = _fixture(case)
    layer = _layer(fx, **OPTION_SETS[option_set])
    T, d = int(fx["T"]), int(fx["d_model"])
    cu = torch.tensor(fx["cu"], dtype=torch.int64)
    gen = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn(1, T, d, device="cuda", generator=gen)
    bf16 = int(fx["head_dim"]) == 128

    def run(inp, packed=True):
        with torch.no_grad(), torch.autocast("cuda", dtype=torch.bfloat16, enabled=bf16):
            return (layer(inp, cu_seqlens=cu.cuda(), cu_seqlens_cpu=cu) if packed else layer(inp)).float()

    out = run(x)
    for start, end, first_unchanged in ((0, 4, 4), (4, 70, 70)):
        x2 = x.clone()
        x2[:, start:end] = torch.randn(1, end - start, d, device="cuda", generator=gen)
        out2 = run(x2)
        assert torch.equal(out[:, first_unchanged:], out2[:, first_unchanged:])
        assert not torch.allclose(out[:, start:end], out2[:, start:end], atol=1e-3)
        leak, leak2 = run(x, packed=False), run(x2, packed=False)
        assert (leak[:, first_unchanged:] - leak2[:, first_unchanged:]).abs().max() > 1e-3


def test_layer_packed_equals_separate():
    """One packed batch with cu_seqlens equals each document run on its own (fp32, bitwise up to 1e-5)."""
    fx = _fixture("hd64_rep2_short_docs")
    layer = _layer(fx, **OPTION_SETS["all"])
    d = int(fx["d_model"])
    x = torch.randn(1, 90, d, device="cuda", generator=torch.Generator(device="cuda").manual_seed(4))
    cu = torch.tensor([0, 7, 90], dtype=torch.int64)
    with torch.no_grad():
        packed = layer(x, cu_seqlens=cu.cuda(), cu_seqlens_cpu=cu)
        separate = torch.cat([layer(x[:, :7].contiguous()), layer(x[:, 7:].contiguous())], dim=1)
        unpacked = layer(x)
    torch.testing.assert_close(packed, separate, atol=1e-5, rtol=0)
    assert not torch.allclose(unpacked[:, 7:], separate[:, 7:], atol=1e-3)
