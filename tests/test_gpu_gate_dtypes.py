"""The chunk kernels and the decode kernel read g and beta in any of fp32, bf16 and fp16 (the kernels keep
the loaded bits and convert at use). Values exactly representable in the narrower dtype must give
bitwise the same outputs, dq, dk and dv as their fp32 copies: the conversion is the only difference.
dg and dbeta come back rounded to the gates' own dtypes; they are compared within one ulp of that dtype
plus 1e-5 x RMS."""
import pytest
import torch

pytestmark = pytest.mark.gpu
D = 128


def _inputs(seed, B=2, T=200, H=2, HV=2):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = {n: torch.randn(B, T, h, D, device="cuda", generator=g).bfloat16()
         for n, h in (("q", H), ("k", H), ("v", HV), ("do", HV))}
    x["g"] = torch.nn.functional.logsigmoid(torch.randn(B, T, HV, device="cuda", generator=g)) / 16
    x["beta"] = torch.sigmoid(torch.randn(B, T, HV, device="cuda", generator=g))
    return x


@pytest.mark.parametrize("g_dtype,b_dtype", [(torch.bfloat16, torch.float32), (torch.float16, torch.float16),
                                             (torch.float32, torch.bfloat16)])
def test_chunk_gate_dtypes_match_fp32_copies(g_dtype, b_dtype):
    from sorernn_b200 import chunk_gated_delta_rule

    x = _inputs(11)
    g_n, b_n = x["g"].to(g_dtype), x["beta"].to(b_dtype)  # the narrow-dtype values
    runs = []
    for g_in, b_in in ((g_n, b_n), (g_n.float(), b_n.float())):  # same values, fp32 storage
        leaves = {n: x[n].clone().requires_grad_(True) for n in ("q", "k", "v")}
        g_l, b_l = g_in.clone().requires_grad_(True), b_in.clone().requires_grad_(True)
        o, _ = chunk_gated_delta_rule(leaves["q"], leaves["k"], leaves["v"], g_l, b_l, use_qk_l2norm_in_kernel=True)
        o.backward(x["do"])
        runs.append((o.detach(), leaves["q"].grad, leaves["k"].grad, leaves["v"].grad, g_l.grad.float(),
                     b_l.grad.float()))
    torch.cuda.synchronize()
    for name, a, b in zip(("o", "dq", "dk", "dv"), runs[0], runs[1]):
        assert torch.equal(a, b), f"{name} differs between the {g_dtype}/{b_dtype} gates and their fp32 copies"
    # dg, dbeta come back in the gates' dtypes
    ulp = {torch.float32: 0.0, torch.bfloat16: 2.0 ** -7, torch.float16: 2.0 ** -10}
    for name, a, b, dt in (("dg", runs[0][4], runs[1][4], g_dtype), ("dbeta", runs[0][5], runs[1][5], b_dtype)):
        excess = ((a - b).abs() - ulp[dt] * b.abs()).max().item()
        assert excess <= 1e-5 * b.pow(2).mean().sqrt().item(), f"{name}: {excess:.3e}"


@pytest.mark.parametrize("g_dtype,b_dtype", [(torch.bfloat16, torch.float32), (torch.float16, torch.float16)])
def test_decode_gate_dtypes_match_fp32_copies(g_dtype, b_dtype):
    from sorernn_b200 import fused_recurrent_gated_delta_rule_step

    g = torch.Generator(device="cuda").manual_seed(5)
    N, H = 300, 4  # more heads than SMs: the persistent kernel walks several heads per CTA
    q, k, v = (torch.randn(N, H, D, device="cuda", generator=g).bfloat16() for _ in range(3))
    gg = (torch.nn.functional.logsigmoid(torch.randn(N, H, device="cuda", generator=g)) / 16).to(g_dtype)
    bb = torch.sigmoid(torch.randn(N, H, device="cuda", generator=g)).to(b_dtype)
    s0 = torch.randn(N, H, D, D, device="cuda", generator=g) * 0.05
    outs = []
    for g_in, b_in in ((gg, bb), (gg.float(), bb.float())):
        st = s0.clone()
        o = fused_recurrent_gated_delta_rule_step(q, k, v, g_in, b_in, st, use_qk_l2norm_in_kernel=True)
        outs.append((o, st))
    torch.cuda.synchronize()
    assert torch.equal(outs[0][0], outs[1][0]), "o"
    assert torch.equal(outs[0][1], outs[1][1]), "state"
