"""Regenerate the GatedDeltaNet layer fixtures (``layer_*.npz``) from the reference layer.

Run in a checkout that has the soreRNN reference importable:

    python tests/golden/make_layer_golden.py --reference <path to soreRNN checkout>

Each case builds the reference's own ``GatedDeltaNet`` (sore/model/gdn.py:92-135) with its pure-PyTorch
backend (``gdn_backend="torch"``: causal conv of sore/model/conv.py, the gated delta rule of
sore/model/gdn_ref.py, RMSNorm(o) * silu(gate)), loads the seeded weights of ``layer_inputs.py``, and runs
forward + backward in fp64 on CPU against a seeded cotangent, with the document boundaries of the
reference's own layer test matrix (tests/model/test_gdn.py:119: documents of 1-3 tokens, or one
document). Stored: the output, the input gradient, and every parameter gradient at the sampled indices of
``grad_sample_indices`` (all elements for the small ones). Weights and inputs are not stored; the tests
regenerate them from the seeds in the file. The test suite never imports the reference.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

sys.path.insert(0, str(Path(__file__).resolve().parent))
from layer_inputs import grad_sample_indices, layer_io, layer_weights  # noqa: E402

HERE = Path(__file__).resolve().parent
T = 256
D_MODEL = 128
CU = {"short_docs": [0, 1, 3, 4, 70, 200, 256], "one_doc": [0, 256]}
# (name, head_dim, qk heads, v heads, document case): head_dim 64 is the reference test's tiny preset;
# head_dim 128 is the head size of the chunked kernels
CASES = [
    ("hd64_rep1_short_docs", 64, 2, 2, "short_docs"),
    ("hd64_rep2_short_docs", 64, 2, 4, "short_docs"),
    ("hd64_rep1_one_doc", 64, 2, 2, "one_doc"),
    ("hd64_rep2_one_doc", 64, 2, 4, "one_doc"),
    ("hd128_rep1_short_docs", 128, 2, 2, "short_docs"),
    ("hd128_rep2_short_docs", 128, 2, 4, "short_docs"),
]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="soreRNN checkout that contains sore/model/gdn.py")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import torch

    from sore.model.config import get_preset
    from sore.model.gdn import GatedDeltaNet

    for i, (name, hd, hqk, hv, cu_case) in enumerate(CASES):
        wseed, xseed = 100 + i, 200 + i
        cfg = get_preset("tiny", gdn_backend="torch", gdn_qk_heads=hqk, gdn_v_heads=hv, gdn_head_dim=hd)
        layer = GatedDeltaNet(cfg).double()
        w = layer_weights(wseed, D_MODEL, hqk, hv, hd, cfg.conv_kernel)
        sd = layer.state_dict()
        assert set(sd) == set(w), (sorted(sd), sorted(w))
        layer.load_state_dict({n: torch.tensor(a, dtype=torch.float64) for n, a in w.items()})
        x_np, cot_np = layer_io(xseed, T, D_MODEL)
        x = torch.tensor(x_np, dtype=torch.float64, requires_grad=True)
        cu = torch.tensor(CU[cu_case], dtype=torch.long)
        out = layer(x, cu_seqlens=cu)
        (out * torch.tensor(cot_np, dtype=torch.float64)).sum().backward()
        rec = dict(wseed=wseed, xseed=xseed, head_dim=hd, qk_heads=hqk, v_heads=hv, d_model=D_MODEL, T=T,
                   conv_kernel=cfg.conv_kernel, norm_eps=cfg.norm_eps, cu=np.array(CU[cu_case]),
                   out=out.detach().numpy().astype(np.float32), gx=x.grad.numpy().astype(np.float32),
                   param_names=np.array(sorted(w)))
        for j, pn in enumerate(sorted(w)):
            g = dict(layer.named_parameters())[pn].grad.numpy().reshape(-1)
            idx = grad_sample_indices(1000 + j, g.size)
            rec["g_" + pn] = g[idx].astype(np.float32)
            rec["gmax_" + pn] = np.float64(np.abs(g).max())
        np.savez_compressed(HERE / f"layer_{name}.npz", **rec)
        print(name, "out max", float(np.abs(rec["out"]).max()))


if __name__ == "__main__":
    main()
