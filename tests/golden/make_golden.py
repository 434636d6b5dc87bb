"""Regenerate the golden fixtures in this folder from the reference implementation.

Run in a checkout that has the soreRNN reference importable (its ``sore`` package on ``sys.path``,
passed with ``--reference``) and, for the initial-state case, flash-linear-attention installed:

    python tests/golden/make_golden.py --reference <path to soreRNN checkout>

Every case draws its inputs with numpy's PCG64 generator (stable across numpy versions), runs the
reference's own ``naive_gated_delta_rule`` (``sore/model/gdn_ref.py:25``) in fp64 on CPU, and takes
gradients with torch autograd against a seeded cotangent. Layer-level cases reproduce the torch
backend's call sequence of ``GatedDeltaNet.forward`` (``sore/model/gdn.py:170-178``): GVA
``repeat_interleave`` then ``F.normalize`` then the oracle. The ``initial_state`` case is pinned on
flash-linear-attention's ``naive_recurrent_gated_delta_rule`` (FLA 0.5.x, a pure-PyTorch function),
because the reference oracle always starts from a zero state.

The inputs are not stored: ``inputs.py`` regenerates them from the seeds in ``golden.json``. The test
suite never imports the reference; it only reads the files written here.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

sys.path.insert(0, str(Path(__file__).resolve().parent))
from inputs import make_inputs, make_state_inputs  # noqa: E402

HERE = Path(__file__).resolve().parent


def _ref_run(ref, inp, scale, cu=None, l2norm=False, rep=1):
    import torch
    import torch.nn.functional as F

    t = {n: torch.tensor(a, dtype=torch.float64, requires_grad=(n != "do")) for n, a in inp.items()}
    q, k = t["q"], t["k"]
    if rep > 1:  # gdn.py:171-174
        q, k = q.repeat_interleave(rep, dim=2), k.repeat_interleave(rep, dim=2)
    if l2norm:  # gdn.py:177
        q, k = F.normalize(q, dim=-1), F.normalize(k, dim=-1)
    cu_t = None if cu is None else torch.tensor(cu, dtype=torch.long)
    o = ref(q, k, t["v"], t["g"], t["beta"], scale=scale, cu_seqlens=cu_t)
    (o * t["do"]).sum().backward()
    out = dict(o=o.detach().numpy())
    for n in ("q", "k", "v", "g", "beta"):
        out["d" + n] = t[n].grad.numpy()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="soreRNN checkout that contains sore/model/gdn_ref.py")
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    import torch
    from sore.model.gdn_ref import naive_gated_delta_rule as ref

    torch.set_num_threads(8)
    cases = {
        # name: (seed, B, T, H, HV, dk, dv, cu, l2norm, g_mode)
        "t1_closed_form": (11, 2, 1, 2, 2, 8, 6, None, False, "uniform"),
        "t2_op_order": (12, 1, 2, 2, 2, 8, 6, None, False, "uniform"),
        "chunk_cross": (13, 2, 130, 1, 1, 16, 16, None, False, "logsigmoid16"),
        "varlen_short_docs": (14, 1, 200, 2, 2, 16, 16, [0, 1, 3, 4, 70, 200], False, "logsigmoid16"),
        "gva2_l2norm": (15, 1, 70, 1, 2, 16, 16, None, True, "logsigmoid16"),
        "varlen_gva2_l2norm": (16, 1, 150, 2, 4, 16, 8, [0, 1, 2, 100, 150], True, "uniform"),
    }
    meta = {}
    for name, (seed, B, T, H, HV, dk, dv, cu, l2, gm) in cases.items():
        inp = make_inputs(seed, B, T, H, HV, dk, dv, normalized=not l2, g_mode=gm)
        scale = dk ** -0.5
        out = _ref_run(ref, inp, scale, cu=cu, l2norm=l2, rep=HV // H)
        np.savez_compressed(HERE / f"{name}.npz", **out)
        meta[name] = dict(seed=seed, B=B, T=T, H=H, HV=HV, dk=dk, dv=dv, cu=cu, l2norm=l2,
                          g_mode=gm, scale=scale, source="sore/model/gdn_ref.py:25 (fp64, autograd)")

    # initial/final state: FLA's naive recurrent function (the reference never seeds a state)
    from fla.ops.gated_delta_rule.naive import naive_recurrent_gated_delta_rule as fla_naive

    seed, B, T, H, dk, dv = 17, 2, 40, 2, 16, 16
    inp = make_inputs(seed, B, T, H, H, dk, dv)
    h0, dht = make_state_inputs(seed, B, H, dk, dv)
    t = {n: torch.tensor(a, dtype=torch.float64, requires_grad=(n != "do")) for n, a in inp.items()}
    h0_t = torch.tensor(h0, requires_grad=True)
    o, ht = fla_naive(t["q"], t["k"], t["v"], t["beta"], t["g"], scale=dk ** -0.5,
                      initial_state=h0_t, output_final_state=True)
    ((o * t["do"]).sum() + (ht * torch.tensor(dht)).sum()).backward()
    out = dict(o=o.detach().numpy(), ht=ht.detach().numpy(), dh0=h0_t.grad.numpy())
    for n in ("q", "k", "v", "g", "beta"):
        out["d" + n] = t[n].grad.numpy()
    np.savez_compressed(HERE / "initial_state.npz", **out)
    meta["initial_state"] = dict(seed=seed, B=B, T=T, H=H, HV=H, dk=dk, dv=dv, cu=None, l2norm=False,
                                 g_mode="logsigmoid16", scale=dk ** -0.5,
                                 source="fla naive_recurrent_gated_delta_rule (secondary pin, FLA 0.5.1)")

    # config 0 (B2 T256 H4 d64 fp32): too large to store; keep a checksum of every output
    seed = 0
    B, T, H, d = 2, 256, 4, 64
    inp = make_inputs(seed, B, T, H, H, d, d)
    inp32 = {n: a.astype(np.float32) for n, a in inp.items()}
    tt = {n: torch.tensor(a, requires_grad=(n != "do")) for n, a in inp32.items()}
    o = ref(tt["q"], tt["k"], tt["v"], tt["g"], tt["beta"], scale=d ** -0.5)
    (o * tt["do"]).sum().backward()
    outs = dict(o=o.detach().numpy(), **{"d" + n: tt[n].grad.numpy() for n in ("q", "k", "v", "g", "beta")})
    idx_rng = np.random.default_rng(1234)
    summary = {}
    for n, a in outs.items():
        flat = a.reshape(-1).astype(np.float64)
        pick = idx_rng.integers(0, flat.size, 64)
        summary[n] = dict(sum=float(flat.sum()), sumsq=float((flat * flat).sum()),
                          absmax=float(np.abs(flat).max()), idx=pick.tolist(), val=flat[pick].tolist())
    meta["config0_checksum"] = dict(seed=seed, B=B, T=T, H=H, HV=H, dk=d, dv=d, dtype="float32",
                                    scale=d ** -0.5, source="sore/model/gdn_ref.py:25 (fp32, autograd)",
                                    outputs=summary)
    (HERE / "golden.json").write_text(json.dumps(meta, indent=1))
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")))


if __name__ == "__main__":
    main()
