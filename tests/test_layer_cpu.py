"""CPU checks of the layer drop-in: its state_dict has exactly the reference layer's parameter names and
shapes (as recorded in the fixtures made from the reference), so the reference's checkpoints load."""
import sys
from pathlib import Path

import numpy as np
import pytest

GOLDEN = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLDEN))
from layer_inputs import layer_weights  # noqa: E402


@pytest.mark.parametrize("case", ["hd64_rep2_short_docs", "hd128_rep1_short_docs"])
def test_state_dict_matches_reference_layout(case):
    import torch

    from sorernn_b200.layer import GatedDeltaNet

    fx = np.load(GOLDEN / f"layer_{case}.npz")
    d, hqk, hv, hd = int(fx["d_model"]), int(fx["qk_heads"]), int(fx["v_heads"]), int(fx["head_dim"])
    layer = GatedDeltaNet(d, hqk, hv, hd, int(fx["conv_kernel"]), float(fx["norm_eps"]))
    sd = layer.state_dict()
    assert sorted(sd) == sorted(str(n) for n in fx["param_names"])
    w = layer_weights(int(fx["wseed"]), d, hqk, hv, hd, int(fx["conv_kernel"]))
    assert all(tuple(sd[n].shape) == w[n].shape for n in w)
    layer.load_state_dict({n: torch.tensor(a, dtype=torch.float32) for n, a in w.items()})


def test_layer_refuses_cpu_tensors():
    import torch

    from sorernn_b200.layer import GatedDeltaNet

    layer = GatedDeltaNet(64, 1, 2, 64)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        layer(torch.randn(1, 8, 64))
