"""CPU checks of the piece decomposition behind sorernn_b200.pieces (no GPU): the forward and reverse scans
that join pieces, run on the oracle's per-piece results in fp64, reproduce the oracle's unsplit forward and
backward (outputs, final state and every gradient, h0 and dht included)."""
import numpy as np
import pytest
import torch

from oracle.gdn_oracle import gdn_backward, gdn_forward
from sorernn_b200.pieces import end_state_grads, incoming_states


def _case(seed, B, T, H, HV, d):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, T, H, d))
    k = rng.standard_normal((B, T, H, d))
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((B, T, HV, d))
    g = np.log(1 / (1 + np.exp(-rng.standard_normal((B, T, HV))))) / 16
    beta = 1 / (1 + np.exp(-rng.standard_normal((B, T, HV))))
    do = rng.standard_normal((B, T, HV, d))
    h0 = rng.standard_normal((B, HV, d, d)) * 0.1
    dht = rng.standard_normal((B, HV, d, d)) * 0.1
    return q, k, v, g, beta, do, h0, dht


def _pieces(x, P):
    B, T = x.shape[:2]
    return x.reshape(B * P, T // P, *x.shape[2:])


@pytest.mark.parametrize("P", [1, 2, 3, 5])
@pytest.mark.parametrize("with_state", [False, True])
def test_piece_scans_reproduce_the_unsplit_oracle(P, with_state):
    B, T, H, HV, d = 2, 30, 1, 2, 4
    q, k, v, g, beta, do, h0, dht = _case(P * 10 + with_state, B, T, H, HV, d)
    if not with_state:
        h0 = dht = None
    o_ref, s_ref = gdn_forward(q, k, v, g, beta, initial_state=h0)
    ref = gdn_backward(q, k, v, g, beta, do, initial_state=h0, dht=dht)

    qs, ks, vs, gs, bs, dos = (_pieces(x, P) for x in (q, k, v, g, beta, do))
    init = np.zeros((B, P, HV, d, d))
    if h0 is not None:
        init[:, 0] = h0
    init = init.reshape(B * P, HV, d, d)
    # every piece's map: C from its own start state (h0 for piece 0), M from the identity with v = 0
    _, C = gdn_forward(qs, ks, vs, gs, bs, initial_state=init)
    eye = np.broadcast_to(np.eye(d), (B * P, HV, d, d))
    _, M = gdn_forward(qs, ks, np.zeros_like(vs), gs, bs, initial_state=eye)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).reshape(B, P, *a.shape[1:])  # noqa: E731
    S_in, S_fin = incoming_states(t(M), t(C), None if h0 is None else torch.from_numpy(h0))
    S_in = S_in.reshape(B * P, HV, d, d).numpy()
    o, _ = gdn_forward(qs, ks, vs, gs, bs, initial_state=S_in)
    np.testing.assert_allclose(o.reshape(o_ref.shape), o_ref, atol=1e-12)
    np.testing.assert_allclose(S_fin.numpy(), s_ref, atol=1e-12)

    # backward: R from a zero end-state gradient, the reverse scan, then every piece from its true dS_end
    R = gdn_backward(qs, ks, vs, gs, bs, dos, initial_state=S_in)[5]
    MT = t(M).transpose(-1, -2)
    X = end_state_grads(MT, t(R), None if dht is None else torch.from_numpy(dht))
    got = gdn_backward(qs, ks, vs, gs, bs, dos, initial_state=S_in, dht=X.reshape(B * P, HV, d, d).numpy())
    for name, a, r in zip(("dq", "dk", "dv", "dg", "dbeta"), got[:5], ref[:5]):
        np.testing.assert_allclose(a.reshape(r.shape), r, atol=1e-11, err_msg=name)
    dh0 = got[5].reshape(B, P, HV, d, d)[:, 0]
    np.testing.assert_allclose(dh0, ref[5], atol=1e-11)


def test_end_state_grads_last_piece_is_dht():
    B, P, HV, d = 1, 4, 1, 3
    MT = torch.randn(B, P, HV, d, d, dtype=torch.float64)
    R = torch.randn(B, P, HV, d, d, dtype=torch.float64)
    dht = torch.randn(B, HV, d, d, dtype=torch.float64)
    X = end_state_grads(MT, R, dht)
    torch.testing.assert_close(X[:, P - 1], dht)
    for p in range(P - 1):  # the defining recurrence, one step at a time
        torch.testing.assert_close(X[:, p], MT[:, p + 1] @ X[:, p + 1] + R[:, p + 1])
