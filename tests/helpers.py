"""Shared test helpers: the north-star tolerance metric and device-side input builders."""
import numpy as np


def rms(x) -> float:
    x = np.asarray(x, dtype=np.float64)
    return float(np.sqrt((x * x).mean())) if x.size else 0.0


def assert_rms_close(actual, ref, tol, name=""):
    """max|actual - ref| <= tol * RMS(ref): the parity bar (fp32 1e-4, bf16 2e-2, bf16 grads 3e-2)."""
    a = np.asarray(actual, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    assert a.shape == r.shape, f"{name}: shape {a.shape} != {r.shape}"
    err = float(np.abs(a - r).max()) if a.size else 0.0
    bound = tol * max(rms(r), 1e-30)
    assert np.isfinite(a).all(), f"{name}: non-finite values"
    assert err <= bound, f"{name}: max abs err {err:.3e} > {tol} * RMS(ref) = {bound:.3e}"
    return err / max(rms(r), 1e-30)


def to_np(t):
    return t.detach().float().cpu().numpy()
