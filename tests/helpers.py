"""Shared test helpers: the north-star tolerance metric and device-side input builders."""
import numpy as np


# Every parity comparison made in this process: (output name, strict max-abs/RMS, error beyond the bf16
# output rounding / RMS or None for fp32 outputs, bar). conftest.py prints the worst per output at the end
# of the run, so the log shows how far each output is from the literal north-star bar and from the bar
# applied beyond rounding.
PARITY_LOG = []
CURRENT_TEST = [""]  # node id of the running test (set by conftest.py)


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
    PARITY_LOG.append((name, err / max(rms(r), 1e-30), None, tol, CURRENT_TEST[0]))
    assert err <= bound, f"{name}: max abs err {err:.3e} > {tol} * RMS(ref) = {bound:.3e}"
    return err / max(rms(r), 1e-30)


def to_np(t):
    return t.detach().float().cpu().numpy()


def assert_bf16_close(actual, ref, tol, name=""):
    """Parity bar for a bf16 output: the error beyond the output's own rounding (half an ulp of a bf16,
    at most 2^-8 |ref|, which the reference's fp32 -> bf16 cast at gdn_ref.py:52 carries too) is at most
    tol x RMS(ref). Returns (strict max-abs/RMS, excess/RMS) for reporting."""
    a = np.asarray(actual, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    assert a.shape == r.shape, f"{name}: shape {a.shape} != {r.shape}"
    assert np.isfinite(a).all(), f"{name}: non-finite values"
    rr = max(rms(r), 1e-30)
    err = np.abs(a - r)
    excess = float((err - 2.0 ** -8 * np.abs(r)).max()) if a.size else 0.0
    PARITY_LOG.append((name, float(err.max() / rr) if a.size else 0.0, excess / rr, tol, CURRENT_TEST[0]))
    assert excess <= tol * rr, (f"{name}: error beyond bf16 output rounding {excess:.3e} > {tol} * RMS(ref) = "
                                f"{tol * rr:.3e} (strict max-abs/RMS {err.max() / rr:.4f})")
    return float(err.max() / rr), excess / rr
