"""pytest configuration: the ``gpu`` marker and shared fixtures/helpers."""
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests" / "golden"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a) and the built extension")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    """Worst parity figure per output over the run: the strict max-abs/RMS beside the error beyond the
    bf16 output rounding (the figure the bf16 bars are applied to); fp32 outputs show the strict one only."""
    from helpers import PARITY_LOG

    if not PARITY_LOG:
        return
    worst = {}
    for name, strict, excess, tol, test in PARITY_LOG:
        w = worst.setdefault(name, [0.0, None, tol, 0, ""])
        key = strict if excess is None else excess
        prev = w[0] if w[1] is None else w[1]
        if w[3] == 0 or key >= prev:
            w[4] = test
        w[0] = max(w[0], strict)
        if excess is not None:
            w[1] = excess if w[1] is None else max(w[1], excess)
        w[2] = max(w[2], tol)
        w[3] += 1
    tr = terminalreporter
    tr.write_sep("-", "parity: worst max-abs error / RMS(reference) per output")
    tr.write_line(f"{'output':<16}{'checks':>8}{'strict':>12}{'beyond bf16 rounding':>24}{'bar':>8}  worst in")
    for name in sorted(worst):
        strict, excess, tol, n, test = worst[name]
        ex = "-" if excess is None else f"{excess:.4f}"
        tr.write_line(f"{name:<16}{n:>8}{strict:>12.4f}{ex:>24}{tol:>8}  {test.split('::')[-1]}")


@pytest.fixture(autouse=True)
def _record_test_name(request):
    from helpers import CURRENT_TEST

    CURRENT_TEST[0] = request.node.nodeid
    yield
