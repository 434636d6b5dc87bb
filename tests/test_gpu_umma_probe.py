"""GPU checks of the sm_100a building blocks (tcgen05.mma operand layouts, TMA swizzle) in isolation.

A wrong shared-memory descriptor or swizzle shows up here as a plain GEMM mismatch against torch,
before it can hide inside the chunk kernels.
"""
import ctypes
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
sys.path.insert(0, str(Path(__file__).resolve().parent / "csrc"))


@pytest.fixture(scope="module")
def probe():
    import build_probe

    lib = ctypes.CDLL(str(build_probe.build()))
    vp = ctypes.c_void_p
    lib.umma_probe.argtypes = [vp, vp, vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, vp, vp]
    lib.tma_probe.argtypes = [vp, ctypes.c_long, ctypes.c_long, ctypes.c_int, ctypes.c_int, ctypes.c_int, vp, vp, vp]
    lib.wait_timeout_probe.argtypes = [vp, vp, ctypes.c_uint, vp]
    return lib


@pytest.mark.parametrize("N", [64, 128])
@pytest.mark.parametrize("K", [64, 128])
@pytest.mark.parametrize("a_mn", [0, 1])
@pytest.mark.parametrize("b_mn", [0, 1])
def test_umma_layouts(probe, N, K, a_mn, b_mn):
    g = torch.Generator(device="cuda").manual_seed(N * 1000 + K + 10 * a_mn + b_mn)
    A = torch.randn(128, K, device="cuda", generator=g).bfloat16()
    B = torch.randn(N, K, device="cuda", generator=g).bfloat16()
    D = torch.empty(128, N, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = probe.umma_probe(A.data_ptr(), B.data_ptr(), D.data_ptr(), N, K, a_mn, b_mn, err.data_ptr(), None)
    torch.cuda.synchronize()
    assert rc == 0 and int(err.item()) == 0
    ref = A.float() @ B.float().T
    torch.testing.assert_close(D, ref, atol=1e-3, rtol=1e-3)


@pytest.mark.parametrize("t0,h,half", [(0, 0, 0), (64, 3, 1), (100, 5, 0), (190, 1, 1)])
def test_tma_sw128_tile(probe, t0, h, half):
    T, H = 200, 6
    src = torch.randn(T, H, 128, device="cuda").bfloat16()
    out = torch.empty(64, 64, device="cuda").bfloat16()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = probe.tma_probe(src.data_ptr(), T, H, t0, h, half, out.data_ptr(), err.data_ptr(), None)
    torch.cuda.synchronize()
    assert rc == 0 and int(err.item()) == 0
    want = torch.zeros(64, 64, device="cuda").bfloat16()
    n = min(64, T - t0)
    want[:n] = src[t0:t0 + n, h, half * 64:(half + 1) * 64]
    assert torch.equal(out, want)


def test_bounded_wait_gives_up_and_reports(probe):
    """A wait that nothing satisfies ends after its poll limit with the error code recorded; the context
    stays usable (a later launch and copy succeed)."""
    lib = probe
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.zeros(2, dtype=torch.int32, device="cuda")
    assert lib.wait_timeout_probe(ctypes.c_void_p(err.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                  ctypes.c_uint(2000), None) == 0
    torch.cuda.synchronize()
    assert err.item() == 77, "the first timed-out wait records its code (first error wins)"
    assert out.tolist() == [0, 0], "neither wait may report success"
    x = torch.arange(1024, device="cuda", dtype=torch.float32)
    assert float((x * 2).sum().item()) == 2.0 * 1023 * 1024 / 2
