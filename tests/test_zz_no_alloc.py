"""gdn_chunk_bwd_noalloc: the backward for callers that cannot allocate device memory.

Such a caller (a host runtime reaching the library over a C FFI with no device allocator, or a plugin
whose execute hook must not allocate) gets gradients from a fixed scratch array inside the library instead
of a workspace it would have to allocate. This test calls the new entry point through the C ABI, twice in
a row, and checks both results against gdn_chunk_bwd run with an ordinary workspace, within the bf16
gradient tolerance the other tests use. It lives in its own file, collected last.
"""
import ctypes

import pytest
import torch

from helpers import assert_bf16_close, assert_rms_close, to_np

pytestmark = pytest.mark.gpu
D = 128


def _problem(_lib, B, T, H, HV, l2):
    return _lib.Problem(B=B, T=T, H=H, HV=HV, DK=D, DV=D, N=B, cu_seqlens=None, max_seqlen=T, scale=D ** -0.5,
                        act_dtype=_lib.BF16, g_dtype=_lib.FP32, beta_dtype=_lib.BF16, use_qk_l2norm=int(l2),
                        ckpt_every=4)


def _inputs(seed, B, T, H, HV, l2):
    g = torch.Generator(device="cuda").manual_seed(seed)
    unit = (lambda t: t) if l2 else (lambda t: torch.nn.functional.normalize(t, dim=-1))  # unit keys if no norm
    x = dict(q=unit(torch.randn(B, T, H, D, device="cuda", generator=g)),
             k=unit(torch.randn(B, T, H, D, device="cuda", generator=g)),
             v=torch.randn(B, T, HV, D, device="cuda", generator=g),
             do=torch.randn(B, T, HV, D, device="cuda", generator=g))
    x = {n: t.bfloat16().contiguous() for n, t in x.items()}
    x["g"] = (torch.nn.functional.logsigmoid(torch.randn(B, T, HV, device="cuda", generator=g)) / 16).contiguous()
    x["beta"] = torch.sigmoid(torch.randn(B, T, HV, device="cuda", generator=g)).bfloat16().contiguous()
    x["h0"] = (torch.randn(B, HV, D, D, device="cuda", generator=g) * 0.05).contiguous()
    x["dht"] = (torch.randn(B, HV, D, D, device="cuda", generator=g) * 0.1).contiguous()
    return x


def _outputs(x, B, HV):
    return dict(dq=torch.empty_like(x["q"]), dk=torch.empty_like(x["k"]), dv=torch.empty_like(x["v"]),
                dg=torch.empty(x["g"].shape, device="cuda"), dbeta=torch.empty(x["beta"].shape, device="cuda"),
                dh0=torch.empty(B, HV, D, D, device="cuda"))


def _ptrs(x, out, ck):
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    return [p(x["q"]), p(x["k"]), p(x["v"]), p(x["g"]), p(x["beta"]), p(x["h0"]), p(ck), p(x["do"]), p(x["dht"]),
            p(out["dq"]), p(out["dk"]), p(out["dv"]), p(out["dg"]), p(out["dbeta"]), p(out["dh0"])]


@pytest.mark.parametrize("B,T,H,HV,l2", [(1, 700, 2, 2, True), (2, 300, 1, 2, False)])
def test_noalloc_backward_matches_workspace_backward_twice(B, T, H, HV, l2):
    from sorernn_b200 import _lib
    from sorernn_b200.gated_delta_rule import gdn_fwd

    lib = _lib.lib()
    x = _inputs(B * 100 + T, B, T, H, HV, l2)
    _, _, ck = gdn_fwd(x["q"], x["k"], x["v"], x["g"], x["beta"], x["h0"], None, D ** -0.5, l2, T, 4)
    p = _problem(_lib, B, T, H, HV, l2)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    ref = _outputs(x, B, HV)
    nbytes = lib.gdn_chunk_bwd_workspace_size(ctypes.byref(p))
    ws = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    _lib.check(lib.gdn_chunk_bwd(ctypes.byref(p), *_ptrs(x, ref, ck), ctypes.c_void_p(ws.data_ptr()), nbytes, stream),
               "gdn_chunk_bwd")
    torch.cuda.synchronize()
    assert all(torch.isfinite(t.float()).all() for t in ref.values())
    for _ in range(2):
        got = _outputs(x, B, HV)
        _lib.check(lib.gdn_chunk_bwd_noalloc(ctypes.byref(p), *_ptrs(x, got, ck), stream), "gdn_chunk_bwd_noalloc")
        torch.cuda.synchronize()
        for n in ("dq", "dk", "dv"):
            assert_bf16_close(to_np(got[n]), to_np(ref[n]), 3e-2, n)
        for n in ("dg", "dbeta", "dh0"):
            assert_rms_close(to_np(got[n]), to_np(ref[n]), 3e-2, n)


def test_noalloc_rejects_problems_beyond_its_scratch():
    from sorernn_b200 import _lib

    lib = _lib.lib()
    p = _problem(_lib, 1, 1 << 16, 16, 16, True)  # 16,384 chunk-heads: far above the 36 MiB array
    vp = ctypes.c_void_p(256)
    st = lib.gdn_chunk_bwd_noalloc(ctypes.byref(p), *([vp] * 15), None)
    assert st == 8, lib.gdn_status_string(st)
    assert b"scratch" in lib.gdn_status_string(8)
