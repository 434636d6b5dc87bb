"""Host-side checks of the Python boundary (no GPU needed): argument validation happens before any
library call, and CPU tensors are refused (no CPU fallback)."""
import pytest
import torch


def _x(B=1, T=8, H=2, HV=2, D=16):
    q = torch.randn(B, T, H, D)
    v = torch.randn(B, T, HV, D)
    return q, q.clone(), v, torch.randn(B, T, HV), torch.rand(B, T, HV)


def test_gate_in_kernel_requires_A_log():
    from sorernn_b200 import chunk_gated_delta_rule

    q, k, v, g, beta = _x()
    with pytest.raises(ValueError, match="A_log"):
        chunk_gated_delta_rule(q, k, v, g, beta, use_gate_in_kernel=True)


def test_unknown_keyword_is_rejected():
    from sorernn_b200 import chunk_gated_delta_rule

    q, k, v, g, beta = _x()
    with pytest.raises(TypeError, match="unexpected keyword"):
        chunk_gated_delta_rule(q, k, v, g, beta, use_gate_in_kernal=True)


def test_cpu_tensors_are_refused():
    from sorernn_b200 import chunk_gated_delta_rule, fused_recurrent_gated_delta_rule_step

    q, k, v, g, beta = _x()
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        chunk_gated_delta_rule(q, k, v, g, beta)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        chunk_gated_delta_rule(q, k, v, g, beta, use_gate_in_kernel=True, A_log=torch.zeros(2))
    state = torch.zeros(1, 2, 16, 16)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        fused_recurrent_gated_delta_rule_step(q[:, 0], k[:, 0], v[:, 0], g[:, 0], beta[:, 0], state)



@pytest.mark.parametrize("B,T,N,K,varlen", [(8, 4096, 8, 8, False), (2, 300, 2, 4, False), (1, 1000, 5, 8, True),
                                            (1, 64, 1, 1, False), (1, 0, 3, 8, True)])
def test_python_checkpoint_count_matches_library(B, T, N, K, varlen):
    import ctypes

    from sorernn_b200 import _lib
    from sorernn_b200.gated_delta_rule import checkpoint_count

    p = _lib.Problem(B=B, T=T, H=2, HV=2, DK=128, DV=128, N=N, cu_seqlens=16 if varlen else None, max_seqlen=T,
                     scale=1.0, act_dtype=_lib.BF16, g_dtype=_lib.FP32, beta_dtype=_lib.BF16, use_qk_l2norm=1,
                     ckpt_every=K)
    assert checkpoint_count(B, T, N, K, varlen) == _lib.lib().gdn_checkpoint_count(ctypes.byref(p))


@pytest.mark.parametrize("B,T,N,HV,varlen", [(8, 4096, 8, 16, False), (2, 300, 2, 4, False), (1, 1000, 5, 2, True),
                                             (1, 0, 3, 2, True)])
def test_python_saved_record_bytes_match_library(B, T, N, HV, varlen):
    import ctypes

    from sorernn_b200 import _lib
    from sorernn_b200.gated_delta_rule import saved_record_bytes

    p = _lib.Problem(B=B, T=T, H=HV, HV=HV, DK=128, DV=128, N=N, cu_seqlens=16 if varlen else None,
                     max_seqlen=T, scale=1.0, act_dtype=_lib.BF16, g_dtype=_lib.FP32, beta_dtype=_lib.BF16,
                     use_qk_l2norm=1, ckpt_every=8)
    assert saved_record_bytes(B, T, N, HV, varlen) == _lib.lib().gdn_chunk_saved_bytes(ctypes.byref(p))


def test_fake_kernels_trace_without_the_library(monkeypatch):
    """The custom ops' fake (meta) kernels compute output shapes in Python, so tracing (torch.compile,
    activation-checkpoint policies) needs neither a GPU nor the CUDA library."""
    from torch._subclasses.fake_tensor import FakeTensorMode

    from sorernn_b200 import _lib
    import sorernn_b200.gated_delta_rule  # noqa: F401  (registers the ops)

    def no_lib():
        raise AssertionError("the CUDA library was called while tracing")

    monkeypatch.setattr(_lib, "lib", no_lib)
    with FakeTensorMode():
        q = torch.empty(1, 300, 2, 128, dtype=torch.bfloat16, device="cuda")
        v = torch.empty(1, 300, 4, 128, dtype=torch.bfloat16, device="cuda")
        g = torch.empty(1, 300, 4, dtype=torch.float32, device="cuda")
        b = torch.empty(1, 300, 4, dtype=torch.bfloat16, device="cuda")
        cu = torch.empty(4, dtype=torch.int64, device="cuda")
        o, ht, ck = torch.ops.sorernn_b200.gdn_fwd(q, q, v, g, b, None, cu, 0.1, True, 300, 8)
        assert o.shape == v.shape and ht.shape == (3, 4, 128, 128)
        assert ck.shape[0] == (300 + 63 * 3) // 64 // 8 + 3 + 1
        dq, dk, dv, dg, db, dh0 = torch.ops.sorernn_b200.gdn_bwd(q, q, v, g, b, None, ck, v, None, cu, 0.1, True,
                                                                 300, 8)
        assert dq.shape == q.shape and dv.shape == v.shape and dh0.shape == (3, 4, 128, 128)
        # saved-record mode (ckpt_every 0): the third output is the byte buffer of the backward records
        o, ht, rec = torch.ops.sorernn_b200.gdn_fwd(q, q, v, g, b, None, cu, 0.1, True, 300, 0)
        assert rec.dtype == torch.uint8 and rec.shape == (((300 + 63 * 3) // 64 + 3) * 4 * 90112,)
        dq, *_ = torch.ops.sorernn_b200.gdn_bwd(q, q, v, g, b, None, rec, v, None, cu, 0.1, True, 300, 0)
        assert dq.shape == q.shape


@pytest.mark.parametrize("B,T,H,dtype,D,varlen,want", [
    (1, 4096, 16, torch.bfloat16, 128, False, 8),   # config 1 over 8 GPUs: 16 pairs
    (2, 4096, 16, torch.bfloat16, 128, False, 4),   # over 4 GPUs: 32 pairs
    (4, 4096, 16, torch.bfloat16, 128, False, 2),   # over 2 GPUs: 64 pairs
    (8, 4096, 16, torch.bfloat16, 128, False, 1),   # 128 pairs (one GPU): whole sequences
    (1, 1024, 16, torch.bfloat16, 128, False, 2),   # pieces of at least 512 tokens
    (1, 640, 2, torch.bfloat16, 128, False, 1),     # too short to cut
    (1, 4096, 16, torch.float32, 128, False, 1),    # recurrent kernels
    (1, 4096, 16, torch.bfloat16, 64, False, 1),    # head size other than 128
    (1, 4096, 16, torch.bfloat16, 128, True, 1),    # packed documents
])
def test_auto_pieces_choice(B, T, H, dtype, D, varlen, want):
    """The op's own choice of pieces per sequence (shape-only; no kernel runs)."""
    from sorernn_b200.gated_delta_rule import auto_pieces

    q = torch.empty(B, T, H, D, dtype=dtype, device="meta")
    v = torch.empty(B, T, H, D, dtype=dtype, device="meta")
    cu = torch.tensor([0, T // 2, T]) if varlen else None
    assert auto_pieces(q, v, cu) == want
