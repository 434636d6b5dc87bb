"""ctypes binding of the C ABI in ``include/gdn_b200.h`` (library ``sorernn_b200/_lib/libgdn_b200.so``).

The library is loaded on first use. There is no fallback: a missing or unloadable library raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libgdn_b200.so"

BF16, FP16, FP32 = 0, 1, 2
NOALLOC_SCRATCH_BYTES = 36 << 20  # GDN_NOALLOC_SCRATCH_BYTES


class Problem(ctypes.Structure):
    """Mirror of ``struct gdn_problem``."""

    _fields_ = [
        ("B", ctypes.c_int64), ("T", ctypes.c_int64), ("H", ctypes.c_int64), ("HV", ctypes.c_int64),
        ("DK", ctypes.c_int64), ("DV", ctypes.c_int64), ("N", ctypes.c_int64),
        ("cu_seqlens", ctypes.c_void_p), ("max_seqlen", ctypes.c_int64), ("scale", ctypes.c_float),
        ("act_dtype", ctypes.c_int32), ("g_dtype", ctypes.c_int32), ("beta_dtype", ctypes.c_int32),
        ("use_qk_l2norm", ctypes.c_int32), ("ckpt_every", ctypes.c_int32),
    ]


# name -> (restype, argtypes)
_P = ctypes.POINTER(Problem)
_vp, _i64, _i32, _f32, _sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_float, ctypes.c_size_t
SIGNATURES = {
    "gdn_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "gdn_uses_chunk_kernels": (ctypes.c_int, [_P]),
    "gdn_checkpoint_count": (_i64, [_P]),
    "gdn_chunk_fwd_workspace_size": (_sz, [_P]),
    "gdn_chunk_bwd_workspace_size": (_sz, [_P]),
    "gdn_chunk_fwd": (ctypes.c_int, [_P] + [_vp] * 10 + [_sz, _vp]),
    "gdn_chunk_bwd": (ctypes.c_int, [_P] + [_vp] * 16 + [_sz, _vp]),
    "gdn_chunk_saved_bytes": (_sz, [_P]),
    "gdn_segment_records_size": (_sz, [_P]),
    "gdn_segment_maps": (ctypes.c_int, [_P] + [_vp] * 9 + [_sz, _vp]),
    "gdn_segment_outputs": (ctypes.c_int, [_P] + [_vp] * 9 + [_sz, _vp]),
    "gdn_segment_maps_save": (ctypes.c_int, [_P] + [_vp] * 10 + [_sz, _vp]),
    "gdn_segment_outputs_save": (ctypes.c_int, [_P] + [_vp] * 10 + [_sz, _vp]),
    "gdn_piece_chain": (ctypes.c_int, [_i64] * 5 + [_vp] * 5 + [_i32, _vp]),
    "gdn_chunk_state_grad_saved": (ctypes.c_int, [_P] + [_vp] * 10 + [_sz, _vp]),
    "gdn_chunk_bwd_saved_workspace_size": (_sz, [_P]),
    "gdn_chunk_fwd_save": (ctypes.c_int, [_P] + [_vp] * 10 + [_sz, _vp]),
    "gdn_chunk_bwd_saved": (ctypes.c_int, [_P] + [_vp] * 15 + [_sz, _vp]),
    "gdn_decode_step": (ctypes.c_int, [_i64] * 5 + [_f32] + [_i32] * 4 + [_vp] * 7 + [_vp]),
    "gdn_segment_transition": (ctypes.c_int, [_P] + [_vp] * 5 + [_sz, _vp]),
    "gdn_segment_apply_state": (ctypes.c_int, [_P] + [_vp] * 8 + [_sz, _vp]),
    "gdn_segment_workspace_size": (_sz, [_P]),
    "gdn_workspace_error": (ctypes.c_int, [_vp, _vp, ctypes.POINTER(_i32)]),
    "gdn_kernel_launches": (ctypes.c_uint64, []),
    "gdn_stream_kernels_error": (ctypes.c_int, [_vp, ctypes.POINTER(_i32)]),
    "gdn_chunk_bwd_noalloc": (ctypes.c_int, [_P] + [_vp] * 16),
    "gdn_gate_fwd": (ctypes.c_int, [_i64, _i64, _vp, _i32, _vp, _vp, _i32, _vp, _vp]),
    "gdn_gate_bwd": (ctypes.c_int, [_i64, _i64, _vp, _i32, _vp, _vp, _i32] + [_vp] * 5),
    "gdn_beta_sigmoid_fwd": (ctypes.c_int, [_i64, _vp, _i32, _vp, _vp]),
    "gdn_beta_sigmoid_bwd": (ctypes.c_int, [_i64, _vp, _i32, _vp, _vp, _vp]),
    "gdn_rms_norm_gated_fwd": (ctypes.c_int, [_i64, _i64, _vp, _vp, _i32, _vp, _i32, _f32, _vp, _vp]),
    "gdn_rms_norm_gated_bwd": (ctypes.c_int, [_i64, _i64, _vp, _vp, _i32, _vp, _i32, _f32] + [_vp] * 5),
    "gdn_causal_conv1d_fwd": (ctypes.c_int, [_i64] * 4 + [_vp, _i32, _vp, _i32, _vp, _i64, _i32, _vp, _vp]),
    "gdn_causal_conv1d_bwd": (ctypes.c_int, [_i64] * 4 + [_vp, _i32, _vp, _i32, _vp, _i64, _i32] + [_vp] * 4),
}

_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python -m sorernn_b200.build` (nvcc, sm_100a)")
        handle = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype, fn.argtypes = res, args
        _lib = handle
    return _lib


def check(status: int, what: str) -> None:
    if status != 0:
        msg = lib().gdn_status_string(status).decode()
        raise RuntimeError(f"{what} failed: {msg} (status {status})")
