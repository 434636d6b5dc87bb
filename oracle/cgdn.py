"""ctypes binding of the C oracle (``oracle/gdn_oracle.c``): TEST INFRASTRUCTURE ONLY.

Same conventions as ``oracle/gdn_oracle.py`` but fp32 and multithreaded, for large parity cases and
for the timed CPU baseline of ``bench.py``. Arrays are numpy float32, laid out ``[B*T, H, d]``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "liboracle.so"
_lib = None


def build():
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def lib():
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        _lib = ctypes.CDLL(str(LIB_PATH))
        i64, f32, i32, vp = ctypes.c_int64, ctypes.c_float, ctypes.c_int, ctypes.c_void_p
        _lib.oracle_gdn_fwd.argtypes = [vp] * 5 + [i64] * 6 + [vp, i64, f32, i32, vp, vp, vp, i32]
        _lib.oracle_gdn_bwd.argtypes = [vp] * 6 + [i64] * 6 + [vp, i64, f32, i32, vp, vp] + [vp] * 6 + [i32]
        _lib.oracle_gdn_decode.argtypes = [vp] * 5 + [i64] * 5 + [f32, i32, vp, vp, i32]
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _f32(a):
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def _threads(n):
    return n if n else (os.cpu_count() or 1)


def forward(q, k, v, g, beta, scale, initial_state=None, cu_seqlens=None, use_qk_l2norm=False, threads=0):
    q, k, v, g, beta, h0 = map(_f32, (q, k, v, g, beta, initial_state))
    B, T, H, dk = q.shape
    HV, dv = v.shape[2], v.shape[3]
    cu = None if cu_seqlens is None else np.ascontiguousarray(cu_seqlens, dtype=np.int64)
    N = B if cu is None else len(cu) - 1
    o = np.zeros((B, T, HV, dv), np.float32)
    ht = np.zeros((N, HV, dk, dv), np.float32)
    lib().oracle_gdn_fwd(_p(q), _p(k), _p(v), _p(g), _p(beta), B, T, H, HV, dk, dv, _p(cu), N, scale,
                         int(use_qk_l2norm), _p(h0), _p(o), _p(ht), _threads(threads))
    return o, ht


def backward(q, k, v, g, beta, do, scale, initial_state=None, dht=None, cu_seqlens=None, use_qk_l2norm=False,
             threads=0):
    q, k, v, g, beta, do, h0, dht = map(_f32, (q, k, v, g, beta, do, initial_state, dht))
    B, T, H, dk = q.shape
    HV, dv = v.shape[2], v.shape[3]
    cu = None if cu_seqlens is None else np.ascontiguousarray(cu_seqlens, dtype=np.int64)
    N = B if cu is None else len(cu) - 1
    dq, dk_ = np.zeros_like(q), np.zeros_like(k)
    dv_, dg, db = np.zeros_like(v), np.zeros_like(g), np.zeros_like(beta)
    dh0 = np.zeros((N, HV, dk, dv), np.float32)
    lib().oracle_gdn_bwd(_p(q), _p(k), _p(v), _p(g), _p(beta), _p(do), B, T, H, HV, dk, dv, _p(cu), N, scale,
                         int(use_qk_l2norm), _p(h0), _p(dht), _p(dq), _p(dk_), _p(dv_), _p(dg), _p(db), _p(dh0),
                         _threads(threads))
    return dq, dk_, dv_, dg, db, dh0


def decode_step(q, k, v, g, beta, state, scale, use_qk_l2norm=False, threads=0):
    """``state`` (float32, C-contiguous) is updated in place."""
    q, k, v, g, beta = map(_f32, (q, k, v, g, beta))
    assert state.dtype == np.float32 and state.flags.c_contiguous
    N, H, dk = q.shape
    HV, dv = v.shape[1], v.shape[2]
    o = np.zeros((N, HV, dv), np.float32)
    lib().oracle_gdn_decode(_p(q), _p(k), _p(v), _p(g), _p(beta), N, H, HV, dk, dv, scale, int(use_qk_l2norm),
                            _p(state), _p(o), _threads(threads))
    return o
