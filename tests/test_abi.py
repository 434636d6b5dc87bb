"""CPU checks of the C-ABI library: it loads, exports every declared symbol, validates arguments.

No kernel runs here (no GPU in this container); argument checks return before any launch.
"""
import ctypes
import re
from pathlib import Path

import pytest

from sorernn_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "gdn_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(gdn_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.lib()
    names = declared_functions()
    assert len(names) >= 10
    for n in names:
        assert hasattr(lib, n), f"{n} declared in gdn_b200.h but not exported"
    assert set(names) == set(_lib.SIGNATURES), "ctypes signature table out of sync with the header"


def test_ctypes_signatures_match_header_arity():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    for name, (_, argtypes) in _lib.SIGNATURES.items():
        m = re.search(rf"\b{name}\s*\(([^)]*)\)", text)
        assert m, name
        params = [x for x in m.group(1).split(",") if x.strip() and x.strip() != "void"]
        assert len(params) == len(argtypes), f"{name}: header has {len(params)} params, ctypes {len(argtypes)}"


def test_status_strings():
    lib = _lib.lib()
    assert lib.gdn_status_string(0) == b"ok"
    assert b"shape" in lib.gdn_status_string(1)
    assert lib.gdn_status_string(999) == b"unknown status"


def _problem(**kw):
    base = dict(B=2, T=256, H=4, HV=4, DK=64, DV=64, N=2, cu_seqlens=None, max_seqlen=256, scale=0.125,
                act_dtype=_lib.FP32, g_dtype=_lib.FP32, beta_dtype=_lib.FP32, use_qk_l2norm=0, ckpt_every=4)
    base.update(kw)
    return _lib.Problem(**base)


def test_checkpoint_count_and_workspace_queries():
    lib = _lib.lib()
    p = _problem()
    assert lib.gdn_checkpoint_count(ctypes.byref(p)) == 2 * 1  # ceil(ceil(256/64)/4) per sequence
    p = _problem(T=4096, B=8, N=8, DK=128, DV=128, H=16, HV=16, act_dtype=_lib.BF16)
    assert lib.gdn_checkpoint_count(ctypes.byref(p)) == 8 * 16
    assert lib.gdn_chunk_fwd_workspace_size(ctypes.byref(p)) >= 256
    assert lib.gdn_chunk_bwd_workspace_size(ctypes.byref(p)) >= 256
    # varlen: an upper bound computed without reading the device cu_seqlens
    p = _problem(B=1, T=1000, N=5, cu_seqlens=16)
    assert lib.gdn_checkpoint_count(ctypes.byref(p)) >= 5


def test_saved_record_queries_and_checks():
    """The saved-record pair: 88 KB (90,112 B) per chunk-head for chunk-kernel problems, nothing for the
    recurrent family (which the pair refuses with GDN_ERR_SHAPE); missing or misaligned record buffers are
    refused before any launch."""
    lib = _lib.lib()
    p = _chunk_problem(4096, 16, B=8)
    assert lib.gdn_chunk_saved_bytes(ctypes.byref(p)) == 8 * 64 * 16 * 90112
    ws_saved = lib.gdn_chunk_bwd_saved_workspace_size(ctypes.byref(p))
    assert 0 < ws_saved < lib.gdn_chunk_bwd_workspace_size(ctypes.byref(p))
    pv = _chunk_problem(1000, 2)
    pv.N, pv.cu_seqlens = 5, 16
    assert lib.gdn_chunk_saved_bytes(ctypes.byref(pv)) == ((1000 + 63 * 5) // 64 + 5) * 2 * 90112
    rec = _problem()  # fp32, head size 64: the recurrent kernels
    assert lib.gdn_chunk_saved_bytes(ctypes.byref(rec)) == 0
    vp = ctypes.c_void_p(16)
    fwd = lambda prob, saved: lib.gdn_chunk_fwd_save(ctypes.byref(prob), vp, vp, vp, vp, vp, None, vp, None,  # noqa
                                                     saved, vp, 1 << 30, None)
    bwd = lambda prob, saved: lib.gdn_chunk_bwd_saved(ctypes.byref(prob), vp, vp, vp, vp, vp, saved, vp, None,  # noqa
                                                      vp, vp, vp, vp, vp, None, vp, 1 << 30, None)
    for call in (fwd, bwd):
        assert call(rec, vp) == 1
        assert call(p, None) == 7
        assert call(p, ctypes.c_void_p(24)) == 3


def test_segment_record_queries_and_checks():
    """The shared-record sequence-split pair: records sized like the forward's workspace for chunk-kernel
    problems, refused with GDN_ERR_SHAPE for the recurrent family; missing, short or misaligned record
    buffers are refused before any launch."""
    lib = _lib.lib()
    p = _chunk_problem(4096, 16, B=8)
    n = lib.gdn_segment_records_size(ctypes.byref(p))
    assert n >= 8 * 64 * 16 * 58368
    rec = _problem()
    assert lib.gdn_segment_records_size(ctypes.byref(rec)) == 0
    vp = ctypes.c_void_p(16)
    maps = lambda prob, buf, nb: lib.gdn_segment_maps(ctypes.byref(prob), vp, vp, vp, vp, vp, None, vp, vp,  # noqa
                                                      buf, nb, None)
    outs = lambda prob, buf, nb: lib.gdn_segment_outputs(ctypes.byref(prob), vp, vp, vp, vp, vp, None, vp,  # noqa
                                                         None, buf, nb, None)
    for call in (maps, outs):
        assert call(rec, vp, 1 << 20) == 1
        assert call(p, None, n) == 6
        assert call(p, vp, n - 1) == 6
        assert call(p, ctypes.c_void_p(24), n) == 3


def test_segment_save_variants_check_their_record_buffer():
    """The saving pair (training on pieces) takes the same arguments plus the backward-record buffer: a
    missing one is GDN_ERR_ARGUMENT, a misaligned one GDN_ERR_ALIGN, both before any launch; the record
    checks of the plain pair still apply."""
    lib = _lib.lib()
    p = _chunk_problem(4096, 16, B=2)
    n = lib.gdn_segment_records_size(ctypes.byref(p))
    vp = ctypes.c_void_p(16)
    maps = lambda saved, buf, nb: lib.gdn_segment_maps_save(ctypes.byref(p), vp, vp, vp, vp, vp, None, vp,  # noqa
                                                            vp, saved, buf, nb, None)
    outs = lambda saved, buf, nb: lib.gdn_segment_outputs_save(ctypes.byref(p), vp, vp, vp, vp, vp, None, vp,  # noqa
                                                               None, saved, buf, nb, None)
    for call in (maps, outs):
        assert call(None, vp, n) == _lib.lib().gdn_chunk_fwd_save(ctypes.byref(p), vp, vp, vp, vp, vp, None, vp,
                                                                  None, None, vp, 1 << 40, None)
        assert call(ctypes.c_void_p(24), vp, n) == 3
        assert call(vp, None, n) == 6


@pytest.mark.parametrize("bad", [dict(HV=6), dict(DK=256), dict(act_dtype=7), dict(N=3), dict(ckpt_every=0),
                                 dict(B=2, cu_seqlens=16)])
def test_invalid_problems_are_rejected_before_launch(bad):
    lib = _lib.lib()
    p = _problem(**bad)
    st = lib.gdn_chunk_fwd(ctypes.byref(p), *([ctypes.c_void_p(16)] * 5), None, ctypes.c_void_p(16), None, None,
                           ctypes.c_void_p(16), 1 << 20, None)
    assert st in (1, 2, 7), lib.gdn_status_string(st)


def test_missing_workspace_is_rejected():
    lib = _lib.lib()
    p = _problem()
    st = lib.gdn_chunk_fwd(ctypes.byref(p), *([ctypes.c_void_p(16)] * 5), None, ctypes.c_void_p(16), None, None,
                           None, 0, None)
    assert st == 6


def test_decode_rejects_bad_shapes():
    lib = _lib.lib()
    vp = ctypes.c_void_p(16)
    assert lib.gdn_decode_step(4, 3, 4, 128, 128, 0.1, 0, 0, 0, 0, vp, vp, vp, vp, vp, vp, vp, None) == 1
    assert lib.gdn_decode_step(4, 4, 4, 128, 128, 0.1, 9, 0, 0, 0, vp, vp, vp, vp, vp, vp, vp, None) == 2
    assert lib.gdn_decode_step(4, 4, 4, 128, 128, 0.1, 0, 0, 0, 0, vp, vp, vp, vp, vp, None, vp, None) == 7


def _chunk_problem(T, H, B=1):
    return _problem(B=B, T=T, H=H, HV=H, N=B, DK=128, DV=128, act_dtype=_lib.BF16, g_dtype=_lib.FP32,
                    beta_dtype=_lib.BF16, max_seqlen=T, ckpt_every=8)


@pytest.mark.parametrize("T,H,fits", [(1024, 16, True), (4096, 6, True), (64, 418, True), (64, 419, False),
                                      (4096, 16, False)])
def test_noalloc_capacity_matches_its_documentation(T, H, fits):
    """The header states the fixed array holds 418 chunk-heads (e.g. T = 1,024 x 16 heads, T = 4,096 x 6):
    those problems' workspaces fit, one chunk-head more does not, and gdn_chunk_bwd_noalloc rejects a problem
    that does not fit with GDN_ERR_SCRATCH_LIMIT before touching the device."""
    lib = _lib.lib()
    p = _chunk_problem(T, H)
    need = lib.gdn_chunk_bwd_workspace_size(ctypes.byref(p))
    assert need > 0
    assert (need <= _lib.NOALLOC_SCRATCH_BYTES) == fits, need
    if not fits:
        vp = ctypes.c_void_p(256)
        assert lib.gdn_chunk_bwd_noalloc(ctypes.byref(p), *([vp] * 15), None) == 8


def test_noalloc_reports_the_same_status_as_the_workspace_backward_for_invalid_problems():
    lib = _lib.lib()
    vp = ctypes.c_void_p(256)
    for bad, want in ((dict(act_dtype=7), 2), (dict(HV=6), 1), (dict(ckpt_every=0), 7)):
        p = _problem(**bad)
        assert lib.gdn_chunk_bwd_noalloc(ctypes.byref(p), *([vp] * 15), None) == want
        assert lib.gdn_chunk_bwd(ctypes.byref(p), *([vp] * 15), vp, 1 << 30, None) == want


def test_piece_chain_checks_its_arguments():
    """gdn_piece_chain: head sizes other than 128, a bad direction flag, missing tensors and misaligned
    pointers are refused before any launch; empty problems are a no-op."""
    lib = _lib.lib()
    vp = ctypes.c_void_p(256)
    assert lib.gdn_piece_chain(1, 4, 2, 64, 64, vp, vp, None, vp, None, 0, None) == 1
    assert lib.gdn_piece_chain(1, 4, 2, 128, 128, vp, vp, None, vp, None, 2, None) == 7
    assert lib.gdn_piece_chain(1, 4, 2, 128, 128, None, vp, None, vp, None, 0, None) == 7
    assert lib.gdn_piece_chain(1, 4, 2, 128, 128, vp, vp, None, None, None, 1, None) == 7
    assert lib.gdn_piece_chain(1, 4, 2, 128, 128, vp, ctypes.c_void_p(260), None, vp, None, 0, None) == 3
    assert lib.gdn_piece_chain(0, 4, 2, 128, 128, None, None, None, None, None, 0, None) == 0


def test_state_grad_sweep_checks_its_arguments():
    """gdn_chunk_state_grad_saved: dh0 and the records are required, the workspace is the saved backward's,
    recurrent-family problems are refused; all before any launch."""
    lib = _lib.lib()
    p = _chunk_problem(1024, 4, B=2)
    n = lib.gdn_chunk_bwd_saved_workspace_size(ctypes.byref(p))
    vp = ctypes.c_void_p(256)
    call = lambda prob, saved, dh0, ws, nb: lib.gdn_chunk_state_grad_saved(  # noqa: E731
        ctypes.byref(prob), vp, vp, vp, vp, vp, saved, vp, None, dh0, ws, nb, None)
    assert call(p, vp, None, vp, n) == 7
    assert call(p, None, vp, vp, n) == 7
    assert call(p, ctypes.c_void_p(264), vp, vp, n) == 3
    assert call(p, vp, vp, None, n) == 6
    assert call(p, vp, vp, vp, n - 1) == 6
    assert call(_problem(), vp, vp, vp, 1 << 30) == 1


def test_header_compiles_as_c_and_a_c_program_links_and_calls_the_queries(tmp_path):
    """A plain C99 caller (what a cgo, JNI or other C FFI binding compiles against): the header builds with gcc
    without C++, the program links against the library, and the host-side queries answer as documented."""
    import shutil
    import subprocess

    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no gcc")
    root = Path(__file__).resolve().parents[1]
    src = tmp_path / "caller.c"
    src.write_text(r'''
#include <stdio.h>
#include <string.h>
#include "gdn_b200.h"
int main(void) {
    gdn_problem p;
    memset(&p, 0, sizeof p);
    p.B = 8; p.T = 4096; p.H = 16; p.HV = 16; p.DK = 128; p.DV = 128; p.N = 8; p.max_seqlen = 4096;
    p.scale = 0.08838834764831845f; p.act_dtype = GDN_BF16; p.g_dtype = GDN_FP32; p.beta_dtype = GDN_BF16;
    p.use_qk_l2norm = 1; p.ckpt_every = 4;
    if (gdn_checkpoint_count(&p) != 8 * 16) return 1;
    if (gdn_chunk_fwd_workspace_size(&p) < 256) return 2;
    if (gdn_chunk_saved_bytes(&p) != (size_t)8 * 64 * 16 * 90112) return 3;
    if (strlen(gdn_status_string(GDN_OK)) == 0) return 4;
    p.DK = 256;  /* rejected by the shape check, before any pointer is used or any kernel launched */
    if (gdn_chunk_fwd(&p, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0) != GDN_ERR_SHAPE) return 5;
    printf("ok\n");
    return 0;
}
''')
    lib_dir = root / "sorernn_b200" / "_lib"
    exe = tmp_path / "caller"
    r = subprocess.run([gcc, "-std=c99", "-Wall", "-Werror", "-I", str(root / "include"), str(src), "-o", str(exe),
                        "-L", str(lib_dir), "-lgdn_b200", f"-Wl,-rpath,{lib_dir}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and r.stdout.strip() == "ok", (r.returncode, r.stdout, r.stderr)
