"""C-ABI library: loads without a GPU, exports every declared symbol, rejects bad arguments."""
import ctypes
import os
import re

import pytest

from conftest import ROOT
from fused_rope_attn_b200 import _lib

HEADER = os.path.join(ROOT, "include", "frattn.h")


def declared_symbols():
    txt = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(frattn_\w+)\s*\(", txt, re.M)))


def test_header_and_binding_agree():
    assert declared_symbols() == sorted(_lib.exported_symbols())


def test_library_exports_every_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.frattn_version() >= 100


def test_workspace_sizes():
    assert _lib.workspace_bytes(0, 1) > 0
    a = _lib.workspace_bytes(4096, 64)
    b = _lib.workspace_bytes(9216, 1)
    assert b > a > 0
    assert _lib.workspace_bytes_pos(4096, 64, 64, 80) > a
    with pytest.raises(ValueError):
        _lib.workspace_bytes(-1, 1)
    with pytest.raises(ValueError):
        _lib.workspace_bytes(10, 0)


def _fwd(lib, **kw):
    a = dict(q=16, k=16, v=16, cos=16, sin=16, cs=_lib.F32, cu=16, nseg=1, T=128, H=2, D=80, ms=0,
             dt=_lib.BF16, out=16, ws=16, wsb=1 << 20, status=None, stream=None)
    a.update(kw)
    return lib.frattn_fwd(a["q"], a["k"], a["v"], a["cos"], a["sin"], a["cs"], a["cu"], a["nseg"], a["T"],
                          a["H"], a["D"], a["ms"], a["dt"], a["out"], a["ws"], a["wsb"], a["status"], a["stream"])


def test_argument_validation_before_launch():
    lib = _lib.load()
    assert _fwd(lib, q=None) == _lib.E_NULL
    assert _fwd(lib, D=72 + 2) == _lib.E_SHAPE
    assert _fwd(lib, H=0) == _lib.E_SHAPE
    assert _fwd(lib, nseg=0) == _lib.E_SHAPE
    assert _fwd(lib, dt=_lib.F32) == _lib.E_DTYPE
    assert _fwd(lib, cs=7) == _lib.E_DTYPE
    assert _fwd(lib, q=24) == _lib.E_ALIGN
    assert _fwd(lib, wsb=8) == _lib.E_WORKSPACE
    assert lib.frattn_selftest_wait_timeout(None, 1000, None) == _lib.E_NULL
    assert lib.frattn_set_wait_limit_ns(0) == _lib.E_SHAPE
    assert lib.frattn_set_wait_limit_ns(2_000_000_000) == 0


def test_error_strings():
    assert _lib.error_string(0) == "ok"
    assert "workspace" in _lib.error_string(_lib.E_WORKSPACE)
    assert "timed out" in _lib.error_string(_lib.STATUS_WAIT_TIMEOUT | 0x21)
    with pytest.raises(ValueError):
        _lib.check(_lib.E_SHAPE, "x")
    with pytest.raises(_lib.FrattnError):
        _lib.check(_lib.E_CUDA, "x")


def test_wrapper_rejects_cpu_tensors():
    import torch
    from fused_rope_attn_b200 import fused_rope_attention
    q = torch.zeros(4, 1, 80, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        fused_rope_attention(q, q, q, torch.zeros(4, 40), torch.zeros(4, 40), torch.tensor([0, 4]))


def test_noalloc_rejects_oversize_before_touching_the_gpu():
    lib = _lib.load()
    rc = lib.frattn_fwd_noalloc(16, 16, 16, 16, 16, _lib.F32, 16, 1, _lib.NOALLOC_MAX_TOKENS + 1, 2, 80, 0,
                                _lib.BF16, 16, None, None)
    assert rc == _lib.E_NOALLOC_LIMIT
    assert "NOALLOC" in _lib.error_string(rc)


def test_strided_entry_point_validates_strides():
    lib = _lib.load()

    def fwd(qs, ks, vs, **kw):
        a = dict(T=128, H=2, D=80)
        a.update(kw)
        return lib.frattn_fwd_strided(16, 16, 16, qs, ks, vs, 16, 16, _lib.F32, 16, 1, a["T"], a["H"], a["D"], 0,
                                      _lib.BF16, 16, 16, 1 << 20, None, None)
    assert fwd(0, 160, 160) == _lib.E_SHAPE          # strides must be given
    assert fwd(150, 160, 160) == _lib.E_SHAPE        # below H * D
    assert fwd(164, 160, 160) == _lib.E_ALIGN        # row starts not 16-byte aligned
    assert lib.frattn_set_timing_events(16, None) == _lib.E_NULL
    assert lib.frattn_set_timing_events(None, None) == 0


def test_window_plan_sizes_match_host():
    import ctypes
    from fused_rope_attn_b200.utils import get_window_index
    lib = _lib.load()
    for grid in ([(1, 32, 32)], [(1, 22, 30), (2, 8, 12)], [(8, 32, 32), (1, 64, 64)]):
        arr = (ctypes.c_int32 * (3 * len(grid)))(*[v for g in grid for v in g])
        u, w, ws = ctypes.c_int64(0), ctypes.c_int64(0), ctypes.c_size_t(0)
        assert lib.frattn_window_plan_sizes(arr, len(grid), 112, 2, 14, ctypes.byref(u), ctypes.byref(w),
                                            ctypes.byref(ws)) == 0
        widx, cu = get_window_index(grid)
        assert u.value == widx.numel() and w.value == cu.numel() - 1 and ws.value >= 32 * len(grid)
    bad = (ctypes.c_int32 * 3)(1, 15, 16)  # h not divisible by the merge size
    assert lib.frattn_window_plan_sizes(bad, 1, 112, 2, 14, ctypes.byref(u), ctypes.byref(w),
                                        ctypes.byref(ws)) == _lib.E_SHAPE


def test_projection_and_rotated_entry_points_validate_arguments():
    lib = _lib.load()

    def qkv(**kw):
        a = dict(x=16, xs=0, w=16, b=None, cos=16, sin=16, cs=_lib.F32, T=128, K=1280, H=16, D=80, dt=_lib.BF16,
                 out=16)
        a.update(kw)
        return lib.frattn_qkv_rope(a["x"], a["xs"], a["w"], a["b"], a["cos"], a["sin"], a["cs"], a["T"], a["K"],
                                   a["H"], a["D"], a["dt"], a["out"], None, None)
    assert qkv(x=None) == _lib.E_NULL
    assert qkv(D=72) == _lib.E_SHAPE            # head dims: multiples of 16
    assert qkv(D=144) == _lib.E_SHAPE
    assert qkv(K=1284) == _lib.E_ALIGN          # rows must be 16-byte multiples
    assert qkv(xs=1000) == _lib.E_SHAPE         # stride below K
    assert qkv(dt=_lib.F32) == _lib.E_DTYPE
    assert qkv(cs=9) == _lib.E_DTYPE
    assert qkv(w=24) == _lib.E_ALIGN
    assert qkv(T=0) == 0                        # nothing to do, nothing launched

    def rot(**kw):
        a = dict(qs=0, T=128, H=2, D=80, dt=_lib.BF16, wsb=1 << 20)
        a.update(kw)
        return lib.frattn_fwd_rotated(16, 16, 16, a["qs"], 0, 0, 16, 1, a["T"], a["H"], a["D"], 0, a["dt"], 16, 16,
                                      a["wsb"], None, None)
    assert rot(qs=-1) == _lib.E_SHAPE
    assert rot(D=74) == _lib.E_SHAPE
    assert rot(dt=_lib.F32) == _lib.E_DTYPE
    assert rot(wsb=8) == _lib.E_WORKSPACE


def test_backward_and_fp8_entry_points_validate_arguments():
    import ctypes
    lib = _lib.load()
    assert _lib.workspace_bytes_bwd(4096, 16, 80) >= 4096 * 16 * 80 * (2 + 2 + 4)
    assert _lib.workspace_bytes_fp8(4096, 1, 16, 80) >= _lib.workspace_bytes(4096, 1) + 2 * 4096 * 16 * 80

    def bwd(**kw):
        a = dict(q=16, T=128, H=2, D=80, dt=_lib.BF16, cs=_lib.F32, lse=16, wsb=1 << 30)
        a.update(kw)
        return lib.frattn_bwd(a["q"], 16, 16, 16, 16, a["cs"], 16, 1, a["T"], a["H"], a["D"], a["dt"], 16, 16,
                              a["lse"], 16, 16, 16, 16, a["wsb"], None, None)
    assert bwd(q=None) == _lib.E_NULL
    assert bwd(D=72) == _lib.E_SHAPE            # backward head dims: multiples of 16
    assert bwd(D=144) == _lib.E_SHAPE
    assert bwd(dt=_lib.F32) == _lib.E_DTYPE
    assert bwd(cs=5) == _lib.E_DTYPE
    assert bwd(lse=18) == _lib.E_ALIGN
    assert bwd(wsb=16) == _lib.E_WORKSPACE

    def fp8(**kw):
        a = dict(D=80, ws=256, wsb=1 << 30, dt=_lib.BF16)
        a.update(kw)
        return lib.frattn_fwd_fp8(16, 16, 16, 16, 16, _lib.F32, 16, 1, 128, 2, a["D"], 0, a["dt"], 16, a["ws"],
                                  a["wsb"], None, None)
    assert fp8(D=72) == _lib.E_SHAPE
    assert fp8(dt=_lib.F32) == _lib.E_DTYPE
    assert fp8(ws=272) == _lib.E_ALIGN          # workspace 256-byte aligned
    assert fp8(wsb=1024) == _lib.E_WORKSPACE
    out = ctypes.c_size_t(0)
    assert lib.frattn_workspace_bytes_fp8(10, 0, 1, 80, ctypes.byref(out)) == _lib.E_SHAPE


def test_training_wrapper_rejects_unsupported_head_dim_on_cpu():
    import torch
    from fused_rope_attn_b200 import fused_rope_attention_train
    q = torch.zeros(4, 1, 80, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        fused_rope_attention_train(q, q, q, torch.zeros(4, 40), torch.zeros(4, 40), torch.tensor([0, 4]))
