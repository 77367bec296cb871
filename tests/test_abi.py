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
