"""ctypes binding of the C-ABI library ``libfrattn.so`` (declared in include/frattn.h).

The library is built in-tree by ``fused_rope_attn_b200.build`` (nvcc, sm_100a).
Nothing here falls back to another implementation: if the shared object is
missing, every entry point raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libfrattn.so")

F32, F16, BF16 = 0, 1, 2

OK = 0
E_SHAPE, E_DTYPE, E_ALIGN, E_NULL, E_WORKSPACE, E_NOALLOC_LIMIT = -1, -2, -3, -4, -5, -6
NOALLOC_MAX_TOKENS = 65536
E_CUDA, E_TMAP = 1, 2
STATUS_WAIT_TIMEOUT = 0x100
STATUS_BAD_SEQLENS = 0x200
STATUS_BAD_POSITIONS = 0x400

# Every symbol include/frattn.h declares, with (restype, argtypes).
_vp, _i, _sz, _u64, _f = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_uint64, ctypes.c_float
_SIGNATURES = {
    "frattn_version": (_i, []),
    "frattn_error_string": (ctypes.c_char_p, [_i]),
    "frattn_workspace_bytes": (_i, [_i, _i, ctypes.POINTER(_sz)]),
    "frattn_workspace_bytes_pos": (_i, [_i, _i, _i, _i, ctypes.POINTER(_sz)]),
    "frattn_workspace_bytes_rotated_k": (_i, [_i, _i, _i, ctypes.POINTER(_sz)]),
    "frattn_fwd": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _vp, _i, _i, _i, _i, _i, _i, _vp, _vp, _sz, _vp, _vp]),
    "frattn_fwd_strided": (_i, [_vp, _vp, _vp, ctypes.c_longlong, ctypes.c_longlong, ctypes.c_longlong, _vp, _vp,
                               _i, _vp, _i, _i, _i, _i, _i, _i, _vp, _vp, _sz, _vp, _vp]),
    "frattn_fwd_pos": (_i, [_vp, _vp, _vp, _vp, _i, _f, _vp, _i, _i, _i, _i, _i, _i, _vp, _vp, _sz, _vp, _vp]),
    "frattn_qkv_rope": (_i, [_vp, ctypes.c_longlong, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp, _vp, _vp]),
    "frattn_qkv_rope_set_pairs": (_i, [_i]),
    "frattn_fwd_rotated": (_i, [_vp, _vp, _vp, ctypes.c_longlong, ctypes.c_longlong, ctypes.c_longlong, _vp, _i,
                               _i, _i, _i, _i, _i, _vp, _vp, _sz, _vp, _vp]),
    "frattn_fwd_lse": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _vp, _i, _i, _i, _i, _i, _i, _vp, _vp, _vp, _sz, _vp, _vp]),
    "frattn_workspace_bytes_bwd": (_i, [_i, _i, _i, ctypes.POINTER(_sz)]),
    "frattn_bwd": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _vp, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _sz,
                       _vp, _vp]),
    "frattn_workspace_bytes_fp8": (_i, [_i, _i, _i, _i, ctypes.POINTER(_sz)]),
    "frattn_fwd_fp8": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _vp, _i, _i, _i, _i, _i, _i, _vp, _vp, _sz, _vp, _vp]),
    "frattn_fwd_noalloc": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _vp, _i, _i, _i, _i, _i, _i, _vp, _vp, _vp]),
    "frattn_window_plan_sizes": (_i, [_vp, _i, _i, _i, _i, ctypes.POINTER(ctypes.c_int64),
                                      ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(_sz)]),
    "frattn_window_plan": (_i, [_vp, _i, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _i, _f, _vp, _sz, _vp]),
    "frattn_window_shuffle": (_i, [_vp, _vp, ctypes.c_int64, _i, ctypes.c_int64, _i, _vp, _vp]),
    "frattn_selftest_wait_timeout": (_i, [_vp, _u64, _vp]),
    "frattn_set_wait_limit_ns": (_i, [_u64]),
    "frattn_set_timing_events": (_i, [_vp, _vp]),
}

_lib = None
_lock = threading.Lock()


class FrattnError(RuntimeError):
    """A C-ABI call returned a non-zero code."""

    def __init__(self, code: int, where: str):
        self.code = code
        super().__init__(f"{where}: {error_string(code)} (code {code})")


def load() -> ctypes.CDLL:
    """Load (once) and return the library; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m fused_rope_attn_b200.build` "
                    "(there is no fallback implementation)"
                )
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def error_string(code: int) -> str:
    try:
        return load().frattn_error_string(int(code)).decode()
    except Exception:  # noqa: BLE001 - used while formatting another error
        return f"error {code}"


def check(code: int, where: str) -> None:
    if code != 0:
        if code == E_SHAPE or code == E_DTYPE or code == E_ALIGN or code == E_NULL:
            raise ValueError(f"{where}: {error_string(code)} (code {code})")
        raise FrattnError(code, where)


def workspace_bytes(total_tokens: int, num_segments: int) -> int:
    out = ctypes.c_size_t(0)
    check(load().frattn_workspace_bytes(int(total_tokens), int(num_segments), ctypes.byref(out)),
          "frattn_workspace_bytes")
    return int(out.value)


def workspace_bytes_pos(total_tokens: int, num_segments: int, max_position: int, head_dim: int) -> int:
    out = ctypes.c_size_t(0)
    check(load().frattn_workspace_bytes_pos(int(total_tokens), int(num_segments), int(max_position),
                                            int(head_dim), ctypes.byref(out)),
          "frattn_workspace_bytes_pos")
    return int(out.value)


def workspace_bytes_rotated_k(total_tokens: int, num_heads: int, head_dim: int) -> int:
    out = ctypes.c_size_t(0)
    check(load().frattn_workspace_bytes_rotated_k(int(total_tokens), int(num_heads), int(head_dim),
                                                  ctypes.byref(out)),
          "frattn_workspace_bytes_rotated_k")
    return int(out.value)


def workspace_bytes_bwd(total_tokens: int, num_heads: int, head_dim: int) -> int:
    out = ctypes.c_size_t(0)
    check(load().frattn_workspace_bytes_bwd(int(total_tokens), int(num_heads), int(head_dim), ctypes.byref(out)),
          "frattn_workspace_bytes_bwd")
    return int(out.value)


def workspace_bytes_fp8(total_tokens: int, num_segments: int, num_heads: int, head_dim: int) -> int:
    out = ctypes.c_size_t(0)
    check(load().frattn_workspace_bytes_fp8(int(total_tokens), int(num_segments), int(num_heads), int(head_dim),
                                            ctypes.byref(out)), "frattn_workspace_bytes_fp8")
    return int(out.value)
