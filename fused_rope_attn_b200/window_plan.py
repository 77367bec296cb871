"""Window plan built on the device (``frattn_window_plan`` / ``frattn_window_shuffle``).

Device counterparts of the host producers of the kernel's inputs:

* ``window_plan_device`` — ``get_window_index`` (reference utils.py:12-102) plus the
  window-ordered ``compute_rope_2d`` tables (fused_attn.py:33-136 with
  ``window_idx``) and the window-ordered (h, w) positions for
  ``fused_rope_attention_pos``; every element is written by a CUDA kernel from a
  closed form, with no host index arithmetic and no large host->device copy.
* ``window_shuffle_device`` / ``window_unshuffle_device`` — utils.py:105-153 as one
  gather / scatter kernel over rows.

Results are identical to the host functions in ``utils.py`` (permutation,
cu_seqlens and positions bit-exact; fp32 tables within fp32 rounding of the
angle evaluation).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .utils import _check_perm, _thw

__all__ = ["window_plan_device", "window_shuffle_device", "window_unshuffle_device"]


def _grid_array(grid_thw):
    thw = _thw(grid_thw)
    if not thw:
        raise ValueError("grid_thw must be non-empty")
    return thw, (ctypes.c_int32 * (3 * len(thw)))(*[v for row in thw for v in row])


def window_plan_device(grid_thw, *, window_size: int = 112, spatial_merge_size: int = 2, patch_size: int = 14,
                       device=None, head_dim: int | None = None, theta: float = 10000.0, positions: bool = True):
    """Window permutation, cu_seqlens, positions and rotary tables on ``device``.

    Returns a dict with ``window_index`` (int64 [T / m^2]), ``cu_seqlens`` (int32),
    ``pos_hw`` (int32 [T, 2] in window order, or None with ``positions=False``) and,
    when ``head_dim`` is given, ``cos`` / ``sin`` (fp32 [T, head_dim // 2] in window
    order, equal to ``compute_rope_2d(..., torch.float32, window_idx=window_index)``).
    """
    device = torch.device("cuda") if device is None else torch.device(device)
    if device.type != "cuda":
        raise ValueError(f"window_plan_device needs a CUDA device, got {device}")
    if head_dim is not None and (head_dim <= 0 or head_dim % 4):
        raise ValueError(f"head_dim must be divisible by 4, got {head_dim}")
    thw, arr = _grid_array(grid_thw)
    lib = _lib.load()
    units, windows, ws = ctypes.c_int64(0), ctypes.c_int64(0), ctypes.c_size_t(0)
    _lib.check(lib.frattn_window_plan_sizes(arr, len(thw), int(window_size), int(spatial_merge_size),
                                            int(patch_size), ctypes.byref(units), ctypes.byref(windows),
                                            ctypes.byref(ws)), "frattn_window_plan_sizes")
    mu = int(spatial_merge_size) ** 2
    T = units.value * mu
    widx = torch.empty(units.value, dtype=torch.int64, device=device)
    cu = torch.empty(windows.value + 1, dtype=torch.int32, device=device)
    pos = torch.empty(T, 2, dtype=torch.int32, device=device) if positions else None
    cos = sin = None
    rd = 0
    if head_dim is not None:
        rd = head_dim // 2
        cos = torch.empty(T, rd, dtype=torch.float32, device=device)
        sin = torch.empty(T, rd, dtype=torch.float32, device=device)
    work = torch.empty(max(ws.value, 256), dtype=torch.uint8, device=device)

    def ptr(t):
        return t.data_ptr() if t is not None else None

    with torch.cuda.device(device):
        rc = lib.frattn_window_plan(arr, len(thw), int(window_size), int(spatial_merge_size), int(patch_size),
                                    widx.data_ptr(), cu.data_ptr(), ptr(pos), ptr(cos), ptr(sin), rd, float(theta),
                                    work.data_ptr(), work.numel(), torch.cuda.current_stream(device).cuda_stream)
    _lib.check(rc, "frattn_window_plan")
    # (``work`` returns to torch's stream-ordered allocator: a later user of the
    # block on this stream runs after the kernels that read it.)
    return {"window_index": widx, "cu_seqlens": cu, "pos_hw": pos, "cos": cos, "sin": sin}


def _shuffle(x: torch.Tensor, window_index: torch.Tensor, merge: int, inverse: int) -> torch.Tensor:
    n, mu = _check_perm(x, window_index, merge)
    if x.device.type != "cuda":
        raise ValueError(f"x must be on CUDA, got {x.device}")
    xc = x.contiguous()
    row_bytes = xc[0].numel() * xc.element_size() if n else 16
    if row_bytes % 16:
        raise ValueError(f"a row of x must be a multiple of 16 bytes, got {row_bytes}")
    idx = window_index.to(device=x.device, dtype=torch.int64).contiguous()
    out = torch.empty_like(xc)
    with torch.cuda.device(x.device):
        rc = _lib.load().frattn_window_shuffle(xc.data_ptr(), idx.data_ptr(), n // mu, mu, row_bytes, inverse,
                                               out.data_ptr(), torch.cuda.current_stream(x.device).cuda_stream)
    _lib.check(rc, "frattn_window_shuffle")
    return out


def window_shuffle_device(x: torch.Tensor, window_index: torch.Tensor, *, spatial_merge_size: int = 2) -> torch.Tensor:
    """Tokens (in groups of merge^2) into window order, one gather kernel (utils.py:105-126)."""
    return _shuffle(x, window_index, spatial_merge_size, 0)


def window_unshuffle_device(x: torch.Tensor, window_index: torch.Tensor, *, spatial_merge_size: int = 2) -> torch.Tensor:
    """Inverse of ``window_shuffle_device`` (utils.py:129-153)."""
    return _shuffle(x, window_index, spatial_merge_size, 1)
