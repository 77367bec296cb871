"""Host-side producers of the kernel's inputs (window order and cu_seqlens).

Mirrors the reference module ``utils.py`` (sdan/fused-rope-attn):

* ``get_window_index`` — utils.py:12-102: Qwen-VL window partition of merge units
  and token-space ``cu_seqlens`` (edge windows truncated, empty windows dropped)
* ``window_shuffle`` / ``window_unshuffle`` — utils.py:105-153
* ``flash_window_attention`` — utils.py:156-195, the unfused comparator
  (FlashAttention varlen). It is a baseline only and never used by the fused path.

The partition is computed with vectorised index arithmetic per image (one
``argsort`` of a window key) rather than padding and reshaping; the output is
identical (tests/test_host_golden.py checks it against vectors produced by the
reference).
"""
from __future__ import annotations

import torch

__all__ = [
    "get_window_index",
    "window_shuffle",
    "window_unshuffle",
    "flash_window_attention",
    "segments_per_image",
]


def _thw(grid_thw):
    if isinstance(grid_thw, torch.Tensor):
        if grid_thw.ndim != 2 or grid_thw.shape[-1] != 3:
            raise ValueError(f"grid_thw must be [N,3], got {tuple(grid_thw.shape)}")
        return [(int(t), int(h), int(w)) for t, h, w in grid_thw.tolist()]
    return [(int(t), int(h), int(w)) for (t, h, w) in grid_thw]


def get_window_index(
    grid_thw,
    *,
    window_size: int = 112,
    spatial_merge_size: int = 2,
    patch_size: int = 14,
    device: torch.device | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """Window permutation of merge units and token-space ``cu_seqlens``.

    Each frame's ``(h/m) x (w/m)`` merge-unit grid is cut into square windows of
    ``window_size // m // patch_size`` units (8 x 8 patches for the Qwen2.5-VL
    defaults). Windows are visited row-major per frame and units row-major per
    window; windows on the right/bottom edge keep only their valid units.
    Returns ``(window_index int64 [T / m^2], cu_seqlens int32)`` where
    ``cu_seqlens`` counts tokens (units x m^2) and skips empty windows.
    """
    if device is None:
        device = grid_thw.device if isinstance(grid_thw, torch.Tensor) else torch.device("cpu")
    thw = _thw(grid_thw)
    if not thw:
        raise ValueError("grid_thw must be non-empty")
    if window_size <= 0:
        raise ValueError(f"window_size must be > 0, got {window_size}")
    if spatial_merge_size <= 0:
        raise ValueError(f"spatial_merge_size must be > 0, got {spatial_merge_size}")
    if patch_size <= 0:
        raise ValueError(f"patch_size must be > 0, got {patch_size}")
    m = spatial_merge_size
    vw = window_size // m // patch_size
    if vw <= 0:
        raise ValueError(
            "vit_window computed as window_size//spatial_merge_size//patch_size must be >= 1, "
            f"got {vw} (window_size={window_size} spatial_merge_size={m} patch_size={patch_size})"
        )
    mu = m * m
    perms, lens = [], []
    base = 0
    for t, h, w in thw:
        if t <= 0:
            raise ValueError(f"grid_thw temporal size must be > 0, got t={t}")
        if h <= 0 or w <= 0:
            raise ValueError(f"grid_thw h/w must be > 0, got h={h} w={w}")
        if h % m or w % m:
            raise ValueError(f"h and w must be divisible by spatial_merge_size={m}, got h={h} w={w}")
        gh, gw = h // m, w // m
        nwh, nww = -(-gh // vw), -(-gw // vw)
        r = torch.arange(gh).view(gh, 1).expand(gh, gw)
        c = torch.arange(gw).view(1, gw).expand(gh, gw)
        # window id (row-major over windows), then position inside the window
        win = (r // vw) * nww + (c // vw)
        inner = (r % vw) * vw + (c % vw)
        key = (win * (vw * vw) + inner).reshape(-1)
        order = torch.argsort(key)                     # unit ids of one frame in window order
        counts = torch.bincount(win.reshape(-1), minlength=nwh * nww)
        frames = torch.arange(t).view(t, 1) * (gh * gw)
        perms.append((order.view(1, -1) + frames).reshape(-1) + base)
        lens.append(counts.repeat(t))
        base += t * gh * gw
    window_index = torch.cat(perms).to(device=device, dtype=torch.long)
    tok = torch.cat(lens) * mu
    cu = torch.cat([torch.zeros(1, dtype=torch.long), torch.cumsum(tok, 0)])
    keep = torch.ones_like(cu, dtype=torch.bool)
    keep[1:] = cu[1:] != cu[:-1]
    return window_index.contiguous(), cu[keep].to(device=device, dtype=torch.int32).contiguous()


def _check_perm(x: torch.Tensor, window_index: torch.Tensor, spatial_merge_size: int) -> tuple[int, int]:
    if x.ndim < 1:
        raise ValueError(f"x must have at least 1 dim, got {tuple(x.shape)}")
    mu = int(spatial_merge_size) ** 2
    if mu <= 0:
        raise ValueError(f"spatial_merge_size must be > 0, got {spatial_merge_size}")
    n = int(x.shape[0])
    if n % mu:
        raise ValueError(f"seq_len must be divisible by merge_unit={mu}, got {n}")
    if window_index.numel() != n // mu:
        raise ValueError(f"window_index length must be {n // mu}, got {window_index.numel()}")
    return n, mu


def window_shuffle(x: torch.Tensor, window_index: torch.Tensor, *, spatial_merge_size: int = 2) -> torch.Tensor:
    """Reorder tokens (in groups of ``merge^2``) into window order (utils.py:105-126)."""
    n, mu = _check_perm(x, window_index, spatial_merge_size)
    return x.reshape(n // mu, mu, *x.shape[1:])[window_index.to(x.device)].reshape(x.shape)


def window_unshuffle(x: torch.Tensor, window_index: torch.Tensor, *, spatial_merge_size: int = 2) -> torch.Tensor:
    """Inverse of ``window_shuffle`` (utils.py:129-153)."""
    n, mu = _check_perm(x, window_index, spatial_merge_size)
    idx = window_index.to(x.device)
    out = torch.empty_like(x).reshape(n // mu, mu, *x.shape[1:])
    out[idx] = x.reshape(n // mu, mu, *x.shape[1:])
    return out.reshape(x.shape)


def segments_per_image(grid_thw, spatial_merge_size: int = 2, device=None) -> torch.Tensor:
    """cu_seqlens with one segment per image (per clip for t > 1): full-attention layers."""
    lens = [t * h * w for t, h, w in _thw(grid_thw)]
    cu = torch.zeros(len(lens) + 1, dtype=torch.int32)
    cu[1:] = torch.cumsum(torch.tensor(lens), 0)
    return cu.to(device) if device is not None else cu


def flash_window_attention(q, k, v, cu_seqlens, num_heads: int, head_dim: int, softmax_scale: float | None = None):
    """Unfused comparator: FlashAttention varlen over window order (utils.py:156-195).

    Used only as the GPU baseline arm; raises if flash_attn cannot be imported.
    """
    try:
        from flash_attn import flash_attn_varlen_func
    except Exception as exc:  # noqa: BLE001
        raise RuntimeError("flash_attn not available") from exc
    n = q.shape[0]
    q = q.view(n, num_heads, head_dim)
    k = k.view(n, num_heads, head_dim)
    v = v.view(n, num_heads, head_dim)
    max_len = int((cu_seqlens[1:] - cu_seqlens[:-1]).max().item())
    scale = head_dim ** -0.5 if softmax_scale is None else softmax_scale
    o = flash_attn_varlen_func(q, k, v, cu_seqlens_q=cu_seqlens, cu_seqlens_k=cu_seqlens,
                               max_seqlen_q=max_len, max_seqlen_k=max_len, dropout_p=0.0,
                               softmax_scale=scale, causal=False)
    return o.view(n, num_heads * head_dim)
