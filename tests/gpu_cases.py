"""Seeded inputs for the GPU parity tests (BASELINE.json configs and edge cases)."""
from __future__ import annotations

import numpy as np
import torch

from fused_rope_attn_b200 import compute_rope_2d
from fused_rope_attn_b200.utils import get_window_index, segments_per_image


def rand_qkv(T, H, D, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(T, H, D, generator=g).to(dtype) for _ in range(3)]


def grid_case(grid, windowed, H=16, D=80, dtype=torch.bfloat16, cs_dtype=torch.float32, seed=0):
    """q/k/v ~N(0,1) in window order, cos/sin from the 2D grid, cu_seqlens (CPU tensors)."""
    if windowed:
        widx, cu = get_window_index(grid)
        cos, sin = compute_rope_2d(grid, D, 2, 10000.0, "cpu", cs_dtype, window_idx=widx)
    else:
        cu = segments_per_image(grid)
        cos, sin = compute_rope_2d(grid, D, 2, 10000.0, "cpu", cs_dtype)
    T = int(cu[-1])
    q, k, v = rand_qkv(T, H, D, dtype, seed)
    return q, k, v, cos, sin, cu


def mixed_sides(seed=0, n=8):
    """Config 3: image sides (patches) drawn from {16,24,32,48,64,96}."""
    return [int(s) for s in np.random.default_rng(seed).choice([16, 24, 32, 48, 64, 96], n)]


def cu_case(cu_list, H=2, D=80, dtype=torch.bfloat16, cs_dtype=torch.float32, T=None, seed=0):
    """Random angles (not a grid) for arbitrary cu_seqlens."""
    T = cu_list[-1] if T is None else T
    q, k, v = rand_qkv(T, H, D, dtype, seed)
    g = torch.Generator().manual_seed(seed + 7)
    ang = torch.rand(T, D // 2, generator=g) * 20.0
    return q, k, v, ang.cos().to(cs_dtype), ang.sin().to(cs_dtype), torch.tensor(cu_list, dtype=torch.int32)
