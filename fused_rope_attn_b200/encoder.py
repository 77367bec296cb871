"""Qwen2.5-VL-shaped vision encoder harness around the fused attention path.

BASELINE configs 4 and 5 need a full vision stack to measure the hot path in
context: 32 pre-norm blocks (RMSNorm eps 1e-6, QKV projection with bias,
attention, output projection, SiLU-gated MLP 1280 -> 3420 -> 1280), hidden
1280, 16 heads of 80, full attention at layers {7, 15, 23, 31} and 8x8-patch
windows elsewhere, random weights ~N(0, 0.02). The reference ships no encoder;
this is harness code, not part of the kernel contract.

Token flow (Qwen2.5-VL): patch embeddings are window-shuffled once (one
gather kernel), every layer runs in window order (windowed layers use the
window ``cu_seqlens``, full layers one segment per image/clip), and the output
is unshuffled at the end. The permutation, the window ``cu_seqlens`` and the
window-ordered cos/sin come from the device window plan (``frattn_window_plan``,
equal to ``get_window_index`` / ``compute_rope_2d`` of the reference).

Attention implementations (``attn=``):
* ``"fused"``    — ``fused_rope_attention`` (this repository's sm_100a kernel);
* ``"fused_fp8"`` — ``fused_rope_attention`` on window layers and the FP8
                   (e4m3 q/k) variant ``fused_rope_attention_fp8`` on full layers;
* ``"fused_qkv"`` — the QKV projection with RoPE in its epilogue
                   (``qkv_rope_projection``, an own tcgen05 GEMM) followed by
                   ``fused_attention_rotated``: no rotation in attention;
* ``"unfused"``  — separate RoPE in the input dtype (torch elementwise, as the
                   reference's baseline ``bench.py:73-78``) + FlashAttention
                   varlen (``flash_attn_varlen_func``; ``torch.nn.attention.varlen``
                   when flash_attn cannot run);
* ``"fp32"``     — RoPE and per-segment attention in fp32 (drift reference).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from .fused_attn import (compute_rope_2d, fused_attention_rotated, fused_rope_attention, fused_rope_attention_fp8,
                         qkv_rope_projection)
from .utils import get_window_index, segments_per_image, window_shuffle, window_unshuffle
from .window_plan import window_plan_device, window_shuffle_device, window_unshuffle_device

__all__ = ["EncoderConfig", "VisionEncoder", "encoder_inputs", "rope_unfused", "attention_fp32"]


@dataclass
class EncoderConfig:
    hidden: int = 1280
    heads: int = 16
    head_dim: int = 80
    mlp: int = 3420
    depth: int = 32
    full_layers: tuple = (7, 15, 23, 31)
    eps: float = 1e-6
    window_size: int = 112
    patch_size: int = 14
    merge: int = 2
    theta: float = 10000.0
    init_std: float = 0.02
    seed: int = 0
    extra: dict = field(default_factory=dict)


def rope_unfused(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Split-half rotation in the dtype of ``x`` (the reference baseline, bench.py:73-78)."""
    half = x.shape[-1] // 2
    c = cos.to(x.dtype)[:, None, :]
    s = sin.to(x.dtype)[:, None, :]
    x0, x1 = x[..., :half], x[..., half:]
    return torch.cat([x0 * c - x1 * s, x0 * s + x1 * c], dim=-1)


def attention_fp32(q, k, v, cos, sin, cu) -> torch.Tensor:
    """RoPE then per-segment softmax attention, all in fp32 (fp32 result).

    The reference's unfused path (bench.py:73-78 + utils.py:178-193) without any
    rounding; runs of equal-length segments are batched into one call.
    """
    qr = rope_unfused(q.float(), cos.float(), sin.float())
    kr = rope_unfused(k.float(), cos.float(), sin.float())
    vf = v.float()
    out = torch.zeros_like(qr)
    cl = cu.tolist()
    i, n = 0, len(cl) - 1
    while i < n:
        L = cl[i + 1] - cl[i]
        j = i
        while j < n and cl[j + 1] - cl[j] == L:
            j += 1
        a, b = cl[i], cl[j]
        if L > 0:
            def seg(x):  # [nseg * L, H, D] -> [nseg, H, L, D]
                return x[a:b].reshape(j - i, L, *x.shape[1:]).transpose(1, 2)
            o = torch.nn.functional.scaled_dot_product_attention(seg(qr), seg(kr), seg(vf))
            out[a:b] = o.transpose(1, 2).reshape(b - a, *qr.shape[1:])
        i = j
    return out


def _attn_fp32(q, k, v, cos, sin, cu):
    return attention_fp32(q, k, v, cos, sin, cu).to(q.dtype)


_FA_OK: bool | None = None


def _attn_unfused(q, k, v, cos, sin, cu, max_len):
    global _FA_OK
    qr, kr = rope_unfused(q, cos, sin), rope_unfused(k, cos, sin)
    scale = q.shape[-1] ** -0.5
    if _FA_OK is not False:
        try:
            from flash_attn import flash_attn_varlen_func
            out = flash_attn_varlen_func(qr, kr, v, cu, cu, max_len, max_len, 0.0, scale, False)
            _FA_OK = True
            return out
        except Exception:  # noqa: BLE001 - flash_attn build without sm_100 kernels
            _FA_OK = False
    from torch.nn.attention.varlen import varlen_attn
    return varlen_attn(qr, kr, v, cu, cu, max_len, max_len, scale=scale)


def unfused_backend() -> str:
    return {None: "unknown", True: "flash_attn_varlen_func", False: "torch.nn.attention.varlen"}[_FA_OK]


class VisionEncoder(torch.nn.Module):
    """32-layer random-weight Qwen2.5-VL-style vision stack (see module docstring)."""

    def __init__(self, cfg: EncoderConfig | None = None, device="cuda", dtype=torch.bfloat16):
        super().__init__()
        self.cfg = cfg = cfg or EncoderConfig()
        g = torch.Generator().manual_seed(cfg.seed)
        hid, mlp = cfg.hidden, cfg.mlp

        def w(*shape):
            return torch.nn.Parameter((torch.randn(*shape, generator=g) * cfg.init_std).to(device=device, dtype=dtype),
                                      requires_grad=False)

        # The MLP width is stored padded to a multiple of 8 with zero rows /
        # columns: silu(0) * 0 = 0 adds nothing, so the function is the
        # cfg.mlp-wide one, while every GEMM operand row is 16-byte aligned
        # (3420 x 2 B is not, and cuBLAS then falls back to sm80 kernels).
        mlp_p = -(-mlp // 8) * 8

        def pad_rows(t):
            return torch.nn.functional.pad(t, (0, 0, 0, mlp_p - mlp)) if mlp_p != mlp else t

        self.layers = []
        for i in range(cfg.depth):
            layer = {
                "n1": torch.ones(hid, device=device, dtype=dtype),
                "n2": torch.ones(hid, device=device, dtype=dtype),
                "qkv_w": w(3 * hid, hid), "qkv_b": w(3 * hid),
                "proj_w": w(hid, hid), "proj_b": w(hid),
            }
            gate, up, down = w(mlp, hid), w(mlp, hid), w(hid, mlp)  # same draw order as unpadded
            layer.update({
                "gate_w": pad_rows(gate.data), "up_w": pad_rows(up.data),
                "down_w": torch.nn.functional.pad(down.data, (0, mlp_p - mlp)) if mlp_p != mlp else down.data,
            })
            self.layers.append(layer)
        self.device, self.dtype = torch.device(device), dtype

    def _rms(self, x, weight):
        # torch's fused RMSNorm (fp32 statistics, one pass over x)
        return torch.nn.functional.rms_norm(x, (x.shape[-1],), weight, self.cfg.eps)

    def plan(self, grid_thw):
        """Window permutation, cu_seqlens of both layer kinds and window-ordered cos/sin,
        built on the device (``frattn_window_plan``: no host index arithmetic, no
        host sync). The longest segments come from the grid: a window holds at
        most (window_size / patch_size)^2 tokens, an image / clip t h w."""
        c = self.cfg
        cu_full = segments_per_image(grid_thw, device=self.device)
        lw = min((c.window_size // c.patch_size) ** 2, max(int(h) * int(w) for _, h, w in grid_thw))
        lf = max(int(t) * int(h) * int(w) for t, h, w in grid_thw)
        if self.device.type != "cuda":  # the fp32 harness on CPU (multi-process tests): host plan
            widx, cu_win = get_window_index(grid_thw, window_size=c.window_size, spatial_merge_size=c.merge,
                                            patch_size=c.patch_size)
            cos, sin = compute_rope_2d(grid_thw, c.head_dim, c.merge, c.theta, self.device, torch.float32,
                                       window_idx=widx)
            return dict(widx=widx, cu_win=cu_win, cu_full=cu_full, max_win=int(lw), max_full=int(lf), cos=cos,
                        sin=sin)
        dp = window_plan_device(grid_thw, window_size=c.window_size, spatial_merge_size=c.merge,
                                patch_size=c.patch_size, device=self.device, head_dim=c.head_dim, theta=c.theta,
                                positions=False)
        return dict(widx=dp["window_index"], cu_win=dp["cu_seqlens"], cu_full=cu_full, max_win=int(lw),
                    max_full=int(lf), cos=dp["cos"], sin=dp["sin"])

    def forward(self, x: torch.Tensor, grid_thw, attn: str = "fused", plan=None, layer_hook=None,
                attn_hook=None):
        """Run the stack. ``layer_hook(i, h)`` sees the hidden states after layer i;
        ``attn_hook(i, q, k, v, cos, sin, cu_seqlens, o)`` sees each attention call's
        inputs and output (window order; with ``"fused_qkv"`` q and k are already
        rotated)."""
        c = self.cfg
        plan = plan or self.plan(grid_thw)
        T = x.shape[0]
        on_gpu = x.device.type == "cuda"
        shuffle = window_shuffle_device if on_gpu else window_shuffle
        h = shuffle(x, plan["widx"], spatial_merge_size=c.merge)
        for i, L in enumerate(self.layers):
            full = i in c.full_layers
            cu = plan["cu_full"] if full else plan["cu_win"]
            max_len = plan["max_full"] if full else plan["max_win"]
            y = self._rms(h, L["n1"])
            if attn == "fused_qkv":  # q, k leave the projection rotated
                qkv = qkv_rope_projection(y, L["qkv_w"], L["qkv_b"], plan["cos"], plan["sin"], c.heads)
            else:
                qkv = torch.nn.functional.linear(y, L["qkv_w"], L["qkv_b"]).view(T, 3, c.heads, c.head_dim)
            q, k, v = qkv[:, 0], qkv[:, 1], qkv[:, 2]
            if attn == "fused_qkv":
                o = fused_attention_rotated(q, k, v, cu, max_seqlen=max_len)
            elif attn == "fused_fp8" and full:
                o = fused_rope_attention_fp8(q, k, v, plan["cos"], plan["sin"], cu, max_seqlen=max_len)
            elif attn in ("fused", "fused_fp8"):
                o = fused_rope_attention(q, k, v, plan["cos"], plan["sin"], cu, max_seqlen=max_len)
            elif attn == "unfused":
                o = _attn_unfused(q, k, v, plan["cos"], plan["sin"], cu, max_len)
            elif attn == "fp32":
                o = _attn_fp32(q, k, v, plan["cos"], plan["sin"], cu)
            else:
                raise ValueError(f"unknown attention implementation {attn!r}")
            if attn_hook is not None:
                attn_hook(i, q, k, v, plan["cos"], plan["sin"], cu, o)
            h = h + torch.nn.functional.linear(o.reshape(T, -1), L["proj_w"], L["proj_b"])
            y = self._rms(h, L["n2"])
            a = torch.nn.functional.silu(torch.nn.functional.linear(y, L["gate_w"])) * \
                torch.nn.functional.linear(y, L["up_w"])
            h = h + torch.nn.functional.linear(a, L["down_w"])
            if layer_hook is not None:
                layer_hook(i, h)
        unshuffle = window_unshuffle_device if on_gpu else window_unshuffle
        return unshuffle(h, plan["widx"], spatial_merge_size=c.merge)


def encoder_inputs(grid_thw, hidden=1280, seed=0, device="cuda", dtype=torch.bfloat16):
    """Seeded N(0, 1) patch embeddings for the given grids, [T, hidden]."""
    T = sum(t * h * w for t, h, w in grid_thw)
    g = torch.Generator().manual_seed(seed)
    return torch.randn(T, hidden, generator=g).to(device=device, dtype=dtype)


def encoder_flops(grid_thw, cfg: EncoderConfig | None = None) -> dict:
    """GEMM and attention FLOPs of one forward (for reporting)."""
    cfg = cfg or EncoderConfig()
    T = sum(t * h * w for t, h, w in grid_thw)
    gemm = 2 * T * cfg.depth * (cfg.hidden * 3 * cfg.hidden + cfg.hidden * cfg.hidden + 3 * cfg.hidden * cfg.mlp)
    _, cu_win = get_window_index(grid_thw, window_size=cfg.window_size, spatial_merge_size=cfg.merge,
                                 patch_size=cfg.patch_size)
    cw = cu_win.tolist()
    cf = segments_per_image(grid_thw).tolist()
    win = 4 * sum((b - a) ** 2 for a, b in zip(cw[:-1], cw[1:])) * cfg.heads * cfg.head_dim
    full = 4 * sum((b - a) ** 2 for a, b in zip(cf[:-1], cf[1:])) * cfg.heads * cfg.head_dim
    nf = len(cfg.full_layers)
    return {"gemm": gemm, "attention": nf * full + (cfg.depth - nf) * win}


def rel_l2(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float(), b.float()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))

