"""CPU oracle for the fused 2D-RoPE + varlen attention path — TEST INFRASTRUCTURE ONLY.

This module is a plain numpy restatement of the reference's algorithm
(sdan/fused-rope-attn). It is the checker that the CUDA path is compared
against, and the timed CPU baseline in ``bench.py``; it is never on the
product path (``fused_rope_attn_b200`` does not import it).

Parity pin: ``tests/golden/`` holds vectors produced by the reference itself
(``tests/golden/make_golden.py`` imports the reference's ``fused_attn.py`` /
``utils.py``: host functions run natively, the Triton kernel runs under
``TRITON_INTERPRET=1`` with fp16/fp32 inputs). ``tests/test_oracle_golden.py``
checks every function here against them.

Functions and the reference lines they restate:

* ``rope_inv_freq``, ``rope_tables_2d`` — fused_attn.py:77-116 (compute_rope_2d)
* ``window_index``                    — utils.py:12-102 (get_window_index)
* ``shuffle`` / ``unshuffle``         — utils.py:105-153
* ``apply_rope``                      — bench.py:73-78 (split-half rotation) and
                                        fused_attn.py:340-345 / 385-390 (fp32 math,
                                        optional rounding to the input type)
* ``varlen_attention``                — utils.py:178-193 (non-causal softmax(QK^T d^-1/2)V
                                        per cu_seqlens segment; scale fused_attn.py:354-355)
* ``rope_attention``                  — the unfused path: apply_rope then varlen_attention
* ``qkv_rope``                        — the caller's projection + separate rotation
                                        (bench.py:72-78: linear output in the input
                                        type, then the split-half rotation of q, k)
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "rope_inv_freq",
    "rope_positions",
    "rope_tables_2d",
    "window_index",
    "shuffle",
    "unshuffle",
    "round_to",
    "apply_rope",
    "varlen_attention",
    "rope_attention",
    "qkv_rope",
    "varlen_attention_rows",
    "attention_flops",
    "attention_bytes",
]


def rope_inv_freq(head_dim: int, theta: float) -> np.ndarray:
    """inv_freq[i] = 1 / theta^(2i / (head_dim/2)), i < head_dim/4, fp32 (fused_attn.py:59,78)."""
    rd = head_dim // 2
    expo = np.arange(0, rd, 2, dtype=np.float32) / np.float32(rd)
    return (np.float32(1.0) / np.power(np.float32(theta), expo, dtype=np.float32)).astype(np.float32)


def rope_positions(grid_thw, merge: int) -> np.ndarray:
    """Per-token (h, w) patch ids in 2x2-merge order, repeated over t (fused_attn.py:84-102)."""
    rows = []
    for t, h, w in grid_thw:
        hh = np.repeat(np.arange(h)[:, None], w, axis=1)
        ww = np.repeat(np.arange(w)[None, :], h, axis=0)
        hh = hh.reshape(h // merge, merge, w // merge, merge).transpose(0, 2, 1, 3).reshape(-1)
        ww = ww.reshape(h // merge, merge, w // merge, merge).transpose(0, 2, 1, 3).reshape(-1)
        hw = np.stack([hh, ww], 1)
        rows.append(np.tile(hw, (t, 1)))
    return np.concatenate(rows, 0).astype(np.int64)


def rope_tables_2d(grid_thw, head_dim: int, merge: int, theta: float, window_idx=None):
    """(cos, sin) fp32 [T, head_dim/2]: h-angles then w-angles (fused_attn.py:105-116, 124-134)."""
    inv = rope_inv_freq(head_dim, theta)
    pos = rope_positions(grid_thw, merge).astype(np.float32)
    ang = np.concatenate([pos[:, :1] * inv[None, :], pos[:, 1:2] * inv[None, :]], axis=1).astype(np.float32)
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    if window_idx is not None:
        mu = merge * merge
        rd = head_dim // 2
        idx = np.asarray(window_idx, dtype=np.int64)
        cos = cos.reshape(-1, mu, rd)[idx].reshape(-1, rd)
        sin = sin.reshape(-1, mu, rd)[idx].reshape(-1, rd)
    return cos, sin


def window_index(grid_thw, window_size: int = 112, merge: int = 2, patch_size: int = 14):
    """(window_index int64 [T/merge^2], cu_seqlens int32) as utils.py:46-102.

    Merge units of each frame are grouped into vit_window x vit_window windows
    (vit_window = window_size // merge // patch_size); windows at the right and
    bottom edges are truncated; lengths are counted in tokens (x merge^2);
    repeated cumulative values (empty windows) are dropped.
    """
    vw = window_size // merge // patch_size
    mu = merge * merge
    idx_all, cu = [], [0]
    offset = 0
    for t, h, w in grid_thw:
        gh, gw = h // merge, w // merge
        nh, nw = -(-gh // vw), -(-gw // vw)
        for f in range(t):
            for wi in range(nh):
                for wj in range(nw):
                    r0, r1 = wi * vw, min(wi * vw + vw, gh)
                    c0, c1 = wj * vw, min(wj * vw + vw, gw)
                    ids = [offset + f * gh * gw + r * gw + c for r in range(r0, r1) for c in range(c0, c1)]
                    idx_all.extend(ids)
                    cu.append(cu[-1] + len(ids) * mu)
        offset += t * gh * gw
    cu = np.asarray(cu, dtype=np.int32)
    keep = np.concatenate([[True], cu[1:] != cu[:-1]])
    return np.asarray(idx_all, dtype=np.int64), cu[keep]


def shuffle(x: np.ndarray, widx: np.ndarray, merge: int = 2) -> np.ndarray:
    mu = merge * merge
    return x.reshape(-1, mu, *x.shape[1:])[widx].reshape(x.shape)


def unshuffle(x: np.ndarray, widx: np.ndarray, merge: int = 2) -> np.ndarray:
    mu = merge * merge
    inv = np.empty_like(widx)
    inv[widx] = np.arange(widx.size)
    return x.reshape(-1, mu, *x.shape[1:])[inv].reshape(x.shape)


def round_to(x: np.ndarray, dtype: str | None) -> np.ndarray:
    """Round fp32 values to bf16 / fp16 (round-to-nearest-even) and back to fp32."""
    x = np.asarray(x, dtype=np.float32)
    if dtype is None or dtype == "float32":
        return x
    if dtype == "float16":
        return x.astype(np.float16).astype(np.float32)
    if dtype == "bfloat16":
        u = x.view(np.uint32).astype(np.uint64)
        nan = np.isnan(x)
        u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
        out = u.astype(np.uint32).view(np.float32)
        return np.where(nan, x, out).astype(np.float32)
    raise ValueError(dtype)


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray, round_dtype: str | None = None) -> np.ndarray:
    """Split-half rotation of x [T, H, D] with cos/sin [T, D/2] broadcast over heads."""
    d = x.shape[-1] // 2
    x = x.astype(np.float32)
    c = cos.astype(np.float32)[:, None, :]
    s = sin.astype(np.float32)[:, None, :]
    x0, x1 = x[..., :d], x[..., d:]
    out = np.concatenate([x0 * c - x1 * s, x0 * s + x1 * c], axis=-1)
    return round_to(out, round_dtype)


def varlen_attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, cu_seqlens, scale: float | None = None,
                     p_round: str | None = None) -> np.ndarray:
    """Per-segment non-causal attention, fp32 math; rows outside all segments are 0."""
    T, H, D = q.shape
    scale = (1.0 / np.sqrt(D)) if scale is None else scale
    out = np.zeros((T, H, D), dtype=np.float32)
    cu = [int(x) for x in cu_seqlens]
    for a, b in zip(cu[:-1], cu[1:]):
        if b <= a:
            continue
        qs = q[a:b].astype(np.float32).transpose(1, 0, 2)
        ks = k[a:b].astype(np.float32).transpose(1, 0, 2)
        vs = v[a:b].astype(np.float32).transpose(1, 0, 2)
        s = np.matmul(qs, ks.transpose(0, 2, 1)) * np.float32(scale)
        s = s - s.max(axis=-1, keepdims=True)
        p = np.exp(s)
        l = p.sum(axis=-1, keepdims=True)
        if p_round is not None:
            p = round_to(p, p_round)
        out[a:b] = (np.matmul(p, vs) / l).transpose(1, 0, 2)
    return out


def varlen_attention_rows(q, k, v, cu_seqlens, rows) -> np.ndarray:
    """``varlen_attention`` evaluated only for the query rows ``rows`` -> [len(rows), H, D]."""
    T, H, D = q.shape
    cu = np.asarray([int(x) for x in cu_seqlens])
    out = np.zeros((len(rows), H, D), dtype=np.float32)
    for n, r in enumerate(rows):
        s = int(np.searchsorted(cu, r, side="right")) - 1
        if s < 0 or s >= len(cu) - 1 or not (cu[s] <= r < cu[s + 1]):
            continue
        a, b = cu[s], cu[s + 1]
        ks = k[a:b].astype(np.float32).transpose(1, 0, 2)          # [H, L, D]
        vs = v[a:b].astype(np.float32).transpose(1, 0, 2)
        sc = np.einsum("hd,hld->hl", q[r].astype(np.float32), ks) / np.float32(np.sqrt(D))
        sc = np.exp(sc - sc.max(axis=-1, keepdims=True))
        out[n] = np.einsum("hl,hld->hd", sc, vs) / sc.sum(axis=-1, keepdims=True)
    return out


def rope_attention(q, k, v, cos, sin, cu_seqlens, round_dtype: str | None = None) -> np.ndarray:
    """The reference's unfused path: RoPE(Q), RoPE(K) then varlen attention (fp32)."""
    qr = apply_rope(q, cos, sin, round_dtype)
    kr = apply_rope(k, cos, sin, round_dtype)
    return varlen_attention(qr, kr, v, cu_seqlens)


def attention_flops(cu_seqlens, heads: int, head_dim: int) -> int:
    """Algorithmic FLOPs: 4 * sum(L^2) * H * D (QK^T and PV, no padding)."""
    cu = [int(x) for x in cu_seqlens]
    return 4 * sum((b - a) ** 2 for a, b in zip(cu[:-1], cu[1:]) if b > a) * heads * head_dim


def attention_bytes(total: int, nseg: int, heads: int, head_dim: int, cs_bytes: int = 4, io_bytes: int = 2) -> int:
    """Algorithmic bytes: Q, K, V read + O written, cos/sin read once, cu_seqlens."""
    return 4 * total * heads * head_dim * io_bytes + 2 * total * (head_dim // 2) * cs_bytes + 4 * (nseg + 1)


def qkv_rope(x, w, b, cos, sin, heads: int, round_dtype: str | None = "bfloat16") -> np.ndarray:
    """[T, 3, H, D]: qkv = x w^T + b (fp32 math) rounded to ``round_dtype``, then q, k
    rotated with apply_rope (fp32, rounded again) and v as projected (bench.py:72-78)."""
    T = x.shape[0]
    y = x.astype(np.float32) @ w.astype(np.float32).T
    if b is not None:
        y = y + b.astype(np.float32)
    y = round_to(y.astype(np.float32), round_dtype).reshape(T, 3, heads, -1)
    q = apply_rope(y[:, 0], cos, sin, round_dtype)
    k = apply_rope(y[:, 1], cos, sin, round_dtype)
    return np.stack([q, k, y[:, 2]], axis=1)
