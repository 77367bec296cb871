"""Host side of the fused 2D-RoPE + varlen attention path.

Mirrors the public interface of the reference module ``fused_attn.py``
(sdan/fused-rope-attn):

* ``compute_rope_2d``      — fused_attn.py:33-136 (2D rotary cos/sin tables, LRU cached)
* ``fused_rope_attention`` — fused_attn.py:139-232 (same signature, argument meaning and
  ``ValueError`` behaviour), launching the sm_100a kernels of ``libfrattn.so`` through
  the C ABI instead of a Triton kernel
* ``next_pow2``            — fused_attn.py:13-15

Additions that keep the call a drop-in:

* keyword ``max_seqlen`` is an optional hint, never required: the on-device
  scheduler derives the work list from ``cu_seqlens`` itself, so no ``.item()``
  host sync is needed (the reference syncs at fused_attn.py:211). A hint of at
  most 128 (window layers) skips the K pre-rotation pass and its workspace;
  results are the same with or without it;
* ``fused_rope_attention_pos`` takes integer (h, w) patch positions instead of
  materialised cos/sin tables and evaluates the rotary angles in the kernel.
"""
from __future__ import annotations

import threading
from collections import OrderedDict

import torch

from . import _lib

__all__ = [
    "next_pow2",
    "compute_rope_2d",
    "rope_positions_2d",
    "fused_rope_attention",
    "fused_rope_attention_pos",
    "last_status",
    "SUPPORTED_HEAD_DIMS",
]

# Head dimensions with compiled sm_100a kernels (multiples of 8 in [32, 128]).
# Any other even head_dim up to 128 runs on the next one through zero padding
# (``_padded_dim``), so every head_dim the reference accepts
# (fused_attn.py:166-168) up to 128 works.
KERNEL_HEAD_DIMS = tuple(range(32, 129, 8))
SUPPORTED_HEAD_DIMS = tuple(range(2, 129, 2))

_DT = {torch.float32: _lib.F32, torch.float16: _lib.F16, torch.bfloat16: _lib.BF16}


def next_pow2(n: int) -> int:
    """Smallest power of two >= n (1 for n <= 0); fused_attn.py:13-15."""
    n = int(n)
    if n <= 1:
        return 1
    return 1 << (n - 1).bit_length()


# --------------------------------------------------------------------------- RoPE tables
_ROPE_CACHE_MAX = 32
_rope_cache: "OrderedDict[tuple, tuple[torch.Tensor, torch.Tensor]]" = OrderedDict()
_rope_lock = threading.Lock()


def _thw_list(grid_thw) -> list[tuple[int, int, int]]:
    if isinstance(grid_thw, torch.Tensor):
        rows = grid_thw.detach().to("cpu").tolist()
    else:
        rows = list(grid_thw)
    return [(int(r[0]), int(r[1]), int(r[2])) for r in rows]


def _device_key(device: torch.device) -> tuple:
    if device.type == "cuda":
        return ("cuda", device.index if device.index is not None else torch.cuda.current_device())
    return (device.type, device.index)


def rope_positions_2d(grid_thw, spatial_merge_size: int = 2, device=None) -> torch.Tensor:
    """(h, w) patch coordinates of every token, int32 ``[T, 2]``, in merge order.

    Tokens of one image are ordered by merge block (row-major over the
    ``h/m x w/m`` block grid) and, inside a block, row-major over its ``m x m``
    patches; frames of a clip repeat the same coordinates
    (the ordering built at fused_attn.py:84-102).
    """
    m = int(spatial_merge_size)
    out = []
    for t, h, w in _thw_list(grid_thw):
        if h % m or w % m:
            raise ValueError(f"h and w must be divisible by spatial_merge_size={m}, got h={h} w={w}")
        bh = torch.arange(h // m).view(-1, 1, 1, 1)
        bw = torch.arange(w // m).view(1, -1, 1, 1)
        ih = torch.arange(m).view(1, 1, -1, 1)
        iw = torch.arange(m).view(1, 1, 1, -1)
        hh = (bh * m + ih).expand(h // m, w // m, m, m).reshape(-1)
        ww = (bw * m + iw).expand(h // m, w // m, m, m).reshape(-1)
        hw = torch.stack([hh, ww], dim=1)
        out.append(hw.repeat(t, 1) if t > 1 else hw)
    pos = torch.cat(out, 0).to(torch.int32) if out else torch.zeros(0, 2, dtype=torch.int32)
    return pos.to(device) if device is not None else pos


def compute_rope_2d(
    grid_thw,
    head_dim: int,
    spatial_merge_size: int,
    theta: float,
    device,
    dtype,
    window_idx: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """2D rotary tables ``(cos, sin)``, each ``[T, head_dim // 2]`` (fused_attn.py:33-136).

    Rotary index ``i < head_dim/4`` rotates with the patch row ``h``, index
    ``head_dim/4 + i`` with the patch column ``w``; both use
    ``inv_freq[i] = 1 / theta^(2i / (head_dim/2))``. Angles are formed in fp32 and
    the tables cast to ``dtype``. Results are cached (32 entries, LRU) per
    (grid, head_dim, merge, theta, device, dtype). ``window_idx`` permutes merge
    units (groups of ``merge^2`` tokens) into window order after the cache.
    """
    if head_dim <= 0 or head_dim % 4 != 0:
        raise ValueError(f"head_dim must be divisible by 4, got {head_dim}")
    device = torch.device(device)
    thw = _thw_list(grid_thw)
    merge = int(spatial_merge_size)
    rd = head_dim // 2
    key = (tuple(thw), int(head_dim), merge, float(theta), *_device_key(device), dtype)
    with _rope_lock:
        hit = _rope_cache.get(key)
        if hit is not None:
            _rope_cache.move_to_end(key)
    if hit is None:
        inv_freq = 1.0 / (theta ** (torch.arange(0, rd, 2, device=device, dtype=torch.float32) / rd))
        pos = rope_positions_2d(thw, merge, device=device).float()
        ang = torch.cat([pos[:, 0:1] * inv_freq[None, :], pos[:, 1:2] * inv_freq[None, :]], dim=-1)
        hit = (ang.cos().to(dtype).contiguous(), ang.sin().to(dtype).contiguous())
        with _rope_lock:
            _rope_cache[key] = hit
            _rope_cache.move_to_end(key)
            while len(_rope_cache) > _ROPE_CACHE_MAX:
                _rope_cache.popitem(last=False)
    cos, sin = hit
    if window_idx is not None:
        mu = merge * merge
        idx = window_idx.to(device=device, dtype=torch.long)
        cos = cos.view(-1, mu, rd)[idx].reshape(-1, rd)
        sin = sin.view(-1, mu, rd)[idx].reshape(-1, rd)
    return cos.contiguous(), sin.contiguous()


# --------------------------------------------------------------------------- op wrapper
_status: dict[int, torch.Tensor] = {}


def _status_word(device: torch.device) -> torch.Tensor:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    s = _status.get(idx)
    if s is None:
        s = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status[idx] = s
    return s


def last_status(device=None, reset: bool = True) -> int:
    """Device status word of the kernels on ``device`` (0 = no device-side error).

    Reading it synchronises with the device. Non-zero values are the
    ``FRATTN_STATUS_*`` codes of include/frattn.h.
    """
    device = torch.device("cuda") if device is None else torch.device(device)
    s = _status_word(device)
    v = int(s.item())
    if reset and v:
        s.zero_()
    return v


def _aligned(t: torch.Tensor) -> torch.Tensor:
    return t if t.data_ptr() % 16 == 0 else t.clone()


def _token_rows(t: torch.Tensor) -> tuple[torch.Tensor, int]:
    """``t`` [T, H, D] as rows the kernel reads in place: (tensor, token stride in
    elements). Views whose heads and dims are packed but whose tokens are spread
    out (q/k/v of one fused QKV projection) are passed as they are; anything
    else is copied to a contiguous tensor (as the reference does for every
    non-contiguous input, fused_attn.py:187-193)."""
    T, H, D = t.shape
    if (t.stride(2) == 1 and t.stride(1) == D and t.stride(0) >= H * D and t.stride(0) % 8 == 0
            and t.data_ptr() % 16 == 0):
        return t, int(t.stride(0))
    t = _aligned(t.contiguous())
    return t, H * D


def _check_qkv(q, k, v):
    if q.device.type != "cuda":
        raise ValueError(f"q must be on CUDA, got device={q.device}")
    if q.shape != k.shape or q.shape != v.shape:
        raise ValueError(f"q/k/v must have same shape, got q={tuple(q.shape)} k={tuple(k.shape)} v={tuple(v.shape)}")
    if q.ndim != 3:
        raise ValueError(f"q/k/v must be [total_seq, num_heads, head_dim], got q.ndim={q.ndim}")
    total, heads, hd = (int(x) for x in q.shape)
    if hd <= 0 or hd % 2 != 0:
        raise ValueError(f"head_dim must be positive and even, got {hd}")
    if q.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError(f"q dtype must be float16 or bfloat16, got {q.dtype}")
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError(f"q/k/v must share dtype, got q={q.dtype} k={k.dtype} v={v.dtype}")
    if k.device != q.device or v.device != q.device:
        raise ValueError(f"q/k/v must share a device, got q={q.device} k={k.device} v={v.device}")
    return total, heads, hd


def _check_cu(cu_seqlens, device):
    if cu_seqlens.ndim != 1 or cu_seqlens.numel() < 2:
        raise ValueError(f"cu_seqlens must be 1D with length >= 2, got {tuple(cu_seqlens.shape)}")
    cu = cu_seqlens
    if cu.dtype != torch.int32:
        cu = cu.to(torch.int32)
    if cu.device != device:
        cu = cu.to(device, non_blocking=True)
    return cu.contiguous()


def _check_out(out, q):
    if out is None:
        return torch.empty_like(q)
    if out.shape != q.shape:
        raise ValueError(f"out must have shape {tuple(q.shape)}, got {tuple(out.shape)}")
    if out.dtype != q.dtype or out.device != q.device:
        raise ValueError(f"out must match q dtype/device, got out={out.dtype}/{out.device} q={q.dtype}/{q.device}")
    if not out.is_contiguous() or out.data_ptr() % 16:
        raise ValueError("out must be contiguous and 16-byte aligned")
    return out


def _check_head_dim(hd):
    if hd not in SUPPORTED_HEAD_DIMS:
        raise ValueError(f"head_dim {hd} is not supported by the sm_100a kernel (even values up to 128)")


def _padded_dim(hd: int) -> int:
    """Kernel head dim for ``hd``: each rotate-half half padded to a multiple of 4, at least 32 in total."""
    return max(32, 2 * (-(-(hd // 2) // 4) * 4))


def _pad_halves(x: torch.Tensor, hd: int, dp: int) -> torch.Tensor:
    """[..., hd] -> [..., dp] with x[:hd/2] at 0 and x[hd/2:] at dp/2, zeros elsewhere."""
    h, hp = hd // 2, dp // 2
    y = x.new_zeros(*x.shape[:-1], dp)
    y[..., :h] = x[..., :h]
    y[..., hp:hp + h] = x[..., h:]
    return y


def _unpad_halves(y: torch.Tensor, hd: int, dp: int) -> torch.Tensor:
    h, hp = hd // 2, dp // 2
    return torch.cat([y[..., :h], y[..., hp:hp + h]], dim=-1)


def fused_rope_attention(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    cu_seqlens: torch.Tensor,
    *,
    out: torch.Tensor | None = None,
    max_seqlen: int | None = None,
) -> torch.Tensor:
    """Fused RoPE + windowed/varlen attention over packed ``cu_seqlens`` segments.

    Same contract as the reference (fused_attn.py:139-232):

    * ``q, k, v``: ``[total_seq, num_heads, head_dim]``, float16 or bfloat16, CUDA
    * ``cos, sin``: ``[total_seq, head_dim // 2]`` (float32, float16 or bfloat16),
      split-half (NeoX) rotary applied to Q and K inside the kernel
    * ``cu_seqlens``: ``[num_windows + 1]`` cumulative lengths (cast to int32)
    * ``out``: optional preallocated output of q's shape/dtype/device

    Returns ``out`` with ``softmax(R(q) R(k)^T / sqrt(head_dim)) v`` per segment and
    head. Rows outside ``[cu_seqlens[0], cu_seqlens[-1])`` are zero.
    """
    total, heads, hd = _check_qkv(q, k, v)
    if cos.shape != (total, hd // 2) or sin.shape != (total, hd // 2):
        raise ValueError(
            f"cos/sin must be [total_seq, head_dim//2]={total, hd // 2}, got cos={tuple(cos.shape)} sin={tuple(sin.shape)}"
        )
    if cu_seqlens.ndim != 1 or cu_seqlens.numel() < 2:
        raise ValueError(f"cu_seqlens must be 1D with length >= 2, got {tuple(cu_seqlens.shape)}")
    if cos.dtype not in _DT:
        raise ValueError(f"cos dtype must be float16, bfloat16 or float32, got {cos.dtype}")
    if sin.dtype not in _DT:
        raise ValueError(f"sin dtype must be float16, bfloat16 or float32, got {sin.dtype}")
    if sin.dtype != cos.dtype:
        sin = sin.to(cos.dtype)
    _check_head_dim(hd)
    if hd not in KERNEL_HEAD_DIMS:
        # Zero-pad each half of q/k/v to the kernel's head dim. Padded lanes
        # contribute nothing to QK^T or PV; the kernel scales scores by
        # 1/sqrt(dp), so cos/sin carry (dp/hd)^(1/4) each to restore
        # 1/sqrt(hd) (fused_attn.py:355). Rotation stays in fp32.
        dp = _padded_dim(hd)
        f = (dp / hd) ** 0.25
        cs = torch.ones(total, dp // 2, dtype=torch.float32, device=q.device)
        sn = torch.zeros(total, dp // 2, dtype=torch.float32, device=q.device)
        cs[:, : hd // 2] = cos.to(q.device, torch.float32)
        sn[:, : hd // 2] = sin.to(q.device, torch.float32)
        _check_out(out, q)
        o = fused_rope_attention(_pad_halves(q, hd, dp), _pad_halves(k, hd, dp), _pad_halves(v, hd, dp),
                                 cs * f, sn * f, cu_seqlens, max_seqlen=max_seqlen)
        res = _unpad_halves(o, hd, dp)
        if out is None:
            return res.contiguous()
        out.copy_(res)
        return out
    (q, qs), (k, ks), (v, vs) = (_token_rows(t) for t in (q, k, v))
    cos = _aligned(cos.to(q.device).contiguous())
    sin = _aligned(sin.to(q.device).contiguous())
    out = _check_out(out, q)
    cu = _check_cu(cu_seqlens, q.device)
    nseg = cu.numel() - 1
    lib = _lib.load()
    ws_bytes = _lib.workspace_bytes(total, nseg)
    if not (max_seqlen and 0 < max_seqlen <= 128):
        ws_bytes += _lib.workspace_bytes_rotated_k(total, heads, hd)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream(q.device).cuda_stream
        if qs == ks == vs == heads * hd:
            rc = lib.frattn_fwd(
                q.data_ptr(), k.data_ptr(), v.data_ptr(), cos.data_ptr(), sin.data_ptr(), _DT[cos.dtype],
                cu.data_ptr(), nseg, total, heads, hd, int(max_seqlen or 0), _DT[q.dtype],
                out.data_ptr(), ws.data_ptr(), ws_bytes, _status_word(q.device).data_ptr(), stream,
            )
        else:
            rc = lib.frattn_fwd_strided(
                q.data_ptr(), k.data_ptr(), v.data_ptr(), qs, ks, vs, cos.data_ptr(), sin.data_ptr(),
                _DT[cos.dtype], cu.data_ptr(), nseg, total, heads, hd, int(max_seqlen or 0), _DT[q.dtype],
                out.data_ptr(), ws.data_ptr(), ws_bytes, _status_word(q.device).data_ptr(), stream,
            )
    _lib.check(rc, "frattn_fwd")
    return out


def fused_rope_attention_pos(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    pos_hw: torch.Tensor,
    cu_seqlens: torch.Tensor,
    *,
    theta: float = 10000.0,
    max_position: int | None = None,
    out: torch.Tensor | None = None,
    max_seqlen: int | None = None,
) -> torch.Tensor:
    """Fused RoPE + varlen attention with the rotary angles built in the kernel.

    ``pos_hw`` is int32 ``[total_seq, 2]`` holding each token's (h, w) patch
    coordinate (``rope_positions_2d`` builds it; window-shuffle it like q/k/v).
    Equivalent to ``fused_rope_attention`` with
    ``compute_rope_2d(..., dtype=torch.float32)`` tables. ``max_position`` bounds
    the coordinates (exclusive); when omitted it is read from ``pos_hw`` (one
    host sync).
    """
    total, heads, hd = _check_qkv(q, k, v)
    if pos_hw.shape != (total, 2):
        raise ValueError(f"pos_hw must be [total_seq, 2]={total, 2}, got {tuple(pos_hw.shape)}")
    if hd % 4 != 0:
        raise ValueError(f"head_dim must be divisible by 4 for 2D RoPE, got {hd}")
    if hd not in KERNEL_HEAD_DIMS:
        raise ValueError(f"head_dim {hd} is not supported by the position entry point (multiples of 8 in [32, 128])")
    pos = _aligned(pos_hw.to(device=q.device, dtype=torch.int32).contiguous())
    if max_position is None:
        max_position = int(pos.max().item()) + 1 if total > 0 else 1
    q, k, v = (_aligned(t.contiguous()) for t in (q, k, v))
    out = _check_out(out, q)
    cu = _check_cu(cu_seqlens, q.device)
    nseg = cu.numel() - 1
    lib = _lib.load()
    ws_bytes = _lib.workspace_bytes_pos(total, nseg, max_position, hd)
    if not (max_seqlen and 0 < max_seqlen <= 128):
        ws_bytes += _lib.workspace_bytes_rotated_k(total, heads, hd)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream(q.device).cuda_stream
        rc = lib.frattn_fwd_pos(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), pos.data_ptr(), int(max_position), float(theta),
            cu.data_ptr(), nseg, total, heads, hd, int(max_seqlen or 0), _DT[q.dtype],
            out.data_ptr(), ws.data_ptr(), ws_bytes, _status_word(q.device).data_ptr(), stream,
        )
    _lib.check(rc, "frattn_fwd_pos")
    return out


# --------------------------------------------------------------------------- rotation in the projection
QKV_ROPE_HEAD_DIMS = (32, 48, 64, 80, 96, 112, 128)


def qkv_rope_projection(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: torch.Tensor | None,
    cos: torch.Tensor,
    sin: torch.Tensor,
    num_heads: int,
    *,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """QKV projection with the 2D rotary embedding applied in the GEMM epilogue.

    ``x`` ``[T, K]`` (rows may be strided), ``weight`` ``[3 * num_heads * head_dim, K]``
    (``nn.Linear`` layout: q rows, then k, then v), ``bias`` ``[3 * H * D]`` or None,
    ``cos``/``sin`` ``[T, head_dim // 2]`` as for ``fused_rope_attention``.
    Returns ``[T, 3, H, D]`` with the q and k heads rotated and v as projected:
    ``linear(x, weight, bias)`` rounded to x's dtype, then rotated in fp32 and
    rounded again (the reference's caller rotates q/k in a separate pass after
    the projection, bench.py:72-78). Feed ``[:, 0]``, ``[:, 1]``, ``[:, 2]`` to
    ``fused_attention_rotated``.
    """
    if x.device.type != "cuda":
        raise ValueError(f"x must be on CUDA, got device={x.device}")
    if x.ndim != 2 or weight.ndim != 2 or weight.shape[1] != x.shape[1]:
        raise ValueError(f"x must be [T, K] and weight [N, K], got x={tuple(x.shape)} weight={tuple(weight.shape)}")
    if x.dtype not in (torch.float16, torch.bfloat16) or weight.dtype != x.dtype:
        raise ValueError(f"x and weight must share dtype float16 or bfloat16, got {x.dtype} / {weight.dtype}")
    T, K = (int(s) for s in x.shape)
    N = int(weight.shape[0])
    if num_heads <= 0 or N % (3 * num_heads):
        raise ValueError(f"weight rows {N} are not 3 * num_heads * head_dim for num_heads={num_heads}")
    hd = N // (3 * num_heads)
    if hd not in QKV_ROPE_HEAD_DIMS:
        raise ValueError(f"head_dim {hd} is not supported by the QKV projection kernel ({QKV_ROPE_HEAD_DIMS})")
    if K % 8:
        raise ValueError(f"K={K} must be a multiple of 8 (16-byte rows)")
    if cos.shape != (T, hd // 2) or sin.shape != (T, hd // 2):
        raise ValueError(f"cos/sin must be [T, head_dim//2]={T, hd // 2}, got cos={tuple(cos.shape)} sin={tuple(sin.shape)}")
    if cos.dtype not in _DT or sin.dtype not in _DT:
        raise ValueError(f"cos/sin dtype must be float16, bfloat16 or float32, got {cos.dtype} / {sin.dtype}")
    if sin.dtype != cos.dtype:
        sin = sin.to(cos.dtype)
    if bias is not None and (bias.shape != (N,) or bias.dtype != x.dtype):
        raise ValueError(f"bias must be [{N}] of dtype {x.dtype}, got {tuple(bias.shape)} {bias.dtype}")
    if not (x.stride(1) == 1 and x.stride(0) >= K and x.stride(0) % 8 == 0 and x.data_ptr() % 16 == 0):
        x = _aligned(x.contiguous())
    xs = int(x.stride(0))
    w = _aligned(weight.contiguous())
    b = _aligned(bias.contiguous()) if bias is not None else None
    cos = _aligned(cos.to(x.device).contiguous())
    sin = _aligned(sin.to(x.device).contiguous())
    if out is None:
        out = torch.empty(T, 3, num_heads, hd, dtype=x.dtype, device=x.device)
    elif out.shape != (T, 3, num_heads, hd) or out.dtype != x.dtype or not out.is_contiguous() or out.data_ptr() % 16:
        raise ValueError(f"out must be a contiguous 16-byte aligned [{T}, 3, {num_heads}, {hd}] {x.dtype} tensor")
    if T == 0:
        return out
    lib = _lib.load()
    with torch.cuda.device(x.device):
        stream = torch.cuda.current_stream(x.device).cuda_stream
        rc = lib.frattn_qkv_rope(
            x.data_ptr(), xs, w.data_ptr(), b.data_ptr() if b is not None else None, cos.data_ptr(),
            sin.data_ptr(), _DT[cos.dtype], T, K, num_heads, hd, _DT[x.dtype], out.data_ptr(),
            _status_word(x.device).data_ptr(), stream,
        )
    _lib.check(rc, "frattn_qkv_rope")
    return out


def fused_attention_rotated(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    cu_seqlens: torch.Tensor,
    *,
    out: torch.Tensor | None = None,
    max_seqlen: int | None = None,
) -> torch.Tensor:
    """Varlen attention for q and k that are already rotated (``qkv_rope_projection``).

    ``fused_rope_attention`` without the tables: same shapes, dtypes, ``cu_seqlens``
    and ``max_seqlen`` contract, same kernels minus the rotation.
    """
    total, heads, hd = _check_qkv(q, k, v)
    if hd not in KERNEL_HEAD_DIMS:
        raise ValueError(f"head_dim {hd} is not supported (multiples of 8 in [32, 128])")
    if cu_seqlens.ndim != 1 or cu_seqlens.numel() < 2:
        raise ValueError(f"cu_seqlens must be 1D with length >= 2, got {tuple(cu_seqlens.shape)}")
    (q, qs), (k, ks), (v, vs) = (_token_rows(t) for t in (q, k, v))
    out = _check_out(out, q)
    cu = _check_cu(cu_seqlens, q.device)
    nseg = cu.numel() - 1
    lib = _lib.load()
    ws_bytes = _lib.workspace_bytes(total, nseg)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    with torch.cuda.device(q.device):
        stream = torch.cuda.current_stream(q.device).cuda_stream
        rc = lib.frattn_fwd_rotated(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), qs, ks, vs, cu.data_ptr(), nseg, total, heads, hd,
            int(max_seqlen or 0), _DT[q.dtype], out.data_ptr(), ws.data_ptr(), ws_bytes,
            _status_word(q.device).data_ptr(), stream,
        )
    _lib.check(rc, "frattn_fwd_rotated")
    return out


# --------------------------------------------------------------------------- backward
BACKWARD_HEAD_DIMS = (32, 48, 64, 80, 96, 112, 128)


def _fwd_lse(q, k, v, cos, sin, cu, max_seqlen):
    """Forward that also returns lse [T, H] (fp32, base-2 log-sum-exp of the scaled scores)."""
    total, heads, hd = (int(x) for x in q.shape)
    out = torch.empty_like(q)
    lse = torch.empty(total, heads, dtype=torch.float32, device=q.device)
    nseg = cu.numel() - 1
    lib = _lib.load()
    ws_bytes = _lib.workspace_bytes(total, nseg)
    if not (max_seqlen and 0 < max_seqlen <= 128):
        ws_bytes += _lib.workspace_bytes_rotated_k(total, heads, hd)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    with torch.cuda.device(q.device):
        rc = lib.frattn_fwd_lse(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), cos.data_ptr(), sin.data_ptr(), _DT[cos.dtype], cu.data_ptr(),
            nseg, total, heads, hd, int(max_seqlen or 0), _DT[q.dtype], out.data_ptr(), lse.data_ptr(),
            ws.data_ptr(), ws_bytes, _status_word(q.device).data_ptr(), torch.cuda.current_stream(q.device).cuda_stream,
        )
    _lib.check(rc, "frattn_fwd_lse")
    return out, lse


def _bwd(q, k, v, cos, sin, cu, out, lse, dout):
    total, heads, hd = (int(x) for x in q.shape)
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    if total == 0:
        return dq, dk, dv
    dout = _aligned(dout.contiguous())
    ws_bytes = _lib.workspace_bytes_bwd(total, heads, hd)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    lib = _lib.load()
    with torch.cuda.device(q.device):
        rc = lib.frattn_bwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), cos.data_ptr(), sin.data_ptr(), _DT[cos.dtype], cu.data_ptr(),
            cu.numel() - 1, total, heads, hd, _DT[q.dtype], out.data_ptr(), dout.data_ptr(), lse.data_ptr(),
            dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), ws.data_ptr(), ws_bytes, _status_word(q.device).data_ptr(),
            torch.cuda.current_stream(q.device).cuda_stream,
        )
    _lib.check(rc, "frattn_bwd")
    return dq, dk, dv


class _FusedRopeAttention(torch.autograd.Function):
    """Autograd node of ``fused_rope_attention``: the forward saves lse, the
    backward runs the sm_100a backward kernels (frattn_bwd). No gradient flows
    to cos/sin or cu_seqlens."""

    @staticmethod
    def forward(ctx, q, k, v, cos, sin, cu, max_seqlen):
        out, lse = _fwd_lse(q, k, v, cos, sin, cu, max_seqlen)
        ctx.save_for_backward(q, k, v, cos, sin, cu, out, lse)
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, cos, sin, cu, out, lse = ctx.saved_tensors
        dq, dk, dv = _bwd(q, k, v, cos, sin, cu, out, lse, dout)
        return dq, dk, dv, None, None, None, None


def fused_rope_attention_train(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    cu_seqlens: torch.Tensor,
    *,
    max_seqlen: int | None = None,
) -> torch.Tensor:
    """``fused_rope_attention`` with gradients for q, k and v (head_dim in
    ``BACKWARD_HEAD_DIMS``). The reference is forward-only; this is the same
    forward recording an autograd node whose backward is the sm_100a backward pass."""
    total, heads, hd = _check_qkv(q, k, v)
    if hd not in BACKWARD_HEAD_DIMS:
        raise ValueError(f"head_dim {hd} has no backward kernel ({BACKWARD_HEAD_DIMS})")
    if cos.shape != (total, hd // 2) or sin.shape != (total, hd // 2):
        raise ValueError(
            f"cos/sin must be [total_seq, head_dim//2]={total, hd // 2}, got cos={tuple(cos.shape)} sin={tuple(sin.shape)}"
        )
    if cos.dtype not in _DT or sin.dtype not in _DT:
        raise ValueError(f"cos/sin dtype must be float16, bfloat16 or float32, got {cos.dtype} / {sin.dtype}")
    if sin.dtype != cos.dtype:
        sin = sin.to(cos.dtype)
    q, k, v = (_aligned(t.contiguous()) for t in (q, k, v))
    cos = _aligned(cos.to(q.device).contiguous()).detach()
    sin = _aligned(sin.to(q.device).contiguous()).detach()
    cu = _check_cu(cu_seqlens, q.device)
    return _FusedRopeAttention.apply(q, k, v, cos, sin, cu, max_seqlen)


# --------------------------------------------------------------------------- FP8 q / k
def fused_rope_attention_fp8(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    cos: torch.Tensor,
    sin: torch.Tensor,
    cu_seqlens: torch.Tensor,
    *,
    out: torch.Tensor | None = None,
    max_seqlen: int | None = None,
) -> torch.Tensor:
    """``fused_rope_attention`` with R(q) R(k)^T on the FP8 tensor cores.

    q and k are rotated and rounded to e4m3 once per call (a scale per q row and
    per k head), P V stays in q's dtype. Same arguments and checks as
    ``fused_rope_attention``; head_dim a multiple of 16 in [32, 128]. Meant for
    long segments (full-attention layers).
    """
    total, heads, hd = _check_qkv(q, k, v)
    if hd % 16 or not 32 <= hd <= 128:
        raise ValueError(f"head_dim {hd} is not supported by the FP8 path (multiples of 16 in [32, 128])")
    if cos.shape != (total, hd // 2) or sin.shape != (total, hd // 2):
        raise ValueError(
            f"cos/sin must be [total_seq, head_dim//2]={total, hd // 2}, got cos={tuple(cos.shape)} sin={tuple(sin.shape)}"
        )
    if cos.dtype not in _DT or sin.dtype not in _DT:
        raise ValueError(f"cos/sin dtype must be float16, bfloat16 or float32, got {cos.dtype} / {sin.dtype}")
    if sin.dtype != cos.dtype:
        sin = sin.to(cos.dtype)
    if cu_seqlens.ndim != 1 or cu_seqlens.numel() < 2:
        raise ValueError(f"cu_seqlens must be 1D with length >= 2, got {tuple(cu_seqlens.shape)}")
    q, k, v = (_aligned(t.contiguous()) for t in (q, k, v))
    cos = _aligned(cos.to(q.device).contiguous())
    sin = _aligned(sin.to(q.device).contiguous())
    out = _check_out(out, q)
    cu = _check_cu(cu_seqlens, q.device)
    nseg = cu.numel() - 1
    lib = _lib.load()
    ws_bytes = _lib.workspace_bytes_fp8(total, nseg, heads, hd)
    ws = torch.empty(ws_bytes + 256, dtype=torch.uint8, device=q.device)
    off = (-ws.data_ptr()) % 256
    with torch.cuda.device(q.device):
        rc = lib.frattn_fwd_fp8(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), cos.data_ptr(), sin.data_ptr(), _DT[cos.dtype], cu.data_ptr(),
            nseg, total, heads, hd, int(max_seqlen or 0), _DT[q.dtype], out.data_ptr(), ws.data_ptr() + off, ws_bytes,
            _status_word(q.device).data_ptr(), torch.cuda.current_stream(q.device).cuda_stream,
        )
    _lib.check(rc, "frattn_fwd_fp8")
    return out
