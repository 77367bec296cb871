"""QKV projection with RoPE in the GEMM epilogue (frattn_qkv_rope) and attention on
pre-rotated q/k (frattn_fwd_rotated), against the CPU oracle.

The oracle restates the reference caller's composition (bench.py:72-78): the
projection's output in the input type, then the split-half rotation of q and k in
fp32 rounded once more. The GPU kernel accumulates in a different order than numpy,
so a value whose fp32 sum lies next to a rounding boundary may land one unit in the
last place away; the tests bound those cases (count and size) instead of asking for
bit equality.
"""
import numpy as np
import pytest
import torch

from gpu_cases import cu_case
from fused_rope_attn_b200 import (fused_attention_rotated, fused_rope_attention, last_status,
                                  qkv_rope_projection)
from fused_rope_attn_b200.utils import get_window_index, segments_per_image
from fused_rope_attn_b200 import compute_rope_2d
from oracle import rope_attn_oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
NP_DT = {torch.bfloat16: "bfloat16", torch.float16: "float16"}


def proj_inputs(T, K, H, D, dtype, cs_dtype=torch.float32, bias=True, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, K, generator=g).to(dtype)
    w = (torch.randn(3 * H * D, K, generator=g) * 0.02).to(dtype)
    b = (torch.randn(3 * H * D, generator=g) * 0.02).to(dtype) if bias else None
    ang = torch.rand(T, D // 2, generator=g) * 20.0
    return x, w, b, ang.cos().to(cs_dtype), ang.sin().to(cs_dtype)


def check_close_to_rounding(got, ref, ulp_frac=0.02):
    """got/ref fp32 arrays of values rounded to a 16-bit type: equal except for a few
    one-rounding-step differences (fp32 summation order)."""
    d = np.abs(got - ref)
    # a rotated value can be a small difference of large products: measure the step
    # against the magnitude of its head row as well as its own
    rms = np.sqrt(np.mean(ref * ref, axis=-1, keepdims=True))
    scale = np.abs(ref) + rms + 1e-6
    diag = f"max abs {d.max():.3e}, max rel {(d / scale).max():.3e}, differing {np.mean(d > 0):.4f}"
    assert np.isfinite(got).all()
    assert (d <= scale * 2.0 ** -6).all(), diag
    assert np.mean(d > 0) <= ulp_frac, diag


@pytest.mark.parametrize("T,K,H,D,dtype,cs_dtype,bias", [
    (300, 256, 2, 80, torch.bfloat16, torch.float32, True),
    (1000, 1280, 16, 80, torch.bfloat16, torch.float32, True),   # encoder width
    (129, 64, 1, 64, torch.bfloat16, torch.bfloat16, False),     # one K block, ragged T
    (257, 200, 3, 128, torch.float16, torch.float16, True),      # K not a multiple of 64
    (64, 512, 5, 32, torch.bfloat16, torch.float32, True),       # 8 heads per N tile, partial tile
    (200, 320, 4, 48, torch.bfloat16, torch.float32, True),
    (190, 96, 2, 96, torch.bfloat16, torch.float32, True),
    (130, 136, 2, 112, torch.float16, torch.float32, False),
])
def test_qkv_rope_matches_oracle(T, K, H, D, dtype, cs_dtype, bias):
    x, w, b, cos, sin = proj_inputs(T, K, H, D, dtype, cs_dtype, bias)
    got = qkv_rope_projection(x.to(DEV), w.to(DEV), b.to(DEV) if b is not None else None, cos.to(DEV),
                              sin.to(DEV), H)
    torch.cuda.synchronize()
    assert last_status(DEV) == 0
    assert got.shape == (T, 3, H, D)
    ref = O.qkv_rope(x.float().numpy(), w.float().numpy(), b.float().numpy() if b is not None else None,
                     cos.float().numpy(), sin.float().numpy(), H, NP_DT[dtype])
    check_close_to_rounding(got.float().cpu().numpy(), ref)


def test_qkv_rope_strided_rows_and_out():
    T, K, H, D = 256, 192, 2, 80
    x, w, b, cos, sin = proj_inputs(T, K, H, D, torch.bfloat16)
    xbig = torch.zeros(T, K + 64, dtype=torch.bfloat16)
    xbig[:, :K] = x
    xv = xbig.to(DEV)[:, :K]                       # row stride K + 64 elements, read in place
    out = torch.empty(T, 3, H, D, dtype=torch.bfloat16, device=DEV)
    got = qkv_rope_projection(xv, w.to(DEV), b.to(DEV), cos.to(DEV), sin.to(DEV), H, out=out)
    assert got.data_ptr() == out.data_ptr()
    ref = O.qkv_rope(x.float().numpy(), w.float().numpy(), b.float().numpy(), cos.numpy(), sin.numpy(), H)
    check_close_to_rounding(got.float().cpu().numpy(), ref)


def test_qkv_rope_empty_and_errors():
    x, w, b, cos, sin = proj_inputs(0, 64, 1, 64, torch.bfloat16)
    out = qkv_rope_projection(x.to(DEV), w.to(DEV), b.to(DEV), cos.to(DEV), sin.to(DEV), 1)
    assert out.shape == (0, 3, 1, 64)
    x, w, b, cos, sin = proj_inputs(8, 64, 1, 72, torch.bfloat16)
    with pytest.raises(ValueError):
        qkv_rope_projection(x.to(DEV), w.to(DEV), b.to(DEV), cos.to(DEV), sin.to(DEV), 1)  # D=72
    x, w, b, cos, sin = proj_inputs(8, 60, 1, 64, torch.bfloat16)
    with pytest.raises(ValueError):
        qkv_rope_projection(x.to(DEV), w.to(DEV), b.to(DEV), cos.to(DEV), sin.to(DEV), 1)  # K % 8
    with pytest.raises(ValueError):
        qkv_rope_projection(x.to(DEV), w.to(DEV), b.to(DEV), cos.to(DEV), sin.to(DEV), 5)  # rows vs heads


def test_qkv_rope_full_encoder_shape_against_cublas():
    """9216 x 1280 -> 3840 (one 1344x1344 layer): the same composition on the GPU with
    cuBLAS in fp32 (size-independent check of every tile of the persistent grid)."""
    T, K, H, D = 9216, 1280, 16, 80
    g = torch.Generator(device=DEV).manual_seed(3)
    x = torch.randn(T, K, generator=g, device=DEV).to(torch.bfloat16)
    w = (torch.randn(3 * H * D, K, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    b = (torch.randn(3 * H * D, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    ang = torch.rand(T, D // 2, generator=g, device=DEV) * 50
    cos, sin = ang.cos(), ang.sin()
    got = qkv_rope_projection(x, w, b, cos, sin, H)
    y = (x.float() @ w.float().T + b.float()).to(torch.bfloat16).float().view(T, 3, H, D)

    def rope(t):
        c, s = cos[:, None, :], sin[:, None, :]
        return torch.cat([t[..., :D // 2] * c - t[..., D // 2:] * s, t[..., :D // 2] * s + t[..., D // 2:] * c], -1)

    ref = torch.stack([rope(y[:, 0]).to(torch.bfloat16).float(), rope(y[:, 1]).to(torch.bfloat16).float(), y[:, 2]],
                      dim=1)
    torch.cuda.synchronize()
    assert last_status(DEV) == 0
    check_close_to_rounding(got.float().cpu().numpy(), ref.cpu().numpy())


def _rotated(q, k, cos, sin, dtype):
    qr = O.apply_rope(q.float().numpy(), cos.float().numpy(), sin.float().numpy(), NP_DT[dtype])
    kr = O.apply_rope(k.float().numpy(), cos.float().numpy(), sin.float().numpy(), NP_DT[dtype])
    return torch.from_numpy(qr).to(dtype), torch.from_numpy(kr).to(dtype)


@pytest.mark.parametrize("cu,H,D,hint", [
    ([0, 64, 128, 192, 256, 300], 2, 80, 64),      # window kernel
    ([0, 64, 128, 192, 256, 300], 2, 80, None),    # general path, packed items
    ([0, 700, 1000], 2, 80, None),                 # long segments
    ([0, 5, 133, 261, 400], 3, 64, None),          # mixed
    ([0, 64, 128, 200], 2, 128, 128),              # head dim without a window kernel
    ([0, 300, 364], 2, 96, None),
    ([0, 1, 2, 130, 258, 259], 1, 48, 128),
])
def test_attention_on_rotated_inputs_matches_oracle(cu, H, D, hint):
    q, k, v, cos, sin, cut = cu_case(cu, H=H, D=D)
    qr, kr = _rotated(q, k, cos, sin, torch.bfloat16)
    out = fused_attention_rotated(qr.to(DEV), kr.to(DEV), v.to(DEV), cut.to(DEV), max_seqlen=hint)
    torch.cuda.synchronize()
    assert last_status(DEV) == 0
    ref = O.varlen_attention(qr.float().numpy(), kr.float().numpy(), v.float().numpy(), cut.numpy())
    err = np.abs(out.float().cpu().numpy() - ref)
    assert err.max() <= 2e-2 and err.mean() <= 2e-3, (float(err.max()), float(err.mean()))


@pytest.mark.parametrize("windowed", [True, False])
def test_projection_then_rotated_attention_matches_unfused(windowed):
    """Encoder block shape at 448x448: the pre-rotated pipeline against the reference's
    unfused path (projection, separate RoPE, attention; fp32 oracle)."""
    grid = [(1, 32, 32)]
    H, D, K = 16, 80, 1280
    if windowed:
        widx, cu = get_window_index(grid)
        cos, sin = compute_rope_2d(grid, D, 2, 10000.0, "cpu", torch.float32, window_idx=widx)
    else:
        cu = segments_per_image(grid)
        cos, sin = compute_rope_2d(grid, D, 2, 10000.0, "cpu", torch.float32)
    T = int(cu[-1])
    x, w, b, _, _ = proj_inputs(T, K, H, D, torch.bfloat16, seed=5)
    qkv = qkv_rope_projection(x.to(DEV), w.to(DEV), b.to(DEV), cos.to(DEV), sin.to(DEV), H)
    hint = 64 if windowed else T
    out = fused_attention_rotated(qkv[:, 0], qkv[:, 1], qkv[:, 2], cu.to(DEV), max_seqlen=hint)
    torch.cuda.synchronize()
    assert last_status(DEV) == 0
    y = O.round_to(x.float().numpy() @ w.float().numpy().T + b.float().numpy(), "bfloat16").reshape(T, 3, H, D)
    ref = O.rope_attention(y[:, 0], y[:, 1], y[:, 2], cos.numpy(), sin.numpy(), cu.numpy())
    err = np.abs(out.float().cpu().numpy() - ref)
    assert err.max() <= 2e-2 and err.mean() <= 2e-3, (float(err.max()), float(err.mean()))
    # and the same numbers as the table-driven kernel on the unrotated projection
    yq = torch.from_numpy(y).to(torch.bfloat16).to(DEV)
    o2 = fused_rope_attention(yq[:, 0], yq[:, 1], yq[:, 2], cos.to(DEV), sin.to(DEV), cu.to(DEV), max_seqlen=hint)
    assert (out.float() - o2.float()).abs().max().item() <= 2e-2


@pytest.mark.parametrize("T,K,H,D", [(9216, 1280, 16, 80), (300, 200, 3, 64), (513, 136, 2, 128), (257, 96, 5, 48)])
def test_cta_pairs_equal_single_ctas(T, K, H, D):
    """The CTA-pair kernel (M = 256 over two SMs) and the single-CTA kernel compute
    every output element with the same K order: identical results, ragged T included."""
    from fused_rope_attn_b200 import _lib
    x, w, b, cos, sin = proj_inputs(T, K, H, D, torch.bfloat16, seed=4)
    args = (x.to(DEV), w.to(DEV), b.to(DEV), cos.to(DEV), sin.to(DEV), H)
    lib = _lib.load()
    try:
        lib.frattn_qkv_rope_set_pairs(0)
        single = qkv_rope_projection(*args)
        lib.frattn_qkv_rope_set_pairs(1)
        pairs = qkv_rope_projection(*args)
        torch.cuda.synchronize()
    finally:
        lib.frattn_qkv_rope_set_pairs(1)
    assert last_status(DEV) == 0
    assert torch.equal(single, pairs), (single.float() - pairs.float()).abs().max().item()
