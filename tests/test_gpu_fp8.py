"""FP8 (e4m3) q/k variant (frattn_fwd_fp8).

Two checks per case:
* against an e4m3-emulated reference: q, k rotated in fp32 and rounded to e4m3
  with the kernel's scales (max |row| / 448 per q row, max |k| / 448 per head),
  then the oracle's attention (utils.py:178-193) on the dequantised values. This
  pins the kernel's FP8 arithmetic (layouts, scales) at the bf16 kernels'
  tolerance: max-abs <= 2e-2, mean-abs <= 2e-3;
* against the fp32 oracle of the reference's unfused path (bench.py:73-78 RoPE +
  attention) at the FP8 bound: mean-abs <= 4e-3 (twice the bf16 bound) and
  max-abs <= 8e-2. e4m3 keeps 3 mantissa bits, so scores carry ~2^-5 relative
  error per product; measured on N(0,1) inputs: mean 0.8e-3 to 2.7e-3, max
  1.4e-2 (4096-token segment) to 6.5e-2 (a 5-token segment, peaky softmax).
Also the 32-layer encoder drift with FP8 full-attention layers."""
import numpy as np
import pytest
import torch

from gpu_cases import cu_case, grid_case
from fused_rope_attn_b200 import fused_rope_attention, fused_rope_attention_fp8, last_status
from fused_rope_attn_b200.encoder import EncoderConfig, VisionEncoder, encoder_inputs, rel_l2
from oracle import rope_attn_oracle as O

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def e4m3(x):
    return torch.from_numpy(np.ascontiguousarray(x)).to(torch.float8_e4m3fn).float().numpy()


def emulate_fp8(qf, kf):
    """Dequantised e4m3 copies of rotated q [T,H,D] and k with the kernel's scales."""
    sq = np.abs(qf).max(axis=-1, keepdims=True) / 448.0
    sq = np.where(sq > 0, sq, 1.0).astype(np.float32)
    sk = np.abs(kf).max(axis=(0, 2), keepdims=True) / 448.0
    sk = np.where(sk > 0, sk, 1.0).astype(np.float32)
    return e4m3(qf / sq) * sq, e4m3(kf / sk) * sk


def check(out, q, k, v, cos, sin, cu, rows=None):
    qf, kf = (O.apply_rope(t.float().numpy(), cos.float().numpy(), sin.float().numpy()) for t in (q, k))
    qe, ke = emulate_fp8(qf, kf)
    vf = v.float().numpy()
    got = out.float().cpu().numpy()
    if rows is None:
        ref = O.varlen_attention(qf, kf, vf, cu.numpy())
        emu = O.varlen_attention(qe, ke, vf, cu.numpy())
    else:
        ref = O.varlen_attention_rows(qf, kf, vf, cu.numpy(), rows)
        emu = O.varlen_attention_rows(qe, ke, vf, cu.numpy(), rows)
        got = got[rows]
    assert np.isfinite(got).all()
    e_emu, e_ref = np.abs(got - emu), np.abs(got - ref)
    assert e_emu.max() <= 2e-2 and e_emu.mean() <= 2e-3, ("vs e4m3 emulation", float(e_emu.max()), float(e_emu.mean()))
    assert e_ref.max() <= 8e-2 and e_ref.mean() <= 4e-3, ("vs fp32 oracle", float(e_ref.max()), float(e_ref.mean()))
    print(f"fp8: vs emulation max {e_emu.max():.3e} mean {e_emu.mean():.3e}; vs fp32 max {e_ref.max():.3e} "
          f"mean {e_ref.mean():.3e}")
    return float(e_ref.max()), float(e_ref.mean())


@pytest.mark.parametrize("cu,H,D,dtype,cs_dtype", [
    ([0, 700, 1000], 2, 80, torch.bfloat16, torch.float32),
    ([0, 5, 133, 261, 400, 1400], 3, 80, torch.bfloat16, torch.float32),   # short and long segments
    ([0, 512, 1024], 2, 64, torch.float16, torch.bfloat16),
    ([0, 300, 900], 2, 128, torch.bfloat16, torch.float32),
    ([0, 640], 2, 96, torch.bfloat16, torch.float16),
    ([0, 0, 257, 257, 600], 1, 48, torch.bfloat16, torch.float32),          # empty segments
])
def test_fp8_matches_oracle(cu, H, D, dtype, cs_dtype):
    q, k, v, cos, sin, cut = cu_case(cu, H=H, D=D, dtype=dtype, cs_dtype=cs_dtype)
    out = fused_rope_attention_fp8(q.to(DEV), k.to(DEV), v.to(DEV), cos.to(DEV), sin.to(DEV), cut.to(DEV))
    torch.cuda.synchronize()
    assert last_status(DEV) == 0
    check(out, q, k, v, cos, sin, cut)


def test_fp8_full_896_layer():
    """Config 2b: one 4096-token segment, 16 heads of 80, 2D-grid RoPE; a row sample
    against the oracle, and the whole output against the bf16 kernel."""
    q, k, v, cos, sin, cu = grid_case([(1, 64, 64)], windowed=False)
    args = [t.to(DEV) for t in (q, k, v, cos, sin, cu)]
    out = fused_rope_attention_fp8(*args)
    ref16 = fused_rope_attention(*args)
    torch.cuda.synchronize()
    rows = np.random.default_rng(0).choice(4096, 256, replace=False)
    mx, mean = check(out, q, k, v, cos, sin, cu, rows)
    d = (out.float() - ref16.float()).abs()
    print(f"fp8 vs oracle (256 rows): max {mx:.3e} mean {mean:.3e}; vs bf16 kernel: max {d.max():.3e} mean {d.mean():.3e}")
    assert d.max().item() <= 4e-2 and d.mean().item() <= 4e-3


def test_fp8_large_values_stay_finite():
    """Per-row q scales and a per-head k scale: inputs 100x larger quantise the same way."""
    q, k, v, cos, sin, cu = cu_case([0, 600], H=2, D=80)
    a = fused_rope_attention_fp8(*(t.to(DEV) for t in (q, k, v, cos, sin, cu)))
    b = fused_rope_attention_fp8(*(t.to(DEV) for t in ((q * 100).to(q.dtype), k, v, cos, sin, cu)))
    torch.cuda.synchronize()
    assert torch.isfinite(a).all() and torch.isfinite(b).all()


def test_fp8_encoder_drift_448():
    """32 layers, full layers through FP8: relative L2 drift from the fp32 stack stays
    within 1.5x of the bf16 fused path's drift (measured and printed)."""
    grid = [(1, 32, 32)]
    cfg = EncoderConfig()
    enc = VisionEncoder(cfg, device="cuda", dtype=torch.bfloat16)
    x = encoder_inputs(grid, cfg.hidden, seed=0, device="cuda")
    plan = enc.plan(grid)
    f16 = enc(x, grid, attn="fused", plan=plan)
    f8 = enc(x, grid, attn="fused_fp8", plan=plan)
    ref = VisionEncoder(cfg, device="cuda", dtype=torch.float32)(x.float(), grid, attn="fp32")
    torch.cuda.synchronize()
    d16, d8 = rel_l2(f16, ref), rel_l2(f8, ref)
    print(f"32-layer relL2 vs fp32: bf16 fused {d16:.4e}, fp8 full layers {d8:.4e}")
    assert torch.isfinite(f8.float()).all()
    assert d8 <= 1.5 * d16 + 2e-3
