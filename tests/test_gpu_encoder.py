"""32-layer random-weight Qwen2.5-VL-style encoder: fused attention vs unfused and fp32.

Drift is the relative L2 distance of the final hidden states. The fused path
must drift from the fp32 stack no more than the unfused (separate RoPE +
FlashAttention varlen) bf16 path does, within 10 % plus a small slack.
Measured on B200 (448x448, 1024 tokens): fused 2.05e-2, unfused 2.05e-2,
fused vs unfused 2.3e-2 (the same at 1344x1344).
"""
import pytest
import torch

from fused_rope_attn_b200.encoder import EncoderConfig, VisionEncoder, encoder_inputs, rel_l2

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def outputs():
    grid = [(1, 32, 32)]
    cfg = EncoderConfig()
    enc = VisionEncoder(cfg, device="cuda", dtype=torch.bfloat16)
    x = encoder_inputs(grid, cfg.hidden, seed=0, device="cuda")
    plan = enc.plan(grid)
    fused = enc(x, grid, attn="fused", plan=plan)
    unfused = enc(x, grid, attn="unfused", plan=plan)
    enc32 = VisionEncoder(cfg, device="cuda", dtype=torch.float32)
    ref = enc32(x.float(), grid, attn="fp32")
    torch.cuda.synchronize()
    return fused, unfused, ref


def test_32_layer_drift_no_worse_than_unfused(outputs):
    fused, unfused, ref = outputs
    d_f, d_u = rel_l2(fused, ref), rel_l2(unfused, ref)
    print(f"relL2 fused-vs-fp32={d_f:.4e} unfused-vs-fp32={d_u:.4e} fused-vs-unfused={rel_l2(fused, unfused):.4e}")
    assert torch.isfinite(fused.float()).all()
    assert d_f <= 1.1 * d_u + 2e-3
    assert d_f < 5e-2


def test_windowed_and_full_layer_match_unfused():
    """One encoder layer of each kind (the attention output feeds the residual)."""
    grid = [(1, 32, 32)]
    for full in ((0,), ()):
        cfg = EncoderConfig(depth=1, full_layers=full)
        enc = VisionEncoder(cfg, device="cuda", dtype=torch.bfloat16)
        x = encoder_inputs(grid, cfg.hidden, seed=1, device="cuda")
        a = enc(x, grid, attn="fused").float()
        b = enc(x, grid, attn="unfused").float()
        err = (a - b).abs()
        assert err.max().item() <= 2e-2 * max(1.0, b.abs().max().item()) and err.mean().item() <= 2e-3
