"""Backward pass (frattn_bwd) and the forward's log-sum-exp (frattn_fwd_lse) against
an fp32 PyTorch autograd reference of the reference's unfused path (separate RoPE,
bench.py:73-78, then per-segment softmax attention, utils.py:178-193).

The reference is forward-only; the gradients are checked against autograd of that
composition in fp32. The kernels round P and dS to the input type before the
tensor-core products (as flash-attention backward passes do), so the bound is
relative: rel-L2 <= 2e-2 per gradient and max-abs <= 5e-2 of the gradient's scale.
"""
import math

import numpy as np
import pytest
import torch

from gpu_cases import cu_case
from fused_rope_attn_b200 import fused_rope_attention, fused_rope_attention_train, last_status
from fused_rope_attn_b200 import fused_attn as FA

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def reference_grads(q, k, v, cos, sin, cu, dout):
    """fp32 autograd of RoPE + per-segment attention; returns (out, lse2, dq, dk, dv)."""
    q32, k32, v32 = (t.detach().float().to(DEV).requires_grad_(True) for t in (q, k, v))
    c, s = cos.float().to(DEV)[:, None, :], sin.float().to(DEV)[:, None, :]
    D = q.shape[-1]

    def rope(x):
        x0, x1 = x[..., :D // 2], x[..., D // 2:]
        return torch.cat([x0 * c - x1 * s, x0 * s + x1 * c], -1)

    qr, kr = rope(q32), rope(k32)
    out = torch.zeros_like(q32)
    lse = torch.full(q.shape[:2], float("-inf"), device=DEV)
    cl = [int(x) for x in cu]
    outs = []
    for a, b in zip(cl[:-1], cl[1:]):
        if b <= a:
            continue
        sc = torch.einsum("qhd,khd->hqk", qr[a:b], kr[a:b]) / math.sqrt(D)
        lse[a:b] = (torch.logsumexp(sc, -1) / math.log(2)).T.detach()
        o = torch.einsum("hqk,khd->qhd", torch.softmax(sc, -1), v32[a:b])
        outs.append((a, b, o))
    parts = []
    prev = 0
    for a, b, o in outs:
        if a > prev:
            parts.append(torch.zeros_like(q32[prev:a]))
        parts.append(o)
        prev = b
    if prev < q.shape[0]:
        parts.append(torch.zeros_like(q32[prev:]))
    out = torch.cat(parts) if parts else torch.zeros_like(q32)
    out.backward(dout.float().to(DEV))
    return out.detach(), lse, q32.grad, k32.grad, v32.grad


def rel_l2(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30))


def run_case(cu_list, H, D, dtype=torch.bfloat16, cs_dtype=torch.float32, T=None, hint=None, seed=0):
    q, k, v, cos, sin, cu = cu_case(cu_list, H=H, D=D, dtype=dtype, cs_dtype=cs_dtype, T=T, seed=seed)
    g = torch.Generator().manual_seed(seed + 11)
    dout = torch.randn(q.shape, generator=g).to(dtype)
    qd, kd, vd = (t.to(DEV).requires_grad_(True) for t in (q, k, v))
    out = fused_rope_attention_train(qd, kd, vd, cos.to(DEV), sin.to(DEV), cu.to(DEV), max_seqlen=hint)
    out.backward(dout.to(DEV))
    torch.cuda.synchronize()
    assert last_status(DEV) == 0
    ro, rl, rdq, rdk, rdv = reference_grads(q, k, v, cos, sin, cu.tolist(), dout)
    err = (out.detach().float() - ro).abs()
    assert err.max().item() <= 2e-2 and err.mean().item() <= 2e-3
    for name, got, ref in (("dq", qd.grad, rdq), ("dk", kd.grad, rdk), ("dv", vd.grad, rdv)):
        assert got.dtype == dtype and got.shape == ref.shape
        r = rel_l2(got, ref)
        m = (got.float() - ref).abs().max().item()
        scale = ref.abs().max().item() + 1e-6
        assert torch.isfinite(got).all(), name
        assert r <= 2e-2 and m <= 5e-2 * scale, (name, r, m, scale)
    return qd, kd, vd, out


@pytest.mark.parametrize("cu,H,D,hint", [
    ([0, 64, 128, 192, 256, 320], 2, 80, 64),          # windows (window kernel forward)
    ([0, 700, 1000], 2, 80, None),                     # long segments, many q tiles per key chunk
    ([0, 5, 133, 261, 400], 3, 80, None),              # mixed, chunks straddling segments
    ([0, 1, 2, 130, 258, 259], 1, 64, None),           # one-token segments
    ([0, 0, 200, 200, 330], 2, 48, None),              # empty segments
    ([0, 256, 512], 2, 32, None),
    ([0, 300, 700], 2, 96, None),
    ([0, 64, 128, 200, 520], 2, 112, 128),
    ([0, 400, 660], 2, 128, None),                     # one Q/dO stage (shared memory)
])
def test_backward_matches_fp32_autograd(cu, H, D, hint):
    run_case(cu, H, D, hint=hint)


def test_backward_fp16_and_bf16_tables():
    run_case([0, 100, 300, 428], 2, 80, dtype=torch.float16, cs_dtype=torch.bfloat16)


def test_backward_rows_outside_segments_get_zero():
    qd, kd, vd, _ = run_case([10, 150, 290], 2, 64, T=300)
    for g in (qd.grad, kd.grad, vd.grad):
        assert g[:10].abs().max().item() == 0 and g[290:].abs().max().item() == 0


def test_backward_full_896_layer():
    """Config 2b (one 4096-token segment, 16 heads of 80) at full size."""
    run_case([0, 4096], 16, 80, seed=3)


def test_forward_lse_and_output():
    q, k, v, cos, sin, cu = cu_case([0, 64, 300, 1000], H=2, D=80)
    out, lse = FA._fwd_lse(*(t.to(DEV) for t in (q, k, v, cos, sin, cu)), None)
    ref_out = fused_rope_attention(*(t.to(DEV) for t in (q, k, v, cos, sin, cu)))
    assert torch.equal(out, ref_out)
    _, rl, *_ = reference_grads(q, k, v, cos, sin, cu.tolist(), torch.zeros(q.shape))
    assert (lse - rl).abs().max().item() <= 1e-2  # log2 units; rotated q/k are rounded to bf16 here
    out2, lse2 = FA._fwd_lse(*(t.to(DEV) for t in (q, k, v, cos, sin, cu)), 64)  # window-hint path
    torch.cuda.synchronize()
    assert torch.isfinite(lse2).all()


def test_backward_rejects_unsupported_head_dim():
    q, k, v, cos, sin, cu = cu_case([0, 64], H=1, D=72)
    with pytest.raises(ValueError):
        fused_rope_attention_train(q.to(DEV), k.to(DEV), v.to(DEV), cos.to(DEV), sin.to(DEV), cu.to(DEV))
