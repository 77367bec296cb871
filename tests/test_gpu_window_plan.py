"""Device window plan (frattn_window_plan / frattn_window_shuffle) against the host
producers (get_window_index, compute_rope_2d with window_idx, window_shuffle), which
are themselves pinned to the reference's outputs in tests/test_host_golden.py."""
import pytest
import torch

from fused_rope_attn_b200 import compute_rope_2d, fused_rope_attention, fused_rope_attention_pos, last_status
from fused_rope_attn_b200.utils import get_window_index, window_shuffle, window_unshuffle
from fused_rope_attn_b200.window_plan import window_plan_device, window_shuffle_device, window_unshuffle_device

pytestmark = pytest.mark.gpu
DEV = "cuda"

GRIDS = {
    "448": [(1, 32, 32)],
    "896": [(1, 64, 64)],
    "1344": [(1, 96, 96)],
    "truncated": [(1, 22, 30), (1, 34, 18)],
    "clip_and_images": [(8, 32, 32), (1, 16, 24), (2, 10, 14)],
    "cfg5_sample": [(1, 64, 64)] * 3 + [(8, 32, 32)],
}


@pytest.mark.parametrize("name", list(GRIDS))
def test_plan_matches_host(name):
    grid = GRIDS[name]
    widx, cu = get_window_index(grid)
    cos, sin = compute_rope_2d(grid, 80, 2, 10000.0, DEV, torch.float32, window_idx=widx)
    from fused_rope_attn_b200 import rope_positions_2d
    pos = rope_positions_2d(grid).reshape(-1, 4, 2)[widx].reshape(-1, 2)
    d = window_plan_device(grid, device=DEV, head_dim=80)
    torch.cuda.synchronize()
    assert torch.equal(d["window_index"].cpu(), widx)
    assert torch.equal(d["cu_seqlens"].cpu(), cu)
    assert torch.equal(d["pos_hw"].cpu(), pos)
    assert (d["cos"] - cos).abs().max().item() <= 2e-6
    assert (d["sin"] - sin).abs().max().item() <= 2e-6


@pytest.mark.parametrize("window_size,patch", [(112, 14), (56, 14), (224, 16)])
def test_plan_other_window_sizes(window_size, patch):
    grid = [(1, 22, 30), (3, 8, 12)]
    widx, cu = get_window_index(grid, window_size=window_size, patch_size=patch)
    d = window_plan_device(grid, window_size=window_size, patch_size=patch, device=DEV, positions=False)
    assert torch.equal(d["window_index"].cpu(), widx)
    assert torch.equal(d["cu_seqlens"].cpu(), cu)
    assert d["pos_hw"] is None and d["cos"] is None


def test_shuffle_roundtrip_matches_host():
    grid = [(1, 22, 30), (2, 8, 8)]
    widx, _ = get_window_index(grid)
    T = int(widx.numel()) * 4
    x = torch.randn(T, 1280, device=DEV).to(torch.bfloat16)
    a = window_shuffle_device(x, widx.to(DEV))
    assert torch.equal(a, window_shuffle(x, widx.to(DEV)))
    b = window_unshuffle_device(a, widx.to(DEV))
    assert torch.equal(b, x)
    assert torch.equal(b, window_unshuffle(a, widx.to(DEV)))


def test_device_plan_drives_the_kernel():
    """The whole window-layer input built on the device feeds both entry points."""
    grid = [(1, 22, 30), (1, 16, 16)]
    d = window_plan_device(grid, device=DEV, head_dim=80)
    T = d["pos_hw"].shape[0]
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(T, 4, 80, generator=g).to(torch.bfloat16).to(DEV) for _ in range(3))
    o1 = fused_rope_attention(q, k, v, d["cos"], d["sin"], d["cu_seqlens"], max_seqlen=64)
    o2 = fused_rope_attention_pos(q, k, v, d["pos_hw"], d["cu_seqlens"], max_position=64)
    widx, cu = get_window_index(grid)
    cos, sin = compute_rope_2d(grid, 80, 2, 10000.0, DEV, torch.float32, window_idx=widx)
    o3 = fused_rope_attention(q, k, v, cos, sin, cu.to(DEV))
    torch.cuda.synchronize()
    assert last_status() == 0
    assert (o1.float() - o3.float()).abs().max().item() <= 2e-2
    assert (o2.float() - o3.float()).abs().max().item() <= 2e-2


def test_plan_rejects_bad_grids():
    with pytest.raises(ValueError):
        window_plan_device([(1, 15, 16)], device=DEV)  # not divisible by merge
    with pytest.raises(ValueError):
        window_plan_device([(0, 16, 16)], device=DEV)
