"""CUDA path (through the C ABI) vs the CPU oracle on the same seeded inputs.

Tolerance (bf16/fp16 outputs vs the fp32 unfused path): max-abs <= 2e-2 and
mean-abs <= 2e-3 per call.
"""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from fused_rope_attn_b200 import fused_rope_attention, fused_rope_attention_pos, last_status, rope_positions_2d
from fused_rope_attn_b200.utils import get_window_index
from gpu_cases import cu_case, grid_case, mixed_sides, rand_qkv
from oracle import rope_attn_oracle as O

pytestmark = pytest.mark.gpu
MAX_ABS, MEAN_ABS = 2e-2, 2e-3
DEV = "cuda"


def run(q, k, v, cos, sin, cu, **kw):
    out = fused_rope_attention(q.to(DEV), k.to(DEV), v.to(DEV), cos.to(DEV), sin.to(DEV), cu.to(DEV), **kw)
    torch.cuda.synchronize()
    assert last_status() == 0
    return out


def oracle(q, k, v, cos, sin, cu):
    return O.rope_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                            cos.float().numpy(), sin.float().numpy(), cu.numpy())


def assert_close(out, ref, max_abs=MAX_ABS, mean_abs=MEAN_ABS):
    o = out.float().cpu().numpy()
    assert np.isfinite(o).all()
    err = np.abs(o - ref)
    assert err.max() <= max_abs and err.mean() <= mean_abs, (float(err.max()), float(err.mean()))


@pytest.mark.parametrize("name,grid,windowed", [
    ("cfg1_448_windowed", [(1, 32, 32)], True),
    ("cfg2a_896_windowed", [(1, 64, 64)], True),
    ("cfg2b_896_full", [(1, 64, 64)], False),
    ("truncated_22x30", [(1, 22, 30)], True),
    ("clip_t2", [(2, 16, 24)], True),
])
def test_config_parity(name, grid, windowed):
    case = grid_case(grid, windowed, seed=hash(name) % 1000)
    assert_close(run(*case), oracle(*case))


@pytest.mark.parametrize("hint", [None, 64])
def test_cfg3_mixed_varlen_batch(hint):
    grid = [(1, s, s) for s in mixed_sides(0)]
    case = grid_case(grid, True, seed=3)
    assert_close(run(*case, max_seqlen=hint), oracle(*case))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("cs_dtype", [torch.float32, torch.bfloat16, torch.float16])
def test_dtypes(dtype, cs_dtype):
    case = cu_case([0, 64, 100, 300, 301, 429], H=3, dtype=dtype, cs_dtype=cs_dtype, seed=5)
    assert_close(run(*case), oracle(*case))


@pytest.mark.parametrize("D", list(range(32, 129, 8)))
def test_head_dims(D):
    """Every compiled kernel head dim (multiples of 8 in [32, 128])."""
    case = cu_case([0, 64, 128, 390, 400], H=2, D=D, seed=D)
    assert_close(run(*case), oracle(*case))


@pytest.mark.parametrize("D", [2, 16, 36, 50, 124])
def test_padded_head_dims(D):
    """Other even head dims (the reference accepts any even D, fused_attn.py:166-168)
    run on the next kernel dim through zero padding; the result is unpadded."""
    case = cu_case([0, 64, 300, 301], H=3, D=D, seed=D + 1)
    out = run(*case)
    assert out.shape == case[0].shape
    assert_close(out, oracle(*case))
    o2 = torch.empty_like(case[0], device=DEV)
    run(*case, out=o2)
    assert torch.equal(o2, out)


@pytest.mark.parametrize("cu_list", [
    [0, 1],                                  # single token
    [0, 127], [0, 128], [0, 129],            # around the long-segment threshold
    [0, 255, 256, 257],                      # long, length-1, length-1
    [0, 0, 64, 64, 64, 130, 130],            # empty segments
    [0, 5, 9, 70, 71, 200, 330, 331, 459],   # ragged, segments crossing 128-row chunks
    list(range(0, 1025, 1)),                 # 1024 length-1 segments
    [0, 3000],                               # one long segment, partial last tile
    list(range(0, 2050, 2)),                 # 1024 two-token segments (cu longer than the staged part)
    [0, 60, 64, 130, 131, 250, 300, 364],    # windows crossing 128-row chunks (two K/V tiles)
])
@pytest.mark.parametrize("hint", [False, True], ids=["general", "max_seqlen_hint"])
def test_edge_segmentations(cu_list, hint):
    # With the hint (the longest segment, as callers pass it) segments of at
    # most 128 tokens take the window kernel, longer ones the general path.
    case = cu_case(cu_list, H=2, seed=len(cu_list))
    kw = {"max_seqlen": max(b - a for a, b in zip(cu_list[:-1], cu_list[1:]))} if hint else {}
    assert_close(run(*case, **kw), oracle(*case))


@pytest.mark.parametrize("hint", [None, 64])
def test_strided_qkv_views_match_contiguous(hint):
    """q/k/v as views of one [T, 3, H, D] projection output (token stride 3 H D)
    are read in place (frattn_fwd_strided) and give the contiguous result."""
    grid = [(1, 22, 30), (1, 16, 16)]
    q, k, v, cos, sin, cu = grid_case(grid, True, H=4, seed=13)
    qkv = torch.stack([q, k, v], dim=1).to(DEV)  # [T, 3, H, D]
    qv, kv_, vv = qkv[:, 0], qkv[:, 1], qkv[:, 2]
    assert not qv.is_contiguous()
    out = run(qv, kv_, vv, cos, sin, cu, max_seqlen=hint)
    ref = run(q, k, v, cos, sin, cu, max_seqlen=hint)
    assert torch.equal(out, ref)
    assert_close(out, oracle(q, k, v, cos, sin, cu))
    # a long segment through the same views (pre-rotated K path)
    cu2 = torch.tensor([0, 300, int(cu[-1])], dtype=torch.int32)
    assert torch.equal(run(qv, kv_, vv, cos, sin, cu2), run(q, k, v, cos, sin, cu2))


@pytest.mark.parametrize("cu_list,H,D,dtype", [
    ([0, 3000, 5000], 16, 80, torch.bfloat16),       # 320 long units, two tile counts
    ([0, 4096], 16, 80, torch.bfloat16),             # BASELINE config 2b shape: 256 units
    ([0, 700, 2600, 2601, 4000], 24, 64, torch.float16),
    ([0, 1500, 3100], 20, 128, torch.bfloat16),      # Q in shared memory (D = 128)
])
def test_many_long_units(cu_list, H, D, dtype):
    """More long (segment, 256-row, head) units than CTAs, ragged tile counts:
    every CTA walks several units (row-subsample check against the oracle)."""
    case = cu_case(cu_list, H=H, D=D, dtype=dtype, seed=H + D)
    q, k, v, cos, sin, cu = case
    out = run(*case)
    rows = np.random.default_rng(1).choice(q.shape[0], 160, replace=False)
    qr = O.apply_rope(q.float().numpy(), cos.numpy(), sin.numpy())
    kr = O.apply_rope(k.float().numpy(), cos.numpy(), sin.numpy())
    ref = O.varlen_attention_rows(qr, kr, v.float().numpy(), cu.numpy(), rows)
    assert_close(out[rows.tolist()], ref)
    # cross-check against the window kernel, which walks every chunk's whole kv
    # range itself (a max_seqlen hint <= 128 selects it; results never depend
    # on the hint)
    assert (run(*case, max_seqlen=1).float() - out.float()).abs().max().item() <= 1e-2


def test_rows_outside_segments_are_zero():
    q, k, v, cos, sin, cu = cu_case([40, 104, 170], H=2, T=256, seed=9)
    out = run(q, k, v, cos, sin, cu).float().cpu()
    ref = oracle(q, k, v, cos, sin, cu)
    assert (out[:40] == 0).all() and (out[170:] == 0).all()
    assert_close(out, ref)


def test_all_empty_returns_zeros():
    q, k, v, cos, sin, _ = cu_case([0, 64], H=2, seed=1)
    out = run(q, k, v, cos, sin, torch.tensor([0, 0, 0], dtype=torch.int32))
    assert (out == 0).all()


def test_many_heads_and_out_param():
    q, k, v, cos, sin, cu = cu_case([0, 64, 192, 250], H=32, seed=11)
    out = torch.full((250, 32, 80), float("nan"), dtype=torch.bfloat16, device=DEV)
    res = run(q, k, v, cos, sin, cu, out=out, max_seqlen=128)
    assert res.data_ptr() == out.data_ptr()
    assert_close(out, oracle(q, k, v, cos, sin, cu))


def test_noncontiguous_and_int64_cpu_cu():
    q, k, v, cos, sin, cu = cu_case([0, 64, 128, 300], H=4, seed=12)
    qt = q.transpose(0, 1).contiguous().transpose(0, 1)  # same values, non-contiguous
    out = fused_rope_attention(qt.to(DEV), k.to(DEV), v.to(DEV), cos.to(DEV), sin.to(DEV), cu.to(torch.int64))
    torch.cuda.synchronize()
    assert_close(out, oracle(q, k, v, cos, sin, cu))


@pytest.mark.parametrize("cs_dtype", [torch.float32, torch.bfloat16])
def test_head_dim_72_fp16_reference_bench_shape(cs_dtype):
    """The reference's own benchmark configuration: fp16, head_dim 72 (bench.py:31-34)."""
    case = grid_case([(1, 32, 32)], True, H=16, D=72, dtype=torch.float16, cs_dtype=cs_dtype, seed=72)
    assert_close(run(*case), oracle(*case))
    case = grid_case([(1, 32, 32)], False, H=4, D=72, dtype=torch.float16, cs_dtype=cs_dtype, seed=73)
    assert_close(run(*case), oracle(*case))


def test_wrapper_value_errors():
    q, k, v, cos, sin, cu = [t.to(DEV) for t in cu_case([0, 64], H=2, seed=1)]
    with pytest.raises(ValueError):
        fused_rope_attention(q, k[:32], v, cos, sin, cu)
    with pytest.raises(ValueError):
        fused_rope_attention(q[:, 0], k[:, 0], v[:, 0], cos, sin, cu)
    with pytest.raises(ValueError):
        fused_rope_attention(q, k, v, cos[:, :20], sin, cu)
    with pytest.raises(ValueError):
        fused_rope_attention(q, k, v, cos, sin, cu[:1])
    with pytest.raises(ValueError):
        fused_rope_attention(q.float(), k.float(), v.float(), cos, sin, cu)
    with pytest.raises(ValueError):
        fused_rope_attention(q, k.half(), v, cos, sin, cu)
    with pytest.raises(ValueError):
        fused_rope_attention(q, k, v, cos.double(), sin, cu)
    with pytest.raises(ValueError):
        fused_rope_attention(q, k, v, cos, sin, cu, out=torch.empty_like(q)[:10])
    with pytest.raises(ValueError):
        fused_rope_attention(q, k, v, cos, sin, cu, out=torch.empty_like(q, dtype=torch.float16))


def test_bad_cu_seqlens_sets_status():
    q, k, v, cos, sin, _ = [t.to(DEV) for t in cu_case([0, 64], H=2, seed=1)]
    fused_rope_attention(q, k, v, cos, sin, torch.tensor([0, 50, 20, 64], dtype=torch.int32, device=DEV))
    torch.cuda.synchronize()
    assert last_status() == 0x200
    assert last_status() == 0  # reset after reading


def test_out_of_table_positions_set_status():
    # A coordinate equal to max_position is one row past the rotary table. The
    # scheduler kernel rejects it before any kernel reads the table (nothing is
    # computed). Were the check missing, the read would still land inside the
    # workspace (the sin half follows the cos half), so the case cannot fault.
    q, k, v, _, _, cu = [t.to(DEV) for t in cu_case([0, 64, 300], H=2, seed=3)]
    pos = torch.randint(0, 16, (300, 2), dtype=torch.int32, device=DEV)
    fused_rope_attention_pos(q, k, v, pos, cu, max_position=16)
    torch.cuda.synchronize()
    assert last_status() == 0
    pos[17, 1] = 16
    fused_rope_attention_pos(q, k, v, pos, cu, max_position=16)
    torch.cuda.synchronize()
    assert last_status() == 0x400


def test_device_wait_timeout_is_reported_not_hung():
    from fused_rope_attn_b200 import _lib
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc = _lib.load().frattn_selftest_wait_timeout(st.data_ptr(), 20_000_000, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    assert int(st.item()) & 0xF00 == _lib.STATUS_WAIT_TIMEOUT
    # the context is still usable
    case = cu_case([0, 64], H=1, seed=2)
    assert_close(run(*case), oracle(*case))


def test_position_entry_point_matches_tables():
    grid = [(1, 22, 30), (2, 8, 8)]
    widx, cu = get_window_index(grid)
    pos = rope_positions_2d(grid).reshape(-1, 4, 2)[widx].reshape(-1, 2)
    q, k, v, cos, sin, _ = grid_case(grid, True, H=4, seed=21)
    out_pos = fused_rope_attention_pos(q.to(DEV), k.to(DEV), v.to(DEV), pos.to(DEV), cu.to(DEV), theta=10000.0)
    torch.cuda.synchronize()
    assert last_status() == 0
    assert_close(out_pos, oracle(q, k, v, cos, sin, cu))
    out_tab = run(q, k, v, cos, sin, cu)
    assert (out_pos.float() - out_tab.float()).abs().max().item() <= 2e-2


@pytest.mark.parametrize("windowed", [True, False])
def test_max_seqlen_hint_changes_nothing(windowed):
    # The hint only decides whether long segments' K is pre-rotated in a
    # separate pass; a true, a missing and a wrong (too small) hint give the
    # same result (the K rotation is the same fp32 arithmetic on either path), and
    # all of them match the oracle.
    case = grid_case([(1, 32, 48)], windowed, H=4, seed=7)
    true_max = int((case[5][1:] - case[5][:-1]).max())
    want = oracle(*case)
    ref = run(*case)
    assert_close(ref, want)
    for hint in (true_max, 64, 1):
        out = run(*case, max_seqlen=hint)
        assert_close(out, want)
        assert (out.float() - ref.float()).abs().max().item() <= 1e-2


def test_deterministic():
    case = grid_case([(1, 32, 32)], False, H=4, seed=4)
    a = run(*case)
    b = run(*case)
    assert torch.equal(a, b)


def test_reference_kernel_golden_vectors():
    """Our kernel on the inputs the reference kernel was run on (fp16 cases)."""
    K = np.load(os.path.join(GOLDEN, "golden_kernel.npz"))
    for name in sorted({key.split("/")[0] for key in K.files}):
        q, k, v = (torch.from_numpy(K[f"{name}/{t}"]) for t in "qkv")
        if q.dtype == torch.float32:
            q, k, v = q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16)
        cos, sin = torch.from_numpy(K[f"{name}/cos"]), torch.from_numpy(K[f"{name}/sin"])
        cu = torch.from_numpy(K[f"{name}/cu_seqlens"])
        out = run(q, k, v, cos, sin, cu).float().cpu().numpy()
        ref = K[f"{name}/out"].astype(np.float32)
        err = np.abs(out - ref)
        assert err.max() <= MAX_ABS and err.mean() <= MEAN_ABS, (name, err.max(), err.mean())


@pytest.mark.parametrize("windowed", [True, False])
@pytest.mark.parametrize("hint", [None, "true"])
def test_cuda_graph_replay_matches_eager(windowed, hint):
    # Replayed from a CUDA graph, the call's kernels launch back to back with
    # programmatic dependent launch; the attention kernel then starts before
    # the work list is written and must still read the finished list.
    case = grid_case([(1, 48, 48)], windowed, H=8, seed=11)
    q, k, v, cos, sin, cu = (t.to(DEV) for t in case)
    ms = int((cu[1:] - cu[:-1]).max()) if hint else None
    eager = fused_rope_attention(q, k, v, cos, sin, cu, max_seqlen=ms)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        fused_rope_attention(q, k, v, cos, sin, cu, max_seqlen=ms)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        out = fused_rope_attention(q, k, v, cos, sin, cu, max_seqlen=ms)
    for _ in range(3):
        g.replay()
        torch.cuda.synchronize()
        assert last_status() == 0
        assert (out.float() - eager.float()).abs().max().item() <= 1e-2
    assert_close(out, oracle(*case))
