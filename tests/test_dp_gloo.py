"""Data-parallel partition + gather on 2 gloo CPU ranks (no GPU)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fused_rope_attn_b200.dp import partition, run_dp
from fused_rope_attn_b200.encoder import EncoderConfig, VisionEncoder, encoder_inputs

CFG = dict(hidden=64, heads=2, head_dim=32, mlp=96, depth=3, full_layers=(1,), seed=3)
GRIDS = [(1, 8, 8), (1, 16, 8), (2, 8, 8), (1, 4, 12), (1, 8, 16)]


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q, fail_rank, timeout_s):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    try:
        if rank == fail_rank:
            raise RuntimeError("injected rank failure")
        enc = VisionEncoder(EncoderConfig(**CFG), device="cpu", dtype=torch.float32)
        res, mine, n = run_dp(enc, GRIDS, attn="fp32", seed=11)
        if rank == 0:
            q.put(("ok", [r.clone() for r in res], mine))
        else:
            q.put(("rank", mine, n))
    except Exception as e:  # noqa: BLE001
        q.put(("error", rank, type(e).__name__))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001
            pass


def _run(world, fail_rank=-1, timeout_s=120):
    # (a generous process-group timeout: a spawned rank can take many seconds to
    # import torch on a loaded machine; the failure test shortens it)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, q, fail_rank, timeout_s)) for r in range(world)]
    for p in ps:
        p.start()
    msgs = [q.get(timeout=120) for _ in range(world)]
    for p in ps:
        p.join(timeout=60)
    return msgs


def test_partition_lpt_balances_and_covers():
    costs = [9, 7, 6, 5, 4, 3, 2, 1]
    parts = partition(costs, 3)
    assert sorted(i for p in parts for i in p) == list(range(8))
    loads = [sum(costs[i] for i in p) for p in parts]
    assert max(loads) - min(loads) <= max(costs)
    assert partition([1.0], 4)[0] == [0] and partition([], 2) == [[], []]
    with pytest.raises(ValueError):
        partition([1.0], 0)


def test_items_are_independent_of_packing():
    enc = VisionEncoder(EncoderConfig(**CFG), device="cpu", dtype=torch.float32)
    xs = [encoder_inputs([g], 64, seed=11 + i, device="cpu", dtype=torch.float32) for i, g in enumerate(GRIDS[:3])]
    packed = enc(torch.cat(xs), GRIDS[:3], attn="fp32")
    off = 0
    for x, g in zip(xs, GRIDS[:3]):
        single = enc(x, [g], attn="fp32")
        assert torch.allclose(packed[off: off + x.shape[0]], single, atol=1e-5, rtol=1e-5)
        off += x.shape[0]


def test_dp_two_ranks_matches_single_process():
    msgs = _run(2)
    ok = [m for m in msgs if m[0] == "ok"]
    assert len(ok) == 1, msgs
    _, res, mine0 = ok[0]
    enc = VisionEncoder(EncoderConfig(**CFG), device="cpu", dtype=torch.float32)
    for i, g in enumerate(GRIDS):
        ref = enc(encoder_inputs([g], 64, seed=11 + i, device="cpu", dtype=torch.float32), [g], attn="fp32")
        assert torch.allclose(res[i], ref, atol=1e-5, rtol=1e-5)
    other = [m for m in msgs if m[0] == "rank"][0]
    assert sorted(mine0 + other[1]) == list(range(len(GRIDS)))


def test_dp_rank_failure_is_reported_not_hung():
    msgs = _run(2, fail_rank=1, timeout_s=20)
    kinds = sorted(m[0] for m in msgs)
    assert kinds == ["error", "error"], msgs
