"""Data-parallel image throughput and its single collective.

Images and clips are independent (no attention crosses them), so the work
shards by item: each rank runs the encoder on its own packed items and the
outputs are gathered to rank 0 once at the end. That gather is the only
collective (NCCL over NVLink on GPUs; gloo in the CPU tests).

* ``partition`` — greedy longest-processing-time assignment of items to ranks by
  a cost model (GEMM FLOPs ∝ tokens, full attention ∝ L², windows ∝ L).
* ``gather_packed`` — variable-length gather: sizes are exchanged first, rows
  are padded to the largest rank, one ``all_gather_into_tensor`` moves them.
* ``run_dp`` — one DP encoder pass; rank 0 returns the per-item outputs in the
  original item order.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .encoder import EncoderConfig, encoder_flops, encoder_inputs

__all__ = ["item_cost", "partition", "gather_packed", "local_inputs", "run_dp"]


def item_cost(grid, cfg: EncoderConfig | None = None) -> float:
    f = encoder_flops([tuple(grid)], cfg)
    return float(f["gemm"] + f["attention"])


def partition(costs, world: int) -> list[list[int]]:
    """Greedy LPT: items by decreasing cost, each to the currently lightest rank.
    Returns per-rank item indices in ascending order (deterministic ties)."""
    if world <= 0:
        raise ValueError("world must be >= 1")
    load = [0.0] * world
    parts: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(costs)), key=lambda j: (-costs[j], j)):
        r = min(range(world), key=lambda k: (load[k], k))
        parts[r].append(i)
        load[r] += costs[i]
    return [sorted(p) for p in parts]


def gather_packed(x: torch.Tensor, group=None) -> list[torch.Tensor] | None:
    """Gather a [n_r, C] tensor of every rank to rank 0 (n_r may differ)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    n = torch.tensor([x.shape[0]], dtype=torch.int64, device=x.device)
    sizes = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(sizes, n, group=group)
    sizes = [int(s.item()) for s in sizes]
    m = max(sizes) if sizes else 0
    pad = torch.zeros(m, *x.shape[1:], dtype=x.dtype, device=x.device)
    pad[: x.shape[0]] = x
    full = torch.empty(world * m, *x.shape[1:], dtype=x.dtype, device=x.device)
    dist.all_gather_into_tensor(full, pad, group=group)
    if rank != 0:
        return None
    return [full[r * m: r * m + sizes[r]] for r in range(world)]


def local_inputs(encoder, grids, parts, rank, seed: int = 0):
    """This rank's packed input embeddings (item i seeded by seed + i) and its grids."""
    cfg = encoder.cfg
    mine = parts[rank]
    dev, dt = encoder.device, encoder.dtype
    if not mine:
        return torch.zeros(0, cfg.hidden, device=dev, dtype=dt), []
    xs = [encoder_inputs([grids[i]], cfg.hidden, seed=seed + i, device=dev, dtype=dt) for i in mine]
    return torch.cat(xs), [grids[i] for i in mine]


def run_dp(encoder, grids, attn: str = "fused", seed: int = 0, group=None, inputs=None, plan=None,
           events=None):
    """One data-parallel encoder pass over ``grids`` (list of (t, h, w)).

    Every item's input embeddings are seeded by its index, so the result does
    not depend on the partition. ``inputs`` / ``plan`` may be prepared ahead
    (``local_inputs``, ``encoder.plan``) so that a timed pass only runs the
    encoder and the gather; ``events`` = three CUDA events recorded before the
    encoder, between encoder and gather, and after the gather. Returns (outputs
    on rank 0 else None, my item indices, local token count).
    """
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    cfg = encoder.cfg
    parts = partition([item_cost(g, cfg) for g in grids], world)
    mine = parts[rank]
    x, my_grids = inputs if inputs is not None else local_inputs(encoder, grids, parts, rank, seed)
    if events:
        events[0].record()
    if mine:
        out = encoder(x, my_grids, attn=attn, plan=plan)
    else:
        out = x
    if events:
        events[1].record()
    gathered = gather_packed(out, group)
    if events:
        events[2].record()
    if gathered is None:
        return None, mine, out.shape[0]
    result: list[torch.Tensor | None] = [None] * len(grids)
    for r, idx in enumerate(parts):
        off = 0
        for i in idx:
            n = grids[i][0] * grids[i][1] * grids[i][2]
            result[i] = gathered[r][off: off + n]
            off += n
    return result, mine, out.shape[0]
