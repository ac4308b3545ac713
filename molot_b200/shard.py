"""Work partitioning for batched decode over several GPUs, one process per GPU.

Two layouts, both host-side (the kernels never see a rank):

* sequence sharding (continuous batching): each rank owns whole sequences
  and their pages; ranks never exchange data on the hot path.  The batch is
  split by longest-processing-time-first greedy over the sequences' KV
  bytes (their lengths), which keeps the slowest rank within 4/3 of optimal.
* kv-head sharding (one model too large for one GPU's HBM): each rank owns a
  contiguous range of kv heads with their grouped q heads, for every
  sequence, and the per-rank attention outputs are all-gathered over NCCL
  into [B][nq][d] after each layer.

The reference runs one process on one CPU and has no counterpart; its
per-head independence (attn.h:125-177 computes every q head from its own kv
head only) is what makes head sharding exact.
"""
from __future__ import annotations

from typing import Sequence


def lpt_partition(lengths: Sequence[int], world: int) -> list[list[int]]:
    """Sequence indices per rank, longest first onto the least-loaded rank.

    Deterministic: ties in length go to the lower index, ties in load to the
    lower rank.  Each rank's list is returned in ascending index order.
    """
    if world < 1:
        raise ValueError("world must be >= 1")
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i))
    load = [0] * world
    parts: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda j: (load[j], j))
        parts[r].append(i)
        load[r] += int(lengths[i])
    return [sorted(p) for p in parts]


def head_shard(nkv: int, world: int, rank: int) -> tuple[int, int]:
    """[g0, g1): the kv heads rank `rank` owns (contiguous, equal counts)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    if nkv % world:
        raise ValueError(f"{nkv} kv heads do not split evenly over {world} ranks")
    per = nkv // world
    return rank * per, (rank + 1) * per


def gather_heads(o_local, group=None, out=None):
    """All-gather per-rank attention outputs [B][nq_local][d] into
    [B][world*nq_local][d], rank r's heads at [r*nq_local, (r+1)*nq_local).

    Uses torch.distributed.all_gather_into_tensor (NCCL on GPUs, gloo on the
    CPU) on a [world][B][nq_local][d] staging buffer, then one permuting
    copy into `out` (allocated when None).
    """
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    B, nql, d = o_local.shape
    stage = torch.empty((world, B, nql, d), dtype=o_local.dtype, device=o_local.device)
    if hasattr(dist, "all_gather_into_tensor") and o_local.device.type == "cuda":
        dist.all_gather_into_tensor(stage, o_local.contiguous(), group=group)
    else:
        dist.all_gather(list(stage.unbind(0)), o_local.contiguous(), group=group)
    if out is None:
        out = torch.empty((B, world * nql, d), dtype=o_local.dtype, device=o_local.device)
    out.view(B, world, nql, d).copy_(stage.permute(1, 0, 2, 3))
    return out
