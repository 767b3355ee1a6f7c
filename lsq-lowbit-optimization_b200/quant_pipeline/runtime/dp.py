"""Data-parallel whole-network inference: one process per GPU.

The batch is partitioned into contiguous per-rank slices (images are
independent, weights are replicated); the only exchange is one all-gather
of the float32 logits. Over NCCL (NVLink / NVSwitch) this is
``all_gather_into_tensor``; other backends (gloo, for host-side tests) use
the list form.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.distributed as dist


def shard_range(total: int, world: int, rank: int) -> Tuple[int, int]:
    """[start, stop) of rank's contiguous slice; sizes differ by at most one."""
    if world < 1 or not 0 <= rank < world or total < 0:
        raise ValueError("bad shard request")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def gather_logits(local: torch.Tensor, out: Optional[torch.Tensor] = None,
                  group: Optional[dist.ProcessGroup] = None) -> torch.Tensor:
    """Concatenates every rank's [b, classes] logits in rank order (equal b)."""
    world = dist.get_world_size(group)
    b, classes = local.shape
    if out is None:
        out = torch.empty((b * world, classes), dtype=local.dtype, device=local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    else:
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local.contiguous(), group=group)
        torch.cat(parts, dim=0, out=out)
    return out
