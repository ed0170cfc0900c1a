"""Image sharding across GPUs, one process per GPU.

Images are independent, so a batch of B images splits into contiguous shards
of B/G images per rank with a full replica of the weights each, and no
collective touches the data path. The one exchange is at the end: every rank
contributes its [B/G, T/4, 1024] fp16 embeddings to an all-gather so every
rank holds the whole batch's output (NCCL over NVLink on the GPUs; any
torch.distributed backend works, gloo on the CPU in the tests).
"""
from __future__ import annotations

import os
from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    start: int
    count: int


def shard(n_total: int, rank: int, world: int) -> Shard:
    """Contiguous shard of `n_total` images for `rank` of `world`. The batch
    must divide evenly: an uneven split would make the all-gather ragged."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if n_total % world:
        raise ValueError(f"{n_total} images do not split evenly over {world} ranks")
    per = n_total // world
    return Shard(rank, world, rank * per, per)


def env_rank() -> tuple[int, int, int]:
    """(rank, local_rank, world_size) from torchrun's environment."""
    r = int(os.environ.get("RANK", "0"))
    lr = int(os.environ.get("LOCAL_RANK", str(r)))
    w = int(os.environ.get("WORLD_SIZE", "1"))
    return r, lr, w


def gather_embeddings(local, group=None):
    """All-gather each rank's [b, ...] tensor into [world*b, ...], in rank
    order. `local` is a torch tensor on this rank's device (or CPU for gloo)."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    if dist.get_backend(group) == "gloo":
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local.contiguous(), group=group)
        return torch.cat(parts, dim=0)
    out = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]),
                      dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    return out
