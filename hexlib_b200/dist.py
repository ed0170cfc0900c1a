"""Image sharding across GPUs, one process per GPU.

Images are independent, so a batch of B images splits into contiguous shards
of B/G images per rank with a full replica of the weights each, and no
collective touches the data path. The one exchange is at the end: every rank
contributes its [B/G, T/4, 1024] fp16 embeddings to an all-gather so every
rank holds the whole batch's output.

On the GPUs that gather is `EmbeddingGather`: libhexlib_b200's NCCL entry
points (non-blocking communicator, a deadline on every wait, abort on expiry
-> ERR_TIMEOUT / ERR_COMM), with rank 0's rendezvous id handed to the other
ranks through whatever channel the caller has (torch.distributed by default).
`gather_embeddings` is the same exchange through any torch.distributed
backend (gloo on the CPU in the tests).
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import Callable


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


class CommError(RuntimeError):
    """A collective of EmbeddingGather failed; `status` is the library's code
    (ERR_TIMEOUT: a peer stopped answering before the deadline; ERR_COMM: NCCL
    reported an error, e.g. a peer that left). The communicator is aborted."""

    def __init__(self, what: str, status: int):
        from hexlib_b200 import _lib
        super().__init__(f"{what}: {_lib.status_name(status)} ({status})")
        self.status = status


def broadcast_from_rank0(value):
    """Rank 0's `value` on every rank, through torch.distributed's default
    group (any backend)."""
    import torch.distributed as dist
    box = [value]
    dist.broadcast_object_list(box, src=0)
    return box[0]


def share_unique_id(rank: int, exchange: Callable = broadcast_from_rank0) -> bytes:
    """Rank 0 makes the NCCL rendezvous id through the library; every rank
    returns it (`exchange(rank 0's bytes or None) -> rank 0's bytes`)."""
    from hexlib_b200 import _lib
    mine = None
    if rank == 0:
        buf = (ctypes.c_uint8 * 128)()
        rc = _lib.lib().hexlib_b200_nccl_unique_id(buf)
        if rc != 1:
            raise CommError("nccl unique id", rc)
        mine = bytes(buf)
    ident = exchange(mine)
    if not isinstance(ident, (bytes, bytearray)) or len(ident) != 128:
        raise ValueError("the rendezvous id did not arrive intact")
    return bytes(ident)


class EmbeddingGather:
    """The all-gather of every rank's embeddings through the library's NCCL
    entry points, every wait bounded by `timeout_s`."""

    def __init__(self, rank: int, world: int, device: int, timeout_s: float = 60.0,
                 exchange: Callable = broadcast_from_rank0):
        from hexlib_b200 import _lib
        self._L = _lib.lib()
        self.rank, self.world, self.device = rank, world, device
        self.timeout_ms = max(1, int(timeout_s * 1000))
        self._h = None
        ident = share_unique_id(rank, exchange)
        h = ctypes.c_void_p()
        rc = self._L.hexlib_b200_nccl_open((ctypes.c_uint8 * 128).from_buffer_copy(ident),
                                           world, rank, device, self.timeout_ms,
                                           ctypes.byref(h))
        if rc != 1:
            raise CommError("nccl open", rc)
        self._h = h

    def gather(self, local, out, stream: int) -> None:
        """Enqueue on `stream` the gather of `local` ([b, ...] fp16, on this
        rank's GPU) into `out` ([world * b, ...]) in rank order."""
        import torch
        if local.dtype != torch.float16 or out.dtype != torch.float16:
            raise TypeError("the embedding gather moves fp16")
        if out.numel() != local.numel() * self.world or not (local.is_contiguous()
                                                             and out.is_contiguous()):
            raise ValueError("out must hold world x local, both contiguous")
        # NCCL's kernel runs on the communicator's device and would otherwise
        # be handed another device's memory
        for t in (local, out):
            if t.device.type != "cuda" or t.device.index != self.device:
                raise ValueError(f"the gather's tensors must be on cuda:{self.device}, "
                                 f"not {t.device}")
        rc = self._L.hexlib_b200_nccl_allgather_f16(self._h, local.data_ptr(), out.data_ptr(),
                                                    local.numel(), stream, self.timeout_ms)
        if rc != 1:
            raise CommError("nccl all-gather", rc)

    def wait(self, stream: int) -> None:
        rc = self._L.hexlib_b200_nccl_wait(self._h, stream, self.timeout_ms)
        if rc != 1:
            raise CommError("nccl wait", rc)

    def abort(self) -> None:
        if self._h:
            self._L.hexlib_b200_nccl_abort(self._h)

    def close(self) -> None:
        if self._h:
            self._L.hexlib_b200_nccl_close(self._h, self.timeout_ms)
            self._h = None
