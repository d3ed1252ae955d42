"""Data-parallel inference across the GPUs of one node.

Each rank holds a full replica of the packed model and runs its own slice of
the image batch; the only collective is one all-gather of the logits per
step (NCCL over NVLink on GPUs, gloo on CPU for the tests). There is no
collective inside a layer: the packed GEMM never talks to another GPU.

The reference's only multi-GPU code is training DDP (RPFQ-ViT-main/scripts/
train.py:949-953) and ``nn.DataParallel`` in validation (validate.py:276-277);
inference sharding by image is this module.
"""

from __future__ import annotations

import os
from datetime import timedelta

import torch
import torch.distributed as dist


def env_rank_world() -> tuple[int, int, int]:
    """(rank, world_size, local_rank) from the torchrun environment."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def init(backend: str, timeout_s: float = 120.0, device: torch.device | None = None) -> None:
    """Initialise the default process group with a short timeout, so that ranks
    waiting for a dead peer end with an error instead of hanging."""
    kw = {"timeout": timedelta(seconds=timeout_s)}
    if device is not None and backend == "nccl":
        kw["device_id"] = device
    dist.init_process_group(backend, **kw)


def shard_range(global_batch: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous slice of the global batch owned by ``rank`` (the first
    ``global_batch % world`` ranks take one extra image)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    base, extra = divmod(global_batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard_sizes(global_batch: int, world: int) -> list[int]:
    """Images per rank under :func:`shard_range`."""
    return [e - s for s, e in (shard_range(global_batch, world, r) for r in range(world))]


class LogitsGather:
    """All-gather of per-rank logits ``[b_r, C]`` (rank r holding the rows
    :func:`shard_range` gives it) into ``[global_batch, C]`` in image order,
    with one collective per call.

    Equal shards gather straight into the output. Uneven shards (a global
    batch that ``world`` does not divide) are padded to ``ceil(B / world)``
    rows in a staging buffer, gathered, and the padding rows dropped. All
    buffers are allocated once, so a step can reuse them."""

    def __init__(self, global_batch: int, classes: int, world: int, rank: int, dtype=torch.float32,
                 device: torch.device | str = "cpu"):
        self.global_batch, self.world, self.rank = global_batch, world, rank
        self.sizes = shard_sizes(global_batch, world)
        self.cap = max(self.sizes) if self.sizes else 0
        self.even = all(s == self.cap for s in self.sizes)
        self.out = torch.empty((global_batch, classes), dtype=dtype, device=device)
        if self.even:
            self.send = self.recv = None
        else:
            self.send = torch.zeros((self.cap, classes), dtype=dtype, device=device)
            self.recv = torch.empty((world * self.cap, classes), dtype=dtype, device=device)

    def __call__(self, local: torch.Tensor) -> torch.Tensor:
        if local.shape[0] != self.sizes[self.rank]:
            raise ValueError(f"rank {self.rank} holds {self.sizes[self.rank]} images of the global batch, "
                             f"got logits for {local.shape[0]}")
        if self.even:
            _all_gather(self.out, local.contiguous(), self.world)
            return self.out
        self.send[: local.shape[0]].copy_(local)
        _all_gather(self.recv, self.send, self.world)
        start = 0
        for r, n in enumerate(self.sizes):
            self.out[start:start + n].copy_(self.recv[r * self.cap:r * self.cap + n])
            start += n
        return self.out


def _all_gather(out: torch.Tensor, local: torch.Tensor, world: int) -> None:
    if dist.get_backend() == "nccl":
        dist.all_gather_into_tensor(out, local)
    else:
        dist.all_gather(list(out.chunk(world, dim=0)), local)


def gather_logits(local: torch.Tensor, global_batch: int | None = None) -> torch.Tensor:
    """All-gather per-rank logits into ``[global_batch, C]`` in image order
    (one collective). ``global_batch`` defaults to ``world * local rows``
    (equal shards); with a global batch that does not divide by the world
    size, each rank passes the rows :func:`shard_range` gave it."""
    world, rank = dist.get_world_size(), dist.get_rank()
    if global_batch is None:
        global_batch = world * local.shape[0]
    return LogitsGather(global_batch, local.shape[1], world, rank, local.dtype, local.device)(local)


def max_over_ranks(value: float, device: torch.device) -> float:
    """Maximum of a per-rank scalar (device timings are reported as the max)."""
    t = torch.tensor([value], dtype=torch.float64, device=device)
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
