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


def gather_logits(local: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """All-gather equal-sized per-rank logits ``[b, C]`` into ``[world * b, C]``
    in rank order (one collective)."""
    world = dist.get_world_size()
    if out is None:
        out = torch.empty((world * local.shape[0], *local.shape[1:]), dtype=local.dtype, device=local.device)
    if dist.get_backend() == "nccl":
        dist.all_gather_into_tensor(out, local.contiguous())
    else:
        parts = list(out.chunk(world, dim=0))
        dist.all_gather(parts, local.contiguous())
    return out


def max_over_ranks(value: float, device: torch.device) -> float:
    """Maximum of a per-rank scalar (device timings are reported as the max)."""
    t = torch.tensor([value], dtype=torch.float64, device=device)
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
