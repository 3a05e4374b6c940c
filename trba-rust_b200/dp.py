"""Host side of data-parallel training: one process per GPU, weak scaling.

Each rank trains the same model on its own batch; libtrba_b200 averages the
fp32 gradient buffer with one NCCL all-reduce per step (trba_dp_init /
trba_model_train_step) before the identical optimiser step on every rank.
BN batch statistics and the dynamic activation scales stay per rank (the
reference's per-replica semantics).  This module holds the plumbing around
that: joining the NCCL communicator through torch.distributed, per-rank data
seeds, and the max-over-ranks step time.
"""
from __future__ import annotations

from typing import Callable


def rank_seed(seed: int, rank: int) -> int:
    """Seed of a rank's synthetic batches: distinct per rank, reproducible."""
    return seed + 1000 * rank + 1


def shard(global_batch: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of rank's lines when a global batch is split evenly;
    the first global_batch % world ranks take one line more."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    base, extra = divmod(global_batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def join(model, unique_id: Callable[[], bytes] | None = None) -> tuple[int, int]:
    """Join `model` to the NCCL communicator of the current torch.distributed
    group: rank 0 draws the 128-byte NCCL id, every rank receives it by
    broadcast and calls model.dp_init(id, rank, world).  Returns (rank, world)."""
    import torch.distributed as dist
    rank, world = dist.get_rank(), dist.get_world_size()
    if unique_id is None:
        from .model import QatModel
        unique_id = QatModel.dp_unique_id
    obj = [unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    if not isinstance(obj[0], (bytes, bytearray)) or len(obj[0]) != 128:
        raise RuntimeError("NCCL unique id broadcast returned a malformed id")
    model.dp_init(bytes(obj[0]), rank, world)
    return rank, world


def max_over_ranks(value: float, device=None) -> float:
    """The largest `value` over all ranks (the step time a job is charged)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
