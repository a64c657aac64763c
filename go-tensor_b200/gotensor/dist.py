"""Host side of data-parallel training: one process per GPU.

go-tensor has no multi-device code; this is what a host needs around the
library's NCCL data path (``gt_comm_init`` / ``gth_dp_init``):

* ``env_ranks`` reads the launcher's rank variables (torchrun's RANK,
  WORLD_SIZE, LOCAL_RANK);
* ``shard`` splits a global batch into equal per-rank row ranges (the mean of
  equal shard means is the global mean, so the averaged gradient equals the
  single-device one up to rounding);
* ``exchange_unique_id`` sends rank 0's 128-byte NCCL id to every rank over
  the host process group (``torch.distributed``, gloo), the only thing NCCL
  needs from the host to form the communicator;
* ``max_over_ranks`` gives the slowest rank's time, the figure a data-parallel
  step is worth.

The host process group carries only these small host messages; gradients
travel over NCCL inside the library.
"""
from __future__ import annotations

import os
from typing import Callable, Optional, Tuple


def env_ranks() -> Tuple[int, int, int]:
    """(rank, world_size, local_rank) from the launcher's environment
    (1-process defaults when unset)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    return rank, world, local


def shard(global_batch: int, rank: int, world: int) -> Tuple[int, int]:
    """Row range [lo, hi) of the global batch that `rank` trains on."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    if global_batch <= 0 or global_batch % world:
        raise ValueError(f"global batch {global_batch} does not split evenly over {world} ranks")
    per = global_batch // world
    return rank * per, (rank + 1) * per


def exchange_unique_id(rank: int, make_id: Optional[Callable[[], bytes]] = None) -> bytes:
    """Rank 0 creates the communicator id (``gt_comm_unique_id`` unless
    `make_id` is given) and every rank returns the same 128 bytes. Needs an
    initialised torch.distributed process group."""
    import torch.distributed as dist
    if make_id is None:
        from .model import unique_id as make_id
    obj = [make_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    uid = obj[0]
    if not isinstance(uid, (bytes, bytearray)) or len(uid) != 128:
        raise ValueError("the communicator id must be 128 bytes")
    return bytes(uid)


def max_over_ranks(x: float) -> float:
    """The largest value of `x` over all ranks (x itself without a process group)."""
    import torch
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier() -> None:
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.barrier()
