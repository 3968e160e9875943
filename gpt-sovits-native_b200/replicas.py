"""Multi-GPU host logic.

Utterances are independent (no exchange step anywhere on the path), so N GPUs
run N replicas of the engines, one process per GPU, each on its own shard of
the utterances.  torch.distributed is used only for start/stop barriers, the
max-over-ranks step time and gathering results on rank 0 — never on the data
path.  The backend is NCCL on GPUs and gloo for the CPU tests of this logic.
"""
from __future__ import annotations

import datetime
import os


def shard(n_items: int, rank: int, world: int) -> range:
    """Contiguous block of the n_items utterances owned by `rank` (sizes
    differ by at most one; every item is owned exactly once)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    base, extra = divmod(n_items, world)
    lo = rank * base + min(rank, extra)
    return range(lo, lo + base + (1 if rank < extra else 0))


def init(backend: str, rank: int, world: int, device=None, timeout_s: int = 180) -> None:
    """Join the process group (MASTER_ADDR defaults to 127.0.0.1)."""
    if world <= 1:
        return
    import torch.distributed as dist

    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    kw = {"device_id": device} if device is not None else {}
    dist.init_process_group(backend, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s), **kw)


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value: float, world: int, device=None) -> float:
    """The largest of the ranks' values (device: where the reduction tensor
    lives — a CUDA device for NCCL, None for gloo)."""
    if world <= 1:
        return float(value)
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(value)], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_to_rank0(obj, rank: int, world: int):
    """Every rank's object, in rank order, on rank 0 (None elsewhere)."""
    if world <= 1:
        return [obj]
    import torch.distributed as dist

    out = [None] * world if rank == 0 else None
    dist.gather_object(obj, out, dst=0)
    return out


def close(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
