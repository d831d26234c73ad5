"""Multi-rank plumbing of the batched decode workload: one process per GPU.

The workload shards by sequence (every sequence's cache lives on one rank), so the data
path has no collective.  What the ranks share is bookkeeping: which global sequences a
rank owns, a barrier around timed regions, the maximum of the per-rank timings, and a
gather of per-rank output checksums for verification.  The helpers take the
``torch.distributed`` module and the device of the collective tensors, so the same code
runs over NCCL on GPUs and over gloo on CPU (the tests).
"""
from __future__ import annotations

import datetime
import os


def sequence_range(per_rank: int, rank: int) -> range:
    """Global sequence ids owned by ``rank`` when every rank holds ``per_rank`` sequences
    (weak scaling: the global batch is ``per_rank * world``)."""
    if per_rank < 0 or rank < 0:
        raise ValueError("per_rank and rank must be non-negative")
    return range(rank * per_rank, (rank + 1) * per_rank)


def split_range(total: int, world: int, rank: int) -> range:
    """Contiguous share of ``total`` sequences for ``rank`` of ``world`` (strong scaling):
    the first ``total % world`` ranks take one extra sequence."""
    if world < 1 or not 0 <= rank < world or total < 0:
        raise ValueError("need world >= 1, 0 <= rank < world, total >= 0")
    base, extra = divmod(total, world)
    first = rank * base + min(rank, extra)
    return range(first, first + base + (1 if rank < extra else 0))


def init_from_env(backend: str, timeout_s: float = 300.0, device=None):
    """Join the process group described by RANK / WORLD_SIZE / MASTER_ADDR / MASTER_PORT
    when WORLD_SIZE > 1; returns ``torch.distributed`` or None for a single process.  The
    short timeout makes ranks that wait for a missing peer fail with an error."""
    world = int(os.environ.get("WORLD_SIZE", 1))
    if world <= 1:
        return None
    import torch.distributed as dist
    kw = {"timeout": datetime.timedelta(seconds=timeout_s)}
    if device is not None and backend == "nccl":
        kw["device_id"] = device
    dist.init_process_group(backend, **kw)
    return dist


def max_over_ranks(values, dist, device):
    """Element-wise maximum of a list of floats over all ranks (float64)."""
    import torch
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(x) for x in t.cpu()]


def gather_checksums(tensors, dist, device):
    """Sum of every tensor in ``tensors`` (float64), gathered from all ranks in rank
    order; a single process returns a one-element list."""
    import torch
    s = torch.zeros(1, dtype=torch.float64, device=device)
    for x in tensors:
        s += x.to(device=device, dtype=torch.float64).sum()
    if dist is None:
        return [float(s)]
    out = [torch.zeros_like(s) for _ in range(dist.get_world_size())]
    dist.all_gather(out, s)
    return [float(o) for o in out]


def barrier(dist, synchronize=None):
    """Device synchronisation, then a barrier over ranks, then synchronisation again, so
    a timed region starts and ends with every rank's queued work finished."""
    if synchronize:
        synchronize()
    if dist is not None:
        dist.barrier()
    if synchronize:
        synchronize()
