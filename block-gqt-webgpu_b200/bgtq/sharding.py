"""Multi-rank plumbing of the batched decode workload: one process per GPU.

The workload shards by sequence (every sequence's cache lives on one rank), so the data
path has no collective.  What the ranks share: which global sequences a rank owns (a
contiguous share of one batch), a barrier around timed regions, the maximum of the
per-rank timings, and, after the timed region, the gather of every rank's attention
outputs to rank 0 with exact per-rank checksums that prove the gathered copy.  The helpers take the
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


def bit_checksum(x) -> int:
    """Order-independent exact checksum of a tensor's bits: the sum of its 32-bit words as
    int64 (integer addition, so every device and reduction order gives the same value)."""
    import torch
    t = x.contiguous().view(-1)
    words = t.view(torch.int32) if t.element_size() == 4 else t.view(torch.int16)
    return int(words.to(torch.int64).sum())


def gather_to_root(x, counts, dist, device, dim: int = 0):
    """Gather every rank's ``x`` to rank 0 along ``dim``: rank r holds ``counts[r]`` entries
    of that dimension (a contiguous share of the batch, ``split_range``).  Returns the
    concatenation in rank order on rank 0 and None elsewhere; a single process returns
    ``x`` itself.  Shares are padded to the largest count so one collective carries them."""
    import torch
    if dist is None:
        return x
    world, rank = dist.get_world_size(), dist.get_rank()
    if len(counts) != world or x.shape[dim] != counts[rank]:
        raise ValueError("counts must give every rank's share of the gathered dimension")
    width = max(counts)
    shape = list(x.shape)
    shape[dim] = width
    padded = torch.zeros(shape, dtype=x.dtype, device=device)
    padded.narrow(dim, 0, counts[rank]).copy_(x)
    parts = [torch.empty_like(padded) for _ in range(world)] if rank == 0 else None
    dist.gather(padded, gather_list=parts, dst=0)
    if rank != 0:
        return None
    return torch.cat([p.narrow(dim, 0, c) for p, c in zip(parts, counts)], dim=dim)


def gather_ints(values, dist, device):
    """Every rank's list of Python ints (equal lengths), in rank order, on every rank."""
    import torch
    t = torch.tensor([int(v) for v in values], dtype=torch.int64, device=device)
    if dist is None:
        return [[int(v) for v in t.cpu()]]
    out = [torch.zeros_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(out, t)
    return [[int(v) for v in o.cpu()] for o in out]


def barrier(dist, synchronize=None):
    """Device synchronisation, then a barrier over ranks, then synchronisation again, so
    a timed region starts and ends with every rank's queued work finished."""
    if synchronize:
        synchronize()
    if dist is not None:
        dist.barrier()
    if synchronize:
        synchronize()
