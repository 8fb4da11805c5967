"""Multi-GPU host logic: independent utterances partitioned over one process per GPU.

The reference runs one ``VoxCPM`` per worker (``README.md:96-103``); there is no exchange
between utterances, so nothing here is on the data path.  ``torch.distributed`` is used only
for timing (barrier, max over ranks) and for the re-queue of work a failed rank returns.
"""
from __future__ import annotations

from typing import Callable, Iterable, List, Sequence


def partition(n_items: int, world: int, rank: int) -> List[int]:
    """Contiguous block of ``range(n_items)`` for ``rank`` (sizes differ by at most one)."""
    base, extra = divmod(n_items, world)
    start = rank * base + min(rank, extra)
    return list(range(start, start + base + (1 if rank < extra else 0)))


def allmax(value: float, group=None, device=None) -> float:
    """Max of a float over the ranks of ``group`` (identity without a process group)."""
    import torch
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def aggregate_rate(local_units: float, local_seconds: float, group=None, device=None) -> float:
    """Whole-job rate: the units all ranks processed over the slowest rank's time."""
    import torch
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return local_units / local_seconds
    t = torch.tensor([float(local_units)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return float(t.item()) / allmax(local_seconds, group, device)


def waves(indices: Sequence[int], size: int) -> List[List[int]]:
    """Consecutive groups of at most ``size`` indices (the utterances decoded together)."""
    return [list(indices[i:i + size]) for i in range(0, len(indices), size)]


def run_partitioned(items: Sequence, work: Callable[[object], object], group=None, batch: int = 1) -> dict:
    """Process this rank's share of ``items`` with ``work``; items whose work raised are
    gathered from every rank and re-run round-robin by the ranks that did not fail (a rank
    that failed once gets no retries).  Returns ``{item_index: result}`` for the items this
    rank completed.  Every rank takes the same collective steps in the same order.

    With ``batch > 1`` the rank's share runs in waves of up to ``batch`` items: ``work``
    receives a list of items and returns one result per item; a wave that raised re-queues
    all of its items (retried one wave per healthy rank, in waves of ``batch`` again)."""
    import torch.distributed as dist
    dist_on = dist.is_available() and dist.is_initialized()
    world = dist.get_world_size(group) if dist_on else 1
    rank = dist.get_rank(group) if dist_on else 0

    def run(idx: List[int], done: dict, failed: list):
        try:
            if batch > 1:
                res = work([items[i] for i in idx])
                for i, r in zip(idx, res):
                    done[i] = r
            else:
                done[idx[0]] = work(items[idx[0]])
        except Exception:
            failed.extend(idx)

    done, failed = {}, []
    for wv in waves(partition(len(items), world, rank), max(1, batch)):
        run(wv, done, failed)
    if not dist_on:
        return done
    gathered: List[Iterable[int]] = [None] * world  # type: ignore[list-item]
    dist.all_gather_object(gathered, failed, group=group)
    healthy = [r for r in range(world) if not gathered[r]]
    retry = sorted(i for lst in gathered for i in lst)
    if healthy:
        for j, wv in enumerate(waves(retry, max(1, batch))):
            if healthy[j % len(healthy)] == rank:
                run(wv, done, [])  # failed twice: reported as missing from every rank's result
    return done
