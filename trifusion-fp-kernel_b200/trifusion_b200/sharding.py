"""Data-parallel inference over the GPUs of one node.

Every clip is independent (each row of the recurrence starts from a zero
state), so batches are partitioned across ranks with no exchange on the data
path: one process per GPU runs its own ``InferenceEngine`` (own CUDA graphs),
and a single collective at the end gathers the ``[n, 5]`` logits with their
clip indices to every rank.

Partitioning is longest-processing-time first on a batch's padded
audio-seconds (batch size × bucket length × channels), which bounds the
slowest rank at 4/3 of the optimum.
"""

from __future__ import annotations

import heapq


def batch_cost(limit_samples, rows):
    """Padded work of one planned batch: clips × samples × channels."""
    return len(rows) * limit_samples * max(r.channels for r in rows)


def lpt_partition(costs, world):
    """Assign item i (cost ``costs[i]``) to a rank; returns ``[[items of rank r]]``.

    Items are taken in decreasing cost (ties by index) and each goes to the
    currently least-loaded rank (ties to the lower rank): deterministic, so
    every rank computes the same assignment without communicating.
    """
    if world < 1:
        raise ValueError("world must be >= 1")
    heap = [(0, r) for r in range(world)]
    owned = [[] for _ in range(world)]
    for i in sorted(range(len(costs)), key=lambda i: (-costs[i], i)):
        load, r = heapq.heappop(heap)
        owned[r].append(i)
        heapq.heappush(heap, (load + costs[i], r))
    return [sorted(items) for items in owned]


def gather_logits(indices, logits, group=None, capacity=None):
    """All-gather each rank's ``(indices [n_r] int64, logits [n_r, 5])`` and
    return them concatenated in clip-index order, on every rank.

    With ``capacity`` (an upper bound on every rank's ``n_r``, e.g. from the
    deterministic partition every rank computes) this is one all-gather: each
    rank sends ``capacity + 1`` rows of float64, the first holding its count.
    Without it, two: the per-rank counts, then the payload padded to the largest.
    Indices travel as float64, exact below 2**53.
    """
    import torch
    import torch.distributed as dist

    world = dist.get_world_size(group)
    dev = logits.device
    width = logits.shape[1] if logits.dim() == 2 else 5
    n_local = indices.numel()
    if capacity is None:
        n = torch.tensor([n_local], device=dev, dtype=torch.int64)
        counts = [torch.zeros_like(n) for _ in range(world)]
        dist.all_gather(counts, n, group=group)
        counts = [int(c.item()) for c in counts]
        top, head = max(counts), 0
    else:
        if n_local > capacity:
            raise ValueError(f"gather_logits: {n_local} rows exceed the capacity {capacity}")
        counts, top, head = None, int(capacity), 1
    pack = torch.zeros(head + top, 1 + width, device=dev, dtype=torch.float64)
    if head:
        pack[0, 0] = n_local
    if n_local:
        pack[head:head + n_local, 0] = indices.to(dev, torch.float64)
        pack[head:head + n_local, 1:] = logits.to(torch.float64)
    parts = [torch.empty_like(pack) for _ in range(world)]
    dist.all_gather(parts, pack, group=group)
    if counts is None:
        counts = [int(p[0, 0].item()) for p in parts]
    rows = torch.cat([p[head:head + c] for p, c in zip(parts, counts)])
    order = rows[:, 0].argsort()
    return rows[order, 0].long(), rows[order, 1:].to(logits.dtype)
