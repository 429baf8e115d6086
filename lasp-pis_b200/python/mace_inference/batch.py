"""Batches of independent cells across GPUs (the C4 workload): LPT sharding by estimated work.

Each rank (one process per GPU, torch.distributed) evaluates its share of the cells with one
``mace_calculate_batch`` call per sub-batch; the only collective is the final gather of the
per-cell results to rank 0 -- cells never exchange data.  Work per cell is estimated as
N * (1 + E/N), with the neighbour count E/N taken from the cell's number density and the
cutoff sphere, since edges are only known after traversal.
"""
import heapq
import math

import numpy as np


def estimated_work(n_atoms, cell, cutoff=6.0):
    """N * (1 + expected neighbours per atom) for a periodic cell of n_atoms."""
    volume = abs(float(np.linalg.det(np.asarray(cell, np.float64).reshape(3, 3))))
    if n_atoms == 0 or volume == 0:
        return float(n_atoms)
    neighbours = 4.0 / 3.0 * math.pi * cutoff ** 3 * n_atoms / volume
    return n_atoms * (1.0 + neighbours)


def lpt_partition(weights, parts):
    """Longest-processing-time-first: each item, heaviest first, goes to the currently lightest
    part (ties to the lowest part index).  Returns one sorted list of item indices per part."""
    if parts < 1:
        raise ValueError("parts must be positive")
    heap = [(0.0, p) for p in range(parts)]
    out = [[] for _ in range(parts)]
    for i in sorted(range(len(weights)), key=lambda k: (-weights[k], k)):
        load, p = heapq.heappop(heap)
        out[p].append(i)
        heapq.heappush(heap, (load + float(weights[i]), p))
    return [sorted(x) for x in out]


def run_sharded(model, cells, rank=0, world=1, cutoff=6.0, gather=None):
    """Evaluate ``cells`` (a sequence of (xyz, Z, cell)) on ``world`` ranks.

    ``model`` is this rank's calculator (``NativeMH1`` on its GPU, or anything with
    ``calculate_batch``); ``gather(obj)`` returns the list of every rank's object on rank 0
    (None elsewhere) -- by default torch.distributed.gather_object when world > 1.  Rank 0
    returns the results in input order; other ranks return None.
    """
    weights = [estimated_work(len(z), c, cutoff) for _, z, c in cells]
    shards = lpt_partition(weights, world)
    mine = shards[rank]
    results = model.calculate_batch([cells[i] for i in mine]) if mine else []
    local = list(zip(mine, results))
    if world == 1:
        gathered = [local]
    else:
        if gather is None:
            import torch.distributed as dist

            def gather(obj):
                box = [None] * world if rank == 0 else None
                dist.gather_object(obj, box, dst=0)
                return box
        gathered = gather(local)
    if rank != 0:
        return None
    out = [None] * len(cells)
    for part in gathered:
        for i, r in part:
            out[i] = r
    return out
