"""FLOP-balanced partition of packed sequences across ranks (multi-GPU bench).

Units are whole sequences (all heads of a sequence stay on one rank, so GQA
groups never split and dK/dV need no cross-GPU reduction).  A unit's cost is
its causal fwd+bwd FLOPs, proportional to L^2.  Longest-processing-time
greedy: sort by cost descending, give each unit to the least loaded rank.

Also the row maps of the multi-GPU data plane: which rows of the global
packed batch a rank owns (scatter), where its results go back (gather), and
the contiguous sequence groups in which rank 0 re-checks the gathered results.
"""
from __future__ import annotations

import heapq
import math
import random
from typing import List, Sequence, Tuple


def lpt_partition(lengths: Sequence[int], world: int) -> List[List[int]]:
    """Return, per rank, the sorted indices of the sequences it owns."""
    if world < 1:
        raise ValueError("world must be >= 1")
    heap = [(0.0, r) for r in range(world)]
    heapq.heapify(heap)
    parts: List[List[int]] = [[] for _ in range(world)]
    order = sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]) ** 2, i))
    for i in order:
        load, r = heapq.heappop(heap)
        parts[r].append(i)
        heapq.heappush(heap, (load + float(lengths[i]) ** 2, r))
    return [sorted(p) for p in parts]


def imbalance(lengths: Sequence[int], parts: List[List[int]]) -> float:
    """max rank cost / mean rank cost (1.0 = perfect)."""
    costs = [sum(float(lengths[i]) ** 2 for i in p) for p in parts]
    mean = sum(costs) / len(costs)
    return max(costs) / mean if mean > 0 else 1.0


def loguniform_lengths(n: int, lo: int, hi: int, seed: int = 0) -> List[int]:
    """n lengths log-uniform in [lo, hi] (fp64 draws, rounded)."""
    rng = random.Random(seed)
    return [int(round(math.exp(rng.uniform(math.log(lo), math.log(hi))))) for _ in range(n)]


def uniform_int_lengths(n: int, lo: int, hi: int, seed: int = 0) -> List[int]:
    """n lengths uniform-int in [lo, hi]."""
    rng = random.Random(seed)
    return [rng.randint(lo, hi) for _ in range(n)]


def cu_seqlens(lengths: Sequence[int]) -> List[int]:
    cu = [0]
    for L in lengths:
        cu.append(cu[-1] + int(L))
    return cu


def shard_token_index(lengths: Sequence[int], part: Sequence[int]) -> List[int]:
    """Rows of the global packed tensor (sequences in index order) that the
    sequences in ``part`` occupy, in the rank-local packing order."""
    cu = cu_seqlens(lengths)
    rows: List[int] = []
    for i in part:
        rows.extend(range(cu[i], cu[i + 1]))
    return rows


def scatter_rows(t, lengths: Sequence[int], parts: List[List[int]], rank: int):
    """Rank-local packed slice of a global packed tensor [T, ...]."""
    import torch
    idx = torch.tensor(shard_token_index(lengths, parts[rank]), dtype=torch.long, device=t.device)
    return t.index_select(0, idx)


def gather_rows(local_tensors, lengths: Sequence[int], parts: List[List[int]]):
    """Inverse of scatter_rows: place every rank's rows back in global order."""
    import torch
    T = sum(int(L) for L in lengths)
    first = local_tensors[0]
    out = first.new_zeros((T,) + tuple(first.shape[1:]))
    for rank, t in enumerate(local_tensors):
        idx = torch.tensor(shard_token_index(lengths, parts[rank]), dtype=torch.long, device=t.device)
        out.index_copy_(0, idx, t)
    return out


def local_rows_of(lengths: Sequence[int], part: Sequence[int], seqs: Sequence[int]) -> List[int]:
    """Rows, in a rank's local packing (its sequences ``part`` in order), of the
    sequences ``seqs`` (a subset of ``part``, in the order given)."""
    pos = {}
    off = 0
    for i in part:
        pos[i] = off
        off += int(lengths[i])
    rows: List[int] = []
    for i in seqs:
        rows.extend(range(pos[i], pos[i] + int(lengths[i])))
    return rows


def sequence_groups(lengths: Sequence[int], n_groups: int) -> List[Tuple[int, int]]:
    """Split the sequences (in global order) into at most ``n_groups``
    contiguous ranges [a, b) of about equal token counts."""
    T = sum(int(L) for L in lengths)
    bounds, acc = [0], 0
    for i, L in enumerate(lengths):
        acc += int(L)
        if acc >= T * len(bounds) / n_groups and len(bounds) < n_groups and i + 1 < len(lengths):
            bounds.append(i + 1)
    bounds.append(len(lengths))
    return [(a, b) for a, b in zip(bounds[:-1], bounds[1:]) if b > a]


def owner_of(parts: List[List[int]]) -> List[int]:
    """Rank owning each sequence."""
    n = sum(len(p) for p in parts)
    own = [-1] * n
    for r, p in enumerate(parts):
        for i in p:
            own[i] = r
    return own
