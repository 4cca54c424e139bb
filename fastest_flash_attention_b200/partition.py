"""Work partitioning across the GPUs of one node (one process per GPU).

Attention over (batch element, kv head) groups is independent: a GQA group
(one kv head with its query heads) reads and writes nothing another group
touches, so prefill forward and backward split across ranks by groups with
no collective on the data path.  Decode splits by request; requests have
very different context lengths, so they are balanced by their K/V bytes
(proportional to the context length) with greedy longest-processing-time
assignment.

The reference has no multi-GPU path; these helpers define the split that
``bench.py --gpus N`` and callers use.  All functions are pure host logic.
"""
from __future__ import annotations

from typing import List, Sequence, Tuple

Block = Tuple[int, int, int, int]  # (b0, b1, h0, h1): batch [b0, b1) x kv heads [h0, h1)


def group_range(n_groups: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous balanced range [g0, g1) of group indices for ``rank``
    (group counts differ by at most one between ranks)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    base, extra = divmod(n_groups, world)
    g0 = rank * base + min(rank, extra)
    return g0, g0 + base + (1 if rank < extra else 0)


def gqa_group_blocks(B: int, Hkv: int, rank: int, world: int) -> List[Block]:
    """This rank's share of the B x Hkv GQA groups (flattened batch-major),
    as the fewest rectangles of whole batch elements and kv-head ranges.
    Each rectangle is one kernel launch over q[b0:b1, h0*G:h1*G] and
    k/v[b0:b1, h0:h1] (G = query heads per kv head)."""
    g0, g1 = group_range(B * Hkv, rank, world)
    blocks: List[Block] = []
    g = g0
    while g < g1:
        b, h = divmod(g, Hkv)
        if h == 0 and g + Hkv <= g1:  # whole batch elements
            nb = (g1 - g) // Hkv
            blocks.append((b, b + nb, 0, Hkv))
            g += nb * Hkv
        else:  # a run of heads inside one batch element
            h1 = min(Hkv, h + (g1 - g))
            blocks.append((b, b + 1, h, h1))
            g += h1 - h
    return blocks


def lpt_partition(costs: Sequence[float], world: int) -> List[List[int]]:
    """Greedy longest-processing-time assignment: items in decreasing cost
    order, each to the currently least-loaded rank (lowest rank on ties).
    Returns, per rank, its item indices in increasing order.  The largest
    load is within max(costs) of the best possible split."""
    if world <= 0:
        raise ValueError("world must be positive")
    order = sorted(range(len(costs)), key=lambda i: (-costs[i], i))
    loads = [0.0] * world
    parts: List[List[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda j: (loads[j], j))
        loads[r] += costs[i]
        parts[r].append(i)
    return [sorted(p) for p in parts]
