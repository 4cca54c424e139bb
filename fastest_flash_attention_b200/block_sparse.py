"""Block-sparse mask generators (ops/block_sparse.py:17-132).

``[n_br, n_bc]`` bool masks, True = the (query block, key block) pair is
computed.  The forward kernel consumes them at the given block granularity
(``block_size`` of the forward call) and skips every 128-key tile that no
kept block touches.
"""
from __future__ import annotations

import math

import torch


def create_causal_block_mask(S_q: int, S_kv: int, block_q: int, block_kv: int, q_offset: int = 0) -> torch.Tensor:
    """(i, j) kept iff some query of block i is >= the first key of block j (block_sparse.py:17-45)."""
    n_br, n_bc = math.ceil(S_q / block_q), math.ceil(S_kv / block_kv)
    q_last = q_offset + torch.clamp((torch.arange(n_br) + 1) * block_q, max=S_q) - 1
    k_first = torch.arange(n_bc) * block_kv
    return q_last[:, None] >= k_first[None, :]


def create_sliding_window_block_mask(S_q: int, S_kv: int, block_q: int, block_kv: int, window_size: int,
                                     q_offset: int = 0) -> torch.Tensor:
    """(i, j) kept iff key block j overlaps [q_first - w + 1, q_last] (block_sparse.py:48-81)."""
    n_br, n_bc = math.ceil(S_q / block_q), math.ceil(S_kv / block_kv)
    i = torch.arange(n_br)
    j = torch.arange(n_bc)
    q_first = q_offset + i * block_q
    q_last = q_offset + torch.clamp((i + 1) * block_q, max=S_q) - 1
    k_first = j * block_kv
    k_last = torch.clamp((j + 1) * block_kv, max=S_kv) - 1
    return (k_last[None, :] >= (q_first[:, None] - window_size + 1)) & (k_first[None, :] <= q_last[:, None])


def create_local_block_mask(S_q: int, S_kv: int, block_q: int, block_kv: int, local_radius: int) -> torch.Tensor:
    """(i, j) kept iff block centres are within radius + max block (block_sparse.py:84-110)."""
    n_br, n_bc = math.ceil(S_q / block_q), math.ceil(S_kv / block_kv)
    qc = torch.arange(n_br) * block_q + block_q // 2
    kc = torch.arange(n_bc) * block_kv + block_kv // 2
    return (qc[:, None] - kc[None, :]).abs() <= local_radius + max(block_q, block_kv)


def combine_block_masks(*masks: torch.Tensor, mode: str = "and") -> torch.Tensor:
    """AND / OR of equally shaped masks (block_sparse.py:113-132)."""
    assert len(masks) >= 1
    out = masks[0]
    for m in masks[1:]:
        if mode == "and":
            out = out & m
        elif mode == "or":
            out = out | m
        else:
            raise ValueError(f"Unknown mode: {mode!r}")
    return out
