"""Shape and numeric helpers mirroring the reference's utils.py."""
from __future__ import annotations

import math
from typing import Tuple

import torch


def check_triton_available() -> bool:
    """Reference name kept for drop-in imports (utils.py:20-29).

    This package has no Triton path; the function reports whether the
    sm_100a kernel library can run here (a CUDA device is present and the
    library is built).
    """
    if not torch.cuda.is_available():
        return False
    from . import _lib

    return _lib.lib_path().exists()


def auto_select_block_size(S_q: int, S_kv: int, D: int, max_block: int = 256, min_block: int = 16) -> int:
    """Block-size heuristic of utils.py:36-67.

    The sm_100a kernels use fixed 128x128 tiles; this value only sets the
    granularity at which a user ``block_mask`` is interpreted, exactly as in
    the reference.
    """
    budget = 4096
    bs = max(min_block, min(budget // max(D, 1), max_block))
    while bs > min_block and math.ceil(S_kv / bs) < 4:
        bs //= 2
    if bs > 0:
        bs = 1 << (bs.bit_length() - 1)
    return max(min_block, min(bs, max_block))


def safe_softmax(x: torch.Tensor, dim: int = -1, dtype: torch.dtype | None = None) -> torch.Tensor:
    """exp(x - max) / sum(exp(x - max)) with NaN rows zeroed (utils.py:74-86)."""
    if dtype is not None:
        x = x.to(dtype)
    x_max = x.max(dim=dim, keepdim=True).values
    e = torch.exp(x - x_max)
    return torch.nan_to_num(e / e.sum(dim=dim, keepdim=True), nan=0.0)


def logaddexp_safe(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return torch.logaddexp(a, b)


def maybe_unsqueeze_head(q, k, v) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, bool]:
    """[B,S,D] -> [B,1,S,D] for q/k/v (utils.py:98-108)."""
    if q.dim() == 3:
        return q.unsqueeze(1), k.unsqueeze(1), v.unsqueeze(1), True
    return q, k, v, False


def repeat_kv(kv: torch.Tensor, num_q_heads: int, num_kv_heads: int) -> torch.Tensor:
    """Materialised GQA head repeat (utils.py:111-130).

    Kept for API compatibility; the kernels read grouped K/V heads directly,
    so nothing in this package calls it on the hot path.
    """
    if num_q_heads == num_kv_heads:
        return kv
    ratio = num_q_heads // num_kv_heads
    B, H_kv, S, D = kv.shape
    return kv[:, :, None, :, :].expand(B, H_kv, ratio, S, D).reshape(B, num_q_heads, S, D)
