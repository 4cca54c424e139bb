"""AttentionConfig — same fields and defaults as the reference's config.py:15-81.

Only the fields the reference's forward dispatch reads are honoured
(causal, softcap, sliding_window, two_pass, compute_dtype, num_kv_heads,
return_lse, block sizes for block-mask granularity); the remaining knobs are
accepted for drop-in compatibility and have no effect on the sm_100a kernels,
whose tiles are fixed by the hardware mapping.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional, Tuple

import torch


@dataclass
class AttentionConfig:
    block_size_q: int = 0
    block_size_kv: int = 0
    causal: bool = False
    sliding_window: Optional[int] = None
    softcap: Optional[float] = None
    num_kv_heads: Optional[int] = None
    compute_dtype: Optional[torch.dtype] = None
    use_triton: bool = True
    two_pass: bool = False
    pipeline_stages: int = 2
    return_lse: bool = False
    dropout_p: float = 0.0
    deterministic: bool = False
    max_seqlen_q: int = 0
    max_seqlen_kv: int = 0
    page_size: int = 64

    def resolve_block_sizes(self, S_q: int, S_kv: int, D: int) -> Tuple[int, int]:
        """(block_q, block_kv), auto-selecting either that is 0 (config.py:75-81)."""
        from .utils import auto_select_block_size

        bq = self.block_size_q or auto_select_block_size(S_q, S_kv, D)
        bkv = self.block_size_kv or auto_select_block_size(S_q, S_kv, D)
        return bq, bkv
