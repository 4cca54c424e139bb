"""B200-native (sm_100a) flash attention with the public API of
MindIntels/fastest_flash_attention (reference __init__.py:40-88)."""
from .config import AttentionConfig
from .utils import auto_select_block_size, check_triton_available
from .attention import (
    fastest_flash_attn_forward,
    fastest_flash_attn_backward,
    fastest_flash_attn_func,
    FastestFlashAttnFunc,
)
from .block_sparse import (
    create_causal_block_mask,
    create_sliding_window_block_mask,
    create_local_block_mask,
    combine_block_masks,
)

__version__ = "1.0.0"
from .kv_cache import PagedKVCache, ContinuousKVCache
from .decode import paged_decode
from .fa4 import FA4AttnFunc, fa4_attn_func, fa4_forward_dispatch
from .modules import FastestFlashMHA, FastestFlashGQA, FastestFlashMLA, FastestFlashFA4, RotaryEmbedding
from .mla import MLADecoder, MLALatentCache, mla_decode, absorbed_weights
from .utils import repeat_kv
from .ring import ring_attention_forward, ring_attention_backward, ring_attention_func, zigzag_shard, zigzag_unshard

__all__ = [
    "AttentionConfig", "fastest_flash_attn_forward", "fastest_flash_attn_backward", "fastest_flash_attn_func",
    "FastestFlashAttnFunc", "fa4_attn_func", "fa4_forward_dispatch", "FA4AttnFunc", "FastestFlashMHA",
    "FastestFlashGQA", "FastestFlashMLA", "FastestFlashFA4", "PagedKVCache", "ContinuousKVCache",
    "create_causal_block_mask", "create_sliding_window_block_mask", "create_local_block_mask",
    "auto_select_block_size", "check_triton_available", "paged_decode", "MLADecoder", "mla_decode",
    "ring_attention_forward", "ring_attention_backward", "ring_attention_func", "zigzag_shard", "zigzag_unshard",
]
