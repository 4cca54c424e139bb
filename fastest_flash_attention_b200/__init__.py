"""B200-native (sm_100a) flash attention with the public API of
MindIntels/fastest_flash_attention (reference __init__.py:40-88)."""
from .config import AttentionConfig
from .utils import auto_select_block_size, check_triton_available
from .attention import fastest_flash_attn_forward

__version__ = "1.0.0"
