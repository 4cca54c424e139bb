"""nn.Module wrappers — drop-ins for the reference's modules/flash_{mha,gqa,mla,fa4}.py.

Parameter names and shapes match the reference so its state_dicts load
unchanged (q_proj/k_proj/v_proj/o_proj; MLA q_rope_proj/kv_down_proj/
kv_up_proj/k_rope_proj and the rope.inv_freq buffer).  Attention runs on the
sm_100a kernels through the functional API; projections are ordinary
nn.Linear layers.

Differences from the reference, all in the direction of less work or more
accuracy:
* GQA does not materialise repeated K/V heads (flash_gqa.py:102-103); the
  kernels read each K/V head once per query-head group.
* The query/key/value views keep the [B, S, H, D] storage of the projections
  (no transpose copy); the output is produced in the layout o_proj reads.
* MLA attends with 128-dim values instead of values zero-padded to 192
  (flash_mla.py:152); the padding columns are re-inserted (as zeros) before
  o_proj so its weight layout is unchanged.  RoPE positions are built in fp32
  (the reference builds them in x.dtype, flash_mla.py:41, which rounds
  positions above 256 in bf16).
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .attention import fastest_flash_attn_forward, fastest_flash_attn_func
from .fa4 import fa4_attn_func, fa4_forward_dispatch


def _heads(x: torch.Tensor, B: int, S: int, H: int, D: int) -> torch.Tensor:
    return x.view(B, S, H, D).transpose(1, 2)


def _merge(o: torch.Tensor, B: int, S: int) -> torch.Tensor:
    return o.transpose(1, 2).reshape(B, S, -1)


class _AttnBase(nn.Module):
    def _attend(self, q, k, v, use_causal, bs, kv_cache, return_lse, fa4: bool = False):
        if self.training and not return_lse and kv_cache is None:
            if fa4:
                out = fa4_attn_func(q, k, v, scale=self.scale, causal=use_causal, block_size=bs or 64,
                                    softcap=self.softcap, sliding_window=self.sliding_window,
                                    use_poly_exp=self.use_poly_exp, rescale_threshold=self.rescale_threshold,
                                    pingpong=self.pingpong, deterministic=self.deterministic)
            else:
                out = fastest_flash_attn_func(q, k, v, scale=self.scale, causal=use_causal, block_size=bs or 64,
                                              softcap=self.softcap, sliding_window=self.sliding_window)
            return out, None
        fn = fa4_forward_dispatch if fa4 else fastest_flash_attn_forward
        return fn(q, k, v, scale=self.scale, causal=use_causal, block_size=bs, softcap=self.softcap,
                  sliding_window=self.sliding_window, kv_cache=kv_cache, return_lse=return_lse)


class FastestFlashMHA(_AttnBase):
    """Multi-head attention (modules/flash_mha.py:20-158)."""

    def __init__(self, hidden_size: int, num_heads: int, head_dim: Optional[int] = None, dropout: float = 0.0,
                 bias: bool = False, causal: bool = False, block_size: int = 0, softcap: Optional[float] = None,
                 sliding_window: Optional[int] = None):
        super().__init__()
        self.hidden_size = hidden_size
        self.num_heads = num_heads
        self.head_dim = head_dim or hidden_size // num_heads
        assert self.head_dim * num_heads == hidden_size, "hidden_size must equal num_heads * head_dim"
        self.default_causal = causal
        self.block_size = block_size
        self.softcap = softcap
        self.sliding_window = sliding_window
        self.q_proj = nn.Linear(hidden_size, hidden_size, bias=bias)
        self.k_proj = nn.Linear(hidden_size, hidden_size, bias=bias)
        self.v_proj = nn.Linear(hidden_size, hidden_size, bias=bias)
        self.o_proj = nn.Linear(hidden_size, hidden_size, bias=bias)
        self.scale = 1.0 / math.sqrt(self.head_dim)

    def load_weights(self, w_q, w_k, w_v, w_o):
        self.q_proj.weight.data.copy_(w_q)
        self.k_proj.weight.data.copy_(w_k)
        self.v_proj.weight.data.copy_(w_v)
        self.o_proj.weight.data.copy_(w_o)

    def forward(self, x: torch.Tensor, causal: Optional[bool] = None, block_size: Optional[int] = None,
                kv_cache: Optional[Tuple[torch.Tensor, torch.Tensor]] = None, return_lse: bool = False):
        B, S, _ = x.shape
        use_causal = causal if causal is not None else self.default_causal
        bs = block_size or self.block_size or None
        H, D = self.num_heads, self.head_dim
        q, k, v = (_heads(p(x), B, S, H, D) for p in (self.q_proj, self.k_proj, self.v_proj))
        out, lse = self._attend(q, k, v, use_causal, bs, kv_cache, return_lse)
        out = self.o_proj(_merge(out, B, S))
        return (out, lse) if return_lse else out

    def extra_repr(self) -> str:
        return (f"hidden={self.hidden_size}, heads={self.num_heads}, head_dim={self.head_dim}, "
                f"block_size={self.block_size}, causal={self.default_causal}, softcap={self.softcap}, "
                f"window={self.sliding_window}")


class FastestFlashGQA(_AttnBase):
    """Grouped-query attention (modules/flash_gqa.py:22-139); K/V heads are not repeated."""

    def __init__(self, hidden_size: int, num_heads: int, num_kv_heads: int, head_dim: Optional[int] = None,
                 bias: bool = False, causal: bool = False, block_size: int = 0, softcap: Optional[float] = None,
                 sliding_window: Optional[int] = None):
        super().__init__()
        self.hidden_size = hidden_size
        self.num_heads = num_heads
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim or hidden_size // num_heads
        self.default_causal = causal
        self.block_size = block_size
        self.softcap = softcap
        self.sliding_window = sliding_window
        assert num_heads % num_kv_heads == 0, "num_heads must be divisible by num_kv_heads"
        self.q_proj = nn.Linear(hidden_size, num_heads * self.head_dim, bias=bias)
        self.k_proj = nn.Linear(hidden_size, num_kv_heads * self.head_dim, bias=bias)
        self.v_proj = nn.Linear(hidden_size, num_kv_heads * self.head_dim, bias=bias)
        self.o_proj = nn.Linear(num_heads * self.head_dim, hidden_size, bias=bias)
        self.scale = 1.0 / math.sqrt(self.head_dim)

    def forward(self, x: torch.Tensor, causal: Optional[bool] = None, block_size: Optional[int] = None,
                kv_cache: Optional[Tuple[torch.Tensor, torch.Tensor]] = None, return_lse: bool = False):
        B, S, _ = x.shape
        use_causal = causal if causal is not None else self.default_causal
        bs = block_size or self.block_size or None
        D = self.head_dim
        q = _heads(self.q_proj(x), B, S, self.num_heads, D)
        k = _heads(self.k_proj(x), B, S, self.num_kv_heads, D)
        v = _heads(self.v_proj(x), B, S, self.num_kv_heads, D)
        out, lse = self._attend(q, k, v, use_causal, bs, kv_cache, return_lse)
        out = self.o_proj(_merge(out, B, S))
        return (out, lse) if return_lse else out

    def extra_repr(self) -> str:
        return (f"hidden={self.hidden_size}, q_heads={self.num_heads}, kv_heads={self.num_kv_heads}, "
                f"head_dim={self.head_dim}, causal={self.default_causal}, softcap={self.softcap}")


class FastestFlashFA4(FastestFlashMHA):
    """FA4 multi-head attention (modules/flash_fa4.py:26-190)."""

    def __init__(self, hidden_size: int, num_heads: int, head_dim: Optional[int] = None, bias: bool = False,
                 causal: bool = False, block_size: int = 0, softcap: Optional[float] = None,
                 sliding_window: Optional[int] = None, use_poly_exp: bool = True, rescale_threshold: float = 0.0,
                 pingpong: bool = True, deterministic: bool = False):
        super().__init__(hidden_size, num_heads, head_dim, bias=bias, causal=causal, block_size=block_size,
                         softcap=softcap, sliding_window=sliding_window)
        self.use_poly_exp = use_poly_exp
        self.rescale_threshold = rescale_threshold
        self.pingpong = pingpong
        self.deterministic = deterministic

    def forward(self, x: torch.Tensor, causal: Optional[bool] = None, block_size: Optional[int] = None,
                kv_cache: Optional[Tuple[torch.Tensor, torch.Tensor]] = None, return_lse: bool = False):
        B, S, _ = x.shape
        use_causal = causal if causal is not None else self.default_causal
        bs = block_size or self.block_size or None
        H, D = self.num_heads, self.head_dim
        q, k, v = (_heads(p(x), B, S, H, D) for p in (self.q_proj, self.k_proj, self.v_proj))
        out, lse = self._attend(q, k, v, use_causal, bs, kv_cache, return_lse, fa4=True)
        out = self.o_proj(_merge(out, B, S))
        return (out, lse) if return_lse else out

    def extra_repr(self) -> str:
        return super().extra_repr() + (f", poly_exp={self.use_poly_exp}, rescale_τ={self.rescale_threshold}, "
                                       f"pingpong={self.pingpong}, deterministic={self.deterministic}")


class RotaryEmbedding(nn.Module):
    """Half-split RoPE (modules/flash_mla.py:29-52); positions in fp32."""

    def __init__(self, dim: int, max_len: int = 8192, base: float = 10000.0):
        super().__init__()
        inv_freq = 1.0 / (base ** (torch.arange(0, dim, 2).float() / dim))
        self.register_buffer("inv_freq", inv_freq)
        self.max_len = max_len

    def cos_sin(self, S: int, offset: int, device) -> Tuple[torch.Tensor, torch.Tensor]:
        t = torch.arange(offset, offset + S, device=device, dtype=torch.float32)
        freqs = torch.outer(t, self.inv_freq.to(device=device, dtype=torch.float32))
        return freqs.cos(), freqs.sin()  # [S, dim/2]

    def forward(self, x: torch.Tensor, offset: int = 0) -> torch.Tensor:
        """Rotate x [..., S, dim]."""
        cos, sin = self.cos_sin(x.size(-2), offset, x.device)
        h = x.size(-1) // 2
        x1, x2 = x[..., :h].float(), x[..., h:].float()
        return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], dim=-1).to(x.dtype)


class FastestFlashMLA(nn.Module):
    """DeepSeek-style multi-latent attention (modules/flash_mla.py:55-179).

    forward(x) is the reference's non-absorbed computation (up-projected K/V)
    on the sm_100a forward at head dims (qk 192, v 128).  ``decode`` /
    ``absorbed_weights`` give the absorbed latent form used for decoding
    (see fastest_flash_attention_b200.mla).
    """

    def __init__(self, hidden_size: int, num_heads: int, head_dim: int = 128, latent_dim: int = 512,
                 rope_dim: int = 64, causal: bool = True, block_size: int = 0):
        super().__init__()
        self.hidden_size = hidden_size
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.latent_dim = latent_dim
        self.rope_dim = rope_dim
        self.default_causal = causal
        self.block_size = block_size
        self.attn_dim = head_dim + rope_dim
        self.scale = 1.0 / math.sqrt(self.attn_dim)
        self.q_proj = nn.Linear(hidden_size, num_heads * head_dim, bias=False)
        self.q_rope_proj = nn.Linear(hidden_size, num_heads * rope_dim, bias=False)
        self.kv_down_proj = nn.Linear(hidden_size, latent_dim, bias=False)
        self.kv_up_proj = nn.Linear(latent_dim, num_heads * (head_dim + head_dim), bias=False)
        self.k_rope_proj = nn.Linear(hidden_size, rope_dim, bias=False)
        self.rope = RotaryEmbedding(rope_dim)
        self.o_proj = nn.Linear(num_heads * (head_dim + rope_dim), hidden_size, bias=False)

    def qkv(self, x: torch.Tensor, offset: int = 0):
        """Q [B,H,S,192], K [B,H,S,192], V [B,H,S,128] as the reference builds them (flash_mla.py:133-150)."""
        B, S, _ = x.shape
        H, d, r = self.num_heads, self.head_dim, self.rope_dim
        q_nope = _heads(self.q_proj(x), B, S, H, d)
        q_rope = self.rope(_heads(self.q_rope_proj(x), B, S, H, r), offset)
        q = torch.cat([q_nope, q_rope], dim=-1)
        kv = _heads(self.kv_up_proj(self.kv_down_proj(x)), B, S, H, 2 * d)
        k_rope = self.rope(self.k_rope_proj(x).unsqueeze(1), offset).expand(-1, H, -1, -1)
        k = torch.cat([kv[..., :d], k_rope], dim=-1)
        v = kv[..., d:]
        return q, k, v

    def forward(self, x: torch.Tensor, causal: Optional[bool] = None, block_size: Optional[int] = None):
        B, S, _ = x.shape
        use_causal = causal if causal is not None else self.default_causal
        bs = block_size or self.block_size or None
        q, k, v = self.qkv(x)
        if self.training:
            out = fastest_flash_attn_func(q, k, v, scale=self.scale, causal=use_causal, block_size=bs or 64)
        else:
            out, _ = fastest_flash_attn_forward(q, k, v, scale=self.scale, causal=use_causal, block_size=bs)
        out = F.pad(out, (0, self.rope_dim))  # the reference's zero value columns (flash_mla.py:152)
        return self.o_proj(_merge(out, B, S))

    def extra_repr(self) -> str:
        return (f"hidden={self.hidden_size}, heads={self.num_heads}, head_dim={self.head_dim}, "
                f"latent={self.latent_dim}, rope_dim={self.rope_dim}")
