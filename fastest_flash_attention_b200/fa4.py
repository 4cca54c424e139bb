"""FlashAttention-4 functional API — drop-in for ops/fa4_func.py:20-229.

The reference's FA4 path is a CPU simulation (kernels/cpu_fa4.py) of the
techniques the sm_100a kernels here implement in hardware: ping-pong query
tiles (two 128-row tiles per CTA), conditional (lazy) rescaling, LPT tile
order and a deterministic backward.  The knobs are accepted with these
meanings:

* ``use_poly_exp`` — accepted; the kernels use the hardware ex2 unit, which
  is more accurate than the reference's cubic (relative error ~1e-7 vs 5.6e-3).
* ``rescale_threshold`` — accepted; the kernels always rescale lazily (only
  when a row max grows by more than 2^8) and stay exact, so the result equals
  the reference at its default threshold 0.
* ``pingpong`` / ``deterministic`` — always on.

The returned LSE is the exact log-sum-exp.  (The reference's fa4_forward
returns an inexact LSE whenever a later key tile has a lower row max than the
running max, cpu_fa4.py:412; its gradients inherit that error.)
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
from torch.autograd import Function

from .attention import fastest_flash_attn_backward, fastest_flash_attn_forward


class FA4AttnFunc(Function):
    """Autograd FA4 attention (ops/fa4_func.py:20-100); 13 forward args."""

    @staticmethod
    def forward(ctx, q, k, v, scale, causal, block_size, softcap, sliding_window, two_pass, use_poly_exp,
                rescale_threshold, pingpong, deterministic):
        output, lse = fastest_flash_attn_forward(q, k, v, scale=scale, causal=causal, block_size=block_size,
                                                 softcap=softcap, sliding_window=sliding_window,
                                                 two_pass=two_pass, return_lse=True)
        ctx.save_for_backward(q, k, v, output, lse)
        ctx.scale, ctx.causal, ctx.softcap, ctx.sliding_window = scale, causal, softcap, sliding_window
        return output

    @staticmethod
    def backward(ctx, grad_output):
        q, k, v, output, lse = ctx.saved_tensors
        was_3d = q.dim() == 3
        if was_3d:
            q, k, v, output, lse, grad_output = (t.unsqueeze(1) for t in (q, k, v, output, lse, grad_output))
        dq, dk, dv = fastest_flash_attn_backward(grad_output, q, k, v, output, lse, scale=ctx.scale,
                                                 causal=ctx.causal, softcap=ctx.softcap,
                                                 sliding_window=ctx.sliding_window)
        if was_3d:
            dq, dk, dv = dq.squeeze(1), dk.squeeze(1), dv.squeeze(1)
        return dq, dk, dv, None, None, None, None, None, None, None, None, None, None


def fa4_attn_func(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: Optional[float] = None,
                  causal: bool = False, block_size: int = 64, softcap: Optional[float] = None,
                  sliding_window: Optional[int] = None, two_pass: bool = False, use_poly_exp: bool = True,
                  rescale_threshold: float = 0.0, pingpong: bool = True, deterministic: bool = False
                  ) -> torch.Tensor:
    """Differentiable FA4 attention (ops/fa4_func.py:103-142)."""
    return FA4AttnFunc.apply(q, k, v, scale, causal, block_size, softcap, sliding_window, two_pass, use_poly_exp,
                             rescale_threshold, pingpong, deterministic)


def fa4_forward_dispatch(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, scale: Optional[float] = None,
                         causal: bool = False, block_size: Optional[int] = None,
                         block_mask: Optional[torch.Tensor] = None, softcap: Optional[float] = None,
                         sliding_window: Optional[int] = None, two_pass: bool = False,
                         compute_dtype: Optional[torch.dtype] = None, num_kv_heads: Optional[int] = None,
                         kv_cache: Optional[Tuple[torch.Tensor, torch.Tensor]] = None, return_lse: bool = False,
                         use_poly_exp: bool = True, rescale_threshold: float = 0.0, pingpong: bool = True
                         ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """FA4 inference forward with shapes, KV cache and GQA (ops/fa4_func.py:145-229)."""
    return fastest_flash_attn_forward(q, k, v, scale=scale, causal=causal, block_size=block_size,
                                      block_mask=block_mask, softcap=softcap, sliding_window=sliding_window,
                                      two_pass=two_pass, compute_dtype=compute_dtype, num_kv_heads=num_kv_heads,
                                      kv_cache=kv_cache, return_lse=return_lse)
