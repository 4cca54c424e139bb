"""Paged-KV decode (one query token per request) on the sm_100a kernels.

The reference decodes by gathering each sequence's pages into a contiguous
tensor (ops/kv_cache.py:208-232) and running the prefill forward with
S_q = 1 (ops/attention_forward.py:23).  ``paged_decode`` computes the same
attention directly from the page pool: a split-KV kernel reads every K/V
byte of the context once per kv head (all query heads of a GQA group share
the read) and a merge kernel combines the splits by LSE.
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from . import _lib


def default_chunks_per_split(ctx_max: int, R: int, Hkv: int, num_sms: int = 148) -> int:
    """16-token chunks per CTA.  Long splits (up to 2048 tokens) keep the
    per-split merge traffic small and measured best on B200; short contexts or
    few requests get smaller splits so every SM still has several CTAs."""
    chunks = max(1, math.ceil(ctx_max / 16))
    target_ctas = 8 * num_sms
    splits = max(1, math.ceil(target_ctas / max(1, R * Hkv)))
    return max(16, min(128, math.ceil(chunks / splits)))


def check_block_table(block_table: torch.Tensor, ctx_lens: torch.Tensor, num_pages: int, page_size: int) -> None:
    """Host-side validation of paging data (CPU tensors): every context length
    in [0, width * page_size] and every page id a request reads in
    [0, num_pages).  Raises ValueError naming the first bad request.  The
    decode kernels repeat these checks on the device (reporting through the
    error word) for tables that never pass through the host."""
    bt = block_table.to("cpu", torch.int64)
    lens = ctx_lens.to("cpu", torch.int64)
    if bt.dim() != 2 or lens.dim() != 1 or lens.numel() != bt.shape[0]:
        raise ValueError("block_table must be [R, max_pages] and ctx_lens [R]")
    width = bt.shape[1]
    bad_len = (lens < 0) | (lens > width * page_size)
    if bool(bad_len.any()):
        r = int(bad_len.nonzero()[0, 0])
        raise ValueError(f"ctx_lens[{r}] = {int(lens[r])} is outside [0, {width * page_size}] "
                         f"({width} pages of {page_size} tokens)")
    used = (torch.arange(width)[None, :] * page_size) < lens[:, None]  # pages each request reads
    bad = used & ((bt < 0) | (bt >= num_pages))
    if bool(bad.any()):
        r, c = (int(x) for x in bad.nonzero()[0])
        raise ValueError(f"block_table[{r}, {c}] = {int(bt[r, c])} is outside [0, {num_pages})")


def paged_decode(q: torch.Tensor, k_pages: torch.Tensor, v_pages: torch.Tensor, block_table: torch.Tensor,
                 ctx_lens: torch.Tensor, *, scale: Optional[float] = None, softcap: Optional[float] = None,
                 return_lse: bool = False, chunks_per_split: Optional[int] = None, max_ctx: Optional[int] = None):
    """Decode attention for R requests.

    q [R, Hq, D]; k_pages/v_pages [P, Hkv, page_size, D] (contiguous);
    block_table [R, max_pages] int32; ctx_lens [R] int32 (device tensors).
    Returns o [R, Hq, D] (q's dtype) and, if requested, lse [R, Hq] fp32.
    """
    _lib.require_cuda(q, k_pages, v_pages, block_table, ctx_lens)
    R, Hq, D = q.shape
    P, Hkv, page_size, Dk = k_pages.shape
    if Dk != D or v_pages.shape != k_pages.shape:
        raise ValueError("q / page pool head dims disagree")
    if q.dtype not in _lib.DTYPE_CODE or k_pages.dtype != q.dtype:
        raise ValueError("paged_decode needs fp16/bf16 q and pages of the same dtype")
    if not (k_pages.is_contiguous() and v_pages.is_contiguous()):
        raise ValueError("page pools must be contiguous")
    bt = block_table.to(torch.int32).contiguous()
    lens = ctx_lens.to(torch.int32).contiguous()
    if q.stride(-1) != 1:
        q = q.contiguous()
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    max_pages = bt.shape[1]
    if chunks_per_split is None:
        ctx_max = max_ctx if max_ctx is not None else max_pages * page_size
        sms = torch.cuda.get_device_properties(q.device).multi_processor_count
        chunks_per_split = default_chunks_per_split(ctx_max, R, Hkv, sms)
    out = torch.empty((R, Hq, D), dtype=q.dtype, device=q.device)
    lse = torch.empty((R, Hq), dtype=torch.float32, device=q.device) if return_lse else None
    lib = _lib.load()
    ws_bytes = lib.ffa_paged_decode_workspace_size(R, Hq, D, max_pages, page_size, chunks_per_split)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    with torch.cuda.device(q.device):
        st = lib.ffa_paged_decode(
            q.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(), bt.data_ptr(), lens.data_ptr(), out.data_ptr(),
            lse.data_ptr() if lse is not None else None, _lib.DTYPE_CODE[q.dtype], R, Hq, Hkv, D, P, page_size,
            max_pages, _lib.i64arr(q.stride(0), q.stride(1)), _lib.i64arr(out.stride(0), out.stride(1)),
            float(scale), float(softcap or 0.0), int(chunks_per_split), ws.data_ptr(), ws_bytes,
            _lib.err_word(q.device).data_ptr(), _lib.stream_of(q))
    _lib.check(st, "ffa_paged_decode")
    if _lib.sync_check_enabled():
        _lib.check_device_errors(q.device)
    return (out, lse) if return_lse else out
