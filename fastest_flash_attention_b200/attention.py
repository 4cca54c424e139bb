"""Forward / backward / autograd API — drop-in for the reference's ops layer.

Mirrors ops/attention_forward.py:23-167, ops/attention_backward.py:19-76 and
ops/attention_func.py:20-125: same names, arguments, shapes and return
values.  The work is done by the sm_100a kernels in libffa_b200.so; there is
no Triton path and no CPU fallback (CPU tensors raise).

Numerics: fp16/bf16 inputs are consumed as-is by the tensor cores with fp32
accumulation.  fp32 inputs are computed in fp32, as the reference does
(kernels/cpu_reference.py:28-32 casts only when a lower ``compute_dtype`` is
given): the fp32 kernels run on the CUDA cores, since the tensor cores take no
fp32 operands.  With ``compute_dtype`` fp16/bf16, fp32 inputs are rounded to
it and run on the tensor cores, and the result is cast back to fp32.
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import torch
from torch.autograd import Function

from . import _lib
from .config import AttentionConfig
from .utils import auto_select_block_size, maybe_unsqueeze_head

_KERNEL_DTYPES = (torch.float16, torch.bfloat16)
# dtype codes of ffa_fwd / ffa_bwd (FFA_DTYPE_*): fp32 selects the CUDA-core kernels
_ATTN_DTYPE_CODE = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}
FWD_HEAD_DIMS = ((64, 64), (128, 128), (192, 128))  # kernel instantiations (qk, v)
MAX_HEAD_DIM = 192  # qk head dim; v head dim up to 128


def kernel_head_dims(D: int, Dv: int) -> Optional[Tuple[int, int]]:
    """Smallest kernel instantiation (qk, v) that holds head dims (D, Dv), or
    None.  Other head dims (the reference computes any D) run on a kernel
    whose tile is wider: q/k (and v) are zero-padded in the head dim, which
    leaves every dot product, the softmax and the kept output columns
    unchanged; the caller's scale (default 1/sqrt(D) of the true D) is passed
    through unchanged."""
    for kd, kv in FWD_HEAD_DIMS:
        if D <= kd and Dv <= kv:
            return kd, kv
    return None


def _pad_last(t: torch.Tensor, width: int) -> torch.Tensor:
    if t.shape[-1] == width:
        return t
    return torch.nn.functional.pad(t, (0, width - t.shape[-1]))


def kernel_dtype(t: torch.Tensor, compute_dtype: Optional[torch.dtype] = None) -> torch.dtype:
    """Dtype the kernels compute in: 16-bit inputs as they are; fp32 (and
    fp64) inputs in fp32 unless ``compute_dtype`` asks for fp16/bf16 (tensor
    cores); other input dtypes in bf16."""
    if t.dtype in _KERNEL_DTYPES:
        return t.dtype
    if compute_dtype in _KERNEL_DTYPES:
        return compute_dtype
    if t.dtype in (torch.float32, torch.float64):
        return torch.float32
    return torch.bfloat16


def _tma_ready(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Cast to the kernel dtype and make the layout TMA-addressable
    (unit stride in D, 16-byte aligned base and outer strides)."""
    if t.dtype != dtype:
        t = t.to(dtype)
    if (t.stride(-1) != 1 or any(s % 8 for s in t.stride()[:-1]) or t.data_ptr() % 16
            or any(s == 0 for s in t.stride()[:-1])):
        t = t.contiguous()
    return t


def _strides_bhs(t: torch.Tensor):
    return _lib.i64arr(t.stride(0), t.stride(1), t.stride(2))


def flash_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, scale: float, causal: bool = False,
              q_offset: int = 0, window: Optional[int] = None, softcap: Optional[float] = None,
              block_mask: Optional[torch.Tensor] = None, mask_block: Tuple[int, int] = (64, 64),
              compute_dtype: Optional[torch.dtype] = None, want_lse: bool = True
              ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Run the sm_100a forward kernel on 4-D [B, H, S, D] tensors.

    Returns (O in the kernel dtype with q's stride order, LSE [B, Hq, Sq] fp32).
    """
    _lib.require_cuda(q, k, v)
    B, Hq, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    Dv = v.shape[3]
    if k.shape[0] != B or v.shape[:3] != k.shape[:3] or k.shape[3] != D:
        raise ValueError(f"incompatible q/k/v shapes {tuple(q.shape)} {tuple(k.shape)} {tuple(v.shape)}")
    if Hq % Hkv != 0:
        raise ValueError(f"query heads ({Hq}) must be a multiple of key/value heads ({Hkv})")
    kdims = kernel_head_dims(D, Dv)
    if kdims is None:
        raise ValueError(f"head dims (qk={D}, v={Dv}) not supported by the sm_100a forward kernel "
                         f"(supported: qk <= {MAX_HEAD_DIM}, v <= 128)")
    dt = kernel_dtype(q, compute_dtype)
    if kdims != (D, Dv):
        o, lse = flash_fwd(_pad_last(q.to(dt), kdims[0]), _pad_last(k.to(dt), kdims[0]),
                           _pad_last(v.to(dt), kdims[1]), scale=scale, causal=causal, q_offset=q_offset,
                           window=window, softcap=softcap, block_mask=block_mask, mask_block=mask_block,
                           compute_dtype=compute_dtype, want_lse=want_lse)
        return o[..., :Dv], lse
    q = _tma_ready(q, dt)
    k = _tma_ready(k, dt)
    v = _tma_ready(v, dt)
    if Dv == D:
        o = torch.empty_like(q)  # keeps q's stride order when q is dense
    else:
        o = torch.empty((B, Sq, Hq, Dv), dtype=dt, device=q.device).transpose(1, 2)
    lse = torch.empty((B, Hq, Sq), dtype=torch.float32, device=q.device) if want_lse else None
    bm_ptr, n_br, n_bc = None, 0, 0
    if block_mask is not None:
        bm = block_mask.to(device=q.device, dtype=torch.uint8).contiguous()
        n_br, n_bc = bm.shape
        bm_ptr = bm.data_ptr()
    lib = _lib.load()
    with torch.cuda.device(q.device):
        st = lib.ffa_fwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr() if lse is not None else None,
            _ATTN_DTYPE_CODE[dt], B, Hq, Hkv, Sq, Skv, D, Dv,
            _strides_bhs(q), _strides_bhs(k), _strides_bhs(v), _strides_bhs(o),
            float(scale), int(bool(causal)), int(q_offset), int(window or 0), float(softcap or 0.0),
            bm_ptr, n_br, n_bc, int(mask_block[0]), int(mask_block[1]),
            _lib.err_word(q.device).data_ptr(), _lib.stream_of(q))
    _lib.check(st, "ffa_fwd")
    if block_mask is not None:
        bm.record_stream(torch.cuda.current_stream(q.device))
    if _lib.sync_check_enabled():
        _lib.check_device_errors(q.device)
    return o, lse


def fastest_flash_attn_forward(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    config: Optional[AttentionConfig] = None,
    *,
    scale: Optional[float] = None,
    causal: bool = False,
    block_size: Optional[int] = None,
    block_mask: Optional[torch.Tensor] = None,
    softcap: Optional[float] = None,
    sliding_window: Optional[int] = None,
    two_pass: bool = False,
    compute_dtype: Optional[torch.dtype] = None,
    num_kv_heads: Optional[int] = None,
    kv_cache: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
    return_lse: bool = False,
) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
    """Forward attention (ops/attention_forward.py:23-167).

    q [B,S_q,D] or [B,H_q,S_q,D]; k/v [B,S_kv,D] or [B,H_kv,S_kv,D].
    Returns (output shaped like q, LSE [B,H,S_q,1] fp32 natural log or None).
    GQA/MQA (H_q a multiple of H_kv) is handled natively without repeating
    K/V; ``num_kv_heads`` is accepted for compatibility.  ``two_pass`` needs
    no second pass here: the kernel's LSE is already exact.
    """
    if config is not None:  # attention_forward.py:66-73
        causal = config.causal
        softcap = config.softcap
        sliding_window = config.sliding_window
        two_pass = config.two_pass
        compute_dtype = config.compute_dtype
        num_kv_heads = config.num_kv_heads
        return_lse = config.return_lse

    in_dtype = q.dtype
    q, k, v, squeezed = maybe_unsqueeze_head(q, k, v)
    B, H_q, S_q, D = q.shape

    q_offset = 0
    if kv_cache is not None:  # attention_forward.py:80-89: cache is prepended, queries sit at the end
        k_cache, v_cache = kv_cache
        if k_cache.dim() == 3:
            k_cache = k_cache.unsqueeze(1)
            v_cache = v_cache.unsqueeze(1)
        k = torch.cat([k_cache.to(k.dtype), k], dim=2)
        v = torch.cat([v_cache.to(v.dtype), v], dim=2)
        q_offset = k.size(2) - S_q
    S_kv = k.size(2)

    if scale is None:
        scale = 1.0 / math.sqrt(D)

    if block_size is None:
        if config is not None:
            bq, bkv = config.resolve_block_sizes(S_q, S_kv, D)
        else:
            bq = bkv = auto_select_block_size(S_q, S_kv, D)
    else:
        bq = bkv = block_size

    o, lse = flash_fwd(q, k, v, scale=scale, causal=causal, q_offset=q_offset, window=sliding_window,
                       softcap=softcap, block_mask=block_mask, mask_block=(bq, bkv),
                       compute_dtype=compute_dtype, want_lse=return_lse)
    if o.dtype != in_dtype:
        o = o.to(in_dtype)
    if lse is not None:
        lse = lse.unsqueeze(-1)
    if squeezed:
        o = o.squeeze(1)
        if lse is not None:
            lse = lse.squeeze(1)
    return o, lse


def flash_bwd(dout: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o: torch.Tensor,
              lse: torch.Tensor, *, scale: float, causal: bool = False, q_offset: int = 0,
              window: Optional[int] = None, softcap: Optional[float] = None,
              block_mask: Optional[torch.Tensor] = None, mask_block: Tuple[int, int] = (64, 64),
              compute_dtype: Optional[torch.dtype] = None) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Run the deterministic sm_100a backward on 4-D tensors.

    lse: [B, Hq, Sq] (or [B, Hq, Sq, 1]) natural-log LSE from the forward.
    block_mask / mask_block: the tile mask the forward was given (masked
    pairs contribute nothing to any gradient).
    Returns (dq, dk, dv) in the kernel dtype; dk/dv have k's head count
    (GQA groups are summed inside the kernel).
    """
    _lib.require_cuda(dout, q, k, v, o, lse)
    B, Hq, Sq, D = q.shape
    Hkv, Skv = k.shape[1], k.shape[2]
    Dv = v.shape[3]
    kdims = kernel_head_dims(D, Dv)
    if kdims is None or o.shape[3] != Dv or dout.shape[3] != Dv:
        raise ValueError(f"head dims (qk={D}, v={Dv}) not supported by the sm_100a backward kernel "
                         f"(supported: qk <= {MAX_HEAD_DIM}, v <= 128)")
    if Hq % Hkv != 0:
        raise ValueError(f"query heads ({Hq}) must be a multiple of key/value heads ({Hkv})")
    dt = kernel_dtype(q, compute_dtype)
    if kdims != (D, Dv):
        # zero columns: Delta, dP and the kept gradient columns are unchanged
        kd, kv = kdims
        dq, dk, dv = flash_bwd(_pad_last(dout.to(dt), kv), _pad_last(q.to(dt), kd), _pad_last(k.to(dt), kd),
                               _pad_last(v.to(dt), kv), _pad_last(o.to(dt), kv), lse, scale=scale, causal=causal,
                               q_offset=q_offset, window=window, softcap=softcap, block_mask=block_mask,
                               mask_block=mask_block, compute_dtype=compute_dtype)
        return dq[..., :D], dk[..., :D], dv[..., :Dv]
    q, k, v, o, dout = (_tma_ready(t, dt) for t in (q, k, v, o, dout))
    if lse.dim() == 4:
        lse = lse[..., 0]
    lse = lse.to(torch.float32).contiguous()
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    lib = _lib.load()
    ws_bytes = lib.ffa_bwd_workspace_size(B, Hq, Sq)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    common = (dout.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), lse.data_ptr(),
              dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), _ATTN_DTYPE_CODE[dt], B, Hq, Hkv, Sq, Skv, D, v.shape[3],
              _strides_bhs(q), _strides_bhs(k), _strides_bhs(v), _strides_bhs(o), _strides_bhs(dout),
              _strides_bhs(dq), _strides_bhs(dk), _strides_bhs(dv),
              float(scale), int(bool(causal)), int(q_offset), int(window or 0), float(softcap or 0.0))
    tail = (ws.data_ptr(), ws_bytes, _lib.err_word(q.device).data_ptr(), _lib.stream_of(q))
    with torch.cuda.device(q.device):
        if block_mask is None:
            st = lib.ffa_bwd(*common, *tail)
        else:
            bm = block_mask.to(device=q.device, dtype=torch.uint8).contiguous()
            st = lib.ffa_bwd_masked(*common, bm.data_ptr(), bm.shape[0], bm.shape[1], int(mask_block[0]),
                                    int(mask_block[1]), *tail)
            bm.record_stream(torch.cuda.current_stream(q.device))
    _lib.check(st, "ffa_bwd")
    if _lib.sync_check_enabled():
        _lib.check_device_errors(q.device)
    return dq, dk, dv


def fastest_flash_attn_backward(
    grad_output: torch.Tensor,
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    output: torch.Tensor,
    lse: torch.Tensor,
    *,
    scale: Optional[float] = None,
    causal: bool = False,
    block_size: int = 64,
    softcap: Optional[float] = None,
    sliding_window: Optional[int] = None,
    q_offset: int = 0,
    block_mask: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Backward (ops/attention_backward.py:19-76): (dq, dk, dv) from the
    forward's output and LSE, recomputing the attention tile by tile.

    ``block_size`` sets the granularity of ``block_mask`` (as in the forward);
    the kernel's own tiles are fixed.  ``block_mask`` goes beyond the
    reference, whose backward ignores it: given the forward's mask, the
    gradients are those of the masked forward.  Gradients come back in the
    dtypes of q, k and v.
    """
    bs = block_size if block_size is not None else auto_select_block_size(q.shape[-2], k.shape[-2], q.shape[-1])
    dq, dk, dv = flash_bwd(grad_output, q, k, v, output, lse, scale=scale if scale is not None else
                           1.0 / math.sqrt(q.shape[-1]), causal=causal, q_offset=q_offset, window=sliding_window,
                           softcap=softcap, block_mask=block_mask, mask_block=(bs, bs))
    return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype)


class FastestFlashAttnFunc(Function):
    """Autograd function (ops/attention_func.py:20-90): saves q, k, v, output
    and LSE; the backward recomputes attention with the sm_100a kernels.
    Accepts GQA (fewer K/V heads than query heads) natively."""

    @staticmethod
    def forward(ctx, q, k, v, scale, causal, block_size, softcap, sliding_window, two_pass, block_mask=None):
        output, lse = fastest_flash_attn_forward(
            q, k, v, scale=scale, causal=causal, block_size=block_size, softcap=softcap,
            sliding_window=sliding_window, two_pass=two_pass, block_mask=block_mask, return_lse=True)
        ctx.save_for_backward(q, k, v, output, lse)
        ctx.block_mask = block_mask
        ctx.scale = scale
        ctx.causal = causal
        ctx.block_size = block_size
        ctx.softcap = softcap
        ctx.sliding_window = sliding_window
        return output

    @staticmethod
    def backward(ctx, grad_output):
        q, k, v, output, lse = ctx.saved_tensors
        was_3d = q.dim() == 3
        if was_3d:
            q, k, v, output, lse, grad_output = (t.unsqueeze(1) for t in (q, k, v, output, lse, grad_output))
        dq, dk, dv = fastest_flash_attn_backward(
            grad_output, q, k, v, output, lse, scale=ctx.scale, causal=ctx.causal, block_size=ctx.block_size,
            softcap=ctx.softcap, sliding_window=ctx.sliding_window, block_mask=ctx.block_mask)
        if was_3d:
            dq, dk, dv = dq.squeeze(1), dk.squeeze(1), dv.squeeze(1)
        return dq, dk, dv, None, None, None, None, None, None, None


def fastest_flash_attn_func(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    scale: Optional[float] = None,
    causal: bool = False,
    block_size: int = 64,
    softcap: Optional[float] = None,
    sliding_window: Optional[int] = None,
    two_pass: bool = False,
    block_mask: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Differentiable attention (ops/attention_func.py:93-125).  The trailing
    ``block_mask`` (tiles of ``block_size``) is an addition: the reference's
    autograd path has no block mask."""
    return FastestFlashAttnFunc.apply(q, k, v, scale, causal, block_size, softcap, sliding_window, two_pass,
                                      block_mask)
