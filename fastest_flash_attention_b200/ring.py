"""Sequence-sharded ("ring") attention across the GPUs of one node: forward,
backward and an autograd function.

The reference has no multi-GPU path; for contexts too long for one GPU the
sequence is split into shards, one per rank: contiguous (rank r holds
positions [r S, (r+1) S)) or zigzag (2 W chunks, rank r holds chunks r and
2 W-1-r, which gives every rank the same work under causal masking).  Each
rank attends its queries to
every rank's K/V block in W steps: the block in hand is sent on to rank r+1
while the local partial attention runs (NCCL point-to-point on its own
stream, so the transfer overlaps the kernel), and partial results are folded
into a running (O, LSE) by log-sum-exp (``ffa_merge_partial``).

Causal masking uses the forward kernel's bottom-right alignment: a key
piece starting at absolute position k0 is attended by a query piece starting
at q0 with ``q_offset = q0 - k0``, which makes every earlier key visible,
masks the diagonal causally and applies a sliding window across piece edges.
Pairs no query can see (later keys under causal masking, or keys entirely
left of the window) are skipped.

Backward: the backward kernel run on one (query piece, key piece) pair with
the pieces' final O and LSE from the forward gives that pair's exact share of
dQ, dK and dV (P = exp(S - LSE) is the global probability, Delta = rowsum(dO O)
the global one).  dQ is summed locally; the dK / dV sums travel around the ring
with their K / V block, gaining each rank's share, and take one last hop home.
Every sum is taken in a fixed order, in fp32, so results are deterministic.
"""
from __future__ import annotations

import math
from typing import Callable, List, Optional, Tuple

import torch

from . import _lib

AttnFn = Callable[..., Tuple[torch.Tensor, torch.Tensor]]
BwdFn = Callable[..., Tuple[torch.Tensor, torch.Tensor, torch.Tensor]]


def piece_starts(rank: int, world: int, S: int, layout: str) -> List[Tuple[int, int]]:
    """(absolute start, length) of the pieces that make up rank ``rank``'s
    shard of S positions, in the order they are concatenated.
    contiguous: one piece [rank S, rank S + S).  zigzag: the sequence is cut
    into 2 world chunks of S / 2 and rank r holds chunks r and 2 world-1-r, so
    that every rank does the same causal work."""
    if layout == "contiguous":
        return [(rank * S, S)]
    if layout == "zigzag":
        if S % 2:
            raise ValueError("zigzag shards need an even number of positions per rank")
        C = S // 2
        return [(rank * C, C), ((2 * world - 1 - rank) * C, C)]
    raise ValueError(f"unknown layout {layout!r}")


def zigzag_shard(x: torch.Tensor, rank: int, world: int, dim: int = 2) -> torch.Tensor:
    """This rank's zigzag shard of a full-sequence tensor (chunks r and 2W-1-r)."""
    c = x.shape[dim] // (2 * world)
    a = x.narrow(dim, rank * c, c)
    b = x.narrow(dim, (2 * world - 1 - rank) * c, c)
    return torch.cat([a, b], dim=dim)


def zigzag_unshard(shards: List[torch.Tensor], dim: int = 2) -> torch.Tensor:
    """Inverse of zigzag_shard over the shards of all ranks (in rank order)."""
    W = len(shards)
    halves = [s.chunk(2, dim=dim) for s in shards]
    return torch.cat([halves[r][0] for r in range(W)] + [halves[r][1] for r in reversed(range(W))], dim=dim)


def _pair_visible(q0: int, lq: int, k0: int, lk: int, causal: bool, window: Optional[int]) -> bool:
    """Whether any query at [q0, q0 + lq) sees any key at [k0, k0 + lk)."""
    if causal and k0 > q0 + lq - 1:
        return False
    if window and k0 + lk - 1 < q0 - window + 1:
        return False
    return True


def _kernel_attn(q, k, v, *, scale, causal, q_offset, window, softcap):
    from .attention import flash_fwd
    # the ring's partial merge takes 16-bit partials: fp32 pieces run on the tensor cores in bf16
    return flash_fwd(q, k, v, scale=scale, causal=causal, q_offset=q_offset, window=window, softcap=softcap,
                     compute_dtype=torch.bfloat16 if q.dtype == torch.float32 else None)


def merge_partial(o_acc: torch.Tensor, lse_acc: torch.Tensor, o_part: torch.Tensor, lse_part: torch.Tensor) -> None:
    """In place: fold (o_part, lse_part) into the running (o_acc fp32, lse_acc fp32)."""
    if o_acc.is_cuda:
        _lib.require_cuda(o_acc, lse_acc, o_part, lse_part)
        op = o_part.contiguous()
        lp = lse_part.to(torch.float32).contiguous()
        rows = lse_acc.numel()
        lib = _lib.load()
        with torch.cuda.device(o_acc.device):
            st = lib.ffa_merge_partial(o_acc.data_ptr(), lse_acc.data_ptr(), op.data_ptr(), lp.data_ptr(),
                                       _lib.DTYPE_CODE[op.dtype], rows, o_acc.shape[-1], _lib.stream_of(o_acc))
        _lib.check(st, "ffa_merge_partial")
        return
    # host ranks (tests on CPU): the same arithmetic in torch
    lp = lse_part.float()
    m = torch.maximum(lse_acc, lp)
    m = torch.where(torch.isinf(m) & (m < 0), torch.zeros_like(m), m)
    wa = torch.exp(lse_acc - m)
    wp = torch.exp(lp - m)
    tot = wa + wp
    keep = tot > 0
    o_new = (o_acc * wa[..., None] + o_part.float() * wp[..., None]) / torch.where(keep, tot, 1.0)[..., None]
    o_acc.copy_(torch.where(keep[..., None], o_new, o_acc))
    lse_acc.copy_(torch.where(keep, m + torch.log(torch.where(keep, tot, 1.0)), lse_acc))


class _Acc:
    """Running (O fp32, LSE fp32) of one query piece."""

    def __init__(self, q: torch.Tensor, dv: int):
        B, H, L, _ = q.shape
        self.o = torch.zeros((B, H, L, dv), dtype=torch.float32, device=q.device)
        self.lse = torch.full((B, H, L), float("-inf"), dtype=torch.float32, device=q.device)


def _attend_block(q_pieces, accs, k, v, kv_pieces, *, attn, scale, causal, window, softcap):
    """Fold one rank's K/V block (pieces at their absolute positions) into the
    running results of this rank's query pieces."""
    off = 0
    for k0, lk in kv_pieces:
        kp, vp = k[:, :, off:off + lk], v[:, :, off:off + lk]
        off += lk
        for (qp, q0), acc in zip(q_pieces, accs):
            if not _pair_visible(q0, qp.shape[2], k0, lk, causal, window):
                continue
            o_p, lse_p = attn(qp, kp, vp, scale=scale, causal=causal, q_offset=q0 - k0, window=window,
                              softcap=softcap)
            merge_partial(acc.o, acc.lse, o_p, lse_p)


def _split_q(q: torch.Tensor, pieces):
    out, off = [], 0
    for q0, l in pieces:
        out.append((q[:, :, off:off + l].contiguous() if len(pieces) > 1 else q, q0))
        off += l
    return out


def ring_attention_local(q: torch.Tensor, kv_blocks: List[Tuple[torch.Tensor, torch.Tensor]], rank: int, *,
                         scale: Optional[float] = None, causal: bool = False, sliding_window: Optional[int] = None,
                         softcap: Optional[float] = None, attn_fn: Optional[AttnFn] = None,
                         layout: str = "contiguous") -> Tuple[torch.Tensor, torch.Tensor]:
    """The ring's arithmetic on one device, with every rank's K/V shard given
    (in rank order, each laid out as ``layout``): rank ``rank``'s output over
    the full sequence.  Used to test the ring's arithmetic on one GPU."""
    W = len(kv_blocks)
    S = q.shape[2]
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    attn = attn_fn or _kernel_attn
    q_pieces = _split_q(q, piece_starts(rank, W, S, layout))
    accs = [_Acc(qp, kv_blocks[0][1].shape[-1]) for qp, _ in q_pieces]
    for step in range(W):
        s = (rank - step) % W
        k, v = kv_blocks[s]
        _attend_block(q_pieces, accs, k, v, piece_starts(s, W, S, layout), attn=attn, scale=scale, causal=causal,
                      window=sliding_window, softcap=softcap)
    return torch.cat([a.o for a in accs], dim=2), torch.cat([a.lse for a in accs], dim=2)


def ring_attention_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, group=None,
                           scale: Optional[float] = None, causal: bool = False,
                           sliding_window: Optional[int] = None, softcap: Optional[float] = None,
                           attn_fn: Optional[AttnFn] = None, return_lse: bool = False,
                           layout: str = "contiguous"):
    """Attention of this rank's query shard over the whole sequence.

    q [B, Hq, S, D], k [B, Hkv, S, D], v [B, Hkv, S, Dv]: this rank's shard
    (every rank holds the same S), laid out as ``layout`` ("contiguous", or
    "zigzag" for balanced causal work; see ``piece_starts`` / ``zigzag_shard``).
    Returns O [B, Hq, S, Dv] in q's dtype, in the same layout (and, with
    return_lse, LSE [B, Hq, S] fp32, natural log).  K/V shards travel
    rank -> rank + 1 around the ring by point-to-point sends issued before
    each step's attention, so the transfer of the next shard overlaps the
    current one's kernels.
    """
    import torch.distributed as dist
    W = dist.get_world_size(group)
    r = dist.get_rank(group)
    S = q.shape[2]
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    attn = attn_fn or _kernel_attn
    nxt = dist.get_global_rank(group, (r + 1) % W) if group is not None else (r + 1) % W
    prv = dist.get_global_rank(group, (r - 1) % W) if group is not None else (r - 1) % W
    q_pieces = _split_q(q, piece_starts(r, W, S, layout))
    accs = [_Acc(qp, v.shape[-1]) for qp, _ in q_pieces]
    # The caller's K / V are only sent; blocks arriving from other ranks land
    # in two buffers of our own, used in turn.
    cur = (k.contiguous(), v.contiguous())
    bufs = [(torch.empty_like(cur[0]), torch.empty_like(cur[1])) for _ in range(2 if W > 2 else 1)]
    for step in range(W):
        s = (r - step) % W
        works = []
        if step < W - 1:
            spare = bufs[step % len(bufs)]
            ops = [dist.P2POp(dist.isend, cur[0], nxt, group), dist.P2POp(dist.irecv, spare[0], prv, group),
                   dist.P2POp(dist.isend, cur[1], nxt, group), dist.P2POp(dist.irecv, spare[1], prv, group)]
            works = dist.batch_isend_irecv(ops)
        _attend_block(q_pieces, accs, cur[0], cur[1], piece_starts(s, W, S, layout), attn=attn, scale=scale,
                      causal=causal, window=sliding_window, softcap=softcap)
        for w in works:
            w.wait()
        if step < W - 1:
            cur = spare
    o_acc = torch.cat([a.o for a in accs], dim=2)
    lse_acc = torch.cat([a.lse for a in accs], dim=2)
    o = o_acc.to(q.dtype) if q.dtype in (torch.bfloat16, torch.float16) else o_acc
    return (o, lse_acc) if return_lse else o


def _kernel_bwd(dout, q, k, v, o, lse, *, scale, causal, q_offset, window, softcap):
    from .attention import flash_bwd
    return flash_bwd(dout, q, k, v, o, lse, scale=scale, causal=causal, q_offset=q_offset, window=window,
                     softcap=softcap, compute_dtype=torch.bfloat16 if q.dtype == torch.float32 else None)


def _split_seq(x: torch.Tensor, pieces) -> List[torch.Tensor]:
    """x [B, H, S(, ...)] cut along dim 2 into the layout's pieces."""
    out, off = [], 0
    for _, l in pieces:
        out.append(x[:, :, off:off + l].contiguous() if len(pieces) > 1 else x)
        off += l
    return out


def _bwd_block(q_pieces, do_pieces, o_pieces, lse_pieces, dq_accs, k, v, dk_acc, dv_acc, kv_pieces, *, bwd,
               scale, causal, window, softcap):
    """Add every visible (query piece, key piece) pair's gradient shares:
    dQ into dq_accs, dK / dV into the travelling block sums dk_acc / dv_acc."""
    off = 0
    for k0, lk in kv_pieces:
        kp, vp = k[:, :, off:off + lk], v[:, :, off:off + lk]
        for i, (qp, q0) in enumerate(q_pieces):
            if not _pair_visible(q0, qp.shape[2], k0, lk, causal, window):
                continue
            dq, dk, dv = bwd(do_pieces[i], qp, kp, vp, o_pieces[i], lse_pieces[i], scale=scale, causal=causal,
                             q_offset=q0 - k0, window=window, softcap=softcap)
            dq_accs[i] += dq.float()
            dk_acc[:, :, off:off + lk] += dk.float()
            dv_acc[:, :, off:off + lk] += dv.float()
        off += lk


def ring_attention_backward(dout: torch.Tensor, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                            o: torch.Tensor, lse: torch.Tensor, *, group=None, scale: Optional[float] = None,
                            causal: bool = False, sliding_window: Optional[int] = None,
                            softcap: Optional[float] = None, bwd_fn: Optional[BwdFn] = None,
                            layout: str = "contiguous"):
    """Gradients of ring_attention_forward for this rank's shards.

    dout, q, o [B, Hq, S, *], k [B, Hkv, S, D], v [B, Hkv, S, Dv] and lse
    [B, Hq, S] (fp32, natural log, as ring_attention_forward returns it):
    this rank's shards in ``layout``.  Returns (dq, dk, dv) in the inputs'
    dtypes and layout.  Each step sends the next K / V block on while the
    current one's pairs are computed; the dK / dV sums follow once they hold
    this rank's share.
    """
    import torch.distributed as dist
    W = dist.get_world_size(group)
    r = dist.get_rank(group)
    S = q.shape[2]
    scale = scale if scale is not None else 1.0 / math.sqrt(q.shape[-1])
    bwd = bwd_fn or _kernel_bwd
    nxt = dist.get_global_rank(group, (r + 1) % W) if group is not None else (r + 1) % W
    prv = dist.get_global_rank(group, (r - 1) % W) if group is not None else (r - 1) % W
    pieces = piece_starts(r, W, S, layout)
    q_pieces = _split_q(q, pieces)
    do_pieces = _split_seq(dout, pieces)
    o_pieces = _split_seq(o, pieces)
    lse_pieces = [x.float() for x in _split_seq(lse if lse.dim() == 3 else lse[..., 0], pieces)]
    dq_accs = [torch.zeros(qp.shape, dtype=torch.float32, device=q.device) for qp, _ in q_pieces]
    # as in the forward, the caller's K / V are only sent
    cur = (k.contiguous(), v.contiguous())
    bufs = [(torch.empty_like(cur[0]), torch.empty_like(cur[1])) for _ in range(2 if W > 2 else 1)]
    acc = (torch.zeros(k.shape, dtype=torch.float32, device=k.device),
           torch.zeros(v.shape, dtype=torch.float32, device=v.device))
    acc_in = (torch.empty_like(acc[0]), torch.empty_like(acc[1]))

    def exchange(send, recv):
        ops = []
        for a, b in zip(send, recv):
            ops += [dist.P2POp(dist.isend, a, nxt, group), dist.P2POp(dist.irecv, b, prv, group)]
        for w in dist.batch_isend_irecv(ops):
            w.wait()

    for step in range(W):
        s = (r - step) % W
        works = []
        if step < W - 1:
            spare = bufs[step % len(bufs)]
            ops = []
            for a, b in zip(cur, spare):
                ops += [dist.P2POp(dist.isend, a, nxt, group), dist.P2POp(dist.irecv, b, prv, group)]
            works = dist.batch_isend_irecv(ops)
        _bwd_block(q_pieces, do_pieces, o_pieces, lse_pieces, dq_accs, cur[0], cur[1], acc[0], acc[1],
                   piece_starts(s, W, S, layout), bwd=bwd, scale=scale, causal=causal, window=sliding_window,
                   softcap=softcap)
        for w in works:
            w.wait()
        # block s's sums (now holding this rank's share) go where block s goes;
        # after the last step they are complete and go to block s's owner, r + 1
        exchange(acc, acc_in)
        acc, acc_in = acc_in, acc
        if step < W - 1:
            cur = spare
    dq = torch.cat(dq_accs, dim=2) if len(dq_accs) > 1 else dq_accs[0]
    return dq.to(q.dtype), acc[0].to(k.dtype), acc[1].to(v.dtype)


def ring_attention_local_backward(douts, qs, kvs, os_, lses, *, scale: Optional[float] = None,
                                  causal: bool = False, sliding_window: Optional[int] = None,
                                  softcap: Optional[float] = None, bwd_fn: Optional[BwdFn] = None,
                                  layout: str = "contiguous"):
    """The ring backward's arithmetic on one device, with every rank's shards
    given (lists in rank order; kvs of (k, v) pairs): (dqs, dks, dvs) per rank.
    Block sums are taken in the order the distributed ring takes them (rank
    s's block gains rank s's share first, then s+1's, ...).  Used to test the
    ring's arithmetic on one GPU."""
    W = len(qs)
    S = qs[0].shape[2]
    scale = scale if scale is not None else 1.0 / math.sqrt(qs[0].shape[-1])
    bwd = bwd_fn or _kernel_bwd
    per_rank = []
    for r in range(W):
        pieces = piece_starts(r, W, S, layout)
        lse = lses[r] if lses[r].dim() == 3 else lses[r][..., 0]
        per_rank.append((_split_q(qs[r], pieces), _split_seq(douts[r], pieces), _split_seq(os_[r], pieces),
                         [x.float() for x in _split_seq(lse, pieces)]))
    dq_accs = [[torch.zeros(qp.shape, dtype=torch.float32, device=qp.device) for qp, _ in pr[0]] for pr in per_rank]
    dks, dvs = [], []
    for s in range(W):
        k, v = kvs[s]
        dk = torch.zeros(k.shape, dtype=torch.float32, device=k.device)
        dv = torch.zeros(v.shape, dtype=torch.float32, device=v.device)
        for t in range(W):
            r = (s + t) % W
            qp, dop, op, lp = per_rank[r]
            _bwd_block(qp, dop, op, lp, dq_accs[r], k, v, dk, dv, piece_starts(s, W, S, layout), bwd=bwd,
                       scale=scale, causal=causal, window=sliding_window, softcap=softcap)
        dks.append(dk.to(k.dtype))
        dvs.append(dv.to(v.dtype))
    dqs = [(torch.cat(a, dim=2) if len(a) > 1 else a[0]).to(qs[r].dtype) for r, a in enumerate(dq_accs)]
    return dqs, dks, dvs


class RingAttnFunc(torch.autograd.Function):
    """Autograd over ring_attention_forward / ring_attention_backward."""

    @staticmethod
    def forward(ctx, q, k, v, group, scale, causal, sliding_window, softcap, layout):
        o, lse = ring_attention_forward(q, k, v, group=group, scale=scale, causal=causal,
                                        sliding_window=sliding_window, softcap=softcap, return_lse=True,
                                        layout=layout)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.args = (group, scale, causal, sliding_window, softcap, layout)
        return o

    @staticmethod
    def backward(ctx, dout):
        q, k, v, o, lse = ctx.saved_tensors
        group, scale, causal, sliding_window, softcap, layout = ctx.args
        dq, dk, dv = ring_attention_backward(dout.contiguous(), q, k, v, o, lse, group=group, scale=scale,
                                             causal=causal, sliding_window=sliding_window, softcap=softcap,
                                             layout=layout)
        return dq, dk, dv, None, None, None, None, None, None


def ring_attention_func(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, group=None,
                        scale: Optional[float] = None, causal: bool = False, sliding_window: Optional[int] = None,
                        softcap: Optional[float] = None, layout: str = "contiguous") -> torch.Tensor:
    """Differentiable ring attention of this rank's shards (sm_100a kernels)."""
    return RingAttnFunc.apply(q, k, v, group, scale, causal, sliding_window, softcap, layout)
