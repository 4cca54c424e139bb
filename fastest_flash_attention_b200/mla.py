"""MLA absorbed-latent decoding for FastestFlashMLA.

The reference's FastestFlashMLA (modules/flash_mla.py:116-172) has no KV
cache: every step up-projects the latent of the whole prefix into per-head
K (128 nope dims + 64 shared rotary dims) and V (128 dims, zero-padded to
192) and runs attention over it.  Here the latent itself is cached, paged,
as [c_kv (latent_dim) | rope(k_rope) (rope_dim)] per token, and the
up-projections are absorbed:

  score_h(t) = q_nope_h . (A_h c_t) + q_rope_h . k_rope_t
             = (A_h^T q_nope_h) . c_t + q_rope_h . k_rope_t       (A_h = W_UK_h)
  out_h      = sum_t p_h(t) (B_h c_t) = B_h (sum_t p_h(t) c_t)     (B_h = W_UV_h)

so one decode step is multi-query attention over the latent cache
(``ffa_mla_decode``) between two small per-head GEMMs.  W_UK_h / W_UV_h are
rows [h*2d, h*2d+d) and [h*2d+d, (h+1)*2d) of kv_up_proj.weight
(flash_mla.py:105-107, 141-143).  The result equals the reference's output
for the last position of the prefix + new tokens (the padded value columns
contribute zeros to o_proj).
"""
from __future__ import annotations

import math
from typing import List, Optional, Sequence

import torch

from . import _lib
from .decode import check_block_table


def mla_chunks_per_split(ctx_max: int, R: int, num_sms: int = 148) -> int:
    """16-token chunks per CTA of the latent decode kernel: whole 128-token
    tiles, and about one CTA per SM (the kernel holds one 147 KB tile in
    shared memory, so one CTA fits an SM)."""
    chunks = max(1, math.ceil(ctx_max / 16))
    splits = max(1, math.ceil(num_sms / max(1, R)))
    return max(8, math.ceil(math.ceil(chunks / splits) / 8) * 8)


def absorbed_weights(mla) -> tuple[torch.Tensor, torch.Tensor]:
    """(W_UK [H, d, latent], W_UV [H, d, latent]) views of kv_up_proj.weight."""
    H, d = mla.num_heads, mla.head_dim
    w = mla.kv_up_proj.weight.view(H, 2 * d, mla.latent_dim)
    return w[:, :d], w[:, d:]


def mla_decode(q: torch.Tensor, ckv_pages: torch.Tensor, block_table: torch.Tensor, ctx_lens: torch.Tensor, *,
               scale: float, return_lse: bool = False, chunks_per_split: Optional[int] = None,
               max_ctx: Optional[int] = None):
    """Latent attention: q [R, H, 576], ckv_pages [P, page_size, 576] -> o_lat [R, H, 512]."""
    _lib.require_cuda(q, ckv_pages, block_table, ctx_lens)
    R, H, DK = q.shape
    P, page_size, DKc = ckv_pages.shape
    if DK != 576 or DKc != 576 or H != 32:
        raise ValueError("the MLA decode kernel serves latent 512 + rope 64 and 32 heads")
    if q.dtype not in _lib.DTYPE_CODE or ckv_pages.dtype != q.dtype or not ckv_pages.is_contiguous():
        raise ValueError("q / latent cache must share an fp16/bf16 dtype; cache contiguous")
    if q.stride(-1) != 1 or q.stride(1) % 8 or q.stride(0) % 8 or q.data_ptr() % 16:
        q = q.contiguous()
    bt = block_table.to(torch.int32).contiguous()
    lens = ctx_lens.to(torch.int32).contiguous()
    max_pages = bt.shape[1]
    if chunks_per_split is None:
        ctx_max = max_ctx if max_ctx is not None else max_pages * page_size
        sms = torch.cuda.get_device_properties(q.device).multi_processor_count
        chunks_per_split = mla_chunks_per_split(ctx_max, R, sms)
    out = torch.empty((R, H, 512), dtype=q.dtype, device=q.device)
    lse = torch.empty((R, H), dtype=torch.float32, device=q.device) if return_lse else None
    lib = _lib.load()
    ws_bytes = lib.ffa_mla_decode_workspace_size(R, H, max_pages, page_size, chunks_per_split)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    with torch.cuda.device(q.device):
        st = lib.ffa_mla_decode(q.data_ptr(), ckv_pages.data_ptr(), bt.data_ptr(), lens.data_ptr(), out.data_ptr(),
                                lse.data_ptr() if lse is not None else None, _lib.DTYPE_CODE[q.dtype], R, H, P,
                                page_size, max_pages, _lib.i64arr(q.stride(0), q.stride(1)),
                                _lib.i64arr(out.stride(0), out.stride(1)), float(scale), int(chunks_per_split),
                                ws.data_ptr(), ws_bytes, _lib.err_word(q.device).data_ptr(), _lib.stream_of(q))
    _lib.check(st, "ffa_mla_decode")
    if _lib.sync_check_enabled():
        _lib.check_device_errors(q.device)
    return (out, lse) if return_lse else out


class MLALatentCache:
    """Paged latent cache [max_pages, page_size, latent + rope] with the same
    FIFO page allocator semantics as PagedKVCache (ops/kv_cache.py:157-168)."""

    def __init__(self, max_pages: int, page_size: int = 64, latent_dim: int = 512, rope_dim: int = 64,
                 dtype: torch.dtype = torch.bfloat16, device="cuda"):
        self.page_size = page_size
        self.latent_dim = latent_dim
        self.rope_dim = rope_dim
        self.pages = torch.zeros(max_pages, page_size, latent_dim + rope_dim, dtype=dtype, device=device)
        self.free_pages: List[int] = list(range(max_pages))
        self.sequences: dict = {}

    def _slots(self, sid: int, n: int) -> List[int]:
        seq = self.sequences.setdefault(sid, {"page_table": [], "len": 0})
        out = []
        for _ in range(n):
            idx, off = divmod(seq["len"], self.page_size)
            while len(seq["page_table"]) <= idx:
                if not self.free_pages:
                    raise RuntimeError("MLALatentCache: out of physical pages")
                seq["page_table"].append(self.free_pages.pop(0))
            out.append(seq["page_table"][idx] * self.page_size + off)
            seq["len"] += 1
        return out

    def append(self, sid: int, entries: torch.Tensor) -> int:
        """entries [n, latent + rope] (rope part already rotated)."""
        slots = torch.tensor(self._slots(sid, entries.shape[0]), dtype=torch.long, device=self.pages.device)
        flat = self.pages.view(-1, self.pages.shape[-1])
        flat[slots] = entries.to(self.pages.dtype)
        return self.sequences[sid]["len"]

    def free_sequence(self, sid: int) -> None:
        if sid in self.sequences:
            self.free_pages.extend(self.sequences.pop(sid)["page_table"])

    def block_table(self, seq_ids: Sequence[int]):
        tables = [self.sequences[s]["page_table"] for s in seq_ids]
        width = max(1, max(len(t) for t in tables))
        bt = torch.zeros(len(seq_ids), width, dtype=torch.int32)
        for i, t in enumerate(tables):
            bt[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
        lens = torch.tensor([self.sequences[s]["len"] for s in seq_ids], dtype=torch.int32)
        check_block_table(bt, lens, self.pages.shape[0], self.page_size)
        return bt.to(self.pages.device), lens.to(self.pages.device)


class MLADecoder:
    """Incremental decoding for a FastestFlashMLA module (no reference counterpart:
    the reference recomputes the full prefix every step)."""

    def __init__(self, mla, max_pages: int, page_size: int = 64, dtype: torch.dtype = torch.bfloat16):
        self.mla = mla
        dev = next(mla.parameters()).device
        self.cache = MLALatentCache(max_pages, page_size, mla.latent_dim, mla.rope_dim, dtype, dev)
        self.dtype = dtype

    def _latent_entries(self, x: torch.Tensor, offset: int) -> torch.Tensor:
        """[S, latent + rope] cache rows for x [S, hidden] at positions offset..offset+S-1."""
        lat = self.mla.kv_down_proj(x)
        kr = self.mla.rope(self.mla.k_rope_proj(x).unsqueeze(0), offset)[0]
        return torch.cat([lat, kr], dim=-1)

    @torch.no_grad()
    def prefill(self, x: torch.Tensor, seq_ids: Sequence[int]) -> torch.Tensor:
        """Run the module on x [B, S, hidden] and cache every position's latent."""
        for b, sid in enumerate(seq_ids):
            self.cache.append(sid, self._latent_entries(x[b], self.cache.sequences.get(sid, {"len": 0})["len"]))
        return self.mla(x)

    @torch.no_grad()
    def step(self, x: torch.Tensor, seq_ids: Sequence[int]) -> torch.Tensor:
        """One new token per sequence: x [R, 1, hidden] -> [R, 1, hidden]."""
        m = self.mla
        R = x.shape[0]
        H, d, r = m.num_heads, m.head_dim, m.rope_dim
        pos = [self.cache.sequences.get(s, {"len": 0})["len"] for s in seq_ids]
        for i, sid in enumerate(seq_ids):
            self.cache.append(sid, self._latent_entries(x[i], pos[i]))
        q_nope = m.q_proj(x[:, 0]).view(R, H, d)
        q_rope = m.q_rope_proj(x[:, 0]).view(R, H, r)
        q_rope = torch.stack([m.rope(q_rope[i:i + 1].unsqueeze(2), pos[i])[0, :, 0] for i in range(R)])
        w_uk, w_uv = absorbed_weights(m)
        q_lat = torch.einsum("rhd,hdl->rhl", q_nope.float(), w_uk.float())
        q = torch.cat([q_lat, q_rope.float()], dim=-1).to(self.dtype)
        bt, lens = self.cache.block_table(seq_ids)
        o_lat = mla_decode(q, self.cache.pages, bt, lens, scale=m.scale, max_ctx=max(pos) + 1)
        o = torch.einsum("rhl,hdl->rhd", o_lat.float(), w_uv.float())
        o = torch.nn.functional.pad(o, (0, r)).reshape(R, 1, H * (d + r)).to(x.dtype)
        return m.o_proj(o)
