"""KV caches — drop-in for the reference's ops/kv_cache.py:18-240.

``ContinuousKVCache``: contiguous [max_batch, H, max_seq, D] buffers with
per-batch lengths (kv_cache.py:18-107).

``PagedKVCache``: page pool [max_pages, H_kv, page_size, D], a FIFO free
list and per-sequence page tables with the reference's exact allocation
semantics (kv_cache.py:110-240: pages popped from the front of the free
list, freed pages appended at its back, tables grown token by token).  Slot
assignment is host bookkeeping; the K/V bytes are scattered on the device
by ``ffa_paged_append`` in one launch per call instead of a per-token loop.
Beyond the reference API, ``block_table()`` exports the tables as an int32
tensor and ``decode()`` runs the sm_100a split-KV decode directly on the
pool, with no gather.
"""
from __future__ import annotations

from typing import List, Optional, Sequence, Tuple

import torch

from . import _lib
from .decode import check_block_table


class ContinuousKVCache:
    """Contiguous KV cache (kv_cache.py:18-107)."""

    def __init__(self, max_batch: int, max_seq_len: int, num_heads: int, head_dim: int,
                 dtype: torch.dtype = torch.float16, device: torch.device | str = "cpu"):
        self.max_batch = max_batch
        self.max_seq_len = max_seq_len
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.k_cache = torch.zeros(max_batch, num_heads, max_seq_len, head_dim, dtype=dtype, device=device)
        self.v_cache = torch.zeros(max_batch, num_heads, max_seq_len, head_dim, dtype=dtype, device=device)
        self.seq_lens = torch.zeros(max_batch, dtype=torch.long, device=device)
        self._host_lens = [0] * max_batch

    def reset(self, batch_indices: Optional[torch.Tensor] = None):
        if batch_indices is None:
            self.seq_lens.zero_()
            self._host_lens = [0] * self.max_batch
        else:
            self.seq_lens[batch_indices] = 0
            for b in torch.as_tensor(batch_indices).flatten().tolist():
                self._host_lens[b] = 0

    def append(self, k_new: torch.Tensor, v_new: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Append [B, H, S_new, D] and return views [B, H, max_len, D] (kv_cache.py:68-97)."""
        B, H, S_new, D = k_new.shape
        starts = self._host_lens[:B]
        for b in range(B):
            assert starts[b] + S_new <= self.max_seq_len, \
                f"KV-cache overflow: {starts[b] + S_new} > {self.max_seq_len}"
        if all(s == starts[0] for s in starts):  # common case: one strided copy
            s0 = starts[0]
            self.k_cache[:B, :, s0:s0 + S_new] = k_new
            self.v_cache[:B, :, s0:s0 + S_new] = v_new
        else:
            for b in range(B):
                self.k_cache[b, :, starts[b]:starts[b] + S_new] = k_new[b]
                self.v_cache[b, :, starts[b]:starts[b] + S_new] = v_new[b]
        for b in range(B):
            self._host_lens[b] += S_new
        self.seq_lens[:B] += S_new
        max_len = max(self._host_lens[:B])
        return self.k_cache[:B, :, :max_len], self.v_cache[:B, :, :max_len]

    def get_cache(self, batch_size: int):
        max_len = max(self._host_lens[:batch_size]) if batch_size else 0
        if max_len == 0:
            return None, None
        return self.k_cache[:batch_size, :, :max_len], self.v_cache[:batch_size, :, :max_len]


class PagedKVCache:
    """Paged KV cache (kv_cache.py:110-240) with device-side append and decode."""

    def __init__(self, max_pages: int = 1024, page_size: int = 64, num_heads: int = 8, head_dim: int = 64,
                 dtype: torch.dtype = torch.float16, device: torch.device | str = "cpu"):
        self.max_pages = max_pages
        self.page_size = page_size
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.k_pages = torch.zeros(max_pages, num_heads, page_size, head_dim, dtype=dtype, device=device)
        self.v_pages = torch.zeros(max_pages, num_heads, page_size, head_dim, dtype=dtype, device=device)
        self.free_pages: List[int] = list(range(max_pages))
        self.sequences: dict = {}

    # ---- allocator (kv_cache.py:157-168) ----
    def allocate_page(self) -> int:
        if not self.free_pages:
            raise RuntimeError("PagedKVCache: out of physical pages")
        return self.free_pages.pop(0)

    def free_sequence(self, seq_id: int):
        if seq_id in self.sequences:
            for page_id in self.sequences[seq_id]["page_table"]:
                self.free_pages.append(page_id)
            del self.sequences[seq_id]

    def _assign_slots(self, seq_id: int, n: int) -> List[int]:
        """Slot (page * page_size + offset) of each appended token, allocating
        pages exactly as the reference's per-token loop does (kv_cache.py:192-204)."""
        seq = self.sequences.setdefault(seq_id, {"page_table": [], "len": 0})
        slots = []
        for _ in range(n):
            idx, off = divmod(seq["len"], self.page_size)
            while len(seq["page_table"]) <= idx:
                seq["page_table"].append(self.allocate_page())
            slots.append(seq["page_table"][idx] * self.page_size + off)
            seq["len"] += 1
        return slots

    def append_tokens(self, seq_id: int, k_tokens: torch.Tensor, v_tokens: torch.Tensor) -> int:
        """Append [num_heads, S_new, head_dim] K/V; returns the new length (kv_cache.py:170-206)."""
        S_new = k_tokens.size(1)
        slots = self._assign_slots(seq_id, S_new)
        if S_new == 0:
            return self.sequences[seq_id]["len"]
        if self.k_pages.is_cuda and self.k_pages.dtype in _lib.DTYPE_CODE and self.head_dim % 8 == 0:
            k_new = k_tokens.to(self.k_pages.device, self.k_pages.dtype).contiguous()
            v_new = v_tokens.to(self.v_pages.device, self.v_pages.dtype).contiguous()
            slot_t = torch.tensor(slots, dtype=torch.int32).to(self.k_pages.device)
            lib = _lib.load()
            with torch.cuda.device(self.k_pages.device):
                st = lib.ffa_paged_append(k_new.data_ptr(), v_new.data_ptr(), self.k_pages.data_ptr(),
                                          self.v_pages.data_ptr(), slot_t.data_ptr(),
                                          _lib.DTYPE_CODE[self.k_pages.dtype], S_new, self.num_heads,
                                          self.head_dim, self.page_size, self.max_pages,
                                          _lib.i64arr(k_new.stride(0), k_new.stride(1)),
                                          _lib.stream_of(self.k_pages))
            _lib.check(st, "ffa_paged_append")
        else:
            # Host-side pool (CPU or fp32): same scatter with tensor indexing.
            slot_t = torch.tensor(slots, dtype=torch.long, device=self.k_pages.device)
            pages, offs = slot_t // self.page_size, slot_t % self.page_size
            self.k_pages[pages, :, offs, :] = k_tokens.permute(1, 0, 2).to(self.k_pages)
            self.v_pages[pages, :, offs, :] = v_tokens.permute(1, 0, 2).to(self.v_pages)
        return self.sequences[seq_id]["len"]

    def get_kv(self, seq_id: int) -> Tuple[Optional[torch.Tensor], Optional[torch.Tensor]]:
        """Contiguous [num_heads, len, head_dim] copies of a sequence (kv_cache.py:208-232)."""
        if seq_id not in self.sequences or self.sequences[seq_id]["len"] == 0:
            return None, None
        seq = self.sequences[seq_id]
        L = seq["len"]
        idx = torch.tensor(seq["page_table"], dtype=torch.long, device=self.k_pages.device)
        k = self.k_pages[idx].permute(1, 0, 2, 3).reshape(self.num_heads, -1, self.head_dim)[:, :L]
        v = self.v_pages[idx].permute(1, 0, 2, 3).reshape(self.num_heads, -1, self.head_dim)[:, :L]
        return k.contiguous(), v.contiguous()

    @property
    def num_free_pages(self) -> int:
        return len(self.free_pages)

    @property
    def total_capacity(self) -> int:
        return self.max_pages * self.page_size

    # ---- device views for the decode kernel ----
    def block_table(self, seq_ids: Sequence[int], device=None) -> Tuple[torch.Tensor, torch.Tensor]:
        """(block_table int32 [R, max_pages_of_batch], ctx_lens int32 [R]) on `device`."""
        device = device or self.k_pages.device
        tables = [self.sequences[s]["page_table"] for s in seq_ids]
        width = max(1, max(len(t) for t in tables))
        bt = torch.zeros(len(seq_ids), width, dtype=torch.int32)
        for i, t in enumerate(tables):
            if t:
                bt[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
        lens = torch.tensor([self.sequences[s]["len"] for s in seq_ids], dtype=torch.int32)
        check_block_table(bt, lens, self.max_pages, self.page_size)
        return bt.to(device), lens.to(device)

    def decode(self, q: torch.Tensor, seq_ids: Sequence[int], *, scale: Optional[float] = None,
               softcap: Optional[float] = None, return_lse: bool = False):
        """One-token attention of q [R, Hq, D] over each sequence's cached K/V."""
        from .decode import paged_decode

        bt, lens = self.block_table(seq_ids, q.device)
        max_ctx = max(self.sequences[s]["len"] for s in seq_ids)
        return paged_decode(q, self.k_pages, self.v_pages, bt, lens, scale=scale, softcap=softcap,
                            return_lse=return_lse, max_ctx=max_ctx)
