"""CPU oracle — TEST INFRASTRUCTURE ONLY.

A numpy restatement of the reference's CPU algorithms for the attention hot
path (MindIntels/fastest_flash_attention, paths relative to its project
root).  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
baseline leg may import this module, and only as the checker / the timed CPU
arm; the product (``fastest_flash_attention_b200``) never calls it.

Parity pinning: every function here is checked against golden vectors that
``tests/golden/make_golden.py`` produced by running the reference itself
(imported from its source tree, CPU, fixed seeds); see
``tests/test_oracle_golden.py``.

Arithmetic follows the reference: fp32 accumulation, tile-by-tile online
softmax with log-sum-exp merging, masks applied with ``-inf``, one cast of
the output at the end.  Inputs are numpy arrays; fp16/bf16 tensors are
passed in already converted to float32 (the reference upcasts every tile with
``.float()`` before its matmuls).
"""
from __future__ import annotations

import math
from typing import List, Optional, Tuple

import numpy as np

NEG_INF = np.float32(-np.inf)


# ---------------------------------------------------------------------------
# helpers — kernels/cpu_reference.py:29-56
# ---------------------------------------------------------------------------

def apply_softcap(s: np.ndarray, cap: float) -> np.ndarray:
    """cap * tanh(s / cap)  (cpu_reference.py:35-37)."""
    return (np.float32(cap) * np.tanh(s / np.float32(cap))).astype(np.float32)


def causal_mask(q_start: int, q_end: int, k_start: int, k_end: int) -> np.ndarray:
    """True where masked: row < col  (cpu_reference.py:40-46)."""
    r = np.arange(q_start, q_end)[:, None]
    c = np.arange(k_start, k_end)[None, :]
    return r < c


def window_mask(q_start: int, q_end: int, k_start: int, k_end: int, w: int) -> np.ndarray:
    """True where the key is outside the window: col < row - w + 1 (cpu_reference.py:49-56)."""
    r = np.arange(q_start, q_end)[:, None]
    c = np.arange(k_start, k_end)[None, :]
    return c < (r - w + 1)


def _logaddexp(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    with np.errstate(invalid="ignore"):
        return np.logaddexp(a, b).astype(np.float32)


def _bf16_round(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even to bfloat16, returned as float32."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    return r.view(np.float32)


def to_compute_dtype(x: np.ndarray, compute_dtype: Optional[str]) -> np.ndarray:
    """cpu_reference.py:29-32: cast to a lower precision before Q·K^T."""
    if compute_dtype is None:
        return x
    if compute_dtype == "float16":
        return x.astype(np.float16).astype(np.float32)
    if compute_dtype == "bfloat16":
        return _bf16_round(x)
    return x


def _tile_masked_scores(qb, kb, scale, softcap, causal, window, q_abs_s, q_abs_e, ks, ke):
    s = np.matmul(qb, np.swapaxes(kb, -1, -2)).astype(np.float32) * np.float32(scale)
    if softcap is not None:
        s = apply_softcap(s, softcap)
    if causal:
        s = np.where(causal_mask(q_abs_s, q_abs_e, ks, ke), NEG_INF, s)
    if window is not None:
        s = np.where(window_mask(q_abs_s, q_abs_e, ks, ke, window), NEG_INF, s)
    return s.astype(np.float32)


def _logsumexp_lastdim(s: np.ndarray) -> np.ndarray:
    m = s.max(axis=-1, keepdims=True)
    m_safe = np.where(np.isfinite(m), m, np.float32(0))
    with np.errstate(divide="ignore"):
        out = m_safe + np.log(np.exp(s - m_safe).sum(axis=-1, keepdims=True))
    return out.astype(np.float32)


# ---------------------------------------------------------------------------
# two-pass LSE — kernels/cpu_reference.py:63-125
# ---------------------------------------------------------------------------

def logsumexp_pass1(q, k, scale, causal, block_q, block_kv, block_mask, softcap, window, q_offset=0):
    B, H, S_q, D = q.shape
    S_k = k.shape[2]
    n_br, n_bc = math.ceil(S_q / block_q), math.ceil(S_k / block_kv)
    blocks = []
    for i in range(n_br):
        qs, qe = i * block_q, min(i * block_q + block_q, S_q)
        qa_s, qa_e = q_offset + qs, q_offset + qe
        lse = np.full((B, H, qe - qs, 1), NEG_INF, np.float32)
        for j in range(n_bc):
            ks, ke = j * block_kv, min(j * block_kv + block_kv, S_k)
            if block_mask is not None and not block_mask[i, j]:
                continue
            if causal and ks > qa_e - 1:
                break
            if window is not None and ke - 1 < qa_s - window + 1:
                continue
            s = _tile_masked_scores(q[:, :, qs:qe], k[:, :, ks:ke], scale, softcap, causal, window, qa_s, qa_e, ks, ke)
            lse = _logaddexp(lse, _logsumexp_lastdim(s))
        blocks.append(lse)
    return np.concatenate(blocks, axis=2)


# ---------------------------------------------------------------------------
# forward — kernels/cpu_reference.py:132-312
# ---------------------------------------------------------------------------

def flash_forward(q, k, v, scale=None, causal=False, block_q=64, block_kv=64, block_mask=None, softcap=None,
                  sliding_window=None, two_pass=False, compute_dtype=None, q_offset=0, return_lse=False):
    """Tiled online-softmax forward; returns (O fp32, LSE [B,H,S_q,1] or None).

    q [B,H,S_q,D], k/v [B,H,S_kv,D] (same H: GQA repetition happens before,
    as in ops/attention_forward.py:94-96).
    """
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    B, H, S_q, D = q.shape
    S_kv = k.shape[2]
    Dv = v.shape[3]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    n_br, n_bc = math.ceil(S_q / block_q), math.ceil(S_kv / block_kv)
    exact = logsumexp_pass1(q, k, scale, causal, block_q, block_kv, block_mask, softcap, sliding_window,
                            q_offset) if two_pass else None
    outs, lses = [], []
    for i in range(n_br):
        qs, qe = i * block_q, min(i * block_q + block_q, S_q)
        qa_s, qa_e = q_offset + qs, q_offset + qe
        qb = to_compute_dtype(q[:, :, qs:qe], compute_dtype)
        O = np.zeros((B, H, qe - qs, Dv), np.float32)
        lse_i = np.full((B, H, qe - qs, 1), NEG_INF, np.float32)
        for j in range(n_bc):
            ks, ke = j * block_kv, min(j * block_kv + block_kv, S_kv)
            if block_mask is not None and not block_mask[i, j]:   # :221-224
                continue
            if causal and ks > qa_e - 1:                           # :226-228
                break
            if sliding_window is not None and ke - 1 < qa_s - sliding_window + 1:  # :230-233
                continue
            kb = to_compute_dtype(k[:, :, ks:ke], compute_dtype)
            s = _tile_masked_scores(qb, kb, scale, softcap, causal, sliding_window, qa_s, qa_e, ks, ke)
            vb = v[:, :, ks:ke]
            if exact is not None:                                   # :282-286
                p = np.exp(s - exact[:, :, qs:qe]).astype(np.float32)
                O = O + np.matmul(p, vb)
            else:                                                   # :287-302
                m = s.max(axis=-1, keepdims=True)
                m = np.where(m == NEG_INF, np.float32(0), m)
                p = np.exp(s - m).astype(np.float32)
                lse_ij = m + np.log(np.maximum(p.sum(axis=-1, keepdims=True), np.float32(1e-30)))
                lse_new = _logaddexp(lse_i, lse_ij)
                with np.errstate(invalid="ignore"):
                    alpha = np.exp(lse_i - lse_new).astype(np.float32)
                    tscale = np.exp(m - lse_new).astype(np.float32)
                O = alpha * O + tscale * np.matmul(p, vb)
                lse_i = lse_new
        outs.append(O)
        if return_lse:
            lses.append(exact[:, :, qs:qe] if exact is not None else lse_i)
    out = np.concatenate(outs, axis=2).astype(np.float32)
    return out, (np.concatenate(lses, axis=2) if return_lse else None)


# ---------------------------------------------------------------------------
# backward — kernels/cpu_reference.py:319-427
# ---------------------------------------------------------------------------

def flash_backward(dout, q, k, v, out, lse, scale=None, causal=False, block_q=64, block_kv=64, softcap=None,
                   sliding_window=None, q_offset=0, exp_fn=np.exp):
    """Recompute-based gradients (dq, dk, dv) in fp32.  ``block_mask`` is not
    an input: the reference backward ignores it."""
    dout, q, k, v, out = (np.asarray(t, np.float32) for t in (dout, q, k, v, out))
    lse = np.asarray(lse, np.float32)
    B, H, S_q, D = q.shape
    S_kv = k.shape[2]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    n_br, n_bc = math.ceil(S_q / block_q), math.ceil(S_kv / block_kv)
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    Di = (dout * out).sum(axis=-1, keepdims=True).astype(np.float32)     # :361
    for i in range(n_br):
        qs, qe = i * block_q, min(i * block_q + block_q, S_q)
        qa_s, qa_e = q_offset + qs, q_offset + qe
        qb, dob, lb, db = q[:, :, qs:qe], dout[:, :, qs:qe], lse[:, :, qs:qe], Di[:, :, qs:qe]
        for j in range(n_bc):
            ks, ke = j * block_kv, min(j * block_kv + block_kv, S_kv)
            if causal and ks > qa_e - 1:
                break
            if sliding_window is not None and ke - 1 < qa_s - sliding_window + 1:
                continue
            kb, vb = k[:, :, ks:ke], v[:, :, ks:ke]
            raw = np.matmul(qb, np.swapaxes(kb, -1, -2)).astype(np.float32) * np.float32(scale)
            s = apply_softcap(raw, softcap) if softcap is not None else raw
            if causal:
                s = np.where(causal_mask(qa_s, qa_e, ks, ke), NEG_INF, s)
            if sliding_window is not None:
                s = np.where(window_mask(qa_s, qa_e, ks, ke, sliding_window), NEG_INF, s)
            p = exp_fn(s - lb).astype(np.float32)                        # :392
            dv[:, :, ks:ke] += np.matmul(np.swapaxes(p, -1, -2), dob)
            dp = np.matmul(dob, np.swapaxes(vb, -1, -2))
            ds = p * (dp - db)
            if softcap is not None:                                     # :407-411
                t = np.tanh(raw / np.float32(softcap))
                ds = ds * (1.0 - t * t)
            dq[:, :, qs:qe] += np.matmul(ds, kb) * np.float32(scale)
            dk[:, :, ks:ke] += np.matmul(np.swapaxes(ds, -1, -2), qb) * np.float32(scale)
    return dq, dk, dv


# ---------------------------------------------------------------------------
# FA4 — kernels/cpu_fa4.py
# ---------------------------------------------------------------------------

# Taylor coefficients of 2^f on [0, 1): ln2^n / n!  (cpu_fa4.py:56-59)
_P = (1.0, 0.6931471805599453, 0.2402265069591007, 0.0555041086648216)


def software_exp2(x: np.ndarray) -> np.ndarray:
    """2^x = 2^floor(x) * poly(frac), x clamped at -126 (cpu_fa4.py:62-80)."""
    x = np.maximum(np.asarray(x, np.float32), np.float32(-126.0))
    n = np.floor(x)
    f = (x - n).astype(np.float32)
    poly = (np.float32(_P[0]) + f * (np.float32(_P[1]) + f * (np.float32(_P[2]) + f * np.float32(_P[3])))).astype(
        np.float32)
    return np.ldexp(poly, n.astype(np.int32)).astype(np.float32)


def fast_exp(x: np.ndarray, use_poly: bool = True) -> np.ndarray:
    """exp(x) via 2^(x*log2 e) (cpu_fa4.py:83-93)."""
    if not use_poly:
        return np.exp(x).astype(np.float32)
    return software_exp2(np.asarray(x, np.float32) * np.float32(1.4426950408889634))


def build_tile_schedule(n_br: int, causal: bool, n_bc: int, reverse_mblocks: bool = True) -> List[int]:
    """LPT order: reversed query tiles under causal masking (cpu_fa4.py:131-146)."""
    if causal and reverse_mblocks:
        return list(range(n_br - 1, -1, -1))
    return list(range(n_br))


def fa4_forward(q, k, v, scale=None, causal=False, block_q=128, block_kv=128, block_mask=None, softcap=None,
                sliding_window=None, two_pass=False, compute_dtype=None, q_offset=0, return_lse=False,
                use_poly_exp=True, rescale_threshold=0.0, pingpong=True):
    """FA4 forward restated from cpu_fa4.py:219-438.

    The per-tile LSE is restated as the reference computes it
    (m_ij + log l_ij with P taken against the running max, cpu_fa4.py:412),
    so the returned LSE reproduces the reference's value — which is not the
    true log-sum-exp whenever a later tile's max is below the running max.
    Use :func:`flash_forward` for the exact LSE.
    """
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    B, H, S_q, D = q.shape
    S_kv = k.shape[2]
    Dv = v.shape[3]
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    n_br, n_bc = math.ceil(S_q / block_q), math.ceil(S_kv / block_kv)
    exact = logsumexp_pass1(q, k, scale, causal, block_q, block_kv, block_mask, softcap, sliding_window,
                            q_offset) if two_pass else None
    order = build_tile_schedule(n_br, causal, n_bc)
    groups = [order[g:g + 2] for g in range(0, len(order), 2)] if (pingpong and len(order) >= 2) else [[i] for i in order]
    outs, lses = {}, {}
    for group in groups:
        acc = {}
        for ti in group:
            qs, qe = ti * block_q, min(ti * block_q + block_q, S_q)
            acc[ti] = dict(qs=qs, qe=qe, O=np.zeros((B, H, qe - qs, Dv), np.float32),
                           m=np.full((B, H, qe - qs, 1), NEG_INF, np.float32),
                           l=np.zeros((B, H, qe - qs, 1), np.float32),
                           lse=np.full((B, H, qe - qs, 1), NEG_INF, np.float32))
        for j in range(n_bc):
            ks, ke = j * block_kv, min(j * block_kv + block_kv, S_kv)
            for ti in group:
                a = acc[ti]
                qs, qe = a["qs"], a["qe"]
                qa_s, qa_e = q_offset + qs, q_offset + qe
                if block_mask is not None and not block_mask[ti, j]:
                    continue
                if causal and ks > qa_e - 1:
                    continue
                if sliding_window is not None and ke - 1 < qa_s - sliding_window + 1:
                    continue
                qb = to_compute_dtype(q[:, :, qs:qe], compute_dtype)
                kb = to_compute_dtype(k[:, :, ks:ke], compute_dtype)
                s = _tile_masked_scores(qb, kb, scale, softcap, causal, sliding_window, qa_s, qa_e, ks, ke)
                vb = v[:, :, ks:ke]
                if exact is not None:
                    p = fast_exp(s - exact[:, :, qs:qe], use_poly_exp)
                    a["O"] = a["O"] + np.matmul(p, vb)
                    continue
                m_ij = s.max(axis=-1, keepdims=True)
                m_ij = np.where(m_ij == NEG_INF, np.float32(0), m_ij)
                m_old = a["m"]
                m_new = np.maximum(m_old, m_ij)
                p = fast_exp(s - m_new, use_poly_exp)
                l_ij = p.sum(axis=-1, keepdims=True).astype(np.float32)
                with np.errstate(invalid="ignore"):
                    jump = np.abs(m_new - m_old)
                first = m_old == NEG_INF
                skip = (jump < rescale_threshold) & (~first)
                with np.errstate(invalid="ignore"):
                    exact_alpha = fast_exp(m_old - m_new, use_poly_exp)
                alpha = np.where(first, np.float32(0), np.where(skip, np.float32(1), exact_alpha)).astype(np.float32)
                a["O"] = alpha * a["O"] + np.matmul(p, vb)
                a["l"] = alpha * a["l"] + l_ij
                a["m"] = m_new
                lse_ij = m_ij + np.log(np.maximum(l_ij, np.float32(1e-30)))   # cpu_fa4.py:412
                a["lse"] = _logaddexp(a["lse"], lse_ij)
        for ti in group:
            a = acc[ti]
            if exact is None:
                a["O"] = a["O"] / np.maximum(a["l"], np.float32(1e-30))
            outs[ti] = a["O"]
            if return_lse:
                lses[ti] = exact[:, :, a["qs"]:a["qe"]] if exact is not None else a["lse"]
    out = np.concatenate([outs[i] for i in range(n_br)], axis=2).astype(np.float32)
    lse = np.concatenate([lses[i] for i in range(n_br)], axis=2) if return_lse else None
    return out, lse


def fa4_backward(dout, q, k, v, out, lse, scale=None, causal=False, block_q=128, block_kv=128, softcap=None,
                 sliding_window=None, q_offset=0, use_poly_exp=True, deterministic=False):
    """FA4 backward (cpu_fa4.py:445-586): the base recompute backward with P
    from the polynomial exp.  The even/odd query-tile split and the
    ``deterministic`` flag change only the summation order of dq/dk/dv."""
    return flash_backward(dout, q, k, v, out, lse, scale=scale, causal=causal, block_q=block_q,
                          block_kv=block_kv, softcap=softcap, sliding_window=sliding_window, q_offset=q_offset,
                          exp_fn=lambda x: fast_exp(x, use_poly_exp))


# ---------------------------------------------------------------------------
# GQA expansion and dispatch shape handling — ops/attention_forward.py:23-167
# ---------------------------------------------------------------------------

def repeat_kv(kv: np.ndarray, hq: int) -> np.ndarray:
    """utils.py:111-130: each KV head repeated for its hq/hkv query heads."""
    hkv = kv.shape[1]
    return np.repeat(kv, hq // hkv, axis=1) if hq != hkv else kv


def attention_forward(q, k, v, *, scale=None, causal=False, block_size=64, block_mask=None, softcap=None,
                      sliding_window=None, two_pass=False, compute_dtype=None, kv_cache=None, return_lse=True):
    """fastest_flash_attn_forward's CPU branch on 4-D arrays (attention_forward.py:76-159)."""
    q_offset = 0
    if kv_cache is not None:
        k = np.concatenate([kv_cache[0], k], axis=2)
        v = np.concatenate([kv_cache[1], v], axis=2)
        q_offset = k.shape[2] - q.shape[2]
    k = repeat_kv(k, q.shape[1])
    v = repeat_kv(v, q.shape[1])
    return flash_forward(q, k, v, scale=scale, causal=causal, block_q=block_size, block_kv=block_size,
                         block_mask=block_mask, softcap=softcap, sliding_window=sliding_window, two_pass=two_pass,
                         compute_dtype=compute_dtype, q_offset=q_offset, return_lse=return_lse)


# ---------------------------------------------------------------------------
# block-mask generators — ops/block_sparse.py:17-132
# ---------------------------------------------------------------------------

def causal_block_mask(S_q, S_kv, bq, bkv, q_offset=0):
    n_br, n_bc = math.ceil(S_q / bq), math.ceil(S_kv / bkv)
    m = np.zeros((n_br, n_bc), bool)
    for i in range(n_br):
        q_end = q_offset + min((i + 1) * bq, S_q) - 1
        for j in range(n_bc):
            if q_end >= j * bkv:
                m[i, j] = True
            else:
                break
    return m


def sliding_window_block_mask(S_q, S_kv, bq, bkv, w, q_offset=0):
    n_br, n_bc = math.ceil(S_q / bq), math.ceil(S_kv / bkv)
    m = np.zeros((n_br, n_bc), bool)
    for i in range(n_br):
        q_start = q_offset + i * bq
        q_end = q_offset + min((i + 1) * bq, S_q) - 1
        for j in range(n_bc):
            k_start, k_end = j * bkv, min((j + 1) * bkv, S_kv) - 1
            m[i, j] = (k_end >= q_start - w + 1) and (k_start <= q_end)
    return m


def local_block_mask(S_q, S_kv, bq, bkv, radius):
    n_br, n_bc = math.ceil(S_q / bq), math.ceil(S_kv / bkv)
    m = np.zeros((n_br, n_bc), bool)
    for i in range(n_br):
        qc = i * bq + bq // 2
        for j in range(n_bc):
            kc = j * bkv + bkv // 2
            m[i, j] = abs(qc - kc) <= radius + max(bq, bkv)
    return m


# ---------------------------------------------------------------------------
# paged KV cache bookkeeping — ops/kv_cache.py:110-240
# ---------------------------------------------------------------------------

class PagedCacheModel:
    """Page allocator semantics of PagedKVCache: FIFO free list popped from the
    front (kv_cache.py:157-161), freed pages appended at the back (:163-168),
    one page table per sequence grown token by token (:192-204)."""

    def __init__(self, max_pages: int, page_size: int, free_pages: Optional[List[int]] = None):
        self.max_pages = max_pages
        self.page_size = page_size
        self.free_pages = list(range(max_pages)) if free_pages is None else list(free_pages)
        self.sequences: dict = {}

    def allocate_page(self) -> int:
        if not self.free_pages:
            raise RuntimeError("PagedKVCache: out of physical pages")
        return self.free_pages.pop(0)

    def free_sequence(self, seq_id: int) -> None:
        if seq_id in self.sequences:
            self.free_pages.extend(self.sequences[seq_id]["page_table"])
            del self.sequences[seq_id]

    def append(self, seq_id: int, n_tokens: int) -> List[Tuple[int, int]]:
        """Returns the (page, offset) slot of every appended token."""
        seq = self.sequences.setdefault(seq_id, {"page_table": [], "len": 0})
        slots = []
        for _ in range(n_tokens):
            idx, off = divmod(seq["len"], self.page_size)
            while len(seq["page_table"]) <= idx:
                seq["page_table"].append(self.allocate_page())
            slots.append((seq["page_table"][idx], off))
            seq["len"] += 1
        return slots


def paged_gather(pages: np.ndarray, page_table: List[int], length: int) -> np.ndarray:
    """get_kv (kv_cache.py:208-232): pages [P,H,page,D] -> contiguous [H,L,D]."""
    page = pages.shape[2]
    parts = []
    pos = 0
    for pid in page_table:
        n = min(page, length - pos)
        if n <= 0:
            break
        parts.append(pages[pid, :, :n])
        pos += n
    return np.concatenate(parts, axis=1)


# ---------------------------------------------------------------------------
# MLA — modules/flash_mla.py:29-179 (fp32; positions in fp32, see note)
# ---------------------------------------------------------------------------

def rope(x: np.ndarray, inv_freq: np.ndarray, offset: int = 0) -> np.ndarray:
    """Half-split rotary embedding (flash_mla.py:37-52) on [..., S, d].

    The reference builds positions in x.dtype (:41); this oracle keeps them in
    fp32, which is what the reference computes when run in fp32.
    """
    S = x.shape[-2]
    t = np.arange(offset, offset + S, dtype=np.float32)
    freqs = np.einsum("i,j->ij", t, inv_freq.astype(np.float32)).astype(np.float32)
    emb = np.concatenate([freqs, freqs], axis=-1)
    cos, sin = np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)
    h = x.shape[-1] // 2
    x1, x2 = x[..., :h], x[..., h:]
    return np.concatenate([x1 * cos[..., :h] - x2 * sin[..., :h], x2 * cos[..., :h] + x1 * sin[..., :h]], axis=-1)


def mla_forward(x, w_q, w_qr, w_down, w_up, w_kr, w_o, inv_freq, num_heads, head_dim, rope_dim, causal=True,
                block_size=64):
    """FastestFlashMLA.forward (flash_mla.py:116-172) in fp32 with explicit
    weights (nn.Linear convention: y = x @ W^T)."""
    x = np.asarray(x, np.float32)
    B, S, _ = x.shape
    H, d, r = num_heads, head_dim, rope_dim
    q_nope = (x @ w_q.T).reshape(B, S, H, d).transpose(0, 2, 1, 3)
    q_rope = rope((x @ w_qr.T).reshape(B, S, H, r).transpose(0, 2, 1, 3), inv_freq)
    q = np.concatenate([q_nope, q_rope], -1)
    lat = x @ w_down.T
    kv = (lat @ w_up.T).reshape(B, S, H, 2 * d).transpose(0, 2, 1, 3)
    k_nope, v = kv[..., :d], kv[..., d:]
    kr = np.broadcast_to((x @ w_kr.T)[:, None], (B, H, S, r))
    kr = rope(kr, inv_freq)
    k = np.concatenate([k_nope, kr], -1)
    v_pad = np.concatenate([v, np.zeros(v.shape[:-1] + (r,), np.float32)], -1)
    o, _ = flash_forward(q.astype(np.float32), k.astype(np.float32), v_pad.astype(np.float32),
                         scale=1.0 / math.sqrt(d + r), causal=causal, block_q=block_size, block_kv=block_size)
    o = o.transpose(0, 2, 1, 3).reshape(B, S, H * (d + r))
    return (o @ w_o.T).astype(np.float32)
