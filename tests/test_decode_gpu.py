"""GPU parity of the paged split-KV decode against the reference decode path
(PagedKVCache.get_kv gather + forward with one query, restated in the
oracle), including config 4 at full size on sampled requests.
Tolerances: O max-abs <= 2e-2, LSE <= 1e-3."""
import math

import numpy as np
import pytest
import torch

from oracle import attention_oracle as O

pytestmark = pytest.mark.gpu


def _ref(q, kg, vg, scale, softcap=None):
    # one request: q [Hq, D], kg/vg [Hkv, L, D]
    hq = q.shape[0]
    kr, vr = O.repeat_kv(kg[None], hq), O.repeat_kv(vg[None], hq)
    o, lse = O.flash_forward(q[None, :, None], kr, vr, scale=scale, softcap=softcap, return_lse=True,
                             block_q=64, block_kv=128)
    return o[0, :, 0], lse[0, :, 0, 0]


@pytest.mark.parametrize("page_size,Hq,Hkv,D,lens,softcap,dtype", [
    (16, 32, 8, 128, [1, 17, 300, 1000], None, torch.bfloat16),
    (64, 8, 8, 64, [5, 64, 65, 700], None, torch.float16),
    (32, 16, 1, 128, [129, 33], 30.0, torch.bfloat16),     # MQA, G = 16
])
def test_decode_vs_reference_path(page_size, Hq, Hkv, D, lens, softcap, dtype):
    from fastest_flash_attention_b200 import PagedKVCache
    g = torch.Generator().manual_seed(0)
    n_pages = sum((L + page_size - 1) // page_size for L in lens) + 3
    cache = PagedKVCache(max_pages=n_pages, page_size=page_size, num_heads=Hkv, head_dim=D, dtype=dtype,
                         device="cuda")
    cache.free_pages = list(torch.randperm(n_pages, generator=g).tolist())  # permuted block tables
    for sid, L in enumerate(lens):
        k = torch.randn(Hkv, L, D, generator=g).to(dtype)
        v = torch.randn(Hkv, L, D, generator=g).to(dtype)
        cache.append_tokens(sid, k.cuda(), v.cuda())
    q = torch.randn(len(lens), Hq, D, generator=g).to(dtype)
    scale = 1 / math.sqrt(D)
    o, lse = cache.decode(q.cuda(), list(range(len(lens))), softcap=softcap, return_lse=True)
    for sid in range(len(lens)):
        kg, vg = cache.get_kv(sid)
        ro, rl = _ref(q[sid].float().numpy(), kg.float().cpu().numpy(), vg.float().cpu().numpy(), scale, softcap)
        assert np.abs(o[sid].float().cpu().numpy() - ro).max() <= 2e-2
        assert np.abs(lse[sid].cpu().numpy() - rl).max() <= 1e-3


def test_decode_config4_full_size_sampled():
    """64 requests, ctx ~ U[512, 32768], page 16, Hq 32 / Hkv 8, D 128, bf16,
    permuted block table; sampled requests checked against fp32 torch."""
    from fastest_flash_attention_b200 import paged_decode
    g = torch.Generator().manual_seed(0)
    R, Hq, Hkv, D, PS = 64, 32, 8, 128, 16
    lens = torch.randint(512, 32769, (R,), generator=g)
    npg = ((lens + PS - 1) // PS)
    P = int(npg.sum())
    perm = torch.randperm(P, generator=g).to(torch.int32)
    bt = torch.zeros(R, int(npg.max()), dtype=torch.int32)
    off = 0
    for r in range(R):
        bt[r, :npg[r]] = perm[off:off + npg[r]]
        off += int(npg[r])
    kp = torch.randn(P, Hkv, PS, D, device="cuda", dtype=torch.bfloat16)
    vp = torch.randn(P, Hkv, PS, D, device="cuda", dtype=torch.bfloat16)
    q = torch.randn(R, Hq, D, device="cuda", dtype=torch.bfloat16)
    o, lse = paged_decode(q, kp, vp, bt.cuda(), lens.to(torch.int32).cuda(), return_lse=True,
                          max_ctx=int(lens.max()))
    for r in (0, 17, 63):
        L = int(lens[r])
        pages = bt[r, :npg[r]].long().cuda()
        k = kp[pages].permute(1, 0, 2, 3).reshape(Hkv, -1, D)[:, :L].float()
        v = vp[pages].permute(1, 0, 2, 3).reshape(Hkv, -1, D)[:, :L].float()
        k, v = k.repeat_interleave(Hq // Hkv, 0), v.repeat_interleave(Hq // Hkv, 0)
        s = torch.einsum("hd,hld->hl", q[r].float(), k) / math.sqrt(D)
        assert (o[r].float() - torch.softmax(s, -1).unsqueeze(1).bmm(v).squeeze(1)).abs().max().item() <= 2e-2
        assert (lse[r] - torch.logsumexp(s, -1)).abs().max().item() <= 1e-3


@pytest.mark.parametrize("page_size,cps", [(16, None), (64, 8), (16, 16)])
def test_mla_latent_decode_vs_fp32(page_size, cps):
    """Latent MQA over a paged [c_kv | k_rope] cache against an fp32 torch
    reference: contexts on and off the 128-token tile and split boundaries,
    permuted page table, O within 2e-2 and LSE within 1e-3."""
    from fastest_flash_attention_b200.mla import mla_decode
    torch.manual_seed(5)
    lens = [1, 127, 128, 129, 700, 2048 + 37]
    R, H = len(lens), 32
    max_pages = max((L + page_size - 1) // page_size for L in lens)
    n_pages = R * max_pages
    perm = torch.randperm(n_pages)
    bt = perm.view(R, max_pages).to(torch.int32).cuda()
    cache = (torch.randn(n_pages, page_size, 576, device="cuda") * 0.5).to(torch.bfloat16)
    q = torch.randn(R, H, 576, device="cuda").to(torch.bfloat16)
    scale = 192 ** -0.5
    lens_t = torch.tensor(lens, dtype=torch.int32, device="cuda")
    o, lse = mla_decode(q, cache, bt, lens_t, scale=scale, return_lse=True, chunks_per_split=cps)
    flat = cache.view(-1, 576).float()
    for i, L in enumerate(lens):
        pages = bt[i, :(L + page_size - 1) // page_size].long()
        rows = (pages[:, None] * page_size + torch.arange(page_size, device="cuda")[None]).reshape(-1)[:L]
        c = flat[rows]
        s = (q[i].float() @ c.T) * scale
        ref_lse = torch.logsumexp(s, dim=-1)
        ref = torch.softmax(s, dim=-1) @ c[:, :512]
        assert (o[i].float() - ref).abs().max().item() <= 2e-2, (L, (o[i].float() - ref).abs().max().item())
        assert (lse[i] - ref_lse).abs().max().item() <= 1e-3, L
