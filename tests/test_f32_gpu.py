"""GPU parity of the fp32 path (CUDA-core kernels behind ffa_fwd / ffa_bwd with
dtype FFA_DTYPE_F32) at the reference's own fp32 tolerances.

The reference computes fp32 inputs in fp32 (kernels/cpu_reference.py:28-32,
132-427) and its tests hold fp32 outputs to atol 1e-5
(tests/test_fastest_flash.py).  Here:
  * forward O max-abs <= 1e-5 and LSE max-abs <= 1e-5 against the reference
    fixtures and the oracle;
  * gradients within 1e-4 relative (max |err| / max |ref|) against the
    reference fixtures and an fp64 torch autograd reference with every mask;
  * the fp32 backward is bit-identical run to run;
  * fp64 callers (computed in fp32) pass torch.autograd.gradcheck at the
    tolerances of the reference's own small gradcheck.
"""
import math

import numpy as np
import pytest
import torch

from conftest import load_golden, golden_params
from oracle import attention_oracle as O

pytestmark = pytest.mark.gpu

O_TOL = 1e-5
LSE_TOL = 1e-5
G_TOL = 1e-4


def ffa():
    import fastest_flash_attention_b200 as m
    return m


def dev(x, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)


def max_abs(a, b):
    a = a.detach().double().cpu().numpy() if isinstance(a, torch.Tensor) else a
    b = b.detach().double().cpu().numpy() if isinstance(b, torch.Tensor) else b
    return float(np.abs(a - b).max()) if a.size else 0.0


def rel_err(a, b):
    b = b.detach().double().cpu().numpy() if isinstance(b, torch.Tensor) else np.asarray(b, np.float64)
    return max_abs(a, b) / max(float(np.abs(b).max()), 1e-6)


GOLDEN_FWD = ["fwd_basic_d16", "fwd_causal_d64", "fwd_causal_d128_ragged", "fwd_window_d64", "fwd_softcap_d64",
              "fwd_gqa_d128", "fwd_noncausal_sq_ne_skv_d64", "fwd_two_pass_d64", "fwd_blockmask_d64",
              "fwd_small_d4_causal", "fwd_small_d8_window_softcap", "fwd_small_d32_mqa_sq_ne_skv"]


@pytest.mark.parametrize("name", GOLDEN_FWD)
def test_f32_forward_matches_reference_golden(name):
    g = load_golden(name)
    p = golden_params(g)
    kw = dict(causal=p.get("causal", False), block_size=p.get("block_size"), softcap=p.get("softcap"),
              sliding_window=p.get("sliding_window"), two_pass=p.get("two_pass", False), return_lse=True)
    if "block_mask" in g:
        kw["block_mask"] = torch.from_numpy(g["block_mask"].astype(bool))
    if g["q"].shape[1] != g["k"].shape[1]:
        kw["num_kv_heads"] = g["k"].shape[1]
    o, lse = ffa().fastest_flash_attn_forward(dev(g["q"]), dev(g["k"]), dev(g["v"]), **kw)
    assert o.dtype == torch.float32 and o.shape == g["q"].shape
    assert max_abs(o, g["o"]) <= O_TOL, f"O err {max_abs(o, g['o']):.3e}"
    assert max_abs(lse, g["lse"]) <= LSE_TOL, f"LSE err {max_abs(lse, g['lse']):.3e}"


def test_f32_forward_kvcache_golden():
    g = load_golden("fwd_kvcache_d64")
    o, lse = ffa().fastest_flash_attn_forward(dev(g["q"]), dev(g["k"]), dev(g["v"]), causal=True, block_size=16,
                                              kv_cache=(dev(g["k_cache"]), dev(g["v_cache"])), return_lse=True)
    assert max_abs(o, g["o"]) <= O_TOL
    assert max_abs(lse, g["lse"]) <= LSE_TOL


@pytest.mark.parametrize("name", ["bwd_causal_d64", "bwd_window_softcap_d128", "bwd_noncausal_d64",
                                  "bwd_small_d8_causal", "bwd_small_d16_window", "bwd_small_d32_softcap"])
def test_f32_backward_matches_reference_golden(name):
    g = load_golden(name)
    p = golden_params(g)
    q, k, v, do, o = (dev(g[x]) for x in ("q", "k", "v", "do", "o"))
    lse = torch.from_numpy(g["lse"]).cuda()
    dq, dk, dv = ffa().fastest_flash_attn_backward(do, q, k, v, o, lse, causal=p.get("causal", False),
                                                   softcap=p.get("softcap"), sliding_window=p.get("sliding_window"))
    for got, ref, nm in ((dq, g["dq"], "dq"), (dk, g["dk"], "dk"), (dv, g["dv"], "dv")):
        assert got.dtype == torch.float32
        e = rel_err(got, ref)
        assert e <= G_TOL, f"{nm}: rel err {e:.3e}"


def test_f32_autograd_func_3d_golden():
    g = load_golden("func_3d_causal_d64")
    q, k, v = (dev(g[x]).requires_grad_(True) for x in ("q", "k", "v"))
    o = ffa().fastest_flash_attn_func(q, k, v, causal=True, block_size=16)
    assert max_abs(o, g["o"]) <= O_TOL
    o.backward(dev(g["do"]))
    for t, nm in ((q, "dq"), (k, "dk"), (v, "dv")):
        e = rel_err(t.grad, g[nm])
        assert e <= G_TOL, f"{nm}: rel err {e:.3e}"


def _torch_ref(q, k, v, *, scale, causal=False, q_offset=0, window=None, softcap=None, block_mask=None,
               mask_block=(64, 64)):
    """fp64 attention with every mask of the kernels (GQA by head index):
    key j visible to query i iff j <= i + q_offset (causal), j >= i + q_offset -
    window + 1 (window), and its block-mask tile is kept.  Rows that see no key
    give O = 0 and LSE = -inf."""
    q, k, v = (t.double() for t in (q, k, v))
    Hq, Hkv = q.shape[1], k.shape[1]
    k = k.repeat_interleave(Hq // Hkv, dim=1)
    v = v.repeat_interleave(Hq // Hkv, dim=1)
    s = torch.matmul(q, k.transpose(-1, -2)) * scale
    if softcap:
        s = softcap * torch.tanh(s / softcap)
    Sq, Skv = q.shape[2], k.shape[2]
    i = torch.arange(Sq, device=q.device)[:, None]
    j = torch.arange(Skv, device=q.device)[None, :]
    keep = torch.ones(Sq, Skv, dtype=torch.bool, device=q.device)
    if causal:
        keep &= j <= i + q_offset
    if window:
        keep &= j >= i + q_offset - window + 1
    if block_mask is not None:
        bm = block_mask.to(q.device).bool()
        keep &= bm[i // mask_block[0], j // mask_block[1]]
    s = s.masked_fill(~keep, float("-inf"))
    lse = torch.logsumexp(s.detach(), dim=-1)
    seen = keep.any(dim=-1)[:, None]  # rows with at least one visible key
    p = torch.softmax(s.masked_fill(~seen, 0.0), dim=-1) * seen
    return torch.matmul(p, v), lse


def _rand(*shape, seed):
    gen = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=gen, dtype=torch.float32)


CASES = [
    # B, Hq, Hkv, Sq, Skv, D, Dv, causal, window, softcap, block mask
    (1, 4, 2, 300, 300, 128, 128, True, None, None, False),    # GQA, ragged
    (2, 2, 1, 130, 257, 64, 64, True, 100, None, False),       # MQA, Sq != Skv (bottom-right), window
    (1, 2, 2, 200, 200, 128, 128, True, 70, 30.0, False),      # config-3 features
    (1, 3, 3, 190, 190, 64, 64, False, None, 5.0, True),       # block mask (with a fully masked row block)
    (1, 4, 2, 160, 160, 192, 128, True, None, None, False),    # MLA shape qk 192 / v 128
    (1, 2, 2, 77, 77, 48, 48, False, None, None, False),       # head dim without its own kernel (padded)
]


@pytest.mark.parametrize("B,Hq,Hkv,Sq,Skv,D,Dv,causal,window,softcap,bm", CASES)
def test_f32_fwd_bwd_vs_fp64_autograd(B, Hq, Hkv, Sq, Skv, D, Dv, causal, window, softcap, bm):
    q, k, v, do = _rand(B, Hq, Sq, D, seed=1), _rand(B, Hkv, Skv, D, seed=2), _rand(B, Hkv, Skv, Dv, seed=3), \
        _rand(B, Hq, Sq, Dv, seed=4)
    scale = 1.0 / math.sqrt(D)
    block_mask = None
    if bm:
        gen = torch.Generator().manual_seed(9)
        block_mask = torch.rand(math.ceil(Sq / 32), math.ceil(Skv / 32), generator=gen) > 0.4
        block_mask[1, :] = False  # rows 32-63 see no key
    kw = dict(scale=scale, causal=causal, q_offset=Skv - Sq, window=window, softcap=softcap)
    from fastest_flash_attention_b200 import attention as m
    qc, kc, vc = (t.cuda() for t in (q, k, v))
    o, lse = m.flash_fwd(qc, kc, vc, block_mask=block_mask, mask_block=(32, 32), **kw)
    assert o.dtype == torch.float32
    qd, kd, vd = (t.double().cuda().requires_grad_(True) for t in (q, k, v))
    ro, rl = _torch_ref(qd, kd, vd, block_mask=block_mask, mask_block=(32, 32), **kw)
    assert max_abs(o, ro) <= O_TOL, f"O err {max_abs(o, ro):.3e}"
    fin = torch.isfinite(rl)
    assert torch.equal(torch.isfinite(lse.cpu()), fin.cpu())
    assert max_abs(lse[fin], rl[fin]) <= LSE_TOL
    if bm:
        assert float(o[:, :, 32:64].abs().max()) == 0.0
    ro.backward(do.double().cuda())
    dq, dk, dv = m.flash_bwd(do.cuda(), qc, kc, vc, o, lse, block_mask=block_mask, mask_block=(32, 32), **kw)
    for got, t, nm in ((dq, qd, "dq"), (dk, kd, "dk"), (dv, vd, "dv")):
        assert got.dtype == torch.float32 and got.shape == t.shape
        e = rel_err(got, t.grad)
        assert e <= G_TOL, f"{nm}: rel err {e:.3e}"


def test_f32_backward_deterministic_bitwise():
    q, k, v, do = (_rand(2, 4, 333, 128, seed=s).cuda() for s in (8, 9, 10, 11))
    k, v = k[:, :2].contiguous(), v[:, :2].contiguous()
    from fastest_flash_attention_b200 import attention as m
    o, lse = m.flash_fwd(q, k, v, scale=128 ** -0.5, causal=True)
    first = m.flash_bwd(do, q, k, v, o, lse, scale=128 ** -0.5, causal=True)
    for _ in range(2):
        again = m.flash_bwd(do, q, k, v, o, lse, scale=128 ** -0.5, causal=True)
        for a, b in zip(first, again):
            assert torch.equal(a, b)


def test_f64_gradcheck_small():
    """fp64 callers run on the fp32 kernels and pass a numerical gradient check
    at the tolerances the reference's own small gradcheck uses (atol = rtol =
    5e-2, eps = 1e-3; tests/test_fastest_flash.py)."""
    gen = torch.Generator().manual_seed(102)
    q, k, v = (torch.randn(1, 1, 4, 4, generator=gen, dtype=torch.float64).cuda().requires_grad_(True)
               for _ in range(3))

    def fn(q, k, v):
        return ffa().fastest_flash_attn_func(q, k, v, block_size=4)

    assert torch.autograd.gradcheck(fn, (q, k, v), atol=5e-2, rtol=5e-2, eps=1e-3)


def test_f32_compute_dtype_bf16_uses_tensor_cores():
    """compute_dtype=torch.bfloat16 still routes fp32 callers to the bf16 tensor-core kernels."""
    q, k, v = (_rand(1, 2, 128, 64, seed=s).cuda() for s in (1, 2, 3))
    o32, _ = ffa().fastest_flash_attn_forward(q, k, v, causal=True)
    o16, _ = ffa().fastest_flash_attn_forward(q, k, v, causal=True, compute_dtype=torch.bfloat16)
    assert o16.dtype == torch.float32
    qb, kb, vb = (t.to(torch.bfloat16).float().cpu().numpy() for t in (q, k, v))
    ro = O.flash_forward(qb, kb, vb, causal=True, return_lse=True)[0]
    assert max_abs(o16, ro) <= 2e-2
    assert max_abs(o32, o16) > 0.0  # the two paths round differently
