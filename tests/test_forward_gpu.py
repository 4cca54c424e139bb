"""GPU parity of the sm_100a forward against the reference (golden fixtures)
and against the pinned numpy oracle.  Mirrors the reference's own forward
tests (tests/test_fastest_flash.py: basic, causal, window, softcap,
block-sparse, two-pass, KV cache, GQA/MQA, edge cases, LSE, stability).

Tolerances (bf16/fp16 kernels vs the fp32 reference): O max-abs <= 2e-2,
LSE max-abs <= 1e-3.
"""
import math

import numpy as np
import pytest
import torch

from conftest import load_golden, golden_params
from oracle import attention_oracle as O

pytestmark = pytest.mark.gpu

O_TOL = 2e-2
LSE_TOL = 1e-3


def ffa():
    import fastest_flash_attention_b200 as m
    return m


def dev(x, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)


def close(a, b, tol, what):
    a = a.detach().float().cpu().numpy() if isinstance(a, torch.Tensor) else a
    err = np.abs(a - b).max() if a.size else 0.0
    assert err <= tol, f"{what}: max abs err {err:.3e} > {tol}"


GOLDEN_FWD = ["fwd_basic_d16", "fwd_causal_d64", "fwd_causal_d128_ragged", "fwd_window_d64", "fwd_softcap_d64", "fwd_gqa_d128",
              "fwd_noncausal_sq_ne_skv_d64", "fwd_two_pass_d64", "fwd_blockmask_d64",
              # the reference's own test sizes (D = 4 / 8 / 32), zero-padded onto the D = 64 kernel
              "fwd_small_d4_causal", "fwd_small_d8_window_softcap", "fwd_small_d32_mqa_sq_ne_skv"]


@pytest.mark.parametrize("name", GOLDEN_FWD)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_forward_matches_reference_golden(name, dtype):
    g = load_golden(name)
    p = golden_params(g)
    kw = dict(causal=p.get("causal", False), block_size=p.get("block_size"), softcap=p.get("softcap"),
              sliding_window=p.get("sliding_window"), two_pass=p.get("two_pass", False), return_lse=True)
    if "block_mask" in g:
        kw["block_mask"] = torch.from_numpy(g["block_mask"].astype(bool))
    if g["q"].shape[1] != g["k"].shape[1]:
        kw["num_kv_heads"] = g["k"].shape[1]
    o, lse = ffa().fastest_flash_attn_forward(dev(g["q"], dtype), dev(g["k"], dtype), dev(g["v"], dtype), **kw)
    assert o.dtype == dtype and o.shape == g["q"].shape
    close(o, g["o"], O_TOL, "O")
    close(lse, g["lse"], LSE_TOL, "LSE")


def test_forward_kvcache_golden():
    g = load_golden("fwd_kvcache_d64")
    o, lse = ffa().fastest_flash_attn_forward(dev(g["q"]), dev(g["k"]), dev(g["v"]), causal=True, block_size=16,
                                              kv_cache=(dev(g["k_cache"]), dev(g["v_cache"])), return_lse=True)
    close(o, g["o"], O_TOL, "O")
    close(lse, g["lse"], LSE_TOL, "LSE")


def test_forward_compute_dtype_fp16_golden():
    """fp32 callers with compute_dtype=torch.float16 (cpu_reference.py:28-32,
    260-261): the kernels run in fp16 and the output comes back in fp32."""
    g = load_golden("fwd_fp16_compute_d16")
    p = golden_params_dtype(g)
    assert p["compute_dtype"] == torch.float16
    q, k, v = (dev(g[x], torch.float32) for x in ("q", "k", "v"))
    o, lse = ffa().fastest_flash_attn_forward(q, k, v, block_size=p["block_size"], compute_dtype=torch.float16,
                                              return_lse=True)
    assert o.dtype == torch.float32
    close(o, g["o"], O_TOL, "O")
    close(lse, g["lse"], LSE_TOL, "LSE")
    # the same through an AttentionConfig
    cfg = ffa().AttentionConfig(compute_dtype=torch.float16, return_lse=True)
    o2, _ = ffa().fastest_flash_attn_forward(q, k, v, config=cfg)
    assert torch.equal(o, o2)


def golden_params_dtype(g):
    import ast
    txt = str(g["params"]).replace("torch.float16", "'float16'").replace("torch.bfloat16", "'bfloat16'")
    p = ast.literal_eval(txt)
    return {k: getattr(torch, v) if k == "compute_dtype" else v for k, v in p.items()}


def _rand(*shape, dtype=torch.bfloat16, scale=1.0, seed=0):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(dtype)


def _oracle_fwd(q, k, v, **kw):
    hq = q.shape[1]
    qn, kn, vn = (t.float().numpy() for t in (q, k, v))
    kn, vn = O.repeat_kv(kn, hq), O.repeat_kv(vn, hq)
    return O.flash_forward(qn, kn, vn, return_lse=True, **kw)


@pytest.mark.parametrize("B,Hq,Hkv,Sq,Skv,D,causal,window,softcap", [
    (2, 8, 8, 1024, 1024, 64, True, None, None),      # config 1 shape (bf16 path)
    (1, 4, 1, 777, 777, 128, True, None, None),        # MQA, ragged
    (1, 2, 2, 1, 300, 128, False, None, None),         # single query row
    (1, 2, 2, 300, 1, 64, False, None, None),          # single key
    (2, 4, 2, 520, 520, 128, True, 130, 30.0),         # config 3 features, small
    (1, 2, 2, 333, 129, 64, False, 50, None),          # window without causal, S_q > S_kv
])
def test_forward_vs_oracle(B, Hq, Hkv, Sq, Skv, D, causal, window, softcap):
    q = _rand(B, Hq, Sq, D, seed=1)
    k = _rand(B, Hkv, Skv, D, seed=2)
    v = _rand(B, Hkv, Skv, D, seed=3)
    o, lse = ffa().fastest_flash_attn_forward(q.cuda(), k.cuda(), v.cuda(), causal=causal, sliding_window=window,
                                              softcap=softcap, return_lse=True)
    ro, rl = _oracle_fwd(q, k, v, causal=causal, sliding_window=window, softcap=softcap, block_q=128,
                         block_kv=128)
    close(o, ro, O_TOL, "O")
    # Rows that see no key at all: the kernel returns LSE = -inf (log of an
    # empty sum); the reference returns -inf or log(1e-30) sums depending on
    # whether its tile loop visited a fully masked tile.
    empty = ~np.isfinite(rl) | (rl < -60)
    got = lse.float().cpu().numpy()
    assert np.isneginf(got[empty]).all()
    close(got[~empty], rl[~empty], LSE_TOL, "LSE")


@pytest.mark.parametrize("D,Dv,causal,window", [
    (16, 16, True, None), (32, 32, True, 40), (8, 8, False, None), (80, 80, True, None), (96, 64, False, None),
    (160, 128, True, None), (100, 100, True, 77),
])
def test_forward_other_head_dims(D, Dv, causal, window):
    """Head dims without their own kernel run zero-padded on the next wider one
    (the reference is shape-generic; its own tests use D = 4/8/16)."""
    B, Hq, Hkv, S = 1, 4, 2, 203
    q = _rand(B, Hq, S, D, seed=21)
    k = _rand(B, Hkv, S, D, seed=22)
    v = _rand(B, Hkv, S, Dv, seed=23)
    o, lse = ffa().fastest_flash_attn_forward(q.cuda(), k.cuda(), v.cuda(), causal=causal, sliding_window=window,
                                              return_lse=True)
    assert o.shape == (B, Hq, S, Dv)
    ro, rl = _oracle_fwd(q, k, v, causal=causal, sliding_window=window, block_q=128, block_kv=128)
    close(o, ro, O_TOL, "O")
    close(lse, rl, LSE_TOL, "LSE")


def test_unsupported_head_dims_raise():
    for D, Dv in ((256, 256), (64, 160), (200, 128)):
        q = torch.zeros(1, 1, 8, D, device="cuda", dtype=torch.bfloat16)
        v = torch.zeros(1, 1, 8, Dv, device="cuda", dtype=torch.bfloat16)
        with pytest.raises(ValueError, match="not supported"):
            ffa().fastest_flash_attn_forward(q, q, v)


def test_3d_input_and_fp32_input():
    """3-D [B,S,D] input (attention_forward.py:76) and fp32 callers (computed
    in fp32, held to the reference's fp32 tolerance of 1e-5)."""
    q = _rand(2, 100, 64, dtype=torch.float32, seed=4)
    k = _rand(2, 100, 64, dtype=torch.float32, seed=5)
    v = _rand(2, 100, 64, dtype=torch.float32, seed=6)
    o, lse = ffa().fastest_flash_attn_forward(q.cuda(), k.cuda(), v.cuda(), causal=True, return_lse=True)
    assert o.shape == q.shape and o.dtype == torch.float32 and lse.shape == (2, 100, 1)
    ro, rl = O.flash_forward(q[:, None].numpy(), k[:, None].numpy(), v[:, None].numpy(), causal=True,
                             return_lse=True)
    close(o, ro[:, 0], 1e-5, "O")
    close(lse, rl[:, 0], 1e-5, "LSE")


def test_transposed_layout_input():
    """[B,S,H,D] storage viewed as [B,H,S,D] (the modules' layout) runs without a copy."""
    x = _rand(2, 200, 4, 128, seed=7).cuda()
    q = x.transpose(1, 2)
    k = _rand(2, 200, 4, 128, seed=8).cuda().transpose(1, 2)
    v = _rand(2, 200, 4, 128, seed=9).cuda().transpose(1, 2)
    o, lse = ffa().fastest_flash_attn_forward(q, k, v, causal=True, return_lse=True)
    assert o.stride() == q.stride()
    ro, rl = _oracle_fwd(q.cpu(), k.cpu(), v.cpu(), causal=True)
    close(o, ro, O_TOL, "O")
    close(lse[..., 0], rl[..., 0], LSE_TOL, "LSE")


def test_block_mask_generators_drive_kernel():
    m = ffa()
    S, bs = 256, 32
    mask = m.create_sliding_window_block_mask(S, S, bs, bs, 64)
    q, k, v = (_rand(1, 2, S, 64, seed=s) for s in (10, 11, 12))
    o, _ = m.fastest_flash_attn_forward(q.cuda(), k.cuda(), v.cuda(), block_size=bs, block_mask=mask)
    ro, _ = _oracle_fwd(q, k, v, block_q=bs, block_kv=bs, block_mask=mask.numpy())
    close(o, ro, O_TOL, "O")


def test_numerical_stability_large_and_zero():
    q = _rand(1, 2, 64, 64, scale=30.0, seed=13)
    k = _rand(1, 2, 64, 64, scale=30.0, seed=14)
    v = _rand(1, 2, 64, 64, seed=15)
    o, lse = ffa().fastest_flash_attn_forward(q.cuda(), k.cuda(), v.cuda(), return_lse=True)
    assert torch.isfinite(o).all() and torch.isfinite(lse).all()
    ro, _ = _oracle_fwd(q, k, v)
    close(o, ro, 5e-2, "O (large logits)")
    z = torch.zeros(1, 2, 64, 64, dtype=torch.bfloat16, device="cuda")
    o, _ = ffa().fastest_flash_attn_forward(z, z, z)
    assert torch.equal(o, z)


def test_config_object():
    m = ffa()
    cfg = m.AttentionConfig(causal=True, sliding_window=100, softcap=20.0, return_lse=True)
    q, k, v = (_rand(1, 2, 300, 64, seed=s) for s in (16, 17, 18))
    o, lse = m.fastest_flash_attn_forward(q.cuda(), k.cuda(), v.cuda(), config=cfg)
    ro, rl = _oracle_fwd(q, k, v, causal=True, sliding_window=100, softcap=20.0)
    close(o, ro, O_TOL, "O")
    close(lse, rl, LSE_TOL, "LSE")


def test_full_size_config2_rows():
    """Config 2 at full size (B=4 Hq=32 Hkv=8 S=8192 D=128 causal): O and LSE
    of sampled heads checked row by row against an fp32 recomputation."""
    B, Hq, Hkv, S, D = 4, 32, 8, 8192, 128
    g = torch.Generator(device="cuda").manual_seed(0)
    sc = D ** -0.25
    q = (torch.randn(B, Hq, S, D, device="cuda", generator=g) * sc).to(torch.bfloat16)
    k = (torch.randn(B, Hkv, S, D, device="cuda", generator=g) * sc).to(torch.bfloat16)
    v = torch.randn(B, Hkv, S, D, device="cuda", generator=g).to(torch.bfloat16)
    o, lse = ffa().fastest_flash_attn_forward(q, k, v, causal=True, return_lse=True)
    for b, h in ((0, 0), (1, 13), (3, 31)):
        rows = torch.arange(0, S, 97, device="cuda")
        s = (q[b, h, rows].float() @ k[b, h // 4].float().T) / math.sqrt(D)
        s = s.masked_fill(torch.arange(S, device="cuda")[None, :] > rows[:, None], float("-inf"))
        rl = torch.logsumexp(s, -1)
        ro = torch.softmax(s, -1) @ v[b, h // 4].float()
        assert (o[b, h, rows].float() - ro).abs().max().item() <= O_TOL
        assert (lse[b, h, rows, 0] - rl).abs().max().item() <= LSE_TOL


def test_cpu_tensors_raise():
    q = torch.randn(1, 1, 8, 64)
    with pytest.raises(RuntimeError, match="CUDA"):
        ffa().fastest_flash_attn_forward(q, q, q)


def test_two_devices_in_one_process():
    """The kernels' shared-memory attribute is per device: forward and backward
    on cuda:0 then cuda:1 (then cuda:0 again) from one process all run and
    agree with fp32 torch."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    m = ffa()
    for d in (0, 1, 0):
        dev = torch.device("cuda", d)
        g = torch.Generator(device=dev).manual_seed(d)
        q, k, v = (torch.randn(1, 2, 300, 128, device=dev, generator=g).to(torch.bfloat16).requires_grad_(True)
                   for _ in range(3))
        o = m.fastest_flash_attn_func(q, k, v, causal=True)
        o.float().sum().backward()
        s = (q.float() @ k.float().transpose(-1, -2)) / math.sqrt(128)
        s = s.masked_fill(torch.ones(300, 300, device=dev, dtype=torch.bool).triu(1), float("-inf"))
        ro = torch.softmax(s, -1) @ v.float()
        assert (o.float() - ro).abs().max().item() <= O_TOL
        assert q.grad is not None and torch.isfinite(q.grad.float()).all()
