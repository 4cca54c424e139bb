"""GPU parity of the deterministic sm_100a backward against the reference
(golden fixtures from kernels/cpu_reference.py:319 flash_attn_cpu_backward and
the autograd path ops/attention_func.py) and the pinned oracle.

Tolerance: gradients within 5e-2 relative (max |err| / max |ref|); the
deterministic backward is checked bit-identical run to run.
"""
import math

import numpy as np
import pytest
import torch

from conftest import load_golden, golden_params
from oracle import attention_oracle as O

pytestmark = pytest.mark.gpu
G_TOL = 5e-2


def ffa():
    import fastest_flash_attention_b200 as m
    return m


def dev(x, dtype=torch.bfloat16):
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)


def rel_err(a, b):
    a = a.detach().float().cpu().numpy() if isinstance(a, torch.Tensor) else a
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-6))


@pytest.mark.parametrize("name", ["bwd_causal_d64", "bwd_window_softcap_d128", "bwd_noncausal_d64",
                                  "bwd_small_d8_causal", "bwd_small_d16_window", "bwd_small_d32_softcap"])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_backward_matches_reference_golden(name, dtype):
    g = load_golden(name)
    p = golden_params(g)
    p.pop("block_size")
    q, k, v, do, o = (dev(g[x], dtype) for x in ("q", "k", "v", "do", "o"))
    lse = torch.from_numpy(g["lse"]).cuda()
    dq, dk, dv = ffa().fastest_flash_attn_backward(do, q, k, v, o, lse, causal=p.get("causal", False),
                                                   softcap=p.get("softcap"), sliding_window=p.get("sliding_window"))
    for got, ref, nm in ((dq, g["dq"], "dq"), (dk, g["dk"], "dk"), (dv, g["dv"], "dv")):
        assert got.dtype == dtype
        e = rel_err(got, ref)
        assert e <= G_TOL, f"{nm}: rel err {e:.3e}"


def test_autograd_func_3d_golden():
    g = load_golden("func_3d_causal_d64")
    q, k, v = (dev(g[x]).requires_grad_(True) for x in ("q", "k", "v"))
    o = ffa().fastest_flash_attn_func(q, k, v, causal=True, block_size=16)
    assert np.abs(o.detach().float().cpu().numpy() - g["o"]).max() <= 2e-2
    o.backward(dev(g["do"]))
    for t, nm in ((q, "dq"), (k, "dk"), (v, "dv")):
        e = rel_err(t.grad, g[nm])
        assert e <= G_TOL, f"{nm}: rel err {e:.3e}"


def _rand(*shape, seed=0, dtype=torch.bfloat16):
    gen = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=gen).to(dtype)


def _oracle_grads(q, k, v, do, hq, **kw):
    qn, kn, vn, don = (t.float().numpy() for t in (q, k, v, do))
    hkv = kn.shape[1]
    kr, vr = O.repeat_kv(kn, hq), O.repeat_kv(vn, hq)
    o, lse = O.flash_forward(qn, kr, vr, return_lse=True, block_q=128, block_kv=128, **kw)
    dq, dk, dv = O.flash_backward(don, qn, kr, vr, o, lse, block_q=128, block_kv=128, **kw)
    g = hq // hkv
    B, _, S, D = dk.shape
    dk = dk.reshape(B, hkv, g, S, D).sum(2)
    dv = dv.reshape(B, hkv, g, dv.shape[2], dv.shape[3]).sum(2)
    return dq, dk, dv


@pytest.mark.parametrize("B,Hq,Hkv,S,D,causal,window,softcap", [
    (1, 4, 2, 300, 128, True, None, None),     # GQA, ragged
    (1, 4, 1, 257, 64, True, 100, None),       # MQA + window
    (1, 2, 2, 384, 128, True, 130, 30.0),      # config-3 features
    (2, 2, 2, 200, 64, False, None, None),
    (1, 2, 1, 150, 16, True, None, None),      # head dims without their own kernel: zero-padded
    (1, 2, 2, 170, 32, True, 50, 20.0),
    (1, 2, 2, 129, 96, False, None, None),
])
def test_backward_vs_oracle(B, Hq, Hkv, S, D, causal, window, softcap):
    q, k, v, do = _rand(B, Hq, S, D, seed=1), _rand(B, Hkv, S, D, seed=2), _rand(B, Hkv, S, D, seed=3), \
        _rand(B, Hq, S, D, seed=4)
    qc, kc, vc = (t.cuda().requires_grad_(True) for t in (q, k, v))
    o = ffa().fastest_flash_attn_func(qc, kc, vc, causal=causal, sliding_window=window, softcap=softcap)
    o.backward(do.cuda())
    rdq, rdk, rdv = _oracle_grads(q, k, v, do, Hq, causal=causal, sliding_window=window, softcap=softcap)
    for t, ref, nm in ((qc, rdq, "dq"), (kc, rdk, "dk"), (vc, rdv, "dv")):
        e = rel_err(t.grad, ref)
        assert e <= G_TOL, f"{nm}: rel err {e:.3e}"


@pytest.mark.parametrize("B,Hq,Hkv,S,causal", [
    (1, 4, 4, 300, True),    # ragged, causal
    (2, 4, 2, 256, False),   # GQA
])
def test_backward_mla_shape_vs_oracle(B, Hq, Hkv, S, causal):
    """qk head dim 192 (128 + 64 rotary), value head dim 128: the MLA training shape."""
    q, k, v, do = _rand(B, Hq, S, 192, seed=11), _rand(B, Hkv, S, 192, seed=12), _rand(B, Hkv, S, 128, seed=13), \
        _rand(B, Hq, S, 128, seed=14)
    qc, kc, vc = (t.cuda().requires_grad_(True) for t in (q, k, v))
    o = ffa().fastest_flash_attn_func(qc, kc, vc, scale=192 ** -0.5, causal=causal)
    assert o.shape[-1] == 128
    o.backward(do.cuda())
    rdq, rdk, rdv = _oracle_grads(q, k, v, do, Hq, causal=causal, scale=192 ** -0.5)
    for t, ref, nm in ((qc, rdq, "dq"), (kc, rdk, "dk"), (vc, rdv, "dv")):
        assert t.grad.shape == t.shape
        e = rel_err(t.grad, ref)
        assert e <= G_TOL, f"{nm}: rel err {e:.3e}"


def test_config1_fp32_full():
    """Config 1 at full size: fp32 [2,8,1024,64], causal, loss = out.sum()."""
    q, k, v = (_rand(2, 8, 1024, 64, seed=s, dtype=torch.float32) for s in (5, 6, 7))
    qc, kc, vc = (t.cuda().requires_grad_(True) for t in (q, k, v))
    out = ffa().fastest_flash_attn_func(qc, kc, vc, causal=True, block_size=64)
    out.sum().backward()
    assert out.dtype == torch.float32 and qc.grad.dtype == torch.float32
    # fp32 inputs are computed in fp32 (CUDA-core kernels): the reference's fp32 tolerance
    qn, kn, vn = (t.numpy() for t in (q, k, v))
    ro, lse = O.flash_forward(qn, kn, vn, causal=True, return_lse=True)
    assert np.abs(out.detach().cpu().numpy() - ro).max() <= 1e-5
    rdq, rdk, rdv = O.flash_backward(np.ones_like(ro), qn, kn, vn, ro, lse, causal=True)
    for t, ref, nm in ((qc, rdq, "dq"), (kc, rdk, "dk"), (vc, rdv, "dv")):
        e = rel_err(t.grad, ref)
        assert e <= 1e-4, f"{nm}: rel err {e:.3e}"


def test_backward_deterministic_bitwise():
    q, k, v, do = (_rand(2, 4, 700, 128, seed=s).cuda() for s in (8, 9, 10, 11))
    k, v = k[:, :2].contiguous(), v[:, :2].contiguous()
    m = ffa()
    o, lse = m.fastest_flash_attn_forward(q, k, v, causal=True, sliding_window=300, softcap=30.0, return_lse=True)
    g1 = m.fastest_flash_attn_backward(do, q, k, v, o, lse, causal=True, sliding_window=300, softcap=30.0)
    g2 = m.fastest_flash_attn_backward(do, q, k, v, o, lse, causal=True, sliding_window=300, softcap=30.0)
    for a, b in zip(g1, g2):
        assert torch.equal(a, b)


def test_config3_slice_full_length():
    """Config 3 features at full length on one head: S=4096, window 1024, softcap 30."""
    q, k, v, do = (_rand(1, 1, 4096, 128, seed=s) for s in (12, 13, 14, 15))
    qc, kc, vc = (t.cuda().requires_grad_(True) for t in (q, k, v))
    o = ffa().fastest_flash_attn_func(qc, kc, vc, causal=True, sliding_window=1024, softcap=30.0)
    o.backward(do.cuda())
    rdq, rdk, rdv = _oracle_grads(q, k, v, do, 1, causal=True, sliding_window=1024, softcap=30.0)
    for t, ref, nm in ((qc, rdq, "dq"), (kc, rdk, "dk"), (vc, rdv, "dv")):
        e = rel_err(t.grad, ref)
        assert e <= G_TOL, f"{nm}: rel err {e:.3e}"


def _masked_attention_fp32(q, k, v, keep, scale):
    """Dense fp32 attention with a boolean [Sq, Skv] keep matrix (GQA by repeat)."""
    g = q.shape[1] // k.shape[1]
    kr, vr = k.repeat_interleave(g, 1), v.repeat_interleave(g, 1)
    s = (q @ kr.transpose(-1, -2)) * scale
    s = s.masked_fill(~keep, float("-inf"))
    return torch.softmax(s, -1) @ vr


@pytest.mark.parametrize("S,Skv,D,bs,causal,window", [
    (300, 300, 64, 32, False, None),
    (333, 333, 128, 64, True, None),
    (256, 200, 64, 16, False, 90),
])
def test_backward_with_block_mask(S, Skv, D, bs, causal, window):
    """Block-sparse training: the gradients of the masked forward (the
    reference backward ignores block_mask; here it is defined as the
    derivative of its masked forward, cpu_reference.py:220-224), against fp32
    autograd through a dense masked attention."""
    m = ffa()
    B, Hq, Hkv = 1, 4, 2
    gen = torch.Generator().manual_seed(31)
    n_br, n_bc = -(-S // bs), -(-Skv // bs)
    bm = torch.rand(n_br, n_bc, generator=gen) < 0.6
    bm[torch.arange(n_br), torch.arange(n_br).clamp(max=n_bc - 1)] = True  # every row keeps a block
    q, k, v, do = _rand(B, Hq, S, D, seed=41), _rand(B, Hkv, Skv, D, seed=42), _rand(B, Hkv, Skv, D, seed=43), \
        _rand(B, Hq, S, D, seed=44)
    qc, kc, vc = (t.cuda().requires_grad_(True) for t in (q, k, v))
    o = m.fastest_flash_attn_func(qc, kc, vc, None, causal, bs, None, window, False, bm)
    o.backward(do.cuda())
    # fp32 reference
    qi, ki = torch.arange(S)[:, None], torch.arange(Skv)[None, :]
    keep = bm.repeat_interleave(bs, 0)[:S].repeat_interleave(bs, 1)[:, :Skv]
    if causal:
        keep &= ki <= qi
    if window:
        keep &= ki > qi - window
    assert keep.any(1).all()
    qf, kf, vf = (t.float().cuda().requires_grad_(True) for t in (q, k, v))
    of = _masked_attention_fp32(qf, kf, vf, keep.cuda(), 1 / math.sqrt(D))
    of.backward(do.float().cuda())
    assert (o.float() - of).abs().max().item() <= 2e-2
    for t, ref, nm in ((qc, qf, "dq"), (kc, kf, "dk"), (vc, vf, "dv")):
        e = rel_err(t.grad, ref.grad.cpu().numpy())
        assert e <= G_TOL, f"{nm}: rel err {e:.3e}"
    # deterministic with a mask too
    g1 = [t.grad.clone() for t in (qc, kc, vc)]
    for t in (qc, kc, vc):
        t.grad = None
    m.fastest_flash_attn_func(qc, kc, vc, None, causal, bs, None, window, False, bm).backward(do.cuda())
    assert all(torch.equal(a, t.grad) for a, t in zip(g1, (qc, kc, vc)))


def test_config3_full_size_sampled_heads():
    """Config 3 at full size (B=8 H=16 S=4096 D=128, causal + window 1024 +
    softcap 30, bf16, dO ~ N(0,1)): one fwd+bwd of the whole batch through the
    autograd function, bit-identical when repeated, and dq/dk/dv of sampled
    (batch, head) slices against fp32 torch autograd of the same attention."""
    m = ffa()
    B, H, S, D, W, cap = 8, 16, 4096, 128, 1024, 30.0
    g = torch.Generator(device="cuda").manual_seed(21)
    q, k, v, do = (torch.randn(B, H, S, D, device="cuda", generator=g).to(torch.bfloat16) for _ in range(4))
    qc, kc, vc = (t.clone().requires_grad_(True) for t in (q, k, v))
    m.fastest_flash_attn_func(qc, kc, vc, causal=True, sliding_window=W, softcap=cap).backward(do)
    grads = [t.grad.clone() for t in (qc, kc, vc)]
    for t in (qc, kc, vc):
        t.grad = None
    m.fastest_flash_attn_func(qc, kc, vc, causal=True, sliding_window=W, softcap=cap).backward(do)
    assert all(torch.equal(a, t.grad) for a, t in zip(grads, (qc, kc, vc)))
    i = torch.arange(S, device="cuda")
    keep = (i[None, :] <= i[:, None]) & (i[None, :] > i[:, None] - W)
    for b, h in ((0, 0), (3, 7), (7, 15)):
        qf, kf, vf = (t[b, h].float().requires_grad_(True) for t in (q, k, v))
        s = (qf @ kf.T) / math.sqrt(D)
        s = cap * torch.tanh(s / cap)
        o = torch.softmax(s.masked_fill(~keep, float("-inf")), -1) @ vf
        o.backward(do[b, h].float())
        for got, ref, nm in ((grads[0][b, h], qf.grad, "dq"), (grads[1][b, h], kf.grad, "dk"),
                             (grads[2][b, h], vf.grad, "dv")):
            e = (got.float() - ref).abs().max().item() / ref.abs().max().item()
            assert e <= G_TOL, f"({b},{h}) {nm}: rel err {e:.3e}"
