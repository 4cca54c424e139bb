"""Sequence-sharded ring attention.

CPU: gloo ranks (world 2 and 3) run the ring's communication and merge with a
plain fp32 torch attention in place of the kernel; every rank's output must
equal its slice of full attention over the concatenated sequence.
GPU (one device): the ring's arithmetic with the sm_100a forward kernel and
the merge kernel, W blocks emulated, against fp32 full attention (O within
2e-2, LSE within 1e-3).  GPU (two devices, NCCL): the distributed ring,
skipped when fewer than two GPUs are visible.
The ring must leave the caller's K / V shards untouched.
Backward: gloo ranks run ring_attention_backward with an fp32 torch backward
of one (query piece, key piece) pair in place of the kernel; every rank's
dQ / dK / dV must equal its slice of the full-sequence autograd gradients.
"""
import math
import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def ref_attn(q, k, v, *, scale, causal=False, q_offset=0, window=None, softcap=None):
    """fp32 attention with the kernel's mask conventions; returns (O, LSE natural log)."""
    g = q.shape[1] // k.shape[1]
    k = k.float().repeat_interleave(g, dim=1)
    v = v.float().repeat_interleave(g, dim=1)
    s = (q.float() @ k.transpose(-1, -2)) * scale
    if softcap:
        s = softcap * torch.tanh(s / softcap)
    Sq, Sk = s.shape[-2:]
    i = torch.arange(Sq, device=s.device)[:, None] + q_offset
    j = torch.arange(Sk, device=s.device)[None]
    keep = torch.ones(Sq, Sk, dtype=torch.bool, device=s.device)
    if causal:
        keep &= j <= i
    if window:
        keep &= j >= i - window + 1
    s = s.masked_fill(~keep, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    p = torch.exp(s - torch.where(torch.isinf(lse), torch.zeros_like(lse), lse)[..., None])
    return p @ v, lse


def ref_attn_bwd(dout, q, k, v, o, lse, *, scale, causal=False, q_offset=0, window=None, softcap=None):
    """fp32 gradients of one (query piece, key piece) pair given the pieces'
    final O and LSE (natural log), with the kernel's mask conventions."""
    g = q.shape[1] // k.shape[1]
    kf = k.float().repeat_interleave(g, dim=1)
    vf = v.float().repeat_interleave(g, dim=1)
    qf, dof, of = q.float(), dout.float(), o.float()
    s = (qf @ kf.transpose(-1, -2)) * scale
    th = torch.tanh(s / softcap) if softcap else None
    sc = softcap * th if softcap else s
    Sq, Sk = s.shape[-2:]
    i = torch.arange(Sq, device=s.device)[:, None] + q_offset
    j = torch.arange(Sk, device=s.device)[None]
    keep = torch.ones(Sq, Sk, dtype=torch.bool, device=s.device)
    if causal:
        keep &= j <= i
    if window:
        keep &= j >= i - window + 1
    lse = lse.float()
    p = torch.exp(sc - torch.where(torch.isinf(lse), torch.zeros_like(lse), lse)[..., None])
    p = torch.where(keep & ~torch.isinf(lse)[..., None], p, torch.zeros_like(p))
    dv = p.transpose(-1, -2) @ dof
    dp = dof @ vf.transpose(-1, -2)
    ds = p * (dp - (dof * of).sum(-1, keepdim=True))
    if softcap:
        ds = ds * (1 - th * th)
    dq = (ds @ kf) * scale
    dk = (ds.transpose(-1, -2) @ qf) * scale
    B, Hkv = k.shape[:2]
    return dq, dk.view(B, Hkv, g, *dk.shape[2:]).sum(2), dv.view(B, Hkv, g, *dv.shape[2:]).sum(2)


def _full(q, k, v, sliding_window=None, **kw):
    return ref_attn(q, k, v, scale=q.shape[-1] ** -0.5, window=sliding_window, **kw)


def _sharder(layout, rank, world, S):
    from fastest_flash_attention_b200.ring import zigzag_shard
    if layout == "zigzag":
        return lambda x: zigzag_shard(x, rank, world, dim=2).contiguous()
    return lambda x: x[:, :, rank * S:(rank + 1) * S].contiguous()


def test_zigzag_shards_roundtrip():
    from fastest_flash_attention_b200.ring import piece_starts, zigzag_shard, zigzag_unshard
    x = torch.arange(48).view(1, 1, 48, 1)
    shards = [zigzag_shard(x, r, 3) for r in range(3)]
    assert torch.equal(zigzag_unshard(shards), x)
    for r in range(3):
        pieces = piece_starts(r, 3, 16, "zigzag")
        got = torch.cat([torch.arange(a, a + l) for a, l in pieces])
        assert torch.equal(shards[r].flatten(), got)


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cpu_worker(rank, world, port, kw, layout, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from fastest_flash_attention_b200.ring import ring_attention_forward
    g = torch.Generator().manual_seed(0)
    B, Hq, Hkv, S, D = 1, 4, 2, 24, 16
    q = torch.randn(B, Hq, S * world, D, generator=g)
    k = torch.randn(B, Hkv, S * world, D, generator=g)
    v = torch.randn(B, Hkv, S * world, D, generator=g)
    shard = _sharder(layout, rank, world, S)
    ks, vs = shard(k), shard(v)
    o, lse = ring_attention_forward(shard(q), ks, vs, attn_fn=ref_attn, return_lse=True, layout=layout, **kw)
    ro, rlse = _full(q, k, v, **kw)
    ok_o = torch.allclose(o, shard(ro), atol=1e-5, rtol=1e-4)
    ok_l = torch.allclose(lse, shard(rlse), atol=1e-5, rtol=1e-4)
    # the caller's K / V shards are left as they were
    ok_kv = torch.equal(ks, shard(k)) and torch.equal(vs, shard(v))
    out.put((rank, bool(ok_o), bool(ok_l and ok_kv)))
    dist.destroy_process_group()


@pytest.mark.parametrize("world,layout", [(2, "contiguous"), (3, "contiguous"), (3, "zigzag")])
@pytest.mark.parametrize("kw", [dict(causal=True), dict(causal=False), dict(causal=True, sliding_window=20),
                                dict(causal=True, softcap=5.0)])
def test_ring_gloo_cpu(world, layout, kw):
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_cpu_worker, args=(r, world, port, kw, layout, out)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(out.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(r[1] and r[2] for r in res), res


def _cpu_bwd_worker(rank, world, port, kw, layout, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from fastest_flash_attention_b200.ring import ring_attention_backward, ring_attention_forward
    g = torch.Generator().manual_seed(0)
    B, Hq, Hkv, S, D = 1, 4, 2, 24, 16
    q = torch.randn(B, Hq, S * world, D, generator=g).requires_grad_()
    k = torch.randn(B, Hkv, S * world, D, generator=g).requires_grad_()
    v = torch.randn(B, Hkv, S * world, D, generator=g).requires_grad_()
    dout = torch.randn(B, Hq, S * world, D, generator=g)
    ro, _ = _full(q, k, v, **kw)
    (ro * dout).sum().backward()
    shard = _sharder(layout, rank, world, S)
    qs, ks, vs = shard(q.detach()), shard(k.detach()), shard(v.detach())
    o, lse = ring_attention_forward(qs, ks, vs, attn_fn=ref_attn, return_lse=True, layout=layout, **kw)
    dq, dk, dv = ring_attention_backward(shard(dout), qs, ks, vs, o, lse, bwd_fn=ref_attn_bwd, layout=layout,
                                         **kw)
    errs = [float((a - shard(b)).abs().max()) for a, b in ((dq, q.grad), (dk, k.grad), (dv, v.grad))]
    out.put((rank, errs))
    dist.destroy_process_group()


@pytest.mark.parametrize("world,layout", [(2, "contiguous"), (3, "contiguous"), (3, "zigzag")])
@pytest.mark.parametrize("kw", [dict(causal=True), dict(causal=False), dict(causal=True, sliding_window=20),
                                dict(causal=True, softcap=5.0)])
def test_ring_backward_gloo_cpu(world, layout, kw):
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_cpu_bwd_worker, args=(r, world, port, kw, layout, out)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(out.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(e <= 1e-4 for r in res for e in r[1]), res


@pytest.mark.gpu
@pytest.mark.parametrize("W,kw,layout", [(4, dict(causal=True), "contiguous"), (3, dict(causal=False), "contiguous"),
                                         (4, dict(causal=True, sliding_window=300), "contiguous"),
                                         (2, dict(causal=True, softcap=20.0), "contiguous"),
                                         (4, dict(causal=True), "zigzag"),
                                         (3, dict(causal=True, sliding_window=300), "zigzag")])
def test_ring_arithmetic_gpu(W, kw, layout):
    from fastest_flash_attention_b200.ring import ring_attention_local
    torch.manual_seed(1)
    B, Hq, Hkv, S, D = 1, 8, 2, 256, 128
    q = torch.randn(B, Hq, S * W, D, device="cuda").to(torch.bfloat16)
    k = torch.randn(B, Hkv, S * W, D, device="cuda").to(torch.bfloat16)
    v = torch.randn(B, Hkv, S * W, D, device="cuda").to(torch.bfloat16)
    blocks = [(_sharder(layout, s, W, S)(k), _sharder(layout, s, W, S)(v)) for s in range(W)]
    ro, rlse = _full(q, k, v, **kw)
    for r in range(W):
        shard = _sharder(layout, r, W, S)
        o, lse = ring_attention_local(shard(q), blocks, r, layout=layout, **kw)
        assert (o - shard(ro)).abs().max().item() <= 2e-2, r
        assert (lse - shard(rlse)).abs().max().item() <= 1e-3, r


@pytest.mark.gpu
@pytest.mark.parametrize("W,kw,layout", [(4, dict(causal=True), "contiguous"), (3, dict(causal=False), "contiguous"),
                                         (4, dict(causal=True, sliding_window=300), "zigzag"),
                                         (2, dict(causal=True, softcap=20.0), "zigzag")])
def test_ring_backward_arithmetic_gpu(W, kw, layout):
    """The ring backward's arithmetic with the sm_100a kernels (W ranks
    emulated on one GPU) against fp32 full-sequence autograd: gradients within
    5e-2 of max|ref|."""
    from fastest_flash_attention_b200.ring import ring_attention_local, ring_attention_local_backward
    torch.manual_seed(2)
    B, Hq, Hkv, S, D = 1, 8, 2, 256, 128
    q = torch.randn(B, Hq, S * W, D, device="cuda").to(torch.bfloat16)
    k = torch.randn(B, Hkv, S * W, D, device="cuda").to(torch.bfloat16)
    v = torch.randn(B, Hkv, S * W, D, device="cuda").to(torch.bfloat16)
    dout = torch.randn(B, Hq, S * W, D, device="cuda").to(torch.bfloat16)
    qf, kf, vf = (t.float().requires_grad_() for t in (q, k, v))
    ro, _ = _full(qf, kf, vf, **kw)
    (ro * dout.float()).sum().backward()
    sh = [_sharder(layout, r, W, S) for r in range(W)]
    kvs = [(sh[r](k), sh[r](v)) for r in range(W)]
    qs = [sh[r](q) for r in range(W)]
    outs = [ring_attention_local(qs[r], kvs, r, layout=layout, **kw) for r in range(W)]
    dqs, dks, dvs = ring_attention_local_backward([sh[r](dout) for r in range(W)], qs, kvs,
                                                  [o.to(torch.bfloat16) for o, _ in outs], [l for _, l in outs],
                                                  layout=layout, **kw)
    for r in range(W):
        for got, ref in ((dqs[r], qf.grad), (dks[r], kf.grad), (dvs[r], vf.grad)):
            ref = sh[r](ref)
            assert (got.float() - ref).abs().max().item() <= 5e-2 * ref.abs().max().item(), r


def _gpu_worker(rank, world, port, out):
    # point-to-point only; NVLS stays off so a failing rank cannot leave
    # multicast-bound memory behind on the other GPU
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import torch.distributed as dist
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    from fastest_flash_attention_b200.ring import ring_attention_forward
    g = torch.Generator().manual_seed(0)
    B, Hq, Hkv, S, D = 1, 8, 2, 512, 128
    q = torch.randn(B, Hq, S * world, D, generator=g).to(torch.bfloat16)
    k = torch.randn(B, Hkv, S * world, D, generator=g).to(torch.bfloat16)
    v = torch.randn(B, Hkv, S * world, D, generator=g).to(torch.bfloat16)
    dev = torch.device("cuda", rank)
    shard = _sharder("zigzag", rank, world, S)
    o, lse = ring_attention_forward(shard(q).to(dev), shard(k).to(dev), shard(v).to(dev), causal=True,
                                    return_lse=True, layout="zigzag")
    ro, rlse = _full(q.to(dev), k.to(dev), v.to(dev), causal=True)
    eo = (o.float() - shard(ro)).abs().max().item()
    el = (lse - shard(rlse)).abs().max().item()
    # backward through autograd (ring_attention_func) against fp32 full-sequence autograd
    from fastest_flash_attention_b200.ring import ring_attention_func
    dout = torch.randn(B, Hq, S * world, D, generator=g).to(torch.bfloat16)
    qs, ks, vs = (shard(t).to(dev).requires_grad_() for t in (q, k, v))
    ring_attention_func(qs, ks, vs, causal=True, layout="zigzag").backward(shard(dout).to(dev))
    qf, kf, vf = (t.to(dev).float().requires_grad_() for t in (q, k, v))
    rof, _ = _full(qf, kf, vf, causal=True)
    (rof * dout.to(dev).float()).sum().backward()
    eg = max((a.grad.float() - shard(b.grad)).abs().max().item() / shard(b.grad).abs().max().item()
             for a, b in ((qs, qf), (ks, kf), (vs, vf)))
    out.put((rank, eo, el, eg))
    dist.destroy_process_group()


@pytest.mark.gpu
def test_ring_nccl_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_gpu_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(out.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for _, eo, el, eg in res:
        assert eo <= 2e-2 and el <= 1e-3 and eg <= 5e-2, res
