"""Benchmark of the attention hot path on B200.

Default workload (the configuration the headline metric is quoted on): GQA
prefill forward, bf16, B=4, Hq=32, Hkv=8, S=8192, D=128, causal, emitting O
and LSE.  A step = one forward over one batch of synthetic inputs (~N(0,1)
scaled by D^-1/4, seeded); inputs (403 MB) exceed the 126 MB L2, so no flush
is needed between steps.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs one process per GPU (torchrun); the one config-2 job is split by
its 32 (batch, kv-head) GQA groups across the ranks (strong scaling, no
collective on the data path) and rank 0 prints the whole-job throughput over
the max-over-ranks time.  N > 1 adds two lines: config 4 decode split by
request (greedy LPT on context length) and the sequence-sharded ring.

--impl reference times the reference's CPU algorithm (the numpy port in
oracle/, the reference being a Python package that cannot travel) on the
host cores, on a bounded sample of the same workload, and reports the same
metric.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "causal attention fwd TFLOP/s (GQA prefill bf16, B=4 Hq=32 Hkv=8 S=8192 D=128)"
UNIT = "TFLOP/s"
CFG = dict(B=4, Hq=32, Hkv=8, S=8192, D=128)
# --case small: same kernel, half the batch (192 MB of inputs, still above L2) for ncu captures
SMALL_CFG = dict(B=2, Hq=32, Hkv=8, S=8192, D=128)
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def causal_pairs(S: int) -> int:
    return S * (S + 1) // 2


def fwd_flops(B, Hq, S, D) -> float:
    # 2 GEMMs (QK^T and PV) of 2*D flops per unmasked (query, key) pair
    return 4.0 * D * causal_pairs(S) * B * Hq


def workload_config(n_gpus: int) -> dict:
    groups = CFG["B"] * CFG["Hkv"]
    return {
        "workload": "GQA causal prefill forward (O + LSE)",
        "batch": CFG["B"], "q_heads": CFG["Hq"], "kv_heads": CFG["Hkv"], "seq_len": CFG["S"],
        "head_dim": CFG["D"], "causal": True,
        "parallelism": f"{groups} (batch, kv-head) GQA groups split over {n_gpus} GPU(s), "
                       f"{groups // n_gpus}-{-(-groups // n_gpus)} per GPU, no collective on the data path",
        "l2": "inputs 403 MB per GPU > 126 MB L2, no flush needed",
        "flop_convention": "4*D*causal_pairs*B*Hq (exact unmasked pairs)",
    }


def load_peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


class ClockSampler:
    """Samples nvidia-smi clocks and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
            time.sleep(0.3)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        mhz, max_mhz, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                mhz.append(float(parts[1]))
                max_mhz = float(parts[2])
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(mhz) if mhz else None, "sm_max_mhz": max_mhz,
                "reasons": sorted(reasons), "samples": len(mhz)}


def dist_init():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import torch.distributed as dist
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if torch.cuda.is_available():
            torch.cuda.set_device(local)
        dist.init_process_group(backend=backend)
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda" if torch.cuda.is_available() else "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def make_inputs(device, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    B, Hq, Hkv, S, D = CFG["B"], CFG["Hq"], CFG["Hkv"], CFG["S"], CFG["D"]
    sc = D ** -0.25
    q = (torch.randn(B, Hq, S, D, generator=g) * sc).to(torch.bfloat16)
    k = (torch.randn(B, Hkv, S, D, generator=g) * sc).to(torch.bfloat16)
    v = torch.randn(B, Hkv, S, D, generator=g).to(torch.bfloat16)
    return q, k, v


# ----------------------------------------------------------------------------
# CPU arm: the reference algorithm (numpy port) on a bounded sample
# ----------------------------------------------------------------------------

def cpu_reference_sample(q, k, v, heads: int = 4, s_len: int = 8192, block: int = 128):
    """Time the oracle forward on `heads` query heads of batch 0 with the
    first `s_len` positions (causal), returning (TFLOP/s, seconds, sample)."""
    from oracle import attention_oracle as O
    D = q.shape[-1]
    g = CFG["Hq"] // CFG["Hkv"]
    qs = q[:1, :heads, :s_len].float().numpy()
    ks = np.repeat(k[:1, :max(1, heads // g), :s_len].float().numpy(), g, axis=1)[:, :heads]
    vs = np.repeat(v[:1, :max(1, heads // g), :s_len].float().numpy(), g, axis=1)[:, :heads]
    t0 = time.perf_counter()
    O.flash_forward(qs, ks, vs, scale=1.0 / math.sqrt(D), causal=True, block_q=block, block_kv=block,
                    return_lse=True)
    dt = time.perf_counter() - t0
    fl = fwd_flops(1, heads, s_len, D)
    sample = f"batch 0, {heads} query head(s), first {s_len} positions, causal, block {block} (numpy fp32)"
    return fl / dt / 1e12, dt, sample


def run_reference(args, world, rank):
    if rank != 0:
        return
    q, k, v = make_inputs("cpu")
    cores = os.cpu_count() or 1
    vals = []
    sample = ""
    for i in range(args.warmup + args.steps):
        tf, dt, sample = cpu_reference_sample(q, k, v, heads=8)
        if i >= args.warmup:
            vals.append(tf)
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1)*D^-1/4, bf16-rounded)",
        "config": workload_config(args.gpus),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------
# GPU arm
# ----------------------------------------------------------------------------

def _time(fn, iters, dev):
    for _ in range(3):
        fn()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize(dev)
    return e0.elapsed_time(e1) / iters


def _time_flushed(fn, iters, dev):
    """Mean device time of fn with L2 flushed (a 512 MB write) before every
    call.  All calls are enqueued before one synchronize, so host-side work of
    the wrapper overlaps the previous flush instead of sitting between the
    events."""
    flush = torch.empty(128 * 1024 * 1024, dtype=torch.float32, device=dev)
    for _ in range(3):
        fn()
    torch.cuda.synchronize(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
    for e0, e1 in ev:
        flush.zero_()
        e0.record()
        fn()
        e1.record()
    torch.cuda.synchronize(dev)
    return sum(e0.elapsed_time(e1) for e0, e1 in ev) / iters


def paged_decode_inputs(dev, seed=0):
    """Config 4: 64 requests, ctx ~ U[512, 32768], page 16, Hq 32 / Hkv 8, D 128,
    pool pages shuffled by the seed (permuted block table)."""
    g = torch.Generator().manual_seed(seed)
    R, Hq, Hkv, D, PS = 64, 32, 8, 128, 16
    lens = torch.randint(512, 32769, (R,), generator=g)
    npg = (lens + PS - 1) // PS
    P = int(npg.sum())
    perm = torch.randperm(P, generator=g).to(torch.int32)
    bt = torch.zeros(R, int(npg.max()), dtype=torch.int32)
    off = 0
    for r in range(R):
        bt[r, :npg[r]] = perm[off:off + npg[r]]
        off += int(npg[r])
    kp = torch.randn(P, Hkv, PS, D, device=dev, dtype=torch.bfloat16)
    vp = torch.randn(P, Hkv, PS, D, device=dev, dtype=torch.bfloat16)
    q = torch.randn(R, Hq, D, device=dev, dtype=torch.bfloat16)
    return q, kp, vp, bt.to(dev), lens.to(torch.int32).to(dev), int(lens.sum()), int(lens.max())


def secondary_lines(dev, peaks, peak_src):
    """The other kernels of the path on their BASELINE configs, timed with CUDA
    events (inputs resident in HBM; each workload exceeds L2)."""
    from fastest_flash_attention_b200.attention import flash_bwd, flash_fwd
    from fastest_flash_attention_b200 import paged_decode
    from fastest_flash_attention_b200.mla import mla_decode
    pk = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    out = {}
    # config 3: training fwd+bwd, causal + window 1024 + softcap 30, deterministic
    B, H, S, D = 8, 16, 4096, 128
    g = torch.Generator(device=dev).manual_seed(3)
    q, k, v, do = (torch.randn(B, H, S, D, device=dev, generator=g).to(torch.bfloat16) for _ in range(4))
    sc = 1 / math.sqrt(D)
    o, lse = flash_fwd(q, k, v, scale=sc, causal=True, window=1024, softcap=30.0)
    f_ms = _time(lambda: flash_fwd(q, k, v, scale=sc, causal=True, window=1024, softcap=30.0), 10, dev)
    b_ms = _time(lambda: flash_bwd(do, q, k, v, o, lse, scale=sc, causal=True, window=1024, softcap=30.0), 10, dev)
    pairs = 1024 * 1025 // 2 + (S - 1024) * 1024
    ff = 4.0 * D * pairs * B * H
    out["train_fwd_bwd_cfg3"] = {
        "workload": "B=8 H=16 S=4096 D=128 causal+window1024+softcap30, deterministic bwd",
        "fwd_ms": f_ms, "bwd_ms": b_ms, "fwd_tflops": ff / f_ms / 1e9, "bwd_tflops": 2.5 * ff / b_ms / 1e9,
        "train_tokens_per_s": B * S / ((f_ms + b_ms) * 1e-3),
        "fwd_bwd_tflops": 3.5 * ff / (f_ms + b_ms) / 1e9,
        "frac_of_peak": 3.5 * ff / (f_ms + b_ms) / 1e9 / pk, "peak": f"{pk} TFLOP/s ({peak_src} bf16)"}
    del q, k, v, do, o, lse
    # config 1 (the reference's CPU-runnable case): fp32 [2, 8, 1024, 64] causal fwd+bwd, computed
    # in fp32 on the CUDA cores (no fp32 tensor-core operands); L2-resident (25 MB of inputs)
    g = torch.Generator(device=dev).manual_seed(1)
    q, k, v, do = (torch.randn(2, 8, 1024, 64, device=dev, generator=g) for _ in range(4))
    o, lse = flash_fwd(q, k, v, scale=0.125, causal=True)
    f1 = _time(lambda: flash_fwd(q, k, v, scale=0.125, causal=True), 20, dev)
    b1 = _time(lambda: flash_bwd(do, q, k, v, o, lse, scale=0.125, causal=True), 20, dev)
    ff1 = 4.0 * 64 * causal_pairs(1024) * 2 * 8
    out["fp32_fwd_bwd_cfg1"] = {
        "workload": "config 1: fp32 B=2 H=8 S=1024 D=64 causal, fp32 arithmetic (CUDA cores), L2-resident",
        "fwd_ms": f1, "bwd_ms": b1, "fwd_tflops": ff1 / f1 / 1e9, "bwd_tflops": 2.5 * ff1 / b1 / 1e9,
        "fwd_bwd_tflops": 3.5 * ff1 / (f1 + b1) / 1e9}
    del q, k, v, do, o, lse
    # config 4: paged decode
    q, kp, vp, bt, lens, tot, mx = paged_decode_inputs(dev)
    d_ms = _time(lambda: paged_decode(q, kp, vp, bt, lens, max_ctx=mx), 20, dev)
    byts = tot * 8 * 128 * 2 * 2 + q.numel() * 2 * 2
    out["paged_decode_cfg4"] = {
        "workload": "64 req, ctx U[512,32768], page 16, Hq 32 / Hkv 8, D 128, bf16, permuted block table",
        "ms": d_ms, "gbs": byts / d_ms / 1e6, "frac_of_hbm": byts / d_ms / 1e6 / hbm,
        "requests_per_s": 64 / d_ms * 1e3, "bytes": byts, "peak": f"{hbm} GB/s ({peak_src})"}
    del q, kp, vp
    # config 5 prefill: the MLA module's attention at (qk 192, v 128), B=16 H=32 S=4096 causal
    B5, H5, S5 = 16, 32, 4096
    g = torch.Generator(device=dev).manual_seed(5)
    q = torch.randn(B5, H5, S5, 192, device=dev, generator=g).to(torch.bfloat16)
    k = torch.randn(B5, H5, S5, 192, device=dev, generator=g).to(torch.bfloat16)
    v = torch.randn(B5, H5, S5, 128, device=dev, generator=g).to(torch.bfloat16)
    p_ms = _time(lambda: flash_fwd(q, k, v, scale=192 ** -0.5, causal=True), 10, dev)
    pf = 2.0 * (192 + 128) * causal_pairs(S5) * B5 * H5
    out["mla_prefill_cfg5"] = {
        "workload": "config 5 prefill attention: B=16 H=32 S=4096 causal, qk 192 / v 128 (unpadded V), bf16",
        "ms": p_ms, "tflops": pf / p_ms / 1e9, "frac_of_peak": pf / p_ms / 1e9 / pk,
        "flops": pf, "peak": f"{pk} TFLOP/s ({peak_src} bf16)"}
    del q, k, v
    # config 5: MLA absorbed decode step, B=16 at context 4096 (latent 512 + rope 64, 32 heads)
    R, L, PS = 16, 4096, 64
    cache = torch.randn(R * L // PS, PS, 576, device=dev, dtype=torch.bfloat16)
    btm = torch.arange(R * L // PS, dtype=torch.int32, device=dev).view(R, L // PS)
    lm = torch.full((R,), L, dtype=torch.int32, device=dev)
    qm = torch.randn(R, 32, 576, device=dev, dtype=torch.bfloat16)
    m_ms = _time_flushed(lambda: mla_decode(qm, cache, btm, lm, scale=1 / math.sqrt(192), max_ctx=L), 20, dev)
    mb = R * L * 576 * 2
    out["mla_decode_cfg5"] = {"workload": "16 req x ctx 4096, latent 512 + rope 64, 32 heads, bf16", "ms": m_ms,
                              "gbs": mb / m_ms / 1e6, "frac_of_hbm": mb / m_ms / 1e6 / hbm,
                              "l2": "cache (75 MB) fits L2: flushed before every timed call",
                              "kernels": "ffa_mla_decode_tc_kernel + ffa_mla_merge_kernel"}
    del cache, btm, lm, qm
    # config 5 decode step end to end through MLADecoder.step (the Python
    # included): one GEMM for the input projections, latent append + k RoPE,
    # query absorption + q RoPE, the paged latent decode, value absorption,
    # o_proj; 16 requests at context 4096 (the cache is filled directly).
    from fastest_flash_attention_b200 import FastestFlashMLA, MLADecoder
    torch.manual_seed(5)
    mod = FastestFlashMLA(hidden_size=4096, num_heads=32, head_dim=128, latent_dim=512, rope_dim=64).to(dev).eval()
    for prm in mod.parameters():
        torch.nn.init.normal_(prm, std=0.02)
    mod = mod.to(torch.bfloat16)
    dec = MLADecoder(mod, max_pages=R * (L + 64) // PS + R, page_size=PS)
    rows = dec.cache.pages.view(-1, 576)
    for sid in range(R):
        slots = torch.tensor(dec.cache._slots(sid, L), dtype=torch.long, device=dev)
        rows[slots] = torch.randn(L, 576, device=dev, dtype=torch.bfloat16)
    x = torch.randn(R, 1, 4096, device=dev, dtype=torch.bfloat16)
    for _ in range(3):
        dec.step(x, list(range(R)))
    torch.cuda.synchronize(dev)
    n_steps = 20
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n_steps):
        dec.step(x, list(range(R)))
    e1.record()
    torch.cuda.synchronize(dev)
    st_ms = e0.elapsed_time(e1) / n_steps
    out["mla_decode_step_cfg5"] = {
        "workload": "MLADecoder.step, 16 requests, context 4096 -> 4116, hidden 4096, 32 heads, latent 512 + rope 64, "
                    "bf16 weights N(0, 0.02)", "ms_per_step": st_ms, "tokens_per_s": R / st_ms * 1e3,
        "timing": "CUDA events around 20 consecutive steps, host work included (the cache grows by a token per step)"}
    # the same step replayed from a CUDA graph (MLADecoder.step_graphed): one
    # pinned metadata copy, one input copy and one graph launch per step
    for _ in range(3):
        dec.step_graphed(x, list(range(R)))
    torch.cuda.synchronize(dev)
    e0.record()
    for _ in range(n_steps):
        dec.step_graphed(x, list(range(R)))
    e1.record()
    torch.cuda.synchronize(dev)
    sg_ms = e0.elapsed_time(e1) / n_steps
    out["mla_decode_step_graphed_cfg5"] = {
        "workload": "MLADecoder.step_graphed, same model and cache as mla_decode_step_cfg5 (context 4119 -> 4142)",
        "ms_per_step": sg_ms, "tokens_per_s": R / sg_ms * 1e3,
        "timing": "CUDA events around 20 consecutive steps, host work included (allocator, metadata copy, replay)"}
    del dec, mod
    return out


def rank_blocks(world: int, rank: int):
    """This rank's (batch x kv-head) rectangles of config 2's GQA groups."""
    from fastest_flash_attention_b200.partition import gqa_group_blocks
    return gqa_group_blocks(CFG["B"], CFG["Hkv"], rank, world)


def block_flops(blocks) -> float:
    G = CFG["Hq"] // CFG["Hkv"]
    return sum(fwd_flops(b1 - b0, (h1 - h0) * G, CFG["S"], CFG["D"]) for b0, b1, h0, h1 in blocks)


def e2e_chunks(blocks, kv_chunk: int):
    """(batch element, kv-head range) chunks of this rank's groups for the e2e
    pipeline: kv_chunk heads each, except that the first and the last chunk
    are cut down to single kv heads.  The first forward can start only once
    its inputs have crossed PCIe, and the last chunk's forward and output copy
    run after all inputs have arrived: small end chunks shorten both exposed
    ends while the middle keeps chunks large enough to hide the per-call host
    work behind the copies."""
    base = [(b, g0, min(g0 + kv_chunk, h1)) for b0, b1, h0, h1 in blocks for b in range(b0, b1)
            for g0 in range(h0, h1, kv_chunk)]

    def split(c, first):
        b, g0, g1 = c
        n = g1 - g0
        if n <= 2:
            return [(b, g, g + 1) for g in range(g0, g1)]
        if first:  # 1, 1, then the rest
            return [(b, g0, g0 + 1), (b, g0 + 1, g0 + 2), (b, g0 + 2, g1)]
        return [(b, g0, g1 - 2), (b, g1 - 2, g1 - 1), (b, g1 - 1, g1)]

    if len(base) == 1:
        return split(base[0], True)
    return split(base[0], True) + base[1:-1] + split(base[-1], False)


def pcie_ceiling(dev, qp, q_d, o_host, stream, h2d, d2h):
    """Pinned-host copy bandwidth of this GPU's link, measured with the e2e
    leg's own buffers: H2D alone, D2H alone, and both at once on two streams.
    The e2e step cannot beat moving its bytes: ceiling = max(h2d / H2D rate,
    d2h / D2H rate) with the directions overlapped (the step's pipeline), and
    the slower of that and the sum if the link cannot run both at full rate."""
    nb = min(qp.numel(), o_host.numel())
    src_h, dst_d = qp.view(-1)[:nb], q_d.view(-1)[:nb]
    dst_h = o_host.view(-1)[:nb]
    byts = nb * 2
    s2 = torch.cuda.Stream(dev)

    def timed(fn, reps=5):
        fn()
        torch.cuda.synchronize(dev)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(reps):
            fn()
        b.record(stream)
        torch.cuda.synchronize(dev)
        return a.elapsed_time(b) / reps

    t_h2d = timed(lambda: dst_d.copy_(src_h, non_blocking=True))
    t_d2h = timed(lambda: dst_h.copy_(dst_d, non_blocking=True))

    def both():
        s2.wait_stream(stream)
        dst_d.copy_(src_h, non_blocking=True)
        with torch.cuda.stream(s2):
            dst_h.copy_(q_d.view(-1)[:nb], non_blocking=True)
        stream.wait_stream(s2)
    t_both = timed(both)
    h2d_gbs, d2h_gbs = byts / t_h2d / 1e6, byts / t_d2h / 1e6
    overlapped = max(h2d / (h2d_gbs * 1e6), d2h / (d2h_gbs * 1e6))
    # both directions together: bytes moved per ms when each direction copies `byts`
    both_gbs = 2 * byts / t_both / 1e6
    ceiling = max(overlapped, (h2d + d2h) / (both_gbs * 1e6))
    return {"h2d_gbs": h2d_gbs, "d2h_gbs": d2h_gbs, "bidirectional_gbs": both_gbs, "ceiling_ms": ceiling,
            "how": f"{byts / 1e6:.0f} MB pinned copies with the e2e buffers, CUDA events, mean of 5"}


def multi_gpu_lines(dev, world, rank, peaks, peak_src):
    """Lines only a multi-GPU run has, every rank taking part: config 4 decode
    split by request (greedy LPT on context length) and the sequence-sharded
    ring (zigzag, forward and backward) on one long causal sequence.  Times
    are CUDA events, max over ranks; values are whole-job aggregates."""
    from fastest_flash_attention_b200 import paged_decode
    from fastest_flash_attention_b200.partition import lpt_partition
    from fastest_flash_attention_b200.ring import ring_attention_backward, ring_attention_forward, zigzag_shard
    hbm = float(peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"]))
    out = {}
    q, kp, vp, bt, lens, tot, mx = paged_decode_inputs(dev)
    lens_h = lens.cpu().tolist()
    mine = lpt_partition([float(x) for x in lens_h], world)[rank]
    idx = torch.tensor(mine, dtype=torch.long, device=dev)
    q_r, bt_r, lens_r = q[idx].contiguous(), bt[idx].contiguous(), lens[idx].contiguous()
    mx_r = max(lens_h[i] for i in mine) if mine else 0
    if mine:
        fn = lambda: paged_decode(q_r, kp, vp, bt_r, lens_r, max_ctx=mx_r)  # noqa: E731
        ms_local = _time(fn, 20, dev)
    else:
        ms_local = 0.0
    ms = max_over_ranks(ms_local, world)
    byts = tot * 8 * 128 * 2 * 2 + q.numel() * 2 * 2
    out["paged_decode_cfg4_split"] = {
        "workload": "config 4 (64 req, ctx U[512,32768], page 16, Hq 32/Hkv 8, D 128, bf16) split by request, "
                    "greedy LPT on context length", "ms": ms, "gbs": byts / ms / 1e6,
        "frac_of_hbm_per_gpu": byts / ms / 1e6 / hbm / world, "requests_this_rank": len(mine),
        "ctx_this_rank": int(sum(lens_h[i] for i in mine))}
    del q, kp, vp, bt, lens, q_r, bt_r, lens_r
    torch.cuda.empty_cache()
    # ring: B=1 Hq=32 Hkv=8 D=128, 65536 causal positions, zigzag shards
    S_tot, Hq, Hkv, D = 65536, 32, 8, 128
    g = torch.Generator().manual_seed(11)
    full = [torch.randn(1, h, S_tot, D, generator=g).to(torch.bfloat16) for h in (Hq, Hkv, Hkv, Hq)]
    qs, ks, vs, dos = (zigzag_shard(t, rank, world).contiguous().to(dev) for t in full)
    del full
    sc = 1 / math.sqrt(D)
    fwd = lambda: ring_attention_forward(qs, ks, vs, scale=sc, causal=True, return_lse=True,  # noqa: E731
                                         layout="zigzag")
    o, lse = fwd()
    bwd = lambda: ring_attention_backward(dos, qs, ks, vs, o, lse, scale=sc, causal=True,  # noqa: E731
                                          layout="zigzag")
    res = {}
    for name, fn in (("fwd", fwd), ("bwd", bwd)):
        fn()
        torch.cuda.synchronize(dev)
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(3):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        res[name] = max_over_ranks(e0.elapsed_time(e1) / 3, world)
    ff = fwd_flops(1, Hq, S_tot, D)
    out["ring_cp_zigzag"] = {
        "workload": f"sequence-sharded ring, B=1 Hq=32 Hkv=8 D=128, {S_tot} causal positions, zigzag over "
                    f"{world} GPUs (NCCL p2p K/V exchange)", "fwd_ms": res["fwd"], "bwd_ms": res["bwd"],
        "fwd_tflops": ff / res["fwd"] / 1e9, "bwd_tflops": 2.5 * ff / res["bwd"] / 1e9}
    return out


def run_ours(args, world, rank, local):
    from fastest_flash_attention_b200 import fastest_flash_attn_forward
    from fastest_flash_attention_b200.attention import flash_fwd
    from fastest_flash_attention_b200 import _lib

    dev = torch.device("cuda", local)
    B, Hq, Hkv, S, D = CFG["B"], CFG["Hq"], CFG["Hkv"], CFG["S"], CFG["D"]
    G = Hq // Hkv
    scale = 1.0 / math.sqrt(D)
    # Every rank draws the same full batch and keeps its GQA groups: strong
    # scaling of one fixed config-2 job, no collective on the data path.
    q_h, k_h, v_h = make_inputs("cpu", seed=0)
    blocks = rank_blocks(world, rank)
    parts = [(q_h[b0:b1, h0 * G:h1 * G].contiguous().to(dev), k_h[b0:b1, h0:h1].contiguous().to(dev),
              v_h[b0:b1, h0:h1].contiguous().to(dev)) for b0, b1, h0, h1 in blocks]
    flops = fwd_flops(B, Hq, S, D)            # the whole job
    flops_rank = block_flops(blocks)          # this rank's launches
    stream = torch.cuda.current_stream(dev)

    def step():
        for q, k, v in parts:
            flash_fwd(q, k, v, scale=scale, causal=True)

    # ---- device-resident timing (value + roofline) ----
    # The clock sampler starts first and the warm-up steps run inside it, so
    # the GPU goes from warm-up to the timed steps with no idle second in
    # between (an idle GPU drops its clocks, and the first timed steps would
    # pay the ramp).  A short device-side sleep after the barrier lets the host
    # enqueue the timed steps ahead of the GPU, so the events measure the
    # kernels and not the host's first launch.
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        for _ in range(args.warmup):
            step()
        torch.cuda.synchronize(dev)
        _lib.check_device_errors(dev)
        barrier(world)
        torch.cuda.synchronize(dev)
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        torch.cuda._sleep(1_000_000)  # ~0.5 ms of device time, outside the timed region
        t0.record(stream)
        for i in range(args.steps):
            starts[i].record(stream)
            step()
            ends[i].record(stream)
        t1.record(stream)
        torch.cuda.synchronize(dev)
    barrier(world)
    _lib.check_device_errors(dev)
    ms_local = t0.elapsed_time(t1) / args.steps
    launch_ms = statistics.mean(s.elapsed_time(e) for s, e in zip(starts, ends))
    ms = max_over_ranks(ms_local, world)
    value = flops / (ms * 1e-3) / 1e12

    if args.kernel_only:
        if rank == 0:
            print(json.dumps({"metric": METRIC, "value": value, "unit": UNIT, "ms_per_step": ms,
                              "config": workload_config(world), "note": "kernel-only run (--kernel-only)"}))
        return

    # ---- end to end through the public API with host buffers ----
    qp, kp, vp = q_h.pin_memory(), k_h.pin_memory(), v_h.pin_memory()
    o_host = torch.empty(q_h.shape, dtype=torch.bfloat16).pin_memory()
    lse_host = torch.empty((B, Hq, S, 1), dtype=torch.float32).pin_memory()

    # Chunks of one batch element and half its kv heads (each kv head with its
    # group of query heads: complete GQA attention problems; the first and
    # last chunks smaller, see e2e_chunks), restricted to this rank's groups,
    # on three streams: the H2D copy of chunk c+1 and the D2H copy of chunk c-1
    # overlap the forward of chunk c, so the step costs about the PCIe time of
    # the inputs plus a small chunk.  (Uniformly smaller chunks were measured
    # slower: the host-side call overhead then no longer hides behind the
    # copies.)  Device input buffers are allocated once, outside the timed
    # region; every byte of input and output still crosses PCIe inside it.
    s_h2d, s_d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    q_d, k_d, v_d = (torch.empty(t.shape, dtype=t.dtype, device=dev) for t in (qp, kp, vp))
    chunks = e2e_chunks(blocks, max(1, Hkv // 2))
    h2d = sum((qp[b, g0 * G:g1 * G].numel() + 2 * kp[b, g0:g1].numel()) * 2 for b, g0, g1 in chunks)
    d2h = sum(o_host[b, g0 * G:g1 * G].numel() * 2 + lse_host[b, g0 * G:g1 * G].numel() * 4 for b, g0, g1 in chunks)

    def e2e_step():
        s_h2d.wait_stream(stream)
        s_d2h.wait_stream(stream)
        for b, g0, g1 in chunks:
            hk = slice(g0, g1)
            hq = slice(g0 * G, g1 * G)
            with torch.cuda.stream(s_h2d):
                q_d[b, hq].copy_(qp[b, hq], non_blocking=True)
                k_d[b, hk].copy_(kp[b, hk], non_blocking=True)
                v_d[b, hk].copy_(vp[b, hk], non_blocking=True)
            stream.wait_stream(s_h2d)
            o, lse = fastest_flash_attn_forward(q_d[b:b + 1, hq], k_d[b:b + 1, hk], v_d[b:b + 1, hk],
                                                causal=True, return_lse=True)
            s_d2h.wait_stream(stream)
            with torch.cuda.stream(s_d2h):
                o.record_stream(s_d2h)
                lse.record_stream(s_d2h)
                o_host[b, hq].copy_(o[0], non_blocking=True)
                lse_host[b, hq].copy_(lse[0], non_blocking=True)
        stream.wait_stream(s_d2h)

    e2e_steps = max(3, min(args.steps, 10))
    for _ in range(2):
        e2e_step()
    torch.cuda.synchronize(dev)
    barrier(world)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps, world)
    e2e_val = flops / (e2e_ms * 1e-3) / 1e12
    _lib.check_device_errors(dev)
    link = pcie_ceiling(dev, qp, q_d, o_host, stream, h2d, d2h)

    peaks, peak_src = load_peaks()
    del parts, q_d, k_d, v_d
    torch.cuda.empty_cache()
    multi = multi_gpu_lines(dev, world, rank, peaks, peak_src) if world > 1 and not args.no_secondary else None
    if rank != 0:
        return
    peak = float(peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]))
    achieved = flops_rank / (launch_ms * 1e-3) / 1e12
    traffic = None
    tf = ROOT / "profiles" / "fwd_gqa_prefill_traffic.json"
    if tf.exists() and world == 1:
        traffic = json.loads(tf.read_text()).get("bytes_per_launch")
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1)*D^-1/4)",
        "tokens_per_s": B * S / (ms * 1e-3), "config": workload_config(world),
        "e2e": {"value": e2e_val, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": e2e_ms, "bytes_are": "rank 0's copies (every rank moves its own groups' share)",
                "link": link,
                "frac_of_link_ceiling": (link["ceiling_ms"] / e2e_ms) if link.get("ceiling_ms") else None,
                "api": "fastest_flash_attn_forward(causal=True, return_lse=True) per (batch element, half its kv "
                       "heads with their query-head groups); H2D, forward and D2H pipelined on three streams"},
        "gpu_launches": args.steps * len(blocks),
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "peak_source": f"{peak_src} bf16_tflops (burst)", "kernel": "ffa_fwd_kernel<bf16,128>",
                     "algorithmic_flops_per_launch": flops_rank / max(1, len(blocks)),
                     "note": "rank 0's launches"},
        "clocks": clk.summary(),
    }
    if not args.no_secondary:
        line["secondary"] = secondary_lines(dev, peaks, peak_src)
        if multi:
            line["secondary"].update(multi)
    if world == 1:
        # about 10-15 s of CPU work: 16 query heads (half of batch element 0), 3 runs
        runs = [cpu_reference_sample(q_h, k_h, v_h, heads=16) for _ in range(3)]
        tfc = statistics.median(r[0] for r in runs)
        line["cpu_baseline"] = {"value": tfc, "unit": UNIT, "cores": os.cpu_count() or 1, "kind": "port",
                                "sample": runs[0][2] + ", median of 3",
                                "seconds": sum(r[1] for r in runs)}
    print(json.dumps(line), flush=True)


def run_profile(args):
    """Capture-sized cases (inputs above L2, a few GB at most) for ncu."""
    from fastest_flash_attention_b200.attention import flash_bwd, flash_fwd
    from fastest_flash_attention_b200 import paged_decode
    from fastest_flash_attention_b200.mla import mla_decode
    dev = torch.device("cuda", 0)
    n = args.warmup + args.steps
    if args.profile == "bwd":
        B, H, S, D = 2, 16, 4096, 128
        q, k, v, do = (torch.randn(B, H, S, D, device=dev).to(torch.bfloat16) for _ in range(4))
        o, lse = flash_fwd(q, k, v, scale=D ** -0.5, causal=True, window=1024, softcap=30.0)
        for _ in range(n):
            flash_bwd(do, q, k, v, o, lse, scale=D ** -0.5, causal=True, window=1024, softcap=30.0)
    elif args.profile == "prefill192":
        # config 5 prefill attention at (qk 192, v 128), B=4 (inputs 540 MB > L2; 2048 CTAs, the
        # L2-grouped CTA order as at B=16)
        q = torch.randn(4, 32, 4096, 192, device=dev).to(torch.bfloat16)
        k = torch.randn(4, 32, 4096, 192, device=dev).to(torch.bfloat16)
        v = torch.randn(4, 32, 4096, 128, device=dev).to(torch.bfloat16)
        for _ in range(n):
            flash_fwd(q, k, v, scale=192 ** -0.5, causal=True)
    elif args.profile == "fp32":
        # config 1: fp32 [2, 8, 1024, 64] causal forward + backward (CUDA-core kernels)
        q, k, v, do = (torch.randn(2, 8, 1024, 64, device=dev) for _ in range(4))
        for _ in range(n):
            o, lse = flash_fwd(q, k, v, scale=0.125, causal=True)
            flash_bwd(do, q, k, v, o, lse, scale=0.125, causal=True)
    elif args.profile == "decode":
        q, kp, vp, bt, lens, tot, mx = paged_decode_inputs(dev)
        for _ in range(n):
            paged_decode(q, kp, vp, bt, lens, max_ctx=mx)
    else:
        R, L, PS = 16, 4096, 64
        cache = torch.randn(R * L // PS, PS, 576, device=dev, dtype=torch.bfloat16)
        bt = torch.arange(R * L // PS, dtype=torch.int32, device=dev).view(R, L // PS)
        lens = torch.full((R,), L, dtype=torch.int32, device=dev)
        qm = torch.randn(R, 32, 576, device=dev, dtype=torch.bfloat16)
        for _ in range(n):
            mla_decode(qm, cache, bt, lens, scale=192 ** -0.5, max_ctx=L)
    torch.cuda.synchronize()
    print(json.dumps({"profile": args.profile, "launches": n}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--case", choices=["full", "small"], default="full")
    ap.add_argument("--kernel-only", action="store_true", help="skip the e2e and CPU legs (profiling runs)")
    ap.add_argument("--profile", choices=["bwd", "decode", "mla", "fp32", "prefill192"], default=None,
                    help="run only that kernel family a few times on a capture-sized case (for ncu)")
    ap.add_argument("--no-secondary", action="store_true", help="skip the other kernels' lines")
    args = ap.parse_args()
    if args.case == "small":
        CFG.update(SMALL_CFG)
    if args.profile:
        run_profile(args)
        return
    args.warmup = max(3, args.warmup)
    world, rank, local = dist_init()
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        else:
            run_ours(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
