"""Generate the golden fixtures in this directory by running the reference.

Usage:  python tests/golden/make_golden.py --reference <path to the
MindIntels/fastest_flash_attention source tree>

The reference is a pure-Python package; it is imported from its source tree
(through a temporary directory holding a symlink named
``fastest_flash_attention``), run on CPU with fixed numpy seeds, and every
input and output is written to ``<case>.npz``.  Inputs are rounded to bf16
values (stored as fp32) so the same numbers can be fed to the bf16 GPU
kernels.  The fixtures, not the reference, travel with the repository.
"""
from __future__ import annotations

import argparse
import os
import sys
import tempfile
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def bf16_vals(rng: np.random.Generator, *shape, scale: float = 1.0) -> np.ndarray:
    x = (rng.standard_normal(shape) * scale).astype(np.float32)
    return torch.from_numpy(x).to(torch.bfloat16).float().numpy()


def T(x: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x))


def N(x) -> np.ndarray:
    return x.detach().float().numpy() if isinstance(x, torch.Tensor) else np.asarray(x)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--out", default=str(HERE))
    args = ap.parse_args()

    tmp = tempfile.mkdtemp()
    os.symlink(os.path.abspath(args.reference), os.path.join(tmp, "fastest_flash_attention"))
    sys.path.insert(0, tmp)
    import fastest_flash_attention as ref  # noqa: E402
    from fastest_flash_attention.kernels import cpu_reference, cpu_fa4  # noqa: E402
    from fastest_flash_attention.ops import block_sparse  # noqa: E402

    out = Path(args.out)
    cases: dict[str, dict] = {}
    rng = np.random.default_rng(1234)

    # ---- base forward (cpu_reference.flash_attn_cpu_forward via the dispatch) ----
    def fwd_case(name, B, Hq, Hkv, Sq, Skv, D, **kw):
        q = bf16_vals(rng, B, Hq, Sq, D)
        k = bf16_vals(rng, B, Hkv, Skv, D)
        v = bf16_vals(rng, B, Hkv, Skv, D)
        extra = {}
        call = dict(kw)
        if "block_mask" in call:
            extra["block_mask"] = call["block_mask"].astype(np.uint8)
            call["block_mask"] = T(call["block_mask"])
        if Hq != Hkv:
            call["num_kv_heads"] = Hkv
        o, lse = ref.fastest_flash_attn_forward(T(q), T(k), T(v), return_lse=True, **call)
        params = {k_: v_ for k_, v_ in kw.items() if k_ != "block_mask"}
        cases[name] = dict(q=q, k=k, v=v, o=N(o), lse=N(lse), **extra,
                           params=np.array(repr(params)))

    fwd_case("fwd_basic_d16", 2, 4, 4, 24, 24, 16, block_size=8)
    fwd_case("fwd_causal_d64", 1, 2, 2, 200, 200, 64, causal=True, block_size=64)
    fwd_case("fwd_causal_d128_ragged", 1, 2, 2, 130, 130, 128, causal=True, block_size=32)
    fwd_case("fwd_window_d64", 1, 2, 2, 160, 160, 64, causal=True, sliding_window=40, block_size=16)
    fwd_case("fwd_softcap_d64", 1, 2, 2, 96, 96, 64, causal=True, softcap=5.0, block_size=32)
    fwd_case("fwd_gqa_d128", 1, 4, 2, 150, 150, 128, causal=True, block_size=64)
    fwd_case("fwd_noncausal_sq_ne_skv_d64", 1, 2, 2, 40, 170, 64, block_size=32)
    fwd_case("fwd_two_pass_d64", 1, 2, 2, 100, 100, 64, causal=True, two_pass=True, block_size=32)
    bm = np.ones((4, 4), bool)
    bm[0, 2] = bm[1, 3] = bm[3, 0] = bm[2, 1] = False
    fwd_case("fwd_blockmask_d64", 1, 2, 2, 128, 128, 64, block_mask=bm, block_size=32)
    fwd_case("fwd_fp16_compute_d16", 1, 2, 2, 32, 32, 16, compute_dtype=torch.float16, block_size=16)

    # KV-cache concat (bottom-right aligned causal through q_offset)
    q = bf16_vals(rng, 1, 2, 20, 64)
    kc, vc = bf16_vals(rng, 1, 2, 90, 64), bf16_vals(rng, 1, 2, 90, 64)
    kn, vn = bf16_vals(rng, 1, 2, 20, 64), bf16_vals(rng, 1, 2, 20, 64)
    o, lse = ref.fastest_flash_attn_forward(T(q), T(kn), T(vn), causal=True, kv_cache=(T(kc), T(vc)),
                                            return_lse=True, block_size=16)
    cases["fwd_kvcache_d64"] = dict(q=q, k=kn, v=vn, k_cache=kc, v_cache=vc, o=N(o), lse=N(lse),
                                    params=np.array(repr(dict(causal=True, block_size=16))))

    # ---- base backward (cpu_reference.flash_attn_cpu_backward) ----
    def bwd_case(name, B, H, S, D, **kw):
        q, k, v = (bf16_vals(rng, B, H, S, D) for _ in range(3))
        do = bf16_vals(rng, B, H, S, D)
        bs = kw.pop("block_size", 64)
        o, lse = cpu_reference.flash_attn_cpu_forward(T(q), T(k), T(v), block_q=bs, block_kv=bs, return_lse=True,
                                                      **kw)
        dq, dk, dv = cpu_reference.flash_attn_cpu_backward(T(do), T(q), T(k), T(v), o, lse, block_q=bs,
                                                           block_kv=bs, **kw)
        cases[name] = dict(q=q, k=k, v=v, do=do, o=N(o), lse=N(lse), dq=N(dq), dk=N(dk), dv=N(dv),
                           params=np.array(repr(dict(block_size=bs, **kw))))

    bwd_case("bwd_causal_d64", 1, 2, 192, 64, causal=True)
    bwd_case("bwd_window_softcap_d128", 1, 2, 200, 128, causal=True, sliding_window=64, softcap=30.0,
             block_size=32)
    bwd_case("bwd_noncausal_d64", 2, 1, 100, 64)

    # autograd path through fastest_flash_attn_func (3-D input)
    q, k, v, do = (bf16_vals(rng, 2, 64, 64) for _ in range(4))
    tq, tk, tv = (T(x).requires_grad_(True) for x in (q, k, v))
    o = ref.fastest_flash_attn_func(tq, tk, tv, causal=True, block_size=16)
    o.backward(T(do))
    cases["func_3d_causal_d64"] = dict(q=q, k=k, v=v, do=do, o=N(o), dq=N(tq.grad), dk=N(tk.grad), dv=N(tv.grad),
                                       params=np.array(repr(dict(causal=True, block_size=16))))

    # ---- FA4 ----
    def fa4_case(name, B, H, S, D, **kw):
        q, k, v = (bf16_vals(rng, B, H, S, D) for _ in range(3))
        do = bf16_vals(rng, B, H, S, D)
        bs = kw.pop("block_size", 64)
        o, lse_fa4 = cpu_fa4.fa4_forward(T(q), T(k), T(v), block_q=bs, block_kv=bs, return_lse=True, **kw)
        fkw = {k_: kw[k_] for k_ in ("causal", "softcap", "sliding_window") if k_ in kw}
        _, lse_exact = cpu_reference.flash_attn_cpu_forward(T(q), T(k), T(v), block_q=bs, block_kv=bs,
                                                            return_lse=True, **fkw)
        dq, dk, dv = cpu_fa4.fa4_backward(T(do), T(q), T(k), T(v), o, lse_exact, block_q=bs, block_kv=bs,
                                          deterministic=True, **fkw)
        cases[name] = dict(q=q, k=k, v=v, do=do, o=N(o), lse_fa4=N(lse_fa4), lse_exact=N(lse_exact),
                           dq=N(dq), dk=N(dk), dv=N(dv), params=np.array(repr(dict(block_size=bs, **kw))))

    fa4_case("fa4_causal_d64", 1, 2, 256, 64, causal=True)
    fa4_case("fa4_window_softcap_d128", 1, 2, 192, 128, causal=True, sliding_window=64, softcap=30.0,
             block_size=32)
    fa4_case("fa4_tau_d64", 1, 2, 128, 64, causal=True, rescale_threshold=0.5, block_size=32)

    xs = np.linspace(-130, 20, 1001).astype(np.float32)
    cases["fa4_software_exp2"] = dict(x=xs, y=N(cpu_fa4._software_exp2(T(xs))))
    cases["fa4_tile_schedule"] = dict(causal=np.array(cpu_fa4._build_tile_schedule(7, True, 7)),
                                      noncausal=np.array(cpu_fa4._build_tile_schedule(7, False, 7)))

    # ---- block-mask generators ----
    cases["block_masks"] = dict(
        causal=N(block_sparse.create_causal_block_mask(100, 130, 16, 32, q_offset=30)).astype(np.uint8),
        window=N(block_sparse.create_sliding_window_block_mask(128, 128, 16, 16, 40)).astype(np.uint8),
        local=N(block_sparse.create_local_block_mask(128, 160, 16, 32, 24)).astype(np.uint8))

    # ---- paged cache bookkeeping + gather ----
    cache = ref.PagedKVCache(max_pages=8, page_size=4, num_heads=2, head_dim=8, dtype=torch.float32)
    toks = {}
    for sid, n in ((0, 6), (1, 3)):
        kt, vt = bf16_vals(rng, 2, n, 8), bf16_vals(rng, 2, n, 8)
        toks[sid] = (kt, vt)
        cache.append_tokens(sid, T(kt), T(vt))
    cache.free_sequence(0)
    k2, v2 = bf16_vals(rng, 2, 10, 8), bf16_vals(rng, 2, 10, 8)
    cache.append_tokens(2, T(k2), T(v2))
    kg, vg = cache.get_kv(2)
    cases["paged_cache"] = dict(
        table1=np.array(cache.sequences[1]["page_table"]), table2=np.array(cache.sequences[2]["page_table"]),
        free=np.array(cache.free_pages), len2=np.array(cache.sequences[2]["len"]), k2=k2, v2=v2, kg=N(kg), vg=N(vg),
        k_pages=N(cache.k_pages), v_pages=N(cache.v_pages))

    # ---- MLA module (fp32) ----
    torch.manual_seed(7)
    mla = ref.FastestFlashMLA(hidden_size=64, num_heads=2, head_dim=64, latent_dim=32, rope_dim=16, causal=True)
    for prm in mla.parameters():
        torch.nn.init.normal_(prm, std=0.1)
    mla.eval()
    x = rng.standard_normal((2, 40, 64)).astype(np.float32)
    with torch.no_grad():
        y = mla(T(x), block_size=16)
    cases["mla_small"] = dict(x=x, y=N(y), w_q=N(mla.q_proj.weight), w_qr=N(mla.q_rope_proj.weight),
                              w_down=N(mla.kv_down_proj.weight), w_up=N(mla.kv_up_proj.weight),
                              w_kr=N(mla.k_rope_proj.weight), w_o=N(mla.o_proj.weight),
                              inv_freq=N(mla.rope.inv_freq),
                              params=np.array(repr(dict(num_heads=2, head_dim=64, rope_dim=16, block_size=16))))

    # ---- small head dims (the sizes the reference's own tests use) ----
    # (after every other case, so the random streams of those stay unchanged)
    fwd_case("fwd_small_d4_causal", 2, 2, 2, 33, 33, 4, causal=True, block_size=8)
    fwd_case("fwd_small_d8_window_softcap", 1, 4, 2, 50, 50, 8, causal=True, sliding_window=12, softcap=5.0,
             block_size=16)
    fwd_case("fwd_small_d32_mqa_sq_ne_skv", 1, 4, 1, 17, 45, 32, block_size=16)
    bwd_case("bwd_small_d8_causal", 2, 2, 40, 8, causal=True, block_size=16)
    bwd_case("bwd_small_d16_window", 1, 2, 70, 16, causal=True, sliding_window=20, block_size=16)
    bwd_case("bwd_small_d32_softcap", 1, 1, 64, 32, softcap=10.0, block_size=32)

    out.mkdir(parents=True, exist_ok=True)
    total = 0
    for name, arrs in cases.items():
        path = out / f"{name}.npz"
        np.savez_compressed(path, **arrs)
        total += path.stat().st_size
    print(f"wrote {len(cases)} fixtures, {total / 1e6:.2f} MB")


if __name__ == "__main__":
    main()
