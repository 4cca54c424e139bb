"""Pins the numpy oracle to the reference's own outputs (golden fixtures made
by running the reference; see golden/make_golden.py).  CPU only."""
import ast

import numpy as np
import pytest

from conftest import load_golden, golden_params
from oracle import attention_oracle as O

FWD_CASES = ["fwd_basic_d16", "fwd_causal_d64", "fwd_causal_d128_ragged", "fwd_window_d64", "fwd_softcap_d64",
             "fwd_gqa_d128", "fwd_noncausal_sq_ne_skv_d64", "fwd_two_pass_d64", "fwd_blockmask_d64",
             "fwd_fp16_compute_d16", "fwd_small_d4_causal", "fwd_small_d8_window_softcap",
             "fwd_small_d32_mqa_sq_ne_skv"]


def _fwd_kwargs(p):
    kw = dict(causal=p.get("causal", False), block_size=p.get("block_size", 64), softcap=p.get("softcap"),
              sliding_window=p.get("sliding_window"), two_pass=p.get("two_pass", False))
    if "compute_dtype" in p:
        kw["compute_dtype"] = "float16"
    return kw


@pytest.mark.parametrize("name", FWD_CASES)
def test_forward_matches_reference(name):
    g = load_golden(name)
    p = ast.literal_eval(str(g["params"]).replace("torch.float16", "'float16'"))
    kw = _fwd_kwargs(p)
    o, lse = O.attention_forward(g["q"], g["k"], g["v"], block_mask=g.get("block_mask"), **kw)
    np.testing.assert_allclose(o, g["o"], atol=2e-5, rtol=0)
    np.testing.assert_allclose(lse, g["lse"], atol=2e-5, rtol=0)


def test_forward_kvcache_matches_reference():
    g = load_golden("fwd_kvcache_d64")
    o, lse = O.attention_forward(g["q"], g["k"], g["v"], causal=True, block_size=16,
                                 kv_cache=(g["k_cache"], g["v_cache"]))
    np.testing.assert_allclose(o, g["o"], atol=2e-5)
    np.testing.assert_allclose(lse, g["lse"], atol=2e-5)


@pytest.mark.parametrize("name", ["bwd_causal_d64", "bwd_window_softcap_d128", "bwd_noncausal_d64",
                                  "bwd_small_d8_causal", "bwd_small_d16_window", "bwd_small_d32_softcap"])
def test_backward_matches_reference(name):
    g = load_golden(name)
    p = golden_params(g)
    bs = p.pop("block_size")
    o, lse = O.flash_forward(g["q"], g["k"], g["v"], block_q=bs, block_kv=bs, return_lse=True, **p)
    np.testing.assert_allclose(o, g["o"], atol=2e-5)
    dq, dk, dv = O.flash_backward(g["do"], g["q"], g["k"], g["v"], o, lse, block_q=bs, block_kv=bs, **p)
    for a, b in ((dq, g["dq"]), (dk, g["dk"]), (dv, g["dv"])):
        np.testing.assert_allclose(a, b, atol=5e-5, rtol=1e-4)


def test_autograd_func_3d_matches_reference():
    g = load_golden("func_3d_causal_d64")
    q, k, v, do = (g[x][:, None] for x in ("q", "k", "v", "do"))
    o, lse = O.flash_forward(q, k, v, causal=True, block_q=16, block_kv=16, return_lse=True)
    np.testing.assert_allclose(o[:, 0], g["o"], atol=2e-5)
    dq, dk, dv = O.flash_backward(do, q, k, v, o, lse, causal=True, block_q=16, block_kv=16)
    np.testing.assert_allclose(dq[:, 0], g["dq"], atol=5e-5, rtol=1e-4)
    np.testing.assert_allclose(dk[:, 0], g["dk"], atol=5e-5, rtol=1e-4)
    np.testing.assert_allclose(dv[:, 0], g["dv"], atol=5e-5, rtol=1e-4)


@pytest.mark.parametrize("name", ["fa4_causal_d64", "fa4_window_softcap_d128", "fa4_tau_d64"])
def test_fa4_matches_reference(name):
    g = load_golden(name)
    p = golden_params(g)
    bs = p.pop("block_size")
    o, lse = O.fa4_forward(g["q"], g["k"], g["v"], block_q=bs, block_kv=bs, return_lse=True, **p)
    np.testing.assert_allclose(o, g["o"], atol=5e-5)
    np.testing.assert_allclose(lse, g["lse_fa4"], atol=5e-5)   # reproduces the reference's own (inexact) LSE
    fkw = {k: p[k] for k in ("causal", "softcap", "sliding_window") if k in p}
    _, lse_exact = O.flash_forward(g["q"], g["k"], g["v"], block_q=bs, block_kv=bs, return_lse=True, **fkw)
    np.testing.assert_allclose(lse_exact, g["lse_exact"], atol=2e-5)
    dq, dk, dv = O.fa4_backward(g["do"], g["q"], g["k"], g["v"], g["o"], lse_exact, block_q=bs, block_kv=bs, **fkw)
    for a, b in ((dq, g["dq"]), (dk, g["dk"]), (dv, g["dv"])):
        np.testing.assert_allclose(a, b, atol=1e-4, rtol=1e-4)


def test_fa4_lse_defect_is_documented():
    """The reference's FA4 LSE differs from the exact LSE over several tiles
    (cpu_fa4.py:412); the oracle reproduces both values."""
    g = load_golden("fa4_causal_d64")
    assert np.abs(g["lse_fa4"] - g["lse_exact"]).max() > 1e-2


def test_software_exp2_and_schedule():
    g = load_golden("fa4_software_exp2")
    np.testing.assert_allclose(O.software_exp2(g["x"]), g["y"], rtol=1e-6, atol=0)
    s = load_golden("fa4_tile_schedule")
    assert O.build_tile_schedule(7, True, 7) == list(s["causal"])
    assert O.build_tile_schedule(7, False, 7) == list(s["noncausal"])


def test_block_mask_generators():
    g = load_golden("block_masks")
    assert (O.causal_block_mask(100, 130, 16, 32, q_offset=30) == g["causal"].astype(bool)).all()
    assert (O.sliding_window_block_mask(128, 128, 16, 16, 40) == g["window"].astype(bool)).all()
    assert (O.local_block_mask(128, 160, 16, 32, 24) == g["local"].astype(bool)).all()


def test_paged_cache_bookkeeping():
    g = load_golden("paged_cache")
    m = O.PagedCacheModel(8, 4)
    m.append(0, 6)
    m.append(1, 3)
    m.free_sequence(0)
    m.append(2, 10)
    assert m.sequences[1]["page_table"] == list(g["table1"])
    assert m.sequences[2]["page_table"] == list(g["table2"])
    assert m.free_pages == list(g["free"])
    kg = O.paged_gather(g["k_pages"], list(g["table2"]), int(g["len2"]))
    np.testing.assert_array_equal(kg, g["kg"])


def test_mla_module_matches_reference():
    g = load_golden("mla_small")
    p = golden_params(g)
    y = O.mla_forward(g["x"], g["w_q"], g["w_qr"], g["w_down"], g["w_up"], g["w_kr"], g["w_o"], g["inv_freq"],
                      p["num_heads"], p["head_dim"], p["rope_dim"], causal=True, block_size=p["block_size"])
    np.testing.assert_allclose(y, g["y"], atol=1e-4, rtol=1e-4)
