"""GPU checks of the device-side paged append (ffa_paged_append) and of the
decode kernels' paging-data guards.

The append kernel writes a bf16 pool on the GPU; the checks compare the pool
against the appended tokens themselves (not against a read-back of the same
pool) and the FIFO tables against the reference's own tables
(tests/golden/paged_cache.npz, made by running ops/kv_cache.py:157-232).
Everything here is bit-exact (torch.equal)."""
import numpy as np
import pytest
import torch

from conftest import load_golden

pytestmark = pytest.mark.gpu


def _slots_of(cache, sid):
    seq = cache.sequences[sid]
    return [(seq["page_table"][t // cache.page_size], t % cache.page_size) for t in range(seq["len"])]


def _assert_pool_holds(cache, sid, k_ref, v_ref):
    # token t of the sequence sits at (page_table[t // ps], t % ps) for every head
    for t, (pg, off) in enumerate(_slots_of(cache, sid)):
        assert torch.equal(cache.k_pages[pg, :, off].cpu(), k_ref[:, t]), (sid, t)
        assert torch.equal(cache.v_pages[pg, :, off].cpu(), v_ref[:, t]), (sid, t)


def test_append_kernel_matches_reference_tables_bitwise():
    from fastest_flash_attention_b200 import PagedKVCache
    g = load_golden("paged_cache")
    c = PagedKVCache(max_pages=8, page_size=4, num_heads=2, head_dim=8, dtype=torch.bfloat16, device="cuda")
    rng = np.random.default_rng(0)
    toks = {}
    for sid, n in ((0, 6), (1, 3)):
        k = torch.from_numpy(rng.standard_normal((2, n, 8)).astype(np.float32)).to(torch.bfloat16)
        v = torch.from_numpy(rng.standard_normal((2, n, 8)).astype(np.float32)).to(torch.bfloat16)
        c.append_tokens(sid, k.cuda(), v.cuda())
        toks[sid] = (k, v)
    c.free_sequence(0)
    k2 = torch.from_numpy(g["k2"]).to(torch.bfloat16)
    v2 = torch.from_numpy(g["v2"]).to(torch.bfloat16)
    c.append_tokens(2, k2.cuda(), v2.cuda())
    torch.cuda.synchronize()
    assert c.sequences[1]["page_table"] == list(g["table1"])
    assert c.sequences[2]["page_table"] == list(g["table2"])
    assert c.free_pages == list(g["free"])
    _assert_pool_holds(c, 1, *toks[1])
    _assert_pool_holds(c, 2, k2, v2)
    k, v = c.get_kv(2)  # the reference's gather of the same sequence, bf16-rounded
    assert torch.equal(k.cpu(), torch.from_numpy(g["kg"]).to(torch.bfloat16))
    assert torch.equal(v.cpu(), torch.from_numpy(g["vg"]).to(torch.bfloat16))


@pytest.mark.parametrize("dtype,page_size,D", [(torch.bfloat16, 16, 128), (torch.float16, 64, 64)])
def test_append_kernel_ragged_appends_bitwise(dtype, page_size, D):
    from fastest_flash_attention_b200 import PagedKVCache
    gen = torch.Generator().manual_seed(5)
    Hkv, n_pages = 4, 64
    c = PagedKVCache(max_pages=n_pages, page_size=page_size, num_heads=Hkv, head_dim=D, dtype=dtype, device="cuda")
    c.free_pages = torch.randperm(n_pages, generator=gen).tolist()
    appended = {0: [], 1: [], 2: []}
    # interleaved appends of ragged sizes, including empty and page-crossing ones
    for sid, n in ((0, 1), (1, 37), (0, 0), (2, page_size), (0, 2 * page_size + 3), (1, 5), (2, 1), (0, 9)):
        k = torch.randn(Hkv, n, D, generator=gen).to(dtype)
        v = torch.randn(Hkv, n, D, generator=gen).to(dtype)
        c.append_tokens(sid, k.cuda(), v.cuda())
        appended[sid].append((k, v))
    torch.cuda.synchronize()
    for sid, parts in appended.items():
        k_ref = torch.cat([p[0] for p in parts], dim=1)
        v_ref = torch.cat([p[1] for p in parts], dim=1)
        assert c.sequences[sid]["len"] == k_ref.shape[1]
        _assert_pool_holds(c, sid, k_ref, v_ref)
    # untouched pages stay zero (no stray writes)
    used = {p for s in c.sequences.values() for p in s["page_table"]}
    for pg in set(range(n_pages)) - used:
        assert not c.k_pages[pg].any() and not c.v_pages[pg].any()


def test_decode_rejects_out_of_range_paging_data():
    """A bad page id or context length is reported through the error word and
    nothing outside the pool is read (the kernels check before loading)."""
    from fastest_flash_attention_b200 import _lib
    from fastest_flash_attention_b200.decode import paged_decode
    from fastest_flash_attention_b200.mla import mla_decode
    dev = torch.device("cuda", 0)

    def expect_error(fn, match):
        # the call itself raises when FFA_SYNC_CHECK is on; else the next check does
        with pytest.raises(RuntimeError, match=match):
            fn()
            _lib.check_device_errors(dev)

    P, Hkv, ps, D, Hq = 4, 2, 16, 128, 8
    kp = torch.randn(P, Hkv, ps, D, device=dev).to(torch.bfloat16)
    vp = torch.randn_like(kp)
    q = torch.randn(2, Hq, D, device=dev).to(torch.bfloat16)
    good_bt = torch.tensor([[0, 1], [2, 3]], dtype=torch.int32, device=dev)
    bad_bt = torch.tensor([[0, 1], [2, P + 5]], dtype=torch.int32, device=dev)
    lens = torch.tensor([20, 32], dtype=torch.int32, device=dev)
    paged_decode(q, kp, vp, good_bt, lens)
    _lib.check_device_errors(dev)  # valid data: no error
    expect_error(lambda: paged_decode(q, kp, vp, bad_bt, lens), "block-table entry is outside")
    expect_error(lambda: paged_decode(q, kp, vp, good_bt, torch.tensor([20, 33], dtype=torch.int32, device=dev)),
                 "context length")
    # the MLA latent decode has the same guards
    ckv = torch.randn(P, ps, 576, device=dev).to(torch.bfloat16)
    qm = torch.randn(2, 32, 576, device=dev).to(torch.bfloat16)
    mla_decode(qm, ckv, good_bt, lens, scale=0.05)
    _lib.check_device_errors(dev)
    expect_error(lambda: mla_decode(qm, ckv, bad_bt, lens, scale=0.05), "block-table entry is outside")
    expect_error(lambda: mla_decode(qm, ckv, good_bt, torch.tensor([-1, 32], dtype=torch.int32, device=dev),
                                    scale=0.05), "context length")
    # the context is still usable
    o = paged_decode(q, kp, vp, good_bt, lens)
    torch.cuda.synchronize()
    _lib.check_device_errors(dev)
    assert torch.isfinite(o.float()).all()
