"""KV-cache host logic: the paged allocator reproduces the reference's FIFO
page tables bit-exactly (golden from ops/kv_cache.py), CPU pools gather the
same bytes, and the continuous cache appends like the reference."""
import numpy as np
import torch

from conftest import load_golden


def test_paged_tables_and_gather_match_reference():
    from fastest_flash_attention_b200 import PagedKVCache
    g = load_golden("paged_cache")
    c = PagedKVCache(max_pages=8, page_size=4, num_heads=2, head_dim=8, dtype=torch.float32)
    rng = np.random.default_rng(0)
    for sid, n in ((0, 6), (1, 3)):
        c.append_tokens(sid, torch.from_numpy(rng.standard_normal((2, n, 8)).astype(np.float32)),
                        torch.from_numpy(rng.standard_normal((2, n, 8)).astype(np.float32)))
    c.free_sequence(0)
    c.append_tokens(2, torch.from_numpy(g["k2"]), torch.from_numpy(g["v2"]))
    assert c.sequences[1]["page_table"] == list(g["table1"])
    assert c.sequences[2]["page_table"] == list(g["table2"])
    assert c.free_pages == list(g["free"])
    k, v = c.get_kv(2)
    np.testing.assert_array_equal(k.numpy(), g["kg"])
    np.testing.assert_array_equal(v.numpy(), g["vg"])
    bt, lens = c.block_table([1, 2])
    assert bt.dtype == torch.int32 and bt[1, :3].tolist() == list(g["table2"]) and lens.tolist() == [3, 10]


def test_paged_out_of_pages_raises():
    from fastest_flash_attention_b200 import PagedKVCache
    c = PagedKVCache(max_pages=1, page_size=2, num_heads=1, head_dim=8, dtype=torch.float32)
    x = torch.zeros(1, 3, 8)
    try:
        c.append_tokens(0, x, x)
    except RuntimeError as e:
        assert "out of physical pages" in str(e)
    else:
        raise AssertionError("expected RuntimeError")


def test_continuous_cache_append():
    from fastest_flash_attention_b200 import ContinuousKVCache
    c = ContinuousKVCache(2, 16, 2, 8, dtype=torch.float32)
    a = torch.randn(2, 2, 3, 8)
    k, v = c.append(a, a + 1)
    assert k.shape == (2, 2, 3, 8) and torch.equal(v, a + 1)
    k, v = c.append(a * 2, a)
    assert k.shape == (2, 2, 6, 8) and torch.equal(k[:, :, 3:], a * 2)
    assert c.seq_lens.tolist() == [6, 6]


def test_block_table_validation_rejects_bad_paging_data():
    import pytest
    from fastest_flash_attention_b200.decode import check_block_table
    bt = torch.tensor([[3, 1, 0], [2, 0, 0]], dtype=torch.int32)
    check_block_table(bt, torch.tensor([9, 4], dtype=torch.int32), num_pages=4, page_size=4)  # valid
    # a page id that the request reads is out of the pool
    with pytest.raises(ValueError, match=r"block_table\[0, 0\] = 3 is outside \[0, 3\)"):
        check_block_table(bt, torch.tensor([9, 4], dtype=torch.int32), num_pages=3, page_size=4)
    # unused trailing entries are not read, so they are not checked
    check_block_table(torch.tensor([[1, -7]], dtype=torch.int32), torch.tensor([4], dtype=torch.int32), 2, 4)
    with pytest.raises(ValueError, match=r"block_table\[0, 1\] = -7"):
        check_block_table(torch.tensor([[1, -7]], dtype=torch.int32), torch.tensor([5], dtype=torch.int32), 2, 4)
    # lengths beyond what the table row covers, or negative
    with pytest.raises(ValueError, match=r"ctx_lens\[1\] = 13 is outside \[0, 12\]"):
        check_block_table(bt, torch.tensor([9, 13], dtype=torch.int32), num_pages=4, page_size=4)
    with pytest.raises(ValueError, match=r"ctx_lens\[0\] = -1"):
        check_block_table(bt, torch.tensor([-1, 0], dtype=torch.int32), num_pages=4, page_size=4)
