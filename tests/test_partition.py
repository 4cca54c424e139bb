"""Host logic of the multi-GPU split (fastest_flash_attention_b200/partition.py):
GQA groups cover the job exactly once with balanced counts, and the decode
request split is greedy LPT on context length."""
import random

import pytest

from fastest_flash_attention_b200.partition import gqa_group_blocks, group_range, lpt_partition


@pytest.mark.parametrize("B,Hkv", [(4, 8), (3, 5), (1, 8), (2, 1), (7, 3)])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_groups_cover_the_job_once(B, Hkv, world):
    seen = []
    counts = []
    for r in range(world):
        n = 0
        for b0, b1, h0, h1 in gqa_group_blocks(B, Hkv, r, world):
            assert 0 <= b0 < b1 <= B and 0 <= h0 < h1 <= Hkv
            assert b1 - b0 == 1 or (h0, h1) == (0, Hkv)  # rectangles: whole batch rows or one row's heads
            seen += [(b, h) for b in range(b0, b1) for h in range(h0, h1)]
            n += (b1 - b0) * (h1 - h0)
        counts.append(n)
    assert sorted(seen) == [(b, h) for b in range(B) for h in range(Hkv)]
    assert max(counts) - min(counts) <= 1


def test_config2_split_is_one_launch_per_rank():
    # config 2: 4 batch x 8 kv heads; at 1/2/4/8 GPUs every rank runs one rectangle
    for world, per in ((1, [(0, 4, 0, 8)]), (2, [(0, 2, 0, 8)]), (4, [(0, 1, 0, 8)]), (8, [(0, 1, 0, 4)])):
        assert gqa_group_blocks(4, 8, 0, world) == per
    assert gqa_group_blocks(4, 8, 7, 8) == [(3, 4, 4, 8)]
    assert group_range(10, 3, 4) == (8, 10)


def test_lpt_partition():
    costs = [5, 9, 1, 7, 3, 3]
    parts = lpt_partition(costs, 2)
    assert sorted(i for p in parts for i in p) == list(range(6))
    loads = [sum(costs[i] for i in p) for p in parts]
    assert loads == [15, 13]  # greedy: 9->0, 7->1, 5->1, 3->0, 3->0 (tie: lower rank), 1->1
    rnd = random.Random(0)
    lens = [rnd.randint(512, 32768) for _ in range(64)]
    for world in (2, 4, 8):
        loads = [sum(lens[i] for i in p) for p in lpt_partition(lens, world)]
        assert max(loads) - min(loads) <= max(lens)
        assert max(loads) <= sum(lens) / world + max(lens)
    with pytest.raises(ValueError):
        lpt_partition([1], 0)


def test_e2e_chunks_cover_each_rank_once():
    """bench.py's e2e pipeline: the chunks of a rank cover exactly its GQA
    groups, with single-kv-head chunks at the ends."""
    import bench
    for world in (1, 2, 4, 8):
        for rank in range(world):
            blocks = bench.rank_blocks(world, rank)
            ch = bench.e2e_chunks(blocks, 4)
            got = sorted((b, g) for b, g0, g1 in ch for g in range(g0, g1))
            want = sorted((b, h) for b0, b1, h0, h1 in blocks for b in range(b0, b1) for h in range(h0, h1))
            assert got == want
            assert ch[0][2] - ch[0][1] == 1


def test_kernel_head_dims():
    from fastest_flash_attention_b200.attention import kernel_head_dims
    assert kernel_head_dims(64, 64) == (64, 64)
    assert kernel_head_dims(4, 4) == (64, 64)
    assert kernel_head_dims(80, 80) == (128, 128)
    assert kernel_head_dims(96, 64) == (128, 128)
    assert kernel_head_dims(160, 128) == (192, 128)
    assert kernel_head_dims(192, 128) == (192, 128)
    assert kernel_head_dims(256, 256) is None
    assert kernel_head_dims(64, 160) is None
