"""Multi-process plumbing of bench.py on CPU: two gloo ranks, as torchrun
would launch them (RANK / WORLD_SIZE / LOCAL_RANK / MASTER_* from the
environment, rendezvous on 127.0.0.1).

Checked: the process group comes up, the timed value is the max over ranks,
barriers pass, every rank draws the same seeded job and keeps a disjoint
share of its GQA groups (strong scaling, no collective on the data path),
and only rank 0 runs the CPU reference arm.
"""
import os
import socket
import sys
from pathlib import Path

import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank),
                      WORLD_SIZE=str(world), LOCAL_RANK=str(rank))
    sys.path.insert(0, str(ROOT))
    import bench
    import torch.distributed as dist
    w, r, _ = bench.dist_init()
    assert (w, r) == (world, rank)
    assert dist.get_backend() == "gloo"
    bench.barrier(w)
    ms = bench.max_over_ranks(1.5 + rank, w)
    q, _, _ = bench.make_inputs("cpu", seed=0)
    digest = float(q[0, 0, :64].float().sum())
    blocks = bench.rank_blocks(w, r)

    class Args:
        gpus, steps, warmup = world, 1, 0
    # the reference arm runs on rank 0 only; other ranks return at once
    ran = None
    if rank != 0:
        ran = bench.run_reference(Args, w, r)
    bench.barrier(w)
    out.put((rank, ms, digest, ran, blocks, bench.block_flops(blocks)))
    dist.destroy_process_group()


def test_two_gloo_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(out.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [r[1] for r in res] == [2.5, 2.5]  # max over ranks, seen by every rank
    assert res[0][2] == res[1][2]             # the same job on every rank
    assert res[1][3] is None                  # rank 1 does not run the CPU arm
    assert res[0][4] == [(0, 2, 0, 8)] and res[1][4] == [(2, 4, 0, 8)]  # batch halves
    assert res[0][5] == res[1][5]             # equal work
