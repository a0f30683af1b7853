"""Multi-process (gloo, world_size 2, CPU) test of the data-parallel host logic: each rank's
utterance slice is disjoint from the others and together they cover the list, every rank
decodes a different prompt, and the timing reduction is the max over ranks."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from syrinx_b200 import dp


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def worker(rank, world, port, n_utt, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        lo, hi = dp.utterance_slice(n_utt, rank, world)
        slices = [None] * world
        dist.all_gather_object(slices, (lo, hi))
        seeds = [None] * world
        dist.all_gather_object(seeds, dp.rank_seed(2, rank))
        t = dp.max_over_ranks(10.0 * (rank + 1), dist)
        q.put((rank, slices, seeds, t))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_utt", [64, 7, 1])
def test_dp_slices_and_max_over_ranks(n_utt):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, n_utt, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, slices, seeds, t in out:
        covered = sorted(u for lo, hi in slices for u in range(lo, hi))
        assert covered == list(range(n_utt))
        sizes = [hi - lo for lo, hi in slices]
        assert max(sizes) - min(sizes) <= 1
        assert len(set(seeds)) == world
        assert t == 10.0 * world


def test_slice_edge_cases():
    assert dp.utterance_slice(0, 0, 1) == (0, 0)
    assert dp.utterance_slice(8, 7, 8) == (7, 8)
    assert [dp.utterance_slice(10, r, 4) for r in range(4)] == [(0, 3), (3, 6), (6, 8), (8, 10)]
    with pytest.raises(ValueError):
        dp.utterance_slice(4, 2, 2)
    assert dp.max_over_ranks(3.5) == 3.5
