"""The multi-rank host logic of a data-parallel run, on two gloo ranks on
the CPU: the stream split covers every stream once, prompts do not depend
on the split, and the timing reduction takes the maximum over ranks."""
import os
import socket

import pytest
import torch.multiprocessing as mp

from trit_b200 import dp


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def worker(rank: int, world: int, port: int, total: int, queue):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    r = dp.init("gloo", timeout_s=60)
    mine = dp.split(total, r)
    dp.barrier(r)
    slowest = dp.reduce(float(10 + rank), r, "max")
    made = dp.reduce(float(len(mine)), r, "sum")
    prompts = {s: dp.stream_prompt(5, s, 8, 1000) for s in mine}
    queue.put((rank, list(mine), slowest, made, prompts))
    dp.barrier(r)
    dp.finish(r)


@pytest.mark.parametrize("total", [64, 7])
def test_two_gloo_ranks(total):
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, total, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = sorted(queue.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    covered = sorted(s for _, mine, _, _, _ in results for s in mine)
    assert covered == list(range(total))
    assert all(slowest == 11.0 for _, _, slowest, _, _ in results)
    assert all(made == total for _, _, _, made, _ in results)
    for _, mine, _, _, prompts in results:
        for s in mine:
            assert prompts[s] == dp.stream_prompt(5, s, 8, 1000)


def test_split_sizes():
    for total in (0, 1, 5, 64, 65):
        for world in (1, 2, 3, 8):
            sizes = [len(dp.split(total, dp.Rank(r, world))) for r in range(world)]
            assert sum(sizes) == total and max(sizes) - min(sizes) <= 1
