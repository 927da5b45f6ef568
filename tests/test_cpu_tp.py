"""The tensor-parallel partition (the optional 2/4-way split of the
largest decoder), on gloo ranks on the CPU: each rank describes its shard
of the Ministral-3B-shaped model of C5 (trit_lm_inspect with tp_size /
tp_rank, no GPU), the ranks gather the shards, and together they cover
every query head, key/value head, FFN unit and output-table row once, with
every query head on the rank of its key/value head (whole GQA groups)."""
import os
import socket
import tempfile

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from tests import synth
from tests.synth import presets

# The C5 shape with two layers and a small vocabulary: the partition does
# not depend on depth, and a small model writes in a second.
SHAPE = dict(presets.MINISTRAL_3B, num_hidden_layers=2, vocab_size=4096)


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def worker(rank: int, world: int, port: int, path: str, queue):
    from trit_b200 import lm

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    mine = lm.inspect(path, tp_size=world, tp_rank=rank)["tp"]
    shards = [None] * world
    dist.all_gather_object(shards, mine)
    if rank == 0:
        queue.put(shards)
    dist.barrier()
    dist.destroy_process_group()


def covers(ranges, total):
    at = 0
    for lo, hi in sorted(ranges):
        assert lo == at and hi > lo, (ranges, total)
        at = hi
    assert at == total


@pytest.mark.parametrize("world", [2, 4])
def test_shards_tile_the_model(world):
    with tempfile.TemporaryDirectory() as tmp:
        path = synth.synthesize(os.path.join(tmp, "m"), SHAPE, "q8_0", 5)
        ctx = mp.get_context("spawn")
        queue = ctx.Queue()
        port = free_port()
        procs = [ctx.Process(target=worker, args=(r, world, port, path, queue)) for r in range(world)]
        for p in procs:
            p.start()
        shards = queue.get(timeout=120)
        for p in procs:
            p.join(timeout=60)
            assert p.exitcode == 0
    assert [s["rank"] for s in shards] == list(range(world))
    qpk = SHAPE["num_attention_heads"] // SHAPE["num_key_value_heads"]
    covers([s["heads"] for s in shards], SHAPE["num_attention_heads"])
    covers([s["kv_heads"] for s in shards], SHAPE["num_key_value_heads"])
    covers([s["ffn_units"] for s in shards], SHAPE["intermediate_size"])
    covers([s["vocab_rows"] for s in shards], SHAPE["vocab_size"])
    for s in shards:
        assert s["heads"] == [s["kv_heads"][0] * qpk, s["kv_heads"][1] * qpk]
        assert (s["ffn_units"][1] - s["ffn_units"][0]) % 128 == 0


def test_a_shard_that_does_not_divide_is_refused():
    from trit_b200 import lm

    with tempfile.TemporaryDirectory() as tmp:
        path = synth.synthesize(os.path.join(tmp, "m"), SHAPE, "q8_0", 5)
        with pytest.raises(lm.TritError, match="key/value heads"):
            lm.inspect(path, tp_size=3, tp_rank=0)
