"""Two-way tensor parallelism on two GPUs (one process each, NCCL): a rank
holds half of the query heads with their key/value heads, half of the FFN
units and half of the output table; o_proj and down_proj partials are
summed by an all-reduce and the best token by a max-reduction of argmax
keys. Both ranks must make the oracle's tokens, for a batch and for one
stream, and agree with each other. A rank that stops answering ends the
other's call with an error after `tp_timeout_s` (the communicator is
aborted), not with a hang. Skipped with fewer than two GPUs."""
import os
import queue as queue_mod
import time

import numpy as np
import pytest
import torch.multiprocessing as mp

from oracle import oracle as O

pytestmark = pytest.mark.gpu

MODEL = "mini_qwen3_q8_0"  # 4 heads, 2 kv heads, 768 FFN units: splits 2 ways


def rank_main(rank, path, tp_id, prompts, queue):
    from trit_b200 import CausalLm

    stage = "load"
    try:
        with CausalLm.load(path, device=rank, kv="f16", max_context=128, max_streams=len(prompts), tp_size=2,
                           tp_rank=rank, tp_id=tp_id, tp_timeout_s=60) as lm:
            stage = "generate_batch"
            batch = lm.generate_batch(prompts, max_new=16)
            stage = "generate"
            one = lm.generate(prompts[0], max_new=16)
            status = lm.status()
        queue.put((rank, batch, one, status, None))
    except Exception as e:  # reported to the test, which fails on it
        queue.put((rank, None, None, None, f"{stage}: {e!r}"))


def quiet_rank_main(rank, path, tp_id, prompt, queue, leave):
    """Rank 1 of the failure test joins the group, then never takes part in
    a step: it waits until the test lets it go, then frees its handle."""
    from trit_b200 import CausalLm

    try:
        with CausalLm.load(path, device=rank, kv="f16", max_context=128, tp_size=2, tp_rank=rank, tp_id=tp_id,
                           tp_timeout_s=10) as lm:
            if rank == 0:
                t0 = time.time()
                try:
                    lm.generate(prompt, max_new=8)
                    queue.put((rank, "no error", time.time() - t0))
                except Exception as e:
                    queue.put((rank, str(e), time.time() - t0))
            else:
                queue.put((rank, "joined", 0.0))
                leave.wait(120)
    except Exception as e:
        queue.put((rank, f"load: {e!r}", 0.0))


def collect(queue, procs, n, seconds):
    """The ranks' reports, as they come; stops early when a rank died
    without one. Ranks still running afterwards are killed."""
    got, deadline = {}, time.time() + seconds
    while len(got) < n and time.time() < deadline:
        try:
            item = queue.get(timeout=2)
            got[item[0]] = item
        except queue_mod.Empty:
            if any(p.exitcode not in (None, 0) for p in procs):
                break
    return got


def finish(procs):
    for p in procs:
        p.join(timeout=30)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join(timeout=10)


def test_two_way_tensor_parallel_tokens(mini_models):
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from trit_b200 import lm

    path = mini_models[MODEL]
    oracle = O.Oracle(path, kv_f16=True)
    rng = np.random.default_rng(51)
    prompts = [rng.integers(0, oracle.vocab, size=n).tolist() for n in (30, 41, 17, 25)]
    want = [oracle.generate(p, 16)["tokens"] for p in prompts]
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    tp_id = lm.tp_id()
    procs = [ctx.Process(target=rank_main, args=(r, path, tp_id, prompts, queue)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        got = collect(queue, procs, 2, 240)
    finally:
        finish(procs)
    errors = {r: g[4] for r, g in got.items() if g[4]}
    assert not errors, f"rank errors: {errors}"
    assert sorted(got) == [0, 1], f"ranks that reported: {sorted(got)}; exit codes {[p.exitcode for p in procs]}"
    for rank in (0, 1):
        _, batch, one, status, _ = got[rank]
        assert batch == want, f"rank {rank}"
        assert one == want[0], f"rank {rank}"
        assert status["decode"] == "layered"


def test_lost_rank_ends_the_call_with_an_error(mini_models):
    """Rank 1 joins and then stops answering (between steps, with nothing in
    flight): rank 0's generate fails after tp_timeout_s (10 s) with the
    tensor-parallel error, instead of waiting for good. NVLS is off, as for
    every test where a rank goes quiet."""
    torch = pytest.importorskip("torch")
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    from trit_b200 import lm

    path = mini_models[MODEL]
    prompt = np.random.default_rng(52).integers(0, 4096, size=20).tolist()
    ctx = mp.get_context("spawn")
    queue, leave = ctx.Queue(), ctx.Event()
    tp_id = lm.tp_id()
    old = os.environ.get("NCCL_NVLS_ENABLE")
    os.environ["NCCL_NVLS_ENABLE"] = "0"  # inherited by the ranks
    try:
        procs = [ctx.Process(target=quiet_rank_main, args=(r, path, tp_id, prompt, queue, leave)) for r in range(2)]
        for p in procs:
            p.start()
    finally:
        if old is None:
            os.environ.pop("NCCL_NVLS_ENABLE", None)
        else:
            os.environ["NCCL_NVLS_ENABLE"] = old
    try:
        got = collect(queue, procs, 2, 120)
    finally:
        leave.set()
        finish(procs)
    assert sorted(got) == [0, 1], f"ranks that reported: {got}"
    assert got[1][1] == "joined", got[1]
    message, seconds = got[0][1], got[0][2]
    assert "tensor parallelism" in message and "did not answer" in message, message
    assert seconds < 60, seconds
