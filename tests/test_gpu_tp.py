"""Two-way tensor parallelism on two GPUs (one process each, NCCL): a rank
holds half of the query heads with their key/value heads, half of the FFN
units and half of the output table; o_proj and down_proj partials are
summed by an all-reduce and the best token by a max-reduction of argmax
keys. Both ranks must make the oracle's tokens, for a batch and for one
stream, and agree with each other. Skipped with fewer than two GPUs."""
import numpy as np
import pytest
import torch.multiprocessing as mp

from oracle import oracle as O

pytestmark = pytest.mark.gpu

MODEL = "mini_qwen3_q8_0"  # 4 heads, 2 kv heads, 768 FFN units: splits 2 ways


def rank_main(rank, path, tp_id, prompts, queue):
    from trit_b200 import CausalLm

    try:
        with CausalLm.load(path, device=rank, kv="f16", max_context=128, max_streams=len(prompts), tp_size=2,
                           tp_rank=rank, tp_id=tp_id) as lm:
            batch = lm.generate_batch(prompts, max_new=16)
            one = lm.generate(prompts[0], max_new=16)
            status = lm.status()
        queue.put((rank, batch, one, status, None))
    except Exception as e:  # reported to the test, which fails on it
        queue.put((rank, None, None, None, repr(e)))


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
    got = sorted([queue.get(timeout=300) for _ in range(2)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
    for rank, batch, one, status, err in got:
        assert err is None, f"rank {rank}: {err}"
        assert batch == want, f"rank {rank}"
        assert one == want[0], f"rank {rank}"
        assert status["decode"] == "layered"
