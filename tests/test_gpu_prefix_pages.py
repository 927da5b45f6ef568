"""Shared prefix pages (CausalLm::prefix / generate with a prefix,
causal_lm.rs:200-249; S1-mini's fixed system prompt, src/cleanup.rs:208,
297-299): a prefix's full KV pages are made once and read in place by every
call and every stream that starts with it. Calls neither copy nor allocate
the prefix again: the kept-page count and the device's free memory stay put
across calls, and the tokens stay the reference's."""
import numpy as np
import pytest

from oracle import oracle as O
from trit_b200 import CausalLm, TritError

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("exact", [True, False])
def test_prefix_pages_are_shared_not_copied(mini_models, exact):
    torch = pytest.importorskip("torch")
    path = mini_models["mini_qwen3_q8_0"]
    oracle = O.Oracle(path, kv_f16=True)
    rng = np.random.default_rng(23)
    system = rng.integers(0, oracle.vocab, size=40).tolist()  # 2 full pages of 16 and a partial one
    prompts = [system + rng.integers(0, oracle.vocab, size=n).tolist() for n in (5, 9, 14)]
    want = [oracle.generate(p, 16)["tokens"] for p in prompts]
    other = rng.integers(0, oracle.vocab, size=30).tolist()
    batch = prompts + [other]
    with CausalLm.load(path, kv="f16", max_context=128, page_tokens=16, max_streams=4, prefix_pages=4,
                       exact=exact) as lm:
        assert lm.prefix_pages() == (0, 4)
        pre = lm.prefix(system)
        assert lm.prefix_pages() == (2, 4)
        # One call of each kind first: the batch decode captures its step
        # graph on first use, which takes device memory once.
        lm.generate(prompts[0], prefix=pre, max_new=16)
        lm.generate_batch(batch, max_new=16, prefix=pre)
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        for _ in range(3):
            for p, w in zip(prompts, want):
                assert lm.generate(p, prefix=pre, max_new=16) == w
        # Batches: the streams that start with the prefix read its pages; a
        # stream that does not runs its whole prompt.
        got = lm.generate_batch(batch, max_new=16, prefix=pre)
        assert got == want + [oracle.generate(other, 16)["tokens"]]
        assert lm.generate_batch(batch, max_new=16) == got
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] == free_before
        assert lm.prefix_pages() == (2, 4)
        # A second prefix takes its own pages; freeing returns them.
        pre2 = lm.prefix(other[:20])
        assert lm.prefix_pages() == (3, 4)
        pre2.close()
        pre.close()
        assert lm.prefix_pages() == (0, 4)
        with pytest.raises(TritError, match="prefix_pages"):
            lm.prefix(rng.integers(0, oracle.vocab, size=5 * 16).tolist())
