"""trit_lm_generate_batch: independent greedy generations decoded side by
side. Every stream's tokens equal the CPU oracle's CausalLm::generate for
that stream alone (causal_lm.rs:217-249,284-302), for ragged prompt
lengths, prefill chunks that span streams, more streams than one table
pass takes (16), and stop tokens."""
import numpy as np
import pytest

from oracle import oracle as O
from trit_b200 import CausalLm

pytestmark = pytest.mark.gpu

FORMATS = ["mini_qwen3_q8_0", "mini_qwen3_int8", "mini_qwen3_ternary", "mini_mistral_q8_0", "mini_granite_q8_0",
           "mini_gqa8_q8_0", "mini_mha_q8_0"]


def _prompts(vocab, lens, seed):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, vocab, size=n).tolist() for n in lens]


@pytest.mark.parametrize("name", FORMATS)
@pytest.mark.parametrize("kv", ["f32", "f16"])
def test_batch_matches_oracle_per_stream(mini_models, name, kv):
    path = mini_models[name]
    oracle = O.Oracle(path, kv_f16=(kv == "f16"))
    prompts = _prompts(oracle.vocab, [1, 7, 20, 33, 64], 11)
    want = [oracle.generate(p, 12)["tokens"] for p in prompts]
    with CausalLm.load(path, kv=kv, max_context=128, max_streams=8, prefill_rows=24) as lm:
        got = lm.generate_batch(prompts, max_new=12)
        assert got == want
        # A second call reuses the captured step.
        assert lm.generate_batch(prompts, max_new=12) == want
        t = lm.last_timing()
        assert t["decode_steps"] == 11 * len(prompts) and t["launches"] > 0


@pytest.mark.parametrize("name", ["mini_qwen3_q8_0", "mini_mistral_q8_0", "mini_gqa8_q8_0", "mini_mha_q8_0"])
@pytest.mark.parametrize("kv", ["f32", "f16"])
@pytest.mark.parametrize("length", [70, 300])
def test_one_row_attention_logits_match_oracle(mini_models, name, kv, length):
    """The one-row attention of decode steps (2, 4, 8 and 1 query heads a kv
    head) through the layered decode loop: tokens and logits bit for bit,
    over cache pages of 64 positions; 300 prompt ids span several staged
    key tiles (256 keys a tile for f16, 128 for f32) with odd and even key
    counts."""
    path = mini_models[name]
    oracle = O.Oracle(path, kv_f16=(kv == "f16"))
    prompt = np.random.default_rng(41).integers(0, oracle.vocab, size=length).tolist()
    ref = oracle.generate(prompt, 10, trace=True)
    with CausalLm.load(path, kv=kv, decode="layered", max_context=length + 90) as lm:
        toks, logits = lm.generate_traced(prompt, max_new=10)
    assert toks == ref["tokens"]
    for i in range(len(toks)):
        assert np.array_equal(logits[i], ref["logits"][i]), f"step {i}"


def test_many_streams_and_stops(mini_models):
    path = mini_models["mini_qwen3_q8_0"]
    oracle = O.Oracle(path)
    prompts = _prompts(oracle.vocab, [5 + 3 * i for i in range(20)], 12)
    want = [oracle.generate(p, 9)["tokens"] for p in prompts]
    stop = [want[3][4], want[17][0]]
    want_stopped = [oracle.generate(p, 9, stop=stop)["tokens"] for p in prompts]
    with CausalLm.load(path, kv="f32", max_context=96, max_streams=20, prefill_rows=64) as lm:
        assert lm.generate_batch(prompts, max_new=9) == want
        assert lm.generate_batch(prompts, max_new=9, stop=stop) == want_stopped
        # Fewer streams than before, and one token each.
        assert lm.generate_batch(prompts[:3], max_new=1) == [w[:1] for w in want[:3]]


def test_batch_equals_single_stream_decode(mini_models):
    path = mini_models["mini_qwen3_int8"]
    prompts = _prompts(4096, [40, 41], 13)
    with CausalLm.load(path, kv="f16", max_context=128, max_streams=2) as lm:
        single = [lm.generate(p, max_new=20) for p in prompts]
        assert lm.generate_batch(prompts, max_new=20) == single


def test_batch_argument_errors(mini_models):
    from trit_b200.lm import TritError

    with CausalLm.load(mini_models["mini_qwen3_q8_0"], max_context=64, max_streams=2) as lm:
        with pytest.raises(TritError, match="exceed max_streams"):
            lm.generate_batch([[1], [2], [3]], max_new=4)
        with pytest.raises(TritError, match="empty"):
            lm.generate_batch([[1], []], max_new=4)
        with pytest.raises(TritError, match="max_context"):
            lm.generate_batch([[1] * 60], max_new=8)
        with pytest.raises(TritError, match="outside the vocabulary"):
            lm.generate_batch([[1, 99999]], max_new=4)
