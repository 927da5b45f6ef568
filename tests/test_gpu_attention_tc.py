"""The tensor-core prompt attention (`"tc_attention": true`, with `"exact":
false`; tcgen05 kind::f16,
flash-style, mma.cu k_attention_tc) against the oracle. The prompt's
attention runs in another order than the reference's (the tensor cores'
sums, per-tile softmax, probabilities rounded to f16), so logits are not
bit-equal: the decode steps after it are the exact layered kernels, and the
test bounds the drift that the prompt's attention leaves in every step's
logits, and checks that the greedy tokens agree with the oracle's until the
first step whose top-1/top-2 logit gap is within that drift. Mini models
with 2, 4, 8 and 1 query heads a kv head, prompts of one and of several
128-key tiles, one stream and a batch."""
import numpy as np
import pytest

from oracle import oracle as O
from trit_b200 import CausalLm

pytestmark = pytest.mark.gpu

# Largest logit difference allowed on the mini models (std 0.15 weights, so
# logits of several units): the prompt's attention in f16 / tensor-core
# order moves an int8 activation code now and then.
TC_MAX_ABS = 0.5
TC_MIN_COS = 0.999


def _agree_until_gap(got, want, gaps, bound):
    for i, (a, b) in enumerate(zip(got, want)):
        if a != b:
            assert gaps[i] < bound, f"token {i} differs at gap {gaps[i]}"
            return
    assert len(got) == len(want)


@pytest.mark.parametrize("name", ["mini_qwen3_q8_0", "mini_mistral_q8_0", "mini_gqa8_q8_0", "mini_mha_q8_0"])
@pytest.mark.parametrize("length", [70, 300])
def test_tc_prompt_attention_logits_near_oracle(mini_models, name, length):
    path = mini_models[name]
    oracle = O.Oracle(path, kv_f16=True)
    prompt = np.random.default_rng(61).integers(0, oracle.vocab, size=length).tolist()
    ref = oracle.generate(prompt, 8, trace=True)
    with CausalLm.load(path, kv="f16", decode="layered", exact=False, tc_attention=True, max_context=length + 64) as lm:
        toks, logits = lm.generate_traced(prompt, max_new=8)
    n = min(len(toks), len(ref["tokens"]))
    worst = 0.0
    for i in range(n):
        a, b = np.asarray(logits[i], np.float64), np.asarray(ref["logits"][i], np.float64)
        worst = max(worst, float(np.max(np.abs(a - b))))
        cos = float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))
        assert cos >= TC_MIN_COS, (i, cos)
        if toks[i] != ref["tokens"][i]:
            break
    print(f"{name} prompt {length}: max |dlogit| {worst:.4g}")
    assert worst <= TC_MAX_ABS, worst
    gaps = [float(np.sort(np.asarray(l))[-1] - np.sort(np.asarray(l))[-2]) for l in ref["logits"]]
    _agree_until_gap(toks, ref["tokens"], gaps, 2 * worst + 1e-6)


def test_tc_prompt_attention_batch_equals_single(mini_models):
    """A row's tensor-core attention does not depend on the tile it is in (the
    key tiles are fixed, and a fully masked tile adds exact zeros), so a batch
    whose prompt passes mix streams makes each stream's tokens of a
    single-stream call with the same option."""
    path = mini_models["mini_qwen3_q8_0"]
    rng = np.random.default_rng(62)
    prompts = [rng.integers(0, 4096, size=n).tolist() for n in (5, 140, 260, 33)]
    with CausalLm.load(path, kv="f16", decode="layered", exact=False, tc_attention=True, max_context=400, max_streams=4,
                       prefill_rows=256) as lm:
        got = lm.generate_batch(prompts, max_new=6)
        single = [lm.generate(p, max_new=6) for p in prompts]
    assert got == single
