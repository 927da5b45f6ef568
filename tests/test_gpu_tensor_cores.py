"""The tensor-core products (tcgen05 kind::i8, or for Q8_0 layers with
"tc_f16" kind::f16 on the codes as f16, mma.cu) against the CPU oracle: prefill chunks and batched decode steps of at least `tc_rows` rows
run on the tensor cores, and the greedy tokens and logits stay identical
to the reference arithmetic (exact i32 group dots, then the f32 chain over
the groups in order, src/cpu/int8.rs:560-570)."""
import numpy as np
import pytest

from oracle import oracle as O
from trit_b200 import CausalLm

pytestmark = pytest.mark.gpu

FORMATS = ["mini_qwen3_q8_0", "mini_qwen3_int8", "mini_qwen3_ternary", "mini_mistral_q8_0", "mini_granite_q8_0"]


@pytest.mark.parametrize("name", FORMATS)
@pytest.mark.parametrize("tc_f16", [True, False])
def test_prefill_on_tensor_cores_matches_oracle(mini_models, name, tc_f16):
    path = mini_models[name]
    oracle = O.Oracle(path)
    prompt = np.random.default_rng(21).integers(0, oracle.vocab, size=150).tolist()
    ref = oracle.generate(prompt, 10, trace=True)
    with CausalLm.load(path, kv="f32", max_context=256, tc_rows=16, prefill_rows=100, tc_f16=tc_f16) as lm:
        toks, logits = lm.generate_traced(prompt, max_new=10)
    assert toks == ref["tokens"]
    for i in range(len(toks)):
        assert np.array_equal(logits[i], ref["logits"][i]), f"step {i}"


@pytest.mark.parametrize("name", ["mini_qwen3_q8_0", "mini_qwen3_int8", "mini_qwen3_ternary"])
@pytest.mark.parametrize("tc_f16", [True, False])
def test_batched_decode_on_tensor_cores_matches_oracle(mini_models, name, tc_f16):
    path = mini_models[name]
    oracle = O.Oracle(path, kv_f16=True)
    rng = np.random.default_rng(22)
    prompts = [rng.integers(0, oracle.vocab, size=int(n)).tolist() for n in rng.integers(1, 40, size=70)]
    want = [oracle.generate(p, 6)["tokens"] for p in prompts]
    with CausalLm.load(path, kv="f16", max_context=64, max_streams=70, tc_rows=16, tc_f16=tc_f16) as lm:
        assert lm.generate_batch(prompts, max_new=6) == want


def test_tensor_cores_on_and_off_agree(mini_models):
    path = mini_models["mini_qwen3_q8_0"]
    prompt = list(np.random.default_rng(23).integers(0, 4096, size=200))
    with CausalLm.load(path, max_context=256, tc_rows=1) as lm:
        a = lm.generate_traced(prompt, max_new=8)
    with CausalLm.load(path, max_context=256, tensor_cores=False) as lm:
        b = lm.generate_traced(prompt, max_new=8)
    assert a[0] == b[0] and np.array_equal(a[1][:len(a[0])], b[1][:len(b[0])])
