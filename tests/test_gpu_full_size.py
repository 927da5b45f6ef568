"""The headline configuration (Qwen3-0.6B shape, Q8_0): the persistent
decode, the layered decode and the CPU oracle make the same tokens. The
small models of test_gpu_generate.py miss size-dependent paths (several
weight batches a block, many attention splits)."""
import numpy as np
import pytest

from oracle import oracle as O
from trit_b200 import CausalLm
from tests.synth import presets

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def c1_path():
    return presets.model_path("c1_qwen3_0.6b_q8_0")


def test_c1_persistent_equals_layered_and_oracle(c1_path):
    prompt = np.random.default_rng(1).integers(0, 151936, size=64).tolist()
    with CausalLm.load(c1_path, kv="f32", decode="persistent", exact=True, max_context=256) as lm:
        p_toks, p_logits = lm.generate_traced(prompt, max_new=12)
    with CausalLm.load(c1_path, kv="f32", decode="layered", max_context=256) as lm:
        l_toks, l_logits = lm.generate_traced(prompt, max_new=12)
    assert p_toks == l_toks
    n = len(p_toks)
    assert np.all(np.isfinite(p_logits[:n]))
    assert np.array_equal(p_logits[:n], l_logits[:n])
    ref = O.Oracle(c1_path).generate(prompt, 6, trace=True)
    assert p_toks[:6] == ref["tokens"]
    assert np.array_equal(p_logits[:6], ref["logits"][:6])


def test_c1_f16_cache_long_generation(c1_path):
    prompt = np.random.default_rng(2).integers(0, 151936, size=64).tolist()
    with CausalLm.load(c1_path, kv="f16", decode="persistent", max_context=256) as lm:
        p = lm.generate(prompt, max_new=128)
    with CausalLm.load(c1_path, kv="f16", decode="layered", max_context=256) as lm:
        q = lm.generate(prompt, max_new=128)
    assert len(p) == 128
    agree = next((i for i, (a, b) in enumerate(zip(p, q)) if a != b), len(p))
    assert agree == len(p), f"persistent and layered differ from token {agree}"
