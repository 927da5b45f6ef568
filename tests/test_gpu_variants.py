"""The rest of the CausalLm interface on the GPU against the oracle:
set_ffn_scales (causal_lm.rs:305-307,458-463), generate_additive
(:317-345, Voxtral Realtime) and bidirectional_tokens (:393-408, Granite
Speech NAR)."""
import numpy as np
import pytest

from oracle import oracle as O
from trit_b200 import CausalLm
from trit_b200.lm import TritError

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("decode", ["persistent", "layered"])
@pytest.mark.parametrize("name", ["mini_qwen3_q8_0", "mini_qwen3_ternary"])
def test_ffn_scales(mini_models, name, decode):
    path = mini_models[name]
    oracle = O.Oracle(path)
    rng = np.random.default_rng(31)
    scales = rng.uniform(0.5, 1.5, (2, oracle.width)).astype(np.float32)
    prompt = rng.integers(0, oracle.vocab, size=30).tolist()
    oracle.set_ffn_scales(scales)
    want = oracle.generate(prompt, 12)["tokens"]
    oracle.set_ffn_scales(None)
    plain = oracle.generate(prompt, 12)["tokens"]
    with CausalLm.load(path, kv="f32", decode=decode, max_context=64) as lm:
        lm.set_ffn_scales(scales)
        assert lm.generate(prompt, max_new=12) == want
        lm.set_ffn_scales(None)
        assert lm.generate(prompt, max_new=12) == plain
        with pytest.raises(TritError, match="layers of width"):
            lm.set_ffn_scales(scales[:, :10])


@pytest.mark.parametrize("name", ["mini_qwen3_q8_0", "mini_mistral_q8_0"])
def test_generate_additive(mini_models, name):
    path = mini_models[name]
    oracle = O.Oracle(path)
    rng = np.random.default_rng(32)
    audio = rng.normal(0, 1, (30, oracle.width)).astype(np.float32)
    prompt = rng.integers(0, oracle.vocab, size=6).tolist()
    ref = oracle.generate_additive(prompt, audio)["tokens"]
    assert len(ref) == 25
    stop = [ref[9]]
    ref_stop = oracle.generate_additive(prompt, audio, stop=stop)["tokens"]
    with CausalLm.load(path, kv="f32", max_context=64) as lm:
        assert lm.generate_additive(prompt, audio) == ref
        assert lm.generate_additive(prompt, audio, stop=stop) == ref_stop
        assert lm.generate_additive(prompt, audio[:5]) == []


@pytest.mark.parametrize("name", ["mini_qwen3_q8_0", "mini_qwen3_int8"])
def test_bidirectional_tokens(mini_models, name):
    path = mini_models[name]
    oracle = O.Oracle(path)
    rows = np.random.default_rng(33).normal(0, 1, (40, oracle.width)).astype(np.float32)
    want = oracle.bidirectional_tokens(rows, 10)
    with CausalLm.load(path, kv="f32", max_context=64, prefill_rows=64) as lm:
        assert lm.bidirectional_tokens(rows, 10) == want
        assert lm.bidirectional_tokens(rows, 40) == []
        # A normal generation afterwards is causal again.
        prompt = [5, 6, 7]
        assert lm.generate(prompt, max_new=5) == oracle.generate(prompt, 5)["tokens"]
