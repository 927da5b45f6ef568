"""Real model files on the GPU: the same seeded decoder as model.gguf with
Hugging Face names, as safetensors (f32 weights quantized to Q8_0 at load
as ggml quantizes them; int8 as stored) and as a transcribe.cpp GGUF file
(dec.* names, settings in metadata) gives the same logits bit for bit; and
the weight cache (the device layout kept in a file, src/cpu/store.rs) gives
what a fresh load gives, and is rewritten when its file is damaged."""
import os
import tempfile

import numpy as np
import pytest

from tests import synth
from tests.synth import presets
from trit_b200 import CausalLm

pytestmark = pytest.mark.gpu

CFG = dict(presets.MINI_QWEN3, num_hidden_layers=2, vocab_size=1024)
SEED = 43
PROMPT = list(range(3, 40))


def traced(path, **opts):
    with CausalLm.load(path, kv="f32", max_context=128, exact=True, **opts) as lm:
        toks, logits = lm.generate_traced(PROMPT, max_new=12)
        return toks, logits[: len(toks)], lm.status()


@pytest.mark.parametrize("fmt", ["q8_0", "int8"])
def test_file_forms_give_the_same_logits(fmt):
    with tempfile.TemporaryDirectory() as tmp:
        base = synth.synthesize(os.path.join(tmp, "gguf"), CFG, fmt, SEED, std=presets.MINI_STD)
        forms = [synth.synthesize(os.path.join(tmp, "st"), CFG, "float" if fmt == "q8_0" else fmt, SEED,
                                  std=presets.MINI_STD, container="safetensors")]
        if fmt == "q8_0":
            forms.append(synth.synthesize(os.path.join(tmp, "tc"), CFG, fmt, SEED, std=presets.MINI_STD,
                                          names="transcribe", arch="qwen3_asr"))
        want_toks, want_logits, st = traced(base)
        assert st["source"] == "gguf" and st["weights_from"] == "files"
        for path in forms:
            toks, logits, st = traced(path)
            assert toks == want_toks, st["source"]
            assert np.array_equal(logits, want_logits), st["source"]


def test_weight_cache_round_trip():
    with tempfile.TemporaryDirectory() as tmp:
        path = synth.synthesize(os.path.join(tmp, "m"), CFG, "q8_0", SEED, std=presets.MINI_STD)
        want = traced(path)
        first = traced(path, weight_cache=True)
        assert first[2]["weights_from"] == "files" and os.path.exists(first[2]["weight_cache"])
        second = traced(path, weight_cache=True)
        assert second[2]["weights_from"] == "cache" and second[2]["weight_cache"] == first[2]["weight_cache"]
        for got in (first, second):
            assert got[0] == want[0] and np.array_equal(got[1], want[1])
        # A damaged file is not used: the load converts the files again and
        # rewrites it.
        cache = second[2]["weight_cache"]
        raw = bytearray(open(cache, "rb").read())
        raw[len(raw) // 2] ^= 0xFF
        open(cache, "wb").write(bytes(raw))
        third = traced(path, weight_cache=True)
        assert third[2]["weights_from"] == "files"
        assert third[0] == want[0] and np.array_equal(third[1], want[1])
        assert traced(path, weight_cache=True)[2]["weights_from"] == "cache"
