"""The three forms of a model folder that the library reads
(include/trit_cuda.h), described without a GPU: config.json + model.gguf,
config.json + safetensors (float weights quantized to Q8_0 at load, as
ggml quantizes; or int8), and one GGUF file as transcribe.cpp writes it
(settings from stt.<arch>.decoder.* metadata, dec.* names mapped as
src/models/gguf/qwen3_asr.rs:103-136 maps them). Each form of the same
seeded model has the same settings and the same device bytes."""
import json
import os
import struct
import tempfile

import pytest

from tests import synth
from tests.synth import presets
from trit_b200 import lm

CFG = dict(presets.MINI_QWEN3, num_hidden_layers=1, vocab_size=512)
SEED = 41


def folder(tmp, name, fmt, **extra):
    path = os.path.join(tmp, name)
    synth.synthesize(path, CFG, fmt, SEED, std=presets.MINI_STD, **extra)
    return path


@pytest.fixture(scope="module")
def forms():
    with tempfile.TemporaryDirectory() as tmp:
        yield {
            "gguf": folder(tmp, "gguf", "q8_0"),
            "safetensors_f32": folder(tmp, "st32", "float", container="safetensors", dtype="f32"),
            "safetensors_bf16": folder(tmp, "stbf", "float", container="safetensors", dtype="bf16"),
            "safetensors_int8": folder(tmp, "st8", "int8", container="safetensors"),
            "transcribe": folder(tmp, "tc", "q8_0", names="transcribe", arch="qwen3_asr"),
            "transcribe_voxtral": folder(tmp, "vx", "q8_0", names="transcribe", arch="voxtral"),
        }


SETTINGS = ["model_type", "hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads",
            "num_key_value_heads", "head_dim", "vocab_size", "rms_norm_eps", "rope_theta", "qk_norm",
            "tie_word_embeddings"]


def test_every_form_describes_the_same_decoder(forms):
    base = lm.inspect(forms["gguf"])
    assert base["source"] == "gguf"
    for name in ["safetensors_f32", "safetensors_bf16", "transcribe"]:
        info = lm.inspect(forms[name])
        assert {k: info[k] for k in SETTINGS} == {k: base[k] for k in SETTINGS}, name
        assert info["products"] == "q8_0" and info["product_bytes"] == base["product_bytes"], name
    assert lm.inspect(forms["safetensors_f32"])["source"] == "safetensors"
    int8 = lm.inspect(forms["safetensors_int8"])
    assert int8["products"] == "int8" and int8["token_table"] == "int8"
    tc = lm.inspect(forms["transcribe"])
    assert tc["source"] == "gguf-transcribe" and tc["tensor_prefix"] == "thinker."
    vx = lm.inspect(forms["transcribe_voxtral"])
    # Voxtral's decoder is a Mistral: no q/k norms, its own prefix.
    assert vx["model_type"] == "mistral" and not vx["qk_norm"] and vx["tensor_prefix"] == "language_model."


def test_transcribe_file_needs_a_known_architecture(forms, tmp_path):
    src = os.path.join(forms["transcribe"], "qwen3_asr.gguf")
    data = open(src, "rb").read().replace(b"qwen3_asr", b"qwen9_asr")
    (tmp_path / "m.gguf").write_bytes(data)
    with pytest.raises(lm.TritError, match="qwen3_asr, moss"):
        lm.inspect(str(tmp_path))


def test_safetensors_header_is_checked(forms, tmp_path):
    raw = open(os.path.join(forms["safetensors_f32"], "model.safetensors"), "rb").read()
    (tmp_path / "config.json").write_text(open(os.path.join(forms["safetensors_f32"], "config.json")).read())
    # A file cut short: a tensor's byte range runs past the end.
    (tmp_path / "model.safetensors").write_bytes(raw[: len(raw) // 2])
    with pytest.raises(lm.TritError, match="byte range"):
        lm.inspect(str(tmp_path))
    # A header length past the end of the file.
    (tmp_path / "model.safetensors").write_bytes(struct.pack("<Q", 1 << 40) + b"{}")
    with pytest.raises(lm.TritError, match="header runs past"):
        lm.inspect(str(tmp_path))


def test_sharded_safetensors_follow_the_index(forms, tmp_path):
    """model.safetensors.index.json names the shards (a split checkpoint)."""
    src = forms["safetensors_f32"]
    raw = open(os.path.join(src, "model.safetensors"), "rb").read()
    n = struct.unpack("<Q", raw[:8])[0]
    header = json.loads(raw[8:8 + n])
    data = raw[8 + n:]
    names = [k for k in header if k != "__metadata__"]
    shards = [names[: len(names) // 2], names[len(names) // 2:]]
    weight_map = {}
    for i, part in enumerate(shards):
        at, h, blobs = 0, {}, []
        for name in part:
            b, e = header[name]["data_offsets"]
            h[name] = dict(header[name], data_offsets=[at, at + e - b])
            blobs.append(data[b:e])
            at += e - b
            weight_map[name] = f"part-{i}.safetensors"
        text = json.dumps(h).encode()
        (tmp_path / f"part-{i}.safetensors").write_bytes(struct.pack("<Q", len(text)) + text + b"".join(blobs))
    (tmp_path / "model.safetensors.index.json").write_text(json.dumps({"weight_map": weight_map}))
    (tmp_path / "config.json").write_text(open(os.path.join(src, "config.json")).read())
    info = lm.inspect(str(tmp_path))
    assert info["source"] == "safetensors" and info["product_bytes"] == lm.inspect(src)["product_bytes"]
