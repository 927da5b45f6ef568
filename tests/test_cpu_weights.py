"""The weight formats on the CPU: synthetic model folders hold the bytes the
reference's quantizers would write, and the oracle reads them back as the
reference does. Each restatement here is numpy, written from the reference:
  Q8_0 blocks     Blocks::quantize, src/cpu/gemm.rs:53-76 (ggml's
                  quantize_row_q8_0_ref: d = max|x|/127 in f32, codes
                  round-half-away(x * (1/d)), d stored as f16)
  per-row int8    group_scale / quantize_code, src/cpu/int8.rs:176-186
                  (scale = max/127 or 1, codes round-half-even, clamp +-127)
  int8 table      Q8::quantize, src/cpu/gemm.rs:117-150 (the same per 32)
  ternary         five base-3 digits a byte, low digit first
                  (DIGITS, src/cpu/kernels.rs:630-643), bytes < 243
"""
import os

import numpy as np
import pytest

from tests.gguf_read import GGML_F32, GGML_I8, GGML_Q8_0, Gguf
from trit_b200 import lm
from tests import synth
from tests.synth import presets


def q8_0_numpy(v: np.ndarray):
    v = v.astype(np.float32).reshape(-1, 32)
    mx = np.abs(v).max(axis=1)
    d = (mx / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, np.float32(1.0) / d, np.float32(0.0)).astype(np.float32)
    prod = (v * inv[:, None]).astype(np.float32)
    codes = (np.sign(prod) * np.floor(np.abs(prod) + np.float32(0.5))).astype(np.float32)  # half away from zero
    codes = np.clip(codes, -128, 127).astype(np.int8)
    return codes.reshape(-1), d.astype(np.float16)


def row_int8_numpy(v: np.ndarray):
    mx = np.float32(np.abs(v).max())
    scale = np.float32(mx / np.float32(127.0)) if mx > 0 else np.float32(1.0)
    codes = np.clip(np.rint((v / scale).astype(np.float32)), -127, 127).astype(np.int8)
    return codes, scale


@pytest.fixture(scope="module")
def folders():
    return {n: presets.model_path(n) for n in ("mini_qwen3_q8_0", "mini_qwen3_int8", "mini_qwen3_ternary",
                                               "mini_mistral_q8_0")}


def test_normal_rows_are_seeded_and_normal():
    a = synth.normal_row(5, "w", 3, 4096)
    b = synth.normal_row(5, "w", 3, 4096)
    c = synth.normal_row(5, "w", 4, 4096)
    assert np.array_equal(a, b) and not np.array_equal(a, c)
    assert abs(a.mean()) < 0.02 * 0.1 and abs(a.std() - 0.02) < 0.02 * 0.05


def test_tensor_names_types_and_shapes(folders):
    for name, folder in folders.items():
        cfg, fmt, _ = presets.CONFIGS[name]
        g = Gguf(os.path.join(folder, "model.gguf"))
        d, hd, ffn = cfg["hidden_size"], cfg["head_dim"], cfg["intermediate_size"]
        qd, kvd = cfg["num_attention_heads"] * hd, cfg["num_key_value_heads"] * hd
        for l in range(cfg["num_hidden_layers"]):
            p = f"model.layers.{l}"
            for part, n, k in (("self_attn.q_proj", qd, d), ("self_attn.k_proj", kvd, d), ("self_attn.v_proj", kvd, d),
                               ("self_attn.o_proj", d, qd), ("mlp.gate_proj", ffn, d), ("mlp.up_proj", ffn, d),
                               ("mlp.down_proj", d, ffn)):
                if fmt == "q8_0":
                    dims, typ, _ = g.tensors[f"{p}.{part}.weight"]
                    assert (dims, typ) == ([k, n], GGML_Q8_0)
                elif fmt == "int8":
                    assert g.tensors[f"{p}.{part}.weight"][:2] == ([k, n], GGML_I8)
                    assert g.tensors[f"{p}.{part}.scales"][:2] == ([n], GGML_F32)
                else:
                    assert g.tensors[f"{p}.{part}.qweight"][:2] == ([(k + 4) // 5, n], GGML_I8)
                    assert g.tensors[f"{p}.{part}.scales"][:2] == ([k // 128, n], GGML_F32)
            assert (f"{p}.self_attn.q_norm.weight" in g.tensors) == (cfg["model_type"] == "qwen3")
        assert ("lm_head.weight" in g.tensors) == (not cfg["tie_word_embeddings"])


def test_q8_0_blocks_are_the_reference_quantizer(folders):
    g = Gguf(os.path.join(folders["mini_qwen3_q8_0"], "model.gguf"))
    seed = presets.CONFIGS["mini_qwen3_q8_0"][2]
    for name, rows in (("model.layers.0.self_attn.q_proj", [0, 1, 511]), ("model.layers.1.mlp.down_proj", [0, 255]),
                       ("model.embed_tokens", [0, 17, 4095])):
        codes, scales = g.q8_0(name + ".weight")
        for r in rows:
            v = synth.normal_row(seed, name, r, codes.shape[1], presets.MINI_STD)
            c, s = q8_0_numpy(v)
            assert np.array_equal(codes[r], c), (name, r)
            assert np.array_equal(scales[r].view(np.uint16), s.view(np.uint16)), (name, r)


def test_q8_0_quantizer_edges():
    # Ties away from zero, zero blocks, a lone maximum, the +-127 ends.
    from oracle import oracle

    cases = [np.zeros(32, np.float32), np.full(32, 1.0, np.float32), np.linspace(-1, 1, 32, dtype=np.float32),
             np.array([127.0, 0.5, -0.5, 1.5, -1.5, 2.5] + [0.0] * 26, np.float32),
             np.array([3e-8] + [0.0] * 31, np.float32), np.array([-65504.0] + [1.0] * 31, np.float32)]
    rng = np.random.default_rng(3)
    cases += [rng.normal(0, 1, 32).astype(np.float32) for _ in range(64)]
    for v in cases:
        c, s = q8_0_numpy(v)
        oc, os_ = oracle.q8_0_quantize(v)
        assert np.array_equal(oc, c) and np.array_equal(os_, s.view(np.uint16)), v


def test_int8_rows_and_table(folders):
    g = Gguf(os.path.join(folders["mini_qwen3_int8"], "model.gguf"))
    seed = presets.CONFIGS["mini_qwen3_int8"][2]
    name = "model.layers.0.mlp.gate_proj"
    codes, scales = g.array(name + ".weight"), g.array(name + ".scales")
    for r in (0, 5, 767):
        c, s = row_int8_numpy(synth.normal_row(seed, name, r, codes.shape[1], presets.MINI_STD))
        assert np.array_equal(codes[r], c) and scales[r] == s
    tcodes, tscales = g.array("model.embed_tokens.weight"), g.array("model.embed_tokens.scales")
    for r in (0, 4095):
        v = synth.normal_row(seed, "model.embed_tokens", r, tcodes.shape[1], presets.MINI_STD)
        for grp in range(tcodes.shape[1] // 32):
            c, s = row_int8_numpy(v[grp * 32:(grp + 1) * 32])
            assert np.array_equal(tcodes[r, grp * 32:(grp + 1) * 32], c) and tscales[r, grp] == s


def test_ternary_digits_and_statistics(folders):
    from oracle import oracle

    g = Gguf(os.path.join(folders["mini_qwen3_ternary"], "model.gguf"))
    name = "model.layers.0.mlp.gate_proj"
    packed = g.array(name + ".qweight").view(np.uint8)
    assert packed.max() < 243
    # Five base-3 digits a byte, the low digit first.
    digits = np.stack([(packed.astype(np.int32) // 3 ** i) % 3 for i in range(5)], axis=-1).reshape(packed.shape[0], -1)
    k = 256
    codes = digits[:, :k] - 1
    frac0 = (codes == 0).mean()
    assert abs(frac0 - 0.4) < 0.02 and abs((codes == 1).mean() - 0.3) < 0.02
    for b in (0, 1, 2, 80, 242):
        out = (np.zeros(5, np.uint8))
        oracle.lib().oracle_base3(b, out.ctypes.data_as(oracle._u8p))
        assert out.tolist() == [(b // 3 ** i) % 3 for i in range(5)]
    scales = g.array(name + ".scales")
    assert np.all(scales == scales[:, :1]) and np.all(scales > 0)


def test_inspect_reads_settings_without_a_gpu(folders):
    info = lm.inspect(folders["mini_qwen3_q8_0"])
    assert info["model_type"] == "qwen3" and info["qk_norm"] and info["tie_word_embeddings"]
    assert info["products"] == "q8_0" and info["output_table"] == "q8_0" and not info["separate_head"]
    cfg = presets.MINI_QWEN3
    d, ffn, L = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"]
    weights = L * ((512 + 512) * d + d * 512 + 2 * ffn * d + d * ffn)  # q 512, k+v 2x256, o, gate_up, down
    assert info["product_bytes"] == weights * 34 // 32
    info = lm.inspect(folders["mini_mistral_q8_0"])
    assert info["model_type"] == "mistral" and not info["qk_norm"] and info["separate_head"]
    assert lm.inspect(folders["mini_qwen3_ternary"])["products"] == "ternary"
    assert lm.inspect(folders["mini_qwen3_int8"])["token_table"] == "int8"
