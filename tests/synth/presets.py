"""The model shapes and workloads of the benchmark configurations: Qwen3
0.6B / 1.7B and Ministral-3B shaped decoders with synthetic weights, and
small shapes of the same families for the parity tests."""
from __future__ import annotations

import hashlib
import json
import os

QWEN3_06B = {
    "model_type": "qwen3", "hidden_size": 1024, "intermediate_size": 3072, "num_hidden_layers": 28,
    "num_attention_heads": 16, "num_key_value_heads": 8, "head_dim": 128, "vocab_size": 151936,
    "rms_norm_eps": 1e-6, "rope_theta": 1e6, "tie_word_embeddings": True,
}
QWEN3_17B = dict(QWEN3_06B, hidden_size=2048, intermediate_size=6144)
MINISTRAL_3B = {
    "model_type": "mistral", "hidden_size": 3072, "intermediate_size": 8192, "num_hidden_layers": 30,
    "num_attention_heads": 32, "num_key_value_heads": 8, "head_dim": 128, "vocab_size": 131072,
    "rms_norm_eps": 1e-6, "rope_theta": 1e6, "tie_word_embeddings": False,
}

# Small shapes of the same families: fast on the CPU oracle.
MINI_QWEN3 = dict(QWEN3_06B, hidden_size=256, intermediate_size=768, num_hidden_layers=2,
                  num_attention_heads=4, num_key_value_heads=2, vocab_size=4096)
MINI_MISTRAL = dict(MINISTRAL_3B, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                    num_attention_heads=4, num_key_value_heads=1, vocab_size=2048)

MINI_GRANITE = dict(MINI_QWEN3, model_type="granite", embedding_multiplier=2.0, attention_multiplier=0.0078125,
                    residual_multiplier=0.8, logits_scaling=4.0)
# Eight query heads a kv head, and one (plain multi-head attention).
MINI_GQA8 = dict(MINI_QWEN3, num_attention_heads=8, num_key_value_heads=1)
MINI_MHA = dict(MINI_QWEN3, num_attention_heads=4, num_key_value_heads=4)

CONFIGS = {
    # name: (config, format, seed)
    "c1_qwen3_0.6b_q8_0": (QWEN3_06B, "q8_0", 20261201),
    "c2_qwen3_0.6b_int8": (QWEN3_06B, "int8", 20261202),
    "c3_qwen3_1.7b_ternary": (QWEN3_17B, "ternary", 20261203),
    "c5_ministral_3b_q8_0": (MINISTRAL_3B, "q8_0", 20261205),
    "mini_qwen3_q8_0": (MINI_QWEN3, "q8_0", 7),
    "mini_qwen3_int8": (MINI_QWEN3, "int8", 8),
    "mini_qwen3_ternary": (MINI_QWEN3, "ternary", 9),
    "mini_mistral_q8_0": (MINI_MISTRAL, "q8_0", 10),
    "mini_granite_q8_0": (MINI_GRANITE, "q8_0", 11),
    "mini_gqa8_q8_0": (MINI_GQA8, "q8_0", 12),
    "mini_mha_q8_0": (MINI_MHA, "q8_0", 13),
}


# The small models draw their weights wider than N(0, 0.02): with tied
# embeddings a narrow draw leaves the last token's embedding dominant and
# the greedy loop repeats one token, which tests the loop poorly.
MINI_STD = 0.15


def weight_std(name: str) -> float:
    return MINI_STD if name.startswith("mini_") else 0.02


def cache_dir() -> str:
    return os.environ.get("TRIT_MODEL_CACHE", os.path.join("/tmp", "trit_b200_models"))


def model_path(name: str) -> str:
    """The folder of a synthetic model, written on first use."""
    from . import synthesize

    config, fmt, seed = CONFIGS[name]
    std = weight_std(name)
    spec = {"c": config, "f": fmt, "s": seed}
    if std != 0.02:
        spec["std"] = std
    spec = json.dumps(spec, sort_keys=True).encode()
    folder = os.path.join(cache_dir(), f"{name}-{hashlib.sha1(spec).hexdigest()[:10]}")
    done = os.path.join(folder, ".complete")
    if not os.path.exists(done):
        os.makedirs(folder, exist_ok=True)
        synthesize(folder, config, fmt, seed, std=std)
        open(done, "w").close()
    return folder
