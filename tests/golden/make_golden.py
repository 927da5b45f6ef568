"""Writes tests/golden/greedy.json: the CPU oracle's greedy generations on
the small seeded models, the fixtures that tests/test_cpu_golden.py holds
the oracle to and that the GPU tests compare the CUDA decoder with.

The reference ships no golden vectors for this path, so these pin the
oracle against itself over time and give the GPU tests expected values
that need no oracle at run time. Each case records the model file's
sha256 (which pins the synthesizer), the prompt, the tokens, the sha256 of
all logits rows (f32 little-endian) and the first logits of each row.

Run from the repository root: python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle  # noqa: E402
from tests.synth import presets  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "greedy.json")
MAX_NEW = 12


def cases():
    """(name, model, kv, kind, prompt args) for every golden case."""
    rng = np.random.default_rng(20261201)
    out = []
    for model in ("mini_qwen3_q8_0", "mini_qwen3_int8", "mini_qwen3_ternary", "mini_mistral_q8_0",
                  "mini_granite_q8_0"):
        vocab = presets.CONFIGS[model][0]["vocab_size"]
        for kv in ("f32", "f16"):
            prompt = rng.integers(0, vocab, 24).tolist()
            out.append({"name": f"{model}/{kv}/generate", "model": model, "kv": kv, "kind": "generate",
                        "prompt": prompt})
    d = presets.CONFIGS["mini_qwen3_q8_0"][0]["hidden_size"]
    rows = rng.normal(0, 1, (20, d)).astype(np.float32)
    out.append({"name": "mini_qwen3_q8_0/f32/answer", "model": "mini_qwen3_q8_0", "kv": "f32", "kind": "answer",
                "head": [11, 12, 13], "rows_seed": 7, "rows": 20, "tail": [21, 22]})
    return out


def answer_rows(case) -> np.ndarray:
    d = presets.CONFIGS[case["model"]][0]["hidden_size"]
    return np.random.default_rng(case["rows_seed"]).normal(0, 1, (case["rows"], d)).astype(np.float32)


def run(case) -> dict:
    folder = presets.model_path(case["model"])
    o = oracle.Oracle(folder, kv_f16=case["kv"] == "f16")
    try:
        if case["kind"] == "generate":
            r = o.generate(case["prompt"], MAX_NEW, trace=True)
        else:
            r = o.answer(case["head"], answer_rows(case), case["tail"], MAX_NEW, trace=True)
    finally:
        o.close()
    n = len(r["tokens"])
    logits = np.ascontiguousarray(r["logits"][:n], dtype="<f4")
    return {"tokens": r["tokens"], "logits_sha256": hashlib.sha256(logits.tobytes()).hexdigest(),
            "logits_head": [[float(v).hex() for v in row[:4]] for row in logits]}


def gguf_sha256(model: str) -> str:
    h = hashlib.sha256()
    with open(os.path.join(presets.model_path(model), "model.gguf"), "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def main():
    out = {"max_new": MAX_NEW, "models": {}, "cases": []}
    for case in cases():
        if case["model"] not in out["models"]:
            out["models"][case["model"]] = gguf_sha256(case["model"])
        case = dict(case, **run(case))
        out["cases"].append(case)
        print(case["name"], case["tokens"])
    with open(OUT, "w") as f:
        json.dump(out, f, indent=1)
        f.write("\n")


if __name__ == "__main__":
    main()
