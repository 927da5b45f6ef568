"""Loading and checking the committed golden fixtures of tests/golden/
(written by tests/golden/make_golden.py from the CPU oracle)."""
from __future__ import annotations

import hashlib
import json
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = os.path.join(HERE, "golden", "greedy.json")


def load() -> dict:
    with open(GOLDEN) as f:
        return json.load(f)


def answer_rows(case: dict, width: int) -> np.ndarray:
    return np.random.default_rng(case["rows_seed"]).normal(0, 1, (case["rows"], width)).astype(np.float32)


def check(case: dict, tokens: list[int], logits: np.ndarray) -> None:
    """Tokens equal; the logits rows of the made tokens bit for bit."""
    assert tokens == case["tokens"], (case["name"], tokens, case["tokens"])
    rows = np.ascontiguousarray(logits[:len(tokens)], dtype="<f4")
    head = [[float(v).hex() for v in row[:4]] for row in rows]
    assert head == case["logits_head"], case["name"]
    assert hashlib.sha256(rows.tobytes()).hexdigest() == case["logits_sha256"], case["name"]
