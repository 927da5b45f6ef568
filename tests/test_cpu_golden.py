"""The CPU oracle against the committed golden fixtures (tests/golden/,
made by tests/golden/make_golden.py): the synthetic model files are the
same bytes, and the oracle's greedy tokens and logits are the same bits.
A change to the oracle or the synthesizer that moves a single bit fails
here first."""
import hashlib
import os

import pytest

from oracle import oracle
from tests import golden_cases
from tests.synth import presets

GOLDEN = golden_cases.load()


@pytest.mark.parametrize("model", sorted(GOLDEN["models"]))
def test_model_files_are_the_golden_bytes(model):
    h = hashlib.sha256()
    with open(os.path.join(presets.model_path(model), "model.gguf"), "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    assert h.hexdigest() == GOLDEN["models"][model]


@pytest.mark.parametrize("case", GOLDEN["cases"], ids=[c["name"] for c in GOLDEN["cases"]])
def test_oracle_reproduces_golden(case):
    o = oracle.Oracle(presets.model_path(case["model"]), kv_f16=case["kv"] == "f16")
    try:
        if case["kind"] == "generate":
            r = o.generate(case["prompt"], GOLDEN["max_new"], trace=True)
        else:
            r = o.answer(case["head"], golden_cases.answer_rows(case, o.width), case["tail"], GOLDEN["max_new"],
                         trace=True)
    finally:
        o.close()
    golden_cases.check(case, r["tokens"], r["logits"])


def test_oracle_scalar_path_reproduces_golden():
    """The scalar (non-VNNI) products give the same bits as the VNNI tile."""
    case = GOLDEN["cases"][0]
    oracle.lib().oracle_force_scalar(1)
    try:
        o = oracle.Oracle(presets.model_path(case["model"]), kv_f16=case["kv"] == "f16")
        r = o.generate(case["prompt"], GOLDEN["max_new"], trace=True)
        o.close()
    finally:
        oracle.lib().oracle_force_scalar(0)
    golden_cases.check(case, r["tokens"], r["logits"])
