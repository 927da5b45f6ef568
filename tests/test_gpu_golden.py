"""The CUDA decoder against the committed golden fixtures: for every golden
case, greedy tokens equal and logits bit-identical, through the C ABI
(trit_lm_generate_traced / trit_lm_answer_traced), with both decode paths."""
import pytest

from tests import golden_cases
from trit_b200 import lm
from tests.synth import presets

GOLDEN = golden_cases.load()


@pytest.mark.gpu
@pytest.mark.parametrize("decode", ["persistent", "layered"])
@pytest.mark.parametrize("case", GOLDEN["cases"], ids=[c["name"] for c in GOLDEN["cases"]])
def test_cuda_reproduces_golden(case, decode):
    with lm.CausalLm.load(presets.model_path(case["model"]), kv=case["kv"], decode=decode, max_context=256) as m:
        if case["kind"] == "generate":
            tokens, logits = m.generate_traced(case["prompt"], max_new=GOLDEN["max_new"])
        else:
            tokens, logits = m.answer(case["head"], golden_cases.answer_rows(case, m.width()), case["tail"],
                                      max_new=GOLDEN["max_new"], trace=True)
    golden_cases.check(case, tokens, logits)
