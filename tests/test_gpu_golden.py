"""The CUDA decoder against the committed golden fixtures, through the C ABI
(trit_lm_generate_traced / trit_lm_answer_traced): on the exact paths
(layered, persistent with "exact": true) greedy tokens equal and logits
bit-identical; on the default persistent decode (tree-order sums) the
tokens equal."""
import pytest

from tests import golden_cases
from trit_b200 import lm
from tests.synth import presets

GOLDEN = golden_cases.load()


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["persistent-exact", "layered", "persistent"])
@pytest.mark.parametrize("case", GOLDEN["cases"], ids=[c["name"] for c in GOLDEN["cases"]])
def test_cuda_reproduces_golden(case, mode):
    opts = {"decode": "layered" if mode == "layered" else "persistent", "exact": mode != "persistent"}
    with lm.CausalLm.load(presets.model_path(case["model"]), kv=case["kv"], max_context=256, **opts) as m:
        if case["kind"] == "generate":
            tokens, logits = m.generate_traced(case["prompt"], max_new=GOLDEN["max_new"])
        else:
            tokens, logits = m.answer(case["head"], golden_cases.answer_rows(case, m.width()), case["tail"],
                                      max_new=GOLDEN["max_new"], trace=True)
    if mode == "persistent":
        assert tokens == case["tokens"], (case["name"], tokens, case["tokens"])
    else:
        golden_cases.check(case, tokens, logits)
