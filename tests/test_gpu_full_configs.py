"""Every benchmarked configuration against the CPU oracle at its real
shape: the tokens the bench times must be the reference decoder's tokens.

- C1 (Qwen3-0.6B shape, Q8_0, batch 1): a 64-id prompt, all 128 greedy
  tokens, f16 KV, through the persistent decode the bench runs: the default
  exact path (logits bit for bit) and the tree-order path (tokens, cosine,
  drift recorded).
- C3 (Qwen3-1.7B shape, ternary): `answer` with 375 N(0,1) rows and 16
  ids, 200 greedy tokens.
- C2 (0.6B, per-row int8, 16 streams of 256 ids, 256 steps) and C5
  (Ministral-3B shape, Q8_0, 64 streams): two streams of the batched
  decode against the oracle's single-stream generation. C5's prompts are
  64 ids instead of 1024 (the oracle's 1024-id prefill of the 3B model
  takes minutes) and it runs 32 steps.

Each test records the oracle's top-1/top-2 logit gap at every step: a
token can only flip where that gap is below the logit error, so the
smallest gap says how close a configuration runs to a near-tie. The gaps
are printed (pytest -s) and, when TRIT_PARITY_LOG names a file, appended
to it as JSON lines.
"""
import json
import os

import numpy as np
import pytest

from oracle import oracle as O
from tests.synth import presets
from trit_b200 import CausalLm

pytestmark = pytest.mark.gpu

# The north-star bar for logits. The exact paths (the default) meet it bit
# for bit; the tree-order decode ("exact": false) keeps the tokens and the
# cosine but its logits drift past the max-abs bar (a reordered sum moves
# int8 activation codes; the oracle with only its RmsNorm sum reordered
# drifts 0.046 on C1), so it is held to TREE_MAX_ABS and the drift is
# recorded.
MAX_ABS = 2e-2
MIN_COS = 0.9995
TREE_MAX_ABS = 0.1


def gaps(logits: np.ndarray) -> np.ndarray:
    s = np.sort(logits, axis=1)
    return s[:, -1] - s[:, -2]


def record(name: str, tokens: int, gap: np.ndarray, **extra) -> None:
    entry = {"config": name, "tokens": tokens, "min_gap": float(gap.min()), "min_gap_step": int(gap.argmin()),
             "median_gap": float(np.median(gap)), **extra}
    print(json.dumps(entry))
    path = os.environ.get("TRIT_PARITY_LOG")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps(entry) + "\n")


def compare(name: str, toks, logits, want: dict, exact: bool) -> None:
    ref_toks = want["tokens"]
    ref_logits = want["logits"][: len(ref_toks)]
    gap = gaps(ref_logits)
    first = next((i for i, (a, b) in enumerate(zip(toks, ref_toks)) if a != b), None)
    assert len(toks) == len(ref_toks) and first is None, (
        f"{name}: tokens differ from step {first} (oracle gap there {gap[first] if first is not None else None})")
    n = len(toks)
    got = logits[:n]
    err = float(np.abs(got - ref_logits).max())
    cos = float(np.min(np.sum(got * ref_logits, axis=1) /
                       (np.linalg.norm(got, axis=1) * np.linalg.norm(ref_logits, axis=1))))
    record(name, n, gap, max_abs=err, min_cos=cos, exact=exact)
    if exact:
        assert np.array_equal(got, ref_logits), f"{name}: logits differ by {err}"
    else:
        assert err <= TREE_MAX_ABS and cos >= MIN_COS, f"{name}: max |dlogit| {err}, min cosine {cos}"


@pytest.fixture(scope="module")
def c1():
    path = presets.model_path("c1_qwen3_0.6b_q8_0")
    prompt = np.random.default_rng(2).integers(0, 151936, size=64).tolist()
    want = O.Oracle(path, kv_f16=True).generate(prompt, 128, trace=True)
    return path, prompt, want


@pytest.mark.parametrize("exact", [False, True])
def test_c1_all_128_tokens_f16_kv(c1, exact):
    path, prompt, want = c1
    with CausalLm.load(path, kv="f16", decode="persistent", exact=exact, max_context=256) as lm:
        toks, logits = lm.generate_traced(prompt, max_new=128)
        # The untraced call (what the bench times) makes the same tokens.
        assert lm.generate(prompt, max_new=128) == toks
    compare("c1" + ("_exact" if exact else ""), toks, logits, want, exact)


def test_c3_answer_391_rows_200_tokens():
    path = presets.model_path("c3_qwen3_1.7b_ternary")
    rows = np.random.default_rng(3).normal(0, 1, (375, 2048)).astype(np.float32)
    tail = np.random.default_rng(4).integers(0, 151936, size=16).tolist()
    want = O.Oracle(path, kv_f16=True).answer([], rows, tail, 200, trace=True)
    with CausalLm.load(path, kv="f16", max_context=640) as lm:
        toks, logits = lm.answer([], rows, tail, max_new=200, trace=True)
        assert lm.answer([], rows, tail, max_new=200) == toks
    compare("c3", toks, logits, want, exact=True)


def batch_against_oracle(name: str, model: str, streams: int, prompt_len: int, new: int, check: list) -> None:
    path = presets.model_path(model)
    vocab = presets.CONFIGS[model][0]["vocab_size"]
    rng = np.random.default_rng(sum(map(ord, name)))
    prompts = [rng.integers(0, vocab, size=prompt_len).tolist() for _ in range(streams)]
    with CausalLm.load(path, kv="f16", max_streams=streams, max_context=prompt_len + new + 8,
                       prefill_rows=max(4096, streams)) as lm:
        got = lm.generate_batch(prompts, max_new=new)
    orc = O.Oracle(path, kv_f16=True)
    for s in check:
        want = orc.generate(prompts[s], new, trace=True)
        gap = gaps(want["logits"][: len(want["tokens"])])
        first = next((i for i, (a, b) in enumerate(zip(got[s], want["tokens"])) if a != b), None)
        record(f"{name}_stream{s}", len(want["tokens"]), gap)
        assert got[s] == want["tokens"], f"{name} stream {s}: tokens differ from step {first}"
    orc.close()


def test_c2_two_of_16_streams_256_steps():
    batch_against_oracle("c2", "c2_qwen3_0.6b_int8", 16, 256, 256, [0, 15])


def test_c5_two_of_64_streams():
    batch_against_oracle("c5", "c5_ministral_3b_q8_0", 64, 64, 32, [0, 63])


# The tensor-core prompt attention (`"tc_attention": true`: f16 operands, the
# tensor cores' sums, a per-tile softmax) is not the reference's arithmetic:
# its logits drift, and where the oracle's top-1/top-2 gap is small a token
# can flip (C5 stream 0 flips at step 12, where the oracle's gap is 0.127;
# max-abs 0.29 and cosine 0.9983 by then). These tests record the drift up
# to and including the first differing step and hold it to TC_MAX_ABS /
# MIN_TC_COS, bounds well outside the north star's logit bar; the
# benchmarks' default numbers come from the exact path.
TC_MAX_ABS = 0.5
MIN_TC_COS = 0.995


def drift_until_divergence(name: str, toks, logits, want: dict) -> None:
    ref_toks = want["tokens"]
    n = min(len(toks), len(ref_toks))
    first = next((i for i in range(n) if toks[i] != ref_toks[i]), None)
    upto = n if first is None else first + 1  # the step that flips still has the same prefix
    got, ref = logits[:upto], want["logits"][:upto]
    gap = gaps(want["logits"][: len(ref_toks)])
    err = float(np.abs(got - ref).max())
    cos = float(np.min(np.sum(got * ref, axis=1) / (np.linalg.norm(got, axis=1) * np.linalg.norm(ref, axis=1))))
    record(name, n, gap, max_abs=err, min_cos=cos, exact=False, first_difference=first,
           gap_there=None if first is None else float(gap[first]))
    assert err <= TC_MAX_ABS and cos >= MIN_TC_COS, f"{name}: max |dlogit| {err}, min cosine {cos}"


def test_c5_tensor_core_prompt_attention_drift():
    """`"tc_attention": true` on C5 (stream 0's 64-id prompt of the batch test):
    the prompt's attention on the tensor cores, the decode steps exact."""
    path = presets.model_path("c5_ministral_3b_q8_0")
    rng = np.random.default_rng(sum(map(ord, "c5")))
    prompt = rng.integers(0, presets.CONFIGS["c5_ministral_3b_q8_0"][0]["vocab_size"], size=64).tolist()
    want = O.Oracle(path, kv_f16=True).generate(prompt, 32, trace=True)
    with CausalLm.load(path, kv="f16", decode="layered", exact=False, tc_attention=True, max_context=128) as lm:
        toks, logits = lm.generate_traced(prompt, max_new=32)
    drift_until_divergence("c5_tc_prompt", toks, logits, want)


def test_c1_tensor_core_prompt_attention_drift():
    """`"tc_attention": true` with layered decode on C1: only the prompt's attention
    (300 ids, three 128-key tiles) runs in another order."""
    path = presets.model_path("c1_qwen3_0.6b_q8_0")
    prompt = np.random.default_rng(5).integers(0, 151936, size=300).tolist()
    want = O.Oracle(path, kv_f16=True).generate(prompt, 32, trace=True)
    with CausalLm.load(path, kv="f16", decode="layered", exact=False, tc_attention=True, max_context=400) as lm:
        toks, logits = lm.generate_traced(prompt, max_new=32)
    drift_until_divergence("c1_tc_prompt", toks, logits, want)
