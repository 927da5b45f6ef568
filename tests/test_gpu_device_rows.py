"""Prompt rows that stay on the GPU (trit_lm_answer_device,
trit_lm_generate_rows_device): Qwen3-ASR hands its encoder's output rows to
the decoder as the prompt (src/models/families/qwen3_asr.rs:321-372,
CausalLm::answer, causal_lm.rs:264-282); an encoder on the same GPU keeps
them there. The device entry points must give what the host ones give."""
import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from trit_b200 import CausalLm, TritError

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("exact", [True, False])
def test_device_rows_match_host_rows(mini_models, exact):
    torch = pytest.importorskip("torch")
    path = mini_models["mini_qwen3_q8_0"]
    oracle = O.Oracle(path)
    rng = np.random.default_rng(17)
    audio = rng.standard_normal((29, oracle.width)).astype(np.float32)
    head, tail = [5, 6, 7], [9, 10, 11]
    want = oracle.answer(head, audio, tail, 24)["tokens"]
    rows_want = oracle.generate_rows(audio, 24)["tokens"]
    with CausalLm.load(path, kv="f32", max_context=256, exact=exact) as lm:
        host = lm.answer(head, audio, tail, max_new=24)
        stream = torch.cuda.Stream()
        with torch.cuda.stream(stream):
            # Written on the caller's stream, as an encoder would: the
            # library orders its reads after this work.
            dev = torch.from_numpy(audio).cuda(non_blocking=True) * 1.0
        got = lm.answer_device(head, dev.data_ptr(), dev.shape[0], tail, max_new=24, stream=stream.cuda_stream)
        assert got == host == want
        assert lm.generate_rows_device(dev.data_ptr(), dev.shape[0], max_new=24) == rows_want
        # Host memory passed as device rows is refused.
        with pytest.raises(TritError, match="not device memory"):
            lm.answer_device(head, audio.ctypes.data_as(ctypes.c_void_p).value, audio.shape[0], tail, max_new=4)
