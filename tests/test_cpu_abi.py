"""The C ABI of libtrit_cuda.so on a host without a GPU: every function
that include/*.h declares is exported, the Python signatures cover them,
and the calls that need no GPU (options, config parsing, argument checks,
model description) behave as the reference's interface does: a failure
returns NULL or -1 with the reason in trit_cuda_last_error (include/trit.h:7-18,
ffi/src/lib.rs:20-45)."""
import ctypes
import glob
import json
import os
import re
import tempfile

import numpy as np
import pytest

from trit_b200 import lm
from tests import synth
from tests.synth import presets

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = {}
    for header in sorted(glob.glob(os.path.join(ROOT, "include", "*.h"))):
        text = re.sub(r"/\*.*?\*/", "", open(header).read(), flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b(trit_\w+)\s*\(", text, flags=re.M):
            names[m.group(1)] = os.path.basename(header)
    return names


def test_every_declared_function_is_exported():
    names = declared_functions()
    assert len(names) >= 25, names
    lib = ctypes.CDLL(lm.LIBRARY)
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_python_signatures_cover_the_headers():
    lib = lm.library()
    for name in declared_functions():
        fn = getattr(lib, name)
        assert fn.argtypes is not None, f"{name} has no ctypes signature in trit_b200/lm.py"


def test_library_is_built_for_sm_100a_only():
    # The library's own build recipe names the one target it compiles for.
    make = open(os.path.join(ROOT, "trit_b200", "csrc", "Makefile")).read()
    assert "arch=compute_100a,code=sm_100a" in make


def last_error() -> str:
    return lm.library().trit_cuda_last_error().decode()


def test_version_and_error_text():
    lib = lm.library()
    assert re.match(r"\d+\.\d+\.\d+", lib.trit_cuda_version().decode())
    assert lib.trit_lm_load(None, None) is None
    assert "model_dir" in last_error()


@pytest.mark.parametrize("options, words", [
    ('{"colour": 1}', "unknown key colour"),
    ('{"kv": "bf16"}', "kv"),
    ('{"max_context": 0}', "max_context"),
    ('{"decode": "fast"}', "decode"),
    ('[1, 2]', "not a JSON object"),
    ('{"device": 1.5}', "device"),
])
def test_bad_options_fail_before_any_device_work(options, words):
    lib = lm.library()
    folder = presets.model_path("mini_qwen3_q8_0")
    assert lib.trit_lm_load(folder.encode(), options.encode()) is None
    assert words in last_error()


def test_inspect_failures():
    lib = lm.library()
    assert lib.trit_lm_inspect(b"/nonexistent/model", None) is None
    assert "config.json" in last_error()
    with pytest.raises(lm.TritError):
        lm.inspect("/nonexistent/model")


def write_config(folder: str, config: dict, gguf_from: str):
    os.makedirs(folder, exist_ok=True)
    with open(os.path.join(folder, "config.json"), "w") as f:
        json.dump(config, f)
    target = os.path.join(folder, "model.gguf")
    if not os.path.exists(target):
        os.symlink(os.path.join(gguf_from, "model.gguf"), target)


def test_config_parse_rules():
    """Config::parse (causal_lm.rs:41-77): q/k norms iff qwen3; llama,
    mistral and granite run without them; other types fail; heads must
    share the key heads evenly; head_dim defaults to hidden / heads; eps
    1e-6 and rope_theta 1e6 by default; tie_word_embeddings false by
    default; Granite's multipliers are read."""
    src = presets.model_path("mini_qwen3_q8_0")
    base = dict(presets.MINI_QWEN3)
    with tempfile.TemporaryDirectory() as tmp:
        for kind, qk in (("qwen3", True), ("llama", False), ("mistral", False), ("granite", False)):
            folder = os.path.join(tmp, kind)
            write_config(folder, dict(base, model_type=kind), src)
            assert lm.inspect(folder)["qk_norm"] is qk
        folder = os.path.join(tmp, "defaults")
        cfg = {k: v for k, v in base.items() if k not in ("head_dim", "rms_norm_eps", "rope_theta",
                                                           "tie_word_embeddings")}
        cfg["hidden_size"] = 512  # head_dim = 512 / 4 = 128
        write_config(folder, cfg, src)
        info = lm.inspect(folder)
        assert info["head_dim"] == 128 and info["rope_theta"] == 1e6
        assert abs(info["rms_norm_eps"] - 1e-6) < 1e-12 and info["tie_word_embeddings"] is False
        folder = os.path.join(tmp, "granite")
        write_config(folder, dict(base, model_type="granite", embedding_multiplier=12.0, attention_multiplier=0.0078125,
                                  residual_multiplier=0.22, logits_scaling=8.0), src)
        info = lm.inspect(folder)
        assert info["embedding_multiplier"] == 12.0 and info["attention_multiplier"] == 0.0078125
        assert abs(info["residual_multiplier"] - 0.22) < 1e-7 and info["logits_scaling"] == 8.0
        for bad, words in ((dict(base, model_type="bert"), "does not describe a language model"),
                           (dict(base, num_key_value_heads=3), "share the key heads evenly"),
                           (dict(base, num_key_value_heads=0), "share the key heads evenly")):
            folder = os.path.join(tmp, "bad")
            write_config(folder, bad, src)
            with pytest.raises(lm.TritError, match=words):
                lm.inspect(folder)


def test_config_at_and_tensor_prefix():
    """from_tensors(t, json, (config_at, prefix)) (causal_lm.rs:141-198):
    settings under a key path and tensor names under a prefix."""
    with tempfile.TemporaryDirectory() as tmp:
        cfg = dict(presets.MINI_QWEN3, num_hidden_layers=1, vocab_size=512)
        synth.synthesize(tmp, cfg, "q8_0", 3, prefix="thinker.", config_at="thinker_config.text_config.")
        with pytest.raises(lm.TritError):
            lm.inspect(tmp)
        info = lm.inspect(tmp, config_at="thinker_config.text_config.", prefix="thinker.")
        assert info["num_hidden_layers"] == 1 and info["vocab_size"] == 512


def test_static_entry_checks_its_limits_before_any_device_work():
    lib = lm.library()
    dummy = ctypes.c_void_p(16)  # never dereferenced: the size checks fail first
    fn = lib.trit_dense_q8_0_forward_static
    assert fn(dummy, dummy, 1024, 1024, dummy, 1024, dummy, None) == -1
    assert "too large for the static scratch" in last_error()
    assert fn(dummy, dummy, 1024, 1000, dummy, 1, dummy, None) == -1
    assert "multiple of 128" in last_error()
    # k = 96 is whole Q8_0 blocks but not whole 128-value chunks: rejected
    # with the reason, before any device work.
    assert fn(dummy, dummy, 1024, 96, dummy, 1, dummy, None) == -1
    assert "multiple of 128" in last_error()
    assert fn(None, dummy, 1024, 1024, dummy, 1, dummy, None) == -1
    assert "NULL" in last_error()


def test_dense_argument_checks():
    lib = lm.library()
    assert lib.trit_dense_q8_0(None, 32, 32, 0, 0) is None
    assert "blocks" in last_error()
    # A W8A8 layer whose k is whole Q8_0 blocks but not whole 128-value
    # chunks fails at creation (before any device work), not at forward.
    blocks = np.zeros(32 * 96 // 32 * 34, np.uint8)
    assert lib.trit_dense_q8_0(blocks.ctypes.data_as(ctypes.c_void_p), 32, 96, 0, 0) is None
    assert "multiple of 128" in last_error()
    assert lib.trit_dense_forward(None, None, 1, None) == -1
    assert "layer" in last_error()


def test_free_functions_accept_null():
    lib = lm.library()
    lib.trit_lm_free(None)
    lib.trit_lm_prefix_free(None)
    lib.trit_dense_free(None)
    lib.trit_cuda_free_text(None)


# The names the reference's own C library (the trit cdylib) exports, from
# its #[no_mangle] functions (ffi/src/lib.rs); tests/golden/reference_ffi_exports.py
# wrote the list.
REFERENCE_EXPORTS = os.path.join(ROOT, "tests", "golden", "reference_ffi_exports.txt")


def test_no_export_collides_with_the_reference_library():
    """A drop-in shares a process with the reference's libtrit (its Rust
    crate links both): no name may be defined by both libraries, or the
    dynamic linker binds one library's callers to the other's function."""
    theirs = set(open(REFERENCE_EXPORTS).read().split())
    assert "trit_last_error" in theirs and "trit_free_text" in theirs
    lib = ctypes.CDLL(lm.LIBRARY)
    clashes = sorted(n for n in theirs if hasattr(lib, n))
    assert not clashes, clashes
    ours = set(declared_functions())
    assert not ours & theirs


def test_only_the_header_names_are_exported():
    import shutil
    import subprocess

    if not shutil.which("nm"):
        pytest.skip("nm is not installed")
    out = subprocess.run(["nm", "-D", "--defined-only", lm.LIBRARY], capture_output=True, text=True, check=True)
    exported = {line.split()[-1] for line in out.stdout.splitlines() if line.strip()}
    assert exported == set(declared_functions())
