"""The Rust FFI crate (rust/trit-cuda-sys) declares every function of
include/trit_cuda.h once, with the same number of parameters. The crate
is not compiled in this image (no cargo), so this is its check."""
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions() -> dict:
    text = open(os.path.join(ROOT, "include", "trit_cuda.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    out = {}
    for m in re.finditer(r"\b(trit_\w+)\s*\(([^;{]*?)\)\s*;", text, flags=re.S):
        params = m.group(2).strip()
        out[m.group(1)] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def rust_functions() -> dict:
    text = open(os.path.join(ROOT, "rust", "trit-cuda-sys", "src", "lib.rs")).read()
    block = text[text.index('extern "C" {'):]
    block = block[:block.index("\n    }\n")]
    out = {}
    for m in re.finditer(r"pub fn (trit_\w+)\s*\(([^)]*)\)", block, flags=re.S):
        params = [p for p in m.group(2).split(",") if p.strip()]
        assert m.group(1) not in out, f"{m.group(1)} declared twice"
        out[m.group(1)] = len(params)
    return out


def test_rust_declarations_match_the_header():
    want, got = header_functions(), rust_functions()
    assert len(want) >= 25
    assert set(got) == set(want), (sorted(set(want) - set(got)), sorted(set(got) - set(want)))
    for name, n in want.items():
        assert got[name] == n, f"{name}: header {n} parameters, Rust {got[name]}"
