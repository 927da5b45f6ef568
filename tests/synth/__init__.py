"""Seeded synthetic decoder models for the tests and benchmarks: the
ctypes binding of tests/synth/libtrit_synth.so (trit_synth.h) and the
model shapes of the benchmark configurations (`presets`).

This is test and benchmark infrastructure, not part of the product
library: it writes model folders (config.json + model.gguf) that
libtrit_cuda.so and the CPU oracle then read."""
from __future__ import annotations

import ctypes
import json
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIBRARY = os.path.join(_HERE, "libtrit_synth.so")
_lib = None


def library() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIBRARY):
            raise RuntimeError(f"{LIBRARY} is missing: build it with `make -C tests/synth`")
        lib = ctypes.CDLL(LIBRARY)
        lib.trit_synth_model.restype = ctypes.c_int
        lib.trit_synth_model.argtypes = [ctypes.c_char_p, ctypes.c_char_p]
        lib.trit_synth_last_error.restype = ctypes.c_char_p
        lib.trit_synth_last_error.argtypes = []
        lib.trit_synth_normal_row.restype = None
        lib.trit_synth_normal_row.argtypes = [ctypes.c_uint64, ctypes.c_char_p, ctypes.c_uint64, ctypes.c_size_t,
                                              ctypes.c_float, ctypes.POINTER(ctypes.c_float)]
        _lib = lib
    return _lib


def synthesize(model_dir: str, config: dict, fmt: str = "q8_0", seed: int = 0, std: float = 0.02,
               prefix: str = "", config_at: str = "", **extra) -> str:
    """Writes a seeded synthetic model folder (trit_synth.h). `extra` keys
    of the spec: container ("gguf", "safetensors"), names ("hf",
    "transcribe"), arch (of a transcribe file), dtype (of fmt "float")."""
    os.makedirs(model_dir, exist_ok=True)
    spec = {"config": config, "format": fmt, "seed": seed, "std": std, **extra}
    if prefix:
        spec["prefix"] = prefix
    if config_at:
        spec["config_at"] = config_at
    lib = library()
    if lib.trit_synth_model(str(model_dir).encode(), json.dumps(spec).encode()) != 0:
        raise RuntimeError(lib.trit_synth_last_error().decode("utf-8", "replace"))
    return model_dir


def normal_row(seed: int, name: str, row: int, k: int, std: float = 0.02) -> np.ndarray:
    """The f32 values of a synthetic tensor's row before quantization."""
    out = np.zeros(k, dtype=np.float32)
    library().trit_synth_normal_row(seed, name.encode(), row, k, std,
                                    out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)))
    return out
