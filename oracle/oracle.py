"""TEST INFRASTRUCTURE ONLY: the Python binding of the CPU oracle
(oracle.cpp, a restatement of Trit's CausalLm decoder path). Only tests/,
__graft_entry__.smoke() and the CPU-baseline legs of bench.py use it, as the
checker or the timed CPU baseline; the product never does.

Parity status: unpinned at the golden-vector level (the reference has no
golden vectors); see the header of oracle.cpp.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIBRARY = os.path.join(HERE, "_build", "liboracle.so")

_i32p = ctypes.POINTER(ctypes.c_int32)
_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_i8p = ctypes.POINTER(ctypes.c_int8)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_size = ctypes.c_size_t
_lib = None


def build() -> None:
    subprocess.run(["make", "-C", HERE], check=True, stdout=subprocess.DEVNULL)


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIBRARY):
        build()
    L = ctypes.CDLL(LIBRARY)
    sig = {
        "oracle_last_error": (ctypes.c_char_p, []),
        "oracle_isa": (ctypes.c_char_p, []),
        "oracle_force_scalar": (None, [ctypes.c_int]),
        "oracle_threads": (ctypes.c_int, []),
        "oracle_set_threads": (None, [ctypes.c_int]),
        "oracle_load": (ctypes.c_void_p, [ctypes.c_char_p, ctypes.c_int]),
        "oracle_free": (None, [ctypes.c_void_p]),
        "oracle_vocab": (ctypes.c_int64, [ctypes.c_void_p]),
        "oracle_width": (ctypes.c_int64, [ctypes.c_void_p]),
        "oracle_layers": (ctypes.c_int64, [ctypes.c_void_p]),
        "oracle_prefix": (ctypes.c_void_p, [ctypes.c_void_p, _i32p, _size]),
        "oracle_prefix_free": (None, [ctypes.c_void_p]),
        "oracle_generate": (ctypes.c_int64, [ctypes.c_void_p, ctypes.c_void_p, _i32p, _size, ctypes.c_int64, _i32p,
                                             _size, _i32p, _f32p, _f32p, _f64p, _f64p]),
        "oracle_generate_rows": (ctypes.c_int64, [ctypes.c_void_p, _f32p, _size, ctypes.c_int64, _i32p, _size, _i32p,
                                                  _f32p, _f32p]),
        "oracle_answer": (ctypes.c_int64, [ctypes.c_void_p, _i32p, _size, _f32p, _size, _i32p, _size, ctypes.c_int64,
                                           _i32p, _size, _i32p, _f32p, _f32p]),
        "oracle_embed": (ctypes.c_int, [ctypes.c_void_p, _i32p, _size, _f32p]),
        "oracle_set_ffn_scales": (None, [ctypes.c_void_p, _f32p]),
        "oracle_generate_additive": (ctypes.c_int64, [ctypes.c_void_p, _i32p, _size, _f32p, _size, _i32p, _size,
                                                      _i32p, _f32p]),
        "oracle_bidirectional_tokens": (ctypes.c_int64, [ctypes.c_void_p, _f32p, _size, _size, _i32p]),
        "oracle_f32_to_f16": (ctypes.c_uint16, [ctypes.c_float]),
        "oracle_f16_to_f32": (ctypes.c_float, [ctypes.c_uint16]),
        "oracle_exp": (ctypes.c_float, [ctypes.c_float]),
        "oracle_silu": (ctypes.c_float, [ctypes.c_float]),
        "oracle_base3": (None, [ctypes.c_uint8, _u8p]),
        "oracle_q8_0_quantize": (None, [_f32p, _size, _i8p, _u16p]),
        "oracle_quantize": (None, [_f32p, _size, _size, _size, ctypes.c_int, _i8p, _f32p, _i32p]),
        "oracle_int_layer": (ctypes.c_void_p, [_i8p, _f32p, _size, _size, _size, _size, ctypes.c_int]),
        "oracle_int_layer_free": (None, [ctypes.c_void_p]),
        "oracle_int_forward": (ctypes.c_int, [ctypes.c_void_p, _f32p, _size, _f32p]),
        "oracle_table": (ctypes.c_void_p, [_i8p, _f32p, _size, _size]),
        "oracle_table_free": (None, [ctypes.c_void_p]),
        "oracle_table_forward": (None, [ctypes.c_void_p, _f32p, _size, _f32p]),
        "oracle_rmsnorm": (None, [_f32p, _f32p, _size, ctypes.c_float]),
        "oracle_attention": (None, [_f32p, _size, _f32p, _f32p, _size, _size, _size, _size, _size, _size,
                                    ctypes.c_int, _f32p]),
        "oracle_rope": (None, [_f32p, _size, _size, _size, _size, _size, ctypes.c_float]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    _lib = L
    return L


def _p(a: np.ndarray, kind):
    return a.ctypes.data_as(kind) if a is not None and a.size else None


def _ids(v) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(v, dtype=np.int32).reshape(-1))


class OracleError(RuntimeError):
    pass


def _err():
    return OracleError(lib().oracle_last_error().decode())


class Oracle:
    """The reference decoder on the CPU for one model folder."""

    def __init__(self, model_dir: str, kv_f16: bool = False):
        self.h = lib().oracle_load(model_dir.encode(), 1 if kv_f16 else 0)
        if not self.h:
            raise _err()
        self.vocab = int(lib().oracle_vocab(self.h))
        self.width = int(lib().oracle_width(self.h))

    def close(self):
        if self.h:
            lib().oracle_free(self.h)
            self.h = None

    def __del__(self):
        self.close()

    def prefix(self, tokens):
        ids = _ids(tokens)
        p = lib().oracle_prefix(self.h, _p(ids, _i32p), ids.size)
        if not p:
            raise _err()
        return (p, ids.tolist())

    def free_prefix(self, p):
        lib().oracle_prefix_free(p[0])

    def generate(self, prompt: Sequence[int], max_new: int, stop=(), prefix=None, trace: bool = False,
                 timing: bool = False):
        ids, st = _ids(prompt), _ids(stop)
        out = np.zeros(max(max_new, 1), dtype=np.int32)
        logits = np.zeros((max(max_new, 1), self.vocab), dtype=np.float32) if trace else None
        gaps = np.zeros(max(max_new, 1), dtype=np.float32)
        secs = np.zeros(max(max_new, 1), dtype=np.float64)
        prefill = ctypes.c_double()
        n = lib().oracle_generate(self.h, prefix[0] if prefix else None, _p(ids, _i32p), ids.size, max_new,
                                  _p(st, _i32p), st.size, _p(out, _i32p), _p(logits, _f32p), _p(gaps, _f32p),
                                  _p(secs, _f64p), ctypes.byref(prefill))
        if n < 0:
            raise _err()
        res = {"tokens": out[:n].tolist(), "gaps": gaps[:max(n, 1)].copy()}
        if trace:
            res["logits"] = logits
        if timing:
            res["seconds"] = secs[:n].copy()
            res["prefill_seconds"] = prefill.value
        return res

    def answer(self, head, audio: np.ndarray, tail, max_new: int, stop=(), trace: bool = False):
        h, t, st = _ids(head), _ids(tail), _ids(stop)
        a = np.ascontiguousarray(audio, dtype=np.float32).reshape(-1, self.width)
        out = np.zeros(max(max_new, 1), dtype=np.int32)
        logits = np.zeros((max(max_new, 1), self.vocab), dtype=np.float32) if trace else None
        gaps = np.zeros(max(max_new, 1), dtype=np.float32)
        n = lib().oracle_answer(self.h, _p(h, _i32p), h.size, _p(a, _f32p), a.shape[0], _p(t, _i32p), t.size,
                                max_new, _p(st, _i32p), st.size, _p(out, _i32p), _p(logits, _f32p), _p(gaps, _f32p))
        if n < 0:
            raise _err()
        res = {"tokens": out[:n].tolist(), "gaps": gaps[:max(n, 1)].copy()}
        if trace:
            res["logits"] = logits
        return res

    def generate_rows(self, rows: np.ndarray, max_new: int, stop=(), trace: bool = False):
        return self.answer([], rows, [], max_new, stop, trace)

    def set_ffn_scales(self, scales) -> None:
        """CausalLm::set_ffn_scales: [layers][width] floats, or None."""
        if scales is None:
            lib().oracle_set_ffn_scales(self.h, None)
            return
        self._ffn = np.ascontiguousarray(scales, dtype=np.float32)
        lib().oracle_set_ffn_scales(self.h, _p(self._ffn, _f32p))

    def generate_additive(self, prompt, audio: np.ndarray, stop=(), trace: bool = False):
        ids, st = _ids(prompt), _ids(stop)
        a = np.ascontiguousarray(audio, dtype=np.float32).reshape(-1, self.width)
        cap = max(a.shape[0] - ids.size + 1, 1)
        out = np.zeros(cap, dtype=np.int32)
        logits = np.zeros((cap, self.vocab), dtype=np.float32) if trace else None
        n = lib().oracle_generate_additive(self.h, _p(ids, _i32p), ids.size, _p(a, _f32p), a.shape[0],
                                           _p(st, _i32p), st.size, _p(out, _i32p), _p(logits, _f32p))
        if n < 0:
            raise _err()
        return {"tokens": out[:n].tolist(), "logits": logits}

    def bidirectional_tokens(self, rows: np.ndarray, start: int) -> list:
        r = np.ascontiguousarray(rows, dtype=np.float32).reshape(-1, self.width)
        out = np.zeros(max(r.shape[0] - start, 1), dtype=np.int32)
        n = lib().oracle_bidirectional_tokens(self.h, _p(r, _f32p), r.shape[0], start, _p(out, _i32p))
        if n < 0:
            raise _err()
        return out[:n].tolist()

    def embed(self, tokens) -> np.ndarray:
        ids = _ids(tokens)
        out = np.zeros((ids.size, self.width), dtype=np.float32)
        if lib().oracle_embed(self.h, _p(ids, _i32p), ids.size, _p(out, _f32p)) != 0:
            raise _err()
        return out


# ---- op-level helpers ----
def q8_0_quantize(values: np.ndarray):
    v = np.ascontiguousarray(values, dtype=np.float32).reshape(-1)
    codes = np.zeros(v.size, dtype=np.int8)
    scales = np.zeros(v.size // 32, dtype=np.uint16)
    lib().oracle_q8_0_quantize(_p(v, _f32p), v.size, _p(codes, _i8p), _p(scales, _u16p))
    return codes, scales


def q8_0_blocks(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """ggml Q8_0 bytes (34 a block: f16 scale little-endian, 32 codes)."""
    nb = scales.size
    out = np.zeros((nb, 34), dtype=np.uint8)
    out[:, 0:2] = scales.astype("<u2").view(np.uint8).reshape(nb, 2)
    out[:, 2:] = codes.reshape(nb, 32).view(np.uint8)
    return out.reshape(-1)


def quantize(x: np.ndarray, group: int, half: bool):
    x = np.ascontiguousarray(x, dtype=np.float32)
    m, k = x.shape
    codes = np.zeros((m, k), dtype=np.int8)
    scales = np.zeros((m, k // group), dtype=np.float32)
    sums = np.zeros((m, k // group), dtype=np.int32)
    lib().oracle_quantize(_p(x, _f32p), m, k, group, 1 if half else 0, _p(codes, _i8p), _p(scales, _f32p),
                          _p(sums, _i32p))
    return codes, scales, sums


def f16_to_f32(h: int) -> float:
    return lib().oracle_f16_to_f32(h)


def f32_to_f16(v: float) -> int:
    return lib().oracle_f32_to_f16(v)


class IntLayer:
    def __init__(self, codes: np.ndarray, scales: np.ndarray, group: int, wgroup: int, half: bool):
        c = np.ascontiguousarray(codes, dtype=np.int8)
        s = np.ascontiguousarray(scales, dtype=np.float32)
        self.n, self.k = c.shape
        self.h = lib().oracle_int_layer(_p(c, _i8p), _p(s, _f32p), self.n, self.k, group, wgroup, 1 if half else 0)
        if not self.h:
            raise _err()

    def forward(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, self.k)
        out = np.zeros((x.shape[0], self.n), dtype=np.float32)
        if lib().oracle_int_forward(self.h, _p(x, _f32p), x.shape[0], _p(out, _f32p)) != 0:
            raise _err()
        return out

    def __del__(self):
        if getattr(self, "h", None):
            lib().oracle_int_layer_free(self.h)


class Table:
    def __init__(self, codes: np.ndarray, scales: np.ndarray):
        c = np.ascontiguousarray(codes, dtype=np.int8)
        s = np.ascontiguousarray(scales, dtype=np.float32)
        self.n, self.k = c.shape
        self.h = lib().oracle_table(_p(c, _i8p), _p(s, _f32p), self.n, self.k)

    def forward(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, self.k)
        out = np.zeros((x.shape[0], self.n), dtype=np.float32)
        lib().oracle_table_forward(self.h, _p(x, _f32p), x.shape[0], _p(out, _f32p))
        return out

    def __del__(self):
        if getattr(self, "h", None):
            lib().oracle_table_free(self.h)
