"""Python host side of libtrit_cuda.so: the `CausalLm` interface of Trit's
decoder (src/models/parts/causal_lm.rs) and `Dense` (src/cpu/gemm.rs) over
the C ABI of include/trit_cuda.h.

Failures raise `TritError` with the library's `trit_cuda_last_error()` text, as
the reference's functions return `Err(String)`. There is no fallback: if
the shared library is missing or no GPU can be used, loading fails.
"""
from __future__ import annotations

import ctypes
import json
import os
from typing import Iterable, Sequence

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
# TRIT_CUDA_LIBRARY names another build of the library (a user's own).
LIBRARY = os.environ.get("TRIT_CUDA_LIBRARY") or os.path.join(_HERE, "libtrit_cuda.so")

_i32p = ctypes.POINTER(ctypes.c_int32)
_f32p = ctypes.POINTER(ctypes.c_float)
_i64p = ctypes.POINTER(ctypes.c_int64)
_f64p = ctypes.POINTER(ctypes.c_double)
_size = ctypes.c_size_t


class TritError(RuntimeError):
    """A failed call into libtrit_cuda (the text of trit_cuda_last_error)."""


_lib = None


def library() -> ctypes.CDLL:
    """The loaded libtrit_cuda.so, with the signatures of include/*.h."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIBRARY):
        raise TritError(f"{LIBRARY} is missing: build it with `make -C trit_b200/csrc`")
    lib = ctypes.CDLL(LIBRARY)
    sig = {
        "trit_cuda_version": (ctypes.c_char_p, []),
        "trit_cuda_last_error": (ctypes.c_char_p, []),
        "trit_lm_inspect": (ctypes.c_void_p, [ctypes.c_char_p, ctypes.c_char_p]),
        "trit_cuda_free_text": (None, [ctypes.c_void_p]),
        "trit_lm_load": (ctypes.c_void_p, [ctypes.c_char_p, ctypes.c_char_p]),
        "trit_lm_free": (None, [ctypes.c_void_p]),
        "trit_lm_width": (ctypes.c_int64, [ctypes.c_void_p]),
        "trit_lm_layers": (ctypes.c_int64, [ctypes.c_void_p]),
        "trit_lm_vocab": (ctypes.c_int64, [ctypes.c_void_p]),
        "trit_lm_prefix": (ctypes.c_void_p, [ctypes.c_void_p, _i32p, _size]),
        "trit_lm_prefix_free": (None, [ctypes.c_void_p]),
        "trit_lm_generate": (ctypes.c_int64, [ctypes.c_void_p, ctypes.c_void_p, _i32p, _size, ctypes.c_int32,
                                              _i32p, _size, _i32p, _size]),
        "trit_lm_generate_traced": (ctypes.c_int64, [ctypes.c_void_p, ctypes.c_void_p, _i32p, _size,
                                                     ctypes.c_int32, _i32p, _size, _i32p, _size, _f32p]),
        "trit_lm_generate_rows": (ctypes.c_int64, [ctypes.c_void_p, _f32p, _size, ctypes.c_int32, _i32p, _size,
                                                   _i32p, _size]),
        "trit_lm_answer": (ctypes.c_int64, [ctypes.c_void_p, _i32p, _size, _f32p, _size, _i32p, _size,
                                            ctypes.c_int32, _i32p, _size, _i32p, _size]),
        "trit_lm_answer_traced": (ctypes.c_int64, [ctypes.c_void_p, _i32p, _size, _f32p, _size, _i32p, _size,
                                                   ctypes.c_int32, _i32p, _size, _i32p, _size, _f32p]),
        "trit_lm_generate_rows_device": (ctypes.c_int64, [ctypes.c_void_p, ctypes.c_void_p, _size, ctypes.c_int32,
                                                          _i32p, _size, _i32p, _size, ctypes.c_void_p]),
        "trit_lm_answer_device": (ctypes.c_int64, [ctypes.c_void_p, _i32p, _size, ctypes.c_void_p, _size, _i32p,
                                                   _size, ctypes.c_int32, _i32p, _size, _i32p, _size,
                                                   ctypes.c_void_p]),
        "trit_lm_embed": (ctypes.c_int, [ctypes.c_void_p, _i32p, _size, _f32p]),
        "trit_lm_generate_batch": (ctypes.c_int, [ctypes.c_void_p, _size, ctypes.POINTER(_i32p),
                                                  ctypes.POINTER(_size), ctypes.c_int32, _i32p, _size, _i32p,
                                                  _i64p]),
        "trit_lm_last_timing": (ctypes.c_int, [ctypes.c_void_p, _f64p, _f64p, _i64p, _i64p]),
        "trit_lm_status": (ctypes.c_void_p, [ctypes.c_void_p]),
        "trit_cuda_tp_id": (ctypes.c_int, [ctypes.c_char_p, _size]),
        "trit_lm_generate_batch_prefix": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, _size,
                                                         ctypes.POINTER(_i32p), ctypes.POINTER(_size), ctypes.c_int32,
                                                         _i32p, _size, _i32p, _i64p]),
        "trit_lm_prefix_pages": (ctypes.c_int, [ctypes.c_void_p, _i64p, _i64p]),
        "trit_lm_set_ffn_scales": (ctypes.c_int, [ctypes.c_void_p, _f32p, _size, _size]),
        "trit_lm_generate_additive": (ctypes.c_int64, [ctypes.c_void_p, _i32p, _size, _f32p, _size, _i32p, _size,
                                                       _i32p, _size]),
        "trit_lm_bidirectional_tokens": (ctypes.c_int64, [ctypes.c_void_p, _f32p, _size, _size, _i32p]),
        "trit_dense_q8_0": (ctypes.c_void_p, [ctypes.c_void_p, _size, _size, ctypes.c_int, ctypes.c_int]),
        "trit_dense_forward": (ctypes.c_int, [ctypes.c_void_p, _f32p, _size, _f32p]),
        "trit_dense_forward_device": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, _size, ctypes.c_void_p,
                                                     ctypes.c_void_p]),
        "trit_dense_free": (None, [ctypes.c_void_p]),
        "trit_dense_q8_0_forward_static": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, _size, _size,
                                                          ctypes.c_void_p, _size, ctypes.c_void_p, ctypes.c_void_p]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def _error() -> TritError:
    return TritError(library().trit_cuda_last_error().decode("utf-8", "replace"))


def _ids(values: Iterable[int]) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(list(values) if not isinstance(values, np.ndarray) else values,
                                           dtype=np.int32).reshape(-1))


def _ptr(a: np.ndarray, kind):
    return a.ctypes.data_as(kind) if a.size else None


class Prefix:
    """A prompt start run once (CausalLm::prefix, causal_lm.rs:200-215)."""

    def __init__(self, lm: "CausalLm", handle: int, tokens: Sequence[int]):
        self._lm = lm
        self._handle = handle
        self.tokens = list(tokens)

    def close(self) -> None:
        if self._handle:
            library().trit_lm_prefix_free(self._handle)
            self._handle = None

    def __del__(self):
        self.close()


class CausalLm:
    """A decoder on one GPU (src/models/parts/causal_lm.rs:92-116)."""

    def __init__(self, handle: int, model_dir: str, options: dict):
        self._handle = handle
        self.model_dir = model_dir
        self.options = options

    @classmethod
    def load(cls, model_dir: str, **options) -> "CausalLm":
        """CausalLm::load (causal_lm.rs:124-130): config.json + model.gguf.
        Options are the keys of trit_lm_load (device, kv, max_context,
        max_streams, page_tokens, prefill_rows, decode)."""
        text = json.dumps(options).encode() if options else None
        handle = library().trit_lm_load(str(model_dir).encode(), text)
        if not handle:
            raise _error()
        return cls(handle, str(model_dir), options)

    def close(self) -> None:
        if getattr(self, "_handle", None):
            library().trit_lm_free(self._handle)
            self._handle = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def width(self) -> int:
        return int(library().trit_lm_width(self._handle))

    def layers(self) -> int:
        return int(library().trit_lm_layers(self._handle))

    def vocab(self) -> int:
        return int(library().trit_lm_vocab(self._handle))

    def prefix(self, tokens: Sequence[int]) -> Prefix:
        ids = _ids(tokens)
        h = library().trit_lm_prefix(self._handle, _ptr(ids, _i32p), ids.size)
        if not h:
            raise _error()
        return Prefix(self, h, ids.tolist())

    def generate(self, prompt: Sequence[int], prefix: Prefix | None = None, max_new: int = 128,
                 stop: Sequence[int] = ()) -> list[int]:
        """CausalLm::generate (causal_lm.rs:217-249)."""
        ids, st = _ids(prompt), _ids(stop)
        out = np.zeros(max(max_new, 1), dtype=np.int32)
        n = library().trit_lm_generate(self._handle, prefix._handle if prefix else None, _ptr(ids, _i32p), ids.size,
                                       max_new, _ptr(st, _i32p), st.size, _ptr(out, _i32p), out.size)
        if n < 0:
            raise _error()
        return out[:n].tolist()

    def generate_traced(self, prompt: Sequence[int], prefix: Prefix | None = None, max_new: int = 128,
                        stop: Sequence[int] = ()) -> tuple[list[int], np.ndarray]:
        """generate with the logits of every made (or stopping) token."""
        ids, st = _ids(prompt), _ids(stop)
        out = np.zeros(max(max_new, 1), dtype=np.int32)
        logits = np.zeros((max(max_new, 1), self.vocab()), dtype=np.float32)
        n = library().trit_lm_generate_traced(self._handle, prefix._handle if prefix else None, _ptr(ids, _i32p),
                                              ids.size, max_new, _ptr(st, _i32p), st.size, _ptr(out, _i32p),
                                              out.size, _ptr(logits, _f32p))
        if n < 0:
            raise _error()
        return out[:n].tolist(), logits

    def generate_rows(self, rows: np.ndarray, max_new: int = 128, stop: Sequence[int] = ()) -> list[int]:
        """CausalLm::generate_rows (causal_lm.rs:251-262)."""
        r = np.ascontiguousarray(rows, dtype=np.float32).reshape(-1, self.width())
        st = _ids(stop)
        out = np.zeros(max(max_new, 1), dtype=np.int32)
        n = library().trit_lm_generate_rows(self._handle, _ptr(r, _f32p), r.shape[0], max_new, _ptr(st, _i32p),
                                            st.size, _ptr(out, _i32p), out.size)
        if n < 0:
            raise _error()
        return out[:n].tolist()

    def answer(self, head: Sequence[int], audio: np.ndarray, tail: Sequence[int], max_new: int = 128,
               stop: Sequence[int] = (), trace: bool = False):
        """CausalLm::answer (causal_lm.rs:264-282); with trace=True also the logits."""
        h, t, st = _ids(head), _ids(tail), _ids(stop)
        a = np.ascontiguousarray(audio, dtype=np.float32).reshape(-1, self.width())
        out = np.zeros(max(max_new, 1), dtype=np.int32)
        lib = library()
        if trace:
            logits = np.zeros((max(max_new, 1), self.vocab()), dtype=np.float32)
            n = lib.trit_lm_answer_traced(self._handle, _ptr(h, _i32p), h.size, _ptr(a, _f32p), a.shape[0],
                                          _ptr(t, _i32p), t.size, max_new, _ptr(st, _i32p), st.size,
                                          _ptr(out, _i32p), out.size, _ptr(logits, _f32p))
        else:
            n = lib.trit_lm_answer(self._handle, _ptr(h, _i32p), h.size, _ptr(a, _f32p), a.shape[0], _ptr(t, _i32p),
                                   t.size, max_new, _ptr(st, _i32p), st.size, _ptr(out, _i32p), out.size)
        if n < 0:
            raise _error()
        return (out[:n].tolist(), logits) if trace else out[:n].tolist()

    def answer_device(self, head: Sequence[int], rows_ptr: int, nrows: int, tail: Sequence[int],
                      max_new: int = 128, stop: Sequence[int] = (), stream: int | None = None) -> list[int]:
        """answer with the rows (nrows x width f32) at a device pointer of
        this model's GPU, read after the work queued on `stream` (a
        cudaStream_t handle, None: the default stream)."""
        h, t, st = _ids(head), _ids(tail), _ids(stop)
        out = np.zeros(max(max_new, 1), dtype=np.int32)
        n = library().trit_lm_answer_device(self._handle, _ptr(h, _i32p), h.size, rows_ptr, nrows, _ptr(t, _i32p),
                                            t.size, max_new, _ptr(st, _i32p), st.size, _ptr(out, _i32p), out.size,
                                            stream)
        if n < 0:
            raise _error()
        return out[:n].tolist()

    def generate_rows_device(self, rows_ptr: int, nrows: int, max_new: int = 128, stop: Sequence[int] = (),
                             stream: int | None = None) -> list[int]:
        """generate_rows with the rows at a device pointer (see answer_device)."""
        st = _ids(stop)
        out = np.zeros(max(max_new, 1), dtype=np.int32)
        n = library().trit_lm_generate_rows_device(self._handle, rows_ptr, nrows, max_new, _ptr(st, _i32p), st.size,
                                                   _ptr(out, _i32p), out.size, stream)
        if n < 0:
            raise _error()
        return out[:n].tolist()

    def embed(self, tokens: Sequence[int]) -> np.ndarray:
        """CausalLm::embed (causal_lm.rs:347-355)."""
        ids = _ids(tokens)
        out = np.zeros((ids.size, self.width()), dtype=np.float32)
        if library().trit_lm_embed(self._handle, _ptr(ids, _i32p), ids.size, _ptr(out, _f32p)) != 0:
            raise _error()
        return out

    def generate_batch(self, prompts: Sequence[Sequence[int]], max_new: int = 128,
                       stop: Sequence[int] = (), prefix: Prefix | None = None) -> list[list[int]]:
        """Independent greedy generations decoded side by side; streams whose
        prompt starts with `prefix` read its KV pages in place."""
        arrays = [_ids(p) for p in prompts]
        ptrs = (_i32p * len(arrays))(*[a.ctypes.data_as(_i32p) for a in arrays])
        lens = (_size * len(arrays))(*[a.size for a in arrays])
        st = _ids(stop)
        out = np.zeros((len(arrays), max(max_new, 1)), dtype=np.int32)
        counts = np.zeros(len(arrays), dtype=np.int64)
        if prefix is not None:
            rc = library().trit_lm_generate_batch_prefix(self._handle, prefix._handle, len(arrays), ptrs, lens,
                                                         max_new, _ptr(st, _i32p), st.size, _ptr(out, _i32p),
                                                         _ptr(counts, _i64p))
        else:
            rc = library().trit_lm_generate_batch(self._handle, len(arrays), ptrs, lens, max_new, _ptr(st, _i32p),
                                                  st.size, _ptr(out, _i32p), _ptr(counts, _i64p))
        if rc != 0:
            raise _error()
        return [out[s, :counts[s]].tolist() for s in range(len(arrays))]

    def set_ffn_scales(self, scales: np.ndarray | None) -> None:
        """CausalLm::set_ffn_scales (causal_lm.rs:305-307): [layers][width], or None."""
        if scales is None:
            rc = library().trit_lm_set_ffn_scales(self._handle, None, 0, 0)
        else:
            s = np.ascontiguousarray(scales, dtype=np.float32)
            rc = library().trit_lm_set_ffn_scales(self._handle, _ptr(s, _f32p), s.shape[0], s.shape[1])
        if rc != 0:
            raise _error()

    def generate_additive(self, prompt: Sequence[int], audio: np.ndarray, stop: Sequence[int] = ()) -> list[int]:
        """CausalLm::generate_additive (causal_lm.rs:317-345)."""
        ids, st = _ids(prompt), _ids(stop)
        a = np.ascontiguousarray(audio, dtype=np.float32).reshape(-1, self.width())
        out = np.zeros(max(a.shape[0] - ids.size + 1, 1), dtype=np.int32)
        n = library().trit_lm_generate_additive(self._handle, _ptr(ids, _i32p), ids.size, _ptr(a, _f32p), a.shape[0],
                                                _ptr(st, _i32p), st.size, _ptr(out, _i32p), out.size)
        if n < 0:
            raise _error()
        return out[:n].tolist()

    def bidirectional_tokens(self, rows: np.ndarray, start: int) -> list[int]:
        """CausalLm::bidirectional_tokens (causal_lm.rs:393-408)."""
        r = np.ascontiguousarray(rows, dtype=np.float32).reshape(-1, self.width())
        out = np.zeros(max(r.shape[0] - start, 1), dtype=np.int32)
        n = library().trit_lm_bidirectional_tokens(self._handle, _ptr(r, _f32p), r.shape[0], start, _ptr(out, _i32p))
        if n < 0:
            raise _error()
        return out[:n].tolist()

    def status(self) -> dict:
        """What the load did (trit_lm_status): the files' form, whether the
        weight cache supplied the weights, the arena size, the settings."""
        lib = library()
        ptr = lib.trit_lm_status(self._handle)
        if not ptr:
            raise _error()
        try:
            return json.loads(ctypes.string_at(ptr).decode())
        finally:
            lib.trit_cuda_free_text(ptr)

    def prefix_pages(self) -> tuple[int, int]:
        """KV pages kept for prefixes: (in use, in all)."""
        used, total = ctypes.c_int64(), ctypes.c_int64()
        if library().trit_lm_prefix_pages(self._handle, ctypes.byref(used), ctypes.byref(total)) != 0:
            raise _error()
        return used.value, total.value

    def last_timing(self) -> dict:
        """Device time of the last generation (CUDA events)."""
        pf, dc = ctypes.c_double(), ctypes.c_double()
        steps, launches = ctypes.c_int64(), ctypes.c_int64()
        if library().trit_lm_last_timing(self._handle, ctypes.byref(pf), ctypes.byref(dc), ctypes.byref(steps),
                                         ctypes.byref(launches)) != 0:
            raise _error()
        return {"prefill_ms": pf.value, "decode_ms": dc.value, "decode_steps": steps.value,
                "launches": launches.value}


class Dense:
    """One product layer from ggml Q8_0 blocks (Dense, src/cpu/gemm.rs:14-24)."""

    def __init__(self, handle: int, n: int, k: int, table: bool):
        self._handle, self.n, self.k, self.table = handle, n, k, table

    @classmethod
    def q8_0(cls, blocks: np.ndarray, n: int, k: int, table: bool = False, device: int = 0) -> "Dense":
        b = np.ascontiguousarray(blocks, dtype=np.uint8)
        if b.size != n * (k // 32) * 34:
            raise TritError(f"{b.size} bytes are not the Q8_0 blocks of a {n}x{k} matrix")
        h = library().trit_dense_q8_0(b.ctypes.data, n, k, 1 if table else 0, device)
        if not h:
            raise _error()
        return cls(h, n, k, table)

    def forward(self, x: np.ndarray) -> np.ndarray:
        """Dense::forward (gemm.rs:500-506): rows x k -> rows x n."""
        xs = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, self.k)
        out = np.zeros((xs.shape[0], self.n), dtype=np.float32)
        if library().trit_dense_forward(self._handle, _ptr(xs, _f32p), xs.shape[0], _ptr(out, _f32p)) != 0:
            raise _error()
        return out

    def forward_device(self, x_ptr: int, rows: int, out_ptr: int, stream: int | None = None) -> None:
        if library().trit_dense_forward_device(self._handle, x_ptr, rows, out_ptr, stream) != 0:
            raise _error()

    def close(self) -> None:
        if getattr(self, "_handle", None):
            library().trit_dense_free(self._handle)
            self._handle = None

    def __del__(self):
        self.close()


def tp_id() -> str:
    """A new tensor-parallel group id (trit_cuda_tp_id): made on one rank,
    passed to every rank's load as tp_id."""
    buf = ctypes.create_string_buffer(512)
    if library().trit_cuda_tp_id(buf, len(buf)) != 0:
        raise _error()
    return buf.value.decode()


def inspect(model_dir: str, **options) -> dict:
    """The settings and weight storage of a model folder, read without a GPU
    (Config::parse, causal_lm.rs:41-77). Options: config_at, prefix."""
    lib = library()
    ptr = lib.trit_lm_inspect(model_dir.encode(), json.dumps(options).encode())
    if not ptr:
        raise _error()
    try:
        return json.loads(ctypes.string_at(ptr).decode())
    finally:
        lib.trit_cuda_free_text(ptr)
