"""A small GGUF v3 reader for the CPU tests: tensor names, ggml types,
dimensions and raw bytes, read independently of the library's C++ reader
(the format the reference parses in src/models/gguf/mod.rs)."""
from __future__ import annotations

import struct

import numpy as np

GGML_F32, GGML_F16, GGML_Q8_0, GGML_I8 = 0, 1, 8, 24
_SCALAR = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}


class Gguf:
    def __init__(self, path: str):
        with open(path, "rb") as f:
            self.data = f.read()
        self.pos = 0
        magic, version = self._take("<4sI")
        assert magic == b"GGUF" and version == 3, (magic, version)
        n_tensors, n_kv = self._take("<QQ")
        self.meta = {}
        for _ in range(n_kv):
            key = self._str()
            self.meta[key] = self._value(self._take("<I")[0])
        self.alignment = int(self.meta.get("general.alignment", 32))
        infos = []
        for _ in range(n_tensors):
            name = self._str()
            (nd,) = self._take("<I")
            dims = list(self._take(f"<{nd}Q"))
            typ, off = self._take("<IQ")
            infos.append((name, dims, typ, off))
        start = (self.pos + self.alignment - 1) // self.alignment * self.alignment
        self.tensors = {}
        for name, dims, typ, off in infos:
            count = int(np.prod(dims))
            size = {GGML_F32: 4 * count, GGML_F16: 2 * count, GGML_I8: count, GGML_Q8_0: count // 32 * 34}[typ]
            self.tensors[name] = (dims, typ, self.data[start + off:start + off + size])

    def _take(self, fmt):
        vals = struct.unpack_from(fmt, self.data, self.pos)
        self.pos += struct.calcsize(fmt)
        return vals

    def _str(self) -> str:
        (n,) = self._take("<Q")
        s = self.data[self.pos:self.pos + n].decode()
        self.pos += n
        return s

    def _value(self, typ):
        if typ in _SCALAR:
            return self._take(_SCALAR[typ])[0]
        if typ == 8:
            return self._str()
        if typ == 9:
            sub, n = self._take("<IQ")
            return [self._value(sub) for _ in range(n)]
        raise ValueError(f"GGUF value type {typ}")

    def array(self, name: str) -> np.ndarray:
        """F32 / I8 tensors as arrays shaped [rows][cols] (ggml dims reversed)."""
        dims, typ, raw = self.tensors[name]
        dt = {GGML_F32: np.float32, GGML_F16: np.float16, GGML_I8: np.int8}[typ]
        return np.frombuffer(raw, dtype=dt).reshape(list(reversed(dims)))

    def q8_0(self, name: str):
        """A Q8_0 tensor as (codes int8 [rows][k], f16 scales [rows][k/32])."""
        dims, typ, raw = self.tensors[name]
        assert typ == GGML_Q8_0
        k, n = dims[0], int(np.prod(dims[1:]))
        blocks = np.frombuffer(raw, dtype=np.uint8).reshape(n, k // 32, 34)
        scales = blocks[:, :, :2].copy().view("<f2").reshape(n, k // 32)
        codes = blocks[:, :, 2:].copy().view(np.int8).reshape(n, k)
        return codes, scales
