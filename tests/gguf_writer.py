"""Minimal GGUF writer for tests (published GGUF layout, versions 2 and 3).

Writes files for the C++ reader to parse: typed metadata, tensor infos and aligned
tensor data, with knobs to produce the malformed variants the reader must reject.
Test infrastructure only.
"""
from __future__ import annotations

import struct

import numpy as np

U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_FMT = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B", U64: "<Q",
        I64: "<q", F64: "<d"}
GGML_F32, GGML_F16, GGML_Q8_0 = 0, 1, 8


def _str(s) -> bytes:
    b = s.encode() if isinstance(s, str) else bytes(s)
    return struct.pack("<Q", len(b)) + b


def _value(t: int, v) -> bytes:
    if t == STRING:
        return _str(v)
    if t == ARRAY:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(_value(et, x) for x in items)
    return struct.pack(_FMT[t], v)


class Writer:
    def __init__(self, version: int = 3, alignment: int = 32):
        self.version = version
        self.alignment = alignment
        self.kv = []  # (key, type, value)
        self.tensors = []  # (name, ne, ggml_type, data bytes, offset override)
        if alignment != 32:
            self.add("general.alignment", U32, alignment)

    def add(self, key: str, t: int, v) -> "Writer":
        self.kv.append((key, t, v))
        return self

    def tensor(self, name: str, ne, ggml_type: int, data: bytes, offset=None) -> "Writer":
        self.tensors.append((name, tuple(int(x) for x in ne), ggml_type, bytes(data), offset))
        return self

    def f32(self, name: str, a: np.ndarray) -> "Writer":
        a = np.ascontiguousarray(a, dtype=np.float32)
        return self.tensor(name, tuple(reversed(a.shape)), GGML_F32, a.tobytes())

    def q8_0(self, name: str, blocks: np.ndarray, k: int) -> "Writer":
        b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1, k // 32 * 34)
        return self.tensor(name, (k, b.shape[0]), GGML_Q8_0, b.tobytes())

    def build(self) -> bytes:
        al = self.alignment
        head = struct.pack("<IIQQ", 0x46554747, self.version, len(self.tensors), len(self.kv))
        for key, t, v in self.kv:
            head += _str(key) + struct.pack("<I", t) + _value(t, v)
        data, offsets = b"", []
        for name, ne, gt, raw, off in self.tensors:
            pad = (-len(data)) % al
            data += b"\0" * pad
            offsets.append(len(data) if off is None else off)
            data += raw
        for (name, ne, gt, raw, off), o in zip(self.tensors, offsets):
            head += _str(name) + struct.pack("<I", len(ne)) + b"".join(struct.pack("<Q", x) for x in ne)
            head += struct.pack("<IQ", gt, o)
        head += b"\0" * ((-len(head)) % al)
        return head + data

    def write(self, path) -> str:
        with open(path, "wb") as f:
            f.write(self.build())
        return str(path)
