"""GGUF files through libq8lin's reader (q8lin_gguf_* in include/q8lin.h).

Mirrors how the reference reaches its weights (crates/voxcpm/src/weights.rs):
``Weights::open`` (:31-41) -> ``GGUFFile(path)``; ``Weights::linear(name, false)``
(:96-115, Q8_0 branch :100-104) -> ``GGUFFile.linear(name)``; ``Weights::tensor``
(:74-95) -> ``GGUFFile.tensor(name)`` for the f32 / f16 vectors (norm weights, RoPE
factors); ``Weights::value`` / ``expect_u32`` / ``expect_string`` (:117-137), with the
reference's error messages.  Parsing and bounds checks are in C++ (gguf.cpp); this
module only converts the results.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from . import _lib
from ._lib import Q8LinError, check
from .qmatmul import QMatMul, _stream_ptr

GGML_F32, GGML_F16, GGML_Q8_0, GGML_BF16 = 0, 1, 8, 30
_U8, _I8, _U16, _I16, _U32, _I32, _F32, _BOOL, _STRING, _ARRAY, _U64, _I64, _F64 = range(13)
_NUMERIC_DTYPES = {_U8: np.uint8, _I8: np.int8, _U16: np.uint16, _I16: np.int16, _U32: np.uint32, _I32: np.int32,
                   _F32: np.float32, _BOOL: np.uint8, _U64: np.uint64, _I64: np.int64, _F64: np.float64}


@dataclass(frozen=True)
class TensorInfo:
    name: str
    ggml_type: int
    ne: tuple  # GGUF order: ne[0] is the contiguous dimension
    nbytes: int

    @property
    def shape(self) -> tuple:
        """Row-major shape (ne reversed), as candle reports it."""
        return tuple(reversed(self.ne))


class GGUFFile:
    """A read-only, memory-mapped GGUF file (versions 2 and 3)."""

    def __init__(self, path: str):
        self.path = str(path)
        h = ctypes.c_void_p()
        check(_lib.lib().q8lin_gguf_open(self.path.encode(), ctypes.byref(h)))
        self._h = h

    def close(self) -> None:
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            _lib.lib().q8lin_gguf_close(h)
        self._h = None

    def __enter__(self) -> "GGUFFile":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _handle(self) -> ctypes.c_void_p:
        if self._h is None:
            raise ValueError("GGUF file is closed")
        return self._h

    # -- header and tensors ----------------------------------------------------------
    @property
    def version(self) -> int:
        v = ctypes.c_uint32()
        check(_lib.lib().q8lin_gguf_version(self._handle(), ctypes.byref(v)))
        return int(v.value)

    def _info(self, index: int) -> TensorInfo:
        name = ctypes.c_char_p()
        t, nd = ctypes.c_uint32(), ctypes.c_uint32()
        dims = (ctypes.c_int64 * 4)()
        nb = ctypes.c_uint64()
        check(_lib.lib().q8lin_gguf_tensor_info(self._handle(), index, ctypes.byref(name), ctypes.byref(t),
                                                ctypes.byref(nd), dims, ctypes.byref(nb)))
        return TensorInfo(name.value.decode(), int(t.value), tuple(int(d) for d in dims[:nd.value]), int(nb.value))

    def tensor_names(self) -> list:
        n = _lib.lib().q8lin_gguf_tensor_count(self._handle())
        return [self._info(i).name for i in range(n)]

    def tensor_info(self, name: str) -> TensorInfo:
        idx = ctypes.c_int64()
        check(_lib.lib().q8lin_gguf_find_tensor(self._handle(), name.encode(), ctypes.byref(idx)))
        return self._info(idx.value)

    def __contains__(self, name: str) -> bool:
        idx = ctypes.c_int64()
        return _lib.lib().q8lin_gguf_find_tensor(self._handle(), name.encode(), ctypes.byref(idx)) == _lib.OK

    def raw(self, name: str) -> np.ndarray:
        """A copy of the tensor's bytes (uint8)."""
        idx = ctypes.c_int64()
        L = _lib.lib()
        check(L.q8lin_gguf_find_tensor(self._handle(), name.encode(), ctypes.byref(idx)))
        ptr, nb = ctypes.c_void_p(), ctypes.c_uint64()
        check(L.q8lin_gguf_tensor_data(self._handle(), idx.value, ctypes.byref(ptr), ctypes.byref(nb)))
        return np.ctypeslib.as_array((ctypes.c_uint8 * nb.value).from_address(ptr.value)).copy()

    def tensor(self, name: str) -> np.ndarray:
        """An f32 / f16 / bf16 tensor as f32 numpy (row-major shape).  Q8_0 matrices are
        kept quantized: use linear() or q8_0_blocks()."""
        info = self.tensor_info(name)
        b = self.raw(name)
        if info.ggml_type == GGML_F32:
            a = b.view(np.float32)
        elif info.ggml_type == GGML_F16:
            a = b.view(np.float16).astype(np.float32)
        elif info.ggml_type == GGML_BF16:
            a = (b.view(np.uint16).astype(np.uint32) << 16).view(np.float32)
        else:
            raise Q8LinError(_lib.ERR_FORMAT, f"tensor '{name}' has ggml type {info.ggml_type}; "
                                              "tensor() reads F32, F16 and BF16")
        return a.reshape(info.shape)

    def q8_0_blocks(self, name: str) -> np.ndarray:
        """The GGUF Q8_0 blocks of a matrix as uint8 [rows, K/32 * 34]."""
        info = self.tensor_info(name)
        if info.ggml_type != GGML_Q8_0:
            raise Q8LinError(_lib.ERR_FORMAT, f"tensor '{name}' has ggml type {info.ggml_type}, not Q8_0")
        k = info.ne[0]
        return self.raw(name).reshape(-1, k // 32 * 34)

    def linear(self, name: str, device: Optional[torch.device | int | str] = None) -> QMatMul:
        """``Weights::linear(name, false)``: the Q8_0 tensor ``{name}.weight`` as a device
        QMatMul (uploaded straight from the mapping)."""
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        device = torch.device(device)
        tname = f"{name}.weight"
        info = self.tensor_info(tname)
        h = ctypes.c_void_p()
        with torch.cuda.device(device):
            check(_lib.lib().q8lin_gguf_weight_create(self._handle(), tname.encode(), device.index,
                                                      ctypes.c_void_p(_stream_ptr(device)), ctypes.byref(h)))
        return QMatMul(h, info.ne[1], info.ne[0], device)

    # -- metadata ----------------------------------------------------------------------
    def value(self, key: str):
        """The metadata value as a Python object (arrays of numbers as numpy, arrays of
        strings as lists)."""
        L, h, k = _lib.lib(), self._handle(), key.encode()
        t = ctypes.c_uint32()
        st = L.q8lin_gguf_metadata_type(h, k, ctypes.byref(t))
        if st == _lib.ERR_NOT_FOUND:
            raise Q8LinError(st, f"missing GGUF metadata {key}")
        check(st)
        t = t.value
        if t == _STRING:
            p, n = ctypes.c_void_p(), ctypes.c_uint64()
            check(L.q8lin_gguf_metadata_string(h, k, ctypes.byref(p), ctypes.byref(n)))
            return ctypes.string_at(p.value, n.value).decode("utf-8", errors="replace") if n.value else ""
        if t == _ARRAY:
            et, cnt, p, nb = ctypes.c_uint32(), ctypes.c_uint64(), ctypes.c_void_p(), ctypes.c_uint64()
            check(L.q8lin_gguf_metadata_array(h, k, ctypes.byref(et), ctypes.byref(cnt), ctypes.byref(p),
                                              ctypes.byref(nb)))
            raw = ctypes.string_at(p.value, nb.value) if nb.value else b""
            if et.value in _NUMERIC_DTYPES:
                a = np.frombuffer(raw, dtype=_NUMERIC_DTYPES[et.value]).copy()
                return a.astype(bool) if et.value == _BOOL else a
            if et.value == _STRING:
                out, off = [], 0
                for _ in range(cnt.value):
                    n = int.from_bytes(raw[off:off + 8], "little")
                    out.append(raw[off + 8:off + 8 + n].decode("utf-8", errors="replace"))
                    off += 8 + n
                return out
            raise Q8LinError(_lib.ERR_FORMAT, f"GGUF metadata {key}: nested arrays are not decoded")
        if t in (_F32, _F64):
            v = ctypes.c_double()
            check(L.q8lin_gguf_metadata_f64(h, k, ctypes.byref(v)))
            return float(v.value)
        v = ctypes.c_int64()
        check(L.q8lin_gguf_metadata_i64(h, k, ctypes.byref(v)))
        return bool(v.value) if t == _BOOL else int(v.value)

    def to_u32(self, key: str) -> int:
        v = ctypes.c_uint32()
        st = _lib.lib().q8lin_gguf_metadata_u32(self._handle(), key.encode(), ctypes.byref(v))
        if st == _lib.ERR_NOT_FOUND:
            raise Q8LinError(st, f"missing GGUF metadata {key}")
        check(st)
        return int(v.value)

    def expect_u32(self, key: str, expected: int) -> None:
        actual = self.to_u32(key)
        if actual != expected:
            raise Q8LinError(_lib.ERR_FORMAT, f"unsupported GGUF {key}={actual}; expected {expected}")

    def expect_string(self, key: str, expected: str) -> None:
        actual = self.value(key)
        if not isinstance(actual, str):
            raise Q8LinError(_lib.ERR_FORMAT, f"GGUF metadata {key} is not a string")
        if actual != expected:
            raise Q8LinError(_lib.ERR_FORMAT, f"unsupported GGUF {key}={actual}; expected {expected}")
