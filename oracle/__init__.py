"""CPU oracle for the Q8_0 quantized linear (TEST INFRASTRUCTURE ONLY).

ctypes bindings over ``oracle/_build/libq8oracle.so`` (built from
``oracle/q8_0_oracle.c`` by ``oracle/Makefile``), a restatement of candle-core
0.11.0's CPU ``QMatMul`` Q8_0 path that talechime calls through
``Linear::forward`` (crates/voxcpm/src/weights.rs:213-229).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may
import this module, and only as the checker or the timed CPU baseline.  The
product package ``talechime_b200`` never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "libq8oracle.so")
_lib = None

QK8_0 = 32
BLOCK_BYTES = 34


def build() -> str:
    """Compile the oracle with its Makefile (idempotent)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _SO


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_SO):
            build()
        L = ctypes.CDLL(_SO)
        L.q8o_f32_to_f16.argtypes = [ctypes.c_float]
        L.q8o_f32_to_f16.restype = ctypes.c_uint16
        L.q8o_f16_to_f32.argtypes = [ctypes.c_uint16]
        L.q8o_f16_to_f32.restype = ctypes.c_float
        L.q8o_quantize_row.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
        L.q8o_quantize_row.restype = ctypes.c_int
        L.q8o_quantize_planes.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                          ctypes.c_void_p, ctypes.c_void_p]
        L.q8o_quantize_planes.restype = ctypes.c_int
        L.q8o_dequantize_row.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
        L.q8o_dequantize_row.restype = ctypes.c_int
        L.q8o_matmul.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p,
                                 ctypes.c_int64, ctypes.c_void_p, ctypes.c_int]
        L.q8o_matmul.restype = ctypes.c_int
        L.q8o_swiglu.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p]
        L.q8o_swiglu.restype = ctypes.c_int
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def quantize(x: np.ndarray) -> np.ndarray:
    """f32 [..., K] -> uint8 GGUF Q8_0 blocks [..., K/32, 34]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    k = x.shape[-1]
    flat = x.reshape(-1, k)
    out = np.empty((flat.shape[0], k // QK8_0, BLOCK_BYTES), dtype=np.uint8)
    for r in range(flat.shape[0]):
        row = np.ascontiguousarray(flat[r])
        o = np.empty((k // QK8_0, BLOCK_BYTES), dtype=np.uint8)
        if lib().q8o_quantize_row(_ptr(row), k, _ptr(o)) != 0:
            raise ValueError(f"K={k} is not a multiple of 32")
        out[r] = o
    return out.reshape(x.shape[:-1] + (k // QK8_0, BLOCK_BYTES))


def quantize_planes(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """f32 [M, K] -> (qs int8 [M, K], d f16 [M, K/32]) with candle's activation rules."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    m, k = x.shape
    qs = np.empty((m, k), dtype=np.int8)
    d = np.empty((m, k // QK8_0), dtype=np.uint16)
    if lib().q8o_quantize_planes(_ptr(x), m, k, _ptr(qs), _ptr(d)) != 0:
        raise ValueError(f"K={k} is not a multiple of 32")
    return qs, d.view(np.float16)


def dequantize(blocks: np.ndarray, k: int) -> np.ndarray:
    """uint8 GGUF Q8_0 blocks for rows of K values -> f32 [rows, K]."""
    b = np.ascontiguousarray(blocks, dtype=np.uint8).reshape(-1, (k // QK8_0) * BLOCK_BYTES)
    out = np.empty((b.shape[0], k), dtype=np.float32)
    for r in range(b.shape[0]):
        row = np.ascontiguousarray(b[r])
        o = np.empty(k, dtype=np.float32)
        if lib().q8o_dequantize_row(_ptr(row), k, _ptr(o)) != 0:
            raise ValueError(f"K={k} is not a multiple of 32")
        out[r] = o
    return out


def matmul(x: np.ndarray, w_blocks: np.ndarray, n: int, threads: int = 1) -> np.ndarray:
    """candle CPU QMatMul::forward: x f32 [M, K] times Q8_0 W [N, K] -> y f32 [M, N]."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    m, k = x.shape
    w = np.ascontiguousarray(w_blocks, dtype=np.uint8)
    if w.size != n * (k // QK8_0) * BLOCK_BYTES:
        raise ValueError("weight block buffer does not match N x K")
    y = np.empty((m, n), dtype=np.float32)
    rc = lib().q8o_matmul(_ptr(x), m, k, _ptr(w), n, _ptr(y), int(threads))
    if rc != 0:
        raise ValueError(f"oracle matmul failed with status {rc}")
    return y


def swiglu(gu: np.ndarray) -> np.ndarray:
    """silu(gate) * up over gu f32 [M, 2I] (gate columns first) -> h f32 [M, I]."""
    gu = np.ascontiguousarray(gu, dtype=np.float32)
    m, two_i = gu.shape
    if two_i % 2:
        raise ValueError("gu must have an even number of columns")
    h = np.empty((m, two_i // 2), dtype=np.float32)
    rc = lib().q8o_swiglu(_ptr(gu), m, two_i // 2, _ptr(h))
    if rc != 0:
        raise ValueError(f"oracle swiglu failed with status {rc}")
    return h


def mlp(x: np.ndarray, gate: np.ndarray, up: np.ndarray, down: np.ndarray, hidden: int, inter: int,
        threads: int = 1) -> np.ndarray:
    """The VoxCPM MLP on the CPU path: down(silu(gate(x)) * up(x)), three candle
    QMatMul::forward calls (crates/voxcpm/src/transformer.rs:147-150)."""
    g = matmul(x, gate, inter, threads)
    u = matmul(x, up, inter, threads)
    return matmul(swiglu(np.concatenate([g, u], axis=1)), down, hidden, threads)


def f32_to_f16_bits(v: float) -> int:
    return int(lib().q8o_f32_to_f16(float(v)))


def f16_bits_to_f32(h: int) -> float:
    return float(lib().q8o_f16_to_f32(int(h)))
