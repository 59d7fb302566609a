"""Seeded synthetic inputs with the shapes and value distributions of the Q8_0 configs.

The reference measures on real VoxCPM2 GGUF weights that are not available offline;
these generators stand in for them:

* activations x: f32 ~ N(0, 1)
* Q8_0 weights: per 32-value block, ``qs`` uniform over the integers [-127, 127] and
  ``d = f16(|N(0, 0.02)| / 127)``, packed in the GGUF byte layout
  ``{f16 d (little endian); int8 qs[32]}`` (34 bytes per block), N rows of K/32
  blocks, as candle's ``QTensor`` holds them (crates/voxcpm/src/weights.rs:100-104).

Draw order for one (seed, M, K, N) case: x first, then qs, then d.
"""
from __future__ import annotations

import numpy as np

QK8_0 = 32
BLOCK_BYTES = 34

# (K, N) projection shapes of the shape sweep: fused QKV, O, fused gate+up, down.
SWEEP_SHAPES = {
    "qkv": (2048, 6144),
    "o": (2048, 2048),
    "gate_up": (2048, 12288),
    "down": (6144, 2048),
}
SWEEP_M = (1, 4, 16, 64, 256, 1024)


def q8_0_blocks(rng: np.random.Generator, n: int, k: int) -> np.ndarray:
    """uint8 [n, k/32, 34] GGUF Q8_0 blocks."""
    if k % QK8_0:
        raise ValueError("K must be a multiple of 32")
    nb = k // QK8_0
    qs = rng.integers(-127, 128, size=(n, nb, QK8_0), dtype=np.int8)
    d = (np.abs(rng.normal(0.0, 0.02, size=(n, nb))) / 127.0).astype(np.float16)
    out = np.empty((n, nb, BLOCK_BYTES), dtype=np.uint8)
    out[:, :, 0:2] = d.view(np.uint8).reshape(n, nb, 2)
    out[:, :, 2:] = qs.view(np.uint8)
    return out


def case(seed: int, m: int, k: int, n: int) -> tuple[np.ndarray, np.ndarray]:
    """(x f32 [m, k], W blocks uint8 [n, k/32, 34]) for one seeded case."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k), dtype=np.float32)
    w = q8_0_blocks(rng, n, k)
    return x, w


def split_blocks(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """GGUF blocks [n, nb, 34] -> (qs int8 [n, nb*32], d f16 [n, nb])."""
    n, nb, _ = w.shape
    d = np.ascontiguousarray(w[:, :, 0:2]).view(np.float16).reshape(n, nb)
    qs = np.ascontiguousarray(w[:, :, 2:]).view(np.int8).reshape(n, nb * QK8_0)
    return qs, d
