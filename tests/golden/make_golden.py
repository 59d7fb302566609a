"""Generate tests/golden/q8_0_golden.npz, the fixtures that pin the CPU oracle.

Run in an environment that has the ``gguf`` Python package (0.19.0 was used):

    python tests/golden/make_golden.py

Sources of truth (independent of oracle/q8_0_oracle.c):

* quantize / dequantize: ``gguf.quants.quantize`` / ``dequantize`` with
  ``GGMLQuantizationType.Q8_0`` -- gguf-py's numpy Q8_0, which states that it is
  bit-exact with ggml-quants.c's reference quantizer (``d = amax/127``,
  ``id = 1/d``, round half away from zero, ``d`` stored f16).  candle-core's
  ``BlockQ8_0::from_float`` follows the same rules.
* matmul: a numpy restatement of candle's scalar ``vec_dot_unopt`` loop written
  here (activations quantized with gguf-py, per-block ``(f32(isum)*dw)*dx`` and
  a sequential f32 sum over blocks).  float64 dequantized products are stored
  beside it as the mathematical reference.

The reference repository has no Q8_0 golden vectors of its own (its Q8 numerical
checks need external weights), so these are the pins.
"""
from __future__ import annotations

import os
import sys

import numpy as np
from gguf import GGMLQuantizationType as QT
from gguf import quants

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from talechime_b200 import synth  # noqa: E402

Q8 = QT.Q8_0


def quant_cases() -> np.ndarray:
    rng = np.random.default_rng(1234)
    rows = []
    rows.append(rng.standard_normal(256, dtype=np.float32))
    rows.append(rng.standard_normal(256, dtype=np.float32) * np.float32(1e-3))
    rows.append(rng.standard_normal(256, dtype=np.float32) * np.float32(300.0))
    rows.append(rng.uniform(-1, 1, 256).astype(np.float32))
    edge = np.zeros(256, dtype=np.float32)
    # block 0: all zero (d = 0, q = 0)
    # block 1: amax = 127 -> d = 1, id = 1: exact half ties round away from zero
    edge[32:64] = np.float32(0.5) * np.arange(-16, 16, dtype=np.float32)
    edge[63] = 127.0
    # block 2: saturating extremes +-amax
    edge[64:96] = np.where(np.arange(32) % 2 == 0, 3.25, -3.25).astype(np.float32)
    # block 3: tiny values -> subnormal f16 scale
    edge[96:128] = rng.standard_normal(32).astype(np.float32) * np.float32(1e-6)
    # block 4: scale that overflows to f16 inf (amax/127 > 65504)
    edge[128:160] = rng.standard_normal(32).astype(np.float32) * np.float32(3e7)
    # block 5: a single non-zero element
    edge[160 + 7] = np.float32(-0.0123)
    # block 6: values at the f16 subnormal/normal boundary of d
    edge[192:224] = np.linspace(-127 * 6.1e-5, 127 * 6.1e-5, 32, dtype=np.float32)
    # block 7: negative zeros and one tie below amax
    edge[224:256] = np.float32(-0.0)
    edge[224] = np.float32(2.0)
    edge[225] = np.float32(-2.0 * 63.5 / 127.0)
    rows.append(edge)
    return np.stack(rows).astype(np.float32)


def dequant_cases() -> np.ndarray:
    rng = np.random.default_rng(99)
    nblk = 64
    out = np.empty((nblk, 34), dtype=np.uint8)
    out[:, 2:] = rng.integers(-128, 128, size=(nblk, 32), dtype=np.int8).view(np.uint8)
    d_bits = rng.integers(0, 0x7c00, size=nblk, dtype=np.uint16)  # finite, incl. subnormal
    sign = rng.integers(0, 2, size=nblk, dtype=np.uint16) << 15
    d_bits = d_bits | sign
    d_bits[0] = 0x0000
    d_bits[1] = 0x0001  # smallest subnormal
    d_bits[2] = 0x03ff  # largest subnormal
    d_bits[3] = 0x7bff  # 65504
    out[:, 0:2] = d_bits.view(np.uint8).reshape(nblk, 2)
    return out


def candle_scalar_matmul(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """numpy restatement of candle's scalar loop (independent of the C oracle)."""
    m, k = x.shape
    n, nb, _ = w.shape
    xb = quants.quantize(x, Q8).reshape(m, nb, 34)
    dx = np.ascontiguousarray(xb[:, :, 0:2]).view(np.float16).reshape(m, nb).astype(np.float32)
    qx = np.ascontiguousarray(xb[:, :, 2:]).view(np.int8).reshape(m, nb, 32).astype(np.int32)
    qw_all, dw_all = synth.split_blocks(w)
    qw = qw_all.reshape(n, nb, 32).astype(np.int32)
    dw = dw_all.astype(np.float32)
    y = np.zeros((m, n), dtype=np.float32)
    for r in range(m):
        isum = np.einsum("nbj,bj->nb", qw, qx[r])  # exact int32
        s = np.zeros(n, dtype=np.float32)
        for b in range(nb):
            term = (isum[:, b].astype(np.float32) * dw[:, b]) * dx[r, b]
            s = (s + term).astype(np.float32)
        y[r] = s
    return y


def main() -> None:
    out = {}
    qx = quant_cases()
    out["quant_x"] = qx
    out["quant_blocks"] = quants.quantize(qx, Q8).reshape(qx.shape[0], -1, 34)
    db = dequant_cases()
    out["dequant_blocks"] = db
    out["dequant_y"] = quants.dequantize(db.reshape(1, -1), Q8).reshape(-1).astype(np.float32)
    mm_shapes = [(1, 64, 8), (3, 256, 17), (16, 512, 33), (5, 2048, 12), (17, 96, 40)]
    for i, (m, k, n) in enumerate(mm_shapes):
        x, w = synth.case(100 + i, m, k, n)
        out[f"mm{i}_x"] = x
        out[f"mm{i}_w"] = w
        out[f"mm{i}_y"] = candle_scalar_matmul(x, w)
        xd = quants.dequantize(quants.quantize(x, Q8), Q8).astype(np.float64)
        wd = quants.dequantize(w.reshape(n, -1), Q8).astype(np.float64)
        out[f"mm{i}_y64"] = xd @ wd.T
    out["mm_shapes"] = np.array(mm_shapes, dtype=np.int64)
    path = os.path.join(HERE, "q8_0_golden.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


if __name__ == "__main__":
    main()
