"""The CPU oracle against the committed golden fixtures (no GPU).

Fixtures: tests/golden/q8_0_golden.npz, made by tests/golden/make_golden.py from
gguf-py 0.19.0's Q8_0 (quantize/dequantize) and a numpy restatement of candle's
scalar vec_dot loop (matmul).
"""
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "q8_0_golden.npz")


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def test_quantize_bit_exact_vs_gguf(oracle_lib, golden):
    got = oracle_lib.quantize(golden["quant_x"])
    assert np.array_equal(got, golden["quant_blocks"])


def test_quantize_planes_agree_with_blocks(oracle_lib, golden):
    x = golden["quant_x"]
    qs, d = oracle_lib.quantize_planes(x)
    blocks = golden["quant_blocks"]
    assert np.array_equal(qs.view(np.uint8).reshape(x.shape[0], -1, 32), blocks[:, :, 2:])
    assert np.array_equal(d.view(np.uint8).reshape(x.shape[0], -1, 2), blocks[:, :, :2])


def test_dequantize_bit_exact_vs_gguf(oracle_lib, golden):
    b = golden["dequant_blocks"]
    got = oracle_lib.dequantize(b.reshape(1, -1), b.shape[0] * 32).reshape(-1)
    assert np.array_equal(got.view(np.uint32), golden["dequant_y"].view(np.uint32))


@pytest.mark.parametrize("i", range(5))
def test_matmul_bit_exact_vs_scalar_restatement(oracle_lib, golden, i):
    m, k, n = (int(v) for v in golden["mm_shapes"][i])
    x, w = golden[f"mm{i}_x"], golden[f"mm{i}_w"]
    for threads in (1, 3):
        y = oracle_lib.matmul(x, w, n, threads=threads)
        assert np.array_equal(y.view(np.uint32), golden[f"mm{i}_y"].view(np.uint32))
    y64 = golden[f"mm{i}_y64"]
    assert np.linalg.norm(y - y64) / np.linalg.norm(y64) < 1e-6


def test_f16_decode_exhaustive(oracle_lib):
    bits = np.arange(65536, dtype=np.uint16)
    ref = bits.view(np.float16).astype(np.float32)
    got = np.array([oracle_lib.f16_bits_to_f32(int(b)) for b in bits], dtype=np.float32)
    finite = np.isfinite(ref)
    assert np.array_equal(got[finite].view(np.uint32), ref[finite].view(np.uint32))
    assert np.all(np.isnan(got[np.isnan(ref)]))
    assert np.array_equal(got[np.isinf(ref)], ref[np.isinf(ref)])


def test_f16_encode_matches_numpy_rne(oracle_lib):
    rng = np.random.default_rng(7)
    vals = np.concatenate([
        rng.standard_normal(4000).astype(np.float32) * np.float32(1e-5),
        rng.standard_normal(4000).astype(np.float32),
        rng.standard_normal(2000).astype(np.float32) * np.float32(3e4),
        # ties at f16 subnormal and normal spacing
        (np.arange(1, 200, dtype=np.float32) + np.float32(0.5)) * np.float32(2.0 ** -24),
        (np.float32(1.0) + (np.arange(0, 200, dtype=np.float32) + np.float32(0.5)) * np.float32(2.0 ** -10)),
        np.array([65504, 65519.99, 65520, 1e10, 2.0 ** -25, 2.0 ** -25 * 1.0001, 0.0, -0.0,
                  6.103515625e-05, 6.1e-05], dtype=np.float32),
    ])
    with np.errstate(over="ignore"):
        ref = vals.astype(np.float16).view(np.uint16)
    got = np.array([oracle_lib.f32_to_f16_bits(float(v)) for v in vals], dtype=np.uint16)
    assert np.array_equal(got, ref)


def test_candle_cast_rules_for_non_finite(oracle_lib):
    # Rust `as i8` saturates and maps NaN to 0; f32::max skips NaN.
    x = np.zeros(32, dtype=np.float32)
    x[0] = np.inf
    x[1] = 1.0
    x[2] = np.nan
    b = oracle_lib.quantize(x)  # one block: shape (1, 34)
    assert b[0, 0:2].view(np.float16)[0] == np.float16(np.inf)
    qs = b[0, 2:].view(np.int8)
    assert qs[0] == 0 and qs[1] == 0 and qs[2] == 0  # id = 1/inf = 0 -> inf*0 = NaN -> 0
    # tiny amax: d subnormal in f32, 1/d overflows to inf -> saturating casts
    x = np.zeros(32, dtype=np.float32)
    x[0] = np.float32(1e-40)
    x[1] = np.float32(-1e-40)
    qs = oracle_lib.quantize(x)[0, 2:].view(np.int8)
    assert qs[0] == 127 and qs[1] == -128 and qs[2] == 0


def test_matmul_rejects_bad_k(oracle_lib):
    with pytest.raises(ValueError):
        oracle_lib.matmul(np.zeros((1, 33), np.float32), np.zeros(34, np.uint8), 1)
