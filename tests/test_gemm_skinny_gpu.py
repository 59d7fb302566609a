"""The small-batch int8 tensor-core path (5 <= M <= 32) against the oracle."""
import ctypes

import numpy as np
import pytest
import torch

from talechime_b200 import QMatMul, _lib, synth
from tests.conftest import assert_close_to_oracle

pytestmark = pytest.mark.gpu


def _run(oracle_lib, dev, seed, m, k, n):
    x, w = synth.case(seed, m, k, n)
    y_ref = oracle_lib.matmul(x, w, n, threads=16)
    q = QMatMul.from_gguf_blocks(w, n, k, device=dev)
    y = q.forward(torch.from_numpy(x).to(dev))
    torch.cuda.synchronize()
    return y.cpu().numpy(), y_ref


@pytest.mark.parametrize("m,k,n", [
    (5, 32, 1),          # one block, one weight row (K <= 2048: the dp4a small-batch kernel)
    (6, 96, 130),        # three blocks, partial row tile (dp4a small-batch kernel)
    (7, 2080, 1),        # int8 tensor-core path from here on (K > 2048 with M > 6, or M > 16)
    (8, 2112, 130),      # partial stage, partial row tile
    (16, 2048, 2048),    # split-K over 16 row tiles
    (17, 2048, 256),     # Np = 32
    (31, 544, 300),      # Np = 32, ragged
    (32, 6144, 2048),    # Np = 32, long K
    (16, 14336, 512),    # config-4 down shard shape class: many blocks per split
])
def test_skinny_matches_oracle(oracle_lib, cuda_device, m, k, n):
    y, y_ref = _run(oracle_lib, cuda_device, 600 + m + k + n, m, k, n)
    assert_close_to_oracle(y, y_ref)


def test_skinny_without_split_is_bit_exact(oracle_lib, cuda_device):
    """150 row tiles fill the SMs without splitting K: one CTA adds every block of a row
    in block order with candle's per-product rounding, so the result is the CPU result.
    (K = 2080 keeps M = 8 on this path: past K = 2048 the dp4a small-batch kernel takes M <= 6.)"""
    y, y_ref = _run(oracle_lib, cuda_device, 611, 8, 2080, 128 * 150)
    assert np.array_equal(y, y_ref)


def test_skinny_repeated_calls_are_deterministic(cuda_device):
    """Split-K partials are added by a separate reduction kernel in split order."""
    x, w = synth.case(612, 8, 4096, 1024)
    q = QMatMul.from_gguf_blocks(w, 1024, 4096, device=cuda_device)
    xt = torch.from_numpy(x).to(cuda_device)
    first = q.forward(xt).cpu().numpy()
    for _ in range(5):
        assert np.array_equal(q.forward(xt).cpu().numpy(), first)


def test_skinny_fault_word_clear(cuda_device):
    _, w = synth.case(613, 1, 256, 256)
    q = QMatMul.from_gguf_blocks(w, 256, 256, device=cuda_device)
    q.forward(torch.randn((5, 256), device=cuda_device))
    flags = ctypes.c_uint32(123)
    _lib.check(_lib.lib().q8lin_fault_status(0, ctypes.byref(flags), 1))
    assert flags.value == 0
