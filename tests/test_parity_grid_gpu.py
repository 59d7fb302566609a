"""Parity of q8lin_forward with the candle-CPU oracle at the benchmark's full sizes.

The benchmark shape sweep is a grid of activation rows M in {1, 4, 16, 64, 256, 1024} over the
VoxCPM-style projection shapes qkv 2048->6144, o 2048->2048, gate_up 2048->12288 and
down 6144->2048, plus the real k/v projection 2048->256
(crates/voxcpm/src/transformer.rs:119-121,146,148-150, called through Linear::forward,
crates/voxcpm/src/weights.rs:213-229).  configs[3] runs M = 4096 and configs[4] the
per-rank shard shapes of the tensor-parallel MLP at hidden 4096 / intermediate 14336 on
P = 1, 2, 4, 8 GPUs.  Every case goes through QMatMul.forward (q8lin_forward) on the
exact weights and activations the oracle sees, at the north-star tolerance, and names
the kernel that served it (q8lin_dispatch_path); the grid must reach every kernel of the
dispatch table at full size.
"""
import numpy as np
import pytest
import torch

from talechime_b200 import QMatMul, _lib, synth
from tests.conftest import assert_close_to_oracle

pytestmark = pytest.mark.gpu

GRID_M = (1, 4, 16, 64, 256, 1024)
GRID_SHAPES = [("qkv", 2048, 6144), ("o", 2048, 2048), ("gate_up", 2048, 12288), ("down", 6144, 2048),
               ("kv", 2048, 256)]
THREADS = 16

_paths_seen = set()


def _check(oracle_lib, q, w, seed, m, k, n, device):
    x = np.random.default_rng(seed).standard_normal((m, k), dtype=np.float32)
    y = q.forward(torch.from_numpy(x).to(device))
    torch.cuda.synchronize()
    path = _lib.lib().q8lin_dispatch_path(m, k, n)
    assert path in _lib.PATH_NAMES
    _paths_seen.add(path)
    y_ref = oracle_lib.matmul(x, w, n, threads=THREADS)
    try:
        assert_close_to_oracle(y.cpu().numpy(), y_ref)
    except AssertionError as e:
        raise AssertionError(f"M={m} K={k} N={n} on {_lib.PATH_NAMES[path]}: {e}") from None


@pytest.mark.parametrize("name,k,n", GRID_SHAPES, ids=[s[0] for s in GRID_SHAPES])
def test_configs1_grid(oracle_lib, cuda_device, name, k, n):
    w = synth.q8_0_blocks(np.random.default_rng(sum(map(ord, name))), n, k)
    q = QMatMul.from_gguf_blocks(w, n, k, device=cuda_device)
    for m in GRID_M:
        _check(oracle_lib, q, w, 31 * m + k + n, m, k, n, cuda_device)


def test_configs3_prefill_rows(oracle_lib, cuda_device):
    """M = 4096 (4 x 1024 tokens) through the widest projection."""
    k, n = 2048, 12288
    w = synth.q8_0_blocks(np.random.default_rng(4096), n, k)
    q = QMatMul.from_gguf_blocks(w, n, k, device=cuda_device)
    _check(oracle_lib, q, w, 4097, 4096, k, n, cuda_device)


@pytest.mark.parametrize("p", [1, 2, 4, 8])
def test_configs4_shard_shapes(oracle_lib, cuda_device, p):
    """Per-rank shards of the tensor-parallel MLP: [gate | up] rows 4096 -> 2 * 14336 / P
    and the down projection's block columns 14336 / P -> 4096."""
    hidden, inter = 4096, 14336
    for name, k, n in (("gate_up", hidden, 2 * inter // p), ("down", inter // p, hidden)):
        w = synth.q8_0_blocks(np.random.default_rng(100 * p + len(name)), n, k)
        q = QMatMul.from_gguf_blocks(w, n, k, device=cuda_device)
        for m in (1, 16, 256):
            _check(oracle_lib, q, w, 7 * m + p + k, m, k, n, cuda_device)
        del q


def test_grid_reached_every_kernel():
    """The full-size cases above were served by every kernel of the dispatch table."""
    if not _paths_seen:
        pytest.skip("grid cases did not run in this session")
    missing = set(_lib.PATH_NAMES) - _paths_seen
    assert not missing, f"kernels not reached at full size: {[_lib.PATH_NAMES[p] for p in missing]}"
