"""The tensor-core batched path (M > 32) against the oracle, plus exact-integer and
determinism checks.  Outputs with fewer than 75 128x128 tiles split K over CTAs; the
split count is min(148 // tiles, scale groups of 8 blocks)."""
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
    return assert_close_to_oracle(y.cpu().numpy(), y_ref)


@pytest.mark.parametrize("m,k,n", [
    (17, 64, 128),      # one stage, partial M tile
    (33, 96, 130),      # odd block count (pad block), partial N tile
    (128, 2048, 256),   # exact tiles
    (200, 544, 300),    # 17 blocks, ragged everything; 3 splits, the last of one stage
    (64, 6144, 256),    # long K (down projection): 2 tiles x 24 splits
    (64, 6144, 2048),   # sweep shape down at M = 64: 16 tiles x 9 splits
    (64, 2048, 2050),   # 17 tiles x 8 splits, ragged last tile, N not a multiple of 4
    (96, 2048, 6144),   # sweep shape qkv: 48 tiles x 3 splits
    (300, 2048, 12288), # 288 tiles: no split
    (4096, 2048, 256),  # configs[3] prefill rows (M = 4096): 64 tiles x 2 splits
    (4096, 6144, 200),  # ... down-projection K, ragged N
])
def test_tc_matches_oracle(oracle_lib, cuda_device, m, k, n):
    _run(oracle_lib, cuda_device, 300 + m + k + n, m, k, n)


def test_tc_sweep_shape_m256(oracle_lib, cuda_device):
    _run(oracle_lib, cuda_device, 401, 256, 2048, 2048)


@pytest.mark.parametrize("k", [256, 2048])
def test_tc_integer_products_are_exact(cuda_device, k):
    """Unit scales: x holds integers with |x| <= 127 and amax 127 in every block, so the
    activation scale is exactly 1 and y is an exact integer dot product (K = 2048 adds
    the split partials, which are exact integers too)."""
    rng = np.random.default_rng(77)
    m, n = 130, 136
    x = rng.integers(-126, 127, size=(m, k)).astype(np.float32)
    x.reshape(m, k // 32, 32)[:, :, 0] = 127.0  # every block has amax 127 -> d = 1
    qs = rng.integers(-127, 128, size=(n, k // 32, 32), dtype=np.int8)
    blocks = np.empty((n, k // 32, 34), dtype=np.uint8)
    blocks[:, :, 0:2] = np.full((n, k // 32), 1.0, dtype=np.float16).view(np.uint8).reshape(n, k // 32, 2)
    blocks[:, :, 2:] = qs.view(np.uint8)
    q = QMatMul.from_gguf_blocks(blocks, n, k, device=cuda_device)
    y = q.forward(torch.from_numpy(x).to(cuda_device)).cpu().numpy()
    ref = x.astype(np.int64) @ qs.reshape(n, k).astype(np.int64).T
    assert np.array_equal(y.astype(np.int64), ref)
    assert np.abs(ref).max() < 2 ** 24  # so the f32 result is exact


def test_tc_split_k_is_deterministic(cuda_device):
    """Split-K partial tiles are added by a separate reduction kernel in split order."""
    x, w = synth.case(403, 64, 6144, 1024)
    q = QMatMul.from_gguf_blocks(w, 1024, 6144, device=cuda_device)
    xt = torch.from_numpy(x).to(cuda_device)
    first = q.forward(xt).cpu().numpy()
    for _ in range(5):
        assert np.array_equal(q.forward(xt).cpu().numpy(), first)


def test_tc_fault_word_clear(cuda_device):
    _, w = synth.case(402, 1, 128, 64)
    q = QMatMul.from_gguf_blocks(w, 64, 128, device=cuda_device)
    q.forward(torch.randn((40, 128), device=cuda_device))
    flags = ctypes.c_uint32(123)
    _lib.check(_lib.lib().q8lin_fault_status(0, ctypes.byref(flags), 1))
    assert flags.value == 0


def test_split_kernel_matches_oracle(cuda_device):
    """The exact-halves kernel (Q8LIN_F16_GEMM=split, read once per process, so in a child):
    parity with the oracle on a partial tile, an odd block count (last stage with one
    block), split-K and a long K over several 4-stage TMEM chunks."""
    import os
    import subprocess
    import sys
    import textwrap

    code = textwrap.dedent("""
        import numpy as np, torch
        from talechime_b200 import QMatMul, _lib, synth
        import oracle
        from tests.conftest import assert_close_to_oracle
        dev = torch.device("cuda", 0)
        for m, k, n in ((64, 2048, 2048), (100, 2080, 300), (33, 4096, 512), (200, 6144, 640)):
            assert _lib.PATH_NAMES[_lib.lib().q8lin_dispatch_path(m, k, n)] == "f16_tc"
            w = synth.q8_0_blocks(np.random.default_rng(m + k + n), n, k)
            q = QMatMul.from_gguf_blocks(w, n, k, device=dev)
            x = np.random.default_rng(m).standard_normal((m, k), dtype=np.float32)
            y = q.forward(torch.from_numpy(x).to(dev)).cpu().numpy()
            assert_close_to_oracle(y, oracle.matmul(x, w, n, threads=16))
        print("ok")
    """)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, Q8LIN_F16_GEMM="split", PYTHONPATH=root)
    r = subprocess.run([sys.executable, "-c", code], cwd=root, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]
