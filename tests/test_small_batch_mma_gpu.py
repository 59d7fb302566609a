"""Small batches on mma.sync int8 (gemm_mma.cu): parity with the candle-CPU oracle.

The path serves 12 <= M <= 16 where the activations fit in shared memory beside the
weight rings (q8lin_dispatch_path == small_batch_mma); the activations are quantized with
candle's Q8_0 rules, once per call into the workspace or -- for small M*K and weights of
8192 rows or more -- by every CTA into its own shared memory, and every output is the sum
over blocks of ((f32(I) * dw) * dx) (candle-core 0.11.0 QMatMul::forward, called from
Linear::forward, crates/voxcpm/src/weights.rs:209-229).  Cases cover partial 16-row
tiles, a partial last 8-block unit, the regime where a CTA holds more tiles than warps
(each warp whole tiles) and the one where warps split a tile's units (partials added in
unit order), determinism, and -- in child processes -- M = 2..11 (Q8LIN_SMALL_MMA=1) and
each quantization variant forced where the default picks the other (Q8LIN_MMA_QUANT).
"""
import ctypes
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest
import torch

from talechime_b200 import QMatMul, _lib, synth
from tests.conftest import assert_close_to_oracle

pytestmark = pytest.mark.gpu

CASES = [
    (12, 2048, 2048),    # o, M = 12
    (16, 2048, 6144),    # qkv, M = 16
    (16, 2048, 12288),   # gate_up, M = 16 (x quantized in the kernel)
    (13, 2080, 100),     # partial tile (100 rows) and a partial last unit (65 blocks)
    (14, 2048, 28672),   # 1792 tiles: a CTA holds more tiles than warps (x in the kernel)
    (15, 512, 48),       # 3 tiles, 2 units each
    (12, 96, 17),        # one 3-block unit, one partial tile
]


@pytest.mark.parametrize("m,k,n", CASES, ids=[f"m{m}_k{k}_n{n}" for m, k, n in CASES])
def test_mma_path_matches_oracle(oracle_lib, cuda_device, m, k, n):
    assert _lib.PATH_NAMES[_lib.lib().q8lin_dispatch_path(m, k, n)] == "small_batch_mma"
    w = synth.q8_0_blocks(np.random.default_rng(m * 131 + k + n), n, k)
    q = QMatMul.from_gguf_blocks(w, n, k, device=cuda_device)
    x = np.random.default_rng(m + k).standard_normal((m, k), dtype=np.float32)
    xt = torch.from_numpy(x).to(cuda_device)
    y = q.forward(xt).cpu().numpy()
    assert_close_to_oracle(y, oracle_lib.matmul(x, w, n, threads=16))
    assert np.array_equal(q.forward(xt).cpu().numpy(), y)  # partial sums in a fixed order


def test_mma_path_needs_the_workspace(cuda_device):
    """The quantized activations live in the workspace: q8lin_forward without a bound one
    is refused (M = 16 here; the dp4a kernel below M = 12 needs none)."""
    m, k, n = 16, 2048, 256
    w = synth.q8_0_blocks(np.random.default_rng(5), n, k)
    L = _lib.lib()
    h = ctypes.c_void_p()
    _lib.check(L.q8lin_weight_create(w.ctypes.data, n, k, cuda_device.index, None, ctypes.byref(h)))
    try:
        assert L.q8lin_workspace_size(h, m) > 0
        assert L.q8lin_workspace_size(h, 11) == 0
        x = torch.zeros((m, k), device=cuda_device)
        y = torch.empty((m, n), device=cuda_device)
        st = L.q8lin_forward(h, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()), m, None)
        assert st == _lib.ERR_WORKSPACE
    finally:
        L.q8lin_weight_destroy(h)


def _child_parity(cases, **env_vars):
    """Run the mma path on `cases` in a child process with the given switches (each is
    read once per process) and check every case against the oracle."""
    code = textwrap.dedent(f"""
        import numpy as np, torch
        from talechime_b200 import QMatMul, _lib, synth
        import oracle
        from tests.conftest import assert_close_to_oracle
        dev = torch.device("cuda", 0)
        for m, k, n in {cases!r}:
            assert _lib.PATH_NAMES[_lib.lib().q8lin_dispatch_path(m, k, n)] == "small_batch_mma"
            w = synth.q8_0_blocks(np.random.default_rng(m + n), n, k)
            q = QMatMul.from_gguf_blocks(w, n, k, device=dev)
            x = np.random.default_rng(m).standard_normal((m, k), dtype=np.float32)
            y = q.forward(torch.from_numpy(x).to(dev)).cpu().numpy()
            assert_close_to_oracle(y, oracle.matmul(x, w, n, threads=16))
        print("ok")
    """)
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, PYTHONPATH=root, **env_vars)
    r = subprocess.run([sys.executable, "-c", code], cwd=root, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "ok" in r.stdout, r.stdout[-2000:] + r.stderr[-2000:]


def test_mma_kernel_below_its_range(cuda_device):
    """M = 2..11 through the same kernel (Q8LIN_SMALL_MMA=1), both quantization variants
    reached by the default choice ((2, 2048, 8192) quantizes x in the kernel)."""
    _child_parity(((2, 2048, 256), (3, 2080, 100), (5, 1024, 333), (8, 2048, 2048), (11, 256, 4100),
                   (2, 2048, 8192)), Q8LIN_SMALL_MMA="1")


def test_mma_quantization_variants_forced(cuda_device):
    """Each quantization variant where the default takes the other: x quantized in every
    CTA for short weights and partial tiles, and by a separate launch for gate_up."""
    _child_parity(((12, 2048, 2048), (13, 2080, 100), (15, 512, 48), (12, 96, 17), (16, 1024, 300)),
                  Q8LIN_MMA_QUANT="kernel")
    _child_parity(((16, 2048, 12288), (14, 2048, 28672)), Q8LIN_MMA_QUANT="launch")
