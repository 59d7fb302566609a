"""q8lin_forward_noalloc: the Q8_0 linear for callers that must not allocate.

Some callers cannot allocate device memory while they run -- a real-time audio
producer cannot stall on cudaMalloc's device synchronisation, and an embedder whose
allocator owns the device memory may forbid allocations behind its back.  For them
the library keeps the activation scratch in a fixed device array and exposes
q8lin_forward_noalloc.  This test calls it through the C ABI and checks it against
the regular q8lin_forward on two calls in a row (the second call reuses the scratch
the first one left behind).  It lives in its own file so that it runs after every
other test in a run that stops at the first failure.
"""
import ctypes

import numpy as np
import pytest
import torch

from talechime_b200 import QMatMul, _lib, synth
from tests.conftest import assert_close_to_oracle

pytestmark = pytest.mark.gpu


def _noalloc(q, x, m):
    y = torch.empty((m, q.n), dtype=torch.float32, device=x.device)
    st = _lib.lib().q8lin_forward_noalloc(q.handle, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()), m,
                                          ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream))
    _lib.check(st)
    return y


def test_noalloc_matches_forward_on_two_calls(cuda_device):
    cases = [(21, 64, 2048, 256), (22, 17, 1024, 130)]  # second call: different shape, same scratch
    for seed, m, k, n in cases:
        x, w = synth.case(seed, m, k, n)
        q = QMatMul.from_gguf_blocks(w, n, k, device=cuda_device)
        xd = torch.from_numpy(x).to(cuda_device)
        y_ref = q.forward(xd)
        y = _noalloc(q, xd, m)
        torch.cuda.synchronize()
        assert_close_to_oracle(y.cpu().numpy(), y_ref.cpu().numpy())


def test_noalloc_is_bit_exact_with_the_cpu_path(oracle_lib, cuda_device):
    """Its matmul adds the block terms in block order with candle's per-product rounding."""
    x, w = synth.case(24, 9, 1024, 200)
    q = QMatMul.from_gguf_blocks(w, 200, 1024, device=cuda_device)
    y = _noalloc(q, torch.from_numpy(x).to(cuda_device), 9)
    torch.cuda.synchronize()
    assert np.array_equal(y.cpu().numpy(), oracle_lib.matmul(x, w, 200, threads=16))


def test_noalloc_rejects_sizes_beyond_its_scratch(cuda_device):
    k, n = 2048, 64
    _, w = synth.case(23, 1, k, n)
    q = QMatMul.from_gguf_blocks(w, n, k, device=cuda_device)
    m = 8388608 // k + 1  # one row past the scratch limit
    x = torch.zeros((m, k), dtype=torch.float32, device=cuda_device)
    y = torch.empty((m, n), dtype=torch.float32, device=cuda_device)
    L = _lib.lib()
    st = L.q8lin_forward_noalloc(q.handle, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()), m, None)
    assert st == _lib.ERR_SHAPE
    assert b"no-allocation scratch limit" in L.q8lin_last_error()
    # at the limit itself the call runs
    m_ok = 8388608 // k
    y_ok = _noalloc(q, x[:m_ok].contiguous(), m_ok)
    torch.cuda.synchronize()
    assert np.all(y_ok.cpu().numpy() == 0.0)
