"""Parity of the CUDA Q8_0 linear (through the C ABI) with the candle-CPU oracle."""
import numpy as np
import pytest
import torch

from talechime_b200 import Linear, Q8LinError, QMatMul, quantize_rows
from talechime_b200 import synth
from tests.conftest import assert_close_to_oracle

pytestmark = pytest.mark.gpu


def run_case(oracle_lib, device, seed, m, k, n, threads=8):
    x, w = synth.case(seed, m, k, n)
    y_ref = oracle_lib.matmul(x, w, n, threads=threads)
    q = QMatMul.from_gguf_blocks(w, n, k, device=device)
    y = q.forward(torch.from_numpy(x).to(device))
    torch.cuda.synchronize()
    return assert_close_to_oracle(y.cpu().numpy(), y_ref)


@pytest.mark.parametrize("m", list(range(1, 17)))
def test_gemv_all_m_small(oracle_lib, cuda_device, m):
    run_case(oracle_lib, cuda_device, 10 + m, m, 256, 67)


@pytest.mark.parametrize("k,n", [(32, 1), (64, 3), (96, 200), (544, 33), (2048, 256), (6144, 40)])
def test_gemv_ragged_shapes(oracle_lib, cuda_device, k, n):
    for m in (1, 3, 16):
        run_case(oracle_lib, cuda_device, k + n + m, m, k, n)


@pytest.mark.parametrize("m,k,n", [
    (3, 2048, 4096),   # M = 3, 4 with N*K >= 8M weights: the dp4a small-batch kernel
    (4, 1024, 8200),   # ... ragged N
    (4, 2048, 2048),   # below 8M weights: the register-streaming GEMV
    (2, 6144, 300),    # K > 2048, M <= 6: the dp4a small-batch kernel
    (4, 6144, 130),
    (6, 4096, 257),
    (2, 2048, 6144),   # M = 2 at K <= 2048: the register-streaming GEMV
])
def test_small_batch_dispatch_shapes(oracle_lib, cuda_device, m, k, n):
    run_case(oracle_lib, cuda_device, 700 + m + k + n, m, k, n, threads=16)


def test_config0_single_linear(oracle_lib, cuda_device):
    # the single-linear benchmark case: x [1,2048], W 2048x2048 Q8_0, seed 0
    run_case(oracle_lib, cuda_device, 0, 1, 2048, 2048)


@pytest.mark.parametrize("m", [17, 33, 64, 100])
def test_batched_path(oracle_lib, cuda_device, m):
    run_case(oracle_lib, cuda_device, 1000 + m, m, 512, 130)


def test_batched_sweep_shape(oracle_lib, cuda_device):
    run_case(oracle_lib, cuda_device, 5, 64, 2048, 2048)


def test_weight_export_round_trip(cuda_device):
    _, w = synth.case(3, 1, 320, 37)
    q = QMatMul.from_gguf_blocks(w, 37, 320, device=cuda_device)
    back = q.to_gguf_blocks().cpu().numpy()
    assert np.array_equal(back, w)
    # device-resident source blocks take the same path
    q2 = QMatMul.from_gguf_blocks(torch.from_numpy(w.reshape(-1)).to(cuda_device), 37, 320, device=cuda_device)
    assert np.array_equal(q2.to_gguf_blocks().cpu().numpy(), w)


def test_dequantize_bit_exact(oracle_lib, cuda_device):
    _, w = synth.case(4, 1, 256, 19)
    q = QMatMul.from_gguf_blocks(w, 19, 256, device=cuda_device)
    got = q.dequantize().cpu().numpy()
    ref = oracle_lib.dequantize(w.reshape(19, -1), 256)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_activation_quantization_bit_exact(oracle_lib, cuda_device):
    g = np.load("tests/golden/q8_0_golden.npz")
    x = g["quant_x"]
    qs, d = quantize_rows(torch.from_numpy(x).to(cuda_device))
    blocks = g["quant_blocks"]
    assert np.array_equal(qs.cpu().numpy().view(np.uint8).reshape(x.shape[0], -1, 32), blocks[:, :, 2:])
    assert np.array_equal(d.cpu().numpy().view(np.uint8).reshape(x.shape[0], -1, 2), blocks[:, :, :2])
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((33, 4096)) * rng.uniform(1e-4, 1e3, (33, 1))).astype(np.float32)
    qs, d = quantize_rows(torch.from_numpy(x).to(cuda_device))
    qs_ref, d_ref = oracle_lib.quantize_planes(x)
    assert np.array_equal(qs.cpu().numpy(), qs_ref)
    assert np.array_equal(d.cpu().numpy().view(np.uint16), d_ref.view(np.uint16))


def test_edge_activations(oracle_lib, cuda_device):
    # zeros, exact-half ties, a saturating block and a huge-scale block in one input
    g = np.load("tests/golden/q8_0_golden.npz")
    x = g["quant_x"].copy()
    x[4, 128:160] = 0.0  # keep d finite so the reference output is finite
    _, w = synth.case(6, 1, x.shape[1], 50)
    y_ref = oracle_lib.matmul(x, w, 50)
    q = QMatMul.from_gguf_blocks(w, 50, x.shape[1], device=cuda_device)
    y = q.forward(torch.from_numpy(x).to(cuda_device)).cpu().numpy()
    assert_close_to_oracle(y, y_ref)


def test_empty_input_is_noop(cuda_device):
    _, w = synth.case(7, 1, 64, 5)
    q = QMatMul.from_gguf_blocks(w, 5, 64, device=cuda_device)
    y = q.forward(torch.empty((0, 64), device=cuda_device))
    assert y.shape == (0, 5)


def test_shape_errors_like_candle(cuda_device):
    _, w = synth.case(8, 1, 64, 5)
    q = QMatMul.from_gguf_blocks(w, 5, 64, device=cuda_device)
    with pytest.raises(Q8LinError):
        q.forward(torch.zeros(64, device=cuda_device))
    with pytest.raises(Q8LinError):
        q.forward(torch.zeros((2, 32), device=cuda_device))
    with pytest.raises(Q8LinError):
        q.forward(torch.zeros((2, 64), device=cuda_device, dtype=torch.float16))
    with pytest.raises(Q8LinError):
        QMatMul.from_gguf_blocks(w.reshape(-1)[:-1], 5, 64, device=cuda_device)


def test_linear_flattens_leading_dims(oracle_lib, cuda_device):
    x, w = synth.case(9, 6, 128, 24)
    y_ref = oracle_lib.matmul(x, w, 24)
    lin = Linear(QMatMul.from_gguf_blocks(w, 24, 128, device=cuda_device))
    y = lin.forward(torch.from_numpy(x).to(cuda_device).reshape(2, 3, 128))
    assert y.shape == (2, 3, 24)
    assert_close_to_oracle(y.reshape(6, 24).cpu().numpy(), y_ref)
    bias = torch.arange(24, dtype=torch.float32, device=cuda_device)
    y2 = Linear(lin.mat, bias).forward(torch.from_numpy(x).to(cuda_device))
    # (y + b) - b re-rounds y in f32, so compare with an absolute tolerance
    assert torch.allclose(y2 - bias, y.reshape(6, 24), rtol=0.0, atol=1e-5)


def test_forward_ws_requires_workspace(cuda_device):
    import ctypes

    from talechime_b200 import _lib

    x, w = synth.case(11, 40, 64, 8)
    q = QMatMul.from_gguf_blocks(w, 8, 64, device=cuda_device)
    xd = torch.from_numpy(x).to(cuda_device)
    y = torch.empty((40, 8), device=cuda_device)
    L = _lib.lib()
    need = L.q8lin_workspace_size(q.handle, 40)
    assert need > 0
    st = L.q8lin_forward_ws(q.handle, ctypes.c_void_p(xd.data_ptr()), ctypes.c_void_p(y.data_ptr()), 40,
                            None, 0, None)
    assert st == _lib.ERR_WORKSPACE
    ws = torch.empty(need, dtype=torch.uint8, device=cuda_device)
    st = L.q8lin_forward_ws(q.handle, ctypes.c_void_p(xd.data_ptr()), ctypes.c_void_p(y.data_ptr()), 40,
                            ctypes.c_void_p(ws.data_ptr()), need,
                            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0
    torch.cuda.synchronize()
    assert torch.equal(y, q.forward(xd))


def test_forward_needs_a_bound_workspace_and_allocates_nothing(oracle_lib, cuda_device):
    """q8lin_forward reads scratch only from the workspace bound to the weight: without one
    it returns Q8LIN_ERR_WORKSPACE; with one it runs inside a CUDA-graph capture in global
    mode, where any device allocation would make the capture fail."""
    import ctypes

    from talechime_b200 import _lib

    m, k, n = 40, 256, 72
    x, w = synth.case(12, m, k, n)
    q = QMatMul.from_gguf_blocks(w, n, k, device=cuda_device)
    xd = torch.from_numpy(x).to(cuda_device)
    y = torch.zeros((m, n), device=cuda_device)
    L = _lib.lib()
    s = torch.cuda.Stream(cuda_device)
    args = (q.handle, ctypes.c_void_p(xd.data_ptr()), ctypes.c_void_p(y.data_ptr()), m, ctypes.c_void_p(s.cuda_stream))
    assert L.q8lin_forward(*args) == _lib.ERR_WORKSPACE
    assert b"q8lin_weight_bind_workspace" in L.q8lin_last_error()
    q.reserve(64)
    _lib.check(L.q8lin_forward(*args))  # eager warm-up (kernel attributes) before the capture
    torch.cuda.synchronize()
    y.zero_()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s, capture_error_mode="global"):
        st = L.q8lin_forward(*args)
    assert st == 0
    g.replay()
    torch.cuda.synchronize()
    assert_close_to_oracle(y.cpu().numpy(), oracle_lib.matmul(x, w, n, threads=8))
