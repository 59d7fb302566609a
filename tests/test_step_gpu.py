"""Persistent decode-step kernel (q8lin_step_*): its GEMV operations against the oracle.

Each program is run through the C ABI; outputs are compared with the CPU restatement at
the linear's tolerance (rel-L2 <= 1e-5), including chained operations (the arrival-
counter barrier between them), K spanning several 2048-value segments, the SwiGLU
epilogue, residual adds, the argmax epilogue + ARGMAX operation, and repeated launches
(counters back at zero after each run).
"""
import ctypes

import numpy as np
import pytest
import torch

from talechime_b200 import QMatMul, _lib, synth
from tests.conftest import assert_close_to_oracle

pytestmark = pytest.mark.gpu


def _p(t):
    return t.data_ptr()


class _Program:
    def __init__(self, ops, dev):
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.token = torch.zeros(1, dtype=torch.int32, device=dev)
        arr = (_lib.Op * len(ops))(*ops)
        self.h = ctypes.c_void_p()
        _lib.check(_lib.lib().q8lin_step_create(arr, len(ops), ctypes.c_void_p(_p(self.pos)),
                                                ctypes.c_void_p(_p(self.token)), dev.index, ctypes.byref(self.h)))

    def run(self):
        _lib.check(_lib.lib().q8lin_step_run(self.h, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
        torch.cuda.synchronize()

    def __del__(self):
        _lib.lib().q8lin_step_destroy(self.h)


def _gemv(q, x, y, **kw):
    return _lib.Op(kind=_lib.OP_GEMV, weight=q.handle.value, x=_p(x), y=_p(y), **kw)


def _fault_clear():
    st = ctypes.c_uint32(0)
    _lib.check(_lib.lib().q8lin_fault_status(torch.cuda.current_device(), ctypes.byref(st), 1))
    return st.value


@pytest.mark.parametrize("k,n", [(2048, 6144), (6144, 2048), (8192, 300), (256, 1000), (1024, 37)])
def test_single_gemv_matches_oracle(oracle_lib, cuda_device, k, n):
    rng = np.random.default_rng(k + n)
    w = synth.q8_0_blocks(rng, n, k)
    q = QMatMul.from_gguf_blocks(w, n, k, device=cuda_device)
    x = rng.standard_normal(k).astype(np.float32)
    xd = torch.from_numpy(x).to(cuda_device)
    y = torch.zeros(n, device=cuda_device)
    prog = _Program([_gemv(q, xd, y)], cuda_device)
    ref = oracle_lib.matmul(x[None, :], w, n)[0]
    for _ in range(3):  # repeated launches: counters reset by the kernel
        y.zero_()
        prog.run()
        assert_close_to_oracle(y.cpu().numpy()[None, :], ref[None, :])
    assert _fault_clear() == 0


def test_chained_gemvs_residual_and_swiglu(oracle_lib, cuda_device):
    """x -> gate|up with the SwiGLU epilogue -> down + residual -> o: every operation
    reads the previous one's output, across the arrival-counter barrier."""
    rng = np.random.default_rng(7)
    H, inter = 2048, 6144
    wgu = synth.q8_0_blocks(rng, 2 * inter, H)
    wd = synth.q8_0_blocks(rng, H, inter)
    wo = synth.q8_0_blocks(rng, H, H)
    dev = cuda_device
    gu = QMatMul.from_gguf_blocks(wgu, 2 * inter, H, device=dev)
    down = QMatMul.from_gguf_blocks(wd, H, inter, device=dev)
    o = QMatMul.from_gguf_blocks(wo, H, H, device=dev)
    x = rng.standard_normal(H).astype(np.float32)
    xd = torch.from_numpy(x).to(dev)
    h = torch.zeros(inter, device=dev)
    r = torch.from_numpy(rng.standard_normal(H).astype(np.float32)).to(dev)
    x2 = r.clone()
    y = torch.zeros(H, device=dev)
    prog = _Program([_gemv(gu, xd, h, epilogue=_lib.EPILOGUE_SWIGLU),
                     _gemv(down, h, x2, residual=_p(x2)),
                     _gemv(o, x2, y)], dev)
    prog.run()
    g_u = oracle_lib.matmul(x[None, :], wgu, 2 * inter)[0]
    h_ref = oracle_lib.swiglu(g_u[None, :])[0]
    assert_close_to_oracle(h.cpu().numpy()[None, :], h_ref[None, :])
    # the next operations against the oracle on the GPU's own inputs
    hg = h.cpu().numpy()
    x2_ref = r.cpu().numpy() + oracle_lib.matmul(hg[None, :], wd, H)[0]
    assert_close_to_oracle(x2.cpu().numpy()[None, :], x2_ref[None, :])
    y_ref = oracle_lib.matmul(x2.cpu().numpy()[None, :], wo, H)[0]
    assert_close_to_oracle(y.cpu().numpy()[None, :], y_ref[None, :])
    assert _fault_clear() == 0


def test_argmax_operation_picks_the_lm_head_maximum(oracle_lib, cuda_device):
    rng = np.random.default_rng(9)
    n, k = 5000, 2048
    w = synth.q8_0_blocks(rng, n, k)
    q = QMatMul.from_gguf_blocks(w, n, k, device=cuda_device)
    x = rng.standard_normal(k).astype(np.float32)
    xd = torch.from_numpy(x).to(cuda_device)
    logits = torch.zeros(n, device=cuda_device)
    prog = _Program([_gemv(q, xd, logits, argmax=1), _lib.Op(kind=_lib.OP_ARGMAX)], cuda_device)
    prog.pos.fill_(11)
    for step in range(2):
        prog.run()
        lg = logits.cpu().numpy()
        assert int(prog.token.item()) == int(np.argmax(lg))
        assert int(prog.pos.item()) == 12 + step
    assert_close_to_oracle(lg[None, :], oracle_lib.matmul(x[None, :], w, n))


def test_rmsnorm_prologue_matches_the_stream_kernel(cuda_device):
    """The rms_norm prologue against q8lin_forward_fused's (same formula, sums of squares
    in a different tree order: within the re-quantization tolerance)."""
    rng = np.random.default_rng(13)
    n, k = 3000, 2048
    w = synth.q8_0_blocks(rng, n, k)
    q = QMatMul.from_gguf_blocks(w, n, k, device=cuda_device)
    xd = torch.from_numpy(rng.standard_normal(k).astype(np.float32)).to(cuda_device)
    nw = torch.from_numpy(rng.uniform(0.5, 1.5, k).astype(np.float32)).to(cuda_device)
    y = torch.zeros(n, device=cuda_device)
    prog = _Program([_gemv(q, xd, y, prologue=_lib.PROLOGUE_RMSNORM, norm_weight=_p(nw), eps=1e-5)], cuda_device)
    prog.run()
    y2 = torch.empty(n, device=cuda_device)
    q.forward_fused(xd, y2, QMatMul.PROLOGUE_RMSNORM, nw, 1e-5)
    torch.cuda.synchronize()
    a, b = y.cpu().numpy().astype(np.float64), y2.cpu().numpy().astype(np.float64)
    assert np.linalg.norm(a - b) / np.linalg.norm(b) <= 2e-3
