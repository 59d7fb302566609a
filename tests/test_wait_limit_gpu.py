"""Failure detection by time-bounded waits, made to run out on purpose without a fault.

The kernels' spin waits give up after q8lin_set_wait_limit_ns nanoseconds, set their bit
of the device fault word and return; the host reads (and clears) the word with
q8lin_fault_status.  Here the wait is for a peer that never arrives: q8lin_forward_allreduce
runs as rank 0 of a two-rank tensor-parallel group on one GPU whose rank 1 does not exist,
so rank 1's flag is never raised.  Every buffer the kernel touches is this GPU's own
memory.  The kernel must come back within the limit, report bit 1, write its rows as NaN,
and leave the context usable.  (Reference pattern: a failure turns into a status the
caller acts on, crates/voxcpm/src/cuda_graph.rs:142-160.)
"""
import ctypes
import time

import pytest
import torch

from talechime_b200 import QMatMul, _lib, synth
from tests.conftest import assert_close_to_oracle

pytestmark = pytest.mark.gpu


def _fault(dev):
    st = ctypes.c_uint32(0)
    _lib.check(_lib.lib().q8lin_fault_status(dev.index, ctypes.byref(st), 1))
    return st.value


def test_peer_wait_runs_out_and_reports(oracle_lib, cuda_device):
    L = _lib.lib()
    k, n, world = 2048, 1024, 2
    x, w = synth.case(77, 1, k, n)
    q = QMatMul.from_gguf_blocks(w, n, k, device=cuda_device)
    xd = torch.from_numpy(x).to(cuda_device)
    y = torch.zeros((1, n), device=cuda_device)
    stage = [torch.zeros(L.q8lin_allreduce_stage_bytes(n, world) // 4, device=cuda_device) for _ in range(world)]
    flags = [torch.zeros(L.q8lin_allreduce_flag_bytes(world) // 4, dtype=torch.int32, device=cuda_device)
             for _ in range(world)]
    sp = torch.tensor([t.data_ptr() for t in stage], dtype=torch.int64, device=cuda_device)
    fp = torch.tensor([t.data_ptr() for t in flags], dtype=torch.int64, device=cuda_device)
    assert _fault(cuda_device) == 0
    old = L.q8lin_wait_limit_ns()
    L.q8lin_set_wait_limit_ns(2_000_000)  # 2 ms
    try:
        t0 = time.perf_counter()
        _lib.check(L.q8lin_forward_allreduce(q.handle, ctypes.c_void_p(xd.data_ptr()), ctypes.c_void_p(y.data_ptr()),
                                             1, ctypes.c_void_p(sp.data_ptr()), ctypes.c_void_p(fp.data_ptr()), n, 0,
                                             world, 1, None, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
    finally:
        L.q8lin_set_wait_limit_ns(old)
    assert elapsed < 5.0
    f = _fault(cuda_device)
    assert f & 2, f"fault word {f:#x} lacks the streaming GEMV's bit"
    assert _fault(cuda_device) == 0  # read-and-clear
    assert torch.isnan(y).all()
    # rank 0's rows were staged on both "ranks" as tagged words (epoch 1, half 1) before the
    # wait for rank 1's words ran out
    for r in range(world):
        words = stage[r].view(torch.int64)
        assert int(words[(1 * world + 0) * n].item()) >> 32 == 1
    # the context is still usable: an ordinary call is exact again
    y2 = q.forward(xd)
    torch.cuda.synchronize()
    assert _fault(cuda_device) == 0
    assert_close_to_oracle(y2.cpu().numpy(), oracle_lib.matmul(x, w, n, threads=16))


def test_staging_smaller_than_the_weight_is_rejected(cuda_device):
    L = _lib.lib()
    k, n = 256, 64
    _, w = synth.case(78, 1, k, n)
    q = QMatMul.from_gguf_blocks(w, n, k, device=cuda_device)
    x = torch.zeros((1, k), device=cuda_device)
    y = torch.zeros((1, n), device=cuda_device)
    p = torch.zeros(2, dtype=torch.int64, device=cuda_device)
    st = L.q8lin_forward_allreduce(q.handle, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(y.data_ptr()), 1,
                                   ctypes.c_void_p(p.data_ptr()), ctypes.c_void_p(p.data_ptr()), n - 1, 0, 2, 1, None,
                                   None)
    assert st == _lib.ERR_SHAPE and b"staging" in L.q8lin_last_error()

