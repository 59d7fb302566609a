"""SwiGLU kernel and the (tensor-parallel) Q8_0 MLP on the GPU against the oracle.

Stage by stage through one rank's QMatMuls (MLPShard, the same kernels), and end to end
through the C-ABI object (SwiGLUMLP over q8lin_mlp_tp_*): on one GPU, and over NCCL with
the sum done by ncclAllReduce or inside the down projection's kernel (fused decode)."""
import ctypes
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch

from talechime_b200 import _lib, synth
from talechime_b200.tp_mlp import MLPShard, SwiGLUMLP, shard_k, shard_rows, swiglu
from tests.conftest import assert_close_to_oracle

pytestmark = pytest.mark.gpu

# End to end, the down projection re-quantizes h: a last-bit difference in the gate/up
# output (tree and split-K summation orders) can move an h value across a Q8_0 rounding
# boundary, a change of one quantization step d in that element.  Each projection is
# held to the per-linear tolerance against the oracle fed with the same input; the whole
# MLP against the all-oracle MLP gets this looser bound.
MLP_E2E_REL_L2 = 1e-3


def _check_stages(oracle_lib, mlp, x_np, gate, up, down, hidden, inter, rank=0, world=1):
    """gate/up, SwiGLU and down of one rank, each against the oracle on the same input."""
    il = inter // world
    xt = torch.from_numpy(x_np).to(mlp.device)
    gu = mlp.gate_up.forward(xt)
    gu_ref = np.concatenate([oracle_lib.matmul(x_np, shard_rows(gate, inter, hidden, rank, world), il, threads=16),
                             oracle_lib.matmul(x_np, shard_rows(up, inter, hidden, rank, world), il, threads=16)],
                            axis=1)
    assert_close_to_oracle(gu.cpu().numpy(), gu_ref)
    h = swiglu(gu, il)
    h_np = h.cpu().numpy()
    h_ref = oracle_lib.swiglu(gu.cpu().numpy())
    assert np.all(np.abs(h_np - h_ref) <= 4e-7 * np.abs(h_ref) + 1e-30)
    part = mlp.down.forward(h).cpu().numpy()
    part_ref = oracle_lib.matmul(h_np, shard_k(down, hidden, inter, rank, world), hidden, threads=16)
    assert_close_to_oracle(part, part_ref)
    return part


def _rel_l2(y, ref):
    return float(np.linalg.norm(y.astype(np.float64) - ref) / np.linalg.norm(ref))


def _weights(seed, hidden, inter, m):
    rng = np.random.default_rng(seed)
    gate = synth.q8_0_blocks(rng, inter, hidden)
    up = synth.q8_0_blocks(rng, inter, hidden)
    down = synth.q8_0_blocks(rng, hidden, inter)
    x = rng.standard_normal((m, hidden)).astype(np.float32)
    return x, gate, up, down


@pytest.mark.parametrize("m,inter", [(3, 256), (2, 30), (5, 4096)])
def test_swiglu_kernel_matches_oracle(oracle_lib, cuda_device, m, inter):
    rng = np.random.default_rng(100 + inter)
    gu = (rng.standard_normal((m, 2 * inter)) * 3).astype(np.float32)
    ref = oracle_lib.swiglu(gu)
    g = torch.from_numpy(gu).to(cuda_device)
    h = torch.empty((m, inter), device=cuda_device)
    _lib.check(_lib.lib().q8lin_swiglu(ctypes.c_void_p(g.data_ptr()), m, inter, ctypes.c_void_p(h.data_ptr()),
                                       ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)))
    got = h.cpu().numpy()
    # expf differs from the CPU libm exp by a few ulp: elementwise relative bound
    assert np.all(np.abs(got - ref) <= 4e-7 * np.abs(ref) + 1e-30)


def test_swiglu_rejects_bad_arguments(cuda_device):
    L = _lib.lib()
    assert L.q8lin_swiglu(None, 1, 4, None, None) == _lib.ERR_INVALID_ARGUMENT
    assert L.q8lin_swiglu(None, -1, 4, None, None) == _lib.ERR_SHAPE


@pytest.mark.parametrize("m", [1, 5, 40, 100])
def test_mlp_single_gpu_matches_oracle(oracle_lib, cuda_device, m):
    hidden, inter = 512, 1024
    x, gate, up, down = _weights(200 + m, hidden, inter, m)
    shard = MLPShard.from_gguf_blocks(gate, up, down, hidden, inter, device=cuda_device)
    part = _check_stages(oracle_lib, shard, x, gate, up, down, hidden, inter)
    ref = oracle_lib.mlp(x, gate, up, down, hidden, inter, threads=16)
    mlp = SwiGLUMLP.from_gguf_blocks(gate, up, down, hidden, inter, device=cuda_device, max_m=128)
    y = mlp.forward(torch.from_numpy(x).to(cuda_device)).cpu().numpy()
    if m > 1:
        assert np.array_equal(y, part)  # the C-ABI MLP runs the same three stages
    # (M = 1: silu(gate) * up is folded into the down projection's quantization)
    assert _rel_l2(y, ref) <= MLP_E2E_REL_L2
    mlp.close()


def test_mlp_decode_row_folds_swiglu(oracle_lib, cuda_device):
    """One activation row: gate|up GEMV, then the down GEMV with silu(gate) * up computed
    in its activation quantization -- the same values q8lin_swiglu feeds the unfused path."""
    hidden, inter = 1024, 2048
    x, gate, up, down = _weights(210, hidden, inter, 1)
    shard = MLPShard.from_gguf_blocks(gate, up, down, hidden, inter, device=cuda_device)
    mlp = SwiGLUMLP.from_gguf_blocks(gate, up, down, hidden, inter, device=cuda_device, max_m=4)
    xt = torch.from_numpy(x).to(cuda_device)
    y = mlp.forward(xt).cpu().numpy()
    h = swiglu(shard.gate_up.forward(xt), inter).cpu().numpy()
    assert_close_to_oracle(y, oracle_lib.matmul(h, down, hidden, threads=16))
    mlp.close()


def test_mlp_rejects_rows_beyond_max_m(cuda_device):
    hidden, inter = 256, 512
    x, gate, up, down = _weights(220, hidden, inter, 9)
    mlp = SwiGLUMLP.from_gguf_blocks(gate, up, down, hidden, inter, device=cuda_device, max_m=8)
    with pytest.raises(_lib.Q8LinError) as e:
        mlp.forward(torch.from_numpy(x).to(cuda_device))
    assert e.value.status == _lib.ERR_SHAPE
    mlp.close()


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_partials_sum_to_oracle(oracle_lib, cuda_device, world):
    """Every rank's shard on one GPU; the host adds the partials (the all-reduce)."""
    hidden, inter, m = 512, 2048, 4
    x, gate, up, down = _weights(300 + world, hidden, inter, m)
    total = np.zeros((m, hidden), dtype=np.float64)
    total_ref = np.zeros((m, hidden), dtype=np.float64)
    xt = torch.from_numpy(x).to(cuda_device)
    for r in range(world):
        part = MLPShard.from_gguf_blocks(gate, up, down, hidden, inter, device=cuda_device, rank=r, world=world)
        p = _check_stages(oracle_lib, part, x, gate, up, down, hidden, inter, rank=r, world=world)
        assert np.array_equal(part.partial(xt).cpu().numpy(), p)
        total += p
        h = swiglu(part.gate_up.forward(xt), inter // world).cpu().numpy()
        total_ref += oracle_lib.matmul(h, shard_k(down, hidden, inter, r, world), hidden, threads=16)
    assert_close_to_oracle(total, total_ref)
    ref = oracle_lib.mlp(x, gate, up, down, hidden, inter, threads=16)
    assert _rel_l2(total, ref) <= MLP_E2E_REL_L2


def test_tp_create_without_process_group_fails_loudly(cuda_device):
    hidden, inter = 256, 512
    _, gate, up, down = _weights(400, hidden, inter, 1)
    with pytest.raises(_lib.Q8LinError):
        SwiGLUMLP.from_gguf_blocks(gate, up, down, hidden, inter, device=cuda_device, rank=0, world=2)
    L = _lib.lib()
    h = ctypes.c_void_p()
    ptrs = [ctypes.c_void_p(b.ctypes.data) for b in (gate, up, down)]
    st = L.q8lin_mlp_tp_create(*ptrs, hidden, inter, 0, 2, None, 0, 4, 0, None, ctypes.byref(h))
    assert st == _lib.ERR_INVALID_ARGUMENT and b"communicator" in L.q8lin_last_error()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank, world, port, result_dir):
    torch.cuda.set_device(rank)
    torch.distributed.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                         world_size=world, timeout=timedelta(seconds=60),
                                         device_id=torch.device("cuda", rank))
    try:
        hidden, inter = 1024, 2048
        _, gate, up, down = _weights(500, hidden, inter, 1)
        dev = torch.device("cuda", rank)
        mlp = SwiGLUMLP.from_gguf_blocks(gate, up, down, hidden, inter, device=dev, rank=rank, world=world,
                                         max_m=64)
        out = {}
        for m in (1, 3, 40):
            x = np.random.default_rng(510 + m).standard_normal((m, hidden)).astype(np.float32)
            out[f"x{m}"] = x
            out[f"y{m}"] = mlp.forward(torch.from_numpy(x).to(dev)).cpu().numpy()
        torch.cuda.synchronize(dev)
        mlp.close()
        np.savez(os.path.join(result_dir, f"y{rank}.npz"), **out)
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_tp_nccl_multi_gpu(oracle_lib, cuda_device, tmp_path, world):
    """The C-ABI MLP over `world` GPUs (ncclAllReduce on torch's communicator)."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    port = _free_port()
    torch.multiprocessing.start_processes(_nccl_rank, args=(world, port, str(tmp_path)), nprocs=world,
                                          join=True, start_method="spawn")
    _, gate, up, down = _weights(500, 1024, 2048, 1)
    res = [np.load(tmp_path / f"y{r}.npz") for r in range(world)]
    for m in (1, 3, 40):
        ref = oracle_lib.mlp(res[0][f"x{m}"], gate, up, down, 1024, 2048, threads=16)
        for r in range(world):
            assert np.array_equal(res[r][f"y{m}"], res[0][f"y{m}"])  # every rank holds the same sum
        assert _rel_l2(res[0][f"y{m}"], ref) <= MLP_E2E_REL_L2


def _fused_rank(rank, world, port, result_dir):
    torch.cuda.set_device(rank)
    torch.distributed.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                         world_size=world, timeout=timedelta(seconds=60),
                                         device_id=torch.device("cuda", rank))
    try:
        hidden, inter = 1024, 2048
        dev = torch.device("cuda", rank)
        _, gate, up, down = _weights(600, hidden, inter, 1)
        fused = SwiGLUMLP.from_gguf_blocks(gate, up, down, hidden, inter, device=dev, rank=rank, world=world,
                                           max_m=4, fused_decode=True)
        plain = SwiGLUMLP.from_gguf_blocks(gate, up, down, hidden, inter, device=dev, rank=rank, world=world,
                                           max_m=4)
        assert fused.fused_decode and not plain.fused_decode
        xs, yf, yn = [], [], []
        for i in range(6):  # several calls: epochs and both staging halves
            x = np.random.default_rng(700 + i).standard_normal((1, hidden)).astype(np.float32)
            xd = torch.from_numpy(x).to(dev)
            yf.append(fused.forward(xd).cpu().numpy())
            yn.append(plain.forward(xd).cpu().numpy())
            xs.append(x)
        st = ctypes.c_uint32(0)
        _lib.check(_lib.lib().q8lin_fault_status(rank, ctypes.byref(st), 1))
        fused.close()
        plain.close()
        np.savez(os.path.join(result_dir, f"f{rank}.npz"), x=np.concatenate(xs), fused=np.concatenate(yf),
                 nccl=np.concatenate(yn), fault=np.array([st.value]))
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_fused_gemv_allreduce_matches_nccl(oracle_lib, cuda_device, tmp_path, world):
    """The down projection with the cross-GPU sum in the same kernel (peer stores over
    NVLink) against the down projection + ncclAllReduce: bit-identical for two ranks (a
    two-term sum does not depend on the order), within f32 tolerance otherwise."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    port = _free_port()
    torch.multiprocessing.start_processes(_fused_rank, args=(world, port, str(tmp_path)), nprocs=world,
                                          join=True, start_method="spawn")
    res = [np.load(tmp_path / f"f{r}.npz") for r in range(world)]
    _, gate, up, down = _weights(600, 1024, 2048, 1)
    for r in range(world):
        assert res[r]["fault"][0] == 0
        assert np.array_equal(res[r]["fused"], res[0]["fused"])  # every rank holds the same sum
        if world == 2:
            assert np.array_equal(res[r]["fused"], res[r]["nccl"])
        else:
            assert_close_to_oracle(res[r]["fused"], res[r]["nccl"])
    ref = oracle_lib.mlp(res[0]["x"], gate, up, down, 1024, 2048, threads=16)
    assert _rel_l2(res[0]["fused"], ref) <= MLP_E2E_REL_L2
