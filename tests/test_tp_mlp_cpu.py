"""Tensor-parallel MLP host logic on the CPU: the C-ABI shard plan (q8lin_mlp_tp_shard)
and the argument checks of q8lin_mlp_tp_create that need no GPU, the SwiGLU oracle, and a
world-size-2 gloo run of the partition -- each rank slices its shards by the C plan,
computes its partial with the oracle, and gloo's all_reduce stands in for NCCL's --
against the unsplit oracle MLP."""
import ctypes
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch

from talechime_b200 import synth
from talechime_b200 import _lib
from talechime_b200._lib import Q8LinError
from talechime_b200.tp_mlp import fuse_rows, shard_k, shard_plan, shard_rows
from tests.conftest import assert_close_to_oracle

HIDDEN, INTER = 256, 512


def _mlp_weights(seed):
    rng = np.random.default_rng(seed)
    gate = synth.q8_0_blocks(rng, INTER, HIDDEN)
    up = synth.q8_0_blocks(rng, INTER, HIDDEN)
    down = synth.q8_0_blocks(rng, HIDDEN, INTER)
    x = rng.standard_normal((3, HIDDEN)).astype(np.float32)
    return x, gate, up, down


def test_row_shards_reassemble():
    _, gate, _, _ = _mlp_weights(1)
    for world in (1, 2, 4, 8):
        parts = [shard_rows(gate, INTER, HIDDEN, r, world) for r in range(world)]
        assert np.array_equal(np.concatenate(parts, axis=0).reshape(-1), gate.reshape(-1))


def test_k_shards_reassemble_blockwise():
    _, _, _, down = _mlp_weights(2)
    for world in (1, 2, 4, 8):
        parts = [shard_k(down, HIDDEN, INTER, r, world) for r in range(world)]
        assert all(p.shape == (HIDDEN, INTER // 32 // world, 34) for p in parts)
        assert np.array_equal(np.concatenate(parts, axis=1).reshape(-1), down.reshape(-1))


def test_c_shard_plan_matches_the_partition():
    for world in (1, 2, 4, 8):
        for r in range(world):
            row0, rows, blk0, blks = shard_plan(4096, 14336, r, world)
            assert (row0, rows) == (14336 // world * r, 14336 // world)
            assert (blk0, blks) == (448 // world * r, 448 // world)


def test_c_shard_plan_rejects_bad_splits():
    L = _lib.lib()
    out = [ctypes.c_int64() for _ in range(4)]
    refs = [ctypes.byref(v) for v in out]
    assert L.q8lin_mlp_tp_shard(4096, 14336, 0, 3, *refs) == _lib.ERR_SHAPE  # 448 blocks over 3
    assert L.q8lin_mlp_tp_shard(4096, 14336, 2, 2, *refs) == _lib.ERR_INVALID_ARGUMENT
    assert L.q8lin_mlp_tp_shard(4096, 14336 + 16, 0, 1, *refs) == _lib.ERR_SHAPE
    assert L.q8lin_mlp_tp_shard(4096, 14336, 0, 1, None, None, None, None) == _lib.ERR_INVALID_ARGUMENT


def test_c_create_checks_arguments_before_the_gpu():
    """Errors the C entry point reports without touching CUDA (no GPU here)."""
    L = _lib.lib()
    h = ctypes.c_void_p()
    buf = (ctypes.c_uint8 * 64)()
    p = ctypes.cast(buf, ctypes.c_void_p)
    assert L.q8lin_mlp_tp_create(p, p, p, 256, 512, 0, 2, None, 0, 8, 0, None, ctypes.byref(h)) == \
        _lib.ERR_INVALID_ARGUMENT  # world > 1 without a communicator
    assert b"communicator" in L.q8lin_last_error()
    assert L.q8lin_mlp_tp_create(None, p, p, 256, 512, 0, 1, None, 0, 8, 0, None, ctypes.byref(h)) == \
        _lib.ERR_INVALID_ARGUMENT
    assert L.q8lin_mlp_tp_create(p, p, p, 256, 512 + 32, 0, 2, None, 0, 8, 0, None, ctypes.byref(h)) == \
        _lib.ERR_SHAPE  # 17 blocks over 2 ranks
    assert L.q8lin_mlp_tp_create(p, p, p, 256, 512, 0, 1, None, 0, 0, 0, None, ctypes.byref(h)) == _lib.ERR_SHAPE
    assert L.q8lin_mlp_tp_create(p, p, p, 256, 512, 0, 1, None, 0, 8, 8, None, ctypes.byref(h)) == \
        _lib.ERR_INVALID_ARGUMENT  # unknown flag
    assert L.q8lin_mlp_tp_forward(None, None, None, 1, None) == _lib.ERR_INVALID_ARGUMENT
    assert L.q8lin_mlp_tp_peer_handle(None, None) == _lib.ERR_INVALID_ARGUMENT
    assert L.q8lin_mlp_tp_destroy(None) == 0
    assert L.q8lin_nccl_available() in (0, 1)


def test_uneven_splits_are_rejected():
    _, gate, _, down = _mlp_weights(3)
    with pytest.raises(Q8LinError):
        shard_rows(gate, INTER, HIDDEN, 0, 3)
    with pytest.raises(Q8LinError):
        shard_k(down, HIDDEN, INTER, 0, 3)  # 16 blocks per row over 3 ranks
    with pytest.raises(Q8LinError):
        shard_k(down, HIDDEN, INTER, 2, 2)


def test_shards_of_torch_tensors_match_numpy():
    _, gate, up, down = _mlp_weights(4)
    t = torch.from_numpy(down)
    assert np.array_equal(shard_k(t, HIDDEN, INTER, 1, 4).numpy(), shard_k(down, HIDDEN, INTER, 1, 4))
    fused = fuse_rows(torch.from_numpy(shard_rows(gate, INTER, HIDDEN, 1, 2)),
                      torch.from_numpy(shard_rows(up, INTER, HIDDEN, 1, 2)))
    assert fused.shape == (INTER, HIDDEN // 32, 34)


def test_swiglu_oracle_formula(oracle_lib):
    rng = np.random.default_rng(5)
    gu = (rng.standard_normal((4, 64)) * 4).astype(np.float32)
    gu[0, :3] = [-100.0, 100.0, 0.0]
    h = oracle_lib.swiglu(gu)
    g, u = gu[:, :32].astype(np.float64), gu[:, 32:].astype(np.float64)
    ref = g / (1.0 + np.exp(-g)) * u
    assert np.max(np.abs(h - ref)) <= 1e-6 * np.max(np.abs(ref))
    assert h[0, 0] == 0.0 or abs(h[0, 0]) < 1e-30  # silu(-100) underflows to -0/0


def test_split_sum_matches_unsplit_oracle(oracle_lib):
    """The sum of per-rank partials (computed serially) equals the unsplit MLP."""
    x, gate, up, down = _mlp_weights(6)
    full = oracle_lib.mlp(x, gate, up, down, HIDDEN, INTER)
    for world in (2, 4):
        total = np.zeros_like(full)
        for r in range(world):
            il = INTER // world
            g = oracle_lib.matmul(x, shard_rows(gate, INTER, HIDDEN, r, world), il)
            u = oracle_lib.matmul(x, shard_rows(up, INTER, HIDDEN, r, world), il)
            h = oracle_lib.swiglu(np.concatenate([g, u], axis=1))
            total += oracle_lib.matmul(h, shard_k(down, HIDDEN, INTER, r, world), HIDDEN)
        assert_close_to_oracle(total, full)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, result_dir):
    import oracle

    torch.distributed.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                                         world_size=world, timeout=timedelta(seconds=60))
    try:
        x, gate, up, down = _mlp_weights(7)
        row0, il, blk0, blks = shard_plan(HIDDEN, INTER, rank, world)  # the C plan of q8lin_mlp_tp_create
        dn = np.ascontiguousarray(down[:, blk0:blk0 + blks])
        gu = np.concatenate([oracle.matmul(x, np.ascontiguousarray(gate[row0:row0 + il]), il),
                             oracle.matmul(x, np.ascontiguousarray(up[row0:row0 + il]), il)], axis=1)
        part = oracle.matmul(oracle.swiglu(gu), dn, HIDDEN)
        y = torch.from_numpy(part.copy())
        torch.distributed.all_reduce(y, op=torch.distributed.ReduceOp.SUM)
        np.save(os.path.join(result_dir, f"y{rank}.npy"), y.numpy())
    finally:
        torch.distributed.destroy_process_group()


def test_gloo_world2_all_reduce_of_partials(oracle_lib, tmp_path):
    world = 2
    port = _free_port()
    torch.multiprocessing.start_processes(_gloo_rank, args=(world, port, str(tmp_path)), nprocs=world,
                                          join=True, start_method="spawn")
    x, gate, up, down = _mlp_weights(7)
    full = oracle_lib.mlp(x, gate, up, down, HIDDEN, INTER)
    y0, y1 = np.load(tmp_path / "y0.npy"), np.load(tmp_path / "y1.npy")
    assert np.array_equal(y0, y1)  # every rank holds the same reduced result
    assert_close_to_oracle(y0, full)
