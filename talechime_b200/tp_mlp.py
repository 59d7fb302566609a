"""Q8_0 SwiGLU MLP on one GPU or tensor-parallel over P GPUs of one node.

The VoxCPM MLP (crates/voxcpm/src/transformer.rs:147-150) is
``down(silu(gate(h)) * up(h))`` with three Q8_0 ``QMatMul``s.  Partition for P ranks
(one exchange step; the plan is ``q8lin_mlp_tp_shard`` in libq8lin.so):

* gate and up are split by output feature (weight rows): rank r holds rows
  [I*r/P, I*(r+1)/P) of each, stored as ONE fused weight [gate rows; up rows] so a
  single linear launch produces both halves;
* SwiGLU is local to the rank;
* down is split by input feature: rank r holds the Q8_0 block columns
  [nb*r/P, nb*(r+1)/P) of every row.  I/P stays a multiple of 32 (14336/8 = 1792 =
  56 blocks), so the rank's slice of h quantizes to exactly the Q8_0 blocks the
  unsplit activation row would have;
* one all-reduce (sum, f32, M x hidden) adds the partial outputs: ncclAllReduce on the
  process group's communicator, or, for one activation row with ``fused_decode``, inside
  the down projection's kernel (each CTA pushes its rows into every rank's staging buffer
  over NVLink and adds the ranks' rows in rank order).  The summation order differs from
  the single-GPU CPU path, so results agree within f32 tolerance.

``SwiGLUMLP`` is the C-ABI object (``q8lin_mlp_tp_*``): the shards, the scratch for up to
``max_m`` rows and the all-reduce live in libq8lin.so, which calls NCCL on the
communicator of torch's NCCL process group; torch carries the staging buffers' IPC
handles between the ranks.  ``MLPShard`` holds one rank's two projections as ``QMatMul``s
(the same kernels) so that tests can check every stage against the oracle and emulate P
shards on one GPU.  x is replicated: every rank quantizes the same activation rows.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np
import torch

from . import _lib
from ._lib import Q8LinError, check
from .qmatmul import BLOCK_BYTES, QK8_0, QMatMul, _stream_ptr

HANDLE_BYTES = 128  # Q8LIN_TP_HANDLE_BYTES


def shard_plan(hidden: int, inter: int, rank: int, world: int) -> tuple[int, int, int, int]:
    """(row0, rows, blk0, blks): rows of gate/up and block columns of down kept by `rank`."""
    v = [ctypes.c_int64() for _ in range(4)]
    check(_lib.lib().q8lin_mlp_tp_shard(hidden, inter, rank, world, *[ctypes.byref(t) for t in v]))
    return tuple(t.value for t in v)


def _blocks3(blocks, n: int, k: int):
    """View GGUF Q8_0 blocks (bytes, numpy or torch uint8) as [n, k/32, 34]."""
    nb = k // QK8_0
    if isinstance(blocks, (bytes, bytearray, memoryview)):
        blocks = np.frombuffer(blocks, dtype=np.uint8)
    if blocks.dtype not in (np.uint8, torch.uint8):
        raise Q8LinError(_lib.ERR_INVALID_ARGUMENT, "Q8_0 blocks must be uint8")
    size = blocks.numel() if isinstance(blocks, torch.Tensor) else blocks.size
    if size != n * nb * BLOCK_BYTES:
        raise Q8LinError(_lib.ERR_SHAPE, f"{size} bytes are not {n} rows of {nb} Q8_0 blocks")
    return blocks.reshape(n, nb, BLOCK_BYTES)


def shard_rows(blocks, n: int, k: int, rank: int, world: int):
    """Output-feature shard of a Q8_0 weight [n, k]: rows [n*rank/world, n*(rank+1)/world)."""
    if world < 1 or not 0 <= rank < world or n % world:
        raise Q8LinError(_lib.ERR_SHAPE, f"{n} output features do not split over {world} ranks")
    b = _blocks3(blocks, n, k)
    step = n // world
    return b[rank * step:(rank + 1) * step]


def shard_k(blocks, n: int, k: int, rank: int, world: int):
    """Input-feature shard of a Q8_0 weight [n, k]: block columns
    [nb*rank/world, nb*(rank+1)/world) of every row (k/32 must split evenly)."""
    nb = k // QK8_0
    if world < 1 or not 0 <= rank < world or k % QK8_0 or nb % world:
        raise Q8LinError(_lib.ERR_SHAPE, f"{nb} Q8_0 blocks per row do not split over {world} ranks")
    b = _blocks3(blocks, n, k)
    step = nb // world
    part = b[:, rank * step:(rank + 1) * step]
    return part.contiguous() if isinstance(part, torch.Tensor) else np.ascontiguousarray(part)


def fuse_rows(a, b):
    """Stack two row blocks of Q8_0 weights ([gate rows; up rows])."""
    if isinstance(a, torch.Tensor):
        return torch.cat([a, b], dim=0).contiguous()
    return np.ascontiguousarray(np.concatenate([a, b], axis=0))


def swiglu(gu: torch.Tensor, inter: int) -> torch.Tensor:
    """h[..., inter] = silu(gu[..., :inter]) * gu[..., inter:] on the device (q8lin_swiglu)."""
    if gu.shape[-1] != 2 * inter or gu.dtype != torch.float32 or not gu.is_contiguous() or not gu.is_cuda:
        raise Q8LinError(_lib.ERR_SHAPE, f"gu {tuple(gu.shape)} is not a contiguous f32 CUDA [..., {2 * inter}]")
    m = gu.numel() // (2 * inter)
    h = torch.empty(gu.shape[:-1] + (inter,), dtype=torch.float32, device=gu.device)
    check(_lib.lib().q8lin_swiglu(ctypes.c_void_p(gu.data_ptr()), m, inter, ctypes.c_void_p(h.data_ptr()),
                                  ctypes.c_void_p(_stream_ptr(gu.device))))
    return h


class MLPShard:
    """One rank's projections as QMatMuls: the fused [gate; up] rows and down's block
    columns (all of the MLP when world = 1).  ``partial`` is the rank's contribution to y."""

    def __init__(self, gate_up: QMatMul, down: QMatMul, hidden: int, inter: int, rank: int, world: int):
        self.gate_up, self.down = gate_up, down
        self.hidden, self.inter, self.rank, self.world = hidden, inter, rank, world
        self.inter_local = inter // world
        self.device = gate_up.device

    @classmethod
    def from_gguf_blocks(cls, gate, up, down, hidden: int, inter: int,
                         device: Optional[torch.device | int | str] = None, rank: int = 0,
                         world: int = 1) -> "MLPShard":
        row0, rows, blk0, blks = shard_plan(hidden, inter, rank, world)
        g = _blocks3(gate, inter, hidden)[row0:row0 + rows]
        u = _blocks3(up, inter, hidden)[row0:row0 + rows]
        d = _blocks3(down, hidden, inter)[:, blk0:blk0 + blks]
        d = d.contiguous() if isinstance(d, torch.Tensor) else np.ascontiguousarray(d)
        gate_up = QMatMul.from_gguf_blocks(fuse_rows(g, u), 2 * rows, hidden, device=device)
        dn = QMatMul.from_gguf_blocks(d, hidden, rows, device=device)
        return cls(gate_up, dn, hidden, inter, rank, world)

    def partial(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        return self.down.forward(swiglu(self.gate_up.forward(x), self.inter_local), out=out)


def _nccl_comm(group, device: torch.device) -> int:
    """The raw ncclComm_t of torch's NCCL process group on `device` (created if needed)."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        raise Q8LinError(_lib.ERR_INVALID_ARGUMENT, "world > 1 needs an initialized torch.distributed NCCL group")
    pg = group if group is not None else dist.distributed_c10d._get_default_group()
    backend = pg._get_backend(device)
    if not hasattr(backend, "_comm_ptr"):
        raise Q8LinError(_lib.ERR_INVALID_ARGUMENT, "the process group has no NCCL backend on this device")
    try:
        ptr = backend._comm_ptr()
    except RuntimeError:
        ptr = 0
    if not ptr:  # communicators are created lazily: one collective makes it
        t = torch.zeros(1, device=device)
        dist.all_reduce(t, group=group)
        torch.cuda.synchronize(device)
        ptr = backend._comm_ptr()
    if not ptr:
        raise Q8LinError(_lib.ERR_NCCL, "no NCCL communicator for this device")
    return ptr


class SwiGLUMLP:
    """One rank's share of ``down(silu(gate(x)) * up(x))`` behind the C ABI
    (q8lin_mlp_tp_*); every rank holds the summed y.  Collective when world > 1."""

    def __init__(self, handle: ctypes.c_void_p, hidden: int, inter: int, rank: int, world: int,
                 device: torch.device, max_m: int, group=None):
        self._handle = handle
        self.hidden, self.inter, self.rank, self.world = hidden, inter, rank, world
        self.inter_local = inter // world
        self.device = device
        self.max_m = max_m
        self._group = group

    @classmethod
    def from_gguf_blocks(cls, gate, up, down, hidden: int, inter: int,
                         device: Optional[torch.device | int | str] = None, rank: int = 0, world: int = 1,
                         group=None, max_m: int = 256, fused_decode: bool = False) -> "SwiGLUMLP":
        """gate, up: Q8_0 [inter, hidden]; down: Q8_0 [hidden, inter] (GGUF block bytes,
        numpy or torch uint8, the full tensors).  Keeps only this rank's shards on `device`."""
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        device = torch.device(device)
        keep = []
        for b, n, k in ((gate, inter, hidden), (up, inter, hidden), (down, hidden, inter)):
            b = _blocks3(b, n, k)
            b = b.contiguous() if isinstance(b, torch.Tensor) else np.ascontiguousarray(b)
            keep.append((b, b.data_ptr() if isinstance(b, torch.Tensor) else b.ctypes.data))
        comm = _nccl_comm(group, device) if world > 1 else None
        handle = ctypes.c_void_p()
        with torch.cuda.device(device):
            check(_lib.lib().q8lin_mlp_tp_create(
                ctypes.c_void_p(keep[0][1]), ctypes.c_void_p(keep[1][1]), ctypes.c_void_p(keep[2][1]), hidden, inter,
                rank, world, ctypes.c_void_p(comm) if comm else None, device.index, max_m,
                1 if fused_decode else 0, ctypes.c_void_p(_stream_ptr(device)), ctypes.byref(handle)))
        mlp = cls(handle, hidden, inter, rank, world, device, max_m, group)
        if fused_decode and world > 1:
            # every rank's staging/flag buffer handles, carried by the process group
            mine = (ctypes.c_uint8 * HANDLE_BYTES)()
            check(_lib.lib().q8lin_mlp_tp_peer_handle(handle, mine))
            gathered = [None] * world
            torch.distributed.all_gather_object(gathered, bytes(mine), group=group)
            allh = (ctypes.c_uint8 * (HANDLE_BYTES * world)).from_buffer_copy(b"".join(gathered))
            check(_lib.lib().q8lin_mlp_tp_connect_peers(handle, allh))
            torch.distributed.barrier(group=group)  # every rank mapped before the first call
        return mlp

    @property
    def fused_decode(self) -> bool:
        f = ctypes.c_int32(0)
        check(_lib.lib().q8lin_mlp_tp_info(self._handle, None, ctypes.byref(f)))
        return bool(f.value)

    def forward(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        if x.shape[-1] != self.hidden or x.dtype != torch.float32 or not x.is_contiguous() or x.device != self.device:
            raise Q8LinError(_lib.ERR_SHAPE, f"x must be a contiguous f32 [..., {self.hidden}] tensor on {self.device}")
        m = x.numel() // self.hidden
        y = out if out is not None else torch.empty(x.shape, dtype=torch.float32, device=self.device)
        check(_lib.lib().q8lin_mlp_tp_forward(self._handle, ctypes.c_void_p(x.data_ptr()),
                                              ctypes.c_void_p(y.data_ptr()), m,
                                              ctypes.c_void_p(_stream_ptr(self.device))))
        return y

    __call__ = forward

    def close(self) -> None:
        """Free the shards and buffers.  With the fused decode path every rank calls it:
        peers unmapped, a barrier, then each rank's own buffers freed."""
        h = getattr(self, "_handle", None)
        if h is None or not h.value:
            return
        if self.world > 1 and self.fused_decode:
            check(_lib.lib().q8lin_mlp_tp_close_peers(h))
            torch.distributed.barrier(group=self._group)
        self._handle = None
        check(_lib.lib().q8lin_mlp_tp_destroy(h))

    def __del__(self):
        h = getattr(self, "_handle", None)
        if h is not None and h.value:
            try:
                # never frees what a peer may still map: that is close()'s job
                _lib.lib().q8lin_mlp_tp_close_peers(h)
                if self.world == 1:
                    _lib.lib().q8lin_mlp_tp_destroy(h)
            except Exception:
                pass
