"""Q8_0 SwiGLU MLP on one GPU or tensor-parallel over P GPUs of one node.

The VoxCPM MLP (crates/voxcpm/src/transformer.rs:147-150) is
``down(silu(gate(h)) * up(h))`` with three Q8_0 ``QMatMul``s.  Partition for P ranks
(one exchange step):

* gate and up are split by output feature (weight rows): rank r holds rows
  [I*r/P, I*(r+1)/P) of each, stored as ONE fused weight [gate rows; up rows] so a
  single linear launch produces both halves, and ``q8lin_swiglu`` combines them;
* SwiGLU is local to the rank;
* down is split by input feature: rank r holds the Q8_0 block columns
  [nb*r/P, nb*(r+1)/P) of every row.  I/P stays a multiple of 32 (14336/8 = 1792 =
  56 blocks), so the rank's slice of h quantizes to exactly the Q8_0 blocks the
  unsplit activation row would have;
* one all-reduce (sum, f32, M x hidden) over the process group (NCCL over NVLink)
  adds the partial outputs.  The summation order differs from the single-GPU CPU
  path, so results agree within f32 tolerance.  For decode rows (M = 1),
  ``enable_fused_allreduce()`` replaces the down projection + NCCL all-reduce with one
  kernel per rank (``q8lin_forward_allreduce``): each CTA pushes its output rows into
  every rank's staging buffer over NVLink (peer stores into IPC-mapped buffers), raises
  a flag on every rank, and adds the ranks' rows in rank order once the same CTA of
  every rank has arrived.

x is replicated: every rank quantizes the same activation rows, so the gate/up
results are the bit-identical rows the single-GPU path computes.  Everything below
is argument checking, slicing of GGUF block arrays and pointer passing; the
arithmetic runs in libq8lin.so and the collective in torch.distributed.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np
import torch

from . import _lib
from ._lib import Q8LinError, check
from .qmatmul import BLOCK_BYTES, QK8_0, QMatMul, _stream_ptr


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


class SwiGLUMLP:
    """One rank's share of ``down(silu(gate(x)) * up(x))`` (all of it when world = 1)."""

    def __init__(self, gate_up: QMatMul, down: QMatMul, hidden: int, inter: int, rank: int = 0,
                 world: int = 1, group=None):
        self.gate_up = gate_up
        self.down = down
        self.hidden = hidden
        self.inter = inter
        self.inter_local = inter // world
        self.rank = rank
        self.world = world
        self.group = group
        self.device = gate_up.device

    @classmethod
    def from_gguf_blocks(cls, gate, up, down, hidden: int, inter: int,
                         device: Optional[torch.device | int | str] = None, rank: int = 0, world: int = 1,
                         group=None) -> "SwiGLUMLP":
        """gate, up: Q8_0 [inter, hidden]; down: Q8_0 [hidden, inter] (GGUF block bytes,
        numpy or torch uint8).  Keeps only this rank's shards on `device`."""
        il = inter // world if inter % world == 0 else -1
        if il <= 0 or il % QK8_0:
            raise Q8LinError(_lib.ERR_SHAPE, f"intermediate {inter} does not split into {world} block-aligned shards")
        gu = fuse_rows(shard_rows(gate, inter, hidden, rank, world), shard_rows(up, inter, hidden, rank, world))
        gate_up = QMatMul.from_gguf_blocks(gu, 2 * il, hidden, device=device)
        dn = QMatMul.from_gguf_blocks(shard_k(down, hidden, inter, rank, world), hidden, il, device=device)
        return cls(gate_up, dn, hidden, inter, rank, world, group)

    def partial(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """This rank's contribution to y (before the all-reduce)."""
        return self.down.forward(swiglu(self.gate_up.forward(x), self.inter_local), out=out)

    def _check_group(self) -> None:
        if self.world > 1 and not (torch.distributed.is_available() and torch.distributed.is_initialized()):
            raise Q8LinError(_lib.ERR_INVALID_ARGUMENT, "world > 1 needs an initialized torch.distributed group")

    def enable_fused_allreduce(self) -> None:
        """Map the staging and flag buffers of every rank (collective: every rank calls
        it) so that M = 1 forwards run the down projection and the cross-GPU sum as one
        kernel.  M > 1 keeps the NCCL all-reduce."""
        self._check_group()
        if self.world == 1 or getattr(self, "_ar", None) is not None:
            return
        L, dev = _lib.lib(), self.device.index
        sizes = {"stage": L.q8lin_allreduce_stage_bytes(self.hidden, self.world),
                 "flags": L.q8lin_allreduce_flag_bytes(self.world)}
        own, handles = {}, {}
        for name, nbytes in sizes.items():
            ptr, h = ctypes.c_void_p(), (ctypes.c_uint8 * 64)()
            check(L.q8lin_peer_alloc(dev, nbytes, ctypes.byref(ptr), h))
            own[name], handles[name] = ptr, bytes(h)
        gathered = [None] * self.world
        torch.distributed.all_gather_object(gathered, handles, group=self.group)
        opened, ptrs = [], {"stage": [], "flags": []}
        for r in range(self.world):
            for name in ("stage", "flags"):
                if r == self.rank:
                    ptrs[name].append(own[name].value)
                    continue
                p = ctypes.c_void_p()
                check(L.q8lin_peer_open(dev, gathered[r][name], ctypes.byref(p)))
                opened.append(p)
                ptrs[name].append(p.value)
        self._ar = {"own": own, "opened": opened, "epoch": 0,
                    "stage": torch.tensor(ptrs["stage"], dtype=torch.int64, device=self.device),
                    "flags": torch.tensor(ptrs["flags"], dtype=torch.int64, device=self.device)}
        torch.cuda.synchronize(self.device)
        torch.distributed.barrier(group=self.group)  # every rank mapped before the first call

    def close_fused_allreduce(self) -> None:
        """Unmap the peers' buffers and free this rank's (collective)."""
        ar = getattr(self, "_ar", None)
        if ar is None:
            return
        torch.cuda.synchronize(self.device)
        torch.distributed.barrier(group=self.group)  # no peer still writes into our buffers
        L, dev = _lib.lib(), self.device.index
        for p in ar["opened"]:
            L.q8lin_peer_close(dev, p)
        for p in ar["own"].values():
            L.q8lin_peer_free(dev, p)
        self._ar = None

    def forward(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        self._check_group()
        ar = getattr(self, "_ar", None)
        if ar is not None and x.dim() == 2 and x.shape[0] == 1:
            h = swiglu(self.gate_up.forward(x), self.inter_local)
            y = out if out is not None else torch.empty((1, self.hidden), dtype=torch.float32, device=self.device)
            ar["epoch"] += 1
            check(_lib.lib().q8lin_forward_allreduce(
                self.down.handle, ctypes.c_void_p(h.data_ptr()), ctypes.c_void_p(y.data_ptr()), 1,
                ctypes.c_void_p(ar["stage"].data_ptr()), ctypes.c_void_p(ar["flags"].data_ptr()), self.rank,
                self.world, ar["epoch"], None, ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)))
            return y
        y = self.partial(x, out=out)
        if self.world > 1:
            torch.distributed.all_reduce(y, op=torch.distributed.ReduceOp.SUM, group=self.group)
        return y

    __call__ = forward
