"""Host-side mirror of the operator surface talechime calls for Q8_0 projections.

* ``QMatMul`` -- candle's ``QMatMul::QTensor(Arc<QTensor>)`` for ``GgmlDType::Q8_0``
  as built at crates/voxcpm/src/weights.rs:103-104: holds one GGUF Q8_0 tensor on a
  B200 and computes ``forward(x[M, K]) -> y[M, N]``.
* ``Linear`` -- ``voxcpm::weights::Linear`` (crates/voxcpm/src/weights.rs:209-229):
  flattens x to ``[rows, in]``, calls ``QMatMul.forward`` and adds an optional bias.

All arithmetic runs in libq8lin.so (hand-written sm_100a kernels); this module only
checks arguments the way candle does, allocates outputs and passes pointers.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np
import torch

from . import _lib
from ._lib import Q8LinError, check

QK8_0 = 32
BLOCK_BYTES = 34


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


class Workspace:
    """Device scratch of the batched paths (q8lin_workspace), sized for every M <= max_m
    and K <= max_k.  ``Workspace.shared(device, m, k)`` is the one this process binds to
    its weights on that device; growing it allocates (so ``QMatMul.reserve`` belongs before
    a CUDA-graph capture), while ``q8lin_forward`` itself only reads it."""

    _shared: dict = {}

    def __init__(self, device: torch.device, max_m: int, max_k: int):
        self.device = device
        self.max_m = max_m
        self.max_k = max_k
        self._handle = ctypes.c_void_p()
        with torch.cuda.device(device):
            check(_lib.lib().q8lin_workspace_create(device.index, max_m, max_k, ctypes.byref(self._handle)))

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._handle

    def covers(self, m: int, k: int) -> bool:
        return m <= self.max_m and k <= self.max_k

    @classmethod
    def shared(cls, device: torch.device, m: int, k: int) -> "Workspace":
        cur = cls._shared.get(device.index)
        if cur is None or not cur.covers(m, k):
            if cur is not None:  # queued kernels may still read the old one
                torch.cuda.synchronize(device)
                m, k = max(m, cur.max_m), max(k, cur.max_k)
            cur = cls(device, m, k)
            cls._shared[device.index] = cur
        return cur

    def __del__(self):
        h = getattr(self, "_handle", None)
        if h is not None and h.value:
            try:
                _lib.lib().q8lin_workspace_destroy(h)
            except Exception:
                pass
            self._handle = None


class QMatMul:
    """One Q8_0 projection resident on one GPU (candle shape ``(n, k)`` = (out, in))."""

    def __init__(self, handle: ctypes.c_void_p, n: int, k: int, device: torch.device):
        self._handle = handle
        self.n = n
        self.k = k
        self.device = device
        self._ws: Optional[Workspace] = None

    def reserve(self, max_m: int) -> None:
        """Bind a workspace covering up to ``max_m`` activation rows (allocates when the
        shared workspace of the device has to grow; q8lin_forward never does)."""
        if _lib.lib().q8lin_workspace_bytes(max_m, self.k) == 0:
            return
        ws = Workspace.shared(self.device, max_m, self.k)
        if ws is not self._ws:
            check(_lib.lib().q8lin_weight_bind_workspace(self._handle, ws.handle))
            self._ws = ws  # keeps it alive while bound

    # -- construction --------------------------------------------------------------
    @classmethod
    def from_gguf_blocks(cls, blocks, n: int, k: int,
                         device: Optional[torch.device | int | str] = None) -> "QMatMul":
        """Upload N rows of K/32 GGUF Q8_0 blocks (34 bytes each).

        ``blocks`` may be ``bytes``, a uint8 numpy array, or a uint8 torch tensor on
        the CPU or on the target GPU.  Mirrors ``Content::tensor`` + ``QTensor``
        construction (crates/voxcpm/src/weights.rs:100-104).
        """
        if device is None:
            device = torch.device("cuda", torch.cuda.current_device())
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("QMatMul lives on a CUDA device; there is no CPU path")
        if k <= 0 or k % QK8_0:
            raise Q8LinError(_lib.ERR_SHAPE, f"in-features {k} is not a multiple of 32")
        nbytes = n * (k // QK8_0) * BLOCK_BYTES
        keep = None
        if isinstance(blocks, (bytes, bytearray, memoryview)):
            arr = np.frombuffer(blocks, dtype=np.uint8)
            keep = arr
            ptr = arr.ctypes.data
            size = arr.size
        elif isinstance(blocks, np.ndarray):
            arr = np.ascontiguousarray(blocks.view(np.uint8) if blocks.dtype != np.uint8 else blocks)
            keep = arr
            ptr = arr.ctypes.data
            size = arr.size
        elif isinstance(blocks, torch.Tensor):
            t = blocks.contiguous()
            if t.dtype != torch.uint8:
                raise TypeError("GGUF blocks must be a uint8 tensor")
            if t.is_cuda and t.device != device:
                raise ValueError(f"blocks are on {t.device}, weight requested on {device}")
            keep = t
            ptr = t.data_ptr()
            size = t.numel()
        else:
            raise TypeError(f"unsupported block container {type(blocks)!r}")
        if size != nbytes:
            raise Q8LinError(_lib.ERR_SHAPE,
                             f"{size} bytes of blocks do not match ({n}, {k}) Q8_0 = {nbytes} bytes")
        handle = ctypes.c_void_p()
        with torch.cuda.device(device):
            check(_lib.lib().q8lin_weight_create(ctypes.c_void_p(ptr), n, k, device.index,
                                                 ctypes.c_void_p(_stream_ptr(device)),
                                                 ctypes.byref(handle)))
        del keep
        return cls(handle, n, k, device)

    def __del__(self):
        h = getattr(self, "_handle", None)
        if h is not None and h.value:
            try:
                _lib.lib().q8lin_weight_destroy(h)
            except Exception:
                pass
            self._handle = None

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._handle

    def shape(self) -> tuple[int, int]:
        return (self.n, self.k)

    def device_bytes(self) -> int:
        out = ctypes.c_size_t()
        check(_lib.lib().q8lin_weight_device_bytes(self._handle, ctypes.byref(out)))
        return out.value

    # -- compute -------------------------------------------------------------------
    def _check_input(self, x: torch.Tensor) -> None:
        # candle QTensor::cpu_fwd / cuda_fwd rules for the quantized matmul
        if x.dim() < 2:
            raise Q8LinError(_lib.ERR_SHAPE, f"input tensor has only one dimension {tuple(x.shape)}")
        if x.shape[-1] != self.k:
            raise Q8LinError(_lib.ERR_SHAPE,
                             f"input tensor {tuple(x.shape)} incompatible with ({self.n}, {self.k})")
        if x.dtype != torch.float32:
            raise Q8LinError(_lib.ERR_INVALID_ARGUMENT, f"input dtype {x.dtype} is not f32")
        if not x.is_contiguous():
            raise Q8LinError(_lib.ERR_INVALID_ARGUMENT, "input tensor is not contiguous")
        if x.device != self.device:
            raise Q8LinError(_lib.ERR_DEVICE, f"input on {x.device}, weight on {self.device}")

    def forward(self, x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """y[..., N] = x[..., K] . W^T with candle's Q8_0 CPU semantics (QMatMul::forward)."""
        self._check_input(x)
        m = x.numel() // self.k
        if out is None:
            out = torch.empty(x.shape[:-1] + (self.n,), dtype=torch.float32, device=self.device)
        elif out.shape != x.shape[:-1] + (self.n,) or out.dtype != torch.float32 or not out.is_contiguous():
            raise Q8LinError(_lib.ERR_SHAPE, "out has the wrong shape, dtype or layout")
        if m > 0 and _lib.lib().q8lin_workspace_size(self._handle, m) > 0 and (
                self._ws is None or not self._ws.covers(m, self.k)
                or self._ws is not Workspace._shared.get(self.device.index)):
            self.reserve(m)
        check(_lib.lib().q8lin_forward(self._handle, ctypes.c_void_p(x.data_ptr()),
                                       ctypes.c_void_p(out.data_ptr()), m,
                                       ctypes.c_void_p(_stream_ptr(self.device))))
        return out

    __call__ = forward

    PROLOGUE_NONE, PROLOGUE_RMSNORM, PROLOGUE_SWIGLU = 0, 1, 2

    def forward_fused(self, x: torch.Tensor, out: torch.Tensor, prologue: int = 0,
                      norm_weight: Optional[torch.Tensor] = None, eps: float = 1e-5,
                      residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Decode-step fusion (one activation row): out = [residual +] W . p(x) with p the
        identity, rms_norm(x, norm_weight, eps) or silu(x[:K]) * x[K:]  (q8lin_forward_fused)."""
        kx = 2 * self.k if prologue == self.PROLOGUE_SWIGLU else self.k
        for name, t, want in (("x", x, kx), ("out", out, self.n), ("norm_weight", norm_weight, self.k),
                              ("residual", residual, self.n)):
            if t is None:
                continue
            if t.numel() != want or t.dtype != torch.float32 or not t.is_contiguous() or t.device != self.device:
                raise Q8LinError(_lib.ERR_SHAPE, f"{name} must be a contiguous f32 tensor of {want} values on "
                                                 f"{self.device} (one activation row)")
        ptr = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None
        check(_lib.lib().q8lin_forward_fused(self._handle, ptr(x), ptr(out), 1, int(prologue), ptr(norm_weight),
                                             float(eps), ptr(residual), ctypes.c_void_p(_stream_ptr(self.device))))
        return out

    def dequantize(self) -> torch.Tensor:
        """f32 [N, K] (QTensor::dequantize, crates/voxcpm/src/weights.rs:79-80,106)."""
        out = torch.empty((self.n, self.k), dtype=torch.float32, device=self.device)
        check(_lib.lib().q8lin_weight_dequantize(self._handle, ctypes.c_void_p(out.data_ptr()),
                                                 ctypes.c_void_p(_stream_ptr(self.device))))
        return out

    def to_gguf_blocks(self) -> torch.Tensor:
        """The weight in GGUF block layout, uint8 [N, K/32, 34] on the device."""
        out = torch.empty((self.n, self.k // QK8_0, BLOCK_BYTES), dtype=torch.uint8, device=self.device)
        check(_lib.lib().q8lin_weight_export_gguf(self._handle, ctypes.c_void_p(out.data_ptr()),
                                                  ctypes.c_void_p(_stream_ptr(self.device))))
        return out


class Linear:
    """voxcpm ``Linear { mat: QMatMul, bias: Option<Tensor> }`` (weights.rs:209-229)."""

    def __init__(self, mat: QMatMul, bias: Optional[torch.Tensor] = None):
        self.mat = mat
        self.bias = bias

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.dim() == 0:
            raise Q8LinError(_lib.ERR_SHAPE, "linear input must have dimensions")
        shape = list(x.shape)
        inp = shape[-1]
        rows = x.numel() // inp if inp else 0
        y = self.mat.forward(x.contiguous().reshape(rows, inp))
        shape[-1] = y.shape[1]
        y = y.reshape(shape)
        if self.bias is not None:
            y = y + self.bias
        return y

    __call__ = forward


def quantize_rows(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Device Q8_0 quantization of f32 rows: (qs int8 [M, K], d f16 [M, K/32])."""
    if x.dim() != 2 or x.dtype != torch.float32 or not x.is_cuda or not x.is_contiguous():
        raise Q8LinError(_lib.ERR_INVALID_ARGUMENT, "quantize_rows needs a contiguous f32 [M, K] CUDA tensor")
    m, k = x.shape
    qs = torch.empty((m, k), dtype=torch.int8, device=x.device)
    d = torch.empty((m, k // QK8_0), dtype=torch.float16, device=x.device)
    check(_lib.lib().q8lin_quantize_rows(ctypes.c_void_p(x.data_ptr()), m, k,
                                         ctypes.c_void_p(qs.data_ptr()), ctypes.c_void_p(d.data_ptr()),
                                         ctypes.c_void_p(_stream_ptr(x.device))))
    return qs, d
