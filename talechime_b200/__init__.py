"""talechime_b200 -- B200-native (sm_100a) Q8_0 quantized linear.

A from-scratch replacement for the Q8_0 GGUF projection path of talechime's VoxCPM2
BaseLM (candle ``QMatMul::forward`` over ``GgmlDType::Q8_0``, reached from
``Linear::forward`` at crates/voxcpm/src/weights.rs:213-229).

    from talechime_b200 import QMatMul, Linear
    w = QMatMul.from_gguf_blocks(blocks, n=2048, k=2048, device="cuda:0")
    y = w.forward(x)            # x: f32 [M, 2048] on cuda:0

The arithmetic is in ``libq8lin.so`` (C ABI in include/q8lin.h); build it with
``python -m talechime_b200.build``.
"""
from ._lib import Q8LinError
from .gguf import GGUFFile
from .qmatmul import Linear, QMatMul, quantize_rows

__all__ = ["QMatMul", "Linear", "Q8LinError", "quantize_rows", "GGUFFile"]
