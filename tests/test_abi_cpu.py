"""libq8lin.so builds, loads and exports the whole C ABI; argument errors (no GPU)."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "q8lin.h")


def header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(q8lin_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from talechime_b200 import _lib, build

    build.build()
    return _lib.lib()


def test_header_declares_expected_surface():
    fns = header_functions()
    for name in ("q8lin_weight_create", "q8lin_forward", "q8lin_weight_destroy", "q8lin_last_error"):
        assert name in fns


def test_library_exports_every_header_symbol(lib):
    from talechime_b200 import _lib

    for name in header_functions():
        assert hasattr(lib, name), f"{name} declared in q8lin.h but not exported"
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"


def test_version(lib):
    assert lib.q8lin_version() == 3


def test_status_strings(lib):
    assert lib.q8lin_status_string(0) == b"Q8LIN_OK"
    assert lib.q8lin_status_string(2) == b"Q8LIN_ERR_SHAPE"
    assert lib.q8lin_status_string(99) == b"Q8LIN_ERR_UNKNOWN"


def test_create_rejects_bad_arguments_before_touching_cuda(lib):
    h = ctypes.c_void_p()
    buf = (ctypes.c_uint8 * 68)()
    assert lib.q8lin_weight_create(None, 2, 32, 0, None, ctypes.byref(h)) == 1
    assert lib.q8lin_weight_create(buf, 2, 33, 0, None, ctypes.byref(h)) == 2
    assert b"multiple of the Q8_0 block size" in lib.q8lin_last_error()
    assert lib.q8lin_weight_create(buf, 0, 32, 0, None, ctypes.byref(h)) == 2
    assert lib.q8lin_weight_create(buf, -1, 32, 0, None, ctypes.byref(h)) == 2
    assert lib.q8lin_weight_create(buf, 2, 32, 0, None, None) == 1
    assert h.value is None


def test_forward_rejects_null_handle(lib):
    assert lib.q8lin_forward(None, None, None, 1, None) == 1
    assert b"null" in lib.q8lin_last_error()
    assert lib.q8lin_workspace_size(None, 100) == 0


def test_quantize_rows_shape_checks(lib):
    assert lib.q8lin_quantize_rows(None, 1, 48, None, None, None) == 2
    assert lib.q8lin_quantize_rows(None, 0, 64, None, None, None) == 0
    assert lib.q8lin_quantize_rows(None, 2, 64, None, None, None) == 1


def test_prefill_entry_points_check_arguments_before_touching_cuda(lib):
    """The prompt-pass kernels refuse a context past max_t (the reference's "Transformer
    context limit exceeded", transformer.rs:110-113), bad head shapes, null and
    misaligned pointers, all before any CUDA call; t = 0 is a no-op."""
    P = ctypes.c_void_p
    good, odd = P(4096), P(4100)
    rope = lambda b, t, p0, hq=4, hkv=2, d=128, mt=16, ptr=good: lib.q8lin_rope_kv_rows(
        ptr, b, t, p0, ptr, ptr, ptr, ptr, hq, hkv, d, mt, ptr, None)
    attn = lambda b, t, p0, hq=4, hkv=2, d=128, mt=16, ptr=good: lib.q8lin_attention_prefill(
        ptr, ptr, ptr, b, t, p0, hq, hkv, d, mt, ptr, None)
    for fn in (rope, attn):
        assert fn(1, 10, 7) == 2  # 7 + 10 > 16
        assert b"context limit" in lib.q8lin_last_error()
        assert fn(1, 4, -1) == 2
        assert fn(0, 4, 0) == 2
        assert fn(1, -1, 0) == 2
        assert fn(1, 4, 0, hq=3) == 2  # not a multiple of hkv
        assert fn(1, 4, 0, ptr=None) == 1
        assert fn(1, 0, 16) == 0  # nothing to do, at the limit
    assert attn(1, 4, 0, d=64) == 2
    assert attn(1, 4, 0, ptr=odd) == 3
    assert lib.q8lin_status_string(3) == b"Q8LIN_ERR_ALIGNMENT"


def test_destroy_null_is_noop(lib):
    assert lib.q8lin_weight_destroy(None) == 0


def test_python_surface_rejects_cpu_device():
    import numpy as np

    from talechime_b200 import QMatMul

    with pytest.raises(ValueError):
        QMatMul.from_gguf_blocks(np.zeros(34, np.uint8), 1, 32, device="cpu")


@pytest.mark.parametrize("m,k,n,path", [
    (1, 2048, 6144, "stream_gemv"),      # decode: bulk-copy ring
    (1, 16384, 2048, "gemv"),            # K beyond the ring: register streaming
    (2, 2048, 6144, "gemv"),             # M = 2 at K <= 2048 keeps the GEMV
    (2, 6144, 2048, "small_batch_dp4a"), # K > 2048, M <= 6: dp4a kernel
    (6, 6144, 2048, "small_batch_dp4a"),
    (7, 6144, 2048, "int8_tc"),          # ... from M = 7 the int8 tensor cores
    (3, 2048, 4096, "small_batch_dp4a"), # M = 3, 4 with N*K >= 8M weights
    (4, 2048, 2048, "gemv"),             # ... but not below
    (5, 2048, 2048, "small_batch_dp4a"), # K <= 2048, 5 <= M <= 11
    (11, 2048, 12288, "small_batch_dp4a"),
    (12, 2048, 2048, "small_batch_mma"),  # 12 <= M <= 16 where x fits in shared memory
    (16, 2048, 12288, "small_batch_mma"),
    (16, 4096, 2048, "small_batch_mma"),  # x fits beside the rings in one CTA up to K ~ 8K
    (12, 6144, 2048, "small_batch_mma"),
    (17, 2048, 2048, "int8_tc"),
    (32, 6144, 2048, "int8_tc"),
    (33, 2048, 2048, "f16_tc"),
    (4096, 6144, 2048, "f16_tc"),
])
def test_dispatch_follows_measured_crossovers(lib, m, k, n, path):
    """The kernel q8lin_forward picks, queried on the host (the crossovers were measured
    on B200 in CUDA graphs; the GPU parity tests cover every path)."""
    from talechime_b200 import _lib
    assert _lib.PATH_NAMES[lib.q8lin_dispatch_path(m, k, n)] == path


def test_dispatch_rejects_invalid_sizes(lib):
    for m, k, n in ((0, 32, 1), (1, 33, 1), (1, 32, 0), (-1, 32, 1)):
        assert lib.q8lin_dispatch_path(m, k, n) == -1


def test_wait_limit_round_trip():
    """q8lin_set_wait_limit_ns: the time bound of the kernels' spin waits (default 1 s)."""
    from talechime_b200 import _lib

    L = _lib.lib()
    old = L.q8lin_wait_limit_ns()
    assert old == 1_000_000_000
    try:
        assert L.q8lin_set_wait_limit_ns(2_000_000) == 0
        assert L.q8lin_wait_limit_ns() == 2_000_000
    finally:
        L.q8lin_set_wait_limit_ns(old)


def test_workspace_sizes_cover_every_m():
    """q8lin_workspace_bytes(max_m, max_k) covers what every M <= max_m, K <= max_k needs."""
    from talechime_b200 import _lib

    L = _lib.lib()
    assert L.q8lin_workspace_bytes(0, 2048) == 0 and L.q8lin_workspace_bytes(8, 33) == 0
    for max_m in (1, 4, 17, 32, 33, 256, 4096):
        for max_k in (256, 2048, 6144):
            total = L.q8lin_workspace_bytes(max_m, max_k)
            for m in (1, 2, 5, 16, 17, 31, 32, 33, 64, 255, 256, 4095, 4096):
                for k in (32, 256, 2048, 6144):
                    if m <= max_m and k <= max_k:
                        assert L.q8lin_workspace_bytes(m, k) <= total
    h = ctypes.c_void_p()
    assert L.q8lin_workspace_create(0, 0, 2048, ctypes.byref(h)) == _lib.ERR_SHAPE
    assert L.q8lin_weight_bind_workspace(None, None) == _lib.ERR_INVALID_ARGUMENT
    assert L.q8lin_workspace_destroy(None) == 0


def _function_body(src, name):
    i = src.index(f"int {name}(")
    return src[i:src.index("\n}\n", i)]


def test_forward_paths_do_not_allocate():
    """The forward entry points and the kernel launchers they reach allocate no device
    memory: no cudaMalloc / cudaFree of any flavour in their bodies."""
    import os
    import re

    csrc = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "talechime_b200", "csrc")
    src = open(os.path.join(csrc, "abi.cu")).read()
    for fn in ("q8lin_forward", "q8lin_forward_ws", "q8lin_forward_fused", "q8lin_forward_allreduce"):
        assert not re.search(r"cuda(Malloc|Free)", _function_body(src, fn)), fn
    for f in ("gemv.cu", "gemv_mrow.cu", "gemm_tc.cu", "gemm_skinny.cu", "mlp.cu", "layout.cu"):
        assert not re.search(r"cuda(Malloc|Free)", open(os.path.join(csrc, f)).read()), f
