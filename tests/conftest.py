import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# Output tolerance of the f32 results against the candle-CPU restatement
# (the parity bar stated for this path): relative L2 <= 1e-5 and max-abs <= 1e-3 * max|y|.
REL_L2_TOL = 1e-5
MAX_ABS_FRAC_TOL = 1e-3


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def oracle_lib():
    import oracle

    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a visible CUDA device")
    major, minor = torch.cuda.get_device_capability(0)
    if (major, minor) != (10, 0):
        pytest.fail(f"GPU tests need sm_100 (B200); found sm_{major}{minor}")
    from talechime_b200 import build

    build.build()
    return torch.device("cuda", 0)


def assert_close_to_oracle(y, y_ref):
    """Tolerance check of an f32 output against the oracle's output."""
    import numpy as np

    y = np.asarray(y, dtype=np.float64)
    y_ref = np.asarray(y_ref, dtype=np.float64)
    assert y.shape == y_ref.shape
    assert np.all(np.isfinite(y)) == np.all(np.isfinite(y_ref))
    denom = np.linalg.norm(y_ref)
    rel = np.linalg.norm(y - y_ref) / denom if denom > 0 else np.linalg.norm(y - y_ref)
    max_abs = np.max(np.abs(y - y_ref)) if y.size else 0.0
    scale = np.max(np.abs(y_ref)) if y.size else 0.0
    assert rel <= REL_L2_TOL, f"relative L2 error {rel:.3e} > {REL_L2_TOL}"
    assert max_abs <= MAX_ABS_FRAC_TOL * scale + 1e-30, (
        f"max abs error {max_abs:.3e} > {MAX_ABS_FRAC_TOL} * max|y| ({scale:.3e})")
    return rel, max_abs
