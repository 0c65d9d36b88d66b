import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


def _has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session")
def backend():
    """One libhachiue_cuda handle on cuda:0 for the GPU tests."""
    if not _has_gpu():
        pytest.fail("GPU test collected without a CUDA device (run with -m 'not gpu' on CPU)")
    from hachiue_b200 import CudaBackend
    be = CudaBackend(0)
    yield be
    be.close()


def rel_l2(a, b) -> float:
    import numpy as np
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
