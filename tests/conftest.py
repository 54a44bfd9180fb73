import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 GPU (B200); run with -m gpu")


@pytest.fixture(scope="session")
def oracle():
    from oracle.oracle import Oracle, build
    if not os.path.exists(os.path.join(ROOT, "oracle", "liboracle.so")):
        build()
    return Oracle()


@pytest.fixture(scope="session")
def ref_kernels():
    """The reference's own kernels compiled from its sources (oracle/_ref);
    present in the build container and wherever the built .so travelled."""
    from oracle.oracle import RefKernels
    if not RefKernels.available():
        pytest.skip("oracle/_ref not built (needs the reference tree: make -C oracle ref)")
    return RefKernels()


@pytest.fixture(scope="session")
def cuda_lib():
    from eosllm_b200 import backend
    if not os.path.exists(backend.LIB_PATH):
        backend.build()
    return backend.load()


@pytest.fixture(scope="session")
def gpu():
    """The CUDA backend on a real GPU.  Fails (never skips) when the GPU path
    is unavailable: a GPU test that silently skipped would hide a fallback."""
    import torch
    from eosllm_b200 import backend
    if not os.path.exists(backend.LIB_PATH):
        backend.build()
    backend.load()
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    assert backend.available(), f"eosi_cuda_probe failed: {backend.last_error()}"
    torch.cuda.init()
    return backend


def golden(name):
    return np.load(os.path.join(GOLDEN, name))


def bits(x: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)


def same_bits(x: np.ndarray, y: np.ndarray) -> bool:
    """Bit-identical float arrays, except that any NaN equals any NaN."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.ascontiguousarray(y, dtype=np.float32)
    if x.shape != y.shape:
        return False
    nx, ny = np.isnan(x), np.isnan(y)
    if not np.array_equal(nx, ny):
        return False
    return np.array_equal(bits(x)[~nx], bits(y)[~ny])
