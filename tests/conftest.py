import os
import sys

import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if REPO not in sys.path:
    sys.path.insert(0, REPO)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (runs the CUDA kernels)")


@pytest.fixture(scope="session")
def built_lib():
    """Build (if needed) and load libhyperion_mlx.so."""
    from hyperion_b200.build import build
    build()
    import hyperion_b200
    return hyperion_b200.lib()


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle.build_oracle import build
    build()
    from oracle import gemma_oracle
    return gemma_oracle.lib()


def has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
