import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA; run with -m 'not gpu'")
    return torch.device("cuda:0")


@pytest.fixture(scope="session")
def oracle_mod():
    from oracle import oracle as O
    O.build()
    return O


@pytest.fixture(scope="session")
def native(cuda_device):
    from kquant_b200 import _native
    _native.load()
    return _native


@pytest.fixture(scope="session")
def ref_ext():
    """The reference's own CUDA extension, compiled from its sources (oracle/_ref)."""
    from oracle import build_ref
    if not build_ref.OUT.exists():
        pytest.skip("reference extension oracle/_ref not built")
    return build_ref.load()
