"""Test configuration.

Markers: ``gpu`` tests need a B200 (they run the CUDA library through the
C-ABI and compare with the CPU oracle); everything else runs on CPU.
The oracle (oracle/) is test infrastructure: tests import it as the checker.
"""
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
for p in (REPO, REPO / "kestrel-q_b200"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def _has_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


HAS_GPU = _has_gpu()


def pytest_collection_modifyitems(config, items):
    if HAS_GPU:
        return
    skip = pytest.mark.skip(reason="no CUDA device in this container")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def kq():
    """The product library binding (builds it if needed)."""
    import kqb200
    from kqb200 import abi
    if not abi.LIB_PATH.exists():
        kqb200.build()
    kqb200.lib()
    return kqb200


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    if not O.PORT_LIB.exists():
        O.build()
    return O
