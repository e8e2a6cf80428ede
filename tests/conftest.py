import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) and the built CUDA library")


@pytest.fixture(scope="session")
def c1_chip():
    from linuxformer_b200 import chip as C

    return C.c1(0)


@pytest.fixture(scope="session")
def real_chip():
    """The real compiled circuit (tests/golden/real_chip.npz, made by the reference's compiler)."""
    from linuxformer_b200 import chip as C

    return C.real()
