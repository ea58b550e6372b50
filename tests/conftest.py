import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = ROOT / "tests" / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (a B200)")


@pytest.fixture(scope="session")
def orc():
    """The C restatement (oracle/restate.c), built on demand."""
    from oracle.oracle import Restated

    return Restated()


@pytest.fixture(scope="session")
def ref():
    """The reference compiled from source (oracle/_ref); skipped when absent."""
    from oracle.oracle import Reference

    try:
        return Reference()
    except FileNotFoundError as ex:
        pytest.skip(str(ex))


@pytest.fixture(scope="session")
def lib():
    """The product library, built in-tree when it is missing."""
    from accelep_b200 import LIB_PATH, build

    if not LIB_PATH.is_file():
        build.build()
    from accelep_b200 import load

    return load()


@pytest.fixture(scope="session")
def cuda():
    import torch

    if not torch.cuda.is_available():
        pytest.fail("GPU test ran without a CUDA device")
    return torch.device("cuda:0")
