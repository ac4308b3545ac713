import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# The parity metric of the path: max|got - want| / max|want| per output
# tensor must stay within this bar against the reference.
PARITY_TOL = 1e-5


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")
    # Keep the in-tree library current with its sources (no-op when it is).
    # The build script is loaded by path: importing the package needs the
    # library to exist already.
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "molot_b200_build", os.path.join(ROOT, "molot_b200", "build.py"))
    build = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(build)
    build.build(quiet=True)


@pytest.fixture(scope="session")
def torch_cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


@pytest.fixture(scope="session")
def mb(torch_cuda):
    """The product library (fails loudly if it is not built)."""
    import molot_b200
    return molot_b200


@pytest.fixture(scope="session")
def orc():
    import oracle
    oracle.port()
    return oracle
