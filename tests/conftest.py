import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100) GPU; runs the CUDA library")


@pytest.fixture(scope="session")
def madi():
    """The CUDA library, bound to cuda:0.  Fails (does not skip) if it is missing."""
    import torch
    from madi_b200 import build
    import madi_b200

    if not os.path.exists(build.LIB):
        build.build()
    assert torch.cuda.is_available(), "gpu tests need a CUDA device"
    torch.cuda.init()
    madi_b200.init(0)
    return madi_b200


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O
    O.build()
    return O
